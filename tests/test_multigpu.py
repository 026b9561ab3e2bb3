"""Multi-GPU paths.

* CPU (gloo, world size 2): the host logic every rank runs — handle exchange
  in rank order, deterministic sequence assignment, the page-split position
  count.
* GPU (2 GPUs, skipped with fewer): KV-sharded decode with the exchange over
  NVLink peer memory (kore_cuda_attn_decode_sharded_dev), one process per
  GPU, checked against the oracle on every rank, and the attention block with
  its projections on the same split (kore_cuda_attn_block_decode_dev).
"""
import datetime
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

from kore_b200.shard import assign_sequences, local_positions

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _FakeCtx:
    def __init__(self, rank):
        self.rank = rank
        self.opened = None

    def peer_handle(self):
        return bytes([self.rank]) * 64

    def peer_open(self, handles):
        self.opened = handles


def _gloo_worker(rank, world, port, q):
    import torch.distributed as dist
    from kore_b200.shard import exchange_handles
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    ctx = _FakeCtx(rank)
    handles = exchange_handles(ctx, dist)
    lengths = list(np.random.default_rng(5).integers(1024, 32768, size=64))
    table = assign_sequences(lengths, world)
    tables = [None] * world
    dist.all_gather_object(tables, table)
    q.put((rank, [h[0] for h in handles], ctx.opened == handles, all(t == table for t in tables)))
    dist.destroy_process_group()


def test_host_logic_on_two_gloo_ranks():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, order, opened, same in res:
        assert order == [0, 1]        # every rank sees all handles in rank order
        assert opened and same        # and opened them; the assignment agrees on all ranks


def test_assign_sequences_balances_and_partitions():
    lengths = list(np.random.default_rng(1).integers(1024, 32768, size=64))
    for n in (1, 2, 4, 8):
        t = assign_sequences(lengths, n)
        assert sorted(i for r in t for i in r) == list(range(64))
        loads = [sum(lengths[i] for i in r) for r in t]
        assert max(loads) - min(loads) <= max(lengths)


def test_page_split_counts_partition_the_positions():
    for n in (1, 2, 3, 8):
        for limit in (0, 1, 255, 256, 257, 2049, 32768):
            assert sum(local_positions(limit, 256, r, n) for r in range(n)) == limit


@pytest.mark.gpu
def test_sharded_decode_with_peer_exchange_on_all_gpus():
    """One rank per visible GPU (2 to 8): the peer exchange for that many ranks."""
    import torch
    n = min(torch.cuda.device_count(), 8)
    if n < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.join(ROOT, "tests", "mp_sharded_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    for rank in range(n):
        assert f"rank {rank} ok" in r.stdout, r.stdout[-2000:]
