"""Worker of tests/test_multigpu.py (one process per GPU, launched by
torch.distributed.run): a KV-sharded context per GPU, handles exchanged over
gloo, decode steps through kore_cuda_attn_decode_sharded_dev compared with
the oracle on every rank."""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import kore_b200 as K  # noqa: E402
from kore_b200.shard import exchange_handles  # noqa: E402
from oracle import oracle as O  # noqa: E402
from tests.attn_check import assert_attn_close, normal  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    H, G, d, ctx_max, cached = 28, 4, 128, 4096, 3000
    ctx = K.KoreCuda(2, H, G, d, ctx_max, device=local, shard_rank=rank, shard_count=world)
    oras = [O.OracleLayer(H, G, d, ctx_max) for _ in range(2)]
    for layer in range(2):
        k, v = normal(500 + layer, (cached, G * d), (cached, G * d))
        ctx.append(0, layer, 0, k, v)
        oras[layer].fill(0, k, v)
    exchange_handles(ctx, dist)
    dev = torch.device("cuda", local)
    out = torch.empty(H * d, device=dev)
    for step in range(3):
        for layer in range(2):
            pos = cached + step
            q, k, v = normal(600 + 10 * step + layer, (H * d,), (G * d,), (G * d,))
            tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q, k, v))
            torch.cuda.synchronize()
            ctx.decode_sharded_dev(0, layer, pos, tq, tk, tv, out)
            ctx.sync()
            assert_attn_close(out.cpu().numpy().reshape(H, d), oras[layer].decode(pos, q, k, v),
                              f"rank {rank} step {step} layer {layer}")
    dist.barrier()
    ctx.close()
    dist.destroy_process_group()
    print(f"rank {rank} ok", flush=True)


if __name__ == "__main__":
    main()
