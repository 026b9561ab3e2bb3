"""Failure detection without a GPU fault.

Every wait inside the decode and exchange kernels is bounded; when a bound
runs out the kernel records an error code, waits for its own copies still in
flight and returns, and the host reports KORE_CUDA_EDEVICE with a message
naming the wait. The context stays usable. The tests make waits run out on
purpose in the two GPU-safe ways:

* a K/V tile wait with a limit far below a copy's latency
  (kore_cuda_set_wait_limit): real copies that land "too late";
* a peer GPU that never sends: a KV-split context of two ranks in two
  processes, where rank 1 maps its exchange buffer and then launches
  nothing, so rank 0's exchange waits on words that nothing writes.

Nothing here traps, faults or hangs a GPU: each kernel returns on its own
after its (short) limit. The host-side failure paths of the split (a rank
that raises or never joins) are covered by the gloo tests.
"""
import os

import numpy as np
import pytest

import kore_b200 as K
from oracle import oracle as O
from tests.attn_check import assert_attn_close, normal

pytestmark = pytest.mark.gpu


def test_tile_wait_limit_expires_then_the_context_recovers():
    import torch
    H, G, d, pos = 28, 4, 128, 32768
    g = K.KoreCuda(1, H, G, d, pos + 1)
    o = O.OracleLayer(H, G, d, pos + 1)
    k, v = normal(41, (pos, G * d), (pos, G * d))
    for p0 in range(0, pos, 8192):
        g.append(0, 0, p0, k[p0:p0 + 8192], v[p0:p0 + 8192])
    o.fill(0, k, v)
    q1, k1, v1 = normal(42, (H * d,), (G * d,), (G * d,))
    dev = torch.device("cuda", 0)
    tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q1, k1, v1))
    out = torch.empty(H * d, device=dev)
    g.set_wait_limit(1e-9)          # 1 ns: far below the latency of any tile copy
    seen = None
    for _ in range(5):
        g.decode_dev(0, 0, pos, tq, tk, tv, out)
        try:
            g.sync()
        except K.KoreCudaError as e:
            seen = e
            break
    assert seen is not None, "no tile wait ran out with a 1 ns limit"
    assert seen.code == -6 and "K/V tile" in str(seen), str(seen)
    g.set_wait_limit(0)             # back to the default
    g.sync()                        # the error was reported once and cleared
    want = o.decode(pos, q1, k1, v1)
    got = g.decode(0, 0, pos, q1, k1, v1)
    assert_attn_close(got, want, "decode after a timed-out call")
    kr, vr = g.kv_read(0, 0, pos - 3, 4)   # the cache around the appended row is intact
    np.testing.assert_array_equal(kr, o.kc[pos - 3:pos + 1])
    np.testing.assert_array_equal(vr, o.vc[pos - 3:pos + 1])
    g.close()


def _silent_peer(device, handle_q, go_q, done_q):
    """Rank 1 of a two-rank KV split: exports its exchange buffer and then
    launches nothing until told to exit."""
    import kore_b200 as K2
    ctx = K2.KoreCuda(1, 28, 4, 128, 1024, device=device, shard_rank=1, shard_count=2)
    handle_q.put(ctx.peer_handle())
    go_q.get(timeout=300)           # rank 0 is done with its check
    ctx.close()
    done_q.put("rank 1 exits")


def test_a_peer_that_never_sends_makes_the_exchange_wait_expire():
    import torch
    import torch.multiprocessing as mp
    n_dev = torch.cuda.device_count()
    d1 = 1 if n_dev > 1 else 0
    mpc = mp.get_context("spawn")
    handle_q, go_q, done_q = mpc.Queue(), mpc.Queue(), mpc.Queue()
    peer = mpc.Process(target=_silent_peer, args=(d1, handle_q, go_q, done_q))
    peer.start()
    try:
        H, G, d = 28, 4, 128
        ctx = K.KoreCuda(1, H, G, d, 1024, device=0, shard_rank=0, shard_count=2)
        k, v = normal(43, (300, G * d), (300, G * d))
        ctx.append(0, 0, 0, k, v)   # this rank keeps page 0; page 1 belongs to the silent peer
        mine = ctx.peer_handle()
        theirs = handle_q.get(timeout=300)
        ctx.peer_open([mine, theirs])
        ctx.set_wait_limit(0.05)    # 50 ms
        dev = torch.device("cuda", 0)
        q1, k1, v1 = normal(44, (H * d,), (G * d,), (G * d,))
        tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q1, k1, v1))
        out = torch.empty(H * d, device=dev)
        ctx.decode_sharded_dev(0, 0, 300, tq, tk, tv, out)
        with pytest.raises(K.KoreCudaError) as e:
            ctx.sync()
        assert e.value.code == -6 and "peer" in str(e.value), str(e.value)
        ctx.set_wait_limit(0)
        ctx.sync()                  # reported once, then cleared: the context is usable
        kr, _ = ctx.kv_read(0, 0, 0, 256)
        assert np.array_equal(kr, O.rope_keys(G, d, O.inv_freq(1e6, d), 0, k[:256]))
        ctx.close()
    finally:
        go_q.put("go")
        peer.join(timeout=120)
    assert peer.exitcode == 0
    assert done_q.get(timeout=10) == "rank 1 exits"
