"""kore_cuda_attn_decode_noalloc: decode for callers that cannot allocate GPU
memory, such as a serving host that carves every device buffer out of its own
pre-reserved pool, or a plugin whose host gives it buffers and a stream but
no permission to allocate. Such a caller lays out the paged KV cache itself
and passes every buffer; the split scratch is a fixed array inside the
library.

Checked through the C ABI against the existing context-based entry point
(kore_cuda_attn_decode) on two decode calls in a row, within the tolerance of
the other parity tests; the second call reads the row that the first one
appended into the caller's pages. Collected last (test_zz_*) so that a run
stopping at the first failure has already run everything else.
"""
import ctypes

import numpy as np
import pytest

import kore_b200 as K
from oracle import oracle as O
from tests.attn_check import assert_attn_close, normal

pytestmark = pytest.mark.gpu


def _caller_owned_cache(torch, H, G, D, P, rows_k, rows_v, n_rope, rope_base=1e6):
    """Pages, page table and RoPE table laid out by the caller, as the view describes.
    Logical page j sits in physical page n_table-1-j, so the indirection is exercised."""
    n_table = (n_rope + P - 1) // P
    perm = np.arange(n_table, dtype=np.int32)[::-1].copy()
    kp = np.zeros((n_table, G, P, D), np.float32)
    vp = np.zeros((n_table, G, P, D), np.float32)
    for t in range(rows_k.shape[0]):
        kp[perm[t // P], :, t % P, :] = rows_k[t].reshape(G, D)
        vp[perm[t // P], :, t % P, :] = rows_v[t].reshape(G, D)
    inv = O.inv_freq(rope_base, D)
    cs = np.empty((n_rope, D // 2, 2), np.float32)
    for p in range(n_rope):
        cs[p, :, 0], cs[p, :, 1] = O.rope_angles(inv, p)
    dev = torch.device("cuda", 0)
    keep = {name: torch.from_numpy(a).to(dev) for name, a in (("k", kp), ("v", vp), ("pt", perm), ("cs", cs))}
    view = K.KvView(keep["k"].data_ptr(), keep["v"].data_ptr(), keep["pt"].data_ptr(), n_table, n_table, P,
                    H, G, D, keep["cs"].data_ptr(), n_rope)
    return view, keep


def test_noalloc_decode_matches_context_entry_point_two_calls():
    import torch
    lib = K.load_library()
    H, G, D, P = 28, 4, 128, 256
    cached = 5000
    n_rope = cached + 2
    ctx = K.KoreCuda(1, H, G, D, n_rope)
    kp, vp = normal(900, (cached, G * D), (cached, G * D))
    ctx.append(0, 0, 0, kp, vp)
    rows_k, rows_v = ctx.kv_read(0, 0, 0, cached)
    view, keep = _caller_owned_cache(torch, H, G, D, P, rows_k, rows_v, n_rope)
    dev = torch.device("cuda", 0)
    for step, pos in enumerate((cached, cached + 1)):
        q, k, v = normal(901 + step, (H * D,), (G * D,), (G * D,))
        want = ctx.decode(0, 0, pos, q, k, v)                     # the existing entry point
        tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q, k, v))
        out = torch.full((H * D,), float("nan"), device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        torch.cuda.synchronize()
        rc = lib.kore_cuda_attn_decode_noalloc(ctypes.byref(view), pos, tq.data_ptr(), tk.data_ptr(),
                                               tv.data_ptr(), out.data_ptr(), status.data_ptr(), None)
        torch.cuda.synchronize()
        assert rc == 0, lib.kore_cuda_last_error(None).decode()
        assert int(status.item()) == 0
        assert_attn_close(out.cpu().numpy().reshape(H, D), want, f"no-alloc decode, call {step + 1}")
    ctx.close()


def test_noalloc_decode_refuses_bad_arguments_with_a_message():
    import torch
    lib = K.load_library()
    H, G, D, P = 28, 4, 128, 256
    rows = np.zeros((1, G * D), np.float32)
    view, keep = _caller_owned_cache(torch, H, G, D, P, rows, rows, 64)
    dev = torch.device("cuda", 0)
    q = torch.zeros(H * D, device=dev)
    kv = torch.zeros(G * D, device=dev)
    out = torch.zeros(H * D, device=dev)
    rc = lib.kore_cuda_attn_decode_noalloc(ctypes.byref(view), 64, q.data_ptr(), kv.data_ptr(), kv.data_ptr(),
                                           out.data_ptr(), None, None)
    assert rc == -2 and b"position" in lib.kore_cuda_last_error(None)
    view.n_head, view.n_head_kv = 36, 4      # a group of 9 query heads: not supported
    rc = lib.kore_cuda_attn_decode_noalloc(ctypes.byref(view), 1, q.data_ptr(), kv.data_ptr(), kv.data_ptr(),
                                           out.data_ptr(), None, None)
    assert rc == -1 and b"geometry" in lib.kore_cuda_last_error(None)


@pytest.mark.parametrize("pos", [0, 20])
def test_noalloc_decode_short_contexts_match_the_oracle(pos):
    """Position 0 (no cached position: the one new row) and a context short
    enough for a single split, whose decode kernel writes the output itself
    with no split merge; checked against the oracle directly, two calls in a
    row (the second reads the row the first appended into the caller's
    pages)."""
    import torch
    lib = K.load_library()
    H, G, D, P = 28, 4, 128, 64
    n_rope = pos + 2
    o = O.OracleLayer(H, G, D, n_rope)
    rows_k = np.zeros((max(pos, 1), G * D), np.float32)
    rows_v = np.zeros((max(pos, 1), G * D), np.float32)
    if pos:
        kp, vp = normal(910, (pos, G * D), (pos, G * D))
        o.fill(0, kp, vp)
        rows_k, rows_v = o.kc[:pos].copy(), o.vc[:pos].copy()
    view, keep = _caller_owned_cache(torch, H, G, D, P, rows_k, rows_v, n_rope)
    dev = torch.device("cuda", 0)
    for step, p in enumerate((pos, pos + 1)):
        q, k, v = normal(911 + step, (H * D,), (G * D,), (G * D,))
        want = o.decode(p, q, k, v)
        tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q, k, v))
        out = torch.full((H * D,), float("nan"), device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        torch.cuda.synchronize()
        rc = lib.kore_cuda_attn_decode_noalloc(ctypes.byref(view), p, tq.data_ptr(), tk.data_ptr(),
                                               tv.data_ptr(), out.data_ptr(), status.data_ptr(), None)
        torch.cuda.synchronize()
        assert rc == 0, lib.kore_cuda_last_error(None).decode()
        assert int(status.item()) == 0
        assert_attn_close(out.cpu().numpy().reshape(H, D), want, f"no-alloc decode at {p}")


def test_noalloc_decode_refuses_a_geometry_beyond_the_scratch_array():
    """32 KV heads of 8 query heads each, 64-token pages: past ~130000 cached
    positions the splits' partial outputs no longer fit the fixed array, and
    the call must say so instead of launching. (The host refuses before any
    device memory is read, so small placeholder buffers stand in for the
    pools.)"""
    import torch
    lib = K.load_library()
    H, G, D, P = 256, 32, 128, 64
    pos = 200000
    dev = torch.device("cuda", 0)
    pool = torch.zeros(4096, device=dev)
    table = torch.zeros(16, dtype=torch.int32, device=dev)
    view = K.KvView(pool.data_ptr(), pool.data_ptr() + 8192, table.data_ptr(), pos // P + 1, 4, P, H, G, D,
                    pool.data_ptr(), pos + 1)
    q = torch.zeros(H * D, device=dev)
    kv = torch.zeros(G * D, device=dev)
    out = torch.zeros(H * D, device=dev)
    rc = lib.kore_cuda_attn_decode_noalloc(ctypes.byref(view), pos, q.data_ptr(), kv.data_ptr(), kv.data_ptr(),
                                           out.data_ptr(), None, None)
    assert rc == -1
    msg = lib.kore_cuda_last_error(None).decode()
    assert "split scratch" in msg and "2359296" in msg, msg
