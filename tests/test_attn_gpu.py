"""GPU parity of the CUDA attention path against the oracle, through the C ABI.

Every case drives kore_b200's C entry points (host buffers, as kore calls
them; device tensors for the *_dev forms) and compares with the C
restatement of kore's attention (oracle/), which is pinned bit-exact to the
reference by tests/test_oracle_pin.py. Tolerance (north star): per head and
token, max-abs error <= 2e-3 and max-abs error / max |reference| <= 1e-3.
Rotated key rows and value rows in the cache must be bit-identical to kore's.
"""
import numpy as np
import pytest

import kore_b200 as K
from oracle import oracle as O
from tests.attn_check import assert_attn_close, attn_errors, normal

pytestmark = pytest.mark.gpu


def make_ctx(H, G, d, ctx, n_layer=1, **kw):
    return K.KoreCuda(n_layer, H, G, d, ctx, **kw)


def fill_both(gpu, ora, seq, layer, n, seed, chunk=4096):
    """Appends n seeded rows at positions 0..n-1 to the GPU cache and the oracle."""
    kvd = gpu.kvd
    k, v = normal(seed, (n, kvd), (n, kvd))
    for p0 in range(0, n, chunk):
        gpu.append(seq, layer, p0, k[p0:p0 + chunk], v[p0:p0 + chunk])
    ora.fill(0, k, v)
    return k, v


# ------------------------------------------------------------------ KV append

@pytest.mark.parametrize("H,G,d", [(14, 2, 64), (28, 4, 128), (16, 2, 128)])
def test_kv_append_rows_bitexact(H, G, d):
    n = 700   # crosses pages at 256 and 512
    g = make_ctx(H, G, d, 1024)
    o = O.OracleLayer(H, G, d, 1024)
    fill_both(g, o, 0, 0, n, 11, chunk=300)
    kr, vr = g.kv_read(0, 0, 0, n)
    np.testing.assert_array_equal(kr, o.kc[:n])
    np.testing.assert_array_equal(vr, o.vc[:n])


# ------------------------------------------------------------------ decode

@pytest.mark.parametrize("pos", [0, 1, 7, 8, 9, 63, 64, 255, 256, 257, 511, 1000, 2047])
def test_decode_positions_and_page_edges_3b(pos):
    H, G, d = 16, 2, 128
    g = make_ctx(H, G, d, 2048 + 8)
    o = O.OracleLayer(H, G, d, 2048 + 8)
    if pos:
        fill_both(g, o, 0, 0, pos, 100 + pos)
    q, k, v = normal(pos, (H * d,), (G * d,), (G * d,))
    out = g.decode(0, 0, pos, q, k, v)
    ref = o.decode(pos, q, k, v)
    assert_attn_close(out, ref, f"decode pos {pos}")
    kr, vr = g.kv_read(0, 0, pos, 1)
    np.testing.assert_array_equal(kr[0], o.kc[pos])
    np.testing.assert_array_equal(vr[0], o.vc[pos])


def test_cfg1_0p5b_prefill128_then_64_decode_steps():
    """Config 1: Qwen2.5-0.5B-shaped layer (14Q/2KV, d 64), prefill 128 tokens
    at positions 0..127, then 64 decode steps at 128..191."""
    H, G, d = 14, 2, 64
    g = make_ctx(H, G, d, 192)
    o = O.OracleLayer(H, G, d, 192)
    q, k, v = normal(12345, (128, H * d), (128, G * d), (128, G * d))
    out = g.prefill(0, 0, 0, q, k, v)
    ref = o.prefill(0, q, k, v)
    assert_attn_close(out, ref, "cfg1 prefill")
    for step in range(64):
        pos = 128 + step
        q1, k1, v1 = normal(777 + step, (H * d,), (G * d,), (G * d,))
        assert_attn_close(g.decode(0, 0, pos, q1, k1, v1), o.decode(pos, q1, k1, v1), f"cfg1 decode {pos}")
    kr, vr = g.kv_read(0, 0, 0, 192)
    np.testing.assert_array_equal(kr, o.kc)
    np.testing.assert_array_equal(vr, o.vc)


@pytest.mark.parametrize("layer", [0, 27])
def test_cfg2_7b_decode_at_8192(layer):
    """Config 2 shape: 28Q/4KV, d 128, 28 layers, decode at position 8192."""
    H, G, d = 28, 4, 128
    g = make_ctx(H, G, d, 8193, n_layer=28)
    o = O.OracleLayer(H, G, d, 8193)
    fill_both(g, o, 0, layer, 8192, 2000 + layer)
    q, k, v = normal(3000 + layer, (H * d,), (G * d,), (G * d,))
    assert_attn_close(g.decode(0, layer, 8192, q, k, v), o.decode(8192, q, k, v), "cfg2 decode")


def test_cfg4_7b_decode_at_32768():
    """Config 4 shape on one GPU: decode at position 32768 (one layer)."""
    H, G, d = 28, 4, 128
    g = make_ctx(H, G, d, 32769)
    o = O.OracleLayer(H, G, d, 32769)
    fill_both(g, o, 0, 0, 32768, 44)
    q, k, v = normal(45, (H * d,), (G * d,), (G * d,))
    assert_attn_close(g.decode(0, 0, 32768, q, k, v), o.decode(32768, q, k, v), "cfg4 decode")


@pytest.mark.parametrize("H,G,d,pos", [(28, 4, 128, 32768), (28, 4, 128, 3000), (14, 2, 64, 191),
                                       (16, 2, 128, 5000), (28, 4, 128, 300)])
def test_fused_split_merge_equals_separate_merge_kernel(H, G, d, pos, monkeypatch):
    """One GPU: the merge CTAs at the end of the decode launch give the same
    bits as split_merge_kernel (the same merge arithmetic), over repeated
    calls (the arrival counters reset themselves), and match the oracle."""
    ctxs = []
    for fused in ("1", "0"):
        monkeypatch.setenv("KORE_CUDA_FUSED_MERGE", fused)
        ctxs.append(make_ctx(H, G, d, pos + 2, n_layer=1))
    o = O.OracleLayer(H, G, d, pos + 2)
    k, v = normal(60 + pos, (pos, G * d), (pos, G * d))
    for g in ctxs:
        for p0 in range(0, pos, 4096):
            g.append(0, 0, p0, k[p0:p0 + 4096], v[p0:p0 + 4096])
    o.fill(0, k, v)
    q, kn, vn = normal(61 + pos, (H * d,), (G * d,), (G * d,))
    outs = [[g.decode(0, 0, pos, q, kn, vn) for _ in range(3)] for g in ctxs]
    for a in outs[0] + outs[1]:
        np.testing.assert_array_equal(a, outs[1][0])
    assert_attn_close(outs[0][0], o.decode(pos, q, kn, vn), f"fused merge pos {pos}")


@pytest.mark.parametrize("H,G,pos", [(28, 4, 0), (28, 4, 1), (28, 4, 15), (28, 4, 16), (28, 4, 17), (28, 4, 255),
                                     (28, 4, 257), (28, 4, 1000), (28, 4, 9001), (16, 2, 777), (16, 4, 4099),
                                     (4, 4, 3000), (8, 8, 65), (24, 4, 2048)])
def test_tensor_core_decode_matches_oracle_and_cuda_core_path(H, G, pos, monkeypatch):
    """Single-query decode at head_dim 128 runs the tensor-core kernel
    (16-token tiles, split-bf16 products); KORE_CUDA_TC_DECODE=0 runs the
    CUDA-core kernel. Both within tolerance of the oracle at tile and page
    edges, for 1, 4, 6, 7 and 8 query heads per KV head; the cached rows are
    kore's bit for bit on both."""
    d = 128
    o = O.OracleLayer(H, G, d, pos + 2)
    k, v = normal(80 + pos, (pos, G * d), (pos, G * d))
    if pos:
        o.fill(0, k, v)
    q, kn, vn = normal(81 + pos, (H * d,), (G * d,), (G * d,))
    ref = o.decode(pos, q, kn, vn)
    for tc in ("1", "0"):
        monkeypatch.setenv("KORE_CUDA_TC_DECODE", tc)
        g = make_ctx(H, G, d, pos + 2)
        for p0 in range(0, pos, 4096):
            g.append(0, 0, p0, k[p0:p0 + 4096], v[p0:p0 + 4096])
        assert_attn_close(g.decode(0, 0, pos, q, kn, vn), ref, f"decode tc={tc} H={H} G={G} pos={pos}")
        kr, vr = g.kv_read(0, 0, pos, 1)
        np.testing.assert_array_equal(kr, o.kc[pos:pos + 1])
        np.testing.assert_array_equal(vr, o.vc[pos:pos + 1])
        g.close()


@pytest.mark.parametrize("pos", [0, 700, 5000])
def test_host_call_mapped_return_equals_copy_back(pos, monkeypatch):
    """The host-buffer decode returns through mapped memory and a polled
    completion word by default; KORE_CUDA_RET_MAPPED=0 copies the output back
    and synchronises. Same bits, over repeated calls, and an error code still
    comes back as an error with the context usable after it."""
    H, G, d = 28, 4, 128
    k, v = normal(90 + pos, (pos, G * d), (pos, G * d))
    q, kn, vn = normal(91 + pos, (H * d,), (G * d,), (G * d,))
    outs = []
    for m in ("1", "0"):
        monkeypatch.setenv("KORE_CUDA_RET_MAPPED", m)
        g = make_ctx(H, G, d, pos + 2)
        if pos:
            g.append(0, 0, 0, k, v)
        outs.append([g.decode(0, 0, pos, q, kn, vn) for _ in range(3)])
        with pytest.raises(K.KoreCudaError):
            g.decode(0, 0, pos + 5, q, kn, vn)   # a position beyond the context: refused
        np.testing.assert_array_equal(g.decode(0, 0, pos, q, kn, vn), outs[-1][0])
        g.close()
    for a in outs[0] + outs[1]:
        np.testing.assert_array_equal(a, outs[1][0])


def test_decode_dev_matches_host_path():
    import torch
    H, G, d = 28, 4, 128
    g = make_ctx(H, G, d, 4096, n_layer=2)
    o = O.OracleLayer(H, G, d, 4096)
    fill_both(g, o, 0, 1, 3000, 5)
    q, k, v = normal(6, (H * d,), (G * d,), (G * d,))
    dev = torch.device("cuda", 0)
    tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q, k, v))
    tout = torch.empty(H * d, device=dev)
    g.decode_dev(0, 1, 3000, tq, tk, tv, tout)
    g.sync()
    assert_attn_close(tout.cpu().numpy().reshape(H, d), o.decode(3000, q, k, v), "decode_dev")


def test_decode_batch_ragged_3b():
    """Config 5 shape (16Q/2KV, d 128), 12 sequences with ragged lengths over a
    shared 256-token page pool, one batched decode call."""
    H, G, d = 16, 2, 128
    rng = np.random.default_rng(55)
    lens = [int(x) for x in rng.integers(1, 3000, size=12)] + [0, 255, 256]
    n = len(lens)
    g = make_ctx(H, G, d, 3072, max_seqs=n)
    oras = []
    for s, L in enumerate(lens):
        o = O.OracleLayer(H, G, d, 3072)
        if L:
            fill_both(g, o, s, 0, L, 900 + s)
        oras.append(o)
    q, k, v = normal(56, (n, H * d), (n, G * d), (n, G * d))
    seqs = np.arange(n, dtype=np.int32)
    out = g.decode_batch(0, seqs, np.array(lens, np.int32), q, k, v)
    for s, L in enumerate(lens):
        assert_attn_close(out[s], oras[s].decode(L, q[s], k[s], v[s]), f"batch seq {s} len {L}")


def test_page_reuse_after_seq_reset():
    H, G, d = 28, 4, 128
    g = make_ctx(H, G, d, 1024, max_seqs=2, n_pages=4)
    o = O.OracleLayer(H, G, d, 1024)
    fill_both(g, o, 0, 0, 1000, 1)
    with pytest.raises(K.KoreCudaError) as e:   # pool of 4 pages is full
        g.append(1, 0, 0, *normal(2, (10, G * d), (10, G * d)))
    assert e.value.code == -3
    g.seq_reset(0)
    o2 = O.OracleLayer(H, G, d, 1024)
    fill_both(g, o2, 1, 0, 600, 3)
    q, k, v = normal(4, (H * d,), (G * d,), (G * d,))
    assert_attn_close(g.decode(1, 0, 600, q, k, v), o2.decode(600, q, k, v), "after reset")


# ------------------------------------------------------------------ prefill

def test_prefill_kore_chunk_onto_4096_7b():
    """A kore-sized 64-token prefill chunk (KORE_BMAX) onto 4096 cached rows."""
    H, G, d = 28, 4, 128
    g = make_ctx(H, G, d, 4160)
    o = O.OracleLayer(H, G, d, 4160)
    fill_both(g, o, 0, 0, 4096, 31)
    q, k, v = normal(32, (64, H * d), (64, G * d), (64, G * d))
    assert_attn_close(g.prefill(0, 0, 4096, q, k, v), o.prefill(4096, q, k, v), "prefill 64 onto 4096")


@pytest.mark.parametrize("pos0,n", [(0, 1), (0, 300), (5, 1), (250, 13), (1000, 257)])
def test_prefill_shapes(pos0, n):
    H, G, d = 14, 2, 64
    g = make_ctx(H, G, d, 2048)
    o = O.OracleLayer(H, G, d, 2048)
    if pos0:
        fill_both(g, o, 0, 0, pos0, 70 + pos0)
    q, k, v = normal(pos0 * 7 + n, (n, H * d), (n, G * d), (n, G * d))
    assert_attn_close(g.prefill(0, 0, pos0, q, k, v), o.prefill(pos0, q, k, v), f"prefill {pos0}+{n}")


# ------------------------------------------------------------------ errors (kore.cpp:1400, :1490)

def test_errors_are_codes_not_crashes():
    H, G, d = 28, 4, 128
    g = make_ctx(H, G, d, 64, n_layer=2)
    q, k, v = normal(1, (H * d,), (G * d,), (G * d,))
    with pytest.raises(K.KoreCudaError) as e:
        g.decode(0, 0, 64, q, k, v)             # pos >= ctx
    assert e.value.code == -2
    with pytest.raises(K.KoreCudaError) as e:
        g.decode(0, 0, 5, q, k, v)              # rows 0..4 never written
    assert e.value.code == -5
    with pytest.raises(K.KoreCudaError) as e:
        g.decode(0, 2, 0, q, k, v)              # layer out of range
    assert e.value.code == -2
    with pytest.raises(K.KoreCudaError) as e:
        g.decode(1, 0, 0, q, k, v)              # seq out of range
    assert e.value.code == -2
    out = g.decode(0, 0, 0, q, k, v)            # the context is still usable
    assert np.isfinite(out).all()


# ------------------------------------------------------------------ KV positions split over GPUs

@pytest.mark.parametrize("n_shards,pos", [(2, 3000), (3, 2049), (8, 700), (8, 100)])
def test_kv_sharded_decode_partials_merge_to_the_full_result(n_shards, pos):
    """Config 4's multi-GPU split, emulated with one context per shard on one
    GPU: each shard holds pages j = rank (mod N) and returns its partial; the
    LSE merge of the partials must equal kore's single softmax. With pos 100
    and 8 shards, seven shards hold no position at all."""
    import torch
    H, G, d = 28, 4, 128
    ctxs = [make_ctx(H, G, d, 4096, shard_rank=r, shard_count=n_shards) for r in range(n_shards)]
    o = O.OracleLayer(H, G, d, 4096)
    k, v = normal(70 + n_shards, (pos, G * d), (pos, G * d))
    for c in ctxs:
        c.append(0, 0, 0, k, v)
    o.fill(0, k, v)
    q1, k1, v1 = normal(71, (H * d,), (G * d,), (G * d,))
    dev = torch.device("cuda", 0)
    tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q1, k1, v1))
    parts = torch.empty(n_shards, ctxs[0].part_floats, device=dev)
    for r, c in enumerate(ctxs):
        c.decode_partial_dev(0, 0, pos, tq, tk, tv, parts[r])
        c.sync()
    out = torch.empty(H * d, device=dev)
    ctxs[0].lse_merge_dev(n_shards, parts, out)
    ctxs[0].sync()
    assert_attn_close(out.cpu().numpy().reshape(H, d), o.decode(pos, q1, k1, v1), f"{n_shards} shards")
    # each row is stored by exactly one shard, the new one included
    rows = np.zeros((pos + 1, G * d), np.float32)
    for r, c in enumerate(ctxs):
        kr, _ = c.kv_read(0, 0, 0, pos + 1)
        owned = (np.arange(pos + 1) // 256) % n_shards == r
        assert not kr[~owned].any()
        rows[owned] = kr[owned]
    np.testing.assert_array_equal(rows, o.kc[:pos + 1])


def test_cfg3_7b_prefill_2048_onto_4096_sampled_rows():
    """Config 3 shape: a 2048-token chunk appended onto 4096 cached rows. Row z
    of a prefill equals a decode at position 4096+z over the same cache, so the
    oracle checks a sample of rows (tile edges included) by its decode."""
    H, G, d = 28, 4, 128
    pos0, n = 4096, 2048
    g = make_ctx(H, G, d, pos0 + n)
    o = O.OracleLayer(H, G, d, pos0 + n)
    fill_both(g, o, 0, 0, pos0, 3000)
    q, k, v = normal(3001, (n, H * d), (n, G * d), (n, G * d))
    out = g.prefill(0, 0, pos0, q, k, v)
    o.fill(pos0, k, v)
    # rows 1408 onwards are in the query tiles split in two key ranges
    for z in (0, 1, 63, 64, 127, 128, 129, 1000, 1023, 1024, 1408, 1535, 1600, 1791, 1800, 2046, 2047):
        assert_attn_close(out[z], o.decode(pos0 + z, q[z], k[z], v[z]), f"prefill row {z}")
    kr, vr = g.kv_read(0, 0, pos0, n)
    np.testing.assert_array_equal(kr, o.kc[pos0:pos0 + n])


def test_cfg5_full_shape_batched_decode():
    """Config 5 at the bench's own shape: the 64 cached lengths ~U{1024..32768}
    (seed 5), 16Q/2KV heads, d 128, 256-token pages, one layer, all 64
    sequences in one batched decode call (the split-length choice and the
    replay of ragged splits at full size). Checked against the oracle on 10
    sequences: the shortest, the longest and 8 in between. Every sequence
    holds a prefix of one seeded block of rows, as in the bench."""
    H, G, d = 16, 2, 128
    lens = np.random.default_rng(5).integers(1024, 32769, 64)
    Lmax = int(lens.max())
    n = lens.size
    g = make_ctx(H, G, d, Lmax + 1, max_seqs=n, n_pages=int(sum((int(x) + 256) // 256 for x in lens)))
    k, v = normal(5005, (Lmax, G * d), (Lmax, G * d))
    for s, ln in enumerate(lens):
        g.append(0 + s, 0, 0, k[:int(ln)], v[:int(ln)])
    q, kn, vn = normal(5006, (n, H * d), (n, G * d), (n, G * d))
    out = g.decode_batch(0, np.arange(n, dtype=np.int32), lens.astype(np.int32), q, kn, vn)
    order = np.argsort(lens, kind="stable")
    check = sorted(set([int(order[0]), int(order[-1])] + [int(order[i]) for i in np.linspace(1, n - 2, 8).astype(int)]))
    o = O.OracleLayer(H, G, d, Lmax + 1)
    o.fill(0, k, v)
    for s in sorted(check, key=lambda s: int(lens[s])):
        p = int(lens[s])
        saved = o.kc[p].copy(), o.vc[p].copy()        # the oracle's decode writes row p
        ref = o.decode(p, q[s], kn[s], vn[s])
        o.kc[p], o.vc[p] = saved
        assert_attn_close(out[s], ref, f"cfg5 sequence {s}, {p} cached positions")


@pytest.mark.parametrize("n_shards,pos0,n", [(2, 2900, 200), (3, 0, 64), (8, 100, 37), (2, 255, 1)])
def test_kv_sharded_prefill_partials_merge_to_the_full_result(n_shards, pos0, n):
    """A prefill chunk on the multi-GPU split, emulated with one context per
    shard on one GPU: every shard stores the chunk rows of its own pages and
    returns its causal partial of the n queries; the LSE merge must equal
    kore's prefill (kore.cpp:1542-1563) row for row."""
    import torch
    H, G, d = 28, 4, 128
    ctxs = [make_ctx(H, G, d, 4096, shard_rank=r, shard_count=n_shards) for r in range(n_shards)]
    o = O.OracleLayer(H, G, d, 4096)
    if pos0:
        k, v = normal(80 + n_shards, (pos0, G * d), (pos0, G * d))
        for c in ctxs:
            c.append(0, 0, 0, k, v)
        o.fill(0, k, v)
    q1, k1, v1 = normal(81 + n, (n, H * d), (n, G * d), (n, G * d))
    ref = o.prefill(pos0, q1, k1, v1)
    dev = torch.device("cuda", 0)
    tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q1, k1, v1))
    pf = n * (H * d + H)
    parts = torch.empty(n_shards * pf, device=dev)
    for r, c in enumerate(ctxs):
        c.prefill_partial_dev(0, 0, pos0, n, tq, tk, tv, parts[r * pf:(r + 1) * pf])
        c.sync()
    out = torch.empty(n * H * d, device=dev)
    ctxs[0].lse_merge_batch_dev(n_shards, n, parts, out)
    ctxs[0].sync()
    assert_attn_close(out.cpu().numpy().reshape(n, H, d), ref, f"{n_shards} shards, prefill {pos0}+{n}")
    # each chunk row is stored by exactly one shard
    rows = np.zeros((n, G * d), np.float32)
    for r, c in enumerate(ctxs):
        kr, _ = c.kv_read(0, 0, pos0, n)
        owned = ((pos0 + np.arange(n)) // 256) % n_shards == r
        assert not kr[~owned].any()
        rows[owned] = kr[owned]
    np.testing.assert_array_equal(rows, o.kc[pos0:pos0 + n])
