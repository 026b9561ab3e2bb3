"""GPU parity of the attention block's quantised projections, through the C ABI.

kore_cuda_qmatvec (kore's mv() + quant() for one uploaded matrix) must equal
the oracle's restatement of kore's Q8_K quantisation and AVX2 dot kernels
(pinned to the reference by tests/test_proj_oracle_pin.py) bit for bit, for
Q4_K and Q6_K at the 7B and 3B shapes. kore_cuda_attn_block_decode (the whole
attention block of a decode step) must equal the composition of the separate
entry points bit for bit, equal the oracle bit for bit where the attention is
exact (position 0: one key, weight 1), and stay within the attention
tolerance of the oracle elsewhere.
"""
import numpy as np
import pytest

import kore_b200 as K
from kore_b200.qweights import Q4_K, Q6_K, random_qmat
from oracle import oracle as O
from tests.attn_check import assert_attn_close, normal

pytestmark = pytest.mark.gpu

# (name, H, G, d, types of wq, wk, wv, wo)
GEOMS = [
    ("7b_q4km", 28, 4, 128, (Q4_K, Q4_K, Q6_K, Q4_K)),
    ("3b_q6k", 16, 2, 128, (Q6_K, Q6_K, Q6_K, Q6_K)),
    ("small_256", 4, 2, 64, (Q6_K, Q4_K, Q4_K, Q6_K)),
]


def make_weights(H, G, d, types, seed):
    E, kvd = H * d, G * d
    rng = np.random.default_rng(seed)
    rows = (E, kvd, kvd, E)
    mats = [random_qmat(t, r, E, rng) for t, r in zip(types, rows)]
    bq, bk, bv = (rng.standard_normal(n).astype(np.float32) * np.float32(0.5) for n in (E, kvd, kvd))
    return mats, (bq, bk, bv)


def setup_ctx(H, G, d, types, seed, ctx=4096, n_layer=1, layer=0):
    g = K.KoreCuda(n_layer, H, G, d, ctx)
    mats, biases = make_weights(H, G, d, types, seed)
    g.set_attn_weights(layer, *mats, *biases)
    return g, mats, biases


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("geo", GEOMS, ids=[g[0] for g in GEOMS])
def test_qmatvec_bitexact_with_oracle(geo):
    name, H, G, d, types = geo
    g, mats, biases = setup_ctx(H, G, d, types, seed=1)
    E = H * d
    rng = np.random.default_rng(2)
    xs = [rng.standard_normal(E).astype(np.float32),
          (rng.standard_normal(E) * 1e-3).astype(np.float32),
          (rng.standard_normal(E) * 40).astype(np.float32)]
    x = rng.standard_normal(E).astype(np.float32)
    x[:256] = 0.0   # an all-zero Q8_K block
    xs.append(x)
    for which in range(4):
        bias = biases[which] if which < 3 else None
        for i, x in enumerate(xs):
            got = g.qmatvec(0, which, x)
            ref = O.qmatvec(mats[which], x, bias, avx2=True)
            mism = np.nonzero(bits(got) != bits(ref))[0]
            assert mism.size == 0, (f"{name} which={which} x#{i}: {mism.size} rows differ, first row {mism[0]}: "
                                    f"{got[mism[0]]!r} vs {ref[mism[0]]!r}")


def test_qmatvec_zero_input_gives_bias():
    g, mats, biases = setup_ctx(28, 4, 128, GEOMS[0][4], seed=3)
    for which in range(3):
        got = g.qmatvec(0, which, np.zeros(28 * 128, np.float32))
        np.testing.assert_array_equal(bits(got), bits(np.float32(0) + biases[which]))
    np.testing.assert_array_equal(g.qmatvec(0, 3, np.zeros(28 * 128, np.float32)), 0)


@pytest.mark.parametrize("geo", GEOMS[:2], ids=[g[0] for g in GEOMS[:2]])
def test_block_decode_at_position_0_bitexact(geo):
    """One key: the attention output is v itself on both sides, so the whole
    block is exact integer/fixed-order float work."""
    name, H, G, d, types = geo
    g, mats, (bq, bk, bv) = setup_ctx(H, G, d, types, seed=4)
    o = O.OracleLayer(H, G, d, 16)
    xb = normal(5, (H * d,))[0]
    got = g.attn_block_decode(0, 0, 0, xb)
    q = O.qmatvec(mats[0], xb, bq)
    k = O.qmatvec(mats[1], xb, bk)
    v = O.qmatvec(mats[2], xb, bv)
    att = o.decode(0, q, k, v).reshape(-1)
    ref = O.qmatvec(mats[3], att)
    mism = np.nonzero(bits(got) != bits(ref))[0]
    assert mism.size == 0, f"{name}: {mism.size} of {ref.size} outputs differ (first {mism[0]})"


@pytest.mark.parametrize("geo,pos", [(GEOMS[0], 1500), (GEOMS[1], 511), (GEOMS[2], 300)],
                         ids=["7b_pos1500", "3b_pos511", "small_pos300"])
def test_block_decode_equals_composition_and_oracle(geo, pos):
    name, H, G, d, types = geo
    E, kvd = H * d, G * d
    ga, mats, (bq, bk, bv) = setup_ctx(H, G, d, types, seed=6)
    gb, _, _ = setup_ctx(H, G, d, types, seed=6)
    o = O.OracleLayer(H, G, d, 4096)
    k0, v0 = normal(7, (pos, kvd), (pos, kvd))
    for g in (ga, gb):
        g.append(0, 0, 0, k0, v0)
    o.fill(0, k0, v0)
    xb = normal(8, (E,))[0]
    blk = ga.attn_block_decode(0, 0, pos, xb)
    # the same step through the separate entry points
    q, k, v = gb.qmatvec(0, 0, xb), gb.qmatvec(0, 1, xb), gb.qmatvec(0, 2, xb)
    att = gb.decode(0, 0, pos, q, k, v).reshape(-1)
    comp = gb.qmatvec(0, 3, att)
    np.testing.assert_array_equal(bits(blk), bits(comp))
    # projections exact, attention within tolerance of the oracle
    rq, rk, rv = O.qmatvec(mats[0], xb, bq), O.qmatvec(mats[1], xb, bk), O.qmatvec(mats[2], xb, bv)
    np.testing.assert_array_equal(bits(q), bits(rq))
    np.testing.assert_array_equal(bits(k), bits(rk))
    np.testing.assert_array_equal(bits(v), bits(rv))
    ratt = o.decode(pos, rq, rk, rv)
    assert_attn_close(att.reshape(H, d), ratt, f"{name} attention at {pos}")
    # the new token's rows in the cache are kore's
    kr, vr = ga.kv_read(0, 0, pos, 1)
    np.testing.assert_array_equal(kr[0], o.kc[pos])
    np.testing.assert_array_equal(vr[0], o.vc[pos])
    # Wo of the attention output: the Q8_K rounding of att can move by one
    # step where att moved within tolerance; the result stays close
    ref = O.qmatvec(mats[3], ratt.reshape(-1))
    err = np.abs(blk.astype(np.float64) - ref).max()
    assert err <= 2e-2 * max(1.0, float(np.abs(ref).max())), (name, err)


def test_block_decode_dev_matches_host():
    import torch
    H, G, d = 28, 4, 128
    E = H * d
    ga, _, _ = setup_ctx(H, G, d, GEOMS[0][4], seed=9, n_layer=2, layer=1)
    gb, _, _ = setup_ctx(H, G, d, GEOMS[0][4], seed=9, n_layer=2, layer=1)
    k0, v0 = normal(10, (700, G * d), (700, G * d))
    for g in (ga, gb):
        g.append(0, 1, 0, k0, v0)
    dev = torch.device("cuda", 0)
    outs_h, outs_d = [], []
    for step in range(3):
        xb = normal(11 + step, (E,))[0]
        outs_h.append(ga.attn_block_decode(0, 1, 700 + step, xb))
        txb = torch.from_numpy(xb).to(dev)
        to = torch.empty(E, device=dev)
        gb.attn_block_decode_dev(0, 1, 700 + step, txb, to)
        gb.sync()
        outs_d.append(to.cpu().numpy())
    for a, b in zip(outs_h, outs_d):
        np.testing.assert_array_equal(bits(a), bits(b))


def test_block_errors_are_reported():
    g = K.KoreCuda(2, 28, 4, 128, 256)
    with pytest.raises(K.KoreCudaError) as e:
        g.attn_block_decode(0, 0, 0, np.zeros(28 * 128, np.float32))
    assert e.value.code == -5   # no weights uploaded: KORE_CUDA_ESTATE
    mats, biases = make_weights(28, 4, 128, GEOMS[0][4], 12)
    with pytest.raises(K.KoreCudaError) as e:
        g.set_attn_weights(0, mats[1], mats[1], mats[2], mats[3], *biases)   # wq with wk's shape
    assert e.value.code == -1
    with pytest.raises(K.KoreCudaError) as e:
        g.set_attn_weights(2, *mats, *biases)   # layer out of range
    assert e.value.code == -2
    g.set_attn_weights(0, *mats, *biases)
    with pytest.raises(K.KoreCudaError) as e:
        g.attn_block_decode(0, 0, 5, np.zeros(28 * 128, np.float32))   # rows 0..4 missing
    assert e.value.code == -5
    with pytest.raises(K.KoreCudaError) as e:
        g.qmatvec(1, 0, np.zeros(28 * 128, np.float32))   # layer 1 has no weights
    assert e.value.code == -5
    # the context stays usable
    out = g.attn_block_decode(0, 0, 0, np.ones(28 * 128, np.float32))
    assert np.isfinite(out).all()
