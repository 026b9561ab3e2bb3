"""Pins the oracle (the C restatement of kore's attention) to the reference.

1. Against the committed golden hashes (tests/golden/kore_attn_golden.json),
   produced by running kore.cpp's own forward()/forward_batch(): the
   restatement's outputs must be bit-identical.
2. Against the reference engine compiled in place (oracle/_ref), live, on
   fresh seeded cases, when that library is present.
CPU only.
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle as O
from tests.golden.make_golden import CASES, case_inputs, run_case, sha

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "kore_attn_golden.json")


@pytest.fixture(scope="module")
def golden():
    with open(GOLDEN) as f:
        return json.load(f)["cases"]


@pytest.mark.parametrize("name", sorted(CASES))
def test_restatement_matches_reference_golden(golden, name):
    H, G, d, ctx, cached, n_pre, n_dec, seed = CASES[name]
    g = golden[name]
    ins = case_inputs(H, G, d, cached, n_pre, n_dec, seed)
    assert sha(*ins) == g["inputs_sha256"], "seeded generator drifted: inputs differ from the golden run"
    layer = O.OracleLayer(H, G, d, ctx)
    if n_pre:
        # the reference picked its AVX2 or scalar hd_dot at run time; restate the same branch
        orig = layer.prefill
        layer.prefill = lambda pos0, q, k, v: orig(pos0, q, k, v, avx2=g["avx2"])
    pre, dec, kc = run_case(layer, H, G, d, cached, n_pre, n_dec, ins)
    assert sha(kc) == g["kcache_sha256"], "rotated key rows differ from kore's cache"
    assert sha(pre) == g["prefill_sha256"], "prefill outputs differ from kore's"
    assert sha(dec) == g["decode_sha256"], "decode outputs differ from kore's"
    np.testing.assert_array_equal(pre.reshape(-1)[:8], np.float32(g["prefill_sample"]))
    np.testing.assert_array_equal(dec.reshape(-1)[:8], np.float32(g["decode_sample"]))


def test_inv_freq_and_angles_match_definition():
    inv = O.inv_freq(1e6, 128)
    want = np.array([np.float32(1e6 ** (-2.0 * i / 128)) for i in range(64)], np.float32)
    np.testing.assert_array_equal(inv, want)
    c, s = O.rope_angles(inv, 8192)
    np.testing.assert_array_equal(c, np.cos(8192.0 * inv.astype(np.float64)).astype(np.float32))
    np.testing.assert_array_equal(s, np.sin(8192.0 * inv.astype(np.float64)).astype(np.float32))


def test_hd_dot_avx2_order_differs_from_scalar_but_both_close():
    a, b = (np.random.default_rng(3).standard_normal((2, 128)).astype(np.float32))
    x = O.lib().korc_hd_dot(O._fp(a), O._fp(b), 128, 1)
    y = O.lib().korc_hd_dot(O._fp(a), O._fp(b), 128, 0)
    assert abs(x - y) < 1e-4 * np.abs(a * b).sum()


def test_argmax_first_of_ties():
    l = np.array([0.0, 3.0, 1.0, 3.0], np.float32)
    assert O.lib().korc_argmax(O._fp(l), 4) == 1


ref = pytest.mark.skipif(not O.ref_available(), reason="reference harness not built (no reference sources)")


@ref
@pytest.mark.parametrize("shape", [(14, 2, 64), (28, 4, 128), (16, 2, 128), (12, 2, 128), (40, 8, 128)])
def test_restatement_bitexact_live(shape):
    H, G, d = shape
    pos = 300
    ctx = 400
    q, k, v, kp, vp, pq, pk, pv = O.seeded_inputs(
        7, (H * d,), (G * d,), (G * d,), (pos, G * d), (pos, G * d), (12, H * d), (12, G * d), (12, G * d))
    a = O.OracleLayer(H, G, d, ctx)
    b = O.RefLayer(H, G, d, ctx)
    a.fill(0, kp, vp)
    b.fill(0, kp, vp)
    np.testing.assert_array_equal(a.kc, b.kc)
    np.testing.assert_array_equal(a.decode(pos, q, k, v), b.decode(pos, q, k, v))
    np.testing.assert_array_equal(a.prefill(pos + 1, pq, pk, pv, avx2=b.avx2), b.prefill(pos + 1, pq, pk, pv))
    np.testing.assert_array_equal(a.kc, b.kc)
    np.testing.assert_array_equal(a.vc, b.vc)


@ref
def test_reference_rejects_out_of_context_position():
    b = O.RefLayer(28, 4, 128, 64)
    q, k, v = O.seeded_inputs(1, (3584,), (512,), (512,))
    with pytest.raises(ValueError):
        b.decode(64, q, k, v)   # kore.cpp:1400: pos >= e.ctx -> forward() returns false
