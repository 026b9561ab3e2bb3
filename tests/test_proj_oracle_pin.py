"""Pins the projection oracle (the C restatement of kore's Q8_K quantisation
and its Q4_K / Q6_K dot kernels) to the reference.

1. Against the committed golden hashes (tests/golden/kore_proj_golden.json),
   produced by running kore.cpp's own quantize_row_q8_K and dot kernels:
   bit-identical outputs.
2. Against the reference compiled in place (oracle/_ref), live, on fresh
   seeded rows, when that library is present: both of kore's kernels (AVX2
   and scalar), including the fused multiply-add kore's compiler forms in the
   AVX2 Q6_K kernel's offset term.
CPU only.
"""
import json
import os

import numpy as np
import pytest

from kore_b200.qweights import Q4_K, Q6_K, QMat, random_qmat
from oracle import oracle as O
from tests.golden.make_proj_golden import MATVEC_CASES, Q8K_CASES, matvec_inputs, q8k_input, sha

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "kore_proj_golden.json")


@pytest.fixture(scope="module")
def golden():
    with open(GOLDEN) as f:
        return json.load(f)


@pytest.mark.parametrize("name", sorted(Q8K_CASES))
def test_q8k_restatement_matches_reference_golden(golden, name):
    g = golden["q8k"][name]
    x = q8k_input(name, Q8K_CASES[name])
    assert sha(x) == g["inputs_sha256"], "seeded generator drifted"
    d, qs, bs = O.q8k_quantize(x)
    assert sha(d) == g["d_sha256"]
    assert sha(qs) == g["qs_sha256"]
    assert sha(bs) == g["bsums_sha256"]


@pytest.mark.parametrize("name", sorted(MATVEC_CASES))
def test_qmatvec_restatement_matches_reference_golden(golden, name):
    g = golden["matvec"][name]
    t, rows, cols, seed = MATVEC_CASES[name]
    m, x = matvec_inputs(t, rows, cols, seed)
    assert sha(m.data, x) == g["inputs_sha256"], "seeded generator drifted"
    for key, avx2 in (("avx2", True), ("scalar", False)):
        if key + "_sha256" in g:
            y = O.qmatvec(m, x, avx2=avx2)
            assert sha(y) == g[key + "_sha256"], f"{key} restatement differs from kore's kernel"


def test_q8k_half_way_values_round_to_even():
    x = q8k_input("half_way", Q8K_CASES["half_way"])
    d, qs, _ = O.q8k_quantize(x)
    # maxv = -127 -> iscale = 1 -> q = rint(-x) ... with the sign flip of -127/maxv = +1
    assert d[0] == np.float32(1.0)
    assert list(qs[1:13]) == [0, 2, 2, 0, -2, -2, 126, -126, 127, 64, -64, 100]


needs_ref = pytest.mark.skipif(not O.ref_available(), reason="reference library not built (make -C oracle ref)")


@needs_ref
@pytest.mark.parametrize("qtype", [Q4_K, Q6_K])
def test_restatement_matches_live_reference(qtype):
    rng = np.random.default_rng(100 + qtype)
    avx2_modes = (True, False) if O.cpu_has_avx2() else (False,)
    for trial in range(60):
        cols = 256 * int(rng.integers(1, 20))
        x = (rng.standard_normal(cols) * rng.uniform(1e-3, 30)).astype(np.float32)
        if trial % 5 == 0:
            x[rng.integers(0, cols, cols // 8)] = 0.0
        xq = O.q8k_quantize(x)
        for a, b in zip(xq, O.ref_q8k_quantize(x)):
            np.testing.assert_array_equal(a, b)
        m = random_qmat(qtype, 8, cols, rng, sigma=float(rng.uniform(1e-3, 0.1)))
        for avx2 in avx2_modes:
            for r in range(m.rows):
                mine, ref = O.qdot(qtype, m.row(r), xq, avx2), O.ref_qdot(qtype, m.row(r), xq, avx2)
                assert mine.view(np.uint32) == ref.view(np.uint32), (trial, r, avx2, mine, ref)


@needs_ref
def test_restatement_matches_live_reference_on_extreme_blocks():
    """All-ones and all-zero nibbles, extreme 6-bit scales and mins, negative
    Q6_K scales of -128: the integer lanes at their limits."""
    rng = np.random.default_rng(7)
    cols = 512
    x = rng.standard_normal(cols).astype(np.float32)
    xq = O.q8k_quantize(x)
    q4 = np.zeros((2 * 2, 144), np.uint8)
    q4[:, 4:16] = 0xFF          # every scale and min 63
    q4[0:2, 16:] = 0xFF         # nibbles 15
    q4[2:4, 16:] = 0x00         # nibbles 0
    q4[:, 0:2] = np.frombuffer(np.float16(0.01).tobytes(), np.uint8)
    q4[:, 2:4] = np.frombuffer(np.float16(0.02).tobytes(), np.uint8)
    q6 = np.full((2 * 2, 210), 0xFF, np.uint8)
    q6[:, 192:208] = 0x80       # scales -128
    q6[:, 208:210] = np.frombuffer(np.float16(0.001).tobytes(), np.uint8)
    for qtype, blocks in ((Q4_K, q4), (Q6_K, q6)):
        m = QMat(qtype, 2, cols, blocks.reshape(-1))
        for avx2 in ((True, False) if O.cpu_has_avx2() else (False,)):
            for r in range(2):
                mine, ref = O.qdot(qtype, m.row(r), xq, avx2), O.ref_qdot(qtype, m.row(r), xq, avx2)
                assert mine.view(np.uint32) == ref.view(np.uint32)
