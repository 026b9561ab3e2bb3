"""Generates tests/golden/kore_proj_golden.json from the REFERENCE engine.

Runs kore's own quantize_row_q8_K and its Q4_K / Q6_K dot kernels (AVX2 and
scalar; oracle/_ref/libkore_ref.so, compiled from the reference sources by
``make -C oracle ref``) on seeded inputs and records the SHA-256 of the
inputs and of the reference's outputs plus a few sample values.
tests/test_proj_oracle_pin.py checks the C restatement against these hashes
where the reference sources are absent.

Usage:  python tests/golden/make_proj_golden.py
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from kore_b200.qweights import Q4_K, Q6_K, random_qmat  # noqa: E402
from oracle import oracle as O  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "kore_proj_golden.json")

# Q8_K cases: name -> seed (inputs built by q8k_input)
Q8K_CASES = {"normal_7b": 1, "tiny_scale": 2, "zeros_and_ties": 3, "half_way": 4}

# product cases: name -> (type, rows, cols, seed)
MATVEC_CASES = {
    "q4k_7b_wk_512x3584": (Q4_K, 512, 3584, 11),
    "q4k_7b_wq_3584x3584": (Q4_K, 3584, 3584, 12),
    "q6k_7b_wv_512x3584": (Q6_K, 512, 3584, 13),
    "q4k_3b_2048x2048": (Q4_K, 256, 2048, 14),
    "q6k_small_16x256": (Q6_K, 16, 256, 15),
}


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def q8k_input(name: str, seed: int) -> np.ndarray:
    g = np.random.default_rng(seed)
    if name == "normal_7b":
        return g.standard_normal(3584, dtype=np.float32)
    if name == "tiny_scale":
        return (g.standard_normal(1024, dtype=np.float32) * np.float32(1e-4)).astype(np.float32)
    if name == "zeros_and_ties":
        x = g.standard_normal(1024, dtype=np.float32)
        x[0:256] = 0.0                         # an all-zero block
        x[256 + 10], x[256 + 20] = 3.0, -3.0   # the first of equal magnitudes wins
        x[256:256 + 5] = 0.0
        x[512 + 7], x[512 + 3] = -5.0, 5.0     # the positive one comes first
        x[768 + 100] = -0.0
        return x
    if name == "half_way":
        # maxv = -127 so that iscale = 1: the values sit on rounding ties
        x = np.zeros(256, np.float32)
        x[0] = -127.0
        ties = [0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 126.5, -126.5, 127.0, 63.5, -63.5, 100.25]
        x[1:1 + len(ties)] = ties
        x[20:] = g.uniform(-127, 127, 236).astype(np.float32)
        return x
    raise KeyError(name)


def matvec_inputs(qtype: int, rows: int, cols: int, seed: int):
    g = np.random.default_rng(seed)
    m = random_qmat(qtype, rows, cols, g)
    x = g.standard_normal(cols, dtype=np.float32)
    return m, x


def ref_matvec(m, x: np.ndarray, avx2: bool) -> np.ndarray:
    xq = O.ref_q8k_quantize(x)
    return np.array([O.ref_qdot(m.type, m.row(r), xq, avx2) for r in range(m.rows)], np.float32)


def main() -> None:
    if not O.ref_available():
        sys.exit("the reference library is missing: make -C oracle ref")
    have_avx2 = O.cpu_has_avx2()
    out = {"generator": "tests/golden/make_proj_golden.py", "avx2_on_generating_cpu": have_avx2,
           "q8k": {}, "matvec": {}}
    for name, seed in sorted(Q8K_CASES.items()):
        x = q8k_input(name, seed)
        d, qs, bs = O.ref_q8k_quantize(x)
        out["q8k"][name] = {"inputs_sha256": sha(x), "d_sha256": sha(d), "qs_sha256": sha(qs),
                            "bsums_sha256": sha(bs), "d_sample": [float(v) for v in d[:4]]}
    for name, (t, rows, cols, seed) in sorted(MATVEC_CASES.items()):
        m, x = matvec_inputs(t, rows, cols, seed)
        rec = {"inputs_sha256": sha(m.data, x)}
        for avx2 in (True, False):
            if avx2 and not have_avx2:
                continue
            y = ref_matvec(m, x, avx2)
            key = "avx2" if avx2 else "scalar"
            rec[key + "_sha256"] = sha(y)
            rec[key + "_sample"] = [float(v) for v in y[:4]]
        out["matvec"][name] = rec
    with open(OUT, "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
        f.write("\n")
    print("wrote", OUT)


if __name__ == "__main__":
    main()
