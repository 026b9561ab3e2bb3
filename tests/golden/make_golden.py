"""Generates tests/golden/kore_attn_golden.json from the REFERENCE engine.

Runs kore's own forward() / forward_batch() (oracle/_ref/libkore_ref.so,
compiled from the reference sources by ``make -C oracle ref``) on seeded
N(0,1) inputs and records, per case, the SHA-256 of the inputs and of the
reference's fp32 outputs plus a few sample values. The C restatement in
oracle/ is bit-exact with the reference, so tests/test_oracle_pin.py checks
it against these hashes on machines where the reference sources are absent.

Usage:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "kore_attn_golden.json")

# name: (H, G, d, ctx, cached rows, prefill tokens, decode steps, seed)
CASES = {
    # Qwen2.5-0.5B-shaped layer: prefill 128 tokens at 0..127, then 64 decode steps
    "cfg1_0p5b_prefill128_decode64": (14, 2, 64, 192, 0, 128, 64, 12345),
    # Qwen2.5-7B-shaped layer, decode at position 8192 over a seeded cache
    "cfg2_7b_decode_at_8192": (28, 4, 128, 8193, 8192, 0, 1, 20001),
    # Qwen2.5-7B-shaped layer, a kore-sized 64-token prefill chunk onto 4096 cached rows
    "cfg3_7b_prefill64_onto_4096": (28, 4, 128, 4160, 4096, 64, 0, 30001),
    # Qwen2.5-3B-shaped layer, decode across page boundaries (255, 256, 257)
    "cfg5_3b_decode_255_to_257": (16, 2, 128, 258, 255, 0, 3, 50001),
    # edge: decode at position 0 (empty cache) and 1
    "edge_7b_decode_pos0": (28, 4, 128, 2, 0, 0, 2, 60001),
}


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a, np.float32).tobytes())
    return h.hexdigest()


def case_inputs(H, G, d, cached, n_pre, n_dec, seed):
    E, kvd = H * d, G * d
    g = np.random.default_rng(seed)
    kc = g.standard_normal((cached, kvd), dtype=np.float32)
    vc = g.standard_normal((cached, kvd), dtype=np.float32)
    pq = g.standard_normal((n_pre, E), dtype=np.float32)
    pk = g.standard_normal((n_pre, kvd), dtype=np.float32)
    pv = g.standard_normal((n_pre, kvd), dtype=np.float32)
    dq = g.standard_normal((n_dec, E), dtype=np.float32)
    dk = g.standard_normal((n_dec, kvd), dtype=np.float32)
    dv = g.standard_normal((n_dec, kvd), dtype=np.float32)
    return kc, vc, pq, pk, pv, dq, dk, dv


def run_case(layer, H, G, d, cached, n_pre, n_dec, ins):
    """Drives `layer` (RefLayer or OracleLayer) through the case; returns
    (prefill outputs [n_pre,H,d], decode outputs [n_dec,H,d], final K cache rows)."""
    kc, vc, pq, pk, pv, dq, dk, dv = ins
    if cached:
        layer.fill(0, kc, vc)
    pre = layer.prefill(cached, pq, pk, pv) if n_pre else np.zeros((0, H, d), np.float32)
    dec = np.stack([layer.decode(cached + n_pre + i, dq[i], dk[i], dv[i]) for i in range(n_dec)]) \
        if n_dec else np.zeros((0, H, d), np.float32)
    end = cached + n_pre + n_dec
    return pre, dec, np.array(layer.kc[:end])


def main() -> None:
    O.build()
    if not O.ref_available():
        sys.exit("the reference harness is not built (needs the reference sources)")
    out = {"generator": "tests/golden/make_golden.py", "source": "kore.cpp forward()/forward_batch() via oracle/_ref",
           "rng": "numpy.random.default_rng(seed).standard_normal(dtype=float32)", "cases": {}}
    for name, (H, G, d, ctx, cached, n_pre, n_dec, seed) in CASES.items():
        ins = case_inputs(H, G, d, cached, n_pre, n_dec, seed)
        ref = O.RefLayer(H, G, d, ctx)
        pre, dec, kcache = run_case(ref, H, G, d, cached, n_pre, n_dec, ins)
        out["cases"][name] = {
            "H": H, "G": G, "d": d, "ctx": ctx, "cached": cached, "prefill": n_pre, "decode": n_dec, "seed": seed,
            "avx2": ref.avx2,
            "inputs_sha256": sha(*ins),
            "prefill_sha256": sha(pre), "decode_sha256": sha(dec), "kcache_sha256": sha(kcache),
            "prefill_sample": [float(x) for x in pre.reshape(-1)[:8]],
            "decode_sample": [float(x) for x in dec.reshape(-1)[:8]],
        }
        print(name, "done", flush=True)
    with open(OUT, "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", OUT)


if __name__ == "__main__":
    main()
