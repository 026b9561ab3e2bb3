"""Shared helpers of the parity tests: seeded inputs and the tolerance of the
attention path (per head and token: max-abs error <= 2e-3 and max-abs error
relative to the largest reference magnitude <= 1e-3)."""
from __future__ import annotations

import numpy as np

ABS_TOL = 2e-3
REL_TOL = 1e-3


def attn_errors(out: np.ndarray, ref: np.ndarray):
    """Worst absolute and relative error over all (token, head) rows."""
    out = np.asarray(out, np.float32)
    ref = np.asarray(ref, np.float32)
    assert out.shape == ref.shape, (out.shape, ref.shape)
    d = out.shape[-1]
    o = out.reshape(-1, d).astype(np.float64)
    r = ref.reshape(-1, d).astype(np.float64)
    err = np.abs(o - r).max(axis=1)
    mag = np.maximum(np.abs(r).max(axis=1), 1e-30)
    return float(err.max()), float((err / mag).max())


def assert_attn_close(out, ref, what: str = "") -> None:
    assert np.isfinite(out).all(), f"{what}: non-finite output"
    a, r = attn_errors(out, ref)
    assert a <= ABS_TOL and r <= REL_TOL, f"{what}: max-abs {a:.3e} (tol {ABS_TOL}), rel {r:.3e} (tol {REL_TOL})"


def normal(seed: int, *shapes):
    g = np.random.default_rng(seed)
    return [g.standard_normal(s, dtype=np.float32) for s in shapes]
