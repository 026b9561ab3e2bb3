"""Pins the restatement of kore's whole decode step (oracle/kore_step_oracle.c:
RMSNorm, Q8_K + Q4_K projections, attention, SwiGLU feed-forward, residual
adds, logits) to the reference: on a seeded random-init model inside the
reference engine (oracle/engine_harness.cpp), kore's own forward() and the
restatement, fed the same tokens at positions 0, 1, 2, ..., must give
bit-identical logits at every step. CPU only; needs the reference library.
"""
import numpy as np
import pytest

import oracle.oracle as O

needs_engine = pytest.mark.skipif(not O.engine_available(), reason="oracle/_ref/libkore_engine.so not built")

# (name, layers, n_embd, heads, kv heads, n_ff, vocab, steps)
GEOMETRIES = [
    ("2-layer d128 GQA 4:1", 2, 1024, 8, 2, 1280, 96, 12),
    ("3-layer d64 GQA 2:1", 3, 512, 8, 4, 768, 64, 10),
]


@needs_engine
@pytest.mark.parametrize("geo", GEOMETRIES, ids=[g[0] for g in GEOMETRIES])
def test_step_restatement_matches_kore_forward(geo):
    name, L, E, H, G, FF, V, steps = geo
    ctx = steps + 4
    eng = O.GreedyEngine(L, E, H, G, FF, V, ctx=ctx, seed=2026, threads=2)
    ora = O.StepOracle(eng, L, E, H, G, FF, V, ctx)
    tokens = np.random.default_rng(31).integers(0, V, steps)
    for pos, tok in enumerate(tokens.tolist()):
        ref = eng.forward_ref(tok, pos)
        got = ora.step(tok, pos)
        assert np.isfinite(ref).all()
        mism = np.nonzero(ref.view(np.uint32) != got.view(np.uint32))[0]
        assert mism.size == 0, (f"{name}, position {pos}: {mism.size} of {V} logits differ, first {mism[0]}: "
                                f"{got[mism[0]]!r} vs kore {ref[mism[0]]!r}")


@needs_engine
def test_step_restatement_greedy_ids_match_kore():
    """The greedy token of each step (kore's argmax rule) from the restatement's
    logits equals kore's own, over a short generation fed back token by token."""
    L, E, H, G, FF, V = 2, 512, 4, 2, 512, 80
    ctx = 20
    eng = O.GreedyEngine(L, E, H, G, FF, V, ctx=ctx, seed=7, threads=1)
    ora = O.StepOracle(eng, L, E, H, G, FF, V, ctx)
    tok_ref = tok_ora = 3
    for pos in range(16):
        lr = eng.forward_ref(tok_ref, pos)
        lo = ora.step(tok_ora, pos)
        tok_ref, tok_ora = O.ref_lib().kref_argmax(O._fp(lr), V), O.lib().korc_argmax(O._fp(lo), V)
        assert tok_ref == tok_ora, pos
