"""The whole decode step on the GPU (kore_cuda_set_model + kore_cuda_decode_step)
against kore itself, through the C ABI.

The model is kore's own: a seeded random-init Qwen2-style model built inside
the reference engine (oracle/engine_harness.cpp, kore.cpp compiled in
place), whose tensors are uploaded as they are. Checks:

* position 0 (one key, so the attention is exact on both sides): the logits
  equal kore's forward() bit for bit (embedding, RMSNorms, Q8_K
  quantisations, Q4_K products, biases, attention, residual adds, SwiGLU
  with the C library's expf, output norm and logits) and the token is kore's
  greedy choice; also with the embedding table in each type get_row reads;
* positions 0..N with the tokens fed in: logits bit-identical to kore's
  control flow with its attention region on the same GPU attention (so
  every other operation is kore's), within 2 % of kore's own logits (kore's
  Q8_K quantisation amplifies the attention's ~1e-7 difference), and the
  greedy token kore's wherever its top-1/top-2 margin is not a near tie;
* greedy generation in kore's own flow (prompt in 64-token chunks, then
  decode steps): identical token IDs with every decode step on the device;
* steps chained on the device (the next token never leaves the GPU) give
  the same tokens as host steps; bad tokens and missing weights are errors.
"""
import os

import numpy as np
import pytest

import kore_b200 as K
import oracle.oracle as O

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not O.engine_available(), reason="oracle/_ref/libkore_engine.so not built")]

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(REPO, "kore_b200", "libkore_cuda.so")


class _Mat:
    """A matrix of the engine's model by address (type, rows, cols, addr)."""

    def __init__(self, t, r, c, addr):
        self.type, self.rows, self.cols, self.addr = t, r, c, addr


def engine_model(eng, n_layer):
    def qm(name):
        return _Mat(*eng.tensor(name))

    def f(name):
        return eng.tensor(name)[3]

    layers = []
    for l in range(n_layer):
        b = f"blk.{l}."
        layers.append(dict(wq=qm(b + "attn_q.weight"), wk=qm(b + "attn_k.weight"), wv=qm(b + "attn_v.weight"),
                           wo=qm(b + "attn_output.weight"), bq=f(b + "attn_q.bias"), bk=f(b + "attn_k.bias"),
                           bv=f(b + "attn_v.bias"), attn_norm=f(b + "attn_norm.weight"),
                           ffn_norm=f(b + "ffn_norm.weight"), w_gate=qm(b + "ffn_gate.weight"),
                           w_up=qm(b + "ffn_up.weight"), w_down=qm(b + "ffn_down.weight")))
    return dict(tok_embd=qm("token_embd.weight"), out_norm=f("output_norm.weight"), out_w=qm("output.weight"),
                layers=layers)


def device_model(eng, L, E, H, G, FF, V, ctx, tok_embd=None):
    g = K.KoreCuda(L, H, G, E // H, ctx, rope_base=1e6)   # inv_freq built as kore.cpp:1339 builds it
    m = engine_model(eng, L)
    if tok_embd is not None:
        m["tok_embd"] = tok_embd
    g.set_model(FF, V, O.engine_lib().keng_rms_eps(eng.h), m["tok_embd"], m["out_norm"], m["out_w"], m["layers"])
    return g


def kore_argmax(logits):
    return int(np.argmax(logits))   # numpy keeps the first of equal maxima, as std::max_element


# (name, layers, n_embd, heads, kv heads, n_ff, vocab, positions)
GEOMETRIES = [
    ("2-layer d128 GQA 4:1", 2, 1024, 8, 2, 1280, 96, 12),
    ("3-layer d64 GQA 2:1", 3, 512, 8, 4, 768, 64, 10),
    ("7B-shaped layer, n_ff 18944", 1, 3584, 28, 4, 18944, 256, 6),
]


@pytest.mark.parametrize("geo", GEOMETRIES, ids=[g[0] for g in GEOMETRIES])
def test_step_tracks_kore_forward(geo):
    """Against kore's own forward() at every position: bit for bit at
    position 0 (one key, so the attention is exact on both sides); beyond it
    the attention differs from kore's scalar loop by ~1e-7 and kore's own
    Q8_K quantisation of the attention output amplifies that into logit
    differences of up to about a percent, so the logits are held to 2 % of
    their scale and the greedy token to kore's wherever kore's top-1/top-2
    margin is not a near tie. Against kore's control flow with its attention
    region on the same GPU attention (keng_forward_cuda): bit for bit at
    every position, which proves every other operation of the step is kore's."""
    import os
    name, L, E, H, G, FF, V, steps = geo
    ctx = steps + 4
    eng = O.GreedyEngine(L, E, H, G, FF, V, ctx=ctx, seed=2026, threads=4)
    twin = O.GreedyEngine(L, E, H, G, FF, V, ctx=ctx, seed=2026, threads=4)   # same model
    twin.attach_cuda(os.path.join(REPO, "kore_b200", "libkore_cuda.so"), 0)
    g = device_model(eng, L, E, H, G, FF, V, ctx)
    tokens = np.random.default_rng(31).integers(0, V, steps).tolist()
    for pos, tok in enumerate(tokens):
        ref = eng.forward_ref(tok, pos)
        iso = twin.forward_cuda(tok, pos)
        nxt, got = g.decode_step(0, tok, pos, want_logits=True)
        assert np.isfinite(got).all()
        mism = np.nonzero(iso.view(np.uint32) != got.view(np.uint32))[0]
        assert mism.size == 0, f"{name}, position {pos}: {mism.size} of {V} logits differ from kore with the GPU attention"
        if pos == 0:   # one key: every step of the computation is kore's own
            mism = np.nonzero(ref.view(np.uint32) != got.view(np.uint32))[0]
            assert mism.size == 0, f"{name}: {mism.size} of {V} logits differ at position 0"
        scale = max(1.0, float(np.abs(ref).max()))
        err = float(np.abs(got.astype(np.float64) - ref).max())
        assert err <= 2e-2 * scale, f"{name}, position {pos}: max |logit error| {err:.3g} (scale {scale:.3g})"
        srt = np.sort(ref)
        if srt[-1] - srt[-2] > 2 * err:
            assert nxt == kore_argmax(ref), f"{name}, position {pos}: token {nxt} vs kore {kore_argmax(ref)}"
    g.close()


def _tables(V, E, rng):
    """An embedding table of each type kore's get_row reads, with its rows
    dequantised by kore's own get_row."""
    from kore_b200.qweights import Q4_K, Q6_K, random_qmat
    out = []
    f16 = rng.standard_normal((V, E)).astype(np.float16)
    out.append(_Mat(1, V, E, 0))
    out[-1].data = f16.view(np.uint8).reshape(-1)
    bf = (rng.standard_normal((V, E)).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    out.append(_Mat(30, V, E, 0))
    out[-1].data = bf.view(np.uint8).reshape(-1)
    for t in (Q4_K, Q6_K):
        m = random_qmat(t, V, E, rng, sigma=1.0)
        out.append(_Mat(t, V, E, 0))
        out[-1].data = m.data
    for m in out:
        m.addr = m.data.ctypes.data
        m.f32 = np.stack([O.ref_get_row(m.type, V, E, m.data, r) for r in range(V)]).astype(np.float32)
    return out


def test_step_embedding_types_bitexact_at_position_0():
    L, E, H, G, FF, V = 2, 512, 4, 2, 512, 32
    eng = O.GreedyEngine(L, E, H, G, FF, V, ctx=8, seed=91, threads=2)
    for tab in _tables(V, E, np.random.default_rng(92)):
        g = device_model(eng, L, E, H, G, FF, V, 8, tok_embd=tab)
        ora = O.StepOracle(eng, L, E, H, G, FF, V, 8)
        ora.model.tok_embd = tab.f32.ctypes.data   # kore's get_row of every row
        for tok in (0, 7, V - 1):
            g.seq_reset(0)
            ora_logits = ora.step(tok, 0)
            nxt, got = g.decode_step(0, tok, 0, want_logits=True)
            assert np.array_equal(got.view(np.uint32), ora_logits.view(np.uint32)), (tab.type, tok)
            assert nxt == kore_argmax(ora_logits)
        g.close()


GREEDY = [
    ("7B-attention", 2, 3584, 28, 4, 3584, 512, 240, 32),
    ("3B-attention", 2, 2048, 16, 2, 2048, 512, 200, 72),
]


@pytest.mark.parametrize("geo", GREEDY, ids=[g[0] for g in GREEDY])
def test_greedy_ids_identical_with_the_decode_step_on_gpu(geo):
    name, L, E, H, G, FF, V, n_prompt, n_gen = geo
    eng = O.GreedyEngine(L, E, H, G, FF, V, ctx=n_prompt + n_gen + 8, seed=12345)
    prompt = np.random.default_rng(2024).integers(0, V, n_prompt)
    ref, margins = eng.generate_ref(prompt, n_gen)
    eng.attach_cuda(LIB, 0)
    got = eng.generate_cuda_step(prompt, n_gen)
    mismatch = np.nonzero(ref != got)[0]
    assert mismatch.size == 0, (
        f"{name}: first mismatch at step {mismatch[0]} (ref {ref[mismatch[0]]}, cuda {got[mismatch[0]]}, "
        f"reference top-1/top-2 margin there {margins[mismatch[0]]:.3g}; min margin {margins.min():.3g})")


def test_steps_chained_on_the_device_match_host_steps():
    import torch
    L, E, H, G, FF, V = 2, 1024, 8, 2, 1280, 96
    n = 20
    eng = O.GreedyEngine(L, E, H, G, FF, V, ctx=n + 4, seed=5, threads=2)
    a = device_model(eng, L, E, H, G, FF, V, n + 4)
    b = device_model(eng, L, E, H, G, FF, V, n + 4)
    toks = [3]
    for pos in range(n):
        toks.append(a.decode_step(0, toks[-1], pos)[0])
    dev = torch.device("cuda", 0)
    t = torch.tensor([3], dtype=torch.int32, device=dev)
    chain = []
    for pos in range(n):
        b.decode_step_dev(0, t, pos, t)      # the next token overwrites the input on the device
        b.sync()
        chain.append(int(t.item()))
    assert chain == toks[1:]
    a.close()
    b.close()


def test_step_errors_are_codes():
    import torch
    L, E, H, G, FF, V = 1, 512, 4, 2, 512, 32
    eng = O.GreedyEngine(L, E, H, G, FF, V, ctx=8, seed=3, threads=1)
    bare = K.KoreCuda(L, H, G, E // H, 8)
    with pytest.raises(K.KoreCudaError) as e:
        bare.n_vocab = V
        bare.decode_step(0, 1, 0)
    assert e.value.code == -5          # no model uploaded
    bare.close()
    g = device_model(eng, L, E, H, G, FF, V, 8)
    with pytest.raises(K.KoreCudaError) as e:
        g.decode_step(0, V, 0)
    assert e.value.code == -2          # forward() returns false for a bad token
    with pytest.raises(K.KoreCudaError) as e:
        g.decode_step(0, 1, 3)
    assert e.value.code == -5          # positions 0..2 were never written
    t = torch.tensor([V + 5], dtype=torch.int32, device="cuda")
    g.decode_step_dev(0, t, 0, t)
    with pytest.raises(K.KoreCudaError) as e:
        g.sync()
    assert e.value.code == -6 and "vocabulary" in str(e.value)
    nxt, _ = g.decode_step(0, 1, 0)    # still usable
    assert 0 <= nxt < V
    g.close()
