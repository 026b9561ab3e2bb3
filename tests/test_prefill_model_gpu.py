"""kore's prefill side on the GPU (kore_cuda_matmul_batch, kore_cuda_prefill)
against kore itself, through the C ABI.

* The float batched product of kore's forward_batch (matmul_batch_float:
  every weight block dequantised to fp32, one fused multiply-add per column
  in column order) is bit-exact with kore's own, for Q4_K and Q6_K matrices,
  the attention and the feed-forward shapes (a 18944-wide down projection)
  and batch sizes from 1 to beyond one 64-token tile.
* The whole prefill (embedding, RMSNorms, the float products, biases, RoPE,
  append, attention, residual adds, SwiGLU, the last token's logits and
  greedy token) is bit-exact with kore's forward_batch() whose attention
  region runs the same GPU attention; a prompt spanning several of kore's
  64-token chunks, done on the device in one call, gives logits within 2 %
  of kore's own chunked prefill.
* Greedy generation with the prompt and every decode step on the device:
  token IDs identical to kore's own flow (forward_batch chunks, then
  forward() + sample_token).
"""
import numpy as np
import pytest

import kore_b200 as K
import oracle.oracle as O
from kore_b200.qweights import Q4_K, Q6_K, random_qmat
from tests.test_step_gpu import device_model

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not O.engine_available(), reason="oracle/_ref/libkore_engine.so not built")]


@pytest.mark.parametrize("B", [1, 7, 64, 100])
def test_matmul_batch_bitexact_with_kore(B):
    H, G, D, E, FF = 28, 4, 128, 3584, 18944
    eng = O.GreedyEngine(1, 512, 4, 2, 512, 32, ctx=8, seed=1, threads=8)   # kore's engine, for its AVX2 choice
    rng = np.random.default_rng(300 + B)
    g = K.KoreCuda(1, H, G, D, 16)
    kvd = G * D
    mats = [random_qmat(Q4_K, E, E, rng), random_qmat(Q4_K, kvd, E, rng), random_qmat(Q6_K, kvd, E, rng),
            random_qmat(Q6_K, E, E, rng)]
    g.set_attn_weights(0, *mats)
    x = rng.standard_normal((B, E)).astype(np.float32)
    for which, m in enumerate(mats):
        got = g.matmul_batch(0, which, x, m.rows)
        ref = eng.matmul_batch_ref(m, x)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (which, B)
    g.close()


def test_matmul_batch_feed_forward_shapes_bitexact():
    L, E, H, G, FF, V = 1, 3584, 28, 4, 18944, 64
    eng = O.GreedyEngine(L, E, H, G, FF, V, ctx=8, seed=3, threads=8)
    g = device_model(eng, L, E, H, G, FF, V, 8)
    rng = np.random.default_rng(7)
    for which, name, cols in ((4, "ffn_gate", E), (5, "ffn_up", E), (6, "ffn_down", FF)):
        t, r, c, addr = eng.tensor(f"blk.0.{name}.weight")

        class M:
            pass
        m = M()
        m.type, m.rows, m.cols, m.addr = t, r, c, addr
        x = rng.standard_normal((9, cols)).astype(np.float32)
        got = g.matmul_batch(0, which, x, r)
        ref = eng.matmul_batch_ref(m, x)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), name
    g.close()


def test_prefill_is_kores_forward_batch_with_the_same_attention():
    """Bit for bit against kore's forward_batch() whose attention region is
    served by the same GPU attention (keng_forward_batch_cuda): every other
    operation of the prefill (embedding, RMSNorms, float products, biases,
    residual adds, SwiGLU, output norm, logits) is kore's own. The prefill
    attention itself is the tensor-core kernel, within tolerance of kore's
    (its split-bf16 operands hold values to ~2^-17), so kore's own
    forward_batch() is matched within 2 % of the logit scale."""
    import os
    L, E, H, G, FF, V = 2, 1024, 8, 2, 1280, 96
    eng = O.GreedyEngine(L, E, H, G, FF, V, ctx=80, seed=11, threads=4)
    eng.attach_cuda(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "kore_b200",
                                 "libkore_cuda.so"), 0)
    g = device_model(eng, L, E, H, G, FF, V, 80)
    toks = np.random.default_rng(12).integers(0, V, 40)
    for p0, n in ((0, 1), (1, 39)):
        iso = eng.forward_batch_cuda(toks[p0:p0 + n], p0)
        nxt, got = g.prefill_tokens(0, toks[p0:p0 + n], p0, want_logits=True)
        assert np.array_equal(got.view(np.uint32), iso.view(np.uint32)), (p0, n)
        assert nxt == int(np.argmax(iso))
    ref = eng.forward_batch_ref(toks[:40], 0)
    err = float(np.abs(got.astype(np.float64) - ref).max())
    assert err <= 2e-2 * max(1.0, float(np.abs(ref).max())), err
    g.close()


def test_prefill_of_several_chunks_in_one_call_tracks_kore():
    """kore prefills in 64-token chunks; the device takes the 150 tokens at
    once. Logits of the last token within the attention tolerance."""
    L, E, H, G, FF, V = 2, 2048, 16, 2, 2048, 128
    n = 150
    eng = O.GreedyEngine(L, E, H, G, FF, V, ctx=n + 8, seed=13, threads=8)
    toks = np.random.default_rng(14).integers(0, V, n)
    for p0 in range(0, n, 64):
        ref = eng.forward_batch_ref(toks[p0:p0 + 64], p0)
    g = device_model(eng, L, E, H, G, FF, V, n + 8)
    nxt, got = g.prefill_tokens(0, toks, 0, want_logits=True)
    scale = max(1.0, float(np.abs(ref).max()))
    err = float(np.abs(got.astype(np.float64) - ref).max())
    assert err <= 2e-2 * scale, err
    srt = np.sort(ref)
    if srt[-1] - srt[-2] > 2 * err:
        assert nxt == int(np.argmax(ref))
    g.close()


GREEDY = [
    ("7B-attention", 2, 3584, 28, 4, 3584, 512, 240, 32),
    ("3B-attention", 2, 2048, 16, 2, 2048, 512, 200, 72),
]


@pytest.mark.parametrize("geo", GREEDY, ids=[g[0] for g in GREEDY])
def test_greedy_ids_identical_with_prefill_and_decode_on_gpu(geo):
    name, L, E, H, G, FF, V, n_prompt, n_gen = geo
    eng = O.GreedyEngine(L, E, H, G, FF, V, ctx=n_prompt + n_gen + 8, seed=12345)
    prompt = np.random.default_rng(2024).integers(0, V, n_prompt)
    ref, margins = eng.generate_ref(prompt, n_gen)
    g = device_model(eng, L, E, H, G, FF, V, n_prompt + n_gen + 8)
    ids = [g.prefill_tokens(0, prompt, 0)[0]]
    for i in range(1, n_gen):
        ids.append(g.decode_step(0, ids[-1], n_prompt + i - 1)[0])
    got = np.array(ids)
    mismatch = np.nonzero(ref != got)[0]
    assert mismatch.size == 0, (
        f"{name}: first mismatch at step {mismatch[0]} (ref {ref[mismatch[0]]}, cuda {got[mismatch[0]]}, "
        f"reference top-1/top-2 margin there {margins[mismatch[0]]:.3g}; min margin {margins.min():.3g})")
    g.close()
