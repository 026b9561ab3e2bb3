// engine_harness.cpp — greedy token-ID parity: the REFERENCE engine against
// the same engine with its attention regions, or its whole attention blocks,
// served by the CUDA library.
//
// TEST INFRASTRUCTURE ONLY. oracle/Makefile compiles this file with kore's own
// flags (build.sh:10, -std=c++20 -O3 -pthread) into
// oracle/_ref/libkore_engine.so; the reference source is included from where
// it lies (KORE_REF_SRC), never copied. Nothing in the product links it.
//
// A seeded random-init Qwen2-style model is built in memory: the tensors
// engine_init asks for (kore.cpp:1316-1330), projection weights as Q4_K blocks
// of random nibbles and scales (valid by construction: every byte pattern
// decodes), norms near 1 and biases as F32, token embeddings as F32. Three
// greedy decoders then run on it:
//   * the reference: kore's forward_batch() over the prompt in chunks of
//     e.bsz tokens, then forward() + sample_token(temp 0) per generated token
//     (the CLI's flow, kore.cpp:1720-1750, :2794-2812);
//   * the CUDA path: the same control flow with the same helpers (get_row,
//     rmsnorm, quant, mv, matmul_batch_float, the SwiGLU and residual adds),
//     where the attention regions kore inlines (kore.cpp:1424-1455 and
//     :1535-1563: RoPE, cache append, attention) are replaced by one call
//     each to kore_cuda_attn_decode / kore_cuda_attn_prefill, resolved from
//     the library with dlopen. The projections see the same inputs in the
//     same order, so the only arithmetic that differs is the attention's.
//   * the CUDA block path: as the CUDA path, but each decode step's whole
//     attention block (kore.cpp:1419-1457: Q8_K quantisation of xb, the
//     Wq/Wk/Wv products and biases, the attention, the quantisation of att
//     and Wo) is one call to kore_cuda_attn_block_decode, with kore's own
//     weight tensors uploaded once by kore_cuda_set_attn_weights.
// The test compares the ID sequences; the reference's top-1/top-2 logit
// margin per step is returned so that a mismatch can be told apart from a
// near tie.

#define main kore_ref_main
#include KORE_REF_SRC
#undef main

#include <dlfcn.h>

#include <memory>
#include <string>

#include "kore_cuda.h"

namespace {

using fn_cfg_default = void (*)(kore_cuda_cfg *, int, int, int, int, int);
using fn_create = int (*)(kore_cuda_ctx **, const kore_cuda_cfg *);
using fn_destroy = void (*)(kore_cuda_ctx *);
using fn_last_error = const char *(*)(const kore_cuda_ctx *);
using fn_seq_reset = int (*)(kore_cuda_ctx *, int);
using fn_decode = int (*)(kore_cuda_ctx *, int, int, int, const float *, const float *, const float *, float *);
using fn_prefill = int (*)(kore_cuda_ctx *, int, int, int, int, const float *, const float *, const float *, float *);
using fn_set_weights = int (*)(kore_cuda_ctx *, int, const kore_cuda_qmat *, const kore_cuda_qmat *,
                               const kore_cuda_qmat *, const kore_cuda_qmat *, const float *, const float *,
                               const float *);
using fn_block = int (*)(kore_cuda_ctx *, int, int, int, const float *, float *);
using fn_set_model = int (*)(kore_cuda_ctx *, const kore_cuda_model *);
using fn_step = int (*)(kore_cuda_ctx *, int, int, int, int *, float *);

struct Harness {
    Model m;
    Engine e;
    std::vector<std::vector<uint8_t>> store;
    std::string err;
    // CUDA library
    void *lib = nullptr;
    kore_cuda_ctx *ctx = nullptr;
    fn_destroy destroy = nullptr;
    fn_last_error last_error = nullptr;
    fn_seq_reset seq_reset = nullptr;
    fn_decode decode = nullptr;
    fn_prefill prefill = nullptr;
    fn_set_weights set_weights = nullptr;
    fn_block block = nullptr;
    fn_set_model set_model = nullptr;
    fn_step step = nullptr;
    bool weights_up = false;
    bool model_up = false;
};

uint16_t f32_to_f16(float f) {   // round to nearest, normal and subnormal range
    uint32_t u;
    memcpy(&u, &f, 4);
    const uint32_t sign = (u >> 16) & 0x8000u;
    const int exp = (int)((u >> 23) & 0xFF) - 127 + 15;
    uint32_t mant = u & 0x7FFFFFu;
    if (exp >= 31) return (uint16_t)(sign | 0x7C00u);
    if (exp <= 0) {
        if (exp < -10) return (uint16_t)sign;
        mant |= 0x800000u;
        const int shift = 14 - exp;
        return (uint16_t)(sign | ((mant + (1u << (shift - 1))) >> shift));
    }
    return (uint16_t)(sign | (uint32_t)(exp << 10) | ((mant + 0x1000u) >> 13));
}

Tensor new_tensor(Harness &hx, uint32_t type, uint64_t cols, uint64_t rows, uint64_t bytes) {
    hx.store.emplace_back(bytes, 0);
    Tensor t;
    t.type = type;
    t.n_dims = rows > 1 ? 2 : 1;
    t.dims[0] = cols;
    t.dims[1] = rows;
    t.nbytes = bytes;
    t.data = hx.store.back().data();
    return t;
}

// Q4_K weights: value = d*sc*q - dmin*mn (kore.cpp:337-354) with random q,
// sc, mn; d and dmin chosen so that the weights have a standard deviation of
// roughly `sigma`.
Tensor q4k_random(Harness &hx, uint64_t cols, uint64_t rows, float sigma, std::mt19937_64 &rng) {
    const uint64_t nb = cols / 256 * rows;
    Tensor t = new_tensor(hx, GGML_Q4_K, cols, rows, nb * 144);
    uint8_t *p = hx.store.back().data();
    const float d = sigma / 270.0f, dmin = 7.5f * d;
    const uint16_t hd = f32_to_f16(d), hm = f32_to_f16(dmin);
    for (uint64_t b = 0; b < nb; b++) {
        uint8_t *blk = p + b * 144;
        for (int i = 4; i < 144; i += 8) {
            const uint64_t r = rng();
            memcpy(blk + i, &r, std::min(8, 144 - i));
        }
        blk[0] = (uint8_t)(hd & 0xFF); blk[1] = (uint8_t)(hd >> 8);
        blk[2] = (uint8_t)(hm & 0xFF); blk[3] = (uint8_t)(hm >> 8);
    }
    return t;
}

Tensor f32_random(Harness &hx, uint64_t cols, uint64_t rows, float mean, float sd, std::mt19937_64 &rng) {
    Tensor t = new_tensor(hx, GGML_F32, cols, rows, cols * rows * 4);
    float *p = (float *)hx.store.back().data();
    std::normal_distribution<float> nd(mean, sd);
    for (uint64_t i = 0; i < cols * rows; i++) p[i] = nd(rng);
    return t;
}

int argmax_margin(const std::vector<float> &logits, float *margin) {
    std::mt19937 rng(0);
    const int best = sample_token(logits, 0.0f, 1, rng);   // kore's greedy rule (kore.cpp:1601-1603)
    float second = -INFINITY;
    for (size_t i = 0; i < logits.size(); i++)
        if ((int)i != best && logits[i] > second) second = logits[i];
    if (margin) *margin = logits[(size_t)best] - second;
    return best;
}

// --- the CUDA path: kore's control flow, attention through the library

bool cuda_forward(Harness &hx, int token, int pos, bool want_logits) {
    Engine &e = hx.e;
    const Hparams &h = e.hp;
    const int E = (int)h.n_embd, FF = (int)h.n_ff, kvd = e.kv_dim;
    if (token < 0 || token >= e.n_vocab || pos < 0 || pos >= e.ctx) return false;
    if (!get_row(*e.tok_embd, (uint64_t)token, e.emb)) return false;
    std::copy(e.emb.begin(), e.emb.begin() + E, e.x.begin());
    for (uint32_t l = 0; l < h.n_layer; l++) {
        const Layer &L = e.layers[l];
        rmsnorm(e.xb.data(), e.x.data(), L.attn_norm, E, h.rms_eps);
        quant(e, e.xb.data(), e.xq_e.data(), E);
        mv(e, *L.wq, e.xb.data(), e.xq_e.data(), e.q.data());
        mv(e, *L.wk, e.xb.data(), e.xq_e.data(), e.k.data());
        mv(e, *L.wv, e.xb.data(), e.xq_e.data(), e.v.data());
        for (int i = 0; i < E; i++) e.q[(size_t)i] += L.bq[i];
        for (int i = 0; i < kvd; i++) {
            e.k[(size_t)i] += L.bk[i];
            e.v[(size_t)i] += L.bv[i];
        }
        if (hx.decode(hx.ctx, 0, (int)l, pos, e.q.data(), e.k.data(), e.v.data(), e.att.data()) != KORE_CUDA_OK) {
            hx.err = hx.last_error(hx.ctx);
            return false;
        }
        quant(e, e.att.data(), e.xq_e.data(), E);
        mv(e, *L.wo, e.att.data(), e.xq_e.data(), e.o.data());
        for (int i = 0; i < E; i++) e.x[(size_t)i] += e.o[(size_t)i];
        rmsnorm(e.xb.data(), e.x.data(), L.ffn_norm, E, h.rms_eps);
        quant(e, e.xb.data(), e.xq_e.data(), E);
        mv(e, *L.w_gate, e.xb.data(), e.xq_e.data(), e.gate.data());
        mv(e, *L.w_up, e.xb.data(), e.xq_e.data(), e.up.data());
        for (int i = 0; i < FF; i++) {
            const float g = e.gate[(size_t)i];
            e.gate[(size_t)i] = g / (1.0f + std::exp(-g)) * e.up[(size_t)i];
        }
        quant(e, e.gate.data(), e.xq_f.data(), FF);
        mv(e, *L.w_down, e.gate.data(), e.xq_f.data(), e.o.data());
        for (int i = 0; i < E; i++) e.x[(size_t)i] += e.o[(size_t)i];
    }
    if (want_logits) {
        rmsnorm(e.xb.data(), e.x.data(), e.out_norm, E, h.rms_eps);
        quant(e, e.xb.data(), e.xq_e.data(), E);
        mv(e, *e.out_w, e.xb.data(), e.xq_e.data(), e.logits.data());
    }
    return true;
}

// kore's forward() with the whole attention block (kore.cpp:1419-1457: the
// quantisation of xb, the q/k/v projections and biases, the attention, the
// quantisation of att and Wo) in one library call, xb in and e.o out.
bool cuda_forward_block(Harness &hx, int token, int pos, bool want_logits) {
    Engine &e = hx.e;
    const Hparams &h = e.hp;
    const int E = (int)h.n_embd, FF = (int)h.n_ff;
    if (token < 0 || token >= e.n_vocab || pos < 0 || pos >= e.ctx) return false;
    if (!get_row(*e.tok_embd, (uint64_t)token, e.emb)) return false;
    std::copy(e.emb.begin(), e.emb.begin() + E, e.x.begin());
    for (uint32_t l = 0; l < h.n_layer; l++) {
        const Layer &L = e.layers[l];
        rmsnorm(e.xb.data(), e.x.data(), L.attn_norm, E, h.rms_eps);
        if (hx.block(hx.ctx, 0, (int)l, pos, e.xb.data(), e.o.data()) != KORE_CUDA_OK) {
            hx.err = hx.last_error(hx.ctx);
            return false;
        }
        for (int i = 0; i < E; i++) e.x[(size_t)i] += e.o[(size_t)i];
        rmsnorm(e.xb.data(), e.x.data(), L.ffn_norm, E, h.rms_eps);
        quant(e, e.xb.data(), e.xq_e.data(), E);
        mv(e, *L.w_gate, e.xb.data(), e.xq_e.data(), e.gate.data());
        mv(e, *L.w_up, e.xb.data(), e.xq_e.data(), e.up.data());
        for (int i = 0; i < FF; i++) {
            const float g = e.gate[(size_t)i];
            e.gate[(size_t)i] = g / (1.0f + std::exp(-g)) * e.up[(size_t)i];
        }
        quant(e, e.gate.data(), e.xq_f.data(), FF);
        mv(e, *L.w_down, e.gate.data(), e.xq_f.data(), e.o.data());
        for (int i = 0; i < E; i++) e.x[(size_t)i] += e.o[(size_t)i];
    }
    if (want_logits) {
        rmsnorm(e.xb.data(), e.x.data(), e.out_norm, E, h.rms_eps);
        quant(e, e.xb.data(), e.xq_e.data(), E);
        mv(e, *e.out_w, e.xb.data(), e.xq_e.data(), e.logits.data());
    }
    return true;
}

kore_cuda_qmat as_qmat(const Tensor &t) {
    kore_cuda_qmat m;
    m.type = (int)t.type;
    m.cols = (int)t.dims[0];
    m.rows = (int)(t.dims[1] * t.dims[2] * t.dims[3]);
    m.data = t.data;
    return m;
}

// Uploads every layer's attention projections and biases (kore's own tensors).
bool upload_attn_weights(Harness &hx) {
    if (hx.weights_up) return true;
    for (uint32_t l = 0; l < hx.e.hp.n_layer; l++) {
        const Layer &L = hx.e.layers[l];
        const kore_cuda_qmat q = as_qmat(*L.wq), k = as_qmat(*L.wk), v = as_qmat(*L.wv), o = as_qmat(*L.wo);
        if (hx.set_weights(hx.ctx, (int)l, &q, &k, &v, &o, L.bq, L.bk, L.bv) != KORE_CUDA_OK) {
            hx.err = hx.last_error(hx.ctx);
            return false;
        }
    }
    hx.weights_up = true;
    return true;
}

// Uploads the whole model (kore's own tensors) for the device-resident step.
bool upload_model(Harness &hx) {
    if (hx.model_up) return true;
    const Engine &e = hx.e;
    std::vector<kore_cuda_layer_weights> lw(e.hp.n_layer);
    for (uint32_t l = 0; l < e.hp.n_layer; l++) {
        const Layer &L = e.layers[l];
        kore_cuda_layer_weights &w = lw[l];
        w.wq = as_qmat(*L.wq);
        w.wk = as_qmat(*L.wk);
        w.wv = as_qmat(*L.wv);
        w.wo = as_qmat(*L.wo);
        w.bq = L.bq;
        w.bk = L.bk;
        w.bv = L.bv;
        w.attn_norm = L.attn_norm;
        w.ffn_norm = L.ffn_norm;
        w.w_gate = as_qmat(*L.w_gate);
        w.w_up = as_qmat(*L.w_up);
        w.w_down = as_qmat(*L.w_down);
    }
    kore_cuda_model m;
    m.n_ff = (int)e.hp.n_ff;
    m.n_vocab = e.n_vocab;
    m.rms_eps = e.hp.rms_eps;
    m.tok_embd = as_qmat(*e.tok_embd);
    m.out_norm = e.out_norm;
    m.out_w = as_qmat(*e.out_w);
    m.layers = lw.data();
    if (hx.set_model(hx.ctx, &m) != KORE_CUDA_OK) {
        hx.err = hx.last_error(hx.ctx);
        return false;
    }
    hx.model_up = true;
    return true;
}

bool cuda_forward_batch(Harness &hx, const int *toks, int nb, int pos0, bool want_logits) {
    Engine &e = hx.e;
    const Hparams &h = e.hp;
    const int E = (int)h.n_embd, FF = (int)h.n_ff, kvd = e.kv_dim;
    if (nb <= 0 || nb > e.bsz || pos0 < 0 || pos0 + nb > e.ctx) return false;
    for (int z = 0; z < nb; z++) {
        if (toks[z] < 0 || toks[z] >= e.n_vocab) return false;
        if (!get_row(*e.tok_embd, (uint64_t)toks[z], e.scratch)) return false;
        std::copy(e.scratch.begin(), e.scratch.begin() + E, e.bx.begin() + (size_t)z * E);
    }
    float *const xt = e.bxt.data();
    for (uint32_t l = 0; l < h.n_layer; l++) {
        const Layer &L = e.layers[l];
        for (int z = 0; z < nb; z++)
            rmsnorm(e.bxb.data() + (size_t)z * E, e.bx.data() + (size_t)z * E, L.attn_norm, E, h.rms_eps);
        matmul_batch_float(*L.wq, e.bxb.data(), nb, xt, e.bq.data(), e.avx2, e.nth);
        matmul_batch_float(*L.wk, e.bxb.data(), nb, xt, e.bk.data(), e.avx2, e.nth);
        matmul_batch_float(*L.wv, e.bxb.data(), nb, xt, e.bv.data(), e.avx2, e.nth);
        for (int z = 0; z < nb; z++) {
            float *q = e.bq.data() + (size_t)z * E;
            float *k = e.bk.data() + (size_t)z * kvd;
            float *v = e.bv.data() + (size_t)z * kvd;
            for (int i = 0; i < E; i++) q[i] += L.bq[i];
            for (int i = 0; i < kvd; i++) {
                k[i] += L.bk[i];
                v[i] += L.bv[i];
            }
        }
        if (hx.prefill(hx.ctx, 0, (int)l, pos0, nb, e.bq.data(), e.bk.data(), e.bv.data(), e.batt.data()) !=
            KORE_CUDA_OK) {
            hx.err = hx.last_error(hx.ctx);
            return false;
        }
        matmul_batch_float(*L.wo, e.batt.data(), nb, xt, e.bo.data(), e.avx2, e.nth);
        for (int z = 0; z < nb; z++)
            for (int i = 0; i < E; i++) e.bx[(size_t)z * E + i] += e.bo[(size_t)z * E + i];
        for (int z = 0; z < nb; z++)
            rmsnorm(e.bxb.data() + (size_t)z * E, e.bx.data() + (size_t)z * E, L.ffn_norm, E, h.rms_eps);
        matmul_batch_float(*L.w_gate, e.bxb.data(), nb, xt, e.bgate.data(), e.avx2, e.nth);
        matmul_batch_float(*L.w_up, e.bxb.data(), nb, xt, e.bup.data(), e.avx2, e.nth);
        for (int z = 0; z < nb; z++)
            for (int i = 0; i < FF; i++) {
                const float g = e.bgate[(size_t)z * FF + i];
                e.bgate[(size_t)z * FF + i] = g / (1.0f + std::exp(-g)) * e.bup[(size_t)z * FF + i];
            }
        matmul_batch_float(*L.w_down, e.bgate.data(), nb, xt, e.bo.data(), e.avx2, e.nth);
        for (int z = 0; z < nb; z++)
            for (int i = 0; i < E; i++) e.bx[(size_t)z * E + i] += e.bo[(size_t)z * E + i];
    }
    if (want_logits) {
        rmsnorm(e.xb.data(), e.bx.data() + (size_t)(nb - 1) * E, e.out_norm, E, h.rms_eps);
        quant(e, e.xb.data(), e.xq_e.data(), E);
        mv(e, *e.out_w, e.xb.data(), e.xq_e.data(), e.logits.data());
    }
    return true;
}

// Greedy generation with either engine: prompt in chunks of e.bsz, then one
// token at a time. Returns the number of generated IDs or -1.
template <class Batch, class Step>
int generate(Harness &hx, const int *prompt, int n_prompt, int n_gen, int *ids, float *margins, Batch batch,
             Step step) {
    Engine &e = hx.e;
    if (n_prompt <= 0 || n_prompt + n_gen > e.ctx) {
        hx.err = "prompt + generation exceed the context";
        return -1;
    }
    for (int p0 = 0; p0 < n_prompt; p0 += e.bsz) {
        const int nb = std::min(e.bsz, n_prompt - p0);
        if (!batch(prompt + p0, nb, p0, p0 + nb == n_prompt)) {
            if (hx.err.empty()) hx.err = "prefill failed";
            return -1;
        }
    }
    int pos = n_prompt;
    for (int i = 0; i < n_gen; i++) {
        ids[i] = argmax_margin(e.logits, margins ? margins + i : nullptr);
        if (i + 1 == n_gen) break;
        if (!step(ids[i], pos++)) {
            if (hx.err.empty()) hx.err = "decode failed";
            return -1;
        }
    }
    return n_gen;
}

}  // namespace

extern "C" {

// A random-init model: n_layer layers of the given geometry (n_embd and n_ff
// multiples of 256, n_ff >= n_embd so that kore's batched projections fit its
// transposed-activation buffer, kore.cpp:1364), vocabulary n_vocab, context
// ctx. Returns nullptr when kore's engine_init refuses it.
void *keng_create(int n_layer, int n_embd, int n_head, int n_head_kv, int n_ff, int n_vocab, int ctx,
                  unsigned long long seed, int n_threads) {
    auto hx = std::make_unique<Harness>();
    std::mt19937_64 rng(seed);
    Hparams &hp = hx->m.hp;
    hp.n_layer = (uint32_t)n_layer; hp.n_embd = (uint32_t)n_embd; hp.n_ff = (uint32_t)n_ff;
    hp.n_head = (uint32_t)n_head; hp.n_head_kv = (uint32_t)n_head_kv; hp.n_ctx = (uint32_t)ctx;
    hp.n_vocab = (uint32_t)n_vocab; hp.rope_base = 1000000.0f; hp.rms_eps = 1e-6f;
    const int hd = n_head > 0 ? n_embd / n_head : 0, kvd = n_head_kv * hd;
    const float se = 1.0f / std::sqrt((float)n_embd), sf = 1.0f / std::sqrt((float)n_ff);
    auto &T = hx->m.tensors;
    T["token_embd.weight"] = f32_random(*hx, n_embd, n_vocab, 0.0f, 1.0f, rng);
    T["output.weight"] = q4k_random(*hx, n_embd, n_vocab, se, rng);
    T["output_norm.weight"] = f32_random(*hx, n_embd, 1, 1.0f, 0.1f, rng);
    for (int l = 0; l < n_layer; l++) {
        const std::string p = "blk." + std::to_string(l) + ".";
        T[p + "attn_q.weight"] = q4k_random(*hx, n_embd, n_embd, se, rng);
        T[p + "attn_k.weight"] = q4k_random(*hx, n_embd, kvd, se, rng);
        T[p + "attn_v.weight"] = q4k_random(*hx, n_embd, kvd, se, rng);
        T[p + "attn_output.weight"] = q4k_random(*hx, n_embd, n_embd, se, rng);
        T[p + "attn_q.bias"] = f32_random(*hx, n_embd, 1, 0.0f, 0.5f, rng);
        T[p + "attn_k.bias"] = f32_random(*hx, kvd, 1, 0.0f, 0.5f, rng);
        T[p + "attn_v.bias"] = f32_random(*hx, kvd, 1, 0.0f, 0.5f, rng);
        T[p + "attn_norm.weight"] = f32_random(*hx, n_embd, 1, 1.0f, 0.1f, rng);
        T[p + "ffn_norm.weight"] = f32_random(*hx, n_embd, 1, 1.0f, 0.1f, rng);
        T[p + "ffn_gate.weight"] = q4k_random(*hx, n_embd, n_ff, se, rng);
        T[p + "ffn_up.weight"] = q4k_random(*hx, n_embd, n_ff, se, rng);
        T[p + "ffn_down.weight"] = q4k_random(*hx, n_ff, n_embd, sf, rng);
    }
    if (!engine_init(hx->e, hx->m, ctx, (unsigned)(n_threads > 0 ? n_threads : 1), false)) return nullptr;
    return hx.release();
}

void keng_destroy(void *h) {
    Harness *hx = (Harness *)h;
    if (!hx) return;
    if (hx->ctx && hx->destroy) hx->destroy(hx->ctx);
    delete hx;   // the library stays loaded: other users in the process may hold it
}

const char *keng_error(void *h) { return ((Harness *)h)->err.c_str(); }
int keng_ctx(void *h) { return ((Harness *)h)->e.ctx; }
int keng_chunk(void *h) { return ((Harness *)h)->e.bsz; }

// Greedy IDs from the reference engine; margins[i] = top-1 minus top-2 logit.
int keng_generate_ref(void *h, const int *prompt, int n_prompt, int n_gen, int *ids, float *margins) {
    Harness &hx = *(Harness *)h;
    hx.err.clear();
    return generate(
        hx, prompt, n_prompt, n_gen, ids, margins,
        [&](const int *t, int nb, int p0, bool last) { return forward_batch(hx.e, t, nb, p0, last); },
        [&](int tok, int pos) { return forward(hx.e, tok, pos, true); });
}

// Loads the CUDA library at `lib_path` and creates a context on `device` for
// this model's geometry, with kore's own inv_freq table.
int keng_attach_cuda(void *h, const char *lib_path, int device) {
    Harness &hx = *(Harness *)h;
    hx.err.clear();
    hx.lib = dlopen(lib_path, RTLD_NOW | RTLD_LOCAL);
    if (!hx.lib) {
        hx.err = std::string("dlopen: ") + dlerror();
        return -1;
    }
    auto cfg_default = (fn_cfg_default)dlsym(hx.lib, "kore_cuda_cfg_default");
    auto create = (fn_create)dlsym(hx.lib, "kore_cuda_create");
    hx.destroy = (fn_destroy)dlsym(hx.lib, "kore_cuda_destroy");
    hx.last_error = (fn_last_error)dlsym(hx.lib, "kore_cuda_last_error");
    hx.seq_reset = (fn_seq_reset)dlsym(hx.lib, "kore_cuda_seq_reset");
    hx.decode = (fn_decode)dlsym(hx.lib, "kore_cuda_attn_decode");
    hx.prefill = (fn_prefill)dlsym(hx.lib, "kore_cuda_attn_prefill");
    hx.set_weights = (fn_set_weights)dlsym(hx.lib, "kore_cuda_set_attn_weights");
    hx.block = (fn_block)dlsym(hx.lib, "kore_cuda_attn_block_decode");
    hx.set_model = (fn_set_model)dlsym(hx.lib, "kore_cuda_set_model");
    hx.step = (fn_step)dlsym(hx.lib, "kore_cuda_decode_step");
    if (!cfg_default || !create || !hx.destroy || !hx.last_error || !hx.seq_reset || !hx.decode || !hx.prefill) {
        hx.err = "missing symbol in the CUDA library";
        return -1;
    }
    const Engine &e = hx.e;
    kore_cuda_cfg cfg;
    cfg_default(&cfg, (int)e.hp.n_layer, (int)e.hp.n_head, (int)e.hp.n_head_kv, e.head_dim, e.ctx);
    cfg.rope_base = e.hp.rope_base;
    cfg.inv_freq = e.inv_freq.data();
    cfg.device = device;
    if (create(&hx.ctx, &cfg) != KORE_CUDA_OK) {
        hx.err = std::string("kore_cuda_create: ") + hx.last_error(nullptr);
        hx.ctx = nullptr;
        return -1;
    }
    return 0;
}

// Greedy IDs from the same engine with the attention on the GPU.
int keng_generate_cuda(void *h, const int *prompt, int n_prompt, int n_gen, int *ids) {
    Harness &hx = *(Harness *)h;
    hx.err.clear();
    if (!hx.ctx) {
        hx.err = "no CUDA context (keng_attach_cuda)";
        return -1;
    }
    if (hx.seq_reset(hx.ctx, 0) != KORE_CUDA_OK) {
        hx.err = hx.last_error(hx.ctx);
        return -1;
    }
    return generate(
        hx, prompt, n_prompt, n_gen, ids, nullptr,
        [&](const int *t, int nb, int p0, bool last) { return cuda_forward_batch(hx, t, nb, p0, last); },
        [&](int tok, int pos) { return cuda_forward(hx, tok, pos, true); });
}

// kore's own forward() of one token at `pos` (kore.cpp:1397-1480) on the
// harness's engine, logits copied out (n_vocab floats). Positions must come
// in order from 0 (forward() appends to the engine's cache).
int keng_forward(void *h, int token, int pos, float *logits) {
    Harness &hx = *(Harness *)h;
    if (!forward(hx.e, token, pos, true)) return -1;
    memcpy(logits, hx.e.logits.data(), hx.e.logits.size() * sizeof(float));
    return 0;
}

// A tensor of the harness's model by GGUF name: its data, type and shape
// (cols = dims[0], rows = the rest), or nullptr.
const void *keng_tensor(void *h, const char *name, int *type, int *rows, int *cols) {
    Harness &hx = *(Harness *)h;
    const auto it = hx.m.tensors.find(name);
    if (it == hx.m.tensors.end()) return nullptr;
    const Tensor &t = it->second;
    *type = (int)t.type;
    *cols = (int)t.dims[0];
    *rows = (int)(t.dims[1] * t.dims[2] * t.dims[3]);
    return t.data;
}

const float *keng_inv_freq(void *h) { return ((Harness *)h)->e.inv_freq.data(); }
int keng_avx2(void *h) { return ((Harness *)h)->e.avx2 ? 1 : 0; }
float keng_rms_eps(void *h) { return ((Harness *)h)->e.hp.rms_eps; }

// Greedy IDs with the attention block of every decode step on the GPU,
// projections included (the prompt's chunks as in keng_generate_cuda).
int keng_generate_cuda_block(void *h, const int *prompt, int n_prompt, int n_gen, int *ids) {
    Harness &hx = *(Harness *)h;
    hx.err.clear();
    if (!hx.ctx || !hx.set_weights || !hx.block) {
        hx.err = "no CUDA context with the attention-block entry points (keng_attach_cuda)";
        return -1;
    }
    if (!upload_attn_weights(hx)) return -1;
    if (hx.seq_reset(hx.ctx, 0) != KORE_CUDA_OK) {
        hx.err = hx.last_error(hx.ctx);
        return -1;
    }
    return generate(
        hx, prompt, n_prompt, n_gen, ids, nullptr,
        [&](const int *t, int nb, int p0, bool last) { return cuda_forward_batch(hx, t, nb, p0, last); },
        [&](int tok, int pos) { return cuda_forward_block(hx, tok, pos, true); });
}

// Greedy IDs with kore's prompt flow (its chunks through the CUDA path, as in
// keng_generate_cuda) and then every decode step wholly on the GPU
// (kore_cuda_decode_step: embedding, every layer, logits and argmax on the
// device; the host passes the token id and gets the next one back).
int keng_generate_cuda_step(void *h, const int *prompt, int n_prompt, int n_gen, int *ids) {
    Harness &hx = *(Harness *)h;
    hx.err.clear();
    if (!hx.ctx || !hx.set_model || !hx.step) {
        hx.err = "no CUDA context with the decode-step entry points (keng_attach_cuda)";
        return -1;
    }
    if (!upload_model(hx)) return -1;
    Engine &e = hx.e;
    if (n_prompt <= 0 || n_prompt + n_gen > e.ctx) {
        hx.err = "prompt + generation exceed the context";
        return -1;
    }
    if (hx.seq_reset(hx.ctx, 0) != KORE_CUDA_OK) {
        hx.err = hx.last_error(hx.ctx);
        return -1;
    }
    for (int p0 = 0; p0 < n_prompt; p0 += e.bsz) {
        const int nb = std::min(e.bsz, n_prompt - p0);
        if (!cuda_forward_batch(hx, prompt + p0, nb, p0, p0 + nb == n_prompt)) {
            if (hx.err.empty()) hx.err = "prefill failed";
            return -1;
        }
    }
    ids[0] = argmax_margin(e.logits, nullptr);
    for (int i = 1; i < n_gen; i++) {
        if (hx.step(hx.ctx, 0, ids[i - 1], n_prompt + i - 1, &ids[i], nullptr) != KORE_CUDA_OK) {
            hx.err = hx.last_error(hx.ctx);
            return -1;
        }
    }
    return n_gen;
}

// kore's get_row (kore.cpp:384-407) of a rows x cols table of GGUF type
// `type` at `data`: the dequantised row into out [cols]. Returns 0 or -1.
int keng_get_row(int type, int rows, int cols, const void *data, int row, float *out) {
    const char *tn;
    uint64_t blk, bpb;
    if (!type_info((uint32_t)type, &tn, &blk, &bpb)) return -1;
    Tensor t;
    t.type = (uint32_t)type;
    t.n_dims = 2;
    t.dims[0] = (uint64_t)cols;
    t.dims[1] = (uint64_t)rows;
    t.nbytes = (uint64_t)rows * ((uint64_t)cols / blk * bpb);
    t.data = (const uint8_t *)data;
    std::vector<float> v;
    if (!get_row(t, (uint64_t)row, v)) return -1;
    memcpy(out, v.data(), (size_t)cols * sizeof(float));
    return 0;
}

// kore's own forward_batch() (kore.cpp:1486-1598) of nb <= e.bsz tokens at
// pos0 (positions before pos0 already in the engine's cache): the last
// token's logits into logits [n_vocab]. Returns 0 or -1.
int keng_forward_batch(void *h, const int *toks, int nb, int pos0, float *logits) {
    Harness &hx = *(Harness *)h;
    if (!forward_batch(hx.e, toks, nb, pos0, true)) return -1;
    memcpy(logits, hx.e.logits.data(), hx.e.logits.size() * sizeof(float));
    return 0;
}

// kore's own matmul_batch_float (kore.cpp:783-845) with the engine's AVX2
// choice: out [B][rows] = rows x [B][cols] of a GGUF matrix at `data`.
int keng_matmul_batch(void *h, int type, int rows, int cols, const void *data, const float *x, int B, float *out) {
    Harness &hx = *(Harness *)h;
    Tensor t;
    t.type = (uint32_t)type;
    t.n_dims = 2;
    t.dims[0] = (uint64_t)cols;
    t.dims[1] = (uint64_t)rows;
    t.data = (const uint8_t *)data;
    std::vector<float> xt((size_t)((B + 7) & ~7) * cols);
    matmul_batch_float(t, x, B, xt.data(), out, hx.e.avx2, hx.e.nth);
    return 0;
}

// One turn of kore's chat flow on the harness's engine: prefill() of ids at
// base (kore.cpp:1720-1737: forward_batch over chunks of e.bsz, the last with
// logits) and then n_gen of its gen_step()s at temperature 0 (kore.cpp:
// 1742-1756: sample_token, append, forward() for the next logits). The
// generated ids go to out. Returns n_gen, or -1 when kore refuses.
int keng_turn_ref(void *h, const int *ids, int n, int base, int n_gen, int *out) {
    Harness &hx = *(Harness *)h;
    Engine &e = hx.e;
    if (n <= 0 || base + n >= e.ctx) return -1;
    for (int i = 0; i < n; i += e.bsz) {
        const int nb = std::min(e.bsz, n - i);
        if (!forward_batch(e, ids + i, nb, base + i, i + nb == n)) return -1;
    }
    int pos = base + n;
    for (int g = 0; g < n_gen; g++) {
        std::mt19937 rng(0);
        const int tok = sample_token(e.logits, 0.0f, 40, rng);
        out[g] = tok;
        if (pos >= e.ctx || !forward(e, tok, pos++, true)) return -1;
    }
    return n_gen;
}

// kore's forward() (kore.cpp:1397-1480) with its attention region served by
// the attached CUDA context (cuda_forward): every other operation is kore's
// own. Its logits isolate the attention: a device step that agrees with
// them bit for bit agrees with kore in everything but the attention. Returns
// 0 or -1.
int keng_forward_cuda(void *h, int token, int pos, float *logits) {
    Harness &hx = *(Harness *)h;
    if (!hx.ctx || !cuda_forward(hx, token, pos, true)) return -1;
    memcpy(logits, hx.e.logits.data(), hx.e.logits.size() * sizeof(float));
    return 0;
}

// The same for forward_batch() (kore.cpp:1486-1598): nb <= e.bsz tokens at
// pos0, attention through the attached CUDA context; the last token's logits.
int keng_forward_batch_cuda(void *h, const int *toks, int nb, int pos0, float *logits) {
    Harness &hx = *(Harness *)h;
    if (!hx.ctx || !cuda_forward_batch(hx, toks, nb, pos0, true)) return -1;
    memcpy(logits, hx.e.logits.data(), hx.e.logits.size() * sizeof(float));
    return 0;
}

}  // extern "C"
