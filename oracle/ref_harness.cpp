// ref_harness.cpp — runs the REFERENCE engine's own attention code on chosen inputs.
//
// TEST INFRASTRUCTURE ONLY. oracle/Makefile compiles this file with kore's own
// flags (build.sh:10, -std=c++20 -O3 -pthread) into oracle/_ref/libkore_ref.so;
// the reference source is included from where it lies (KORE_REF_SRC), never
// copied. Nothing in the product links this library.
//
// kore has no attention function: the attention is inlined in forward()
// (kore.cpp:1397-1480, decode) and forward_batch() (kore.cpp:1486-1598,
// prefill). To run exactly that code on arbitrary q/k/v, the harness builds an
// in-memory one-layer Model whose Q4_K projection weights are all zero, so
// that q = Wq*x + bq = bq, k = bk, v = bv (kore.cpp:1419-1423, :1524-1536),
// and sets the layer biases to the caller's bias-added, pre-RoPE q/k/v before
// each call. forward() then rotates, appends and attends with kore's code,
// and e.att / e.batt hold the attention output.
//
// forward_batch() shares one bias across the tokens of a batch, so a prefill
// chunk is run as successive nb = 1 batches; each (head, token) computation of
// kore.cpp:1542-1563 is independent of the batch size (the loop only shares
// the appended cache), so this reproduces the reference's prefill arithmetic
// (hd_dot / hd_fma) token for token.
//
// Shapes whose n_head*head_dim is not a multiple of 256 (Qwen2.5-0.5B: 14*64 =
// 896) are rejected by engine_init (kore.cpp:1283-1286). For those the engine
// is initialised with the next multiple of 256 and then narrowed (n_embd,
// n_head, n_rep); the attention loops read only those fields, and the zero
// weights keep the wider projections inert.

#define main kore_ref_main
#include KORE_REF_SRC
#undef main

#include <memory>

namespace {

struct RefEngine {
    Model m;
    Engine e;
    std::vector<std::vector<uint8_t>> store;
    int H = 0, G = 0, d = 0, E_init = 0;
    float *bq = nullptr, *bk = nullptr, *bv = nullptr;
};

Tensor make_tensor(RefEngine &r, uint32_t type, uint64_t cols, uint64_t rows, uint64_t bytes) {
    r.store.emplace_back(bytes, 0);
    Tensor t;
    t.type = type;
    t.n_dims = rows > 1 ? 2 : 1;
    t.dims[0] = cols;
    t.dims[1] = rows;
    t.nbytes = bytes;
    t.data = r.store.back().data();
    return t;
}

uint64_t q4k_bytes(uint64_t cols, uint64_t rows) { return cols / 256 * 144 * rows; }

}  // namespace

extern "C" {

// Creates a one-layer kore Engine with the given attention geometry and
// context. Returns nullptr if kore's engine_init refuses it.
void *kref_create(int n_head, int n_head_kv, int head_dim, int ctx, float rope_base, int n_threads) {
    if (n_head <= 0 || n_head_kv <= 0 || head_dim <= 0 || n_head % n_head_kv || ctx <= 0) return nullptr;
    auto r = std::make_unique<RefEngine>();
    r->H = n_head; r->G = n_head_kv; r->d = head_dim;
    int E = n_head * head_dim;
    int Hi = n_head;
    if (E % 256 != 0) {                       // widen to a shape engine_init accepts
        int Ei = (E + 255) / 256 * 256;
        while (Ei % head_dim != 0 || (Ei / head_dim) % n_head_kv != 0) Ei += 256;
        Hi = Ei / head_dim;
        E = Ei;
    }
    r->E_init = E;
    // kore sizes its transposed-activation buffer as [bsz rounded to 8][n_ff]
    // (kore.cpp:1364) and fills [n][B8] of it for every batched projection,
    // so n_ff must be at least n_embd/8 (n_embd itself for tiny contexts).
    const int FF = ctx >= 64 ? std::max(256, (E / 4 + 255) / 256 * 256) : E;
    const int kvd = n_head_kv * head_dim, V = 16;
    Hparams &hp = r->m.hp;
    hp.n_layer = 1; hp.n_embd = (uint32_t)E; hp.n_ff = FF; hp.n_head = (uint32_t)Hi;
    hp.n_head_kv = (uint32_t)n_head_kv; hp.n_ctx = (uint32_t)ctx; hp.n_vocab = V;
    hp.rope_base = rope_base; hp.rms_eps = 1e-6f;

    auto &T = r->m.tensors;
    T["token_embd.weight"] = make_tensor(*r, GGML_F32, E, V, (uint64_t)E * V * 4);
    T["output.weight"] = make_tensor(*r, GGML_Q4_K, E, V, q4k_bytes(E, V));
    T["output_norm.weight"] = make_tensor(*r, GGML_F32, E, 1, (uint64_t)E * 4);
    const std::string p = "blk.0.";
    T[p + "attn_q.weight"] = make_tensor(*r, GGML_Q4_K, E, E, q4k_bytes(E, E));
    T[p + "attn_k.weight"] = make_tensor(*r, GGML_Q4_K, E, kvd, q4k_bytes(E, kvd));
    T[p + "attn_v.weight"] = make_tensor(*r, GGML_Q4_K, E, kvd, q4k_bytes(E, kvd));
    T[p + "attn_output.weight"] = make_tensor(*r, GGML_Q4_K, E, E, q4k_bytes(E, E));
    T[p + "attn_q.bias"] = make_tensor(*r, GGML_F32, E, 1, (uint64_t)E * 4);
    T[p + "attn_k.bias"] = make_tensor(*r, GGML_F32, kvd, 1, (uint64_t)kvd * 4);
    T[p + "attn_v.bias"] = make_tensor(*r, GGML_F32, kvd, 1, (uint64_t)kvd * 4);
    T[p + "attn_norm.weight"] = make_tensor(*r, GGML_F32, E, 1, (uint64_t)E * 4);
    T[p + "ffn_norm.weight"] = make_tensor(*r, GGML_F32, E, 1, (uint64_t)E * 4);
    T[p + "ffn_gate.weight"] = make_tensor(*r, GGML_Q4_K, E, FF, q4k_bytes(E, FF));
    T[p + "ffn_up.weight"] = make_tensor(*r, GGML_Q4_K, E, FF, q4k_bytes(E, FF));
    T[p + "ffn_down.weight"] = make_tensor(*r, GGML_Q4_K, FF, E, q4k_bytes(FF, E));

    if (!engine_init(r->e, r->m, ctx, (unsigned)(n_threads > 0 ? n_threads : 1), false)) return nullptr;
    if (Hi != n_head) {                       // narrow to the requested head count
        r->e.hp.n_head = (uint32_t)n_head;
        r->e.hp.n_embd = (uint32_t)(n_head * head_dim);
        r->e.n_rep = n_head / n_head_kv;
    }
    r->bq = (float *)T[p + "attn_q.bias"].data;
    r->bk = (float *)T[p + "attn_k.bias"].data;
    r->bv = (float *)T[p + "attn_v.bias"].data;
    return r.release();
}

void kref_destroy(void *h) { delete (RefEngine *)h; }

int kref_avx2(void *h) { return ((RefEngine *)h)->e.avx2 ? 1 : 0; }
int kref_ctx(void *h) { return ((RefEngine *)h)->e.ctx; }
const float *kref_inv_freq(void *h) { return ((RefEngine *)h)->e.inv_freq.data(); }
float *kref_kcache(void *h) { return ((RefEngine *)h)->e.kcache.data(); }
float *kref_vcache(void *h) { return ((RefEngine *)h)->e.vcache.data(); }

// Writes post-RoPE key rows and value rows for positions [pos0, pos0+n) of the
// cache directly, rotating with kore's own rope_neox and the angle tables
// built as kore.cpp:1405-1410 builds them. Used to stand up long contexts
// without running n full forward() calls.
int kref_fill(void *h, int pos0, int n, const float *k_pre, const float *v) {
    RefEngine &r = *(RefEngine *)h;
    Engine &e = r.e;
    const int kvd = e.kv_dim, half = e.head_dim / 2;
    if (pos0 < 0 || n < 0 || pos0 + n > e.ctx) return -1;
    std::vector<float> c((size_t)half), s((size_t)half);
    for (int z = 0; z < n; z++) {
        const int pos = pos0 + z;
        for (int i = 0; i < half; i++) {
            const double a = (double)pos * e.inv_freq[(size_t)i];
            c[(size_t)i] = (float)std::cos(a);
            s[(size_t)i] = (float)std::sin(a);
        }
        float *kd = e.kcache.data() + (size_t)pos * kvd;
        memcpy(kd, k_pre + (size_t)z * kvd, (size_t)kvd * sizeof(float));
        rope_neox(kd, (int)e.hp.n_head_kv, e.head_dim, c.data(), s.data());
        memcpy(e.vcache.data() + (size_t)pos * kvd, v + (size_t)z * kvd, (size_t)kvd * sizeof(float));
    }
    return 0;
}

// One decode step through kore's forward(): RoPE of q/k at `pos`, append of
// k/v to row `pos`, attention over rows 0..pos (kore.cpp:1424-1455).
int kref_decode(void *h, int pos, const float *q, const float *k, const float *v, float *out) {
    RefEngine &r = *(RefEngine *)h;
    Engine &e = r.e;
    const int E = r.H * r.d, kvd = e.kv_dim;
    memcpy(r.bq, q, (size_t)E * sizeof(float));
    memcpy(r.bk, k, (size_t)kvd * sizeof(float));
    memcpy(r.bv, v, (size_t)kvd * sizeof(float));
    if (!forward(e, 0, pos, false)) return -1;
    memcpy(out, e.att.data(), (size_t)E * sizeof(float));
    return 0;
}

// A prefill chunk through kore's forward_batch(), one token per batch (see
// the header comment): tokens at positions pos0..pos0+n-1.
int kref_prefill(void *h, int pos0, int n, const float *q, const float *k, const float *v, float *out) {
    RefEngine &r = *(RefEngine *)h;
    Engine &e = r.e;
    const int E = r.H * r.d, kvd = e.kv_dim;
    for (int z = 0; z < n; z++) {
        memcpy(r.bq, q + (size_t)z * E, (size_t)E * sizeof(float));
        memcpy(r.bk, k + (size_t)z * kvd, (size_t)kvd * sizeof(float));
        memcpy(r.bv, v + (size_t)z * kvd, (size_t)kvd * sizeof(float));
        const int tok = 0;
        if (!forward_batch(e, &tok, 1, pos0 + z, false)) return -1;
        memcpy(out + (size_t)z * E, e.batt.data(), (size_t)E * sizeof(float));
    }
    return 0;
}

// kore's greedy choice (kore.cpp:1601-1603, temp <= 0).
int kref_argmax(const float *logits, int n) {
    std::vector<float> l(logits, logits + n);
    std::mt19937 rng(0);
    return sample_token(l, 0.0f, 1, rng);
}

double kref_now_ms(void) { return now_ms(); }

// kore's own Q8_K quantisation (kore.cpp:422-447), unpacked into the arrays
// d[n/256], qs[n], bsums[n/16].
void kref_q8k_quantize(const float *x, int n, float *d, int8_t *qs, int16_t *bsums) {
    std::vector<BlockQ8K> y((size_t)(n / 256));
    quantize_row_q8_K(x, y.data(), n);
    for (size_t i = 0; i < y.size(); i++) {
        d[i] = y[i].d;
        memcpy(qs + 256 * i, y[i].qs, 256);
        memcpy(bsums + 16 * i, y[i].bsums, sizeof(y[i].bsums));
    }
}

// kore's own dot product of one quantised row (type 12 = Q4_K, 14 = Q6_K)
// with Q8_K x given as arrays: the AVX2 kernel (kore.cpp:540-640) when avx2
// is set and the CPU has AVX2/FMA, else the scalar one (kore.cpp:451-507).
float kref_qdot(int type, int n, const uint8_t *w, const float *d, const int8_t *qs, const int16_t *bsums,
                int avx2) {
    std::vector<BlockQ8K> y((size_t)(n / 256));
    for (size_t i = 0; i < y.size(); i++) {
        y[i].d = d[i];
        memcpy(y[i].qs, qs + 256 * i, 256);
        memcpy(y[i].bsums, bsums + 16 * i, sizeof(y[i].bsums));
    }
    const bool v = avx2 && cpu_has_avx2();
    if (type == GGML_Q4_K) return v ? dot_q4_K_q8_K_avx2(n, w, y.data()) : dot_q4_K_q8_K_ref(n, w, y.data());
    return v ? dot_q6_K_q8_K_avx2(n, w, y.data()) : dot_q6_K_q8_K_ref(n, w, y.data());
}

// kore's own mv() + quant() for one quantised matrix (quantize_row_q8_K and
// matvec_mt with n_threads threads, kore.cpp:422-447, :679-682; its AVX2
// kernels when the CPU has them): out = W x, best wall time of `reps` runs in ms.
double kref_qmatvec_ms(int type, int rows, int cols, const uint8_t *data, const float *x, float *out,
                       int n_threads, int reps) {
    Tensor t;
    t.type = (uint32_t)type;
    t.n_dims = 2;
    t.dims[0] = (uint64_t)cols;
    t.dims[1] = (uint64_t)rows;
    t.nbytes = (uint64_t)rows * (uint64_t)(cols / 256) * (type == GGML_Q4_K ? 144 : 210);
    t.data = data;
    std::vector<BlockQ8K> xq((size_t)(cols / 256));
    const bool avx2 = cpu_has_avx2();
    double best = 1e30;
    for (int r = 0; r < reps; r++) {
        const double t0 = now_ms();
        quantize_row_q8_K(x, xq.data(), cols);
        matvec_mt(t, xq.data(), out, avx2, (unsigned)(n_threads > 0 ? n_threads : 1));
        best = std::min(best, now_ms() - t0);
    }
    return best;
}

}  // extern "C"
