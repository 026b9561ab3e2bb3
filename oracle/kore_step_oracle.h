/*
 * kore_step_oracle.h — CPU restatement of kore's whole decode step.
 *
 * TEST INFRASTRUCTURE ONLY: the checker a device-resident decode step is to
 * be compared against; nothing in the product links or calls it. Only tests/
 * use it.
 *
 * kore's forward() (kore.cpp:1397-1480) for one token through every layer:
 * RMSNorm (kore.cpp:1367-1372), the quantised projections (kore_proj_oracle),
 * the attention (kore_attn_oracle), the SwiGLU feed-forward
 * (kore.cpp:1462-1472), the residual adds and the logits. Pinned bit for bit
 * to the reference's own forward() by tests/test_step_oracle_pin.py.
 */
#ifndef KORE_STEP_ORACLE_H
#define KORE_STEP_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* A quantised matrix: GGUF type 12 (Q4_K) or 14 (Q6_K), rows x cols. */
typedef struct korc_qw {
    int type, rows, cols;
    const uint8_t *data;
} korc_qw;

typedef struct korc_layer {
    const float *attn_norm, *ffn_norm;   /* [n_embd] */
    const float *bq, *bk, *bv;           /* [n_embd], [kv_dim], [kv_dim] */
    korc_qw wq, wk, wv, wo, w_gate, w_up, w_down;
} korc_layer;

typedef struct korc_model {
    int n_layer, n_embd, n_ff, n_head, n_head_kv, n_vocab;
    float rms_eps;
    const float *tok_embd;   /* F32 [n_vocab][n_embd] */
    const float *out_norm;   /* [n_embd] */
    korc_qw out_w;           /* [n_vocab x n_embd] */
    const korc_layer *layers;
    const float *inv_freq;   /* [head_dim/2], kore.cpp:1339 */
} korc_model;

/* kore.cpp:1367-1372: out = x * (1 / sqrt(mean(x^2) + eps)) * w, the sum of
 * squares in double, sequentially. */
void korc_rmsnorm(float *out, const float *x, const float *w, int n, float eps);

/* kore.cpp:1465-1468: gate[i] = gate[i] / (1 + exp(-gate[i])) * up[i]. */
void korc_swiglu(float *gate, const float *up, int n);

/* kore.cpp:1397-1480: token at `pos` through every layer; kc[l], vc[l] are
 * layer l's cache rows [ctx][kv_dim] (rows 0..pos-1 filled, row pos written);
 * logits [n_vocab]. avx2 selects kore's AVX2 or scalar dot kernels. Returns 0,
 * or -1 on a bad argument or allocation failure. */
int korc_decode_step(const korc_model *m, float *const *kc, float *const *vc, int token, int pos, float *logits,
                     int avx2);

#ifdef __cplusplus
}
#endif

#endif
