/*
 * kore_step_oracle.c — CPU restatement of kore's whole decode step.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the thing measured or shipped).
 * Built by oracle/Makefile with -ffp-contract=off, like the other
 * restatements: kore's code outside its AVX2 kernels is compiled for baseline
 * x86-64, where nothing is fused.
 */
#include "kore_step_oracle.h"

#include <math.h>
#include <stddef.h>
#include <stdlib.h>
#include <string.h>

#include "kore_attn_oracle.h"
#include "kore_proj_oracle.h"

void korc_rmsnorm(float *out, const float *x, const float *w, int n, float eps) {
    /* kore.cpp:1367-1372 */
    double ss = 0;
    for (int i = 0; i < n; i++) ss += (double)x[i] * x[i];
    const float ms = (float)(ss / n);
    const float scale = 1.0f / sqrtf(ms + eps);
    for (int i = 0; i < n; i++) {
        const float a = x[i] * scale;
        out[i] = a * w[i];
    }
}

void korc_swiglu(float *gate, const float *up, int n) {
    /* kore.cpp:1465-1468 */
    for (int i = 0; i < n; i++) {
        const float g = gate[i];
        const float den = 1.0f + expf(-g);
        const float sg = g / den;
        gate[i] = sg * up[i];
    }
}

static int mv(const korc_qw *w, const float *x, const float *bias, float *out, int avx2) {
    return korc_qmatvec(w->type, w->rows, w->cols, w->data, x, bias, out, avx2);
}

int korc_decode_step(const korc_model *m, float *const *kc, float *const *vc, int token, int pos, float *logits,
                     int avx2) {
    if (!m || token < 0 || token >= m->n_vocab || pos < 0 || m->n_head <= 0 || m->n_embd % m->n_head) return -1;
    const int E = m->n_embd, FF = m->n_ff, H = m->n_head, G = m->n_head_kv, hd = E / H, kvd = G * hd;
    float *buf = (float *)malloc(sizeof(float) * ((size_t)5 * E + 2 * (size_t)kvd + 2 * (size_t)FF + pos + 1));
    if (!buf) return -1;
    float *x = buf, *xb = x + E, *q = xb + E, *att = q + E, *o = att + E, *k = o + E, *v = k + kvd;
    float *gate = v + kvd, *up = gate + FF, *scores = up + FF;
    int rc = 0;
    /* kore.cpp:1402-1403: the token's embedding row (F32) */
    memcpy(x, m->tok_embd + (size_t)token * E, (size_t)E * sizeof(float));
    for (int l = 0; l < m->n_layer && !rc; l++) {
        const korc_layer *L = &m->layers[l];
        /* attention block, kore.cpp:1418-1457 (the bias adds ride on the products) */
        korc_rmsnorm(xb, x, L->attn_norm, E, m->rms_eps);
        rc |= mv(&L->wq, xb, L->bq, q, avx2);
        rc |= mv(&L->wk, xb, L->bk, k, avx2);
        rc |= mv(&L->wv, xb, L->bv, v, avx2);
        rc |= korc_attn_decode(H, G, hd, m->inv_freq, pos, q, k, v, kc[l], vc[l], att, scores);
        rc |= mv(&L->wo, att, NULL, o, avx2);
        for (int i = 0; i < E; i++) x[i] += o[i];
        /* SwiGLU feed-forward, kore.cpp:1460-1472 */
        korc_rmsnorm(xb, x, L->ffn_norm, E, m->rms_eps);
        rc |= mv(&L->w_gate, xb, NULL, gate, avx2);
        rc |= mv(&L->w_up, xb, NULL, up, avx2);
        korc_swiglu(gate, up, FF);
        rc |= mv(&L->w_down, gate, NULL, o, avx2);
        for (int i = 0; i < E; i++) x[i] += o[i];
    }
    if (!rc) {
        /* kore.cpp:1475-1479 */
        korc_rmsnorm(xb, x, m->out_norm, E, m->rms_eps);
        rc |= mv(&m->out_w, xb, NULL, logits, avx2);
    }
    free(buf);
    return rc ? -1 : 0;
}
