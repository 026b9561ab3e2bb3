/*
 * kore_attn_oracle.c — CPU restatement of kore's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the thing measured or shipped).
 * Build: oracle/Makefile, with -ffp-contract=off so that every product and
 * sum is rounded on its own, as in the reference's baseline x86-64 build;
 * the only fused operations are the explicit fmaf() calls that restate the
 * reference's _mm256_fmadd_ps.
 */
#include "kore_attn_oracle.h"

#include <math.h>
#include <stddef.h>
#include <stdlib.h>
#include <string.h>

void korc_inv_freq(float rope_base, int head_dim, float *inv_freq) {
    /* kore.cpp:1339 */
    for (int i = 0; i < head_dim / 2; i++)
        inv_freq[i] = (float)pow((double)rope_base, -2.0 * i / head_dim);
}

void korc_rope_angles(const float *inv_freq, int half, int pos, float *c, float *s) {
    /* kore.cpp:1405-1409: angle in double, cos/sin in double, stored as float */
    for (int i = 0; i < half; i++) {
        const double a = (double)pos * (double)inv_freq[i];
        c[i] = (float)cos(a);
        s[i] = (float)sin(a);
    }
}

void korc_rope_neox(float *vec, int n_heads, int hd, const float *c, const float *s) {
    /* kore.cpp:1374-1384 */
    const int half = hd / 2;
    for (int h = 0; h < n_heads; h++) {
        float *p = vec + (size_t)h * hd;
        for (int i = 0; i < half; i++) {
            const float x0 = p[i], x1 = p[i + half];
            const float a = x0 * c[i], b = x1 * s[i];
            const float e = x0 * s[i], f = x1 * c[i];
            p[i] = a - b;
            p[i + half] = e + f;
        }
    }
}

int korc_cpu_has_avx2(void) {
#if defined(__x86_64__)
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
#else
    return 0;
#endif
}

float korc_hd_dot(const float *a, const float *b, int n, int avx2) {
    if (avx2) {
        /* kore.cpp:693-703: lane j of acc0 sums a[i+j]*b[i+j], lane j of acc1
         * sums a[i+8+j]*b[i+8+j], over i = 0, 16, 32, ... with fused FMAs. */
        float acc0[8] = {0}, acc1[8] = {0};
        int i = 0;
        for (; i + 16 <= n; i += 16) {
            for (int j = 0; j < 8; j++) {
                acc0[j] = fmaf(a[i + j], b[i + j], acc0[j]);
                acc1[j] = fmaf(a[i + 8 + j], b[i + 8 + j], acc1[j]);
            }
        }
        float v[8];
        for (int j = 0; j < 8; j++) v[j] = acc0[j] + acc1[j];
        /* kore.cpp:521-528 (hsum256): low half + high half, then
         * (l0 + l2) + (l1 + l3). */
        float l[4];
        for (int j = 0; j < 4; j++) l[j] = v[j] + v[j + 4];
        const float m0 = l[0] + l[2], m1 = l[1] + l[3];
        float s = m0 + m1;
        for (; i < n; i++) s += a[i] * b[i];
        return s;
    }
    /* kore.cpp:707-709 */
    float s = 0;
    for (int i = 0; i < n; i++) s += a[i] * b[i];
    return s;
}

void korc_hd_fma(float *o, const float *v, float p, int n, int avx2) {
    if (avx2) {
        /* kore.cpp:712-720: o = fma(p, v, o) per element */
        for (int i = 0; i < n; i++) o[i] = fmaf(p, v[i], o[i]);
        return;
    }
    /* kore.cpp:724 */
    for (int i = 0; i < n; i++) o[i] += p * v[i];
}

void korc_rope_key(int G, int d, const float *inv_freq, int pos, const float *k_pre, float *k_out) {
    float c[256], s[256];
    korc_rope_angles(inv_freq, d / 2, pos, c, s);
    memcpy(k_out, k_pre, (size_t)G * d * sizeof(float));
    korc_rope_neox(k_out, G, d, c, s);
}

static int shape_ok(int H, int G, int d) {
    return H > 0 && G > 0 && H % G == 0 && d > 0 && d % 2 == 0 && d <= 512;
}

int korc_attn_decode(int H, int G, int d, const float *inv_freq, int pos,
                     const float *q, const float *k, const float *v,
                     float *kc, float *vc, float *out, float *scores) {
    if (!shape_ok(H, G, d) || pos < 0) return -1;
    const int kvd = G * d, n_rep = H / G, half = d / 2;
    float c[256], s[256];
    korc_rope_angles(inv_freq, half, pos, c, s);
    /* kore.cpp:1411: the scale is applied after the dot product */
    const float inv_sqrt = 1.0f / sqrtf((float)d);

    float *qr = (float *)malloc(((size_t)H * d + kvd) * sizeof(float));
    if (!qr) return -1;
    float *kr = qr + (size_t)H * d;
    memcpy(qr, q, (size_t)H * d * sizeof(float));
    memcpy(kr, k, (size_t)kvd * sizeof(float));
    korc_rope_neox(qr, H, d, c, s);                              /* kore.cpp:1424 */
    korc_rope_neox(kr, G, d, c, s);                              /* kore.cpp:1425 */
    memcpy(kc + (size_t)pos * kvd, kr, (size_t)kvd * sizeof(float));  /* :1429 */
    memcpy(vc + (size_t)pos * kvd, v, (size_t)kvd * sizeof(float));   /* :1430 */

    for (int hh = 0; hh < H; hh++) {                             /* kore.cpp:1432-1455 */
        const float *qh = qr + (size_t)hh * d;
        const int kvh = hh / n_rep;
        float mx = -INFINITY;
        for (int t = 0; t <= pos; t++) {
            const float *kt = kc + (size_t)t * kvd + (size_t)kvh * d;
            float acc = 0;
            for (int i = 0; i < d; i++) acc += qh[i] * kt[i];
            acc *= inv_sqrt;
            scores[t] = acc;
            if (acc > mx) mx = acc;
        }
        float sum = 0;
        for (int t = 0; t <= pos; t++) { scores[t] = expf(scores[t] - mx); sum += scores[t]; }
        const float inv = 1.0f / sum;
        float *oh = out + (size_t)hh * d;
        for (int i = 0; i < d; i++) oh[i] = 0;
        for (int t = 0; t <= pos; t++) {
            const float p = scores[t] * inv;
            const float *vt = vc + (size_t)t * kvd + (size_t)kvh * d;
            for (int i = 0; i < d; i++) oh[i] += p * vt[i];
        }
    }
    free(qr);
    return 0;
}

int korc_attn_prefill(int H, int G, int d, const float *inv_freq, int pos0, int n,
                      const float *q, const float *k, const float *v,
                      float *kc, float *vc, float *out, float *scores, int avx2) {
    if (!shape_ok(H, G, d) || pos0 < 0 || n <= 0) return -1;
    const int kvd = G * d, n_rep = H / G, half = d / 2, E = H * d;
    const float inv_sqrt = 1.0f / sqrtf((float)d);              /* kore.cpp:1513 */
    float c[256], s[256];

    /* kore.cpp:1527-1539: RoPE per token and append. The rotated queries are
     * kept in `out` until the attention below overwrites row by row; a
     * token's output row is written only after all of its heads have read
     * their query, so a separate buffer is used instead. */
    float *qr = scores + (size_t)(pos0 + n);  /* caller provides (pos0+n) + n*E floats */
    for (int z = 0; z < n; z++) {
        korc_rope_angles(inv_freq, half, pos0 + z, c, s);
        float *qz = qr + (size_t)z * E;
        memcpy(qz, q + (size_t)z * E, (size_t)E * sizeof(float));
        korc_rope_neox(qz, H, d, c, s);
        float *kd = kc + (size_t)(pos0 + z) * kvd;
        memcpy(kd, k + (size_t)z * kvd, (size_t)kvd * sizeof(float));
        korc_rope_neox(kd, G, d, c, s);
        memcpy(vc + (size_t)(pos0 + z) * kvd, v + (size_t)z * kvd, (size_t)kvd * sizeof(float));
    }

    for (int hh = 0; hh < H; hh++) {                             /* kore.cpp:1542-1563 */
        const int kvh = hh / n_rep;
        for (int z = 0; z < n; z++) {
            const int lim = pos0 + z;
            const float *qh = qr + (size_t)z * E + (size_t)hh * d;
            float mx = -INFINITY;
            for (int t = 0; t <= lim; t++) {
                const float *kt = kc + (size_t)t * kvd + (size_t)kvh * d;
                const float sc = korc_hd_dot(qh, kt, d, avx2) * inv_sqrt;
                scores[t] = sc;
                if (sc > mx) mx = sc;
            }
            float sum = 0;
            for (int t = 0; t <= lim; t++) { scores[t] = expf(scores[t] - mx); sum += scores[t]; }
            const float inv = 1.0f / sum;
            float *oh = out + (size_t)z * E + (size_t)hh * d;
            memset(oh, 0, (size_t)d * sizeof(float));
            for (int t = 0; t <= lim; t++)
                korc_hd_fma(oh, vc + (size_t)t * kvd + (size_t)kvh * d, scores[t] * inv, d, avx2);
        }
    }
    return 0;
}

int korc_argmax(const float *logits, int n) {
    /* std::max_element: the first of equal maxima wins */
    int best = 0;
    for (int i = 1; i < n; i++)
        if (logits[i] > logits[best]) best = i;
    return best;
}
