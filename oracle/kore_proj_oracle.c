/*
 * kore_proj_oracle.c — CPU restatement of kore's quantised projections.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the thing measured or shipped).
 * Built by oracle/Makefile with -ffp-contract=off: every product and sum is
 * rounded on its own, and the only fused operations are the explicit fmaf()
 * calls restating the reference's _mm256_fmadd_ps / _mm_fmadd_ps.
 */
#include "kore_proj_oracle.h"

#include <math.h>
#include <stddef.h>
#include <stdlib.h>
#include <string.h>

float korc_f16_to_f32(uint16_t h) {
    /* kore.cpp:297-316, exact: sign, exponent rebias, subnormals normalised */
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu, bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            /* value man * 2^-24: shift the leading one to bit 10 */
            int shift = 0;
            while (!(man & 0x400u)) {
                man <<= 1;
                shift++;
            }
            bits = sign | ((uint32_t)(127 - 14 - shift) << 23) | ((man & 0x3FFu) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static float rd_f16(const uint8_t *p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return korc_f16_to_f32(h);
}

void korc_q8k_quantize(const float *x, int n, float *d, int8_t *qs, int16_t *bsums) {
    /* kore.cpp:422-447: the first value of largest magnitude maps to -127 */
    for (int i = 0; i < n / 256; i++, x += 256) {
        float amax = 0, maxv = 0;
        for (int j = 0; j < 256; j++) {
            const float ax = fabsf(x[j]);
            if (ax > amax) {
                amax = ax;
                maxv = x[j];
            }
        }
        int8_t *q = qs + (size_t)i * 256;
        int16_t *bs = bsums + (size_t)i * 16;
        if (amax == 0) {
            d[i] = 0;
            memset(q, 0, 256);
            memset(bs, 0, 16 * sizeof(int16_t));
            continue;
        }
        const float iscale = -127.0f / maxv;
        for (int j = 0; j < 256; j++) {
            const int v = (int)nearbyintf(iscale * x[j]);   /* round half to even */
            q[j] = (int8_t)(v > 127 ? 127 : v);
        }
        for (int j = 0; j < 16; j++) {
            int s = 0;
            for (int l = 0; l < 16; l++) s += q[16 * j + l];
            bs[j] = (int16_t)s;
        }
        d[i] = 1.0f / iscale;
    }
}

/* kore.cpp:326-335: the 6-bit scale and min of sub-block j (0..7) */
static void scale_min_k4(int j, const uint8_t *q, int *sc, int *mn) {
    if (j < 4) {
        *sc = q[j] & 63;
        *mn = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0x0F) | ((q[j - 4] >> 6) << 4);
        *mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

/* hsum256 of kore.cpp:521-528: ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)) */
static float hsum8(const float a[8]) {
    const float l0 = a[0] + a[4], l1 = a[1] + a[5], l2 = a[2] + a[6], l3 = a[3] + a[7];
    const float m0 = l0 + l2, m1 = l1 + l3;
    return m0 + m1;
}

/* hsum128 of kore.cpp:534-538: (v0+v2) + (v1+v3) */
static float hsum4(const float v[4]) {
    const float a = v[0] + v[2], b = v[1] + v[3];
    return a + b;
}

float korc_dot_q4k(int n, const uint8_t *w, const float *dx, const int8_t *qs, const int16_t *bsums, int avx2) {
    const int nb = n / 256;
    if (!avx2) {
        /* kore.cpp:451-477 */
        float sumf = 0;
        for (int i = 0; i < nb; i++) {
            const uint8_t *b = w + (size_t)i * 144;
            const float d = rd_f16(b) * dx[i];
            const float dmin = rd_f16(b + 2) * dx[i];
            const uint8_t *q = b + 16;
            const int8_t *q8b = qs + (size_t)i * 256;
            const int16_t *bs = bsums + (size_t)i * 16;
            int32_t isum = 0, imin = 0;
            for (int c = 0; c < 4; c++) {
                int sc0, m0, sc1, m1;
                scale_min_k4(2 * c, b + 4, &sc0, &m0);
                scale_min_k4(2 * c + 1, b + 4, &sc1, &m1);
                const int8_t *q8 = q8b + 64 * c;
                int32_t lo = 0, hi = 0;
                for (int l = 0; l < 32; l++) {
                    lo += (q[32 * c + l] & 0x0F) * q8[l];
                    hi += (q[32 * c + l] >> 4) * q8[32 + l];
                }
                isum += sc0 * lo + sc1 * hi;
                imin += m0 * (bs[4 * c] + bs[4 * c + 1]) + m1 * (bs[4 * c + 2] + bs[4 * c + 3]);
            }
            const float t1 = d * (float)isum, t2 = dmin * (float)imin;
            sumf += t1 - t2;
        }
        return sumf;
    }
    /* kore.cpp:540-590: eight int32 lanes, lane k holding the scale-weighted
     * products of bytes 4k..4k+3 of each 32-byte nibble row; four lanes of
     * minimum terms; one fused multiply-add per lane and block */
    float acc[8] = {0}, accm[4] = {0};
    for (int i = 0; i < nb; i++) {
        const uint8_t *b = w + (size_t)i * 144;
        const float d = rd_f16(b) * dx[i];
        const float dmin = rd_f16(b + 2) * dx[i];
        int sc[8], mn[8];
        for (int j = 0; j < 8; j++) scale_min_k4(j, b + 4, &sc[j], &mn[j]);
        const int16_t *bs = bsums + (size_t)i * 16;
        for (int m = 0; m < 4; m++) {
            const int s0 = (int16_t)(bs[4 * m] + bs[4 * m + 1]), s1 = (int16_t)(bs[4 * m + 2] + bs[4 * m + 3]);
            const int32_t prod = mn[2 * m] * s0 + mn[2 * m + 1] * s1;
            accm[m] = fmaf(-dmin, (float)prod, accm[m]);
        }
        const uint8_t *q4 = b + 16;
        const int8_t *q8 = qs + (size_t)i * 256;
        int32_t sumi[8] = {0};
        for (int c = 0; c < 4; c++)
            for (int k = 0; k < 8; k++) {
                int32_t lo = 0, hi = 0;
                for (int e = 4 * k; e < 4 * k + 4; e++) {
                    lo += (q4[32 * c + e] & 0x0F) * q8[64 * c + e];
                    hi += (q4[32 * c + e] >> 4) * q8[64 * c + 32 + e];
                }
                sumi[k] += sc[2 * c] * lo;
                sumi[k] += sc[2 * c + 1] * hi;
            }
        for (int k = 0; k < 8; k++) acc[k] = fmaf(d, (float)sumi[k], acc[k]);
    }
    const float a = hsum8(acc), m = hsum4(accm);
    return a + m;
}

/* the unsigned 6-bit value of element e (0..255) of a Q6_K block */
static int q6_value(const uint8_t *b, int e) {
    const int h = e / 128, r = e % 128, k = r / 32, l = r % 32;
    const uint8_t *ql = b + 64 * h, *qh = b + 128 + 32 * h;
    const int lo = (k & 1) ? ql[l + 32] : ql[l];
    const int nib = (k >= 2) ? (lo >> 4) : (lo & 0x0F);
    return nib | (((qh[l] >> (2 * k)) & 3) << 4);
}

float korc_dot_q6k(int n, const uint8_t *w, const float *dx, const int8_t *qs, const int16_t *bsums, int avx2) {
    const int nb = n / 256;
    if (!avx2) {
        /* kore.cpp:480-507 */
        float sumf = 0;
        for (int i = 0; i < nb; i++) {
            const uint8_t *b = w + (size_t)i * 210;
            const int8_t *sc = (const int8_t *)(b + 192);
            const float d = rd_f16(b + 208) * dx[i];
            const int8_t *q8 = qs + (size_t)i * 256;
            int32_t isum = 0;
            for (int j = 0; j < 16; j++) {
                int32_t s = 0;
                for (int l = 0; l < 16; l++) s += (q6_value(b, 16 * j + l) - 32) * q8[16 * j + l];
                isum += sc[j] * s;
            }
            sumf += d * (float)isum;
        }
        return sumf;
    }
    /* kore.cpp:594-640: unsigned 6-bit values in eight int32 lanes (lane n:
     * elements 4n..4n+3 of each 32-value group, weighted by the scale of its
     * 16-value half), the -32 offset as a separate float sum over blocks */
    float acc[8] = {0}, summ = 0;
    for (int i = 0; i < nb; i++) {
        const uint8_t *b = w + (size_t)i * 210;
        const int8_t *sc = (const int8_t *)(b + 192);
        const float d = rd_f16(b + 208) * dx[i];
        const int16_t *bs = bsums + (size_t)i * 16;
        int32_t ibias = 0;
        for (int j = 0; j < 16; j++) ibias += sc[j] * bs[j];
        /* summ -= d * 32.0f * (float)ibias: the reference build (g++ -O3,
         * inside a function compiled for FMA) fuses the product into the
         * subtraction, one rounding */
        const float d32 = d * 32.0f;
        summ = fmaf(-d32, (float)ibias, summ);
        const int8_t *q8 = qs + (size_t)i * 256;
        int32_t sumi[8] = {0};
        for (int h = 0; h < 2; h++)
            for (int k = 0; k < 4; k++)
                for (int nn = 0; nn < 8; nn++) {
                    const int s = sc[8 * h + 2 * k + (nn >= 4)];
                    int32_t p = 0;
                    for (int e = 4 * nn; e < 4 * nn + 4; e++)
                        p += q6_value(b, 128 * h + 32 * k + e) * q8[128 * h + 32 * k + e];
                    sumi[nn] += s * p;
                }
        for (int k = 0; k < 8; k++) acc[k] = fmaf(d, (float)sumi[k], acc[k]);
    }
    const float a = hsum8(acc);
    return a + summ;
}

int korc_qmatvec(int type, int rows, int cols, const uint8_t *w, const float *x, const float *bias, float *out,
                 int avx2) {
    if ((type != 12 && type != 14) || cols <= 0 || cols % 256 || rows < 0) return -1;
    const int nb = cols / 256;
    float *d = (float *)malloc(sizeof(float) * (size_t)nb);
    int8_t *qs = (int8_t *)malloc((size_t)cols);
    int16_t *bs = (int16_t *)malloc(sizeof(int16_t) * 16 * (size_t)nb);
    if (!d || !qs || !bs) {
        free(d);
        free(qs);
        free(bs);
        return -1;
    }
    korc_q8k_quantize(x, cols, d, qs, bs);
    const size_t row_bytes = (size_t)nb * (type == 12 ? 144 : 210);
    for (int r = 0; r < rows; r++) {
        const uint8_t *wr = w + (size_t)r * row_bytes;
        float v = type == 12 ? korc_dot_q4k(cols, wr, d, qs, bs, avx2) : korc_dot_q6k(cols, wr, d, qs, bs, avx2);
        if (bias) v = v + bias[r];
        out[r] = v;
    }
    free(d);
    free(qs);
    free(bs);
    return 0;
}
