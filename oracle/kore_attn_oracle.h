/*
 * kore_attn_oracle.h — CPU restatement of kore's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This is the checker the CUDA path is compared
 * against; nothing in the product (kore_b200/, include/) links or calls it.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline use it.
 *
 * Every function restates, in plain C, the arithmetic of one region of the
 * reference engine (kore.cpp, BJZR/kore); the cited lines are the ones it
 * follows. Parity of this restatement with the reference itself is pinned by
 * tests/test_oracle_pin.py (against the reference compiled in place by
 * oracle/Makefile into oracle/_ref/) and by the committed golden vectors in
 * tests/golden/ (generated from that same compiled reference).
 */
#ifndef KORE_ATTN_ORACLE_H
#define KORE_ATTN_ORACLE_H

#ifdef __cplusplus
extern "C" {
#endif

/* kore.cpp:1337-1339: inv_freq[i] = (float)pow((double)rope_base, -2.0*i/head_dim). */
void korc_inv_freq(float rope_base, int head_dim, float *inv_freq);

/* kore.cpp:1405-1410 (decode) and :1503-1512 (prefill): per-position angle
 * tables, c[i] = (float)cos((double)pos * inv_freq[i]), s[i] likewise. */
void korc_rope_angles(const float *inv_freq, int half, int pos, float *c, float *s);

/* kore.cpp:1374-1384: NEOX rotation of pairs (i, i+hd/2), in place, fp32,
 * products and the difference/sum rounded separately (no fused multiply-add,
 * matching the reference's baseline x86-64 build of this function). */
void korc_rope_neox(float *vec, int n_heads, int hd, const float *c, const float *s);

/* Returns 1 when kore would pick its AVX2/FMA kernels on this CPU
 * (kore.cpp:516-519, :1294: e.avx2 = KORE_HAVE_AVX2 && cpu_has_avx2()). */
int korc_cpu_has_avx2(void);

/* kore.cpp:693-710: hd_dot. avx2 != 0 restates hd_dot_avx2 (two 8-lane fused
 * accumulators over a 16-element stride, then the hsum256 pairing order of
 * kore.cpp:521-528); avx2 == 0 restates the sequential scalar loop. */
float korc_hd_dot(const float *a, const float *b, int n, int avx2);

/* kore.cpp:712-725: hd_fma, o[i] += p*v[i] (fused per element when avx2). */
void korc_hd_fma(float *o, const float *v, float p, int n, int avx2);

/*
 * Decode step for one layer, kore.cpp:1424-1455.
 *   q   [H*d]   bias-added, pre-RoPE query of the token at `pos`
 *   k,v [G*d]   bias-added, pre-RoPE key and value of that token
 *   kc,vc       this layer's cache, [ctx][G*d] rows (kore.cpp:1427-1428);
 *               rows 0..pos-1 hold post-RoPE keys / values, row `pos` is
 *               written here (kore.cpp:1429-1430)
 *   out [H*d]   attention output (e.att, kore.cpp:1447)
 *   scores      scratch of at least pos+1 floats (e.scores)
 * Returns 0, or -1 on a bad argument.
 */
int korc_attn_decode(int H, int G, int d, const float *inv_freq, int pos,
                     const float *q, const float *k, const float *v,
                     float *kc, float *vc, float *out, float *scores);

/*
 * Batched prefill chunk for one layer, kore.cpp:1527-1563: appends the n
 * tokens at positions pos0..pos0+n-1 (RoPE on q and k, kore.cpp:1527-1539),
 * then causal attention for each (head, token) with limit pos0+z, dot
 * products by hd_dot and the P.V accumulation by hd_fma.
 *   q [n][H*d], k,v [n][G*d]  bias-added, pre-RoPE
 *   out [n][H*d]              e.batt rows
 *   scores                    scratch of at least (pos0+n) + n*H*d floats
 *                             (score row, then the rotated queries, e.bq)
 */
int korc_attn_prefill(int H, int G, int d, const float *inv_freq, int pos0, int n,
                      const float *q, const float *k, const float *v,
                      float *kc, float *vc, float *out, float *scores, int avx2);

/* Post-RoPE key row for position pos, exactly as kore stores it in the cache
 * (kore.cpp:1424, :1429): k_out[G*d] = rope_neox(k_pre) with pos's tables. */
void korc_rope_key(int G, int d, const float *inv_freq, int pos, const float *k_pre, float *k_out);

/* kore.cpp:1601-1603 with temp <= 0: index of the first maximum. */
int korc_argmax(const float *logits, int n);

#ifdef __cplusplus
}
#endif
#endif
