/*
 * kore_proj_oracle.h — CPU restatement of kore's quantised projections.
 *
 * TEST INFRASTRUCTURE ONLY. This is the checker the CUDA projections are
 * compared against; nothing in the product (kore_b200/, include/) links or
 * calls it. Only tests/ use it.
 *
 * kore's decode step runs every projection as W * x with W in a GGUF k-quant
 * format (Q4_K or Q6_K, blocks of 256 values) and x quantised to Q8_K
 * (kore.cpp:1388-1394 mv/quant). The integer parts (Q8_K quantisation, the
 * per-block integer dot products) are exact; the float parts follow kore's
 * AVX2 kernels lane by lane (kore picks them on every AVX2/FMA CPU,
 * kore.cpp:1294), with fmaf() exactly where kore uses _mm256_fmadd_ps /
 * _mm_fmadd_ps, or its scalar reference kernels when avx2 == 0. Parity with
 * the reference itself is pinned by tests/test_proj_oracle_pin.py against the
 * reference compiled in place (oracle/_ref/libkore_ref.so) and by golden
 * hashes in tests/golden/.
 *
 * Q8_K is held as three arrays per vector of n = 256*nb values: d[nb]
 * (block scale), qs[nb*256] (int8), bsums[nb*16] (int16 sums of 16 values),
 * the fields of kore's BlockQ8K (kore.cpp:415-420).
 */
#ifndef KORE_PROJ_ORACLE_H
#define KORE_PROJ_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* kore.cpp:297-316: IEEE half to float, exact. */
float korc_f16_to_f32(uint16_t h);

/* kore.cpp:422-447: quantize_row_q8_K. n a multiple of 256. */
void korc_q8k_quantize(const float *x, int n, float *d, int8_t *qs, int16_t *bsums);

/* kore.cpp:451-477 (avx2 == 0) and :540-590 (avx2 != 0): one Q4_K row of
 * n values (n/256 blocks of 144 bytes) against Q8_K x. */
float korc_dot_q4k(int n, const uint8_t *w, const float *d, const int8_t *qs, const int16_t *bsums, int avx2);

/* kore.cpp:480-507 (avx2 == 0) and :594-640 (avx2 != 0): one Q6_K row of
 * n values (n/256 blocks of 210 bytes) against Q8_K x. */
float korc_dot_q6k(int n, const uint8_t *w, const float *d, const int8_t *qs, const int16_t *bsums, int avx2);

/* kore.cpp:1388-1394 + :650-662: out[r] = row r of W (type 12 = Q4_K,
 * 14 = Q6_K; rows x cols, cols a multiple of 256) . quantize(x), then
 * out[r] += bias[r] when bias is not NULL (kore.cpp:1422-1423). Returns 0, or
 * -1 for an unsupported type or shape. */
int korc_qmatvec(int type, int rows, int cols, const uint8_t *w, const float *x, const float *bias, float *out,
                 int avx2);

#ifdef __cplusplus
}
#endif

#endif
