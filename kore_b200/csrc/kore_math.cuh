// kore_math.cuh — kore's own scalar arithmetic, restated for the device
// kernels that must match it bit for bit: RMSNorm's rounded mean square, the
// C library's expf as kore's SwiGLU calls it, and the dequantisation of
// GGUF Q4_K / Q6_K blocks. Every operation is an explicit round-to-nearest
// intrinsic, so the compiler fuses nothing that kore does not.
#pragma once

#include <cstdint>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace kore {

// The float kore's rmsnorm (kore.cpp:1369-1370) makes of its sequential
// double sum of squares, (float)(ss / n), given a sum S of the same squares
// in another order. Every square of a float is exact in double, so the two
// sums differ by at most (n + log2 n) units of 2^-53 of the sum: when the
// rounded mean cannot change within that bound (checked with margin) the
// float is returned, else NaN (the caller then sums in kore's order).
__device__ __forceinline__ float mean_square_float(double S, int n) {
    const double v = __ddiv_rn(S, (double)n);
    const float f = __double2float_rn(v);
    const double lo = ((double)f + (double)nextafterf(f, -INFINITY)) * 0.5;
    const double hi = ((double)f + (double)nextafterf(f, INFINITY)) * 0.5;
    const double m = v * (double)(n + 64) * 0x1p-52;
    return (v - m > lo && v + m < hi) ? f : __int_as_float(0x7fffffff);
}

// kore's rmsnorm scale 1 / sqrt(mean(x^2) + eps) (kore.cpp:1367-1370) for a
// CTA of nthreads (a multiple of 32): every thread gets the same float.
// red: shared scratch of nthreads/32 doubles, s_out: one shared float.
__device__ __forceinline__ float block_rms_scale(const float *__restrict__ x, int n, float eps, double *red,
                                                 float *s_out) {
    const int tid = threadIdx.x, nthreads = blockDim.x;
    double ss = 0.0;
    for (int i = tid; i < n; i += nthreads) {
        const double xi = (double)x[i];
        ss = __dadd_rn(ss, __dmul_rn(xi, xi));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss = __dadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    if (tid == 0) {
        double S = 0.0;
        for (int w = 0; w < nthreads / 32; ++w) S = __dadd_rn(S, red[w]);
        float f = mean_square_float(S, n);
        if (f != f) {   // too close to a rounding boundary (or not finite): kore's order
            double seq = 0.0;
            for (int i = 0; i < n; ++i) {
                const double xi = (double)x[i];
                seq = __dadd_rn(seq, __dmul_rn(xi, xi));
            }
            f = __double2float_rn(__ddiv_rn(seq, (double)n));
        }
        *s_out = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(f, eps)));
    }
    __syncthreads();
    return *s_out;
}

// kore's std::exp(float) is the C library's expf, which on glibc (2.27 and
// later) is the table-driven method of ARM's optimized-routines (Szabolcs
// Nagy): x * 32/ln2 = k + r, the reduced argument formed with one fused
// multiply-add, 2^(k/32) from a table of 2^(i/32), a cubic in r, all in
// double, one rounding to float at the end. Restated here with each double
// operation rounded as the library rounds it; tab[i] = bits(2^(i/32)) -
// (i << 47) from the host's exp2. Checked against the host's expf on all 2^32
// floats: identical except NaN payloads.
__device__ __forceinline__ float kore_expf(float x, const unsigned long long *tab) {
    if (x != x) return x + x;
    if (x > 0x1.62e42ep6f) return __int_as_float(0x7f800000);   // overflow: +inf
    if (x < -0x1.9fe368p6f) return 0.0f;                          // below half the smallest subnormal
    constexpr double kShift = 0x1.8p52, kInvLn2N = 0x1.71547652b82fep+0 * 32;
    constexpr double kC0 = 0x1.c6af84b912394p-5 / 32768, kC1 = 0x1.ebfce50fac4f3p-3 / 1024,
                     kC2 = 0x1.62e42ff0c52d6p-1 / 32;
    const double xd = (double)x;
    double kd = __dadd_rn(__dmul_rn(kInvLn2N, xd), kShift);
    const unsigned long long ki = (unsigned long long)__double_as_longlong(kd);
    kd = __dsub_rn(kd, kShift);
    const double r = __fma_rn(kInvLn2N, xd, -kd);
    const double s = __longlong_as_double((long long)(tab[ki & 31] + (ki << 47)));
    const double r2 = __dmul_rn(r, r);
    const double y = __dadd_rn(__dmul_rn(__dadd_rn(__dmul_rn(kC0, r), kC1), r2), __dadd_rn(__dmul_rn(kC2, r), 1.0));
    return __double2float_rn(__dmul_rn(y, s));
}

// kore.cpp:1465-1468 (and :1578-1584): g / (1 + exp(-g)) * u.
__device__ __forceinline__ float kore_swiglu(float g, float u, const unsigned long long *tab) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, kore_expf(-g, tab))), u);
}

// ---------------------------------------------------------------- GGUF blocks

__device__ __forceinline__ float f16_at(const uint8_t *p) {
    return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

// kore's get_scale_min_k4 (kore.cpp:327-335): the 6-bit scale and min of
// sub-block j from the 12 packed bytes q.
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t *q, int &sc, int &mn) {
    if (j < 4) {
        sc = q[j] & 63;
        mn = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 0x0F) | ((q[j - 4] >> 6) << 4);
        mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// Value j (0..255) of a Q4_K block, as dequant_block_q4_K (kore.cpp:337-354):
// (d * scale) * q - dmin * min, each product and the difference rounded.
__device__ __forceinline__ float q4k_value(const uint8_t *b, int j) {
    const int chunk = j >> 6, jj = j & 63, l = jj & 31;
    int sc, mn;
    scale_min_k4(2 * chunk + (jj >> 5), b + 4, sc, mn);
    const float d1 = __fmul_rn(f16_at(b), (float)sc), m1 = __fmul_rn(f16_at(b + 2), (float)mn);
    const int q = b[16 + 32 * chunk + l];
    const int nib = jj < 32 ? (q & 0x0F) : (q >> 4);
    return __fsub_rn(__fmul_rn(d1, (float)nib), m1);
}

// Value j (0..255) of a Q6_K block, as dequant_block_q6_K (kore.cpp:359-381):
// (d * scale) * (q - 32).
__device__ __forceinline__ float q6k_value(const uint8_t *b, int j) {
    const int half = j >> 7, jj = j & 127, g = jj >> 5, l = jj & 31;
    const uint8_t *ql = b + 64 * half, *qh = b + 128 + 32 * half;
    const int8_t *sc = reinterpret_cast<const int8_t *>(b + 192 + 8 * half);
    const int lo = (g & 1) ? ql[l + 32] : ql[l];
    const int q = (((g & 2) ? (lo >> 4) : (lo & 0x0F)) | (((qh[l] >> (2 * g)) & 3) << 4)) - 32;
    return __fmul_rn(__fmul_rn(f16_at(b + 208), (float)sc[(l >> 4) + 2 * g]), (float)q);
}

}  // namespace kore
