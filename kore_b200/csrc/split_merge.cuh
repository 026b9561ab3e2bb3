// split_merge.cuh — merge of one query head's KV-split partials (one CTA,
// one thread per dim), shared by split_merge_kernel and the cross-GPU
// exchange kernel.
#pragma once

#include "attn.cuh"
#include "common.cuh"

namespace kore {

// For a CTA of D threads: thread t's dim of split s is po[s * stride], the
// split's (max, sum) is ml[s * ml_stride]. Returns the normalised output of
// dim t, out = sum_s 2^(m_s - M) o_s / sum_s 2^(m_s - M) l_s, and (in every
// thread) the merged log2-domain log-sum-exp M + log2(L). All partial loads
// of a thread (up to 64 splits) are issued before the weights are known.
template <int D>
__device__ __forceinline__ void merge_head_splits(const float *__restrict__ po, size_t stride,
                                                  const float2 *__restrict__ ml, size_t ml_stride, int n_splits,
                                                  float &out, float &lse) {
    constexpr int CH = 64;
    constexpr unsigned FULLM = 0xffffffffu;
    __shared__ float w[kMaxSplits];
    __shared__ float red[D / 32];
    __shared__ float s_M, s_L;
    const int tid = threadIdx.x;
    constexpr int MLP = (kMaxSplits + D - 1) / D;   // split (max, sum) pairs held per thread
    // every load of this thread issued at once: its dim of up to CH splits and
    // the (max, sum) pairs of the splits it weighs; one round trip in total
    float v[CH];
#pragma unroll
    for (int s = 0; s < CH; ++s) v[s] = s < n_splits ? __ldcg(po + (size_t)s * stride) : 0.f;
    float2 mls[MLP];
#pragma unroll
    for (int k = 0; k < MLP; ++k) {
        const int s = tid + k * D;
        mls[k] = s < n_splits ? __ldcg(ml + (size_t)s * ml_stride) : make_float2(-INFINITY, 0.f);
    }
    float M = -INFINITY;
#pragma unroll
    for (int k = 0; k < MLP; ++k) M = fmaxf(M, mls[k].x);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(FULLM, M, off));
    if ((tid & 31) == 0) red[tid >> 5] = M;
    __syncthreads();
    if (tid == 0) {
        float m = red[0];
        for (int i = 1; i < D / 32; ++i) m = fmaxf(m, red[i]);
        s_M = m;
    }
    __syncthreads();
    M = s_M;
    float L = 0.f;
#pragma unroll
    for (int k = 0; k < MLP; ++k) {
        const int s = tid + k * D;
        if (s < n_splits) {
            const float ws = M == -INFINITY ? 0.f : fast_exp2(mls[k].x - M);
            w[s] = ws;
            L = fmaf(mls[k].y, ws, L);
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(FULLM, L, off);
    __syncthreads();
    if ((tid & 31) == 0) red[tid >> 5] = L;
    __syncthreads();
    if (tid == 0) {
        float l = 0.f;
        for (int i = 0; i < D / 32; ++i) l += red[i];
        s_L = l;
    }
    __syncthreads();
    L = s_L;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
    for (int s = 0; s < CH; s += 4) {
        if (s < n_splits) a0 = fmaf(w[s], v[s], a0);
        if (s + 1 < n_splits) a1 = fmaf(w[s + 1], v[s + 1], a1);
        if (s + 2 < n_splits) a2 = fmaf(w[s + 2], v[s + 2], a2);
        if (s + 3 < n_splits) a3 = fmaf(w[s + 3], v[s + 3], a3);
    }
    for (int c0 = CH; c0 < n_splits; c0 += CH) {
#pragma unroll
        for (int s = 0; s < CH; ++s) v[s] = c0 + s < n_splits ? __ldcg(po + (size_t)(c0 + s) * stride) : 0.f;
#pragma unroll
        for (int s = 0; s < CH; ++s)
            if (c0 + s < n_splits) a0 = fmaf(w[c0 + s], v[s], a0);
    }
    const float acc = (a0 + a1) + (a2 + a3);
    out = L > 0.f ? acc / L : 0.f;
    lse = L > 0.f ? M + __log2f(L) : -INFINITY;
}

}  // namespace kore
