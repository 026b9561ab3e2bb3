// lse_merge.cu — merges partial attention results of disjoint KV shards.
//
// Each shard r contributes a partial output O_r (normalised by its own
// softmax sum) and its log2-domain log-sum-exp L_r = m_r + log2(l_r) per
// query head. The full softmax over the union of the shards is
//   out = sum_r 2^(L_r - L) O_r,   L = log2 sum_r 2^L_r,
// which is the same arithmetic kore's single softmax (kore.cpp:1437-1454)
// performs, regrouped by shard. Shards holding none of a head's positions
// carry L_r = -inf and weigh nothing.
//
// Packed layout of a partial of n_q queries: [n_q][H*D] floats of O, then
// [n_q][H] floats of L, so that one all-gather moves a rank's whole
// contribution.

#include "attn.cuh"
#include "common.cuh"

namespace kore {
namespace {

__global__ void lse_merge_kernel(const float *__restrict__ parts, int n_parts, int n_q, int H, int D,
                                 float *__restrict__ out) {
    const int h = blockIdx.x, qi = blockIdx.y;
    const size_t stride = (size_t)n_q * ((size_t)H * D + H);          // one part
    const size_t o_off = (size_t)qi * H * D + (size_t)h * D;          // this (query, head) in a part
    const size_t l_off = (size_t)n_q * H * D + (size_t)qi * H + h;
    float M = -INFINITY;
    for (int r = 0; r < n_parts; ++r) M = fmaxf(M, parts[r * stride + l_off]);
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        float acc = 0.f, wsum = 0.f;
        if (M != -INFINITY) {
            for (int r = 0; r < n_parts; ++r) {
                const float w = fast_exp2(parts[r * stride + l_off] - M);
                wsum += w;
                acc = fmaf(w, parts[r * stride + o_off + i], acc);
            }
        }
        out[o_off + i] = wsum > 0.f ? acc / wsum : 0.f;
    }
}

}  // namespace

cudaError_t launch_lse_merge(const float *parts, int n_parts, int n_q, int H, int D, float *out, cudaStream_t s) {
    if (n_q <= 0 || n_q > 65535) return cudaErrorInvalidValue;
    lse_merge_kernel<<<dim3(H, n_q), D, 0, s>>>(parts, n_parts, n_q, H, D, out);
    return cudaGetLastError();
}

}  // namespace kore
