// exchange.cuh — the cross-GPU exchange of one (query, head) partial over
// NVLink peer memory, shared by peer_exchange_kernel (its own launch) and the
// decode kernel's exchange CTAs (one launch with the decode on a KV-split
// context). See peer_exchange.cu for the protocol.
#pragma once

#include "attn.cuh"
#include "common.cuh"

namespace kore {

// One (value, epoch) pair as a single 64-bit word: one scalar access, which
// is single-copy atomic (a vector access of two 32-bit halves would not be).
__device__ __forceinline__ void st_pair_sys(uint64_t *p, uint32_t value, uint32_t epoch) {
    const uint64_t w = (uint64_t)value | ((uint64_t)epoch << 32);
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ uint64_t ld_pair_sys(const uint64_t *p) {
    uint64_t w;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

// Waits (bounded by limit_ns) until the word at p carries `epoch`; returns its value.
__device__ __forceinline__ float await_pair(const uint64_t *p, uint32_t epoch, int *err, uint64_t limit_ns) {
    uint64_t w = ld_pair_sys(p);
    if ((uint32_t)(w >> 32) == epoch) return __uint_as_float((uint32_t)w);
    const uint64_t t0 = global_ns();
    for (;;) {
        w = ld_pair_sys(p);
        if ((uint32_t)(w >> 32) == epoch) return __uint_as_float((uint32_t)w);
        if (global_ns() - t0 > limit_ns) {
            raise_error(err, DEV_PEER_TIMEOUT);
            return 0.f;
        }
    }
}

// For D threads (thread tid = one dim): given this rank's partial (o_me,
// lse_me) of (query slot qi, head h) and the step's epoch e, pushes it into
// every peer's slot, collects every peer's partial of the same (qi, h) and
// writes the merged output (kore's single softmax regrouped by rank):
// out = sum_r 2^(L_r - L) O_r. s_lse: shared [kMaxRanks].
template <int D>
__device__ __forceinline__ void exchange_and_merge(float o_me, float lse_me, unsigned e, float *own,
                                                   float *const *peers, int N, int me, int H, int qi, int h,
                                                   int *err, uint64_t wait_ns, float *out, float *s_lse) {
    constexpr int SLOT = D + 1;   // words per (rank, query, head): D outputs, then the LSE
    constexpr int Q = kExchangeQueries;
    const int tid = threadIdx.x;
    const int par = e & 1u;
    // 1. push it to every peer: one 64-bit (value, epoch) store per element
    for (int r = 0; r < N; ++r) {
        if (r == me) continue;
        uint64_t *dst = reinterpret_cast<uint64_t *>(peers[r]) + ((((size_t)par * N + me) * Q + qi) * H + h) * SLOT;
        st_pair_sys(dst + tid, __float_as_uint(o_me), e);
        if (tid == 0) st_pair_sys(dst + D, __float_as_uint(lse_me), e);
    }
    // 2. collect every peer's element tid (thread 0 also the LSEs)
    const uint64_t *ownw = reinterpret_cast<const uint64_t *>(own);
    float x[kMaxRanks];
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
        x[r] = 0.f;
        if (r < N && r != me) {
            const uint64_t *src = ownw + ((((size_t)par * N + r) * Q + qi) * H + h) * SLOT;
            x[r] = await_pair(src + tid, e, err, wait_ns);
            if (tid == 0) s_lse[r] = await_pair(src + D, e, err, wait_ns);
        }
    }
    if (tid == 0) s_lse[me] = lse_me;
    __syncthreads();
    // 3. merge the N partials
    float M = -INFINITY;
    for (int r = 0; r < N; ++r) M = fmaxf(M, s_lse[r]);
    float acc = 0.f, wsum = 0.f;
    if (M != -INFINITY) {
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r) {
            if (r >= N) break;
            const float w = fast_exp2(s_lse[r] - M);
            wsum += w;
            acc = fmaf(w, r == me ? o_me : x[r], acc);
        }
    }
    out[((size_t)qi * H + h) * D + tid] = wsum > 0.f ? acc / wsum : 0.f;
}

}  // namespace kore
