// peer_exchange.cu — exchange and merge of KV-sharded decode partials over
// NVLink peer memory, one kernel per layer (sm_100a).
//
// A decode step on a context whose KV positions are split over N GPUs leaves
// each rank's partial result — output normalised by its own softmax sum, and
// the log2-domain log-sum-exp per query head — in a local buffer. Every
// rank's exchange buffer is mapped into every other rank (CUDA IPC), so this
// kernel, one CTA per query head:
//   1. stores the partial into this rank's slot of every peer's buffer (plain
//      NVLink stores, no multicast), then raises a per-(rank, head) flag there
//      with a system-scope release;
//   2. waits, bounded by 2 s of %globaltimer, for every peer's flag in its own
//      buffer (system-scope acquire);
//   3. merges the N partials: out = sum_r 2^(L_r - L) O_r, L = log2 sum 2^L_r,
//      which is kore's single softmax (kore.cpp:1437-1454) regrouped by shard.
// The flag value is a per-head epoch kept on the device (the CTA of head h is
// its only reader and writer), so a CUDA graph can replay the step. Two slot
// sets, selected by the epoch's parity, stop a fast rank from overwriting a
// slot that a peer has not read yet: it can reuse a set only after receiving
// the peer's next partial, which the peer sends after finishing this one.

#include "attn.cuh"
#include "common.cuh"
#include "split_merge.cuh"

namespace kore {
namespace {

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

template <int D>
__global__ void __launch_bounds__(D) peer_exchange_kernel(const __grid_constant__ ExchangeParams p) {
    const int h = blockIdx.x, tid = threadIdx.x;
    const int N = p.n_ranks, me = p.rank, H = p.H;
    const size_t PF = (size_t)H * D + H;
    __shared__ unsigned s_epoch;
    __shared__ float s_lse[kMaxRanks];

    grid_dep_launch();     // the next decode may prefetch KV of its own layer meanwhile
    grid_dep_wait();       // this rank's partial is complete and visible

    unsigned *epochs = reinterpret_cast<unsigned *>(reinterpret_cast<char *>(p.own) + p.epoch_off);
    if (tid == 0) s_epoch = epochs[h] + 1u;
    __syncthreads();
    const unsigned e = s_epoch;
    const int par = e & 1u;
    // this rank's partial of head h: the decode's own output (one split) or
    // the merge of its splits, kept in registers
    float o_me, lse_me;
    if (p.n_splits > 1) {
        const int R = p.n_rep, g = h / R, r = h - g * R;
        const size_t base = (size_t)g * p.max_splits;
        merge_head_splits<D>(p.part_o + base * R * D + (size_t)r * D + tid, (size_t)R * D, p.part_ml + base * R + r,
                             (size_t)R, p.n_splits, o_me, lse_me);
    } else {
        o_me = __ldcg(p.local + (size_t)h * D + tid);
        lse_me = __ldcg(p.local + (size_t)H * D + h);
    }

    // 1. push it to every peer, then raise this rank's flag there
    for (int r = 0; r < N; ++r) {
        if (r == me) continue;
        float *dst = p.peers[r] + ((size_t)par * N + me) * PF;
        dst[(size_t)h * D + tid] = o_me;
        if (tid == 0) dst[(size_t)H * D + h] = lse_me;
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence_system();
        for (int r = 0; r < N; ++r) {
            if (r == me) continue;
            unsigned *flags = reinterpret_cast<unsigned *>(reinterpret_cast<char *>(p.peers[r]) + p.flag_off);
            st_release_sys(flags + ((size_t)par * N + me) * H + h, e);
        }
    }

    // 2. wait for every peer's partial of head h (bounded)
    if (tid < N && tid != me) {
        const unsigned *flag =
            reinterpret_cast<const unsigned *>(reinterpret_cast<const char *>(p.own) + p.flag_off) +
            ((size_t)par * N + tid) * H + h;
        const uint64_t t0 = global_ns();
        while ((int)(ld_acquire_sys(flag) - e) < 0) {
            if (global_ns() - t0 > kWaitNs) {
                raise_error(p.err, DEV_PEER_TIMEOUT);
                break;
            }
            __nanosleep(64);
        }
    }
    __syncthreads();

    // 3. merge the N partials of head h
    if (tid < N) s_lse[tid] = tid == me ? lse_me : __ldcg(p.own + ((size_t)par * N + tid) * PF + (size_t)H * D + h);
    __syncthreads();
    float M = -INFINITY;
    for (int r = 0; r < N; ++r) M = fmaxf(M, s_lse[r]);
    float acc = 0.f, wsum = 0.f;
    if (M != -INFINITY) {
        for (int r = 0; r < N; ++r) {
            const float w = fast_exp2(s_lse[r] - M);
            wsum += w;
            const float x = r == me ? o_me : __ldcg(p.own + ((size_t)par * N + r) * PF + (size_t)h * D + tid);
            acc = fmaf(w, x, acc);
        }
    }
    p.out[(size_t)h * D + tid] = wsum > 0.f ? acc / wsum : 0.f;
    __syncthreads();
    if (tid == 0) epochs[h] = e;
}

}  // namespace

cudaError_t launch_peer_exchange(const ExchangeParams &p, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.H);
    cfg.blockDim = dim3(p.D);
    if (p.D != 64 && p.D != 128) return cudaErrorInvalidValue;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return p.D == 128 ? cudaLaunchKernelEx(&cfg, peer_exchange_kernel<128>, p)
                      : cudaLaunchKernelEx(&cfg, peer_exchange_kernel<64>, p);
}

}  // namespace kore
