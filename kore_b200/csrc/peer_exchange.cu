// peer_exchange.cu — exchange and merge of KV-sharded attention partials over
// NVLink peer memory, one kernel per layer (sm_100a).
//
// A decode step, or a piece of a prefill chunk, on a context whose KV
// positions are split over N GPUs leaves each rank's partial result — output
// normalised by its own softmax sum, and the log2-domain log-sum-exp per
// (query, head) — in a local buffer (or as the decode's unmerged splits).
// Every rank's exchange buffer is mapped into every other rank (CUDA IPC), so
// this kernel, one CTA per (query head, query):
//   1. merges this rank's splits of the (query, head) when the decode left
//      several (the split count is derived as the decode kernel derives it);
//   2. stores the partial into this rank's slot of every peer's buffer as
//      (value, epoch) pairs packed into one 64-bit word each (value in the
//      low half) — plain NVLink stores, no multicast. Each word is written by
//      one scalar st.relaxed.sys.b64 and read by one scalar ld.relaxed.sys.b64,
//      which the PTX memory model makes single-copy atomic, so a reader that
//      sees this step's epoch sees this step's value with it, and no fence or
//      flag is needed;
//   3. polls its own buffer, bounded by the context's wait limit (2 s unless
//      set otherwise) of %globaltimer, until every peer's words for the
//      (query, head) carry this step's epoch;
//   4. merges the N partials: out = sum_r 2^(L_r - L) O_r, L = log2 sum 2^L_r,
//      which is kore's single softmax (kore.cpp:1437-1454, and per prefill
//      row :1542-1563) regrouped by shard.
// The epochs are counters per (query slot, head) kept on the device (the CTA
// of that pair is their only reader and writer), so a CUDA graph can replay
// a step. Two slot sets, selected by the epoch's parity, stop a fast rank from
// overwriting a slot that a peer has not read yet: it writes a set again only
// after receiving the peer's next partial for the same slot, which the peer
// sends in a later kernel, after this one's reads of that set completed.

#include "attn.cuh"
#include "common.cuh"
#include "split_merge.cuh"

namespace kore {
namespace {

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

template <int D>
__global__ void __launch_bounds__(D) peer_exchange_kernel(const __grid_constant__ ExchangeParams p) {
    const int h = blockIdx.x, qi = blockIdx.y, tid = threadIdx.x;
    const int N = p.n_ranks, me = p.rank, H = p.H;
    constexpr int SLOT = D + 1;   // words per (rank, query, head): D outputs, then the LSE
    constexpr int Q = kExchangeQueries;
    __shared__ unsigned s_epoch;
    __shared__ float s_lse[kMaxRanks];

    grid_dep_launch();     // the next decode may prefetch KV of its own layer meanwhile
    // the epoch of (qi, h) was last written by this CTA's predecessor, an
    // exchange that finished before the decode this kernel depends on
    // started: it can be read before the wait
    unsigned *epochs = reinterpret_cast<unsigned *>(reinterpret_cast<char *>(p.own) + p.epoch_off);
    if (tid == 0) s_epoch = epochs[qi * H + h] + 1u;
    grid_dep_wait();       // this rank's partial is complete and visible
    __syncthreads();
    const unsigned e = s_epoch;
    const int par = e & 1u;
    // this rank's partial of (qi, h): the decode's own output (one split) or
    // the merge of its splits, kept in registers
    const int pos = p.pos0 + qi;
    const int count = shard_count_below(p.append_new ? pos : pos + 1, p.P, N, me);
    const int n_splits = count > 0 ? (count + p.split_tokens - 1) / p.split_tokens : 1;
    float o_me, lse_me;
    if (n_splits > 1) {
        const int R = p.n_rep, g = h / R, r = h - g * R;
        const size_t base = ((size_t)qi * (H / R) + g) * p.max_splits;
        merge_head_splits<D>(p.part_o + base * R * D + (size_t)r * D + tid, (size_t)R * D, p.part_ml + base * R + r,
                             (size_t)R, n_splits, o_me, lse_me);
    } else {
        o_me = __ldcg(p.local + ((size_t)qi * H + h) * D + tid);
        lse_me = __ldcg(p.local + (size_t)Q * H * D + (size_t)qi * H + h);
    }

    // 1. push it to every peer: one 64-bit (value, epoch) store per element
    for (int r = 0; r < N; ++r) {
        if (r == me) continue;
        uint64_t *dst = reinterpret_cast<uint64_t *>(p.peers[r]) + ((((size_t)par * N + me) * Q + qi) * H + h) * SLOT;
        st_pair_sys(dst + tid, __float_as_uint(o_me), e);
        if (tid == 0) st_pair_sys(dst + D, __float_as_uint(lse_me), e);
    }

    // 2. collect every peer's element tid (thread 0 also the LSEs)
    const uint64_t *own = reinterpret_cast<const uint64_t *>(p.own);
    float x[kMaxRanks];
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
        x[r] = 0.f;
        if (r < N && r != me) {
            const uint64_t *src = own + ((((size_t)par * N + r) * Q + qi) * H + h) * SLOT;
            x[r] = await_pair(src + tid, e, p.err, p.wait_ns);
            if (tid == 0) s_lse[r] = await_pair(src + D, e, p.err, p.wait_ns);
        }
    }
    if (tid == 0) s_lse[me] = lse_me;
    __syncthreads();

    // 3. merge the N partials of (qi, h)
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
    p.out[((size_t)qi * H + h) * D + tid] = wsum > 0.f ? acc / wsum : 0.f;
    if (tid == 0) epochs[qi * H + h] = e;
}

}  // namespace

cudaError_t launch_peer_exchange(const ExchangeParams &p, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.H, p.n_q);
    cfg.blockDim = dim3(p.D);
    if ((p.D != 64 && p.D != 128) || p.n_q <= 0 || p.n_q > kExchangeQueries || p.split_tokens <= 0)
        return cudaErrorInvalidValue;
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
