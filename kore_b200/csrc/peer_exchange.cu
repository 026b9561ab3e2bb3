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
#include "exchange.cuh"
#include "split_merge.cuh"

namespace kore {
namespace {

template <int D>
__global__ void __launch_bounds__(D) peer_exchange_kernel(const __grid_constant__ ExchangeParams p) {
    const int h = blockIdx.x, qi = blockIdx.y, tid = threadIdx.x;
    const int N = p.n_ranks, me = p.rank, H = p.H;
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

    exchange_and_merge<D>(o_me, lse_me, e, p.own, p.peers, N, me, H, qi, h, p.err, p.wait_ns, p.out, s_lse);
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
