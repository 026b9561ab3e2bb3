// attn_decode.cu — split-KV flash-decode over the paged fp32 KV cache (sm_100a).
//
// Replaces kore's decode attention (kore.cpp:1424-1455): RoPE of q and of the
// new k at `pos`, append of k/v at `pos`, then softmax(q k^T / sqrt(d)) v over
// positions 0..pos for every query head. kore reads each KV head once per
// query head of its group (n_rep times); here one CTA serves the whole group,
// so every K/V byte crosses HBM once. The kernel is HBM-bound: per cached
// position it reads 2*d*4 bytes and does 2*R*d FMAs (R = n_rep).
//
// Work decomposition
//   grid = (splits, n_head_kv, queries). A CTA owns one KV head of one query
//   and a contiguous range of `split_tokens` cached positions, cut into
//   TT-token tiles; tile i goes to warp i % NW. Every warp streams its own
//   tiles into a private ring of SPW shared-memory stages with 1-D bulk copies
//   (cp.async.bulk, mbarrier completion, L2 evict-first), refilling a stage as
//   soon as it has consumed it, so no warp ever waits for another.
//
// Lane layout inside a warp (D = 128: VEC = 4 dims per lane)
//   lane owns dims [VEC*lane, VEC*lane+VEC) of q (R heads, pre-scaled by
//   log2(e)/sqrt(d)) and of the output accumulator o. A K row is one 16-byte
//   shared load per lane. The scores of 4 tokens x R heads are reduced across
//   the warp by a butterfly reduce-scatter (xor 16, 8 split tokens; xor 4, 2,
//   1 split heads): 28 shuffles per 4 tokens for R = 7, after which lane L
//   holds the full score of token L>>3 for head L&7. Probabilities go through
//   a small per-warp buffer so that every lane accumulates p*v for all R
//   heads over its VEC dims.
//
// Softmax: online, with a lazily moved reference maximum. Probabilities are
// exp2(s - m_ref); m_ref and the accumulators are rescaled only when a score
// exceeds m_ref by more than 8 (log2 domain; checked with one warp vote per
// tile), so the common tile needs no maximum reduction at all. The final
// division by the running sum cancels m_ref exactly, as in any online softmax.
//
// Merge: warps merge in shared memory; with one split the CTA writes the
// normalised output, otherwise it writes (max, sum, o) to scratch. A
// single-query decode then counts its arrival per query head, and one merge
// CTA per query head at the end of the same grid waits for its head's splits
// and combines them (fused_exchange_cta; on a KV-split context it also runs
// the cross-GPU exchange). Otherwise split_merge_kernel — launched next with
// a programmatic dependency, one CTA per query head with every partial load
// in flight at once — combines the splits. The merge in the decode's own
// launch lets the next layer's dependency wait return ~4 us earlier (traced:
// the separate kernel's CTAs sit behind the decode grid, then wait for its
// completion). (A last-arriving-CTA merge, ordered by an atomic, measured ~8 us of
// serial tail per launch on B200: the release atomic drains the CTA's stores
// and one SM then pulls every partial of its head.) In a KV-sharded context
// (positions split over GPUs) the output is the normalised partial plus its
// log2-domain log-sum-exp.

#include "../../include/kore_cuda.h"
#include "attn.cuh"
#include "common.cuh"
#include "exchange.cuh"
#include "split_merge.cuh"

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

namespace kore {
namespace {

constexpr unsigned FULL = 0xffffffffu;
constexpr float kRescaleLog2 = 8.0f;   // accumulators may grow by up to 2^8 before a rescale
constexpr int kSplitPagesMax = 128;    // page ids of one split kept in shared memory

template <int D, int NW, int TT, int SPW>
struct DecodeSmem {
    static constexpr int TILE_F = TT * D;
    static constexpr size_t stage_floats = (size_t)NW * SPW * 2 * TILE_F;
    static constexpr size_t new_floats = 2 * 4 * D;
    static constexpr size_t pbuf_floats = (size_t)NW * TT * 8;
    // q of the whole group (up to 8 heads), the RoPE row of pos, new k and v
    static constexpr size_t qsm_floats = (size_t)11 * D;
    static constexpr size_t bar_off = (stage_floats + new_floats + pbuf_floats + qsm_floats) * 4;
    static constexpr size_t bytes = bar_off + (size_t)NW * SPW * 8 + kSplitPagesMax * 4;
};

template <int D, int R>
struct WarpState {
    static constexpr int VEC = D / 32;
    float q[R][VEC];
    float o[R][VEC];
    float m[R];     // reference maximum of every head (same in all lanes)
    float mo;       // reference maximum of this lane's head (lane & 7)
    float l;        // lane-partial running sum of this lane's head
};

template <int VEC>
__device__ __forceinline__ void load_row(const float *p, float (&x)[VEC]) {
    if constexpr (VEC == 4) {
        const float4 v = *reinterpret_cast<const float4 *>(p);
        x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
    } else {
        const float2 v = *reinterpret_cast<const float2 *>(p);
        x[0] = v.x; x[1] = v.y;
    }
}

// One tile of nv (1..TT) tokens for one warp: K rows at Ks, V rows at Vs
// (shared memory, row stride D). Rows at and past nv are never accumulated.
template <int D, int R, int TT>
__device__ __forceinline__ void process_tile(WarpState<D, R> &st, const float *__restrict__ Ks,
                                             const float *__restrict__ Vs, int nv, float *__restrict__ pbuf,
                                             int lane) {
    constexpr int VEC = D / 32;
    constexpr int ROUNDS = TT / 4;
    const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4, b1 = lane & 2, b0 = lane & 1;
    const int tl = lane >> 3;   // token (within a round) whose score this lane ends up with

    float sc[ROUNDS];
#pragma unroll
    for (int r = 0; r < ROUNDS; ++r) {
        float part[4][R];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            float kv[VEC];
            load_row<VEC>(Ks + (r * 4 + t) * D + lane * VEC, kv);
#pragma unroll
            for (int h = 0; h < R; ++h) {
                float a = st.q[h][0] * kv[0];
#pragma unroll
                for (int j = 1; j < VEC; ++j) a = fmaf(st.q[h][j], kv[j], a);
                part[t][h] = a;
            }
        }
        float a1[2][R];   // xor 16: keep tokens {2,3} (bit set) or {0,1}
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int h = 0; h < R; ++h) {
                const float mine = b4 ? part[2 + j][h] : part[j][h];
                const float other = b4 ? part[j][h] : part[2 + j][h];
                a1[j][h] = mine + __shfl_xor_sync(FULL, other, 16);
            }
        float a2[8];      // xor 8: keep token {1} or {0}
#pragma unroll
        for (int h = 0; h < R; ++h) {
            const float mine = b3 ? a1[1][h] : a1[0][h];
            const float other = b3 ? a1[0][h] : a1[1][h];
            a2[h] = mine + __shfl_xor_sync(FULL, other, 8);
        }
#pragma unroll
        for (int h = R; h < 8; ++h) a2[h] = 0.f;
        float a3[4];      // xor 4: keep heads {4..7} or {0..3}
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float mine = b2 ? a2[4 + j] : a2[j];
            const float other = b2 ? a2[j] : a2[4 + j];
            a3[j] = j < R ? mine + __shfl_xor_sync(FULL, other, 4) : 0.f;
        }
        float a4[2];      // xor 2: keep heads {2,3} or {0,1} of those
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const float mine = b1 ? a3[2 + j] : a3[j];
            const float other = b1 ? a3[j] : a3[2 + j];
            a4[j] = j < R ? mine + __shfl_xor_sync(FULL, other, 2) : 0.f;
        }
        const float mine = b0 ? a4[1] : a4[0];
        const float other = b0 ? a4[0] : a4[1];
        const float s = mine + __shfl_xor_sync(FULL, other, 1);
        sc[r] = r * 4 + tl < nv ? s : -INFINITY;
    }

    // lazy rescale: only when some score exceeds its head's reference by 2^8
    bool need = false;
#pragma unroll
    for (int r = 0; r < ROUNDS; ++r) need |= sc[r] > st.mo + kRescaleLog2;
    if (__any_sync(FULL, need)) {
        float tm = sc[0];
#pragma unroll
        for (int r = 1; r < ROUNDS; ++r) tm = fmaxf(tm, sc[r]);
        tm = fmaxf(tm, __shfl_xor_sync(FULL, tm, 8));
        tm = fmaxf(tm, __shfl_xor_sync(FULL, tm, 16));
        const float mnew = fmaxf(st.mo, tm);
        st.l *= fast_exp2(st.mo - mnew);
        st.mo = mnew;
#pragma unroll
        for (int h = 0; h < R; ++h) {
            const float mh = __shfl_sync(FULL, mnew, h);
            const float alpha = fast_exp2(st.m[h] - mh);
            st.m[h] = mh;
#pragma unroll
            for (int j = 0; j < VEC; ++j) st.o[h][j] *= alpha;
        }
    }
#pragma unroll
    for (int r = 0; r < ROUNDS; ++r) {
        const float p = fast_exp2(sc[r] - st.mo);
        st.l += p;
        pbuf[(r * 4 + tl) * 8 + (lane & 7)] = p;
    }
    __syncwarp();

    auto pv_row = [&](int t) {
        const float4 p0 = *reinterpret_cast<const float4 *>(pbuf + t * 8);
        const float4 p1 = *reinterpret_cast<const float4 *>(pbuf + t * 8 + 4);
        const float pr[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
        float vv[VEC];
        load_row<VEC>(Vs + t * D + lane * VEC, vv);
#pragma unroll
        for (int h = 0; h < R; ++h)
#pragma unroll
            for (int j = 0; j < VEC; ++j) st.o[h][j] = fmaf(pr[h], vv[j], st.o[h][j]);
    };
    if (nv == TT) {
#pragma unroll
        for (int t = 0; t < TT; ++t) pv_row(t);
    } else {
        for (int t = 0; t < nv; ++t) pv_row(t);
    }
    __syncwarp();
}

#ifdef KORE_TRACE
// Trace build: every decode, split-merge and merge CTA stamps (TraceRec::t)
// entry, dependency wait returned, inputs staged / arrivals seen, tiles done,
// end. Kinds: 0 decode, 1 split_merge_kernel, 2 merge CTA of a fused launch.
KORE_TRACE_BUFFER();
#endif

// The merge CTA of query head h at the end of a fused decode launch (the
// first D threads; the others leave): waits for the head's splits to arrive
// and merges them (as split_merge_kernel would). On a KV-split context it then
// exchanges and merges the ranks' partials (exchange.cuh), as
// peer_exchange_kernel does for one query; on one GPU it writes the output.
template <int D, int R>
__device__ __forceinline__ void fused_exchange_cta(const DecodeParams &p, int h) {
    __shared__ unsigned s_epoch;
    __shared__ float s_lse[kMaxRanks];
    KTRACE_OPEN(2);
    grid_dep_launch();
    grid_dep_wait();   // the previous step's exchange (the epochs) and this step's inputs
    KTRACE(1);
    const int tid = threadIdx.x;
    if (tid >= D) return;
    const PagedKv &kv = p.kv;
    const int pos = p.pos0;
    const int count = shard_count_below(p.append_new ? pos : pos + 1, kv.P, kv.shard_count, kv.shard_rank);
    int n_splits = (count + p.split_tokens - 1) / p.split_tokens;
    if (n_splits == 0) n_splits = 1;
    const bool xchg = p.x_ranks > 1;
    unsigned *epochs =
        xchg ? reinterpret_cast<unsigned *>(reinterpret_cast<char *>(p.x_own) + p.x_epoch_off) : nullptr;
    if (tid == 0) {
        if (xchg) s_epoch = epochs[h] + 1u;
        // bounded wait for the head's n_splits partials (their writes are
        // released by a fence before each arrival is counted)
        int seen = 0;
        const uint64_t t0 = global_ns();
        for (uint32_t it = 0;; ++it) {
            asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(seen) : "l"(p.x_arrivals + h) : "memory");
            if (seen >= n_splits) break;
            if ((it & 15) == 15 && global_ns() - t0 > p.wait_ns) {
                raise_error(p.err, DEV_WAIT_FULL_TIMEOUT);
                break;
            }
        }
        p.x_arrivals[h] = 0;   // for the next launch (stream-ordered after this one)
    }
    __syncthreads();
    KTRACE(2);
    const int g = h / R, r = h - g * R;
    if (!xchg) {   // one GPU: the merged splits are the output (one split wrote it directly)
        if (n_splits > 1) {
            const size_t base = (size_t)g * p.max_splits;
            float o, lse;
            merge_head_splits<D>(p.part_o + base * R * D + (size_t)r * D + tid, (size_t)R * D,
                                 p.part_ml + base * R + r, (size_t)R, n_splits, o, lse);
            p.out[(size_t)h * D + tid] = o;
            if (p.lse && tid == 0) p.lse[h] = lse;
        }
        KTRACE(4);
        return;
    }
    const unsigned e = s_epoch;
    float o_me, lse_me;
    if (n_splits > 1) {
        const size_t base = (size_t)g * p.max_splits;
        merge_head_splits<D>(p.part_o + base * R * D + (size_t)r * D + tid, (size_t)R * D, p.part_ml + base * R + r,
                             (size_t)R, n_splits, o_me, lse_me);
    } else {
        o_me = __ldcg(p.out + (size_t)h * D + tid);
        lse_me = __ldcg(p.lse + h);
    }
    exchange_and_merge<D>(o_me, lse_me, e, p.x_own, p.x_peers, p.x_ranks, kv.shard_rank, p.H, 0, h, p.err, p.wait_ns,
                          p.x_out, s_lse);
    if (tid == 0) epochs[h] = e;
    KTRACE(4);
}

// The CTA merge of its NW warps' states, left in shared memory as cm [NW][8]
// reference maxima, cl [NW][8] sums and co [NW][R][D] unnormalised outputs:
// the query's normalised output (one split; plus its log2-domain LSE when
// asked) or the split's partial (max, sum, o) in the split scratch; in a
// fused launch the split's arrival is then counted for the heads' merge CTAs.
// The weights 2^(m_w - M) and the sums are formed once per (warp, head) in
// shared memory (wsm: [NW][8] weights, then [8] maxima and [8] sums), then
// each thread combines float4 runs of dims, every product in warp order.
template <int D, int R, int NW>
__device__ __forceinline__ void cta_merge_write(const DecodeParams &p, const float *cm, float *wsm, int qi, int g,
                                                int split, int n_splits) {
    constexpr int NT = NW * 32;
    const int tid = threadIdx.x;
    const float *cl = cm + NW * 8;
    const float *co = cl + NW * 8;
    float *sM = wsm + NW * 8, *sL = sM + 8;
    const size_t qh0 = (size_t)qi * p.H + (size_t)g * R;     // first query head of the group
    const size_t part_base = ((size_t)qi * p.kv.G + g) * p.max_splits;
    if (tid < R) {
        const int h = tid;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; ++w) M = fmaxf(M, cm[w * 8 + h]);
        float L = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const float e = M == -INFINITY ? 0.f : fast_exp2(cm[w * 8 + h] - M);
            wsm[w * 8 + h] = e;
            L = fmaf(cl[w * 8 + h], e, L);
        }
        sM[h] = M;
        sL[h] = L;
        if (n_splits == 1) {
            if (p.lse) p.lse[qh0 + h] = L > 0.f ? M + __log2f(L) : -INFINITY;
        } else {
            p.part_ml[(part_base + split) * R + h] = make_float2(M, L);
        }
    }
    __syncthreads();
    float *dst = n_splits == 1 ? p.out + qh0 * D : p.part_o + (part_base + split) * R * D;
    const bool vec = (reinterpret_cast<uintptr_t>(dst) & 15) == 0;
    for (int i4 = tid; i4 < R * D / 4; i4 += NT) {
        const int h = i4 / (D / 4);
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const float e = wsm[w * 8 + h];
            const float4 x = reinterpret_cast<const float4 *>(co + (size_t)w * R * D)[i4];
            a.x = fmaf(x.x, e, a.x);
            a.y = fmaf(x.y, e, a.y);
            a.z = fmaf(x.z, e, a.z);
            a.w = fmaf(x.w, e, a.w);
        }
        if (n_splits == 1) {
            const float L = sL[h];
            a = L > 0.f ? make_float4(a.x / L, a.y / L, a.z / L, a.w / L) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if (vec) {
            reinterpret_cast<float4 *>(dst)[i4] = a;
        } else {
            dst[4 * i4] = a.x;
            dst[4 * i4 + 1] = a.y;
            dst[4 * i4 + 2] = a.z;
            dst[4 * i4 + 3] = a.w;
        }
    }
    if (p.fused_exchange) {
        // this split's partial is written (the barrier orders the CTA's stores
        // before thread 0's release fence): count its arrival per query head
        __syncthreads();
        if (tid == 0) {
            __threadfence();
#pragma unroll
            for (int h = 0; h < R; ++h) atomicAdd(p.x_arrivals + g * R + h, 1);
        }
    }
}

template <int D, int R, int NW, int TT, int SPW>
__global__ void __launch_bounds__(NW * 32, 1) attn_decode_kernel(const __grid_constant__ DecodeParams p) {
    constexpr int VEC = D / 32;
    constexpr int HALF = D / 2;
    constexpr int NT = NW * 32;
    using SM = DecodeSmem<D, NW, TT, SPW>;
    extern __shared__ __align__(128) float smem[];
    float *stages = smem;
    float *newk = stages + SM::stage_floats;
    float *newv = newk + 4 * D;
    float *pbuf_all = newv + 4 * D;
    float *qsm = pbuf_all + SM::pbuf_floats;   // [R*D q][D: HALF (cos, sin)][D k_new][D v_new]
    uint64_t *full = reinterpret_cast<uint64_t *>(reinterpret_cast<char *>(smem) + SM::bar_off);
    int *pages = reinterpret_cast<int *>(full + NW * SPW);

    int split = blockIdx.x, g = blockIdx.y, qi = blockIdx.z;
    if (p.fused_exchange) {   // one query; CTAs [0, max_splits * G) decode, the last H exchange
        const int nd = p.max_splits * p.kv.G;
        if ((int)blockIdx.x >= nd) {
            fused_exchange_cta<D, R>(p, (int)blockIdx.x - nd);
            return;
        }
        split = (int)blockIdx.x % p.max_splits;
        g = (int)blockIdx.x / p.max_splits;
        qi = 0;
    }
    KTRACE_OPEN(0);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int seq = p.contiguous ? p.seq0 : p.seq[qi];
    const int pos = p.contiguous ? p.pos0 + qi : p.pos[qi];
    const PagedKv &kv = p.kv;
    const int P = kv.P, NS = kv.shard_count, rank = kv.shard_rank;

    // cached positions read here: [0, limit) of those this shard holds
    const int limit = p.append_new ? pos : pos + 1;
    const int count = shard_count_below(limit, P, NS, rank);
    const bool own_new = p.append_new && ((pos / P) % NS == rank);
    const int ST = p.split_tokens;
    int n_splits = (count + ST - 1) / ST;
    if (n_splits == 0) n_splits = 1;
    if (split >= n_splits) return;
    const int u_begin = split * ST;
    const int u_end = min(count, u_begin + ST);
    const int n_tiles = u_end > u_begin ? (u_end - u_begin + TT - 1) / TT : 0;
    const bool do_new = own_new && split == n_splits - 1;
    const int lp_first = u_begin / P;
    const int n_pages_split = n_tiles > 0 ? (u_end - 1) / P - lp_first + 1 : 0;
    const int *pt = kv.page_table + (size_t)seq * kv.pt_stride;

    // Without prefetch_ok nothing is known about the preceding kernel on the
    // stream: it may still be writing the page table (a caller's kernel that
    // let this one start early), so every input is read after the wait.
    if (!p.prefetch_ok) grid_dep_wait();

    // page ids of this split (checked; the host keeps a split within
    // kSplitPagesMax pages), barrier init
    for (int j = tid; j < n_pages_split && j < kSplitPagesMax; j += NT) {
        int ph = pt[lp_first + j];
        if (ph < 0 || ph >= kv.n_pages) {
            raise_error(p.err, DEV_BAD_PAGE);
            ph = 0;
        }
        pages[j] = ph;
    }
    if (lane == 0)
        for (int s = 0; s < SPW; ++s) mbar_init(&full[warp * SPW + s], 1);
    if (tid == 0) mbar_fence_init();
    __syncthreads();

    // this warp's tiles: i = warp, warp + NW, ...; its j-th tile uses stage j % SPW
    const int my_tiles = n_tiles > warp ? (n_tiles - warp + NW - 1) / NW : 0;
    const float *kbase = kv.k + (size_t)g * P * D;
    float *my_stages = stages + (size_t)warp * SPW * 2 * SM::TILE_F;
    uint64_t *my_full = full + warp * SPW;
    const uint64_t pol = l2_evict_first_policy();
    auto issue = [&](int j) {   // lane 0 only
        const int i = warp + j * NW;
        const int u0 = u_begin + i * TT;
        const int nv = min(TT, u_end - u0);
        const int lp = u0 / P;
        const int off = u0 - lp * P;
        const int pj = min(lp - lp_first, kSplitPagesMax - 1);
        const float *src = kbase + ((size_t)pages[pj] * kv.G * P + off) * D;
        const uint32_t bytes = (uint32_t)(nv * D * 4);
        float *dst = my_stages + (size_t)(j % SPW) * 2 * SM::TILE_F;
        uint64_t *bar = my_full + (j % SPW);
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(bar, 2 * bytes);
        bulk_g2s(dst, src, bytes, bar, pol);
        bulk_g2s(dst + SM::TILE_F, src + kv.v_off, bytes, bar, pol);
    };
    // KV of this layer is streamed before waiting for the preceding kernel only
    // when the host knows that no kernel still possibly running writes KV of
    // this layer: a decode kernel lets its successor (a split-merge or
    // exchange kernel, or the next decode) start only after its own wait
    // returned, and a split-merge or exchange kernel lets the next decode start
    // The CTA's inputs from the preceding kernel (q of the group, the new
    // token) and its RoPE row are asked into L2 before the K/V copies below,
    // so that the loads after the wait find them there instead of queueing
    // behind the streamed K/V. L2 is where every SM's accesses meet, so a line
    // fetched early still holds the preceding kernel's stores when it is read.
    if (p.prefetch_ok && p.l2_inputs && tid == 0) {
        bulk_prefetch_l2(p.q + (size_t)qi * p.H * D + (size_t)g * R * D, (uint32_t)(R * D * 4));
        bulk_prefetch_l2(p.rope + (size_t)pos * HALF, (uint32_t)(HALF * 8));
        if (do_new) {
            bulk_prefetch_l2(p.k_new + (size_t)qi * kv.G * D + (size_t)g * D, (uint32_t)(D * 4));
            bulk_prefetch_l2(p.v_new + (size_t)qi * kv.G * D + (size_t)g * D, (uint32_t)(D * 4));
        }
    }
    // at once, so at most the previous decode and its merge can still run
    const int pre = p.prefetch_ok ? min(SPW, p.prefetch_stages) : 0;
    if (lane == 0)
        for (int j = 0; j < pre && j < my_tiles; ++j) issue(j);
    // and the positions after those first ring stages, up to the host's L2
    // budget, are asked into L2: HBM keeps streaming this layer's K/V while
    // the preceding kernels (the last layer's merge or exchange) finish
    if (p.prefetch_ok && tid == NT - 1 && p.l2_prefetch_tokens > 0) {
        const int a = min(u_end, u_begin + SPW * NW * TT);
        const int b = min(u_end, u_begin + p.l2_prefetch_tokens);
        for (int u = a; u < b;) {
            const int lp = u / P, off = u - lp * P;
            const int n = min(b - u, P - off);   // within one page
            const int pj = min(lp - lp_first, kSplitPagesMax - 1);
            const char *src = reinterpret_cast<const char *>(kbase + ((size_t)pages[pj] * kv.G * P + off) * D);
            const uint32_t bytes = (uint32_t)n * D * 4;
            for (uint32_t o = 0; o < bytes; o += 65536u) {
                const uint32_t c = min(65536u, bytes - o);
                bulk_prefetch_l2(src + o, c);
                bulk_prefetch_l2(src + (size_t)kv.v_off * 4 + o, c);
            }
            u += n;
        }
    }
    if (p.prefetch_ok) grid_dep_wait();
    KTRACE(1);
    grid_dep_launch();
    if (lane == 0)
        for (int j = pre; j < SPW && j < my_tiles; ++j) issue(j);

    // q of the group, the RoPE row and the new token's k/v: loaded once per
    // CTA with 16-byte loads (every warp of every split reads the same few
    // lines, so per-warp loads would pile onto a handful of L2 lines)
    {
        const float4 *q4 = reinterpret_cast<const float4 *>(p.q + (size_t)qi * p.H * D + (size_t)g * R * D);
        float4 *d4 = reinterpret_cast<float4 *>(qsm);
        for (int i = tid; i < R * D / 4; i += NT) d4[i] = __ldg(q4 + i);
        const float4 *c4 = reinterpret_cast<const float4 *>(p.rope + (size_t)pos * HALF);
        for (int i = tid; i < D / 4; i += NT) d4[R * D / 4 + i] = __ldg(c4 + i);
        if (do_new) {
            const float4 *k4 = reinterpret_cast<const float4 *>(p.k_new + (size_t)qi * kv.G * D + (size_t)g * D);
            const float4 *v4 = reinterpret_cast<const float4 *>(p.v_new + (size_t)qi * kv.G * D + (size_t)g * D);
            for (int i = tid; i < D / 4; i += NT) {
                d4[(R + 1) * D / 4 + i] = __ldg(k4 + i);
                d4[(R + 2) * D / 4 + i] = __ldg(v4 + i);
            }
        }
    }
    __syncthreads();
    KTRACE(2);
    const float2 *cs = reinterpret_cast<const float2 *>(qsm + R * D);

    WarpState<D, R> st;
#pragma unroll
    for (int h = 0; h < R; ++h)
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
            const int i = lane * VEC + j;
            const float x = qsm[h * D + i];
            const float y = qsm[h * D + (i ^ HALF)];
            const float2 a = cs[i & (HALF - 1)];
            const float r = i < HALF ? rope_lo(x, y, a.x, a.y) : rope_hi(y, x, a.x, a.y);
            st.q[h][j] = r * p.scale_log2;
            st.o[h][j] = 0.f;
        }
#pragma unroll
    for (int h = 0; h < R; ++h) st.m[h] = -INFINITY;
    st.mo = -INFINITY;
    st.l = 0.f;
    float *pbuf = pbuf_all + (size_t)warp * TT * 8;

    if (do_new && warp == 0) {
        // the token at pos: rotate k, stage k/v as a 1-token tile, append to the cache
        const float *ks = qsm + (R + 1) * D;
        const float *vs = qsm + (R + 2) * D;
        const int lp = (pos / P) / NS, off = pos % P;
        const int ph = pt[lp];
        const bool ok = ph >= 0 && ph < kv.n_pages;
        if (!ok && lane == 0) raise_error(p.err, DEV_BAD_PAGE);
        float *kd = kv.k + (((size_t)(ok ? ph : 0) * kv.G + g) * P + off) * D;
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
            const int i = lane * VEC + j;
            const float x = ks[i], y = ks[i ^ HALF];
            const float2 a = cs[i & (HALF - 1)];
            const float kr = i < HALF ? rope_lo(x, y, a.x, a.y) : rope_hi(y, x, a.x, a.y);
            const float vr = vs[i];
            newk[i] = kr;
            newv[i] = vr;
            if (ok) {
                kd[i] = kr;
                kd[i + kv.v_off] = vr;
            }
        }
        __syncwarp();
        process_tile<D, R, 4>(st, newk, newv, 1, pbuf, lane);
    }

    for (int j = 0; j < my_tiles; ++j) {
        const int s = j % SPW;
        if (!__all_sync(FULL, mbar_wait(my_full + s, (j / SPW) & 1, p.err, DEV_WAIT_FULL_TIMEOUT, p.wait_ns))) {
            // gave up (the error word says so): tiles j .. j+SPW-1 may still be
            // landing in this warp's stages; wait for them before the stage
            // memory is reused below or the block exits
            for (int t = j; t < my_tiles && t < j + SPW; ++t) mbar_drain(my_full + t % SPW, (t / SPW) & 1);
            break;
        }
        const int nv = min(TT, u_end - (u_begin + (warp + j * NW) * TT));
        const float *tile = my_stages + (size_t)s * 2 * SM::TILE_F;
        process_tile<D, R, TT>(st, tile, tile + SM::TILE_F, nv, pbuf, lane);
        if (lane == 0 && j + SPW < my_tiles) issue(j + SPW);
    }

    // lane-partial sums -> per head (lanes with equal lane & 7); lane h < 8 then holds head h
    st.l += __shfl_xor_sync(FULL, st.l, 8);
    st.l += __shfl_xor_sync(FULL, st.l, 16);
    __syncthreads();   // every tile consumed: the stage memory is free
    KTRACE(3);
    {
        float *cm = stages;              // [NW][8]
        float *cl = cm + NW * 8;         // [NW][8]
        float *co = cl + NW * 8;         // [NW][R][D]
        if (lane < R) cl[warp * 8 + lane] = st.l;
        if (lane == 0)
#pragma unroll
            for (int h = 0; h < R; ++h) cm[warp * 8 + h] = st.m[h];
#pragma unroll
        for (int h = 0; h < R; ++h)
#pragma unroll
            for (int j = 0; j < VEC; ++j) co[(warp * R + h) * D + lane * VEC + j] = st.o[h][j];
    }
    __syncthreads();

    // ---------------------------------------------------------------- CTA merge
    cta_merge_write<D, R, NW>(p, stages, pbuf_all, qi, g, split, n_splits);
#ifdef KORE_TRACE
    __syncthreads();
    KTRACE(4);
#endif
}

// ---------------------------------------------------------------- tensor-core decode
//
// attn_decode_tc_kernel: the same split-KV decode for one query at D = 128,
// with the two contractions of a tile on the tensor cores (mma.sync
// m16n8k16, bf16 operands, fp32 accumulation). The CUDA-core kernel above
// spends most of its issue slots on the 7-head group's FMAs and the shuffle
// reductions of the scores (measured: at the same KV bytes a layer takes
// 28.2 us with 7 query heads per KV head and 23.8 us with 1); here a 16-token
// tile costs 48 MMAs, the operand splits and the fragment loads.
//  * Precision: every fp32 operand x is split into bf16 hi = rn(x) and
//    lo = rn(x - hi) (x = hi + lo to 2^-16 relative) and each product is
//    hi*hi + lo*hi + hi*lo, accumulated in fp32: the error of a product is
//    ~2^-16 relative, far inside the 1e-3 bound (as in the prefill).
//  * Layout: a warp's stage holds a 16-token tile of K and of V, each loaded
//    by four 2-D TMA boxes of 32 floats x 16 rows with the 128-byte swizzle:
//    [column group q][token r][32 floats], the 16-byte chunk j of row r
//    stored at chunk j ^ (r % 8). Every fragment load below then touches 32
//    distinct banks.
//  * Scores: S^T (16 tokens x 8 heads) = K (16 x 128) . Q^T, tokens on M and
//    the group's heads on N (R <= 8 of 8 columns used); k-step s = 2q + e
//    gives thread (g, c) the 4 dims of chunk 8q + 2c + e of its rows g, g+8
//    (the k index of the fragment permuted onto those dims, the same
//    permutation for Q), so one 16-byte load feeds one A register pair.
//  * Output: O^T (128 dims x 8 heads) += V^T (128 x 16 tokens) . P^T; the
//    probabilities move from the score fragment (tokens on rows) to the B
//    fragment (tokens on k) with eight shuffles.
//  * Softmax as in the CUDA-core kernel: online, the reference maximum moved
//    lazily (when a score exceeds it by 2^8); the new token at pos is taken
//    in fp32 by warp 0 before the tiles.

constexpr int kTcTT = 16;   // tokens per tile

// 2-D TMA load of one box into this CTA's shared memory (no multicast).
__device__ __forceinline__ void tma_load_2d(void *dst, const TmaDesc *map, int x, int y, uint64_t *bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// x0, x1 -> bf16x2 hi = (rn(x0), rn(x1)) and lo = (rn(x0 - hi0), rn(x1 - hi1)),
// element 0 in the low half (the lower k index of a fragment pair).
__device__ __forceinline__ void split_bf16x2(float x0, float x1, uint32_t &hi, uint32_t &lo) {
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(x1), "f"(x0));
    const float h0 = __uint_as_float(hi << 16), h1 = __uint_as_float(hi & 0xffff0000u);
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(__fsub_rn(x1, h1)), "f"(__fsub_rn(x0, h0)));
}

// d += a . b, m16n8k16, bf16 inputs, fp32 accumulators.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int R, int NW, int SPW>
struct TcSmem {
    static constexpr int D = 128;
    static constexpr size_t tile_bytes = (size_t)kTcTT * D * 4;   // 8 KB: K or V of a tile
    static constexpr size_t stage_bytes = 2 * tile_bytes;
    static constexpr size_t stages_bytes = (size_t)NW * SPW * stage_bytes;
    static constexpr size_t qsm_off = stages_bytes;               // q [R*D], RoPE row [D], k_new, v_new, k rotated
    static constexpr size_t bar_off = qsm_off + (size_t)12 * D * 4;
    static constexpr size_t pages_off = bar_off + (size_t)NW * SPW * 8;
    static constexpr size_t bytes = pages_off + (size_t)kSplitPagesMax * 4 + 1024;   // + alignment of the stages
    static_assert(stages_bytes >= (size_t)NW * 8 * 32 * 16 + (size_t)NW * 16 * 4, "CTA merge scratch");
};

template <int R, int NW, int SPW>
__global__ void __launch_bounds__(NW * 32, 1) attn_decode_tc_kernel(const __grid_constant__ DecodeParams p) {
    constexpr int D = 128, HALF = 64, TT = kTcTT, NT = NW * 32;
    using SM = TcSmem<R, NW, SPW>;
    extern __shared__ __align__(128) unsigned char tc_smem[];
    // the stages start on a 1024-byte boundary: the 128-byte swizzle pattern
    // repeats every 1024 bytes of shared memory address
    unsigned char *base = tc_smem + ((1024u - (smem_u32(tc_smem) & 1023u)) & 1023u);
    float *qsm = reinterpret_cast<float *>(base + SM::qsm_off);   // q [R*D], RoPE row [D], k_new [D], v_new [D]
    uint64_t *full = reinterpret_cast<uint64_t *>(base + SM::bar_off);
    int *pages = reinterpret_cast<int *>(base + SM::pages_off);

    int split = blockIdx.x, g = blockIdx.y;
    if (p.fused_exchange) {   // CTAs [0, max_splits * G) decode, the last H merge (and exchange)
        const int nd = p.max_splits * p.kv.G;
        if ((int)blockIdx.x >= nd) {
            fused_exchange_cta<D, R>(p, (int)blockIdx.x - nd);
            return;
        }
        split = (int)blockIdx.x % p.max_splits;
        g = (int)blockIdx.x / p.max_splits;
    }
    KTRACE_OPEN(0);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gq = lane >> 2, cq = lane & 3;   // fragment row group, thread in group
    const int seq = p.seq0, pos = p.pos0;
    const PagedKv &kv = p.kv;
    const int P = kv.P, NS = kv.shard_count, rank = kv.shard_rank;

    const int limit = p.append_new ? pos : pos + 1;
    const int count = shard_count_below(limit, P, NS, rank);
    const bool own_new = p.append_new && ((pos / P) % NS == rank);
    const int ST = p.split_tokens;
    int n_splits = (count + ST - 1) / ST;
    if (n_splits == 0) n_splits = 1;
    if (split >= n_splits) return;
    const int u_begin = split * ST;
    const int u_end = min(count, u_begin + ST);
    const int n_tiles = u_end > u_begin ? (u_end - u_begin + TT - 1) / TT : 0;
    const bool do_new = own_new && split == n_splits - 1;
    const int lp_first = u_begin / P;
    const int n_pages_split = n_tiles > 0 ? (u_end - 1) / P - lp_first + 1 : 0;
    const int *pt = kv.page_table + (size_t)seq * kv.pt_stride;

    if (!p.prefetch_ok) grid_dep_wait();
    for (int j = tid; j < n_pages_split && j < kSplitPagesMax; j += NT) {
        int ph = pt[lp_first + j];
        if (ph < 0 || ph >= kv.n_pages) {
            raise_error(p.err, DEV_BAD_PAGE);
            ph = 0;
        }
        pages[j] = ph;
    }
    if (lane == 0)
        for (int s = 0; s < SPW; ++s) mbar_init(&full[warp * SPW + s], 1);
    if (tid == 0) mbar_fence_init();
    __syncthreads();

    // this warp's tiles: i = warp, warp + NW, ...; its j-th tile uses stage j % SPW
    const int my_tiles = n_tiles > warp ? (n_tiles - warp + NW - 1) / NW : 0;
    unsigned char *my_stages = base + (size_t)warp * SPW * SM::stage_bytes;
    uint64_t *my_full = full + warp * SPW;
    const uint64_t pol = l2_evict_first_policy();
    auto issue = [&](int j) {   // lane 0 only: K and V of tile j, four boxes each
        const int i = warp + j * NW;
        const int u0 = u_begin + i * TT;
        const int lp = u0 / P;
        const int off = u0 - lp * P;
        const int pj = min(lp - lp_first, kSplitPagesMax - 1);
        const long long row = ((long long)pages[pj] * kv.G + g) * P + off;
        unsigned char *dst = my_stages + (size_t)(j % SPW) * SM::stage_bytes;
        uint64_t *bar = my_full + (j % SPW);
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(bar, (uint32_t)SM::stage_bytes);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            tma_load_2d(dst + q * 2048, &p.tm_k, 32 * q, (int)(p.k_row0 + row), bar, pol);
            tma_load_2d(dst + SM::tile_bytes + q * 2048, &p.tm_v, 32 * q, (int)(p.v_row0 + row), bar, pol);
        }
    };
    if (p.prefetch_ok && p.l2_inputs && tid == 0) {   // as in attn_decode_kernel
        bulk_prefetch_l2(p.q + (size_t)g * R * D, (uint32_t)(R * D * 4));
        bulk_prefetch_l2(p.rope + (size_t)pos * HALF, (uint32_t)(HALF * 8));
        if (do_new) {
            bulk_prefetch_l2(p.k_new + (size_t)g * D, (uint32_t)(D * 4));
            bulk_prefetch_l2(p.v_new + (size_t)g * D, (uint32_t)(D * 4));
        }
    }
    const int pre = p.prefetch_ok ? min(SPW, p.prefetch_stages) : 0;
    if (lane == 0)
        for (int j = 0; j < pre && j < my_tiles; ++j) issue(j);
    if (p.prefetch_ok) grid_dep_wait();
    KTRACE(1);
    grid_dep_launch();
    if (lane == 0)
        for (int j = pre; j < SPW && j < my_tiles; ++j) issue(j);

    // q of the group, the RoPE row and the new token's k/v, once per CTA
    {
        const float4 *q4 = reinterpret_cast<const float4 *>(p.q + (size_t)g * R * D);
        float4 *d4 = reinterpret_cast<float4 *>(qsm);
        for (int i = tid; i < R * D / 4; i += NT) d4[i] = __ldg(q4 + i);
        const float4 *c4 = reinterpret_cast<const float4 *>(p.rope + (size_t)pos * HALF);
        for (int i = tid; i < D / 4; i += NT) d4[R * D / 4 + i] = __ldg(c4 + i);
        if (do_new) {
            const float4 *k4 = reinterpret_cast<const float4 *>(p.k_new + (size_t)g * D);
            const float4 *v4 = reinterpret_cast<const float4 *>(p.v_new + (size_t)g * D);
            for (int i = tid; i < D / 4; i += NT) {
                d4[(R + 1) * D / 4 + i] = __ldg(k4 + i);
                d4[(R + 2) * D / 4 + i] = __ldg(v4 + i);
            }
        }
    }
    __syncthreads();
    KTRACE(2);
    const float2 *cs = reinterpret_cast<const float2 *>(qsm + R * D);
    auto qrot = [&](int h, int d) -> float {   // q of head h, dim d: rotated at pos, scaled to log2 units
        const float x = qsm[h * D + d], y = qsm[h * D + (d ^ HALF)];
        const float2 a = cs[d & (HALF - 1)];
        const float r = d < HALF ? rope_lo(x, y, a.x, a.y) : rope_hi(y, x, a.x, a.y);
        return r * p.scale_log2;
    };

    // B fragments of Q^T for the 8 k-steps (k-step s = 2q + e: this thread's
    // dims 32q + 8c + 4e .. +3, in the order of its K loads); heads >= R zero
    uint32_t qb_hi[8][2], qb_lo[8][2];
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        const int d0 = 32 * (s >> 1) + 8 * cq + 4 * (s & 1);
        float x[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) x[i] = gq < R ? qrot(gq, d0 + i) : 0.f;
        split_bf16x2(x[0], x[1], qb_hi[s][0], qb_lo[s][0]);
        split_bf16x2(x[2], x[3], qb_hi[s][1], qb_lo[s][1]);
    }

    // O^T fragments: m-tile mt holds dims 16mt + gq (+8) of heads 2cq, 2cq+1:
    // o[mt][0] (dim 16mt+gq, head 2cq), [1] (.., 2cq+1), [2] (dim +8, 2cq), [3] (dim +8, 2cq+1)
    float o[8][4];
#pragma unroll
    for (int mt = 0; mt < 8; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) o[mt][i] = 0.f;
    const bool hv0 = 2 * cq < R, hv1 = 2 * cq + 1 < R;   // this thread's two head columns exist
    // reference maxima (a column without a head: +inf, so its p is 0 and it never rescales)
    float mr0 = hv0 ? -INFINITY : INFINITY, mr1 = hv1 ? -INFINITY : INFINITY;
    float l0 = 0.f, l1 = 0.f;   // thread-partial sums of heads 2cq, 2cq+1

    if (do_new && warp == 0) {
        // the token at pos in fp32: rotate k, append k/v to the cache, fold it in
        const float *ks = qsm + (R + 1) * D;
        const float *vs = qsm + (R + 2) * D;
        const int lp = (pos / P) / NS, off = pos % P;
        const int ph = pt[lp];
        const bool ok = ph >= 0 && ph < kv.n_pages;
        if (!ok && lane == 0) raise_error(p.err, DEV_BAD_PAGE);
        float *kd = kv.k + (((size_t)(ok ? ph : 0) * kv.G + g) * P + off) * D;
        float part[R];
#pragma unroll
        for (int h = 0; h < R; ++h) part[h] = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = lane * 4 + j;
            const float x = ks[i], y = ks[i ^ HALF];
            const float2 a = cs[i & (HALF - 1)];
            const float kr = i < HALF ? rope_lo(x, y, a.x, a.y) : rope_hi(y, x, a.x, a.y);
            if (ok) {
                kd[i] = kr;
                kd[i + kv.v_off] = vs[i];
            }
#pragma unroll
            for (int h = 0; h < R; ++h) part[h] = fmaf(qrot(h, i), kr, part[h]);
        }
#pragma unroll
        for (int h = 0; h < R; ++h)
#pragma unroll
            for (int m = 16; m > 0; m >>= 1) part[h] += __shfl_xor_sync(FULL, part[h], m);
        float sn0 = 0.f, sn1 = 0.f;
#pragma unroll
        for (int h = 0; h < R; ++h) {
            if (h == 2 * cq) sn0 = part[h];
            if (h == 2 * cq + 1) sn1 = part[h];
        }
        if (hv0) {
            mr0 = sn0;   // the first score of this warp: exact reference
            if (gq == 0) l0 = 1.f;
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
                o[mt][0] = vs[16 * mt + gq];
                o[mt][2] = vs[16 * mt + gq + 8];
            }
        }
        if (hv1) {
            mr1 = sn1;
            if (gq == 0) l1 = 1.f;
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
                o[mt][1] = vs[16 * mt + gq];
                o[mt][3] = vs[16 * mt + gq + 8];
            }
        }
    }

    // per-thread byte offsets of the fragment loads within a tile (see the layout above)
    //  K, k-step (q, e): row gq at q*2048 + gq*128 + (((2c ^ gq) ^ e) << 4); row gq+8 at +1024
    const uint32_t kofs0 = gq * 128 + ((((2 * cq) ^ gq)) << 4);
    const uint32_t kofs1 = kofs0 ^ 16u;
    //  V, element (token t = 2c + i (+8), dim 16mt + gq (+8)): (mt >> 1)*2048 + t*128 +
    //  ((chunk(dim) ^ (t & 7)) << 4) + (gq & 3)*4, chunk(dim) = 4(mt & 1) | 2(+8) | (gq >> 2)
    uint32_t vofs[2];
#pragma unroll
    for (int i = 0; i < 2; ++i)
        vofs[i] = (uint32_t)((2 * cq + i) * 128 + ((((gq >> 2) ^ (2 * cq + i)) & 7) << 4) + (gq & 3) * 4);

    for (int j = 0; j < my_tiles; ++j) {
        const int s = j % SPW;
        if (!__all_sync(FULL, mbar_wait(my_full + s, (j / SPW) & 1, p.err, DEV_WAIT_FULL_TIMEOUT, p.wait_ns))) {
            // gave up (the error word says so): let the copies in flight land first
            for (int t = j; t < my_tiles && t < j + SPW; ++t) mbar_drain(my_full + t % SPW, (t / SPW) & 1);
            break;
        }
        const int nv = min(TT, u_end - (u_begin + (warp + j * NW) * TT));
        const unsigned char *Kt = my_stages + (size_t)s * SM::stage_bytes;
        const unsigned char *Vt = Kt + SM::tile_bytes;

        // S^T (16 tokens x 8 heads) = K . Q^T; the hi.hi and the two cross
        // products in separate accumulators (independent MMA chains)
        float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f}, sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int st = 0; st < 8; ++st) {
            const uint32_t ko = ((st & 1) ? kofs1 : kofs0) + (uint32_t)(st >> 1) * 2048u;
            const float4 r0 = *reinterpret_cast<const float4 *>(Kt + ko);          // token gq
            const float4 r1 = *reinterpret_cast<const float4 *>(Kt + ko + 1024);   // token gq + 8
            uint32_t ah[4], al[4];
            split_bf16x2(r0.x, r0.y, ah[0], al[0]);
            split_bf16x2(r1.x, r1.y, ah[1], al[1]);
            split_bf16x2(r0.z, r0.w, ah[2], al[2]);
            split_bf16x2(r1.z, r1.w, ah[3], al[3]);
            mma_16816(sa, ah[0], ah[1], ah[2], ah[3], qb_hi[st][0], qb_hi[st][1]);
            mma_16816(sb, al[0], al[1], al[2], al[3], qb_hi[st][0], qb_hi[st][1]);
            mma_16816(sc, ah[0], ah[1], ah[2], ah[3], qb_lo[st][0], qb_lo[st][1]);
        }
        // sv: (token gq, head 2c), (gq, 2c+1), (gq+8, 2c), (gq+8, 2c+1)
        float sv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) sv[i] = sa[i] + (sb[i] + sc[i]);
        if (nv < TT) {
            if (gq >= nv) sv[0] = sv[1] = -INFINITY;
            if (gq + 8 >= nv) sv[2] = sv[3] = -INFINITY;
        }

        // lazy rescale: only when a score exceeds its head's reference by 2^8
        const bool need = sv[0] > mr0 + kRescaleLog2 || sv[2] > mr0 + kRescaleLog2 || sv[1] > mr1 + kRescaleLog2 ||
                          sv[3] > mr1 + kRescaleLog2;
        if (__any_sync(FULL, need)) {
            float t0 = fmaxf(sv[0], sv[2]), t1 = fmaxf(sv[1], sv[3]);
#pragma unroll
            for (int m = 4; m < 32; m <<= 1) {
                t0 = fmaxf(t0, __shfl_xor_sync(FULL, t0, m));
                t1 = fmaxf(t1, __shfl_xor_sync(FULL, t1, m));
            }
            if (hv0) {
                const float mn = fmaxf(mr0, t0);
                const float al = fast_exp2(mr0 - mn);
                l0 *= al;
#pragma unroll
                for (int mt = 0; mt < 8; ++mt) {
                    o[mt][0] *= al;
                    o[mt][2] *= al;
                }
                mr0 = mn;
            }
            if (hv1) {
                const float mn = fmaxf(mr1, t1);
                const float al = fast_exp2(mr1 - mn);
                l1 *= al;
#pragma unroll
                for (int mt = 0; mt < 8; ++mt) {
                    o[mt][1] *= al;
                    o[mt][3] *= al;
                }
                mr1 = mn;
            }
        }
        float pv[4];
        pv[0] = fast_exp2(sv[0] - mr0);
        pv[1] = fast_exp2(sv[1] - mr1);
        pv[2] = fast_exp2(sv[2] - mr0);
        pv[3] = fast_exp2(sv[3] - mr1);
        l0 += pv[0] + pv[2];
        l1 += pv[1] + pv[3];

        // P^T as a B fragment: this thread needs P[head gq][tokens 2c, 2c+1,
        // 2c+8, 2c+9]; P[h][t] sits in lane (t & 7)*4 + (h >> 1), value
        // (t >> 3)*2 + (h & 1) of the score fragment
        const int srcA = 8 * cq + (gq >> 1), srcB = srcA + 4;
        const bool odd = gq & 1;
        const float xa0 = __shfl_sync(FULL, pv[0], srcA), xa1 = __shfl_sync(FULL, pv[1], srcA);
        const float xb0 = __shfl_sync(FULL, pv[0], srcB), xb1 = __shfl_sync(FULL, pv[1], srcB);
        const float xa2 = __shfl_sync(FULL, pv[2], srcA), xa3 = __shfl_sync(FULL, pv[3], srcA);
        const float xb2 = __shfl_sync(FULL, pv[2], srcB), xb3 = __shfl_sync(FULL, pv[3], srcB);
        uint32_t pbh[2], pbl[2];
        split_bf16x2(odd ? xa1 : xa0, odd ? xb1 : xb0, pbh[0], pbl[0]);
        split_bf16x2(odd ? xa3 : xa2, odd ? xb3 : xb2, pbh[1], pbl[1]);

        // O^T (128 dims x 8 heads) += V^T . P^T, one m-tile of 16 dims at a time
        const bool t0ok = 2 * cq < nv, t1ok = 2 * cq + 1 < nv, t8ok = 2 * cq + 8 < nv, t9ok = 2 * cq + 9 < nv;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
            const uint32_t mb = (uint32_t)(mt >> 1) * 2048u;
            const uint32_t x0 = (uint32_t)(4 * (mt & 1)) << 4, x8 = (uint32_t)(4 * (mt & 1) + 2) << 4;
            // (token, dim): a0 (2c, d) (2c+1, d), a1 (2c, d+8) (2c+1, d+8), a2 (2c+8, d) (2c+9, d), a3 (2c+8, d+8) (2c+9, d+8)
            float v00 = *reinterpret_cast<const float *>(Vt + mb + (vofs[0] ^ x0));
            float v01 = *reinterpret_cast<const float *>(Vt + mb + (vofs[1] ^ x0));
            float v10 = *reinterpret_cast<const float *>(Vt + mb + (vofs[0] ^ x8));
            float v11 = *reinterpret_cast<const float *>(Vt + mb + (vofs[1] ^ x8));
            float v20 = *reinterpret_cast<const float *>(Vt + mb + 1024 + (vofs[0] ^ x0));
            float v21 = *reinterpret_cast<const float *>(Vt + mb + 1024 + (vofs[1] ^ x0));
            float v30 = *reinterpret_cast<const float *>(Vt + mb + 1024 + (vofs[0] ^ x8));
            float v31 = *reinterpret_cast<const float *>(Vt + mb + 1024 + (vofs[1] ^ x8));
            if (nv < TT) {   // rows past the split's end hold other positions: never multiplied in
                v00 = t0ok ? v00 : 0.f;
                v10 = t0ok ? v10 : 0.f;
                v01 = t1ok ? v01 : 0.f;
                v11 = t1ok ? v11 : 0.f;
                v20 = t8ok ? v20 : 0.f;
                v30 = t8ok ? v30 : 0.f;
                v21 = t9ok ? v21 : 0.f;
                v31 = t9ok ? v31 : 0.f;
            }
            uint32_t vh[4], vl[4];
            split_bf16x2(v00, v01, vh[0], vl[0]);
            split_bf16x2(v10, v11, vh[1], vl[1]);
            split_bf16x2(v20, v21, vh[2], vl[2]);
            split_bf16x2(v30, v31, vh[3], vl[3]);
            mma_16816(o[mt], vh[0], vh[1], vh[2], vh[3], pbh[0], pbh[1]);
            mma_16816(o[mt], vl[0], vl[1], vl[2], vl[3], pbh[0], pbh[1]);
            mma_16816(o[mt], vh[0], vh[1], vh[2], vh[3], pbl[0], pbl[1]);
        }
        __syncwarp();   // every lane is done with the stage
        if (lane == 0 && j + SPW < my_tiles) issue(j + SPW);
    }

    // sums of heads 2c, 2c+1 over the warp's tokens (lanes of equal c)
#pragma unroll
    for (int m = 4; m < 32; m <<= 1) {
        l0 += __shfl_xor_sync(FULL, l0, m);
        l1 += __shfl_xor_sync(FULL, l1, m);
    }
    __syncthreads();   // every tile consumed: the stage memory is free
    KTRACE(3);

    // CTA merge, position-wise: thread (gq, c) of every warp holds the same
    // (dim, head) positions, so warp w finalises m-tiles w, w + NW, ... from
    // the NW warps' fragments, weighted by 2^(m_w - M) per head.
    float4 *xo = reinterpret_cast<float4 *>(base);                    // [NW][8 m-tiles][32 lanes]
    float *xm = reinterpret_cast<float *>(base + (size_t)NW * 8 * 32 * 16);   // [NW][8]
    float *xl = xm + NW * 8;                                          // [NW][8]
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) xo[(warp * 8 + mt) * 32 + lane] = make_float4(o[mt][0], o[mt][1], o[mt][2], o[mt][3]);
    if (gq == 0) {
        xm[warp * 8 + 2 * cq] = hv0 ? mr0 : -INFINITY;
        xm[warp * 8 + 2 * cq + 1] = hv1 ? mr1 : -INFINITY;
        xl[warp * 8 + 2 * cq] = l0;
        xl[warp * 8 + 2 * cq + 1] = l1;
    }
    __syncthreads();
    float M0 = -INFINITY, M1 = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
        M0 = fmaxf(M0, xm[w * 8 + 2 * cq]);
        M1 = fmaxf(M1, xm[w * 8 + 2 * cq + 1]);
    }
    float e0[NW], e1[NW], L0 = 0.f, L1 = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
        e0[w] = M0 == -INFINITY ? 0.f : fast_exp2(xm[w * 8 + 2 * cq] - M0);
        e1[w] = M1 == -INFINITY ? 0.f : fast_exp2(xm[w * 8 + 2 * cq + 1] - M1);
        L0 = fmaf(xl[w * 8 + 2 * cq], e0[w], L0);
        L1 = fmaf(xl[w * 8 + 2 * cq + 1], e1[w], L1);
    }
    const size_t qh0 = (size_t)g * R;   // first query head of the group
    const size_t part_base = (size_t)g * p.max_splits;
    for (int mt = warp; mt < 8; mt += NW) {
        float a[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const float4 x = xo[(w * 8 + mt) * 32 + lane];
            a[0] = fmaf(x.x, e0[w], a[0]);
            a[1] = fmaf(x.y, e1[w], a[1]);
            a[2] = fmaf(x.z, e0[w], a[2]);
            a[3] = fmaf(x.w, e1[w], a[3]);
        }
        const int d0 = 16 * mt + gq;
        if (n_splits == 1) {
            if (hv0) {
                p.out[(qh0 + 2 * cq) * D + d0] = L0 > 0.f ? a[0] / L0 : 0.f;
                p.out[(qh0 + 2 * cq) * D + d0 + 8] = L0 > 0.f ? a[2] / L0 : 0.f;
            }
            if (hv1) {
                p.out[(qh0 + 2 * cq + 1) * D + d0] = L1 > 0.f ? a[1] / L1 : 0.f;
                p.out[(qh0 + 2 * cq + 1) * D + d0 + 8] = L1 > 0.f ? a[3] / L1 : 0.f;
            }
        } else {
            float *po = p.part_o + (part_base + split) * R * D;
            if (hv0) {
                po[(2 * cq) * D + d0] = a[0];
                po[(2 * cq) * D + d0 + 8] = a[2];
            }
            if (hv1) {
                po[(2 * cq + 1) * D + d0] = a[1];
                po[(2 * cq + 1) * D + d0 + 8] = a[3];
            }
        }
    }
    if (warp == 0 && gq == 0) {
        if (n_splits == 1) {
            if (p.lse && hv0) p.lse[qh0 + 2 * cq] = L0 > 0.f ? M0 + __log2f(L0) : -INFINITY;
            if (p.lse && hv1) p.lse[qh0 + 2 * cq + 1] = L1 > 0.f ? M1 + __log2f(L1) : -INFINITY;
        } else {
            if (hv0) p.part_ml[(part_base + split) * R + 2 * cq] = make_float2(M0, L0);
            if (hv1) p.part_ml[(part_base + split) * R + 2 * cq + 1] = make_float2(M1, L1);
        }
    }
    if (p.fused_exchange) {
        // this split's partial is written (the barrier orders the CTA's stores
        // before thread 0's release fence): count its arrival per query head
        __syncthreads();
        if (tid == 0) {
            __threadfence();
#pragma unroll
            for (int h = 0; h < R; ++h) atomicAdd(p.x_arrivals + g * R + h, 1);
        }
    }
#ifdef KORE_TRACE
    __syncthreads();
    KTRACE(4);
#endif
}

// Merges the per-split partials of one query head (one CTA, one thread per
// dim): out = sum_s 2^(m_s - M) o_s / sum_s 2^(m_s - M) l_s. Launched right
// after the decode kernel with a programmatic dependency; waits for it first.
template <int D, int R>
__global__ void __launch_bounds__(D) split_merge_kernel(const __grid_constant__ DecodeParams p) {
    // the next decode may start as soon as this kernel is resident: it only
    // prefetches KV of a layer that neither this kernel nor the decode before
    // it writes (checked on the host), and waits for this kernel before
    // anything else
    KTRACE_OPEN(1);
    grid_dep_launch();
    grid_dep_wait();
    KTRACE(1);
    const int h = blockIdx.x % R, g = blockIdx.x / R, qi = blockIdx.y, tid = threadIdx.x;
    const int pos = p.contiguous ? p.pos0 + qi : p.pos[qi];
    const PagedKv &kv = p.kv;
    const int P = kv.P, NS = kv.shard_count, rank = kv.shard_rank;
    const int count = shard_count_below(p.append_new ? pos : pos + 1, P, NS, rank);
    const int n_splits = (count + p.split_tokens - 1) / p.split_tokens;
    if (n_splits <= 1) return;   // the decode kernel wrote this output directly
    const size_t base = ((size_t)qi * kv.G + g) * p.max_splits;
    float o, lse;
    merge_head_splits<D>(p.part_o + base * R * D + (size_t)h * D + tid, (size_t)R * D, p.part_ml + base * R + h,
                         (size_t)R, n_splits, o, lse);
    const size_t qh = (size_t)qi * p.H + (size_t)g * R + h;
    p.out[qh * D + tid] = o;
    if (p.lse && tid == 0) p.lse[qh] = lse;
    KTRACE(4);
}

#ifndef KORE_DECODE_NW
#define KORE_DECODE_NW 8
#endif
#ifndef KORE_DECODE_TT
#define KORE_DECODE_TT 8
#endif
#ifndef KORE_DECODE_SPW
#define KORE_DECODE_SPW 3
#endif
// Decode pipeline shape: NW warps per CTA, TT-token tiles, SPW stages per warp.
constexpr int kNW = KORE_DECODE_NW, kTT = KORE_DECODE_TT, kSPW = KORE_DECODE_SPW;
static_assert(kTT % 4 == 0, "tiles are processed in 4-token rounds");
static_assert(64 % kTT == 0, "a tile must not cross a page (pages are multiples of 64 positions)");
static_assert(DecodeSmem<128, kNW, kTT, kSPW>::bytes <= 227 * 1024, "decode stages exceed shared memory");
static_assert(DecodeSmem<64, kNW, kTT, kSPW>::stage_floats >= (size_t)kMaxSplits * 8 + 16 + 8 * 64 + 64,
              "split merge needs room for the weights and one staged partial");

// Batches of sequences at arbitrary positions use more warps with fewer
// stages each: the same K/V bytes in flight per SM, more tiles in work at
// once (measured 5-8 % faster for ragged batches, slower for one sequence).
#ifndef KORE_DECODE_BATCH_NW
#define KORE_DECODE_BATCH_NW 12
#endif
#ifndef KORE_DECODE_BATCH_SPW
#define KORE_DECODE_BATCH_SPW 2
#endif
constexpr int kNWb = KORE_DECODE_BATCH_NW, kSPWb = KORE_DECODE_BATCH_SPW;
static_assert(DecodeSmem<128, kNWb, kTT, kSPWb>::bytes <= 227 * 1024, "batch decode stages exceed shared memory");
static_assert(DecodeSmem<64, kNWb, kTT, kSPWb>::stage_floats >= (size_t)kMaxSplits * 8 + 16 + 8 * 64 + 64,
              "split merge needs room for the weights and one staged partial");

template <int D, int R, int NW, int SPW>
cudaError_t launch_shape(const DecodeParams &p, int grid_x, cudaStream_t s, bool merge) {
    using SM = DecodeSmem<D, NW, kTT, SPW>;
    auto kern = attn_decode_kernel<D, R, NW, kTT, SPW>;
    if (cudaError_t e = ensure_smem_limit(reinterpret_cast<const void *>(kern), (int)SM::bytes)) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = p.fused_exchange ? dim3(grid_x * p.kv.G + p.H) : dim3(grid_x, p.kv.G, p.n_q);
    cfg.blockDim = dim3(NW * 32);
    cfg.dynamicSmemBytes = SM::bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess || grid_x == 1 || !merge || p.fused_exchange) return e;
    cudaLaunchConfig_t mcfg = cfg;
    mcfg.gridDim = dim3(p.kv.G * R, p.n_q);
    mcfg.blockDim = dim3(D);
    mcfg.dynamicSmemBytes = 0;
    return cudaLaunchKernelEx(&mcfg, split_merge_kernel<D, R>, p);
}

// Tensor-core decode shape: NW warps of 16-token tiles, SPW stages each
// (192 KB of K/V in flight per SM at 4 x 3, as the CUDA-core kernel's 8 x 8-token x 3).
#ifndef KORE_DECODE_TC_NW
#define KORE_DECODE_TC_NW 4
#endif
#ifndef KORE_DECODE_TC_SPW
#define KORE_DECODE_TC_SPW 3
#endif
constexpr int kNWt = KORE_DECODE_TC_NW, kSPWt = KORE_DECODE_TC_SPW;
static_assert(TcSmem<8, kNWt, kSPWt>::bytes <= 227 * 1024, "tensor-core decode stages exceed shared memory");
static_assert(kNWt * 32 >= 128, "a merge CTA of a fused launch needs one thread per dim");

template <int R>
cudaError_t launch_tc(const DecodeParams &p, int grid_x, cudaStream_t s, bool merge) {
    using SM = TcSmem<R, kNWt, kSPWt>;
    auto kern = attn_decode_tc_kernel<R, kNWt, kSPWt>;
    if (cudaError_t e = ensure_smem_limit(reinterpret_cast<const void *>(kern), (int)SM::bytes)) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = p.fused_exchange ? dim3(grid_x * p.kv.G + p.H) : dim3(grid_x, p.kv.G, 1);
    cfg.blockDim = dim3(kNWt * 32);
    cfg.dynamicSmemBytes = SM::bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess || grid_x == 1 || !merge || p.fused_exchange) return e;
    cudaLaunchConfig_t mcfg = cfg;
    mcfg.gridDim = dim3(p.kv.G * R, 1);
    mcfg.blockDim = dim3(128);
    mcfg.dynamicSmemBytes = 0;
    return cudaLaunchKernelEx(&mcfg, split_merge_kernel<128, R>, p);
}

template <int D, int R>
cudaError_t launch_dr(const DecodeParams &p, int grid_x, cudaStream_t s, bool merge) {
    if constexpr (D == 128)
        if (p.tc) return launch_tc<R>(p, grid_x, s, merge);
    if (p.n_q > 1 && !p.contiguous) return launch_shape<D, R, kNWb, kSPWb>(p, grid_x, s, merge);
    return launch_shape<D, R, kNW, kSPW>(p, grid_x, s, merge);
}

template <int D>
cudaError_t launch_d(const DecodeParams &p, int n_rep, int grid_x, cudaStream_t s, bool merge) {
    switch (n_rep) {
        case 1: return launch_dr<D, 1>(p, grid_x, s, merge);
        case 2: return launch_dr<D, 2>(p, grid_x, s, merge);
        case 3: return launch_dr<D, 3>(p, grid_x, s, merge);
        case 4: return launch_dr<D, 4>(p, grid_x, s, merge);
        case 5: return launch_dr<D, 5>(p, grid_x, s, merge);
        case 6: return launch_dr<D, 6>(p, grid_x, s, merge);
        case 7: return launch_dr<D, 7>(p, grid_x, s, merge);
        case 8: return launch_dr<D, 8>(p, grid_x, s, merge);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

cudaError_t launch_attn_decode(const DecodeParams &p, int n_rep, int grid_x, cudaStream_t s, bool merge) {
    if (p.kv.D == 128) return launch_d<128>(p, n_rep, grid_x, s, merge);
    if (p.kv.D == 64) return launch_d<64>(p, n_rep, grid_x, s, merge);
    return cudaErrorInvalidValue;
}

int decode_ctas_per_sm(int head_dim, int) {
    const size_t b = head_dim == 128 ? DecodeSmem<128, kNW, kTT, kSPW>::bytes : DecodeSmem<64, kNW, kTT, kSPW>::bytes;
    return b * 2 <= 227 * 1024 && kNW <= 8 ? 2 : 1;
}

int decode_tile_tokens() { return kTT; }

int decode_tc_tile_tokens() { return kTcTT; }

int decode_split_pages_max() { return kSplitPagesMax; }

size_t decode_smem_bytes(int head_dim) {
    return head_dim == 128 ? DecodeSmem<128, kNW, kTT, kSPW>::bytes : DecodeSmem<64, kNW, kTT, kSPW>::bytes;
}

// ---------------------------------------------------------------- no-allocation decode
//
// kore_cuda_attn_decode_noalloc runs the decode and split-merge kernels above
// for callers that cannot allocate device memory (see include/kore_cuda.h);
// their KV-split scratch is this fixed array instead of a context's buffers.

namespace {

constexpr size_t kNoallocFloats = KORE_CUDA_NOALLOC_SCRATCH_BYTES / sizeof(float);
constexpr size_t kNoallocPartFloats = (size_t)1 << 19;                          // split outputs: 2 MiB
constexpr size_t kNoallocMlPairs = (kNoallocFloats - kNoallocPartFloats) / 2;   // split (max, sum) pairs
static_assert(kNoallocFloats > kNoallocPartFloats, "scratch layout");

static __device__ __align__(256) float g_noalloc_scratch[kNoallocFloats];

// The array's device address, looked up once per device and CUDA context
// (the library's device code, the array with it, is loaded per context).
struct NoallocDevice {
    int dev = -1;
    uintptr_t cuda_ctx = 0;
    float *scratch = nullptr;   // device address of g_noalloc_scratch in that context
    int num_sms = 0;
};
std::mutex g_noalloc_mu;
std::vector<NoallocDevice> g_noalloc_dev;

int noalloc_fail(int code, const char *fmt, long long a = 0, long long b = 0) {
    char buf[256];
    snprintf(buf, sizeof buf, fmt, a, b);
    set_ctxless_error(buf);
    return code;
}

}  // namespace
}  // namespace kore

extern "C" int kore_cuda_attn_decode_noalloc(const kore_cuda_kv_view *kv, int pos, const float *q, const float *k,
                                             const float *v, float *out, int *dev_status, void *stream) {
    using namespace kore;
    if (!kv || !q || !k || !v || !out || !kv->k_pages || !kv->v_pages || !kv->page_table || !kv->rope_cs)
        return noalloc_fail(KORE_CUDA_EINVAL, "null argument");
    const int H = kv->n_head, G = kv->n_head_kv, D = kv->head_dim, P = kv->page_tokens;
    if (G <= 0 || H <= 0 || H % G || H / G > 8 || (D != 64 && D != 128))
        return noalloc_fail(KORE_CUDA_EINVAL, "unsupported geometry: n_head %lld, n_head_kv %lld", H, G);
    if (P <= 0 || P % 64 || kv->n_pages <= 0)
        return noalloc_fail(KORE_CUDA_EINVAL, "page_tokens %lld must be a positive multiple of 64", P);
    if ((reinterpret_cast<uintptr_t>(kv->k_pages) | reinterpret_cast<uintptr_t>(kv->v_pages)) & 15)
        return noalloc_fail(KORE_CUDA_EINVAL, "page pools must be 16-byte aligned");
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
         reinterpret_cast<uintptr_t>(kv->rope_cs)) & 15)
        return noalloc_fail(KORE_CUDA_EINVAL, "q, k, v and rope_cs must be 16-byte aligned");
    if (pos < 0 || pos >= kv->n_rope || pos / P >= kv->n_table)
        return noalloc_fail(KORE_CUDA_ERANGE, "position %lld outside the RoPE table or the page table", pos);

    const uintptr_t vdiff = reinterpret_cast<uintptr_t>(kv->v_pages) - reinterpret_cast<uintptr_t>(kv->k_pages);
    if (vdiff % 16)
        return noalloc_fail(KORE_CUDA_EINVAL, "v_pages - k_pages must be a multiple of 16 bytes");

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0)
        return noalloc_fail(KORE_CUDA_ECUDA, "no current CUDA device");
    const uintptr_t cctx = current_cuda_context();
    NoallocDevice nd;
    {
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        for (const NoallocDevice &d : g_noalloc_dev)
            if (d.dev == dev && d.cuda_ctx == cctx) nd = d;
        if (!nd.scratch) {   // set-up: once per device (and context), with that device current
            void *ptr = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
            if (e != cudaSuccess)
                return noalloc_fail(KORE_CUDA_ECUDA, "cudaGetSymbolAddress of the scratch array failed (error %lld)",
                                    (long long)e);
            e = cudaDeviceGetAttribute(&nd.num_sms, cudaDevAttrMultiProcessorCount, dev);
            if (e != cudaSuccess)
                return noalloc_fail(KORE_CUDA_ECUDA, "cudaDeviceGetAttribute failed (error %lld)", (long long)e);
            nd.dev = dev;
            nd.cuda_ctx = cctx;
            nd.scratch = static_cast<float *>(ptr);
            g_noalloc_dev.push_back(nd);
        }
    }

    const int R = H / G, TT = decode_tile_tokens();
    const int count = pos;   // cached positions 0..pos-1; the token at pos comes from k/v
    // splits: enough CTAs to fill the GPU, within the scratch array and the
    // per-split page list
    long long splits = std::max(1, (nd.num_sms + G - 1) / G);
    const long long cap_o = (long long)(kNoallocPartFloats / ((size_t)G * R * D));
    const long long cap_ml = (long long)(kNoallocMlPairs / ((size_t)G * R));
    splits = std::min(std::min(splits, (long long)kMaxSplits), std::min(cap_o, cap_ml));
    long long st = (count + splits - 1) / splits;
    st = std::max<long long>((st + TT - 1) / TT * TT, 4 * TT);
    const long long st_cap = (long long)(decode_split_pages_max() - 1) * P / TT * TT;
    if (st > st_cap) st = st_cap;
    const int grid_x = std::max(1, (int)((count + st - 1) / st));
    if ((size_t)G * grid_x * R * D > kNoallocPartFloats || (size_t)G * grid_x * R > kNoallocMlPairs ||
        grid_x > kMaxSplits)
        return noalloc_fail(KORE_CUDA_EINVAL, "%lld cached positions need more split scratch than the %lld-byte array",
                            count, (long long)KORE_CUDA_NOALLOC_SCRATCH_BYTES);

    DecodeParams p;
    memset(&p, 0, sizeof p);
    p.kv.k = kv->k_pages;
    // the distance between the pools in floats, from their byte addresses
    // (two separate allocations: no pointer difference between them)
    p.kv.v_off = (long long)(intptr_t)vdiff / (long long)sizeof(float);
    p.kv.page_table = kv->page_table;
    p.kv.pt_stride = kv->n_table;
    p.kv.P = P;
    p.kv.G = G;
    p.kv.D = D;
    p.kv.n_pages = kv->n_pages;
    p.kv.shard_rank = 0;
    p.kv.shard_count = 1;
    p.q = q;
    p.k_new = k;
    p.v_new = v;
    p.out = out;
    p.lse = nullptr;
    p.rope = reinterpret_cast<const float2 *>(kv->rope_cs);
    p.part_o = nd.scratch;
    p.part_ml = reinterpret_cast<float2 *>(nd.scratch + kNoallocPartFloats);
    p.err = dev_status;
    p.wait_ns = kWaitNs;
    p.scale_log2 = (1.0f / sqrtf((float)D)) * 1.4426950408889634f;
    p.H = H;
    p.n_q = 1;
    p.split_tokens = (int)st;
    p.max_splits = grid_x;
    p.append_new = 1;
    p.contiguous = 1;
    p.seq0 = 0;
    p.pos0 = pos;
    p.prefetch_ok = 0;   // nothing is known about the previous kernel on the caller's stream
    p.l2_prefetch_tokens = 0;
    const cudaError_t e = launch_attn_decode(p, R, grid_x, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return noalloc_fail(KORE_CUDA_ECUDA, "decode launch failed (error %lld)", (long long)e);
    return KORE_CUDA_OK;
}

#ifdef KORE_TRACE
// Trace build only: the stamps of the CTAs run since the last reset, as
// kore::TraceRec records of 64 bytes: the decode and merge CTAs in the order
// they claimed them, then the product CTAs (proj.cu) in theirs. Not part of
// the ABI.
extern "C" int kore_trace_read(void *host, int max_recs, int *n_recs) {
    using namespace kore;
    static_assert(sizeof(TraceRec) == 64, "trace record layout");
    unsigned n = 0;
    if (cudaDeviceSynchronize() != cudaSuccess || cudaMemcpyFromSymbol(&n, g_trace_n, sizeof n) != cudaSuccess)
        return KORE_CUDA_ECUDA;
    n = n < kTraceRecs ? n : kTraceRecs;
    const unsigned m = max_recs < 0 ? 0u : ((unsigned)max_recs < n ? (unsigned)max_recs : n);
    if (m && cudaMemcpyFromSymbol(host, g_trace, (size_t)m * sizeof(TraceRec)) != cudaSuccess) return KORE_CUDA_ECUDA;
    unsigned m2 = 0;
    if (max_recs > (int)m && proj_trace_read(static_cast<TraceRec *>(host) + m, (unsigned)max_recs - m, &m2))
        return KORE_CUDA_ECUDA;
    if (n_recs) *n_recs = (int)(m + m2);
    return KORE_CUDA_OK;
}

extern "C" int kore_trace_reset(void) {
    using namespace kore;
    const unsigned z = 0;
    if (cudaDeviceSynchronize() != cudaSuccess || cudaMemcpyToSymbol(g_trace_n, &z, sizeof z) != cudaSuccess ||
        proj_trace_reset())
        return KORE_CUDA_ECUDA;
    return KORE_CUDA_OK;
}
#endif
