// attn_decode.cu — split-KV flash-decode over the paged fp32 KV cache (sm_100a).
//
// Replaces kore's decode attention (kore.cpp:1424-1455): RoPE of q and of the
// new k at `pos`, append of k/v at `pos`, then softmax(q k^T / sqrt(d)) v over
// positions 0..pos for every query head. kore reads each KV head once per
// query head of its group (n_rep times); here one CTA serves the whole group,
// so every K/V byte crosses HBM once.
//
// Work decomposition
//   grid = (splits, n_head_kv, queries). A CTA owns one KV head of one query
//   and a contiguous range of `split_tokens` cached positions. Warp NW is the
//   producer: one lane streams TT-token K and V tiles into an S-stage ring of
//   shared memory with 1-D bulk copies (cp.async.bulk, mbarrier completion,
//   L2 evict-first). Warps 0..NW-1 consume: tile i goes to stage i % S and to
//   warp i % NW, and each warp keeps its own online-softmax state (running max
//   m, running sum l, output o) for the R = n_rep heads of the group.
//
// Lane layout inside a consumer warp (D = 128: VEC = 4 dims per lane)
//   lane owns dims [VEC*lane, VEC*lane+VEC) of q (R heads, pre-scaled by
//   log2(e)/sqrt(d)) and of o. A K row is read with one 16-byte LDS per lane.
//   Scores of 8 tokens x R heads are reduced across the warp by a butterfly
//   reduce-scatter (xor 16, 8, 4 split tokens; xor 2, 1 split head pairs):
//   55 shuffles per 8 tokens for R = 7 instead of 35 per token, after which
//   lane L holds the full scores of token L>>2 for heads 2(L&3), 2(L&3)+1.
//   Probabilities go through a tiny per-warp shared buffer so that every lane
//   can accumulate p * v for all R heads over its VEC dims.
//
// Merge: the warps of a CTA merge in shared memory; with more than one split
// each CTA writes (m, l, o) to scratch and the last CTA to arrive for its
// (query, KV head) — ordered by an atomic counter — merges the splits and
// writes the normalised output, then resets the counter. In a KV-sharded
// context (positions split over GPUs) the output is the normalised partial
// plus its log2-domain LSE, merged across GPUs afterwards.

#include "attn.cuh"
#include "common.cuh"

#include <cfloat>

namespace kore {
namespace {

constexpr unsigned FULL = 0xffffffffu;

template <int D, int NW, int TT, int S>
struct DecodeSmem {
    static constexpr int TILE_F = TT * D;
    static constexpr size_t stage_floats = (size_t)S * 2 * TILE_F;
    static constexpr size_t new_floats = 2 * 8 * D;
    static constexpr size_t pbuf_floats = (size_t)NW * TT * 8;
    static constexpr size_t bytes = (stage_floats + new_floats + pbuf_floats) * 4 + 2 * S * 8;
};

template <int D, int R, int TT>
struct WarpState {
    static constexpr int VEC = D / 32;
    float q[R][VEC];
    float o[R][VEC];
    float m[R];
    float mA, mB;   // running max of the two heads whose scores this lane owns
    float lA, lB;   // lane-partial running sums of those heads
};

// Processes one tile of `nv` (1..TT) tokens whose K rows start at Ks and V rows
// at Vs (shared memory, row stride D) for one consumer warp.
template <int D, int R, int TT>
__device__ __forceinline__ void process_tile(WarpState<D, R, TT> &st, const float *__restrict__ Ks,
                                             const float *__restrict__ Vs, int nv, float *__restrict__ pbuf,
                                             int lane) {
    constexpr int VEC = D / 32;
    constexpr int ROUNDS = TT / 8;
    const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4, b1 = lane & 2, b0 = lane & 1;

    float sc[ROUNDS][2];
#pragma unroll
    for (int r = 0; r < ROUNDS; ++r) {
        float part[8][R];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            float kv[VEC];
            const float *kr = Ks + (r * 8 + t) * D + lane * VEC;
            if constexpr (VEC == 4) {
                const float4 x = *reinterpret_cast<const float4 *>(kr);
                kv[0] = x.x; kv[1] = x.y; kv[2] = x.z; kv[3] = x.w;
            } else {
                const float2 x = *reinterpret_cast<const float2 *>(kr);
                kv[0] = x.x; kv[1] = x.y;
            }
#pragma unroll
            for (int h = 0; h < R; ++h) {
                float a = st.q[h][0] * kv[0];
#pragma unroll
                for (int j = 1; j < VEC; ++j) a = fmaf(st.q[h][j], kv[j], a);
                part[t][h] = a;
            }
        }
        // reduce-scatter over tokens: xor 16 keeps tokens {4..7} or {0..3}
        float a1[4][R];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int h = 0; h < R; ++h) {
                const float mine = b4 ? part[4 + j][h] : part[j][h];
                const float other = b4 ? part[j][h] : part[4 + j][h];
                a1[j][h] = mine + __shfl_xor_sync(FULL, other, 16);
            }
        float a2[2][R];
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int h = 0; h < R; ++h) {
                const float mine = b3 ? a1[2 + j][h] : a1[j][h];
                const float other = b3 ? a1[j][h] : a1[2 + j][h];
                a2[j][h] = mine + __shfl_xor_sync(FULL, other, 8);
            }
        float a3[8];
#pragma unroll
        for (int h = 0; h < R; ++h) {
            const float mine = b2 ? a2[1][h] : a2[0][h];
            const float other = b2 ? a2[0][h] : a2[1][h];
            a3[h] = mine + __shfl_xor_sync(FULL, other, 4);
        }
#pragma unroll
        for (int h = R; h < 8; ++h) a3[h] = 0.f;
        // reduce-scatter over heads: xor 2 keeps heads {4..7} or {0..3}, xor 1 a pair
        float a4[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float mine = b1 ? a3[4 + j] : a3[j];
            const float other = b1 ? a3[j] : a3[4 + j];
            a4[j] = (4 + j < R || j < R) ? mine + __shfl_xor_sync(FULL, other, 2) : 0.f;
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const float mine = b0 ? a4[2 + j] : a4[j];
            const float other = b0 ? a4[j] : a4[2 + j];
            sc[r][j] = mine + __shfl_xor_sync(FULL, other, 1);
        }
        if (r * 8 + (lane >> 2) >= nv) { sc[r][0] = -INFINITY; sc[r][1] = -INFINITY; }
    }

    // tile max of the lane's two heads, then of every head in every lane
    float tA = sc[0][0], tB = sc[0][1];
#pragma unroll
    for (int r = 1; r < ROUNDS; ++r) { tA = fmaxf(tA, sc[r][0]); tB = fmaxf(tB, sc[r][1]); }
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
        tA = fmaxf(tA, __shfl_xor_sync(FULL, tA, off));
        tB = fmaxf(tB, __shfl_xor_sync(FULL, tB, off));
    }
    float alpha[R];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float xa = __shfl_sync(FULL, tA, k);
        const float xb = __shfl_sync(FULL, tB, k);
        if (2 * k < R) {
            const float mn = fmaxf(st.m[2 * k], xa);
            alpha[2 * k] = fast_exp2(st.m[2 * k] - mn);
            st.m[2 * k] = mn;
        }
        if (2 * k + 1 < R) {
            const float mn = fmaxf(st.m[2 * k + 1], xb);
            alpha[2 * k + 1] = fast_exp2(st.m[2 * k + 1] - mn);
            st.m[2 * k + 1] = mn;
        }
    }
    {
        const float nA = fmaxf(st.mA, tA), nB = fmaxf(st.mB, tB);
        st.lA *= fast_exp2(st.mA - nA);
        st.lB *= fast_exp2(st.mB - nB);
        st.mA = nA;
        st.mB = nB;
    }
#pragma unroll
    for (int r = 0; r < ROUNDS; ++r) {
        const float pa = fast_exp2(sc[r][0] - st.mA);
        const float pb = fast_exp2(sc[r][1] - st.mB);
        st.lA += pa;
        st.lB += pb;
        *reinterpret_cast<float2 *>(pbuf + (r * 8 + (lane >> 2)) * 8 + 2 * (lane & 3)) = make_float2(pa, pb);
    }
#pragma unroll
    for (int h = 0; h < R; ++h)
#pragma unroll
        for (int j = 0; j < VEC; ++j) st.o[h][j] *= alpha[h];
    __syncwarp();

    auto pv_row = [&](int t) {
        const float4 p0 = *reinterpret_cast<const float4 *>(pbuf + t * 8);
        const float4 p1 = *reinterpret_cast<const float4 *>(pbuf + t * 8 + 4);
        const float pr[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
        float vv[VEC];
        const float *vr = Vs + t * D + lane * VEC;
        if constexpr (VEC == 4) {
            const float4 x = *reinterpret_cast<const float4 *>(vr);
            vv[0] = x.x; vv[1] = x.y; vv[2] = x.z; vv[3] = x.w;
        } else {
            const float2 x = *reinterpret_cast<const float2 *>(vr);
            vv[0] = x.x; vv[1] = x.y;
        }
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

template <int D, int R, int NW, int TT, int S>
__global__ void __launch_bounds__((NW + 1) * 32, 1) attn_decode_kernel(const __grid_constant__ DecodeParams p) {
    constexpr int VEC = D / 32;
    constexpr int HALF = D / 2;
    constexpr int NT = (NW + 1) * 32;
    using SM = DecodeSmem<D, NW, TT, S>;
    extern __shared__ __align__(128) float smem[];
    float *stages = smem;
    float *newk = stages + SM::stage_floats;
    float *newv = newk + 8 * D;
    float *pbuf_all = newv + 8 * D;
    uint64_t *full = reinterpret_cast<uint64_t *>(pbuf_all + SM::pbuf_floats);
    uint64_t *empty = full + S;
    __shared__ int s_last;

    const int split = blockIdx.x, g = blockIdx.y, qi = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int seq = p.contiguous ? p.seq0 : p.seq[qi];
    const int pos = p.contiguous ? p.pos0 + qi : p.pos[qi];
    const PagedKv &kv = p.kv;
    const int P = kv.P, NS = kv.shard_count, rank = kv.shard_rank;

    // cached positions read here: [0, limit) of those this shard holds
    const int limit = p.append_new ? pos : pos + 1;
    const int F = limit / P, rem = limit - F * P;
    const int nfull_local = F > rank ? (F - rank + NS - 1) / NS : 0;
    const int count = nfull_local * P + ((F % NS == rank) ? rem : 0);
    const bool own_new = p.append_new && ((pos / P) % NS == rank);
    const int ST = p.split_tokens;
    int n_splits = (count + ST - 1) / ST;
    if (n_splits == 0) n_splits = 1;
    if (split >= n_splits) return;
    const int u_begin = split * ST;
    const int u_end = min(count, u_begin + ST);
    const int n_tiles = u_end > u_begin ? (u_end - u_begin + TT - 1) / TT : 0;
    const bool do_new = own_new && split == n_splits - 1;
    const int *pt = kv.page_table + (size_t)seq * kv.pt_stride;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_fence_init();
    }
    __syncthreads();

    const float *kbase = kv.k + (size_t)g * P * D;
    WarpState<D, R, TT> st;
    if (warp == NW) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            // walks the page table as it goes: the raw id of the next page is
            // loaded when a page is entered and checked only when it is used,
            // one page (P/TT tiles) later, so the load latency stays hidden
            auto checked = [&](int ph) {
                if (ph < 0 || ph >= kv.n_pages) {
                    raise_error(p.err, DEV_BAD_PAGE);
                    ph = 0;
                }
                return ph;
            };
            const int last_lp = n_tiles > 0 ? (u_end - 1) / P : 0;
            const uint64_t pol = l2_evict_first_policy();
            int cur_lp = u_begin / P;
            int cur_ph = n_tiles > 0 ? checked(pt[cur_lp]) : 0;
            int next_raw = cur_lp < last_lp ? pt[cur_lp + 1] : 0;
            for (int i = 0; i < n_tiles; ++i) {
                const int s = i % S;
                if (i >= S && !mbar_wait(&empty[s], ((i / S) - 1) & 1, p.err, DEV_WAIT_EMPTY_TIMEOUT)) break;
                const int u0 = u_begin + i * TT;
                const int nv = min(TT, u_end - u0);
                const int lp = u0 / P;
                if (lp != cur_lp) {
                    cur_lp = lp;
                    cur_ph = checked(next_raw);
                    if (lp < last_lp) next_raw = pt[lp + 1];
                }
                const int off = u0 - lp * P;
                const float *src = kbase + ((size_t)cur_ph * kv.G * P + off) * D;
                const uint32_t bytes = (uint32_t)(nv * D * 4);
                float *dst = stages + (size_t)s * 2 * SM::TILE_F;
                mbar_arrive_expect_tx(&full[s], 2 * bytes);
                bulk_g2s(dst, src, bytes, &full[s], pol);
                bulk_g2s(dst + SM::TILE_F, src + kv.v_off, bytes, &full[s], pol);
            }
        }
    } else {
        // ------------------------------------------------------------ consumers
        const float2 *cs = p.rope + (size_t)pos * HALF;
        const float *qsrc = p.q + (size_t)qi * p.H * D + (size_t)g * R * D;
#pragma unroll
        for (int h = 0; h < R; ++h)
#pragma unroll
            for (int j = 0; j < VEC; ++j) {
                const int i = lane * VEC + j;
                const float x = __ldg(qsrc + h * D + i);
                const float y = __ldg(qsrc + h * D + (i ^ HALF));
                const float2 a = __ldg(cs + (i & (HALF - 1)));
                const float r = i < HALF ? rope_lo(x, y, a.x, a.y) : rope_hi(y, x, a.x, a.y);
                st.q[h][j] = r * p.scale_log2;
                st.o[h][j] = 0.f;
            }
#pragma unroll
        for (int h = 0; h < R; ++h) st.m[h] = -INFINITY;
        st.mA = st.mB = -INFINITY;
        st.lA = st.lB = 0.f;
        float *pbuf = pbuf_all + (size_t)warp * TT * 8;

        if (do_new && warp == 0) {
            // the token at pos: rotate k, stage k/v as a 1-token tile, append to the cache
            const float *ks = p.k_new + (size_t)qi * kv.G * D + (size_t)g * D;
            const float *vs = p.v_new + (size_t)qi * kv.G * D + (size_t)g * D;
            const int lp = (pos / P) / NS, off = pos % P;
            const int ph = pt[lp];
            const bool ok = ph >= 0 && ph < kv.n_pages;
            if (!ok && lane == 0) raise_error(p.err, DEV_BAD_PAGE);
            float *kd = kv.k + (((size_t)(ok ? ph : 0) * kv.G + g) * P + off) * D;
#pragma unroll
            for (int j = 0; j < VEC; ++j) {
                const int i = lane * VEC + j;
                const float x = __ldg(ks + i), y = __ldg(ks + (i ^ HALF));
                const float2 a = __ldg(cs + (i & (HALF - 1)));
                const float kr = i < HALF ? rope_lo(x, y, a.x, a.y) : rope_hi(y, x, a.x, a.y);
                const float vr = __ldg(vs + i);
                newk[i] = kr;
                newv[i] = vr;
                if (ok) {
                    kd[i] = kr;
                    kd[i + kv.v_off] = vr;
                }
            }
            __syncwarp();
            process_tile<D, R, TT>(st, newk, newv, 1, pbuf, lane);
        }

        for (int i = warp; i < n_tiles; i += NW) {
            const int s = i % S;
            if (!mbar_wait(&full[s], (i / S) & 1, p.err, DEV_WAIT_FULL_TIMEOUT)) break;
            const int nv = min(TT, u_end - (u_begin + i * TT));
            const float *tile = stages + (size_t)s * 2 * SM::TILE_F;
            process_tile<D, R, TT>(st, tile, tile + SM::TILE_F, nv, pbuf, lane);
            if (lane == 0) mbar_arrive(&empty[s]);
        }

        // lane-partial sums -> per head pair (lanes with equal lane & 3)
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
            st.lA += __shfl_xor_sync(FULL, st.lA, off);
            st.lB += __shfl_xor_sync(FULL, st.lB, off);
        }
    }
    __syncthreads();   // every tile consumed: the stage memory is free
    if (warp < NW) {
        float *cm = stages;              // [NW][8]
        float *cl = cm + NW * 8;         // [NW][8]
        float *co = cl + NW * 8;         // [NW][R][D]
        if (lane == 0)
#pragma unroll
            for (int h = 0; h < R; ++h) cm[warp * 8 + h] = st.m[h];
        if (lane < 4) {
            cl[warp * 8 + 2 * lane] = st.lA;
            cl[warp * 8 + 2 * lane + 1] = st.lB;
        }
#pragma unroll
        for (int h = 0; h < R; ++h)
#pragma unroll
            for (int j = 0; j < VEC; ++j) co[(warp * R + h) * D + lane * VEC + j] = st.o[h][j];
    }
    __syncthreads();

    // ---------------------------------------------------------------- CTA merge
    const float *cm = stages;
    const float *cl = cm + NW * 8;
    const float *co = cl + NW * 8;
    const int Hq = p.H;
    const size_t qh0 = (size_t)qi * Hq + (size_t)g * R;     // first query head of the group
    const size_t part_base = ((size_t)qi * kv.G + g) * p.max_splits;
    for (int idx = tid; idx < R * D; idx += NT) {
        const int h = idx / D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; ++w) M = fmaxf(M, cm[w * 8 + h]);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < NW; ++w) {
                const float e = fast_exp2(cm[w * 8 + h] - M);
                L = fmaf(cl[w * 8 + h], e, L);
                O = fmaf(co[(w * R + h) * D + (idx - h * D)], e, O);
            }
        }
        if (n_splits == 1) {
            p.out[qh0 * D + idx] = L > 0.f ? O / L : 0.f;
            if (p.lse && idx - h * D == 0) p.lse[qh0 + h] = L > 0.f ? M + __log2f(L) : -INFINITY;
        } else {
            p.part_o[(part_base + split) * R * D + idx] = O;
            if (idx - h * D == 0) p.part_ml[(part_base + split) * R + h] = make_float2(M, L);
        }
    }
    if (n_splits == 1) return;

    // ---------------------------------------------------------------- split merge
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned prev = atomicAdd(&p.counters[(size_t)qi * kv.G + g], 1u);
        s_last = prev == (unsigned)(n_splits - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    float *wts = stages;                       // [n_splits][8] split weights
    float *linv = wts + (size_t)n_splits * 8;  // [8] 1/L per head
    float *mh = linv + 8;                      // [8] merged max per head
    for (int h = warp; h < R; h += NW + 1) {
        float M = -INFINITY;
        for (int s = lane; s < n_splits; s += 32) M = fmaxf(M, __ldcg(&p.part_ml[(part_base + s) * R + h]).x);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(FULL, M, off));
        float L = 0.f;
        for (int s = lane; s < n_splits; s += 32) {
            const float2 ml = __ldcg(&p.part_ml[(part_base + s) * R + h]);
            const float w = M == -INFINITY ? 0.f : fast_exp2(ml.x - M);
            wts[s * 8 + h] = w;
            L = fmaf(ml.y, w, L);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(FULL, L, off);
        if (lane == 0) {
            linv[h] = L > 0.f ? 1.f / L : 0.f;
            mh[h] = L > 0.f ? M + __log2f(L) : -INFINITY;
        }
    }
    __syncthreads();
    for (int idx = tid; idx < R * D; idx += NT) {
        const int h = idx / D;
        float O = 0.f;
        for (int s = 0; s < n_splits; ++s) O = fmaf(wts[s * 8 + h], __ldcg(&p.part_o[(part_base + s) * R * D + idx]), O);
        p.out[qh0 * D + idx] = O * linv[h];
        if (p.lse && idx - h * D == 0) p.lse[qh0 + h] = mh[h];
    }
    if (tid == 0) p.counters[(size_t)qi * kv.G + g] = 0u;
}

// Tuning of the decode pipeline: 8 consumer warps, 8-token tiles, 16 stages
// (two per consumer warp, so each warp's next tile loads while it computes).
constexpr int kNW = 8, kTT = 8, kS = 16;
static_assert(kS % kNW == 0, "a warp's tiles must cycle through its own stages");

template <int D, int R>
cudaError_t launch_dr(const DecodeParams &p, int grid_x, cudaStream_t s) {
    using SM = DecodeSmem<D, kNW, kTT, kS>;
    auto kern = attn_decode_kernel<D, R, kNW, kTT, kS>;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SM::bytes);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) configured[dev] = true;
    }
    dim3 grid(grid_x, p.kv.G, p.n_q);
    kern<<<grid, (kNW + 1) * 32, SM::bytes, s>>>(p);
    return cudaGetLastError();
}

template <int D>
cudaError_t launch_d(const DecodeParams &p, int n_rep, int grid_x, cudaStream_t s) {
    switch (n_rep) {
        case 1: return launch_dr<D, 1>(p, grid_x, s);
        case 2: return launch_dr<D, 2>(p, grid_x, s);
        case 3: return launch_dr<D, 3>(p, grid_x, s);
        case 4: return launch_dr<D, 4>(p, grid_x, s);
        case 5: return launch_dr<D, 5>(p, grid_x, s);
        case 6: return launch_dr<D, 6>(p, grid_x, s);
        case 7: return launch_dr<D, 7>(p, grid_x, s);
        case 8: return launch_dr<D, 8>(p, grid_x, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

cudaError_t launch_attn_decode(const DecodeParams &p, int n_rep, int grid_x, cudaStream_t s) {
    if (p.kv.D == 128) return launch_d<128>(p, n_rep, grid_x, s);
    if (p.kv.D == 64) return launch_d<64>(p, n_rep, grid_x, s);
    return cudaErrorInvalidValue;
}

int decode_ctas_per_sm(int head_dim, int) {
    const size_t b = head_dim == 128 ? DecodeSmem<128, kNW, kTT, kS>::bytes : DecodeSmem<64, kNW, kTT, kS>::bytes;
    return b * 2 <= 227 * 1024 ? 2 : 1;
}

int decode_tile_tokens() { return kTT; }

size_t decode_smem_bytes(int head_dim) {
    return head_dim == 128 ? DecodeSmem<128, kNW, kTT, kS>::bytes : DecodeSmem<64, kNW, kTT, kS>::bytes;
}

}  // namespace kore
