// attn_prefill.cu — causal GQA prefill attention on the 5th-generation tensor
// cores (tcgen05 MMA, accumulators in tensor memory), sm_100a.
//
// Replaces kore's prefill attention (kore.cpp:1542-1563): for query row z of a
// chunk at positions pos0..pos0+n-1 and every head, softmax(q k^T / sqrt(d)) v
// over positions 0..pos0+z (the chunk's K/V are appended first, kore.cpp:
// 1527-1539). Algorithmic work: 4*d FLOPs per unmasked (query, key) pair.
//
// Precision. kore computes in fp32 and the parity bound is 1e-3 relative per
// head. Each fp32 operand x is split into two bf16 parts, hi = bf16(x) and
// mid = bf16(x - hi), so that x = hi + mid to 2^-16, and every product is
// formed with three bf16 MMAs (hi*hi + hi*mid + mid*hi) accumulating in fp32:
// error ~2^-16 per product, for 1.5 tf32-equivalents of tensor time (three
// tf32 MMAs would cost twice that).
//
// Data path.
//   kv_split_kernel   converts this layer's K (as [key][d]) and V (transposed,
//                     [d][key]) for positions 0..pos0+n-1, 64 keys per tile,
//                     into hi/mid bf16 tiles laid out in global memory exactly
//                     as the MMA reads them from shared memory (K-major,
//                     128-byte swizzle), so the attention kernel fetches a
//                     tile with plain bulk copies. Keys past the last position
//                     are zero, so they never reach an output through 0 * NaN.
//   prefill_kernel    one CTA per (128-row query tile, query head):
//     warps 0-3   softmax: thread t owns query row t. Prologue: RoPE of its q
//                 row, scale by log2(e)/sqrt(d), hi/mid split into the Q
//                 operand. Per key tile: S row from tensor memory, causal
//                 mask, online softmax with a lazily moved reference maximum
//                 (O in tensor memory is rescaled only when a score exceeds
//                 the reference by 2^8), P split into the P operand.
//                 Epilogue: O / l to global memory.
//     warps 4, 6  producers: K hi/mid and V^T hi/mid of a tile in separate
//                 three-stage rings (a K stage frees as soon as its S is
//                 done), bulk copies completing on mbarriers.
//     warp 5      allocates tensor memory; one lane issues the MMAs:
//                 S[j%4] = Q K_j^T (128 x 64), then O += P_j V_j (128 x d),
//                 issuing S for tile j+2 together with O for tile j after a
//                 single wait point per tile, so that the softmax of tiles
//                 j+1, j+2 overlaps them. Two tcgen05.commits per tile
//                 signal completion to the softmax warps and free K/V
//                 stages and S buffers.
//   Tensor memory: Q hi/mid (the A operand of S = Q K^T), four S buffers (64
//   columns each; a tile's P hi/mid, the A operand of O += P V, overwrites
//   its S) and O (d columns): 512 columns. Only K and V^T are read from
//   shared memory, which halves the operand traffic per MMA.
// Every mbarrier wait is bounded (2 s), after which the CTA records an error
// and drains out; tensor memory is always released.

#include "attn.cuh"
#include "common.cuh"

#include <cuda_bf16.h>

namespace kore {
namespace {

constexpr int kRows = 128;        // query rows per CTA (TMEM lanes)
constexpr int kKeys = 64;         // keys per tile
constexpr int kStages = 3;        // K and V ring stages
constexpr int kBufs = 4;          // S/P buffers in tensor memory
constexpr float kRescale = 8.0f;  // log2-domain slack before O is rescaled
constexpr unsigned FULLMASK = 0xffffffffu;

// ---------------------------------------------------------------- layouts

// Byte offset of 16-byte chunk c (0..7) of row r in a K-major, 128-byte
// swizzled operand whose rows are 128 bytes: 8-row atoms of 1024 bytes, the
// chunk index XOR-ed with the row within the atom.
__device__ __forceinline__ uint32_t sw128(int r, int c) {
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (stride byte offset), Blackwell descriptor version 1.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor: bf16 x bf16 -> fp32, both operands K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

template <int D>
struct PrefillSmem {
    static constexpr int QATOMS = D / 64;                                // 64-element K atoms of K
    static constexpr uint32_t K_PART = (uint32_t)QATOMS * kKeys * 128;   // one of hi/mid
    static constexpr uint32_t V_PART = (uint32_t)D * 128;                // V^T: d rows x 64 keys
    static constexpr uint32_t TILE = 2 * K_PART + 2 * V_PART;            // one global tile: K half, V half
    static constexpr uint32_t k_off = 0;                                 // K ring: kStages x (hi, mid)
    static constexpr uint32_t v_off = k_off + kStages * 2 * K_PART;      // V ring: kStages x (hi, mid)
    static constexpr uint32_t bar_off = v_off + kStages * 2 * V_PART;
    // barriers, TMEM base, alignment slack; at least 116 KB so that one CTA
    // holds an SM (a second would only wait in tcgen05.alloc for the 512
    // tensor-memory columns the first holds)
    static constexpr uint32_t bytes = bar_off + 512 + 1024 > 116u * 1024 ? bar_off + 512 + 1024 : 116u * 1024;
    // tensor memory columns: Q hi/mid as MMA A operand (bf16 pairs), kBufs S
    // buffers (fp32; the tile's P hi/mid, bf16 pairs, overwrite them), O
    static constexpr uint32_t T_Q = 0, T_S = 128, T_O = T_S + kBufs * 64;
    static constexpr uint32_t TMEM_COLS = 512;
};

// ---------------------------------------------------------------- tcgen05 helpers

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

// A operand from tensor memory (bf16 pairs, row m in lane m, element k in
// column k/2, even k in the low half), B from shared memory.
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 bits, 32 consecutive columns: thread (lane i of the warp)
// gets row (warp quarter * 32 + i), columns col..col+31.
__device__ __forceinline__ void tc_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tc_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])),
        "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
        "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])),
        "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}

__device__ __forceinline__ void tc_st32u(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
        "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
        "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}

// hi/mid bf16 split of 2 fp32 values, each part packed as one 32-bit word
// (first value in the low half)
__device__ __forceinline__ void split2(float x0, float x1, uint32_t &hi, uint32_t &mid) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(x0, x1);
    const float2 af = __bfloat1622float2(a);
    const __nv_bfloat162 b = __floats2bfloat162_rn(x0 - af.x, x1 - af.y);
    hi = *reinterpret_cast<const uint32_t *>(&a);
    mid = *reinterpret_cast<const uint32_t *>(&b);
}

__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// hi/mid bf16 split of 8 consecutive fp32 values, packed as two 16-byte chunks
__device__ __forceinline__ void split8(const float *x, uint4 &hi, uint4 &mid) {
    uint32_t h[4], m[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __nv_bfloat162 a = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
        const float2 af = __bfloat1622float2(a);
        const __nv_bfloat162 b = __floats2bfloat162_rn(x[2 * i] - af.x, x[2 * i + 1] - af.y);
        h[i] = *reinterpret_cast<const uint32_t *>(&a);
        m[i] = *reinterpret_cast<const uint32_t *>(&b);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    mid = make_uint4(m[0], m[1], m[2], m[3]);
}

// ---------------------------------------------------------------- K/V split pre-pass

// One CTA per (64-key tile, KV head): gathers the tile's K and V rows from the
// paged pool and writes the four operand images (K hi, K mid, V^T hi, V^T
// mid) of the tile to split + (g * tiles + j) * TILE.
template <int D>
__global__ void __launch_bounds__(256) kv_split_kernel(const __grid_constant__ PrefillParams p) {
    using SM = PrefillSmem<D>;
    __shared__ float vs[kKeys][D + 1];
    const int j = blockIdx.x, g = blockIdx.y, tid = threadIdx.x;
    const PagedKv &kv = p.kv;
    const int n_keys = p.pos0 + p.n;
    const int *pt = kv.page_table + (size_t)p.seq * kv.pt_stride;
    uint8_t *tile = reinterpret_cast<uint8_t *>(p.split) + ((size_t)g * p.tiles + j) * SM::TILE;
    constexpr int CH = D / 8;   // 16-byte bf16 chunks per K row
    // K: row = key, 8 d values per chunk; V rows staged in shared memory
    for (int w = tid; w < kKeys * CH; w += blockDim.x) {
        const int r = w / CH, c = w - r * CH;
        const int key = j * kKeys + r;
        float x[8] = {0, 0, 0, 0, 0, 0, 0, 0}, y[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (key < n_keys) {
            int ph = pt[key / kv.P];
            if (ph < 0 || ph >= kv.n_pages) {
                raise_error(p.err, DEV_BAD_PAGE);
                ph = 0;
            }
            const float *src = kv.k + (((size_t)ph * kv.G + g) * kv.P + (key % kv.P)) * D + c * 8;
            const float4 a = __ldg(reinterpret_cast<const float4 *>(src));
            const float4 b = __ldg(reinterpret_cast<const float4 *>(src + 4));
            const float4 e = __ldg(reinterpret_cast<const float4 *>(src + kv.v_off));
            const float4 f = __ldg(reinterpret_cast<const float4 *>(src + kv.v_off + 4));
            x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
            y[0] = e.x; y[1] = e.y; y[2] = e.z; y[3] = e.w; y[4] = f.x; y[5] = f.y; y[6] = f.z; y[7] = f.w;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) vs[r][c * 8 + i] = y[i];
        uint4 hi, mid;
        split8(x, hi, mid);
        const uint32_t off = (uint32_t)(c >> 3) * (kKeys * 128) + sw128(r, c & 7);
        *reinterpret_cast<uint4 *>(tile + off) = hi;
        *reinterpret_cast<uint4 *>(tile + SM::K_PART + off) = mid;
    }
    __syncthreads();
    // V^T: row = d, 8 keys per chunk
    for (int w = tid; w < D * 8; w += blockDim.x) {
        const int r = w >> 3, c = w & 7;
        float x[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = vs[c * 8 + i][r];
        uint4 hi, mid;
        split8(x, hi, mid);
        const uint32_t off = 2 * SM::K_PART + sw128(r, c);
        *reinterpret_cast<uint4 *>(tile + off) = hi;
        *reinterpret_cast<uint4 *>(tile + SM::V_PART + off) = mid;
    }
}

// ---------------------------------------------------------------- attention

template <int D>
__global__ void __launch_bounds__(224, 1) prefill_kernel(const __grid_constant__ PrefillParams p) {
    using SM = PrefillSmem<D>;
    constexpr int HALF = D / 2;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(smem);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + SM::bar_off);
    // Two commits per tile carry every completion (each commit and each
    // mbarrier access of the MMA thread costs tensor-pipe time):
    //   s_full[j % 4]  after S_j = Q K_j^T: the softmax may read S_j, and the
    //                  K stage of tile j may take tile j + 3;
    //   p_free[j % 4]  after O += P_j V_j: S buffer j % 4 may take S_{j+4},
    //                  the V stage of tile j may take tile j + 3, and O holds
    //                  every tile up to j.
    // A parity wait is exact only within one phase of the barrier's count.
    // Every wait below is: each waiter has already seen the completion four
    // tiles earlier on the same barrier (or it is the first), and the
    // completion four tiles later needs something the waiter has not done
    // yet (the next K or V tile, or the next P).
    uint64_t *k_full = bars;               // [3] K producer -> MMA
    uint64_t *v_full = bars + 3;           // [3] V producer -> MMA
    uint64_t *s_full = bars + 6;           // [4]
    uint64_t *p_free = bars + 10;          // [4]
    uint64_t *p_full = bars + 14;          // [4] softmax (4 warps) -> MMA: P of a buffer written
    uint64_t *q_ready = bars + 18;         // softmax (4 warps) -> MMA
    uint64_t *mma_drained = bars + 19;     // MMA commit -> MMA issuer, before TMEM is freed
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 20);
    int *abort_flag = reinterpret_cast<int *>(bars + 21);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qt = gridDim.x - 1 - blockIdx.x;   // heaviest (last) query tiles first
    const int h = blockIdx.y;
    const int g = h / p.n_rep;
    const int z0 = qt * kRows;
    const int rows = min(kRows, p.n - z0);
    const int last_key = p.pos0 + z0 + rows - 1;                // causal limit of the last row
    const int n_tiles = last_key / kKeys + 1;
    const int first_masked = (p.pos0 + z0) / kKeys;              // tiles from here need the mask

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&v_full[i], 1);
        }
        for (int i = 0; i < kBufs; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&p_free[i], 1);
            mbar_init(&p_full[i], 4);
        }
        mbar_init(q_ready, 4);
        mbar_init(mma_drained, 1);
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 5) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(SM::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t t_q = tmem + SM::T_Q, t_o = tmem + SM::T_O;   // S buffer b at tmem + T_S + 64 * b

    // a completed phase costs one try_wait; the abort flag is read only on
    // the slow path
    auto bounded_wait = [&](uint64_t *bar, uint32_t parity) -> bool {
        if (mbar_try_wait(bar, parity)) return true;
        if (*reinterpret_cast<volatile int *>(abort_flag)) return false;
        if (mbar_wait(bar, parity, p.err, DEV_WAIT_FULL_TIMEOUT)) return true;
        *reinterpret_cast<volatile int *>(abort_flag) = 1;
        return false;
    };

    if (warp == 4 || warp == 6) {
        // ------------------------------------------------------------ producers
        // warp 4 streams the K halves of the tiles, warp 6 the V^T halves: a K
        // stage is free again once its S = Q K^T is done, long before the P.V
        // that frees a V stage, so K runs ahead of V
        if (lane == 0) {
            const bool is_k = warp == 4;
            const uint32_t half = is_k ? 2 * SM::K_PART : 2 * SM::V_PART;
            uint64_t *full = is_k ? k_full : v_full;
            uint64_t *done = is_k ? s_full : p_free;   // tile j - kStages no longer needs the stage
            const uint8_t *src0 = reinterpret_cast<const uint8_t *>(p.split) + (size_t)g * p.tiles * SM::TILE +
                                  (is_k ? 0 : 2 * SM::K_PART);
            uint8_t *ring = smem + (is_k ? SM::k_off : SM::v_off);
            for (int j = 0; j < n_tiles; ++j) {
                const int s = j % kStages;
                const int jp = j - kStages;
                if (jp >= 0 && !bounded_wait(&done[jp % kBufs], (jp / kBufs) & 1)) break;
                uint8_t *dst = ring + s * half;
                mbar_arrive_expect_tx(&full[s], half);
#pragma unroll
                for (int part = 0; part < 2; ++part)   // kept in L2: every query tile and head reads it
                    bulk_g2s_plain(dst + part * (half / 2), src0 + (size_t)j * SM::TILE + part * (half / 2), half / 2,
                                   &full[s]);
            }
        }
    } else if (warp == 5) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t ID_S = idesc_bf16(kRows, kKeys), ID_O = idesc_bf16(kRows, D);
            bool ok = bounded_wait(q_ready, 0);
            tc_fence_after();
            auto issue_s = [&](int j) {   // S_j = Q K_j^T into buffer j % kBufs
                const uint32_t kb = sbase + SM::k_off + (j % kStages) * 2 * SM::K_PART;
                const uint32_t ts = tmem + SM::T_S + 64 * (j % kBufs);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t ko = (kk >> 2) * (kKeys * 128) + (kk & 3) * 32;
                    tc_mma_ts(ts, t_q + kk * 8, sdesc(kb + ko), ID_S, kk > 0);                        // hi*hi
                    tc_mma_ts(ts, t_q + kk * 8, sdesc(kb + SM::K_PART + ko), ID_S, 1);                // hi*mid
                    tc_mma_ts(ts, t_q + HALF + kk * 8, sdesc(kb + ko), ID_S, 1);                      // mid*hi
                }
                tc_commit(&s_full[j % kBufs]);
            };
            auto issue_pv = [&](int j) {   // O += P_j V_j, P_j in buffer j % kBufs
                const uint32_t vb = sbase + SM::v_off + (j % kStages) * 2 * SM::V_PART;
                const uint32_t tp = tmem + SM::T_S + 64 * (j % kBufs);   // P hi in columns 0-31, P mid in 32-63
#pragma unroll
                for (int kk = 0; kk < kKeys / 16; ++kk) {
                    const uint32_t o = kk * 32;
                    tc_mma_ts(t_o, tp + kk * 8, sdesc(vb + o), ID_O, (j > 0 || kk > 0));               // hi*hi
                    tc_mma_ts(t_o, tp + kk * 8, sdesc(vb + SM::V_PART + o), ID_O, 1);                  // hi*mid
                    tc_mma_ts(t_o, tp + 32 + kk * 8, sdesc(vb + o), ID_O, 1);                          // mid*hi
                }
                tc_commit(&p_free[j % kBufs]);
            };
            for (int j = 0; ok && j < 2 && j < n_tiles; ++j) {
                ok = bounded_wait(&k_full[j % kStages], (j / kStages) & 1);
                if (ok) issue_s(j);
            }
            // One wait point per tile: the first mbarrier access after a burst
            // of MMAs waits for the burst to drain from the issue queue, so
            // every wait of an iteration is taken at once, then S two tiles
            // ahead and O for this tile are issued back to back.
            for (int j = 0; ok && j < n_tiles; ++j) {
                const int j2 = j + 2;
                ok = bounded_wait(&p_full[j % kBufs], (j / kBufs) & 1) &&
                     bounded_wait(&v_full[j % kStages], (j / kStages) & 1);
                if (ok && j2 < n_tiles)
                    ok = bounded_wait(&k_full[j2 % kStages], (j2 / kStages) & 1) &&
                         (j2 < kBufs || bounded_wait(&p_free[j2 % kBufs], ((j2 / kBufs) - 1) & 1));
                if (!ok) break;
                tc_fence_after();
                if (j2 < n_tiles) issue_s(j2);
                issue_pv(j);
            }
            // tensor memory is released below only after every MMA issued here is done
            tc_commit(mma_drained);
            mbar_wait(mma_drained, 0, p.err, DEV_WAIT_FULL_TIMEOUT);
        }
    } else {
        // ------------------------------------------------------------ softmax (warps 0-3)
        const int t = threadIdx.x;                  // query row, TMEM lane
        const int z = z0 + t;
        const bool valid = t < rows;
        const int lim = p.pos0 + z;                 // last key this row attends to
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        // Q row: RoPE at its position, scale, hi/mid split into tensor memory
        {
            float qv[D];
            const float *qsrc = p.q + ((size_t)z * p.H + h) * D;
            const float2 *cs = p.rope + (size_t)(valid ? lim : 0) * HALF;
#pragma unroll
            for (int i = 0; i < D; i += 4) {
                const float4 a = valid ? __ldg(reinterpret_cast<const float4 *>(qsrc + i)) : make_float4(0, 0, 0, 0);
                qv[i] = a.x; qv[i + 1] = a.y; qv[i + 2] = a.z; qv[i + 3] = a.w;
            }
#pragma unroll
            for (int i = 0; i < HALF; ++i) {
                const float2 a = __ldg(cs + i);
                const float x0 = qv[i], x1 = qv[i + HALF];
                qv[i] = rope_lo(x0, x1, a.x, a.y) * p.scale_log2;
                qv[i + HALF] = rope_hi(x0, x1, a.x, a.y) * p.scale_log2;
            }
#pragma unroll
            for (int c0 = 0; c0 < HALF; c0 += 32) {   // 32 columns = 64 elements per store
                uint32_t hi[32], mid[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) split2(qv[2 * (c0 + i)], qv[2 * (c0 + i) + 1], hi[i], mid[i]);
                tc_st32u(t_q + lane_off + c0, hi);
                tc_st32u(t_q + lane_off + HALF + c0, mid);
            }
            tc_wait_st();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(q_ready);

        float m_ref = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < n_tiles; ++j) {
            const int b = j % kBufs;
            const uint32_t ts = tmem + SM::T_S + 64 * b + lane_off;
            if (!bounded_wait(&s_full[b], (j / kBufs) & 1)) { ok = false; break; }
            tc_fence_after();
            float sv[64];
            tc_ld32(ts, *reinterpret_cast<float(*)[32]>(sv));
            tc_ld32(ts + 32, *reinterpret_cast<float(*)[32]>(sv + 32));
            tc_wait_ld();
            if (j >= first_masked) {
#pragma unroll
                for (int i = 0; i < 64; ++i)
                    if (j * kKeys + i > lim) sv[i] = -INFINITY;
            }
            // row maximum as a tree (8 independent chains, then pairs)
            float mx8[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) mx8[c] = sv[c];
#pragma unroll
            for (int i = 8; i < 64; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], sv[i]);
            const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                                   fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
            const bool need = mx > m_ref + kRescale;
            const bool any_need = __any_sync(FULLMASK, need);
            const float m_new = need ? mx : m_ref;
            const float alpha = fast_exp2(m_ref - m_new);   // 0 for the first tile, 1 where not needed
            float l8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
            for (int i = 0; i < 64; ++i) {
                sv[i] = fast_exp2(sv[i] - m_new);
                l8[i & 7] += sv[i];
            }
            l = fmaf(l, alpha, ((l8[0] + l8[1]) + (l8[2] + l8[3])) + ((l8[4] + l8[5]) + (l8[6] + l8[7])));
            m_ref = m_new;
            // P of this tile into its own S buffer (S has been read above)
            {
                uint32_t hi[32], mid[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) split2(sv[2 * i], sv[2 * i + 1], hi[i], mid[i]);
                tc_st32u(ts, hi);
                tc_st32u(ts + 32, mid);
            }
            // O is stable only once the previous tile's P.V is done
            if (any_need && j > 0) {
                if (!bounded_wait(&p_free[(j - 1) % kBufs], ((j - 1) / kBufs) & 1)) { ok = false; break; }
                tc_fence_after();
#pragma unroll
                for (int c0 = 0; c0 < D; c0 += 32) {
                    float o[32];
                    tc_ld32(t_o + lane_off + c0, o);
                    tc_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] *= alpha;
                    tc_st32(t_o + lane_off + c0, o);
                }
            }
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[b]);
        }
        // epilogue: O / l
        if (ok && n_tiles > 0 && bounded_wait(&p_free[(n_tiles - 1) % kBufs], ((n_tiles - 1) / kBufs) & 1)) {
            tc_fence_after();
            const float inv = l > 0.f ? 1.f / l : 0.f;
            float *dst = p.out + ((size_t)z * p.H + h) * D;
#pragma unroll
            for (int c0 = 0; c0 < D; c0 += 32) {
                float o[32];
                tc_ld32(t_o + lane_off + c0, o);
                tc_wait_ld();
                if (valid) {
#pragma unroll
                    for (int i = 0; i < 32; i += 4)
                        *reinterpret_cast<float4 *>(dst + c0 + i) =
                            make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(SM::TMEM_COLS)
                     : "memory");
    }
}

template <int D>
cudaError_t launch_prefill_d(const PrefillParams &p, cudaStream_t s) {
    using SM = PrefillSmem<D>;
    const int tiles_needed = (p.pos0 + p.n + kKeys - 1) / kKeys;
    if (tiles_needed > p.tiles) return cudaErrorInvalidValue;
    kv_split_kernel<D><<<dim3(tiles_needed, p.kv.G), 256, 0, s>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !configured[dev]) {
        e = cudaFuncSetAttribute(prefill_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SM::bytes);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) configured[dev] = true;
    }
    const int q_tiles = (p.n + kRows - 1) / kRows;
    prefill_kernel<D><<<dim3(q_tiles, p.H), 224, SM::bytes, s>>>(p);
    return cudaGetLastError();
}

}  // namespace

size_t prefill_tile_bytes(int head_dim) {
    return head_dim == 128 ? PrefillSmem<128>::TILE : PrefillSmem<64>::TILE;
}
int prefill_tile_keys() { return kKeys; }

cudaError_t launch_prefill(const PrefillParams &p, cudaStream_t s) {
    if (p.kv.D == 128) return launch_prefill_d<128>(p, s);
    if (p.kv.D == 64) return launch_prefill_d<64>(p, s);
    return cudaErrorInvalidValue;
}

}  // namespace kore
