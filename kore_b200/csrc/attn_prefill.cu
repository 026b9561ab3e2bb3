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
//   kv_split_kernel   converts this layer's K and V for positions
//                     0..pos0+n-1, 128 keys per tile, into hi/mid bf16 operand
//                     images laid out in global memory exactly as the MMA
//                     reads them from shared memory (K-major, 128-byte
//                     swizzle): per tile, K as d/64 chunks [128 keys][64 d]
//                     and V^T as two chunks [d][64 keys], so the attention
//                     kernel fetches each with one bulk copy. Keys past the
//                     last position are zero, so they never reach an output
//                     through 0 * NaN.
//   prefill_kernel    one CTA per work item (prefill_plan): a (128-row query
//                 tile, query head) over all its key tiles, or, for the
//                 heaviest query tiles, over one of two key ranges. With
//                 3 waves of 148 CTAs the last wave's few CTAs set the time;
//                 splitting the longest tiles and ordering the items by a
//                 replay of the in-order CTA dispatch levels the SMs' ends.
//     warps 0-3   softmax: thread t owns query row t. Prologue: RoPE of its q
//                 row, scale by log2(e)/sqrt(d), hi/mid split into tensor
//                 memory (the A operand of S = Q K^T). Per key tile: S row
//                 from tensor memory, causal mask, online softmax with a
//                 lazily moved reference maximum (O in tensor memory is
//                 rescaled only when a score exceeds the reference by 2^8),
//                 P hi/mid written over the tile's S (the A operand of
//                 O += P V). Epilogue: O / l to global memory; a split half
//                 writes O / l and its log-sum-exp to its slot, and the
//                 second half to finish (an atomic count per slot) merges
//                 both into the output.
//     warp 4      producer: the operand chunks of every MMA group, in the
//                 order the MMAs consume them, into a three-stage ring of
//                 bulk copies completing on mbarriers.
//     warp 5      allocates tensor memory; one lane issues the MMAs in the
//                 order S_0, S_1, O+=P_0V_0, S_2, O+=P_1V_1, S_3, ...:
//                 S_j = Q K_j^T (128 x 128) into buffer j % 2, O += P_j V_j
//                 (128 x d). Two tcgen05.commits per tile carry every
//                 completion (softmax, ring stages, buffer reuse).
//   Tensor memory (512 columns): Q hi/mid, S/P buffers 0 and 1, O.
//   MMA issue is the limit of this kernel, so the design keeps the MMA
//   thread's work minimal: 48 MMAs of N = 128 per 128 keys and two wait
//   points (its first mbarrier access after a burst of MMAs waits for the
//   burst to leave the issue queue, so every such access costs pipe time).
// Every mbarrier wait is bounded (2 s), after which the CTA records an error
// and drains out; tensor memory is always released.

#include "attn.cuh"
#include "common.cuh"

#include <cuda_bf16.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <functional>
#include <vector>

namespace kore {
namespace {

constexpr int kRows = 128;        // query rows per CTA (TMEM lanes)
constexpr int kKeys = 128;        // keys per tile
constexpr int kStages = 3;        // operand ring stages (one MMA group each)
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
// 1024 bytes apart (stride byte offset), Blackwell descriptor version 1. The
// start address is its low 14 bits (address / 16), so adding offset / 16 to
// a descriptor moves its start within shared memory.
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
    static constexpr int QATOMS = D / 64;                       // 64-element K atoms of d
    static constexpr uint32_t KCH = (uint32_t)kKeys * 128 * 2;   // K chunk: [128 keys][64 d] hi, then mid
    static constexpr uint32_t VCH = (uint32_t)D * 128 * 2;       // V^T chunk: [d][64 keys] hi, then mid
    static constexpr uint32_t K_BYTES = QATOMS * KCH;            // all K chunks of a tile
    static constexpr uint32_t V_BYTES = 2 * VCH;                 // both V^T chunks of a tile
    static constexpr uint32_t TILE = K_BYTES + V_BYTES;          // one global tile
    static constexpr uint32_t STAGE = K_BYTES > V_BYTES ? K_BYTES : V_BYTES;
    static constexpr uint32_t ring_off = 0;
    static constexpr uint32_t bar_off = ring_off + kStages * STAGE;
    // barriers, TMEM base, alignment slack; at least 116 KB so that one CTA
    // holds an SM (a second would only wait in tcgen05.alloc for the 512
    // tensor-memory columns the first holds)
    static constexpr uint32_t bytes = bar_off + 512 + 1024 > 116u * 1024 ? bar_off + 512 + 1024 : 116u * 1024;
    // tensor memory columns: Q hi/mid (bf16 pairs), two S buffers (fp32; a
    // tile's P hi/mid, bf16 pairs, overwrite its S), O
    static constexpr uint32_t T_Q = 0, T_S = 128, T_O = 384;
    static constexpr uint32_t TMEM_COLS = 512;
};

// ---------------------------------------------------------------- tcgen05 helpers

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

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

__device__ __forceinline__ void tc_st16u(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
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

// Packed fp32 pairs (Blackwell's two-lane fp32 add/sub/mul: each lane rounds
// as the scalar instruction does) and a three-input max, to cut the softmax's
// instruction count.
__device__ __forceinline__ unsigned long long pk2(float a, float b) {
    unsigned long long u;
    asm("mov.b64 %0, {%1, %2};" : "=l"(u) : "f"(a), "f"(b));
    return u;
}
__device__ __forceinline__ void upk2(unsigned long long u, float &a, float &b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(u));
}
__device__ __forceinline__ unsigned long long sub2(unsigned long long a, unsigned long long b) {
    unsigned long long r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ unsigned long long add2(unsigned long long a, unsigned long long b) {
    unsigned long long r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ unsigned long long mul2(unsigned long long a, unsigned long long b) {
    unsigned long long r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// split2 with the residual formed by one packed subtraction (the bf16 -> fp32
// widening of hi is exact: its 16 bits moved to the top half)
__device__ __forceinline__ void split2p(float x0, float x1, uint32_t &hi, uint32_t &mid) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(x0, x1);
    const uint32_t ab = *reinterpret_cast<const uint32_t *>(&a);
    float r0, r1;
    upk2(sub2(pk2(x0, x1), pk2(__uint_as_float(ab << 16), __uint_as_float(ab & 0xFFFF0000u))), r0, r1);
    const __nv_bfloat162 b = __floats2bfloat162_rn(r0, r1);
    hi = ab;
    mid = *reinterpret_cast<const uint32_t *>(&b);
}

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

// One CTA per (128-key tile, KV head, half of the tile's keys): gathers 64
// keys' K and V rows from the paged pool and writes their part of the tile's
// operand images at split + (g * tiles + j) * TILE: rows 64*half.. of every K
// chunk, and V^T chunk `half`.
template <int D>
__global__ void __launch_bounds__(256) kv_split_kernel(const __grid_constant__ PrefillParams p) {
    using SM = PrefillSmem<D>;
    constexpr int HK = kKeys / 2;   // keys per CTA
    __shared__ float vs[HK][D + 1];
    const int j = blockIdx.x, g = blockIdx.y, half = blockIdx.z, tid = threadIdx.x;
    const PagedKv &kv = p.kv;
    const int n_keys = p.pos0 + p.n;
    const int *pt = kv.page_table + (size_t)p.seq * kv.pt_stride;
    uint8_t *tile = reinterpret_cast<uint8_t *>(p.split) + ((size_t)g * p.tiles + j) * SM::TILE;
    constexpr int CH = D / 8;   // 16-byte bf16 chunks per K row
    // K: row = key, 8 d values per 16-byte chunk; V rows staged in shared memory
    for (int w = tid; w < HK * CH; w += blockDim.x) {
        const int rl = w / CH, c = w - rl * CH;
        const int r = half * HK + rl;   // row within the tile
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
        for (int i = 0; i < 8; ++i) vs[rl][c * 8 + i] = y[i];
        uint4 hi, mid;
        split8(x, hi, mid);
        const uint32_t off = (uint32_t)(c >> 3) * SM::KCH + sw128(r, c & 7);
        *reinterpret_cast<uint4 *>(tile + off) = hi;
        *reinterpret_cast<uint4 *>(tile + off + SM::KCH / 2) = mid;
    }
    __syncthreads();
    // V^T chunk `half`: row = d, 8 keys per 16-byte chunk
    uint8_t *vch = tile + SM::K_BYTES + half * SM::VCH;
    for (int w = tid; w < D * 8; w += blockDim.x) {
        const int r = w >> 3, c = w & 7;
        float x[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = vs[c * 8 + i][r];
        uint4 hi, mid;
        split8(x, hi, mid);
        const uint32_t off = sw128(r, c);
        *reinterpret_cast<uint4 *>(vch + off) = hi;
        *reinterpret_cast<uint4 *>(vch + SM::VCH / 2 + off) = mid;
    }
}

// ---------------------------------------------------------------- attention

template <int D>
__global__ void __launch_bounds__(192, 1) prefill_kernel(const __grid_constant__ PrefillParams p) {
    using SM = PrefillSmem<D>;
    constexpr int HALF = D / 2;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(smem);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + SM::bar_off);
    // MMA groups run in the order S_0, S_1, then for j = 0..n_tiles-1:
    // O += P_j V_j, S_{j+2} (while j + 2 < n_tiles); group i's operands sit in
    // ring stage i % 3. Two commits per tile carry every completion:
    //   s_full[j % 2]   after S_j: the softmax may read S_j; its ring stage
    //                   is free;
    //   pv_done[j % 2]  after O += P_j V_j: S buffer j % 2 may take S_{j+2},
    //                   O holds every tile up to j; its ring stage is free.
    // A parity wait is exact only within one phase of the barrier's count.
    // Each wait below is: its waiter has already seen (or ordered after)
    // the completion two uses earlier on the same barrier, and the one two
    // uses later needs something the waiter has not done yet (the next
    // stage's operands, the next P, or the next S it issues itself).
    uint64_t *full = bars;              // [3] producer -> MMA: a group's operands landed
    uint64_t *s_full = bars + 3;        // [2]
    uint64_t *pv_done = bars + 5;       // [2]
    uint64_t *p_full = bars + 7;        // [2] softmax (4 warps) -> MMA: P_j written
    uint64_t *q_ready = bars + 9;       // softmax (4 warps) -> MMA
    uint64_t *mma_drained = bars + 10;  // MMA commit -> MMA issuer, before TMEM is freed
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 11);
    int *abort_flag = reinterpret_cast<int *>(bars + 12);
    int *arrival = reinterpret_cast<int *>(bars + 13);   // split halves: 1 for the second to finish

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // work item (prefill_plan): query head, query tile, key tiles [t0, t1),
    // and for a query tile split in two key ranges its slot and half
    const int4 item = p.items[blockIdx.x];
    const int h = item.x, qt = item.y;
    const int t0 = item.z & 0xFFFF, t1 = (int)((unsigned)item.z >> 16);
    const int slot = item.w < 0 ? -1 : item.w >> 1, part = item.w & 1;
    const int g = h / p.n_rep;
    const int z0 = qt * kRows;
    const int rows = min(kRows, p.n - z0);
    const int n_tiles = t1 - t0;                                 // key tiles of this CTA
    const int first_masked = (p.pos0 + z0) / kKeys;              // tiles from here need the mask

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) mbar_init(&full[i], 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&pv_done[i], 1);
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
    const uint32_t t_q = tmem + SM::T_Q, t_o = tmem + SM::T_O;   // S buffer b at tmem + T_S + 128 * b

    // a completed phase costs one try_wait; the abort flag is read only on
    // the slow path
    auto bounded_wait = [&](uint64_t *bar, uint32_t parity) -> bool {
        if (mbar_try_wait(bar, parity)) return true;
        if (*reinterpret_cast<volatile int *>(abort_flag)) return false;
        if (mbar_wait(bar, parity, p.err, DEV_WAIT_FULL_TIMEOUT)) return true;
        *reinterpret_cast<volatile int *>(abort_flag) = 1;
        return false;
    };

    if (warp == 4) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const uint8_t *src0 = reinterpret_cast<const uint8_t *>(p.split) + (size_t)g * p.tiles * SM::TILE;
            int gi = 0;
            int h0 = 0, h1 = 0, h2 = 0;   // the last three groups, as 2 * tile + (1 for S, 0 for O)
            auto load = [&](bool is_s, int j) -> bool {
                const int st = gi % kStages;
                if (gi >= kStages) {   // the group that used this stage is done
                    const int jj = h0 >> 1;
                    uint64_t *bar = (h0 & 1) ? &s_full[jj & 1] : &pv_done[jj & 1];
                    if (!bounded_wait(bar, (jj >> 1) & 1)) return false;
                }
                h0 = h1;
                h1 = h2;
                h2 = 2 * j + (is_s ? 1 : 0);
                const uint32_t bytes = is_s ? SM::K_BYTES : SM::V_BYTES;
                uint8_t *dst = smem + SM::ring_off + st * SM::STAGE;
                const uint8_t *src = src0 + (size_t)(t0 + j) * SM::TILE + (is_s ? 0 : SM::K_BYTES);
                mbar_arrive_expect_tx(&full[st], bytes);
                for (uint32_t o = 0; o < bytes; o += 16384)   // kept in L2: every query tile and head reads it
                    bulk_g2s_plain(dst + o, src + o, 16384, &full[st]);
                ++gi;
                return true;
            };
            bool ok = load(true, 0) && (n_tiles < 2 || load(true, 1));
            for (int j = 0; ok && j < n_tiles; ++j) ok = load(false, j) && (j + 2 >= n_tiles || load(true, j + 2));
        }
    } else if (warp == 5) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t ID_S = idesc_bf16(kRows, kKeys), ID_O = idesc_bf16(kRows, D);
            int gi = 0;
            auto wait_full = [&]() { return bounded_wait(&full[gi % kStages], (gi / kStages) & 1); };
            auto issue_s = [&](int j) {   // S_j = Q K_j^T into buffer j % 2
                const uint64_t kd = sdesc(sbase + SM::ring_off + (gi % kStages) * SM::STAGE);
                const uint32_t ts = tmem + SM::T_S + 128 * (j & 1);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    constexpr uint32_t MID = SM::KCH / 2 / 16;
                    const uint32_t o = ((kk >> 2) * SM::KCH + (kk & 3) * 32) / 16;
                    tc_mma_ts(ts, t_q + kk * 8, kd + o, ID_S, kk > 0);                 // hi*hi
                    tc_mma_ts(ts, t_q + kk * 8, kd + o + MID, ID_S, 1);                // hi*mid
                    tc_mma_ts(ts, t_q + HALF + kk * 8, kd + o, ID_S, 1);               // mid*hi
                }
                tc_commit(&s_full[j & 1]);
                ++gi;
            };
            auto issue_pv = [&](int j) {   // O += P_j V_j, P_j in buffer j % 2
                const uint64_t vd = sdesc(sbase + SM::ring_off + (gi % kStages) * SM::STAGE);
                // P of keys 16kk..16kk+15: hi in columns 16kk..+7, mid in 16kk+8..+15
                const uint32_t tp = tmem + SM::T_S + 128 * (j & 1);
#pragma unroll
                for (int kk = 0; kk < kKeys / 16; ++kk) {
                    constexpr uint32_t MID = SM::VCH / 2 / 16;
                    const uint32_t o = ((kk >> 2) * SM::VCH + (kk & 3) * 32) / 16;
                    tc_mma_ts(t_o, tp + 16 * kk, vd + o, ID_O, (j > 0 || kk > 0));    // hi*hi
                    tc_mma_ts(t_o, tp + 16 * kk, vd + o + MID, ID_O, 1);               // hi*mid
                    tc_mma_ts(t_o, tp + 16 * kk + 8, vd + o, ID_O, 1);                 // mid*hi
                }
                tc_commit(&pv_done[j & 1]);
                ++gi;
            };
            bool ok = bounded_wait(q_ready, 0) && wait_full();
            if (ok) {
                tc_fence_after();
                issue_s(0);
            }
            if (ok && n_tiles > 1) {
                ok = wait_full();
                if (ok) issue_s(1);
            }
            for (int j = 0; ok && j < n_tiles; ++j) {
                ok = bounded_wait(&p_full[j & 1], (j >> 1) & 1) && wait_full();
                if (!ok) break;
                tc_fence_after();
                issue_pv(j);
                if (j + 2 < n_tiles) {
                    // buffer j % 2 takes S_{j+2} only once O += P_j V_j has read it
                    ok = bounded_wait(&pv_done[j & 1], (j >> 1) & 1) && wait_full();
                    if (!ok) break;
                    tc_fence_after();
                    issue_s(j + 2);
                }
            }
            // tensor memory is released below only after every MMA issued here is done
            tc_commit(mma_drained);
            mbar_wait(mma_drained, 0, p.err, DEV_WAIT_FULL_TIMEOUT);
        }
    } else if (warp < 4) {
        // ------------------------------------------------------------ softmax (warps 0-3)
        const int t = threadIdx.x;                  // query row, TMEM lane
        const int z = z0 + t;
        const bool valid = t < rows;
        const int lim = p.pos0 + z;                 // last key this row attends to
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        // Q row: RoPE at its position, scale, hi/mid split into tensor memory.
        // In phases of (up to) 32 rotation pairs, each issuing all its 16-byte
        // loads (the pair's q elements and the (cos, sin) table entries) before
        // using any, so that the row costs one memory round trip per phase
        {
            constexpr int PH = HALF < 32 ? HALF : 32;
            const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 *q4 = reinterpret_cast<const float4 *>(p.q + ((size_t)z * p.H + h) * D);
            const float4 *cs4 = reinterpret_cast<const float4 *>(p.rope + (size_t)(valid ? lim : 0) * HALF);
#pragma unroll
            for (int ph = 0; ph < HALF / PH; ++ph) {
                const int e0 = ph * PH;
                float4 a[PH / 4], b[PH / 4], c[PH / 2];   // q[e0..], q[HALF+e0..], (cos, sin) x2
#pragma unroll
                for (int i = 0; i < PH / 4; ++i) {
                    a[i] = valid ? __ldg(q4 + e0 / 4 + i) : zero;
                    b[i] = valid ? __ldg(q4 + (HALF + e0) / 4 + i) : zero;
                }
#pragma unroll
                for (int i = 0; i < PH / 2; ++i) c[i] = __ldg(cs4 + e0 / 2 + i);
                float lo[PH], hi[PH];
#pragma unroll
                for (int i = 0; i < PH; ++i) {
                    const float4 &qa = a[i / 4], &qb = b[i / 4], &cc = c[i / 2];
                    const float x0 = (i & 3) == 0 ? qa.x : (i & 3) == 1 ? qa.y : (i & 3) == 2 ? qa.z : qa.w;
                    const float x1 = (i & 3) == 0 ? qb.x : (i & 3) == 1 ? qb.y : (i & 3) == 2 ? qb.z : qb.w;
                    const float co = (i & 1) ? cc.z : cc.x, si = (i & 1) ? cc.w : cc.y;
                    lo[i] = rope_lo(x0, x1, co, si) * p.scale_log2;
                    hi[i] = rope_hi(x0, x1, co, si) * p.scale_log2;
                }
                // column k of Q hi (mid: + HALF) holds elements 2k, 2k+1
                uint32_t wh[PH / 2], wm[PH / 2];
#pragma unroll
                for (int i = 0; i < PH / 2; ++i) split2(lo[2 * i], lo[2 * i + 1], wh[i], wm[i]);
                tc_st16u(t_q + lane_off + e0 / 2, wh);
                tc_st16u(t_q + lane_off + HALF + e0 / 2, wm);
#pragma unroll
                for (int i = 0; i < PH / 2; ++i) split2(hi[2 * i], hi[2 * i + 1], wh[i], wm[i]);
                tc_st16u(t_q + lane_off + (HALF + e0) / 2, wh);
                tc_st16u(t_q + lane_off + HALF + (HALF + e0) / 2, wm);
            }
            tc_wait_st();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(q_ready);

        // causal mask of 64 scores of keys key0..key0+63
        auto mask64 = [&](float (&v)[64], int key0) {
#pragma unroll
            for (int i = 0; i < 64; ++i)
                if (key0 + i > lim) v[i] = -INFINITY;
        };
        auto max64 = [](const float (&v)[64]) {   // 8 independent chains of three-input maxima
            float m8[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) m8[c] = v[c];
#pragma unroll
            for (int i = 8; i < 64; i += 2) m8[(i >> 1) & 7] = max3(m8[(i >> 1) & 7], v[i], v[i + 1]);
            return max3(max3(m8[0], m8[1], m8[2]), max3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
        };
        // P of 64 keys from their scores, written over them: for each 16 keys,
        // 8 columns of hi pairs then 8 of mid pairs; returns the sum of P
        auto p64 = [&](float (&v)[64], uint32_t col, float m) {
            // sums in 8 chains (keys = c mod 8), as pairs: acc[j] holds chains 2j, 2j+1
            const unsigned long long mm = pk2(m, m);
            unsigned long long acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                float a0, a1;
                upk2(sub2(pk2(v[2 * i], v[2 * i + 1]), mm), a0, a1);
                v[2 * i] = fast_exp2(a0);
                v[2 * i + 1] = fast_exp2(a1);
                acc[i & 3] = add2(acc[i & 3], pk2(v[2 * i], v[2 * i + 1]));
            }
            float l8[8];
#pragma unroll
            for (int j = 0; j < 4; ++j) upk2(acc[j], l8[2 * j], l8[2 * j + 1]);
#pragma unroll
            for (int s = 0; s < 2; ++s) {
                uint32_t w[32];
#pragma unroll
                for (int gq = 0; gq < 2; ++gq)
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int k = 32 * s + 16 * gq + 2 * i;
                        split2p(v[k], v[k + 1], w[16 * gq + i], w[16 * gq + 8 + i]);
                    }
                tc_st32u(col + 32 * s, w);
            }
            return ((l8[0] + l8[1]) + (l8[2] + l8[3])) + ((l8[4] + l8[5]) + (l8[6] + l8[7]));
        };

        float m_ref = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < n_tiles; ++j) {
            const int b = j & 1;
            const uint32_t ts = tmem + SM::T_S + 128 * b + lane_off;
            if (!bounded_wait(&s_full[b], (j >> 1) & 1)) { ok = false; break; }
            tc_fence_after();
            const bool masked = t0 + j >= first_masked;
            const int key0 = (t0 + j) * kKeys;
            float sv[64];
            // pass 1: the row maximum over keys 0-63 (scores dropped) and
            // 64-127 (kept for pass 2)
            tc_ld32(ts, *reinterpret_cast<float(*)[32]>(sv));
            tc_ld32(ts + 32, *reinterpret_cast<float(*)[32]>(sv + 32));
            tc_wait_ld();
            if (masked) mask64(sv, key0);
            float mx = max64(sv);
            tc_ld32(ts + 64, *reinterpret_cast<float(*)[32]>(sv));
            tc_ld32(ts + 96, *reinterpret_cast<float(*)[32]>(sv + 32));
            tc_wait_ld();
            if (masked) mask64(sv, key0 + 64);
            mx = fmaxf(mx, max64(sv));
            const bool need = mx > m_ref + kRescale;
            const bool any_need = __any_sync(FULLMASK, need);
            const float m_new = need ? mx : m_ref;
            // 0 for the first tile, 1 where not needed; a row with no key yet
            // (every key so far masked) keeps 1 and P = 0
            const float alpha = m_new == -INFINITY ? 1.f : fast_exp2(m_ref - m_new);
            const float m_use = m_new == -INFINITY ? 0.f : m_new;
            // pass 2: keys 64-127 from registers, then keys 0-63 again
            float ls = p64(sv, ts + 64, m_use);
            tc_ld32(ts, *reinterpret_cast<float(*)[32]>(sv));
            tc_ld32(ts + 32, *reinterpret_cast<float(*)[32]>(sv + 32));
            tc_wait_ld();
            if (masked) mask64(sv, key0);
            ls += p64(sv, ts, m_use);
            l = fmaf(l, alpha, ls);
            m_ref = m_new;
            // O is stable only once the previous tile's P.V is done
            if (any_need && j > 0) {
                if (!bounded_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1)) { ok = false; break; }
                tc_fence_after();
#pragma unroll
                for (int c0 = 0; c0 < D; c0 += 32) {
                    float o[32];
                    tc_ld32(t_o + lane_off + c0, o);
                    tc_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; i += 2) upk2(mul2(pk2(o[i], o[i + 1]), pk2(alpha, alpha)), o[i], o[i + 1]);
                    tc_st32(t_o + lane_off + c0, o);
                }
            }
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[b]);
        }
        // epilogue: O / l to the output, or for a split query tile to its half's
        // slot, the second half to finish merging both into the output. The
        // split path's barriers are taken by all four softmax warps whatever
        // happened before (a warp whose wait gave up has already raised the
        // error; the results are then not used).
        const bool epi = ok && n_tiles > 0 && bounded_wait(&pv_done[(n_tiles - 1) & 1], ((n_tiles - 1) >> 1) & 1);
        if (epi) tc_fence_after();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        float *dst = p.out + ((size_t)z * p.H + h) * D;
        if (slot < 0) {
            if (epi) {
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
        } else {
            // a half's slot: [kRows][D] outputs normalised by its own sum, then
            // [kRows] log2-domain log-sum-exps
            const float lse = l > 0.f ? m_ref + __log2f(l) : -INFINITY;
            float *mine = p.part + ((size_t)slot * 2 + part) * kRows * (D + 1);
            const float *other = p.part + ((size_t)slot * 2 + (part ^ 1)) * kRows * (D + 1);
            if (epi) {
#pragma unroll
                for (int c0 = 0; c0 < D; c0 += 32) {
                    float o[32];
                    tc_ld32(t_o + lane_off + c0, o);
                    tc_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; i += 4)
                        *reinterpret_cast<float4 *>(mine + (size_t)t * D + c0 + i) =
                            make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv);
                }
                mine[kRows * D + t] = lse;
            }
            __threadfence();
            asm volatile("bar.sync 1, 128;" ::: "memory");   // the four softmax warps
            if (t == 0) *arrival = atomicAdd(p.counters + slot, 1);
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (*reinterpret_cast<volatile int *>(arrival) == 1) {
                __threadfence();
                const float lo = __ldcg(other + kRows * D + t);
                const float M = fmaxf(lse, lo);
                const float wm = M == -INFINITY ? 0.f : fast_exp2(lse - M);
                const float wo = M == -INFINITY ? 0.f : fast_exp2(lo - M);
                const float inv2 = wm + wo > 0.f ? 1.f / (wm + wo) : 0.f;
#pragma unroll
                for (int c0 = 0; c0 < D; c0 += 32) {
                    float o[32];
                    tc_ld32(t_o + lane_off + c0, o);
                    tc_wait_ld();
                    if (valid) {
#pragma unroll
                        for (int i = 0; i < 32; i += 4) {
                            const float4 x = __ldcg(reinterpret_cast<const float4 *>(other + (size_t)t * D + c0 + i));
                            *reinterpret_cast<float4 *>(dst + c0 + i) = make_float4(
                                (wm * o[i] * inv + wo * x.x) * inv2, (wm * o[i + 1] * inv + wo * x.y) * inv2,
                                (wm * o[i + 2] * inv + wo * x.z) * inv2, (wm * o[i + 3] * inv + wo * x.w) * inv2);
                        }
                    }
                }
                if (t == 0) p.counters[slot] = 0;   // ready for the next call
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
    kv_split_kernel<D><<<dim3(tiles_needed, p.kv.G, 2), 256, 0, s>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    e = ensure_smem_limit(reinterpret_cast<const void *>(prefill_kernel<D>), (int)SM::bytes);
    if (e != cudaSuccess) return e;
    if (p.n_items <= 0 || !p.items) return cudaErrorInvalidValue;
    prefill_kernel<D><<<dim3(p.n_items), 192, SM::bytes, s>>>(p);
    return cudaGetLastError();
}

}  // namespace

int prefill_plan(int pos0, int n, int H, int num_sms, std::vector<int4> &items) {
    const int q_tiles = (n + kRows - 1) / kRows;
    std::vector<int> nt(q_tiles), fm(q_tiles);
    int max_nt = 0;
    for (int qt = 0; qt < q_tiles; ++qt) {
        const int z0 = qt * kRows, rows = std::min(kRows, n - z0);
        nt[qt] = (pos0 + z0 + rows - 1) / kKeys + 1;
        fm[qt] = (pos0 + z0) / kKeys;   // keys below this tile are unmasked for every row
        max_nt = std::max(max_nt, nt[qt]);
    }
    struct Work {
        int h, qt, t0, t1, split;
    };
    // A query tile with at least `thr` key tiles is split at its middle, but
    // no later than its first masked tile: the first half is then unmasked
    // and every row has keys in the second.
    auto build = [&](int thr, std::vector<Work> &w) {
        w.clear();
        int slots = 0;
        for (int h = 0; h < H; ++h)
            for (int qt = q_tiles - 1; qt >= 0; --qt) {
                const int mid = std::min(nt[qt] / 2, fm[qt]);
                if (nt[qt] >= thr && mid >= 4 && nt[qt] - mid >= 4) {
                    w.push_back({h, qt, 0, mid, 2 * slots});
                    w.push_back({h, qt, mid, nt[qt], 2 * slots + 1});
                    ++slots;
                } else {
                    w.push_back({h, qt, 0, nt[qt], -1});
                }
            }
        return slots;
    };
    // completion time of the work in launch order, each SM taking the next
    // CTA when it frees, a CTA costing its key tiles plus a start-up cost
    const long long ovh = 4;
    std::vector<long long> sm;
    auto makespan = [&](const std::vector<Work> &w) {
        sm.assign((size_t)std::max(1, num_sms), 0);
        std::make_heap(sm.begin(), sm.end(), std::greater<long long>());
        long long end = 0;
        for (const Work &x : w) {
            std::pop_heap(sm.begin(), sm.end(), std::greater<long long>());
            sm.back() += ovh + (x.t1 - x.t0);
            end = std::max(end, sm.back());
            std::push_heap(sm.begin(), sm.end(), std::greater<long long>());
        }
        return end;
    };
    std::vector<Work> best, w;
    long long best_t = -1;
    for (const double f : {2.0, 1.0, 0.95, 0.9, 0.85, 0.8, 0.7}) {
        const int thr = f > 1.5 ? INT_MAX : (int)std::ceil(f * max_nt);
        build(thr, w);
        for (int order = 0; order < 2; ++order) {
            if (order == 1)   // heaviest first over all heads (the build order is per head)
                std::stable_sort(w.begin(), w.end(),
                                 [](const Work &a, const Work &b) { return a.t1 - a.t0 > b.t1 - b.t0; });
            const long long t = makespan(w);
            if (best_t < 0 || t < best_t) {
                best_t = t;
                best = w;
            }
        }
    }
    items.clear();
    int slots = 0;
    for (const Work &x : best) {
        items.push_back(make_int4(x.h, x.qt, x.t0 | (x.t1 << 16), x.split));
        if (x.split >= 0) slots = std::max(slots, x.split / 2 + 1);
    }
    return slots;
}

size_t prefill_slot_bytes(int head_dim) { return (size_t)2 * kRows * (head_dim + 1) * sizeof(float); }

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
