// proj.cu — kore's quantised projections on the GPU: Q8_K quantisation of an
// activation vector and the Q4_K / Q6_K matrix-vector products, sm_100a.
//
// Replaces mv() + quant() of kore's decode step (kore.cpp:1388-1394) for the
// attention block's projections (kore.cpp:1418-1423 q/k/v + bias, :1456-1457
// Wo): out[r] = row r of W . quantize_q8_K(x) (+ bias[r]).
//
// Exactness. The Q8_K quantisation (kore.cpp:422-447) is reproduced bit for
// bit: the first value of largest magnitude, an IEEE division for the scale,
// round-half-even, the same clamp. The dot products follow kore's AVX2
// kernels (kore.cpp:540-640; kore selects them on every AVX2/FMA CPU) lane by
// lane: per 256-value block, eight int32 lanes (lane k: bytes 4k..4k+3 of
// every 32-value group, weighted by its sub-block scale) and, for Q4_K, four
// lanes of minimum terms (for Q6_K one scalar term for the -32 offset), are
// exact integers; each lane then accumulates d * lane in block order with one
// fused multiply-add, and the lanes are summed in kore's horizontal-sum order.
// Every float operation below is an explicit round-to-nearest intrinsic, so
// the compiler fuses nothing that kore does not. Results equal kore's bit for
// bit; tests/test_proj_gpu.py checks it against the oracle, which is pinned
// to the reference's compiled kernels.
//
// Data path. Weights stay in HBM in the GGUF block layout (Q4_K: 144-byte
// blocks, Q6_K: 210-byte blocks, row-major). One CTA of 16 warps per SM; a
// warp takes 2 consecutive rows at a time, 16 lanes per row: lane (h, k)
// computes AVX2 lane k over half h of the row's blocks, and the second
// half's lane continues the first half's fused multiply-add chains (one
// shuffle), so the float order stays kore's. The 2 rows are one contiguous
// byte range: one bulk copy per warp stages them in shared memory, issued
// before the kernel waits for its predecessor (programmatic dependent
// launch), since weights do not depend on it. Meanwhile every CTA quantises
// the fp32 input vector to Q8_K in shared memory itself (14 KB at 7B: cheaper
// than a kernel boundary), transposed so that each lane reads its 8 words of
// a block with two 16-byte loads on distinct banks. The per-block loop is
// compact, which keeps this short-lived kernel out of instruction-cache
// misses. Memory-bound: algorithmic bytes = the weight bytes (+ the small
// vector), read once.

#include "attn.cuh"
#include "common.cuh"

#include <cuda_fp16.h>

namespace kore {
namespace {

constexpr int kWarps = 16;   // warps per CTA (one CTA per SM)

__device__ __forceinline__ float half_bits(uint32_t h) { return __half2float(__ushort_as_half((unsigned short)h)); }

// ---------------------------------------------------------------- Q8_K

// Staged Q8_K block in shared memory, transposed for the product lanes:
// AVX2 lane k of either format reads the 8 words k, k+8, ..., k+56 of the
// block's 64 qs words (Q4_K: lo/hi of each 64-value chunk; Q6_K: the four
// 32-value groups of each half), in that order. They are stored at
// [k][0..7] with a 48-byte row so that the 8 lanes' 16-byte reads fall on
// distinct banks.
constexpr int kQ8Row = 48;
constexpr int kQ8Block = 8 * kQ8Row;   // 384 bytes

// One warp quantises one 256-value block of x (lane l: values 8l..8l+7) into
// a staged Q8_K block: transposed qs, its scale, its 16 group sums and the 8
// sums of adjacent group pairs.
__device__ __forceinline__ void q8k_block(const float *__restrict__ x, int lane, uint8_t *qt, float *xd,
                                          int16_t *bsums, int16_t *pairs) {
    const float4 *src = reinterpret_cast<const float4 *>(x + 8 * lane);
    const float4 a = src[0], b = src[1];
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    // the first value of largest magnitude (strict >, in index order)
    float amax = 0.f, maxv = 0.f;
    int idx = 1 << 30;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float ax = fabsf(v[i]);
        if (ax > amax) {
            amax = ax;
            maxv = v[i];
            idx = 8 * lane + i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float am = __shfl_xor_sync(0xffffffffu, amax, o);
        const float mv = __shfl_xor_sync(0xffffffffu, maxv, o);
        const int ix = __shfl_xor_sync(0xffffffffu, idx, o);
        if (am > amax || (am == amax && ix < idx)) {
            amax = am;
            maxv = mv;
            idx = ix;
        }
    }
    int q[8];
    float d = 0.f;
    if (amax == 0.f) {
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = 0;
    } else {
        const float iscale = __fdiv_rn(-127.0f, maxv);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int t = __float2int_rn(__fmul_rn(iscale, v[i]));   // round half to even
            q[i] = t > 127 ? 127 : t;
        }
        d = __fdiv_rn(1.0f, iscale);
    }
    int s = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += q[i];
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    const uint32_t w0 = (uint32_t)(q[0] & 0xFF) | (uint32_t)(q[1] & 0xFF) << 8 | (uint32_t)(q[2] & 0xFF) << 16 |
                        (uint32_t)(q[3] & 0xFF) << 24;
    const uint32_t w1 = (uint32_t)(q[4] & 0xFF) | (uint32_t)(q[5] & 0xFF) << 8 | (uint32_t)(q[6] & 0xFF) << 16 |
                        (uint32_t)(q[7] & 0xFF) << 24;
    // words 2l and 2l+1: word w goes to row w % 8, column w / 8
    const int wa = 2 * lane, wb = 2 * lane + 1;
    *reinterpret_cast<uint32_t *>(qt + (wa & 7) * kQ8Row + 4 * (wa >> 3)) = w0;
    *reinterpret_cast<uint32_t *>(qt + (wb & 7) * kQ8Row + 4 * (wb >> 3)) = w1;
    if ((lane & 1) == 0) bsums[lane >> 1] = (int16_t)s;
    // bsums[2j] + bsums[2j+1] as int16 (the Q4_K minimum terms' operands, kore.cpp:563-567)
    const int s2 = (int)(int16_t)s + (int)(int16_t)__shfl_xor_sync(0xffffffffu, s, 2);
    if ((lane & 3) == 0) pairs[lane >> 2] = (int16_t)s2;
    if (lane == 0) *xd = d;
}

// ---------------------------------------------------------------- products

// A lane's weight words of one block (kW words, the larger format's count).
// Q4_K: w[0..3] the 4 nibble words of its byte column (bytes 4k..4k+3 of
// each 32-byte group), w[4..7] the header (d, dmin, 12 scale bytes). Q6_K:
// w[0..5] its ql / qh words in both halves, w[6..9] the 16 scale bytes,
// w[10] d.
constexpr int kW = 11;

__device__ __forceinline__ uint32_t lds_u32(const uint8_t *p) { return *reinterpret_cast<const uint32_t *>(p); }

// 32-bit word at a 2-byte aligned shared-memory address: two aligned loads
// and a byte permute.
__device__ __forceinline__ uint32_t lds_u32_a2(const uint8_t *p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *b = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    return __byte_perm(b[0], b[1], (a & 2) ? 0x5432 : 0x3210);
}

template <int TYPE>
__device__ __forceinline__ void lds_block(const uint8_t *blk, int k, uint32_t (&w)[kW]) {
    if (TYPE == 12) {
#pragma unroll
        for (int c = 0; c < 4; ++c) w[c] = lds_u32(blk + 16 + 32 * c + 4 * k);
        const uint4 h = *reinterpret_cast<const uint4 *>(blk);
        w[4] = h.x;
        w[5] = h.y;
        w[6] = h.z;
        w[7] = h.w;
    } else {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            w[3 * h + 0] = lds_u32_a2(blk + 64 * h + 4 * k);
            w[3 * h + 1] = lds_u32_a2(blk + 64 * h + 32 + 4 * k);
            w[3 * h + 2] = lds_u32_a2(blk + 128 + 32 * h + 4 * k);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) w[6 + i] = lds_u32_a2(blk + 192 + 4 * i);
        w[10] = lds_u32_a2(blk + 208) & 0xFFFFu;
    }
}

// One block's terms for AVX2 lane k of kore's kernels: the exact integers s
// (the lane) and e (Q4_K: minimum lane k & 3; Q6_K: the -32 offset integer,
// the same on every lane) and the float factors, which the lane's chains
// take in block order as acc += d * s and accm += dm * e.
//  Q4_K (kore.cpp:553-586): s = sum_c sc[2c] * <lo nibbles, q8> +
//   sc[2c+1] * <hi nibbles, q8> over bytes 4k..4k+3 of each 32-byte group;
//   e = mn[2m] * (bs[4m] + bs[4m+1]) + mn[2m+1] * (bs[4m+2] + bs[4m+3]);
//   d = d_w * xd, dm = -(dmin_w * xd).
//  Q6_K (kore.cpp:603-636): s = unsigned 6-bit values times q8 over bytes
//   4k..4k+3 of each 32-value group, weighted by the scale of the 16-value
//   half that holds them; e = sum_j sc[j] * bsums[j]; d = d_w * xd,
//   dm = -(d * 32).
struct Terms {
    int s, e;
    float d, dm;
};

template <int TYPE>
__device__ __forceinline__ Terms block_terms(const uint32_t (&w)[kW], int k, const uint8_t *qt, const int16_t *bs,
                                             const int16_t *pr, float xd) {
    const uint4 qa = *reinterpret_cast<const uint4 *>(qt + k * kQ8Row);
    const uint4 qb = *reinterpret_cast<const uint4 *>(qt + k * kQ8Row + 16);
    const uint32_t q8[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    Terms t;
    if (TYPE == 12) {
        const uint32_t u0 = w[5], u1 = w[6], u2 = w[7];
        const uint32_t sc_lo = u0 & 0x3F3F3F3Fu;                                // scales 0-3
        const uint32_t sc_hi = (u2 & 0x0F0F0F0Fu) | ((u0 >> 2) & 0x30303030u);  // scales 4-7
        int s = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            // sc[2c] * <lo nibbles, q8> + sc[2c+1] * <hi nibbles, q8> in one
            // two-way product of the packed 16-bit partial sums (|.| <= 7620)
            const int lo = __dp4a((int)(w[c] & 0x0F0F0F0Fu), (int)q8[2 * c], 0);
            const int hi = __dp4a((int)((w[c] >> 4) & 0x0F0F0F0Fu), (int)q8[2 * c + 1], 0);
            const int pk = (int)__byte_perm((uint32_t)lo, (uint32_t)hi, 0x5410);
            const uint32_t scw = c < 2 ? sc_lo : sc_hi;
            s = (c & 1) ? __dp2a_hi(pk, (int)scw, s) : __dp2a_lo(pk, (int)scw, s);
        }
        const int m = k & 3;
        const uint32_t mnw = m < 2 ? (u1 & 0x3F3F3F3Fu) : (((u2 >> 4) & 0x0F0F0F0Fu) | ((u1 >> 2) & 0x30303030u));
        // mn[2m] * pairs[2m] + mn[2m+1] * pairs[2m+1]
        t.s = s;
        t.e = __dp2a_lo(*reinterpret_cast<const int *>(pr + 2 * m), (int)(mnw >> (16 * (m & 1))), 0);
        t.d = __fmul_rn(half_bits(w[4] & 0xFFFFu), xd);
        t.dm = -__fmul_rn(half_bits(w[4] >> 16), xd);
    } else {
        const uint32_t o = k >= 4 ? 0x31u : 0x20u;   // this lane's scale of each 32-value group: bytes o, o+2
        int s = 0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t qla = w[3 * h], qlb = w[3 * h + 1], qh = w[3 * h + 2];
            int part[4];
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const uint32_t ql = (kk & 1) ? qlb : qla;
                const uint32_t v = ((ql >> (4 * (kk >> 1))) & 0x0F0F0F0Fu) | (((qh >> (2 * kk)) & 0x03030303u) << 4);
                part[kk] = __dp4a((int)v, (int)q8[4 * h + kk], 0);   // |.| <= 4*63*127 = 32004
            }
            // group kk's scale is sc[8h + 2kk + (k >= 4)]: groups 0, 1 in word 6+2h, 2, 3 in word 7+2h
            const int scA = (int)__byte_perm(w[6 + 2 * h], 0u, o), scB = (int)__byte_perm(w[7 + 2 * h], 0u, o);
            s = __dp2a_lo((int)__byte_perm((uint32_t)part[0], (uint32_t)part[1], 0x5410), scA, s);
            s = __dp2a_lo((int)__byte_perm((uint32_t)part[2], (uint32_t)part[3], 0x5410), scB, s);
        }
        const uint4 ba = *reinterpret_cast<const uint4 *>(bs);
        const uint4 bb = *reinterpret_cast<const uint4 *>(bs + 8);
        const uint32_t bw[8] = {ba.x, ba.y, ba.z, ba.w, bb.x, bb.y, bb.z, bb.w};
        // sum_j sc[j] * bsums[j]: bsums pairs (2i, 2i+1) with scale bytes 2i, 2i+1
        int ib = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i)
            ib = (i & 1) ? __dp2a_hi((int)bw[i], (int)w[6 + (i >> 1)], ib) : __dp2a_lo((int)bw[i], (int)w[6 + (i >> 1)], ib);
        t.s = s;
        t.e = ib;
        t.d = __fmul_rn(half_bits(w[10]), xd);
        t.dm = -__fmul_rn(t.d, 32.0f);
    }
    return t;
}

__device__ __forceinline__ void take(const Terms &t, float &acc, float &accm) {
    acc = __fmaf_rn(t.d, __int2float_rn(t.s), acc);
    accm = __fmaf_rn(t.dm, __int2float_rn(t.e), accm);
}

// The row's dot product from its lanes' chains: kore's horizontal sums over
// the row's 8 lanes, ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)), plus for Q4_K
// ((m0+m2)+(m1+m3)), for Q6_K the offset sum. Valid on lane 0 of the group.
template <int TYPE>
__device__ __forceinline__ float row_sum(float acc, float accm) {
    const float t4 = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4, 8));
    const float t2 = __fadd_rn(t4, __shfl_down_sync(0xffffffffu, t4, 2, 8));
    const float a = __fadd_rn(t2, __shfl_down_sync(0xffffffffu, t2, 1, 8));
    float m = accm;
    if (TYPE == 12) {
        const float m2 = __fadd_rn(accm, __shfl_down_sync(0xffffffffu, accm, 2, 8));
        m = __fadd_rn(m2, __shfl_down_sync(0xffffffffu, m2, 1, 8));
    }
    return __fadd_rn(a, m);
}

// The row's product from its staged bytes. Lane (h2, k) computes the terms
// of AVX2 lane k for blocks [h2*hb, min(nb, (h2+1)*hb)); the h2 = 0 lane
// runs the chains over its blocks, the h2 = 1 lane parks its terms in
// `park` and, given the h2 = 0 lane's chains, continues them over its
// blocks: block order, as kore's loop. The result is on the h2 = 1, k = 0
// lane.
template <int TYPE>
__device__ __forceinline__ float row_dot(const uint8_t *row, int nb, int h2, int k, const uint8_t *q8t,
                                         const float *xds, const int16_t *bss, const int16_t *prs, uint4 *park) {
    constexpr int BB = TYPE == 12 ? 144 : 210;
    const int hb = (nb + 1) >> 1, b0 = h2 * hb, b1 = min(nb, b0 + hb);
    float acc = 0.f, accm = 0.f;
#pragma unroll 2
    for (int b = b0; b < b1; ++b) {
        uint32_t w[kW];
        lds_block<TYPE>(row + (size_t)b * BB, k, w);
        const Terms t =
            block_terms<TYPE>(w, k, q8t + (size_t)b * kQ8Block, bss + (size_t)b * 16, prs + (size_t)b * 8, xds[b]);
        if (h2 == 0) take(t, acc, accm);
        else park[b - b0] = make_uint4((uint32_t)t.s, (uint32_t)t.e, __float_as_uint(t.d), __float_as_uint(t.dm));
    }
    const float acc0 = __shfl_xor_sync(0xffffffffu, acc, 8), accm0 = __shfl_xor_sync(0xffffffffu, accm, 8);
    if (h2 == 1) {
        acc = acc0;
        accm = accm0;
        for (int b = b0; b < b1; ++b) {
            const uint4 v = park[b - b0];
            take(Terms{(int)v.x, (int)v.y, __uint_as_float(v.z), __uint_as_float(v.w)}, acc, accm);
        }
    }
    return row_sum<TYPE>(acc, accm);
}

// Global row g of the launch (the segments' rows one after another): its
// segment and row within it.
__device__ __forceinline__ int find_seg(const QMatvecParams &p, int g, int &row) {
    int s = 0;
    row = g;
    while (s + 1 < p.n_seg && row >= p.seg[s].rows) {
        row -= p.seg[s].rows;
        ++s;
    }
    return s;
}

// One CTA per SM, kWarps warps. A warp takes groups of 2 consecutive rows
// (16 lanes per row: lane (h2, k) computes AVX2 lane k over one half of the
// blocks), group warp*grid + cta first and then every TW-th. Every segment's
// row count is even, so a group lies in one segment and its rows are one
// contiguous byte range, which one bulk copy brings into the warp's
// shared-memory slot. The first group's copy is issued before the dependency
// wait (weights do not depend on the preceding kernel).
__global__ void __launch_bounds__(32 * kWarps) qmatvec_kernel(const __grid_constant__ QMatvecParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int nb = p.cols / 256, hb = (nb + 1) >> 1;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);                   // [kWarps]
    uint8_t *q8t = smem + 8 * kWarps;                                     // [nb][kQ8Block]
    float *xds = reinterpret_cast<float *>(q8t + (size_t)nb * kQ8Block);  // [nb]
    int16_t *bss = reinterpret_cast<int16_t *>(xds + ((nb + 3) & ~3));    // [nb][16]
    int16_t *prs = bss + (size_t)nb * 16;                                 // [nb][8]
    uint4 *parks = reinterpret_cast<uint4 *>(prs + (size_t)nb * 8);       // [kWarps][2 rows][8 lanes][hb]
    uint8_t *slots = reinterpret_cast<uint8_t *>(parks + (size_t)kWarps * 16 * hb);   // [kWarps][p.slot_bytes]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rr = lane >> 4, h2 = (lane >> 3) & 1, k = lane & 7;
    uint64_t *bar = bars + warp;
    uint8_t *slot = slots + (size_t)warp * p.slot_bytes;
    uint4 *park = parks + ((size_t)warp * 16 + rr * 8 + k) * hb;
    int R = 0;
    for (int s = 0; s < p.n_seg; ++s) R += p.seg[s].rows;
    const int n_groups = R / 2, TW = (int)gridDim.x * kWarps;
    // groups warp-major over the grid: consecutive groups (and so each
    // matrix's rows, e.g. a Q6_K Wv among Q4_K ones) spread over all SMs
    const int gg0 = warp * (int)gridDim.x + (int)blockIdx.x;
    if (lane == 0) {
        mbar_init(bar, 1);
        mbar_fence_init();
    }
    __syncwarp();
    // the bulk copy of group gg; returns the offset of its first row in the slot
    auto issue = [&](int gg) -> uint32_t {
        int row0;
        const QSeg &sg = p.seg[find_seg(p, 2 * gg, row0)];
        const size_t rb = (size_t)nb * (sg.type == 12 ? 144 : 210);
        const uintptr_t a = reinterpret_cast<uintptr_t>(sg.w + (size_t)row0 * rb);
        const uintptr_t a0 = a & ~uintptr_t(15);
        const uint32_t bytes = (uint32_t)(((a - a0) + 2 * rb + 15) & ~size_t(15));
        if (lane == 0) {
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(bar, bytes);
            bulk_g2s_plain(slot, reinterpret_cast<const void *>(a0), bytes, bar);
        }
        return (uint32_t)(a - a0);
    };
    uint32_t delta = 0, phase = 0;
    if (gg0 < n_groups) delta = issue(gg0);
    grid_dep_wait();
    // x quantised to Q8_K in shared memory, one warp per block
    for (int b = warp; b < nb; b += kWarps)
        q8k_block(p.x + (size_t)b * 256, lane, q8t + (size_t)b * kQ8Block, xds + b, bss + (size_t)b * 16,
                  prs + (size_t)b * 8);
    __syncthreads();
    grid_dep_launch();
    for (int gg = gg0; gg < n_groups; gg += TW) {
        if (gg != gg0) {
            __syncwarp();   // every lane is done with the slot
            delta = issue(gg);
        }
        const bool ok = mbar_wait(bar, phase, p.err, DEV_WAIT_FULL_TIMEOUT);
        if (!__all_sync(0xffffffffu, ok)) {
            mbar_drain(bar, phase);   // the copy may still land: not into a block that has exited
            break;
        }
        phase ^= 1;
        int row;
        const QSeg &sg = p.seg[find_seg(p, 2 * gg + rr, row)];
        float r;
        if (sg.type == 12) r = row_dot<12>(slot + delta + (size_t)rr * nb * 144, nb, h2, k, q8t, xds, bss, prs, park);
        else r = row_dot<14>(slot + delta + (size_t)rr * nb * 210, nb, h2, k, q8t, xds, bss, prs, park);
        if (h2 == 1 && k == 0) {
            if (sg.bias) r = __fadd_rn(r, sg.bias[row]);
            sg.out[row] = r;
        }
    }
}

cudaLaunchAttribute pdl_attr() {
    cudaLaunchAttribute a;
    a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    a.val.programmaticStreamSerializationAllowed = 1;
    return a;
}

}  // namespace

size_t qmatvec_smem_bytes(int cols, int max_block_bytes, int *slot_bytes) {
    const int nb = cols / 256, hb = (nb + 1) / 2;
    // a group's copy starts up to 15 bytes before its first row and ends up to
    // 15 bytes after its last; the Q6_K word reads reach 6 bytes past a block
    const size_t slot = ((size_t)2 * nb * max_block_bytes + 32 + 15) & ~size_t(15);
    if (slot_bytes) *slot_bytes = (int)slot;
    return (size_t)8 * kWarps + (size_t)nb * kQ8Block + (size_t)((nb + 3) & ~3) * 4 + (size_t)nb * 48 +
           (size_t)kWarps * 16 * hb * 16 + (size_t)kWarps * slot;
}

cudaError_t launch_qmatvec(const QMatvecParams &p, int grid, cudaStream_t s) {
    if (p.n_seg <= 0 || p.n_seg > 3 || p.cols <= 0 || p.cols % 256 || !p.x || grid <= 0) return cudaErrorInvalidValue;
    int bb = 0;
    for (int i = 0; i < p.n_seg; ++i) {
        if ((p.seg[i].type != 12 && p.seg[i].type != 14) || p.seg[i].rows < 0 || p.seg[i].rows % 2 || !p.seg[i].w ||
            !p.seg[i].out)
            return cudaErrorInvalidValue;
        bb = max(bb, p.seg[i].type == 12 ? 144 : 210);
    }
    int slot = 0;
    const size_t smem = qmatvec_smem_bytes(p.cols, bb, &slot);
    if (slot != p.slot_bytes || smem > kQmatvecMaxSmem) return cudaErrorInvalidValue;
    if (cudaError_t e = ensure_smem_limit(reinterpret_cast<const void *>(qmatvec_kernel), (int)kQmatvecMaxSmem))
        return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(32 * kWarps);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr = pdl_attr();
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, qmatvec_kernel, p);
}

}  // namespace kore
