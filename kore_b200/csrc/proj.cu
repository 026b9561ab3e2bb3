// proj.cu — kore's quantised products on the GPU: Q8_K quantisation of an
// activation vector and the Q4_K / Q6_K matrix-vector products, sm_100a,
// with the steps of kore's decode step that sit around them fused in.
//
// Replaces mv() + quant() of kore's decode step (kore.cpp:1388-1394):
// out[r] = row r of W . quantize_q8_K(x), for the attention projections
// (kore.cpp:1418-1423 q/k/v + bias, :1456-1457 Wo), the feed-forward
// products (:1462-1471 gate, up, down) and the logits (:1475-1478). What kore
// does next to a product is folded into the same kernel:
//   input   the plain vector, or RMSNorm(x) (kore.cpp:1367-1372) computed from
//           the residual stream by every block itself;
//   output  the row plus its bias; the residual add x[r] += row (kore.cpp:1457,
//           :1471); the SwiGLU of a gate row and the same up row,
//           g / (1 + exp(-g)) * u (kore.cpp:1465-1468); or the logits with
//           their greedy argmax (sample_token at temperature 0,
//           kore.cpp:1601-1603: the first index of the largest value).
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
// the compiler fuses nothing that kore does not.
//  * RMSNorm: kore sums the squares in double, sequentially. Every square of
//    a float is exact in double, so a tree sum differs from kore's sum by at
//    most (n + log2 n) units of 2^-53 of the sum; the block checks that the
//    mean, rounded to float as kore rounds it, cannot change within that
//    bound, and otherwise (about one vector in 10^5) sums sequentially in
//    kore's order. Then (float) mean + eps, sqrtf, 1/x, (x * scale) * w.
//  * SwiGLU: kore's std::exp is the C library's expf, which on glibc (2.27
//    and later) is the table-driven method of ARM's optimized-routines
//    (Szabolcs Nagy): x * 32/ln2 = k + r with the reduced argument formed by
//    one fused multiply-add, 2^(k/32) from a 32-entry table of 2^(i/32), a
//    cubic in r, all in double, one rounding to float at the end. It is
//    restated here (kore_expf) with the table built on the host from exp2;
//    the restatement was checked against the host's expf on all 2^32 floats
//    (identical except NaN payloads).
// Results equal kore's bit for bit; the tests check them against the oracle,
// which is pinned to the reference's compiled code.
//
// Data path. Weights stay in HBM in the GGUF block layout (Q4_K: 144-byte
// blocks, Q6_K: 210-byte blocks, row-major). One CTA of 16 warps per SM. A
// warp takes a group of 2 rows at a time (2 consecutive rows, or row i of
// two matrices for the SwiGLU pair), 16 lanes per row: lane (h, k) computes
// AVX2 lane k over half h of the blocks of each chunk, and the second half's
// lane continues the first half's fused multiply-add chains (one shuffle
// each way per chunk), so the float order stays kore's. Rows are streamed in
// chunks (a whole row of up to 16 blocks, else 8 blocks) through a ring of
// stages per warp (one bulk copy per row and chunk, issued by the row's first
// lane, mbarrier completion), refilled as soon as a chunk has been consumed
// and running on into the warp's next group, so long rows (the 18944-wide
// down projection) fit and every warp keeps several copies in flight. The
// copies are marked first to evict from L2: every weight byte is read once,
// and weights left in L2 at normal priority slowed the decode that follows
// the products by ~5 us per layer. A launch whose matrices share one block
// format runs a kernel compiled for that format alone. The first stages are
// issued before the kernel waits for its predecessor (programmatic dependent
// launch): weights do not depend on it. Meanwhile every CTA builds the Q8_K
// input in shared memory itself (build_q8_input; 14 KB at 7B, 28 KB for the
// feed-forward width: cheaper than a kernel boundary), transposed so that
// each lane reads its 8 words of a block with two 16-byte loads on distinct
// banks. Memory-bound: algorithmic bytes = the weight bytes (+ the small
// vectors), read once.

#include "attn.cuh"
#include "common.cuh"
#include "kore_math.cuh"

#include <cuda_fp16.h>

#include <type_traits>

namespace kore {
namespace {

constexpr int kWarps = 16;   // warps per CTA (one CTA per SM)
constexpr unsigned FULLW = 0xffffffffu;

#ifdef KORE_TRACE
// Trace build: every product CTA stamps (TraceRec::t) entry, dependency wait
// returned, Q8_K input built, warp 0's first weights landed, end (after a
// barrier over the CTA). Kinds: 3 qmatvec_kernel, 4 qmatvec_rows_kernel;
// tag = the first segment's rows, pad2 = cols | out_mode << 32 | n_seg << 40.
KORE_TRACE_BUFFER();
#define KTRACE_PRODUCT(kind) \
    KTRACE_OPEN_TAGGED(kind, (unsigned)p.seg[0].rows, \
                       (unsigned long long)p.cols | (unsigned long long)p.out_mode << 32 | (unsigned long long)p.n_seg << 40)
#define KTRACE_FIRST_LANDED(it) \
    if ((it) == 0) KTRACE(3)
#define KTRACE_END() \
    __syncthreads(); \
    KTRACE(4)
#else
#define KTRACE_PRODUCT(kind)
#define KTRACE_FIRST_LANDED(it)
#define KTRACE_END()
#endif

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

// One warp quantises one 256-value block (lane l holds values 8l..8l+7 in v)
// into a staged Q8_K block: transposed qs, its scale, its 16 group sums and
// the 8 sums of adjacent group pairs.
__device__ __forceinline__ void q8k_block(const float (&v)[8], int lane, uint8_t *qt, float *xd, int16_t *bsums,
                                          int16_t *pairs) {
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
        const float am = __shfl_xor_sync(FULLW, amax, o);
        const float mv = __shfl_xor_sync(FULLW, maxv, o);
        const int ix = __shfl_xor_sync(FULLW, idx, o);
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
    s += __shfl_xor_sync(FULLW, s, 1);
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
    const int s2 = (int)(int16_t)s + (int)(int16_t)__shfl_xor_sync(FULLW, s, 2);
    if ((lane & 3) == 0) pairs[lane >> 2] = (int16_t)s2;
    if (lane == 0) *xd = d;
}

// Orderable key of (value, row) for the greedy argmax: larger value first,
// then smaller row (std::max_element keeps the first of equal maxima; -0
// equals +0 there, so it is keyed as +0).
__device__ __forceinline__ unsigned long long argmax_key(float v, int row) {
    const uint32_t u = __float_as_uint(v == 0.f ? 0.f : v);
    const uint32_t o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)o << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)row);
}

// ---------------------------------------------------------------- products

// A lane's weight words of one block (kW words, the larger format's count).
// Q4_K: w[0..3] the 4 nibble words of its byte column (bytes 4k..4k+3 of
// each 32-byte group), w[4..7] the header (d, dmin, 12 scale bytes). Q6_K:
// w[0..5] its ql / qh words in both halves, w[6..9] the 16 scale bytes,
// w[10] d.
constexpr int kW = 11;

__device__ __forceinline__ uint32_t lds_u32(const uint8_t *p) { return *reinterpret_cast<const uint32_t *>(p); }

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
    } else {   // uploaded Q6_K blocks are 4-byte aligned (kQ6Stride)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            w[3 * h + 0] = lds_u32(blk + 64 * h + 4 * k);
            w[3 * h + 1] = lds_u32(blk + 64 * h + 32 + 4 * k);
            w[3 * h + 2] = lds_u32(blk + 128 + 32 * h + 4 * k);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) w[6 + i] = lds_u32(blk + 192 + 4 * i);   // 4-byte aligned only
        w[10] = lds_u32(blk + 208) & 0xFFFFu;
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
// ((m0+m2)+(m1+m3)), for Q6_K the offset sum. Every lane of the warp runs
// the same shuffles (the two rows of a group may differ in type); valid on
// lane 0 of each 8-lane group.
__device__ __forceinline__ float row_sum(float acc, float accm, bool q4) {
    const float t4 = __fadd_rn(acc, __shfl_down_sync(FULLW, acc, 4, 8));
    const float t2 = __fadd_rn(t4, __shfl_down_sync(FULLW, t4, 2, 8));
    const float a = __fadd_rn(t2, __shfl_down_sync(FULLW, t2, 1, 8));
    const float m2 = __fadd_rn(accm, __shfl_down_sync(FULLW, accm, 2, 8));
    const float m4 = __fadd_rn(m2, __shfl_down_sync(FULLW, m2, 1, 8));
    return __fadd_rn(a, q4 ? m4 : accm);
}

// Row r (0 or 1) of group gg: its segment and row within it, or -1.
__device__ __forceinline__ int group_row(const QMatvecParams &p, int gg, int rr, int total_rows, int &row) {
    if (p.pair_segments) {
        row = gg;
        return rr;
    }
    int g = 2 * gg + rr;
    if (g >= total_rows) return -1;
    int s = 0;
    while (s + 1 < p.n_seg && g >= p.seg[s].rows) {
        g -= p.seg[s].rows;
        ++s;
    }
    row = g;
    return s;
}

// ---------------------------------------------------------------- the Q8_K input

__device__ __forceinline__ void ld8(const float *base, int b, int lane, float (&o)[8]) {
    const float4 *s = reinterpret_cast<const float4 *>(base + (size_t)b * 256 + 8 * lane);
    const float4 a = s[0], c = s[1];
    o[0] = a.x;
    o[1] = a.y;
    o[2] = a.z;
    o[3] = a.w;
    o[4] = c.x;
    o[5] = c.y;
    o[6] = c.z;
    o[7] = c.w;
}

// The RMSNorm weights of a warp's first KW blocks (w, w + NW, ...): loaded
// before the kernel waits for its predecessor (weights do not depend on it).
template <int NW, int KW>
__device__ __forceinline__ void load_norm_first(const QMatvecParams &p, int nb, float (&nw)[KW][8]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int k = 0; k < KW; ++k)
        if (warp + k * NW < nb) ld8(p.norm_w, warp + k * NW, lane, nw[k]);
}

// The product's Q8_K input: x, or RMSNorm(x) * norm_w (kore.cpp:1367-1372),
// handed block by block to quant(b, v) (v: this lane's values 8 lane ..
// 8 lane + 7 of block b). Warp w takes blocks w, w + NW, ...; KB of them at a
// time are loaded before any is used, so their latencies overlap (one or two
// rounds for the inputs of kore's products). The RMSNorm scale: each warp sums
// the squares of its blocks in double, and after one barrier every warp adds
// the warps' partial sums in the same butterfly order, so all form the same
// float; mean_square_float then proves it equal to kore's (sequential sum,
// rounded mean), else (about one vector in 10^5, or always under
// rms_sequential) each warp sums in kore's order. Then (float) mean + eps,
// sqrtf, 1/x, (x * scale) * w, as kore. nw: load_norm_first's registers.
template <int NW, int KB, int KW, class Quant>
__device__ __forceinline__ void build_q8_input(const QMatvecParams &p, int nb, double *red, const float (&nw)[KW][8],
                                               Quant &&quant) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool norm = p.in_mode == QIN_RMSNORM;
    float v[KB][8];
    auto load_x = [&](int b0) {
#pragma unroll
        for (int k = 0; k < KB; ++k)
            if (b0 + k * NW < nb) ld8(p.x, b0 + k * NW, lane, v[k]);
    };
    load_x(warp);
    float scale = 1.f;
    if (norm) {
        double ss = 0.0;
        for (int b0 = warp; b0 < nb; b0 += NW * KB) {
            if (b0 != warp) load_x(b0);
#pragma unroll
            for (int k = 0; k < KB; ++k)
                if (b0 + k * NW < nb)
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const double xi = (double)v[k][i];
                        ss = __dadd_rn(ss, __dmul_rn(xi, xi));
                    }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss = __dadd_rn(ss, __shfl_xor_sync(FULLW, ss, o));
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        double S = lane < NW ? red[lane] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) S = __dadd_rn(S, __shfl_xor_sync(FULLW, S, o));
        float f = p.rms_sequential ? __int_as_float(0x7fffffff) : mean_square_float(S, p.cols);
        if (f != f) {   // too close to a rounding boundary (or not finite): kore's order
            float fs = 0.f;
            if (lane == 0) {
                double seq = 0.0;
                for (int i = 0; i < p.cols; ++i) {
                    const double xi = (double)p.x[i];
                    seq = __dadd_rn(seq, __dmul_rn(xi, xi));
                }
                fs = __double2float_rn(__ddiv_rn(seq, (double)p.cols));
            }
            f = __shfl_sync(FULLW, fs, 0);
        }
        scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(f, p.eps)));
        if (nb > NW * KB) load_x(warp);   // later rounds overwrote the first blocks
    }
    for (int b0 = warp; b0 < nb; b0 += NW * KB) {
        if (b0 != warp) load_x(b0);
#pragma unroll
        for (int k = 0; k < KB; ++k) {
            const int b = b0 + k * NW;
            if (b < nb) {
                if (norm) {
                    float w[8];
                    if (b0 == warp && k < KW) {
#pragma unroll
                        for (int i = 0; i < 8; ++i) w[i] = nw[k < KW ? k : 0][i];
                    } else {
                        ld8(p.norm_w, b, lane, w);
                    }
#pragma unroll
                    for (int i = 0; i < 8; ++i) v[k][i] = __fmul_rn(__fmul_rn(v[k][i], scale), w[i]);
                }
                quant(b, v[k]);
            }
        }
    }
}

// One product launch. TYPES: 12 or 14 when every segment is Q4_K or Q6_K
// (the kernel then carries one format's code only), 0 for a mix (each group
// lies in one segment, so the branch is uniform over a warp). CB: blocks of
// a row per ring stage.
template <int TYPES, int CB>
__global__ void __launch_bounds__(32 * kWarps, 1) qmatvec_kernel(const __grid_constant__ QMatvecParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    KTRACE_PRODUCT(3);
    const int nb = p.cols / 256, S = p.stages;
    const int n_chunks = (nb + CB - 1) / CB;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);                                  // [kWarps][S]
    unsigned long long *wkeys = reinterpret_cast<unsigned long long *>(bars + kWarps * S);   // [kWarps]
    double *red = reinterpret_cast<double *>(wkeys + kWarps);                            // [kWarps]
    float *s_scale = reinterpret_cast<float *>(red + kWarps);                             // [4]
    uint8_t *q8t = reinterpret_cast<uint8_t *>(s_scale + 4);                              // [nb][kQ8Block]
    float *xds = reinterpret_cast<float *>(q8t + (size_t)nb * kQ8Block);                  // [nb]
    int16_t *bss = reinterpret_cast<int16_t *>(xds + ((nb + 3) & ~3));                    // [nb][16]
    int16_t *prs = bss + (size_t)nb * 16;                                                 // [nb][8]
    uint8_t *slots = reinterpret_cast<uint8_t *>(prs + (size_t)nb * 8);                   // [kWarps][S][2][row_slot]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rr = lane >> 4, h2 = (lane >> 3) & 1, k = lane & 7;
    uint64_t *mybar = bars + warp * S;
    const size_t stage_bytes = (size_t)2 * p.row_slot;
    uint8_t *myslots = slots + (size_t)warp * S * stage_bytes;

    int total_rows = 0;
    for (int s = 0; s < p.n_seg; ++s) total_rows += p.seg[s].rows;
    const int n_groups = p.pair_segments ? p.seg[0].rows : (total_rows + 1) / 2;
    const int TW = (int)gridDim.x * kWarps;
    // groups warp-major over the grid: consecutive groups (and so each
    // matrix's rows, e.g. a Q6_K Wv among Q4_K ones) spread over all SMs
    const int gg0 = warp * (int)gridDim.x + (int)blockIdx.x;
    const int my_groups = gg0 < n_groups ? (n_groups - gg0 + TW - 1) / TW : 0;
    const int n_items = my_groups * n_chunks;   // (group, chunk) in order
    if (lane == 0) {
        for (int s = 0; s < S; ++s) mbar_init(mybar + s, 1);
        mbar_fence_init();
    }
    __syncwarp();

    // The byte range of row rr of group gg, chunk c: its 16-aligned start and
    // the copy's length (0 when the group has no such row).
    auto chunk_src = [&](int gg, int r, int c, uintptr_t &a0, uint32_t &bytes) -> uint32_t {
        int row;
        const int sg = group_row(p, gg, r, total_rows, row);
        if (sg < 0) {
            bytes = 0;
            return 0;
        }
        const QSeg &q = p.seg[sg];
        const size_t BB = TYPES ? block_stride(TYPES) : block_stride(q.type);
        const int c0 = c * CB, cb = min(CB, nb - c0);
        const uintptr_t a = reinterpret_cast<uintptr_t>(q.w) + ((size_t)row * nb + c0) * BB;
        a0 = a & ~uintptr_t(15);
        bytes = (uint32_t)(((a - a0) + cb * BB + 15) & ~uintptr_t(15));
        return (uint32_t)(a - a0);
    };
    // bulk copies of item (group t, chunk c) into stage s: lane 0 arms the
    // stage's barrier with both rows' bytes, then lanes 0 and 16 each copy
    // their row's chunk
    auto issue = [&](int t, int c, int s) {
        const int gg = gg0 + t * TW;
        uintptr_t a0 = 0, b0 = 0;
        uint32_t by = 0, by_other = 0;
        if ((lane & 15) == 0) {
            chunk_src(gg, rr, c, a0, by);
            chunk_src(gg, rr ^ 1, c, b0, by_other);
            if (lane == 0) {
                fence_proxy_async_smem();
                mbar_arrive_expect_tx(mybar + s, by + by_other);
            }
        }
        __syncwarp();
        if ((lane & 15) == 0 && by) {
            if (lane == 16) fence_proxy_async_smem();
            bulk_g2s(myslots + s * stage_bytes + (size_t)rr * p.row_slot, reinterpret_cast<const void *>(a0), by,
                     mybar + s, l2_evict_first_policy());
        }
    };
    // the next item to issue, as (group, chunk), advanced incrementally
    int iss_t = 0, iss_c = 0;
    auto advance = [&](int &t, int &c) {
        if (++c == n_chunks) {
            c = 0;
            ++t;
        }
    };
    for (int it = 0; it < S && it < n_items; ++it) {
        issue(iss_t, iss_c, it);
        advance(iss_t, iss_c);
    }
    float nw[1][8];
    if (p.in_mode == QIN_RMSNORM) load_norm_first<kWarps, 1>(p, nb, nw);
    grid_dep_wait();
    KTRACE(1);

    // ------------------------------------------------------------ the Q8_K input
    build_q8_input<kWarps, 3, 1>(p, nb, red, nw, [&](int b, const float (&v)[8]) {
        q8k_block(v, lane, q8t + (size_t)b * kQ8Block, xds + b, bss + (size_t)b * 16, prs + (size_t)b * 8);
    });
    __syncthreads();
    grid_dep_launch();
    KTRACE(2);

    // ------------------------------------------------------------ the rows
    unsigned long long best = 0;   // argmax key of this lane's rows (QOUT_ARGMAX)
    float acc = 0.f, accm = 0.f;
    int it = 0, s = 0;
    uint32_t ph = 0;   // item it sits in stage s = it % S with barrier parity ph = (it / S) & 1
    for (int t = 0; t < my_groups; ++t) {
        const int gg = gg0 + t * TW;
        int row;
        const int sg = group_row(p, gg, rr, total_rows, row);
        const bool valid = sg >= 0;
        const bool q4 = TYPES == 12 || (TYPES == 0 && valid && p.seg[sg].type == 12);
        const uint8_t *wrow = valid ? p.seg[sg].w + (size_t)row * nb * (q4 ? kQ4Stride : kQ6Stride) : nullptr;
        acc = 0.f;
        accm = 0.f;
        bool gave_up = false;
        for (int c = 0; c < n_chunks; ++c) {
            if (!__all_sync(FULLW, mbar_wait(mybar + s, ph, p.err, DEV_WAIT_FULL_TIMEOUT))) {
                // gave up (recorded): let the copies still in flight land first
                for (int u = it; u < n_items && u < it + S; ++u) mbar_drain(mybar + u % S, (u / S) & 1);
                gave_up = true;
                break;
            }
            KTRACE_FIRST_LANDED(it);
            const int c0 = c * CB, cb = min(CB, nb - c0), half0 = (cb + 1) >> 1;
            const uintptr_t a = reinterpret_cast<uintptr_t>(wrow) + (size_t)c0 * (q4 ? kQ4Stride : kQ6Stride);
            const uint8_t *blk0 = myslots + s * stage_bytes + (size_t)rr * p.row_slot + (a & 15);
            // this half's blocks of the chunk: the first half feeds the
            // chains, the second half parks its terms until the chains reach it
            const int j0 = h2 ? half0 : 0, j1 = h2 ? cb : half0;
            Terms park[(CB + 1) / 2];
            auto run_half = [&](auto type_tag) {
                constexpr int T = decltype(type_tag)::value;
                constexpr int BB = block_stride(T);
#pragma unroll
                for (int jj = 0; jj < (CB + 1) / 2; ++jj) {
                    const int j = j0 + jj;
                    if (valid && j < j1) {
                        const int b = c0 + j;
                        uint32_t w[kW];
                        lds_block<T>(blk0 + (size_t)j * BB, k, w);
                        const Terms tm = block_terms<T>(w, k, q8t + (size_t)b * kQ8Block, bss + (size_t)b * 16,
                                                        prs + (size_t)b * 8, xds[b]);
                        if (h2 == 0) take(tm, acc, accm);
                        else park[jj] = tm;
                    }
                }
            };
            if (q4) run_half(std::integral_constant<int, 12>());
            else run_half(std::integral_constant<int, 14>());
            {
                const float a1 = __shfl_xor_sync(FULLW, acc, 8), m1 = __shfl_xor_sync(FULLW, accm, 8);
                if (h2) {
                    acc = a1;
                    accm = m1;
#pragma unroll
                    for (int jj = 0; jj < (CB + 1) / 2; ++jj)
                        if (valid && j0 + jj < j1) take(park[jj], acc, accm);
                }
                const float a2 = __shfl_xor_sync(FULLW, acc, 8), m2 = __shfl_xor_sync(FULLW, accm, 8);
                if (!h2) {
                    acc = a2;
                    accm = m2;
                }
            }
            __syncwarp();   // every lane is done with the stage
            if (it + S < n_items) {
                issue(iss_t, iss_c, s);   // item it + S reuses this stage
                advance(iss_t, iss_c);
            }
            ++it;
            if (++s == S) {
                s = 0;
                ph ^= 1u;
            }
        }
        if (gave_up) break;

        // ------------------------------------------------ the group's results
        const float r = row_sum(acc, accm, q4);
        const float other = __shfl_xor_sync(FULLW, r, 16);   // the other row's result (lane 0 <-> 16)
        if (h2 == 0 && k == 0 && valid) {
            const QSeg &q = p.seg[sg];
            switch (p.out_mode) {
                case QOUT_STORE:
                    q.out[row] = q.bias ? __fadd_rn(r, q.bias[row]) : r;
                    break;
                case QOUT_RESIDUAL:
                    q.out[row] = __fadd_rn(p.resid[row], r);
                    break;
                case QOUT_SWIGLU:   // lane 0 holds the gate row, lane 16 the up row
                    if (rr == 0) q.out[row] = kore_swiglu(r, other, p.exp_tab);
                    break;
                case QOUT_ARGMAX: {
                    q.out[row] = r;
                    int g = row;
                    for (int s2 = 0; s2 < sg; ++s2) g += p.seg[s2].rows;
                    const unsigned long long key = argmax_key(r, g);
                    best = key > best ? key : best;
                    break;
                }
                default:
                    break;
            }
        }
    }
    if (p.out_mode == QOUT_ARGMAX) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long x = __shfl_xor_sync(FULLW, best, o);
            best = x > best ? x : best;
        }
        if (lane == 0) wkeys[warp] = best;
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned long long m = 0;
            for (int w = 0; w < kWarps; ++w) m = wkeys[w] > m ? wkeys[w] : m;
            if (m) atomicMax(p.argmax, m);
        }
    }
    KTRACE_END();
}

// ---------------------------------------------------------------- row-task products
//
// qmatvec_rows_kernel: the same products with 16 rows per warp task, for
// Q4_K launches with many rows (the 7B feed-forward gate/up pair; launch_qmatvec
// keeps the Q6_K launches, whose blocks this kernel reads word by word, on the
// group kernel). Lane (slot, kh) = (lane & 15, lane >> 4) owns row slot `slot` of
// the task and kore's AVX2 lanes k = 4 kh .. 4 kh + 3 of every block of that
// row: it forms those lanes' exact integers for each block and advances their
// fused multiply-add chains in block order itself, so no chain is handed
// between lanes and the block header and scales are unpacked by 2 lanes of a
// row instead of 16. The row's kore sums then take one shuffle (the other
// half's lanes); the epilogue runs on all 16 row lanes at once. A warp's
// items (task, chunk of kRCB blocks) stream through a private ring of
// stages, 16 rows per stage, one bulk copy per row issued by that row's lane.
// The Q8_K input is staged per CTA in natural order (word w = values 4w ..
// 4w+3), which every lane reads as 16-byte runs.

#ifndef KORE_ROWS_WARPS
#define KORE_ROWS_WARPS 8
#endif
constexpr int kRW = KORE_ROWS_WARPS;   // warps per CTA

// Shared-memory loads by 32-bit shared address (no generic addressing).
__device__ __forceinline__ uint4 ld_sh128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t ld_sh32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ float ld_shf(uint32_t a) { return __uint_as_float(ld_sh32(a)); }
constexpr int kRSlots = 16;     // row slots per task (pair mode: 8 gate rows, then the same 8 up rows)
#ifndef KORE_ROWS_CB
#define KORE_ROWS_CB 2
#endif
constexpr int kRCB = KORE_ROWS_CB;   // blocks per row per ring stage
constexpr int kQ8N = 320;       // staged Q8_K block: qs [256], bsums [16] int16, pairs [8] int16, d, pad

// One warp quantises one 256-value block (lane l holds values 8l..8l+7) into
// a natural-order staged Q8_K block (the same arithmetic as q8k_block).
__device__ __forceinline__ void q8k_block_nat(const float (&v)[8], int lane, uint8_t *blk) {
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
        const float am = __shfl_xor_sync(FULLW, amax, o);
        const float mv = __shfl_xor_sync(FULLW, maxv, o);
        const int ix = __shfl_xor_sync(FULLW, idx, o);
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
    s += __shfl_xor_sync(FULLW, s, 1);
    uint2 w;
    w.x = (uint32_t)(q[0] & 0xFF) | (uint32_t)(q[1] & 0xFF) << 8 | (uint32_t)(q[2] & 0xFF) << 16 |
          (uint32_t)(q[3] & 0xFF) << 24;
    w.y = (uint32_t)(q[4] & 0xFF) | (uint32_t)(q[5] & 0xFF) << 8 | (uint32_t)(q[6] & 0xFF) << 16 |
          (uint32_t)(q[7] & 0xFF) << 24;
    reinterpret_cast<uint2 *>(blk)[lane] = w;
    int16_t *bsums = reinterpret_cast<int16_t *>(blk + 256);
    int16_t *pairs = reinterpret_cast<int16_t *>(blk + 288);
    if ((lane & 1) == 0) bsums[lane >> 1] = (int16_t)s;
    const int s2 = (int)(int16_t)s + (int)(int16_t)__shfl_xor_sync(FULLW, s, 2);
    if ((lane & 3) == 0) pairs[lane >> 2] = (int16_t)s2;
    if (lane == 0) *reinterpret_cast<float *>(blk + 304) = d;
}

// Shared memory of a row-task launch: the Q8_K input, then per warp S stages
// of kRSlots row slots; a slot's byte stride is 16 x an odd number, so that
// the 16-byte loads of 8 consecutive row slots fall on distinct banks.
__host__ __device__ constexpr int rows_slot_bytes(int type) {
    return type == 12 ? (kRCB * kQ4Stride + 15) / 16 % 2 ? (kRCB * kQ4Stride + 15) / 16 * 16
                                                          : ((kRCB * kQ4Stride + 15) / 16 + 1) * 16
                      : ((kRCB * kQ6Stride + 15 + 15) / 16) % 2 ? ((kRCB * kQ6Stride + 15 + 15) / 16) * 16
                                                                  : ((kRCB * kQ6Stride + 15 + 15) / 16 + 1) * 16;
}
static_assert(rows_slot_bytes(12) / 16 % 2 == 1 && rows_slot_bytes(14) / 16 % 2 == 1, "row slot strides");
constexpr size_t rows_fixed_smem(int nb, int S) {
    return (size_t)8 * kRW * S + 8 * kRW + 8 * kRW + 16 + (size_t)nb * kQ8N;
}

// One Q4_K block of a row for this lane's AVX2 lanes k = 4 kh + kl
// (kore.cpp:553-586, as block_terms<12>): the exact integers of each lane,
// then each lane's chains acc += d * s, accm += dm * e in block order.
__device__ __forceinline__ void rows_block_q4(uint32_t blk, uint32_t q8, int kh, float (&acc)[4], float (&accm)[4]) {
    const uint4 h = ld_sh128(blk);
    const uint32_t u0 = h.y, u1 = h.z, u2 = h.w;
    const uint32_t sc_lo = u0 & 0x3F3F3F3Fu, sc_hi = (u2 & 0x0F0F0F0Fu) | ((u0 >> 2) & 0x30303030u);
    const uint32_t mn_lo = u1 & 0x3F3F3F3Fu, mn_hi = ((u2 >> 4) & 0x0F0F0F0Fu) | ((u1 >> 2) & 0x30303030u);
    const float xd = ld_shf(q8 + 304);
    const float d = __fmul_rn(half_bits(h.x & 0xFFFFu), xd);
    const float dm = -__fmul_rn(half_bits(h.x >> 16), xd);
    const uint4 pr = ld_sh128(q8 + 288);   // bsum pairs (2m, 2m+1) in word m
    const uint32_t pm[4] = {pr.x, pr.y, pr.z, pr.w};
    int s[4] = {0, 0, 0, 0};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint4 W = ld_sh128(blk + 16 + 32 * c + 16 * kh);
        const uint4 L = ld_sh128(q8 + 4 * (16 * c + 4 * kh));
        const uint4 H = ld_sh128(q8 + 4 * (16 * c + 8 + 4 * kh));
        const uint32_t w[4] = {W.x, W.y, W.z, W.w}, lo8[4] = {L.x, L.y, L.z, L.w}, hi8[4] = {H.x, H.y, H.z, H.w};
        const uint32_t scw = c < 2 ? sc_lo : sc_hi;
#pragma unroll
        for (int kl = 0; kl < 4; ++kl) {
            const int lo = __dp4a((int)(w[kl] & 0x0F0F0F0Fu), (int)lo8[kl], 0);
            const int hi = __dp4a((int)((w[kl] >> 4) & 0x0F0F0F0Fu), (int)hi8[kl], 0);
            const int pk = (int)__byte_perm((uint32_t)lo, (uint32_t)hi, 0x5410);
            s[kl] = (c & 1) ? __dp2a_hi(pk, (int)scw, s[kl]) : __dp2a_lo(pk, (int)scw, s[kl]);
        }
    }
#pragma unroll
    for (int kl = 0; kl < 4; ++kl) {
        // minimum lane m = k & 3 = kl: mn[2m] * pairs[2m] + mn[2m+1] * pairs[2m+1]
        const uint32_t mnw = kl < 2 ? mn_lo : mn_hi;
        const int e = __dp2a_lo((int)pm[kl], (int)(mnw >> (16 * (kl & 1))), 0);
        acc[kl] = __fmaf_rn(d, __int2float_rn(s[kl]), acc[kl]);
        accm[kl] = __fmaf_rn(dm, __int2float_rn(e), accm[kl]);
    }
}

// Two consecutive Q4_K blocks of a row, their integer work interleaved (two
// independent sets of lane sums), then the chains in block order: the same
// values as rows_block_q4 twice.
__device__ __forceinline__ void rows_block2_q4(uint32_t blk, uint32_t q8, int kh, float (&acc)[4], float (&accm)[4]) {
    uint32_t sc[2][2], mn[2][2];
    float d[2], dm[2];
    uint32_t pm[2][4];
#pragma unroll
    for (int b = 0; b < 2; ++b) {
        const uint4 h = ld_sh128(blk + b * kQ4Stride);
        const uint32_t u0 = h.y, u1 = h.z, u2 = h.w;
        sc[b][0] = u0 & 0x3F3F3F3Fu;
        sc[b][1] = (u2 & 0x0F0F0F0Fu) | ((u0 >> 2) & 0x30303030u);
        mn[b][0] = u1 & 0x3F3F3F3Fu;
        mn[b][1] = ((u2 >> 4) & 0x0F0F0F0Fu) | ((u1 >> 2) & 0x30303030u);
        const float xd = ld_shf(q8 + b * kQ8N + 304);
        d[b] = __fmul_rn(half_bits(h.x & 0xFFFFu), xd);
        dm[b] = -__fmul_rn(half_bits(h.x >> 16), xd);
        const uint4 pr = ld_sh128(q8 + b * kQ8N + 288);
        pm[b][0] = pr.x;
        pm[b][1] = pr.y;
        pm[b][2] = pr.z;
        pm[b][3] = pr.w;
    }
    int s[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int b = 0; b < 2; ++b) {
            const uint4 W = ld_sh128(blk + b * kQ4Stride + 16 + 32 * c + 16 * kh);
            const uint4 L = ld_sh128(q8 + b * kQ8N + 4 * (16 * c + 4 * kh));
            const uint4 H = ld_sh128(q8 + b * kQ8N + 4 * (16 * c + 8 + 4 * kh));
            const uint32_t w[4] = {W.x, W.y, W.z, W.w}, lo8[4] = {L.x, L.y, L.z, L.w}, hi8[4] = {H.x, H.y, H.z, H.w};
            const uint32_t scw = sc[b][c >> 1];
#pragma unroll
            for (int kl = 0; kl < 4; ++kl) {
                const int lo = __dp4a((int)(w[kl] & 0x0F0F0F0Fu), (int)lo8[kl], 0);
                const int hi = __dp4a((int)((w[kl] >> 4) & 0x0F0F0F0Fu), (int)hi8[kl], 0);
                const int pk = (int)__byte_perm((uint32_t)lo, (uint32_t)hi, 0x5410);
                s[b][kl] = (c & 1) ? __dp2a_hi(pk, (int)scw, s[b][kl]) : __dp2a_lo(pk, (int)scw, s[b][kl]);
            }
        }
    }
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int kl = 0; kl < 4; ++kl) {
            const int e = __dp2a_lo((int)pm[b][kl], (int)(mn[b][kl >> 1] >> (16 * (kl & 1))), 0);
            acc[kl] = __fmaf_rn(d[b], __int2float_rn(s[b][kl]), acc[kl]);
            accm[kl] = __fmaf_rn(dm[b], __int2float_rn(e), accm[kl]);
        }
}

// One Q6_K block (kore.cpp:603-636, as block_terms<14>); the block is 4-byte
// aligned (212-byte stride), so its words are read one by one.
__device__ __forceinline__ void rows_block_q6(uint32_t blk, uint32_t q8, int kh, float (&acc)[4], float &accm) {
    uint32_t sw[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) sw[i] = ld_sh32(blk + 192 + 4 * i);
    const float xd = ld_shf(q8 + 304);
    const float d = __fmul_rn(half_bits(ld_sh32(blk + 208) & 0xFFFFu), xd);
    const float dm = -__fmul_rn(d, 32.0f);
    const uint32_t o = kh ? 0x31u : 0x20u;   // this lane group's scale of each 32-value group: bytes o, o+2
    int s[4] = {0, 0, 0, 0};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        uint32_t Q[4][4];
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            const uint4 q = ld_sh128(q8 + 4 * (8 * (4 * h + kk) + 4 * kh));
            Q[kk][0] = q.x;
            Q[kk][1] = q.y;
            Q[kk][2] = q.z;
            Q[kk][3] = q.w;
        }
        const int scA = (int)__byte_perm(sw[2 * h], 0u, o), scB = (int)__byte_perm(sw[2 * h + 1], 0u, o);
#pragma unroll
        for (int kl = 0; kl < 4; ++kl) {
            const int k4 = 16 * kh + 4 * kl;
            const uint32_t qla = ld_sh32(blk + 64 * h + k4), qlb = ld_sh32(blk + 64 * h + 32 + k4);
            const uint32_t qh = ld_sh32(blk + 128 + 32 * h + k4);
            int part[4];
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const uint32_t ql = (kk & 1) ? qlb : qla;
                const uint32_t v = ((ql >> (4 * (kk >> 1))) & 0x0F0F0F0Fu) | (((qh >> (2 * kk)) & 0x03030303u) << 4);
                part[kk] = __dp4a((int)v, (int)Q[kk][kl], 0);
            }
            s[kl] = __dp2a_lo((int)__byte_perm((uint32_t)part[0], (uint32_t)part[1], 0x5410), scA, s[kl]);
            s[kl] = __dp2a_lo((int)__byte_perm((uint32_t)part[2], (uint32_t)part[3], 0x5410), scB, s[kl]);
        }
    }
    const uint4 ba = ld_sh128(q8 + 256);
    const uint4 bb = ld_sh128(q8 + 272);
    const uint32_t bw[8] = {ba.x, ba.y, ba.z, ba.w, bb.x, bb.y, bb.z, bb.w};
    int ib = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i)
        ib = (i & 1) ? __dp2a_hi((int)bw[i], (int)sw[i >> 1], ib) : __dp2a_lo((int)bw[i], (int)sw[i >> 1], ib);
#pragma unroll
    for (int kl = 0; kl < 4; ++kl) acc[kl] = __fmaf_rn(d, __int2float_rn(s[kl]), acc[kl]);
    accm = __fmaf_rn(dm, __int2float_rn(ib), accm);
}

template <int TYPE>
__global__ void __launch_bounds__(32 * kRW, 1) qmatvec_rows_kernel(const __grid_constant__ QMatvecParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    KTRACE_PRODUCT(4);
    constexpr int BB = block_stride(TYPE);
    constexpr int SLOT = rows_slot_bytes(TYPE);
    constexpr size_t STAGE = (size_t)kRSlots * SLOT;
    const int nb = p.cols / 256, S = p.stages;
    const int n_chunks = (nb + kRCB - 1) / kRCB;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);                                 // [kRW][S]
    unsigned long long *wkeys = reinterpret_cast<unsigned long long *>(bars + kRW * S);   // [kRW]
    double *red = reinterpret_cast<double *>(wkeys + kRW);                              // [kRW]
    float *s_scale = reinterpret_cast<float *>(red + kRW);                               // [4]
    uint8_t *q8n = reinterpret_cast<uint8_t *>(s_scale + 4);                             // [nb][kQ8N]
    uint8_t *stages = q8n + (size_t)nb * kQ8N;                                           // [kRW][S][slots]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int slot = lane & 15, kh = lane >> 4;
    uint64_t *mybar = bars + warp * S;
    uint8_t *mystages = stages + (size_t)warp * S * STAGE;
    const uint32_t stage_sa = smem_u32(mystages) + (uint32_t)slot * SLOT;   // this lane's row slot in stage 0
    const uint32_t q8_sa = smem_u32(q8n);

    // tasks: 16 rows of one segment, or (pair mode) the same 8 rows of both
    int n_tasks = 0;
    if (p.pair_segments) n_tasks = (p.seg[0].rows + 7) / 8;
    else
        for (int s = 0; s < p.n_seg; ++s) n_tasks += (p.seg[s].rows + kRSlots - 1) / kRSlots;
    const int TW = (int)gridDim.x * kRW;
    const int t0 = warp * (int)gridDim.x + (int)blockIdx.x;   // tasks warp-major over the grid
    const int my_tasks = t0 < n_tasks ? (n_tasks - t0 + TW - 1) / TW : 0;
    const int n_items = my_tasks * n_chunks;
    // this lane's row (within its segment) in task t; false: the slot has no row
    auto task_row = [&](int t, int &seg, int &row) -> bool {
        if (p.pair_segments) {
            seg = slot < 8 ? 0 : 1;
            row = t * 8 + (slot & 7);
            return row < p.seg[0].rows;
        }
        int s = 0;
        while (s + 1 < p.n_seg && t >= (p.seg[s].rows + kRSlots - 1) / kRSlots) {
            t -= (p.seg[s].rows + kRSlots - 1) / kRSlots;
            ++s;
        }
        seg = s;
        row = t * kRSlots + slot;
        return row < p.seg[s].rows;
    };
    if (lane == 0) {
        for (int s = 0; s < S; ++s) mbar_init(mybar + s, 1);
        mbar_fence_init();
    }
    __syncwarp();

    // item (task, chunk) into stage s: each row lane copies its row's chunk;
    // lane 0 arms the stage's barrier with the warp's total
    auto issue = [&](int ti, int c, int s) {
        int seg = 0, row = 0;
        uint32_t bytes = 0;
        uintptr_t a0 = 0;
        if (kh == 0 && task_row(t0 + ti * TW, seg, row)) {
            const int c0 = c * kRCB, cb = min(kRCB, nb - c0);
            const uintptr_t a = reinterpret_cast<uintptr_t>(p.seg[seg].w) + ((size_t)row * nb + c0) * BB;
            a0 = a & ~uintptr_t(15);
            bytes = (uint32_t)(((a - a0) + cb * BB + 15) & ~uintptr_t(15));
        }
        const uint32_t total = __reduce_add_sync(FULLW, bytes);
        if (lane == 0) {
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(mybar + s, total);
        }
        if (bytes) {
            if (lane) fence_proxy_async_smem();
            bulk_g2s(mystages + (size_t)s * STAGE + (size_t)slot * SLOT, reinterpret_cast<const void *>(a0), bytes,
                     mybar + s, l2_evict_first_policy());
        }
    };
    int iss_t = 0, iss_c = 0;
    auto advance = [&](int &t, int &c) {
        if (++c == n_chunks) {
            c = 0;
            ++t;
        }
    };
    for (int it = 0; it < S && it < n_items; ++it) {
        issue(iss_t, iss_c, it);
        advance(iss_t, iss_c);
    }
    float nw[2][8];
    if (p.in_mode == QIN_RMSNORM) load_norm_first<kRW, 2>(p, nb, nw);
    grid_dep_wait();
    KTRACE(1);

    // ------------------------------------------------------------ the Q8_K input
    build_q8_input<kRW, 4, 2>(p, nb, red, nw,
                              [&](int b, const float (&v)[8]) { q8k_block_nat(v, lane, q8n + (size_t)b * kQ8N); });
    __syncthreads();
    grid_dep_launch();
    KTRACE(2);

    // ------------------------------------------------------------ the rows
    unsigned long long best = 0;   // argmax key of this lane's rows (QOUT_ARGMAX)
    int it = 0, s = 0;
    uint32_t ph = 0;
    bool gave_up = false;
    for (int ti = 0; ti < my_tasks && !gave_up; ++ti) {
        int seg = 0, row = 0;
        const bool valid = task_row(t0 + ti * TW, seg, row);
        const uintptr_t rbase = valid ? reinterpret_cast<uintptr_t>(p.seg[seg].w) + (size_t)row * nb * BB : 0;
        float acc[4] = {0.f, 0.f, 0.f, 0.f}, accm[4] = {0.f, 0.f, 0.f, 0.f};
        for (int c = 0; c < n_chunks; ++c) {
            if (!__all_sync(FULLW, mbar_wait(mybar + s, ph, p.err, DEV_WAIT_FULL_TIMEOUT))) {
                // gave up (recorded): let the copies still in flight land first
                for (int u = it; u < n_items && u < it + S; ++u) mbar_drain(mybar + u % S, (u / S) & 1);
                gave_up = true;
                break;
            }
            KTRACE_FIRST_LANDED(it);
            const int c0 = c * kRCB, cb = min(kRCB, nb - c0);
            if (valid) {
                const uint32_t blk0 = stage_sa + (uint32_t)s * (uint32_t)STAGE + (uint32_t)((rbase + (size_t)c0 * BB) & 15);
                const uint32_t q8c = q8_sa + (uint32_t)c0 * kQ8N;
                if (TYPE == 12 && cb == 2) {
                    rows_block2_q4(blk0, q8c, kh, acc, accm);
                } else {
#pragma unroll
                    for (int j = 0; j < kRCB; ++j) {
                        if (j < cb) {
                            if (TYPE == 12) rows_block_q4(blk0 + j * BB, q8c + j * kQ8N, kh, acc, accm);
                            else rows_block_q6(blk0 + j * BB, q8c + j * kQ8N, kh, acc, accm[0]);
                        }
                    }
                }
            }
            __syncwarp();   // every lane is done with the stage
            if (it + S < n_items) {
                issue(iss_t, iss_c, s);   // item it + S reuses this stage
                advance(iss_t, iss_c);
            }
            ++it;
            if (++s == S) {
                s = 0;
                ph ^= 1u;
            }
        }
        if (gave_up) break;

        // kore's horizontal sums: ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)), plus
        // for Q4_K ((m0+m2)+(m1+m3)), for Q6_K the offset chain
        float other[4];
#pragma unroll
        for (int kl = 0; kl < 4; ++kl) other[kl] = __shfl_xor_sync(FULLW, acc[kl], 16);
        const float t0s = __fadd_rn(acc[0], other[0]), t1s = __fadd_rn(acc[1], other[1]);
        const float t2s = __fadd_rn(acc[2], other[2]), t3s = __fadd_rn(acc[3], other[3]);
        const float a = __fadd_rn(__fadd_rn(t0s, t2s), __fadd_rn(t1s, t3s));
        const float m = TYPE == 12 ? __fadd_rn(__fadd_rn(accm[0], accm[2]), __fadd_rn(accm[1], accm[3])) : accm[0];
        const float r = __fadd_rn(a, m);   // valid on kh == 0 lanes
        const float up = __shfl_sync(FULLW, r, (lane & 7) + 8);   // pair mode: the up row of this gate row
        if (kh == 0 && valid) {
            const QSeg &q = p.seg[seg];
            switch (p.out_mode) {
                case QOUT_STORE:
                    q.out[row] = q.bias ? __fadd_rn(r, q.bias[row]) : r;
                    break;
                case QOUT_RESIDUAL:
                    q.out[row] = __fadd_rn(p.resid[row], r);
                    break;
                case QOUT_SWIGLU:
                    if (slot < 8) q.out[row] = kore_swiglu(r, up, p.exp_tab);
                    break;
                case QOUT_ARGMAX: {
                    q.out[row] = r;
                    int g = row;
                    for (int s2 = 0; s2 < seg; ++s2) g += p.seg[s2].rows;
                    const unsigned long long key = argmax_key(r, g);
                    best = key > best ? key : best;
                    break;
                }
                default:
                    break;
            }
        }
    }
    if (p.out_mode == QOUT_ARGMAX) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long x = __shfl_xor_sync(FULLW, best, o);
            best = x > best ? x : best;
        }
        if (lane == 0) wkeys[warp] = best;
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned long long mx = 0;
            for (int w = 0; w < kRW; ++w) mx = wkeys[w] > mx ? wkeys[w] : mx;
            if (mx) atomicMax(p.argmax, mx);
        }
    }
    KTRACE_END();
}

cudaLaunchAttribute pdl_attr() {
    cudaLaunchAttribute a;
    a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    a.val.programmaticStreamSerializationAllowed = 1;
    return a;
}

size_t fixed_smem(int nb, int stages) {
    return (size_t)8 * kWarps * stages + 8 * kWarps + 8 * kWarps + 16 + (size_t)nb * kQ8Block +
           (size_t)((nb + 3) & ~3) * 4 + (size_t)nb * 32 + (size_t)nb * 16;
}

}  // namespace

// Blocks per ring stage: a whole row of up to 16 blocks when two stages of
// that size fit beside the Q8_K input (one chunk per group: the least
// bookkeeping per block), else 8.
static int chunk_blocks(int nb, int max_block_bytes) {
    if (nb > 16) return 8;
    const int slot = (int)(((size_t)16 * max_block_bytes + 32 + 15) & ~size_t(15));
    return fixed_smem(nb, 2) + (size_t)kWarps * 2 * 2 * slot <= kQmatvecMaxSmem ? 16 : 8;
}

size_t qmatvec_config(int cols, int max_block_bytes, int *stages, int *row_slot) {
    const int nb = cols / 256;
    const int cb = chunk_blocks(nb, max_block_bytes);
    // a row's chunk copy starts up to 15 bytes before its first block and ends
    // up to 15 bytes after its last; the Q6_K word reads reach 6 bytes past a block
    const int slot = (int)(((size_t)cb * max_block_bytes + 32 + 15) & ~size_t(15));
    int S = 4;
    while (S > 1 && fixed_smem(nb, S) + (size_t)kWarps * S * 2 * slot > kQmatvecMaxSmem) --S;
    if (stages) *stages = S;
    if (row_slot) *row_slot = slot;
    return fixed_smem(nb, S) + (size_t)kWarps * S * 2 * slot;
}

// Ring stages of the row-task kernel over cols in one block format; returns
// the dynamic shared memory it needs.
static size_t rows_config(int cols, int type, int *stages) {
    const int nb = cols / 256;
    const size_t per = (size_t)kRW * kRSlots * rows_slot_bytes(type);
    int S = 6;
    while (S > 2 && rows_fixed_smem(nb, S) + per * S > kQmatvecMaxSmem) --S;
    if (stages) *stages = S;
    return rows_fixed_smem(nb, S) + per * S;
}

cudaError_t launch_qmatvec(const QMatvecParams &p_in, int grid, cudaStream_t s) {
    // KORE_CUDA_RMS_SEQUENTIAL=1: every RMSNorm input sums its squares in
    // kore's order (the path a mean next to a rounding boundary takes; tests)
    static const int rms_seq = [] {
        const char *e = getenv("KORE_CUDA_RMS_SEQUENTIAL");
        return e && atoi(e) != 0 ? 1 : 0;
    }();
    QMatvecParams p = p_in;
    p.rms_sequential = rms_seq;
    if (p.n_seg <= 0 || p.n_seg > 3 || p.cols <= 0 || p.cols % 256 || !p.x || grid <= 0) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(p.x) & 15) || (p.in_mode == QIN_RMSNORM && (!p.norm_w ||
        (reinterpret_cast<uintptr_t>(p.norm_w) & 15))))
        return cudaErrorInvalidValue;
    int bb = 0;
    for (int i = 0; i < p.n_seg; ++i) {
        if ((p.seg[i].type != 12 && p.seg[i].type != 14) || p.seg[i].rows < 0 || !p.seg[i].w || !p.seg[i].out)
            return cudaErrorInvalidValue;
        bb = max(bb, block_stride(p.seg[i].type));
    }
    if (p.pair_segments && (p.n_seg != 2 || p.seg[0].rows != p.seg[1].rows)) return cudaErrorInvalidValue;
    if (p.out_mode == QOUT_SWIGLU && !p.pair_segments) return cudaErrorInvalidValue;
    if (p.out_mode == QOUT_RESIDUAL && !p.resid) return cudaErrorInvalidValue;
    if (p.out_mode == QOUT_ARGMAX && !p.argmax) return cudaErrorInvalidValue;
    int stages = 0, slot = 0;
    const size_t smem = qmatvec_config(p.cols, bb, &stages, &slot);
    if (slot != p.row_slot || stages != p.stages || smem > kQmatvecMaxSmem) return cudaErrorInvalidValue;
    bool all4 = true, all6 = true;
    for (int i = 0; i < p.n_seg; ++i) {
        all4 = all4 && p.seg[i].type == 12;
        all6 = all6 && p.seg[i].type == 14;
    }
    // Many Q4_K rows: the row-task kernel (every warp gets at least two
    // 16-row tasks; measured 29.4 against 32.2 us on the 7B gate/up pair, and
    // 2 % slower than the group kernel on the Q6_K output matrix, whose
    // blocks it reads word by word). KORE_CUDA_ROW_PRODUCTS=0 keeps the group
    // kernel for every launch, 2 takes the row-task kernel for every launch
    // of one block format (tests/test_product_switches_gpu.py runs the
    // product and step tests under both).
    static const int rows_mode = [] {
        const char *e = getenv("KORE_CUDA_ROW_PRODUCTS");
        return e ? atoi(e) : 1;
    }();
    if (rows_mode == 2 ? (all4 || all6) : (rows_mode == 1 && all4)) {
        int n_tasks = 0;
        if (p.pair_segments) n_tasks = (p.seg[0].rows + 7) / 8;
        else
            for (int i = 0; i < p.n_seg; ++i) n_tasks += (p.seg[i].rows + kRSlots - 1) / kRSlots;
        QMatvecParams q = p;
        const size_t rsmem = rows_config(p.cols, all4 ? 12 : 14, &q.stages);
        if ((rows_mode == 2 || n_tasks >= 2 * grid * kRW) && rsmem <= kQmatvecMaxSmem) {
            void (*rk)(QMatvecParams) = all4 ? qmatvec_rows_kernel<12> : qmatvec_rows_kernel<14>;
            if (cudaError_t e = ensure_smem_limit(reinterpret_cast<const void *>(rk), (int)kQmatvecMaxSmem)) return e;
            cudaLaunchConfig_t rcfg = {};
            rcfg.gridDim = dim3(grid);
            rcfg.blockDim = dim3(32 * kRW);
            rcfg.dynamicSmemBytes = rsmem;
            rcfg.stream = s;
            cudaLaunchAttribute rattr = pdl_attr();
            rcfg.attrs = &rattr;
            rcfg.numAttrs = 1;
            return cudaLaunchKernelEx(&rcfg, rk, q);
        }
    }
    const bool wide = chunk_blocks(p.cols / 256, bb) == 16;
    void (*kern)(QMatvecParams) = all4 ? (wide ? qmatvec_kernel<12, 16> : qmatvec_kernel<12, 8>)
                                  : all6 ? (wide ? qmatvec_kernel<14, 16> : qmatvec_kernel<14, 8>)
                                         : (wide ? qmatvec_kernel<0, 16> : qmatvec_kernel<0, 8>);
    if (cudaError_t e = ensure_smem_limit(reinterpret_cast<const void *>(kern), (int)kQmatvecMaxSmem)) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(32 * kWarps);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr = pdl_attr();
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

#ifdef KORE_TRACE
// Trace build only: the product CTAs' records since the last reset (read
// after the decode's by kore_trace_read).
int proj_trace_read(void *host, unsigned max_recs, unsigned *n_recs) {
    unsigned n = 0;
    if (cudaMemcpyFromSymbol(&n, g_trace_n, sizeof n) != cudaSuccess) return -1;
    n = n < kTraceRecs ? n : kTraceRecs;
    const unsigned m = max_recs < n ? max_recs : n;
    if (m && cudaMemcpyFromSymbol(host, g_trace, (size_t)m * sizeof(TraceRec)) != cudaSuccess) return -1;
    *n_recs = m;
    return 0;
}

int proj_trace_reset() {
    const unsigned z = 0;
    return cudaMemcpyToSymbol(g_trace_n, &z, sizeof z) == cudaSuccess ? 0 : -1;
}
#endif

}  // namespace kore
