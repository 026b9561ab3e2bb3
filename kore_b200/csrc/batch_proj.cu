// batch_proj.cu — kore's prefill-side products on the GPU: the float-activation
// batched matmul of forward_batch() and the row-wise RMSNorm around it, sm_100a.
//
// kore's forward_batch() (kore.cpp:1486-1598) projects a chunk of B tokens
// with matmul_batch_float (kore.cpp:783-845) instead of the Q8_K products of
// the decode step: each 256-value block of a weight row is dequantised to
// fp32 (dequant_block_q4_K / _q6_K, kore.cpp:337-381) and every output
// out[b][r] accumulates w[r][j] * x[b][j] with one fused multiply-add per
// column, in column order, from 0 (the AVX2 rank-1 kernels, kore.cpp:738-781;
// kore selects them on every AVX2/FMA CPU). The result of an output depends
// only on that chain, so any assignment of outputs to threads gives kore's
// values bit for bit as long as each thread keeps the chain's order — which
// is what batch_matmul_kernel does: a CTA holds a tile of 32 weight rows x
// up to 64 tokens, dequantises the tile's rows one block at a time into
// shared memory with kore's rounding (each thread one row's 64 values, the
// sub-block scales computed once), transposed so that a thread reads the 4
// rows it serves at a column with one 16-byte load, stages the tokens'
// matching 256 columns transposed beside them (conflict-free stores), and
// each thread advances 16 chains (4 rows x 4 tokens) through the block; two
// CTAs per SM overlap one's staging with the other's products. CUDA cores,
// not tensor cores: a tensor-core product sums in its own order and could not
// give kore's values.
//
// The epilogues do what forward_batch does next to each product: the bias
// add (kore.cpp:1530-1532), the residual add x += o (:1568-1571, :1588-1591)
// and, for the gate/up pair (a tile of 16 gate rows and the same 16 up rows),
// the SwiGLU g / (1 + exp(-g)) * u (:1578-1584) with the C library's expf.
//
// rmsnorm_rows_kernel: kore's rmsnorm (kore.cpp:1367-1372) of each token's
// row, one CTA per row, with the double-precision sum of squares checked as
// in proj.cu (tree sum, then kore's sequential order only when the rounded
// mean could differ).

#include "attn.cuh"
#include "common.cuh"
#include "kore_math.cuh"

namespace kore {
namespace {

constexpr int kRT = 32;          // weight rows per tile (pair mode: 16 gate + 16 up rows, interleaved)
constexpr int kBT = 64;          // tokens per tile
constexpr int kNT = 128;         // threads: (kRT / 4) row quads x (kBT / 4) token quads
constexpr int kWP = kRT + 4;     // shared pitch of the transposed weights Wt[j][row] (16-byte rows)
constexpr int kXP = kBT + 4;     // shared pitch of the transposed tokens Xs[j][token] (16-byte rows)

constexpr size_t kXsFloats = (size_t)256 * kXP;
constexpr size_t kBatchSmem = (kXsFloats + (size_t)256 * kWP) * sizeof(float);   // 106.5 KB: two CTAs per SM

// Dequantises the 64 values [64 qq, 64 qq + 64) of a Q4_K block into Wt
// column s (kore.cpp:337-354: d1 = d * scale, m1 = dmin * min per 32-value
// sub-block, value = d1 * q - m1, each product and the difference rounded).
__device__ __forceinline__ void dequant_q4k_quarter(const uint8_t *b, int qq, float *Wt, int s) {
    int sc, mn;
    scale_min_k4(2 * qq, b + 4, sc, mn);
    const float d = f16_at(b), dmin = f16_at(b + 2);
    const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)mn);
    scale_min_k4(2 * qq + 1, b + 4, sc, mn);
    const float d2 = __fmul_rn(d, (float)sc), m2 = __fmul_rn(dmin, (float)mn);
    const uint32_t *qw = reinterpret_cast<const uint32_t *>(b + 16 + 32 * qq);
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        const uint32_t q = qw[w];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int l = 4 * w + k;
            const int byte = (q >> (8 * k)) & 0xFF;
            Wt[(64 * qq + l) * kWP + s] = __fsub_rn(__fmul_rn(d1, (float)(byte & 0x0F)), m1);
            Wt[(64 * qq + 32 + l) * kWP + s] = __fsub_rn(__fmul_rn(d2, (float)(byte >> 4)), m2);
        }
    }
}

// The same for a Q6_K block (kore.cpp:359-381: value = (d * scale) * (q - 32)).
// Quarter qq: half qq >> 1, groups 2 (qq & 1) and 2 (qq & 1) + 1 of it.
__device__ __forceinline__ void dequant_q6k_quarter(const uint8_t *b, int qq, float *Wt, int s) {
    const int half = qq >> 1, g0 = 2 * (qq & 1);
    // uploaded Q6_K blocks are 4-byte aligned (kQ6Stride): read words
    const uint32_t *ql = reinterpret_cast<const uint32_t *>(b + 64 * half);
    const uint32_t *qh = reinterpret_cast<const uint32_t *>(b + 128 + 32 * half);
    const int8_t *sc = reinterpret_cast<const int8_t *>(b + 192 + 8 * half);
    const float d = f16_at(b + 208);
#pragma unroll
    for (int gg = 0; gg < 2; ++gg) {
        const int g = g0 + gg;
        const float ds0 = __fmul_rn(d, (float)sc[2 * g]), ds1 = __fmul_rn(d, (float)sc[1 + 2 * g]);
        const uint32_t *lo_src = (g & 1) ? ql + 8 : ql;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            const uint32_t lw = lo_src[w], hw = qh[w];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int l = 4 * w + k;
                const int lo = (lw >> (8 * k)) & 0xFF, hi2 = ((hw >> (8 * k)) >> (2 * g)) & 3;
                const int q = (((g & 2) ? (lo >> 4) : (lo & 0x0F)) | (hi2 << 4)) - 32;
                Wt[(128 * half + 32 * g + l) * kWP + s] = __fmul_rn(l < 16 ? ds0 : ds1, (float)q);
            }
        }
    }
}

__global__ void __launch_bounds__(kNT, 2) batch_matmul_kernel(const __grid_constant__ BatchMatmulParams p) {
    extern __shared__ __align__(16) float bsm[];
    float *Xs = bsm;               // [256][kXP]: the tokens' 256 columns of one block, transposed
    float *Wt = bsm + kXsFloats;   // [256][kWP]: the tile's rows of that block, dequantised, transposed
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rq = tid >> 4, tq = tid & 15;            // row quad, token quad of this thread's 16 chains
    const int b0 = blockIdx.y * kBT;
    const int nb = p.cols / 256;
    // the tile's weight rows: slot s holds (segment, row), or none
    auto slot_row = [&](int s, int &row) -> int {
        if (p.pair) {
            row = blockIdx.x * (kRT / 2) + (s >> 1);
            return row < p.seg[0].rows ? (s & 1) : -1;
        }
        row = blockIdx.x * kRT + s;
        return row < p.seg[0].rows ? 0 : -1;
    };
    // dequantisation: thread (quarter qq = warp, slot s = lane) owns 64
    // values of one row's block, so that a warp's stores fill one Wt row
    const int ds = lane, dqq = warp;
    int drow;
    const int dsg = slot_row(ds, drow);
    const uint8_t *dbase = nullptr;
    bool dq4 = true;
    if (dsg >= 0) {
        const QSeg &q = p.seg[dsg];
        dq4 = q.type == 12;
        dbase = q.w + (size_t)drow * nb * block_stride(q.type);
    }
    float acc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int t = 0; t < 4; ++t) acc[a][t] = 0.f;

    for (int i = 0; i < nb; ++i) {
        if (dsg < 0) {
            for (int j = 0; j < 64; ++j) Wt[(64 * dqq + j) * kWP + ds] = 0.f;
        } else if (dq4) {
            dequant_q4k_quarter(dbase + (size_t)i * kQ4Stride, dqq, Wt, ds);
        } else {
            dequant_q6k_quarter(dbase + (size_t)i * kQ6Stride, dqq, Wt, ds);
        }
        // the tokens' columns of block i, transposed: a warp moves 4 tokens x 8
        // columns per pass (coalesced 32-byte reads, conflict-free stores)
        // (16-byte loads, a round of them in flight per thread); a warp moves 4
        // tokens x 32 columns per pass, 8 lanes per token. The token index is
        // stored XOR-swizzled by the column's quad, x' = x ^ 4 ((j >> 2) & 7),
        // so that the scattered stores fall on distinct banks while a token
        // quad stays one 16-byte group for the product loop
        constexpr int kPasses = (kBT * 256) / (kNT * 4), kDepth = 16;
        for (int p0 = 0; p0 < kPasses; p0 += kDepth) {
            float4 v[kDepth];
#pragma unroll
            for (int u = 0; u < kDepth; ++u) {
                const int pair = (p0 + u) * 4 + warp;       // (32-column group, token quad), 0..127
                const int j = (pair & 7) * 32 + 4 * (lane & 7), b = (pair >> 3) * 4 + (lane >> 3);
                v[u] = b0 + b < p.B ? __ldg(reinterpret_cast<const float4 *>(p.x + (size_t)(b0 + b) * p.cols +
                                                                              (size_t)i * 256 + j))
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < kDepth; ++u) {
                const int pair = (p0 + u) * 4 + warp;
                const int j = (pair & 7) * 32 + 4 * (lane & 7), b = (pair >> 3) * 4 + (lane >> 3);
                const int bs = b ^ (4 * ((j >> 2) & 7));
                Xs[(j + 0) * kXP + bs] = v[u].x;
                Xs[(j + 1) * kXP + bs] = v[u].y;
                Xs[(j + 2) * kXP + bs] = v[u].z;
                Xs[(j + 3) * kXP + bs] = v[u].w;
            }
        }
        __syncthreads();
        const float *wj = Wt + 4 * rq;
#pragma unroll 4
        for (int j = 0; j < 256; ++j) {
            const float4 w4 = *reinterpret_cast<const float4 *>(wj + j * kWP);
            const float4 x4 = *reinterpret_cast<const float4 *>(Xs + j * kXP + 4 * (tq ^ ((j >> 2) & 7)));
            const float w[4] = {w4.x, w4.y, w4.z, w4.w}, x[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int t = 0; t < 4; ++t) acc[a][t] = __fmaf_rn(w[a], x[t], acc[a][t]);
        }
        __syncthreads();
    }

    // epilogue: bias, residual add or SwiGLU, as forward_batch does next
    if (p.pair) {
#pragma unroll
        for (int a = 0; a < 4; a += 2) {   // slots 4rq + a (gate) and 4rq + a + 1 (up) of one index
            int row;
            if (slot_row(4 * rq + a, row) < 0) continue;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const int b = b0 + 4 * tq + t;
                if (b < p.B)
                    p.seg[0].out[(size_t)b * p.out_stride + row] = kore_swiglu(acc[a][t], acc[a + 1][t], p.exp_tab);
            }
        }
        return;
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        int row;
        if (slot_row(4 * rq + a, row) < 0) continue;
        const QSeg &q = p.seg[0];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int b = b0 + 4 * tq + t;
            if (b >= p.B) continue;
            const size_t o = (size_t)b * p.out_stride + row;
            float v = acc[a][t];
            if (p.out_mode == QOUT_RESIDUAL) v = __fadd_rn(p.resid[o], v);
            else if (q.bias) v = __fadd_rn(v, q.bias[row]);
            q.out[o] = v;
        }
    }
}

// out[b] = rmsnorm(x[b]) * w for each of the rows (kore.cpp:1367-1372), one CTA per row.
__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(const float *__restrict__ x, const float *__restrict__ w,
                                                           float *__restrict__ out, int n, float eps) {
    __shared__ double red[8];
    __shared__ float s_scale;
    const float *xr = x + (size_t)blockIdx.x * n;
    const float scale = block_rms_scale(xr, n, eps, red, &s_scale);
    float *o = out + (size_t)blockIdx.x * n;
    for (int i = threadIdx.x; i < n; i += blockDim.x) o[i] = __fmul_rn(__fmul_rn(xr[i], scale), w[i]);
}

}  // namespace

cudaError_t launch_batch_matmul(const BatchMatmulParams &p, cudaStream_t s) {
    if (!p.x || p.B <= 0 || p.cols <= 0 || p.cols % 256 || !p.seg[0].w || !p.seg[0].out || p.out_stride <= 0)
        return cudaErrorInvalidValue;
    if (p.pair && (!p.seg[1].w || p.seg[1].rows != p.seg[0].rows)) return cudaErrorInvalidValue;
    for (int i = 0; i < (p.pair ? 2 : 1); ++i)
        if (p.seg[i].type != 12 && p.seg[i].type != 14) return cudaErrorInvalidValue;
    if (p.out_mode == QOUT_RESIDUAL && !p.resid) return cudaErrorInvalidValue;
    if (cudaError_t e = ensure_smem_limit(reinterpret_cast<const void *>(batch_matmul_kernel), (int)kBatchSmem))
        return e;
    const int per = p.pair ? kRT / 2 : kRT;
    const dim3 grid((p.seg[0].rows + per - 1) / per, (p.B + kBT - 1) / kBT);
    batch_matmul_kernel<<<grid, kNT, kBatchSmem, s>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_rmsnorm_rows(const float *x, const float *w, float *out, int rows, int n, float eps,
                                cudaStream_t s) {
    if (!x || !w || !out || rows <= 0 || n <= 0) return cudaErrorInvalidValue;
    rmsnorm_rows_kernel<<<rows, 256, 0, s>>>(x, w, out, n, eps);
    return cudaGetLastError();
}

}  // namespace kore
