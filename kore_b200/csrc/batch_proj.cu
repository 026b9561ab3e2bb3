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
// is what batch_matmul_kernel does: a CTA holds a tile of 16 weight rows x
// up to 64 tokens, dequantises the tile's rows one block at a time into
// shared memory with kore's rounding, stages the tokens' matching 256
// columns transposed beside them, and each thread advances 8 chains (2 rows
// x 4 tokens) through the block. CUDA cores, not tensor cores: a tensor-core
// product sums in its own order and could not give kore's values.
//
// The epilogues do what forward_batch does next to each product: the bias
// add (kore.cpp:1530-1532), the residual add x += o (:1568-1571, :1588-1591)
// and, for the gate/up pair (a tile of 8 gate rows and the same 8 up rows),
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

constexpr int kRT = 16;          // weight rows per tile (pair mode: 8 gate + 8 up rows)
constexpr int kBT = 64;          // tokens per tile
constexpr int kNT = 128;         // threads: (kRT / 2) row pairs x (kBT / 4) token quads
constexpr int kWPitch = 257;     // shared row pitch of the dequantised weights (bank spread)
constexpr int kXPitch = kBT + 4; // shared row pitch of the transposed tokens (16-byte rows)

constexpr size_t kXsFloats = (size_t)256 * kXPitch;
constexpr size_t kBatchSmem = (kXsFloats + (size_t)kRT * kWPitch) * sizeof(float);

__global__ void __launch_bounds__(kNT) batch_matmul_kernel(const __grid_constant__ BatchMatmulParams p) {
    extern __shared__ __align__(16) float bsm[];
    float *Xs = bsm;               // [256][kXPitch]: the tokens' 256 columns of one block, transposed
    float *Ws = bsm + kXsFloats;   // [kRT][kWPitch]: the tile's rows of that block, dequantised
    const int tid = threadIdx.x;
    const int rp = tid >> 4, bq = tid & 15;          // row pair, token quad
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
    float acc[2][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int t = 0; t < 4; ++t) acc[a][t] = 0.f;

    for (int i = 0; i < nb; ++i) {
        // dequantise block i of the tile's rows, kore's rounding (8 threads per row)
        {
            const int s = tid >> 3, j0 = (tid & 7) * 32;
            int row;
            const int sg = slot_row(s, row);
            float *dst = Ws + s * kWPitch;
            if (sg < 0) {
                for (int j = j0; j < j0 + 32; ++j) dst[j] = 0.f;
            } else {
                const QSeg &q = p.seg[sg];
                const bool q4 = q.type == 12;
                const uint8_t *blk = q.w + ((size_t)row * nb + i) * block_stride(q.type);
                if (q4)
                    for (int j = j0; j < j0 + 32; ++j) dst[j] = q4k_value(blk, j);
                else
                    for (int j = j0; j < j0 + 32; ++j) dst[j] = q6k_value(blk, j);
            }
        }
        // the tokens' columns of block i, transposed: Xs[j][b]
        for (int e = tid; e < kBT * 256; e += kNT) {
            const int b = e >> 8, j = e & 255;
            Xs[j * kXPitch + b] = b0 + b < p.B ? p.x[(size_t)(b0 + b) * p.cols + (size_t)i * 256 + j] : 0.f;
        }
        __syncthreads();
        const float *w0 = Ws + (2 * rp) * kWPitch, *w1 = w0 + kWPitch;
        const float *xs = Xs + 4 * bq;
#pragma unroll 8
        for (int j = 0; j < 256; ++j) {
            const float a = w0[j], c = w1[j];
            const float4 xv = *reinterpret_cast<const float4 *>(xs + j * kXPitch);
            acc[0][0] = __fmaf_rn(a, xv.x, acc[0][0]);
            acc[0][1] = __fmaf_rn(a, xv.y, acc[0][1]);
            acc[0][2] = __fmaf_rn(a, xv.z, acc[0][2]);
            acc[0][3] = __fmaf_rn(a, xv.w, acc[0][3]);
            acc[1][0] = __fmaf_rn(c, xv.x, acc[1][0]);
            acc[1][1] = __fmaf_rn(c, xv.y, acc[1][1]);
            acc[1][2] = __fmaf_rn(c, xv.z, acc[1][2]);
            acc[1][3] = __fmaf_rn(c, xv.w, acc[1][3]);
        }
        __syncthreads();
    }

    // epilogue: bias, residual add or SwiGLU, as forward_batch does next
    if (p.pair) {
        int row;
        if (slot_row(2 * rp, row) < 0) return;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int b = b0 + 4 * bq + t;
            if (b < p.B) p.seg[0].out[(size_t)b * p.out_stride + row] = kore_swiglu(acc[0][t], acc[1][t], p.exp_tab);
        }
        return;
    }
#pragma unroll
    for (int a = 0; a < 2; ++a) {
        int row;
        if (slot_row(2 * rp + a, row) < 0) continue;
        const QSeg &q = p.seg[0];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int b = b0 + 4 * bq + t;
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
