// step.cu — the two small kernels around the device-resident decode step:
// the token's embedding row at its start and the greedy token at its end.
//
// kore's forward() begins with get_row(tok_embd, token) (kore.cpp:1402-1403,
// get_row kore.cpp:384-407): the token's row of the embedding table,
// dequantised to fp32, becomes the residual stream x. embed_kernel does that
// on the device for every table type kore reads (F32, F16, BF16, Q4_K,
// Q6_K), with kore's own rounding: Q4_K values are d1 * q - m1 with
// d1 = d * scale and m1 = dmin * min rounded separately (kore.cpp:337-354),
// Q6_K values are (d * scale) * (q - 32) (kore.cpp:359-381). It also clears
// the argmax key that the logits product fills.
//
// The logits product (proj.cu, QOUT_ARGMAX) leaves the greedy choice of
// sample_token at temperature 0 (kore.cpp:1601-1603) as a key: the largest
// logit, then the smallest index. token_kernel turns the key into the token.

#include "attn.cuh"
#include "common.cuh"

#include <cuda_fp16.h>

namespace kore {
namespace {

__device__ __forceinline__ float f16_at(const uint8_t *p) {
    return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

// kore's get_scale_min_k4 (kore.cpp:327-335): the 6-bit scale and min of
// sub-block j from the 12 packed bytes q.
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t *q, int &sc, int &mn) {
    if (j < 4) {
        sc = q[j] & 63;
        mn = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 0x0F) | ((q[j - 4] >> 6) << 4);
        mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// Value j (0..255) of a Q4_K block (kore.cpp:337-354).
__device__ __forceinline__ float q4k_value(const uint8_t *b, int j) {
    const int chunk = j >> 6, jj = j & 63, l = jj & 31;
    int sc, mn;
    scale_min_k4(2 * chunk + (jj >> 5), b + 4, sc, mn);
    const float d1 = __fmul_rn(f16_at(b), (float)sc), m1 = __fmul_rn(f16_at(b + 2), (float)mn);
    const int q = b[16 + 32 * chunk + l];
    const int nib = jj < 32 ? (q & 0x0F) : (q >> 4);
    return __fsub_rn(__fmul_rn(d1, (float)nib), m1);
}

// Value j (0..255) of a Q6_K block (kore.cpp:359-381).
__device__ __forceinline__ float q6k_value(const uint8_t *b, int j) {
    const int half = j >> 7, jj = j & 127, g = jj >> 5, l = jj & 31;
    const uint8_t *ql = b + 64 * half, *qh = b + 128 + 32 * half;
    const int8_t *sc = reinterpret_cast<const int8_t *>(b + 192 + 8 * half);
    const int lo = (g & 1) ? ql[l + 32] : ql[l];
    const int q = (((g & 2) ? (lo >> 4) : (lo & 0x0F)) | (((qh[l] >> (2 * g)) & 3) << 4)) - 32;
    return __fmul_rn(__fmul_rn(f16_at(b + 208), (float)sc[(l >> 4) + 2 * g]), (float)q);
}

__global__ void __launch_bounds__(256) embed_kernel(const __grid_constant__ EmbedParams p) {
    int t = p.token_dev ? *p.token_dev : p.token;
    if (t < 0 || t >= p.n_vocab) {
        if (threadIdx.x == 0) raise_error(p.err, DEV_BAD_TOKEN);
        t = 0;
    }
    const uint8_t *row = p.table + (size_t)t * p.row_bytes;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.n_embd; i += gridDim.x * blockDim.x) {
        float v;
        switch (p.type) {
            case 0: v = reinterpret_cast<const float *>(row)[i]; break;
            case 1: v = f16_at(row + 2 * i); break;
            case 30: v = __uint_as_float((uint32_t)(row[2 * i] | (row[2 * i + 1] << 8)) << 16); break;
            case 12: v = q4k_value(row + (size_t)(i >> 8) * 144, i & 255); break;
            default: v = q6k_value(row + (size_t)(i >> 8) * 210, i & 255); break;
        }
        p.x[i] = v;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0 && p.key) *p.key = 0ull;
}

__global__ void token_kernel(const unsigned long long *key, int *token) {
    grid_dep_wait();
    const unsigned long long k = *key;
    *token = k ? (int)(0xFFFFFFFFu - (uint32_t)k) : -1;
}

}  // namespace

cudaError_t launch_embed(const EmbedParams &p, cudaStream_t s) {
    if (!p.table || !p.x || p.n_embd <= 0 || p.n_vocab <= 0) return cudaErrorInvalidValue;
    if (p.type != 0 && p.type != 1 && p.type != 30 && p.type != 12 && p.type != 14) return cudaErrorInvalidValue;
    embed_kernel<<<(p.n_embd + 255) / 256 < 32 ? (p.n_embd + 255) / 256 : 32, 256, 0, s>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_token(const unsigned long long *key, int *token, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(1);
    cfg.stream = s;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, token_kernel, key, token);
}

}  // namespace kore
