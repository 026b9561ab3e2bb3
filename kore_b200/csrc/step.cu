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
#include "kore_math.cuh"

namespace kore {
namespace {

__global__ void __launch_bounds__(256) embed_kernel(const __grid_constant__ EmbedParams p) {
    const int z = blockIdx.y;   // token z of the batch: row z of x
    int t = p.token_dev ? p.token_dev[z] : p.token;
    if (t < 0 || t >= p.n_vocab) {
        if (threadIdx.x == 0) raise_error(p.err, DEV_BAD_TOKEN);
        t = 0;
    }
    const uint8_t *row = p.table + (size_t)t * p.row_bytes;
    float *x = p.x + (size_t)z * p.n_embd;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.n_embd; i += gridDim.x * blockDim.x) {
        float v;
        switch (p.type) {
            case 0: v = reinterpret_cast<const float *>(row)[i]; break;
            case 1: v = f16_at(row + 2 * i); break;
            case 30: v = __uint_as_float((uint32_t)(row[2 * i] | (row[2 * i + 1] << 8)) << 16); break;
            case 12: v = q4k_value(row + (size_t)(i >> 8) * 144, i & 255); break;
            default: v = q6k_value(row + (size_t)(i >> 8) * 210, i & 255); break;
        }
        x[i] = v;
    }
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0 && p.key) *p.key = 0ull;
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
    if (p.n_tokens <= 0 || p.n_tokens > 65535 || (p.n_tokens > 1 && !p.token_dev)) return cudaErrorInvalidValue;
    const dim3 grid((p.n_embd + 255) / 256 < 32 ? (p.n_embd + 255) / 256 : 32, p.n_tokens);
    embed_kernel<<<grid, 256, 0, s>>>(p);
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
