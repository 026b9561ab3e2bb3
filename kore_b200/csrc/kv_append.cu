// kv_append.cu — RoPE of new keys and their store, with the values, into the
// paged fp32 KV pool (sm_100a).
//
// Replaces kore.cpp:1425 + :1429-1430 (one token) and :1534-1538 (a prefill
// batch): k is rotated with the angle tables of its own position and stored,
// v is stored unrotated. One warp per (token, KV head); lane j handles dims
// [VEC*j, VEC*j+VEC) and reads the partner element (i xor D/2) of the NEOX
// pair directly, so no shuffle is needed. The rotation is rounded exactly as
// kore's rope_neox, so the stored keys are bit-identical to kore's cache rows.

#include "attn.cuh"
#include "common.cuh"

namespace kore {
namespace {

template <int D>
__global__ void __launch_bounds__(256) kv_append_kernel(const __grid_constant__ AppendParams p) {
    constexpr int VEC = D / 32, HALF = D / 2;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const PagedKv &kv = p.kv;
    const int G = kv.G, P = kv.P, NS = kv.shard_count;
    if (warp >= p.n * G) return;
    const int z = warp / G, g = warp - z * G;
    const int pos = p.pos0 + z;
    const int gp = pos / P;
    if (gp % NS != kv.shard_rank) return;              // another shard holds this position
    const int ph = kv.page_table[(size_t)p.seq * kv.pt_stride + gp / NS];
    if (ph < 0 || ph >= kv.n_pages) {
        if (lane == 0) raise_error(p.err, DEV_BAD_PAGE);
        return;
    }
    const float *ks = p.k + ((size_t)z * G + g) * D;
    const float *vs = p.v + ((size_t)z * G + g) * D;
    const float2 *cs = p.rope + (size_t)pos * HALF;
    float *kd = kv.k + (((size_t)ph * G + g) * P + (pos - gp * P)) * D;
    float kr[VEC], vr[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
        const int i = lane * VEC + j;
        const float x = __ldg(ks + i), y = __ldg(ks + (i ^ HALF));
        const float2 a = __ldg(cs + (i & (HALF - 1)));
        kr[j] = i < HALF ? rope_lo(x, y, a.x, a.y) : rope_hi(y, x, a.x, a.y);
        vr[j] = __ldg(vs + i);
    }
    if constexpr (VEC == 4) {
        *reinterpret_cast<float4 *>(kd + lane * 4) = make_float4(kr[0], kr[1], kr[2], kr[3]);
        *reinterpret_cast<float4 *>(kd + kv.v_off + lane * 4) = make_float4(vr[0], vr[1], vr[2], vr[3]);
    } else {
        *reinterpret_cast<float2 *>(kd + lane * 2) = make_float2(kr[0], kr[1]);
        *reinterpret_cast<float2 *>(kd + kv.v_off + lane * 2) = make_float2(vr[0], vr[1]);
    }
}

}  // namespace

cudaError_t launch_kv_append(const AppendParams &p, cudaStream_t s) {
    const long long warps = (long long)p.n * p.kv.G;
    const int blocks = (int)((warps * 32 + 255) / 256);
    if (blocks == 0) return cudaSuccess;
    if (p.kv.D == 128) kv_append_kernel<128><<<blocks, 256, 0, s>>>(p);
    else if (p.kv.D == 64) kv_append_kernel<64><<<blocks, 256, 0, s>>>(p);
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
}

}  // namespace kore
