// attn.cuh — parameter blocks and launchers of the attention kernels.
#pragma once

#include <cstddef>
#include <cstdint>
#include <vector>

#include <cuda_runtime.h>

struct kore_cuda_ctx;

namespace kore {

constexpr int kMaxBatch = 256;    // queries per decode launch given by (seq, pos) list
constexpr int kMaxRanksDecode = 8;   // ranks of a KV split (kMaxRanks)
constexpr int kMaxSplits = 256;   // KV splits per (query, kv head)

// One layer's slice of the paged KV pool.
//   K of (page, head g, token t) at k[((page*G + g)*P + t)*D], V likewise at
//   k + v_off: every head's run of P tokens in a page is contiguous, so a
//   tile of consecutive tokens of one head is one linear bulk copy.
struct PagedKv {
    float *k;
    long long v_off;           // floats from the K pool to the V pool
    const int *page_table;     // [max_seqs][pt_stride] physical page per local page
    int pt_stride;
    int P, G, D, n_pages;
    int shard_rank, shard_count;
};

// An encoded TMA tensor map (the driver's 128-byte CUtensorMap), opaque here.
struct alignas(64) TmaDesc {
    unsigned long long w[16];
};

struct DecodeParams {
    // Tensor-core decode (attn_decode_tc_kernel, D = 128, one query): the
    // pools' K and V rows of 128 floats as 2-D TMA tensor maps (boxes of 32
    // floats x 16 rows, 128-byte swizzle); row of (page, g, t) in this
    // layer = k_row0 (v_row0) + (page*G + g)*P + t.
    TmaDesc tm_k, tm_v;
    long long k_row0, v_row0;
    int tc;                    // 1: launch the tensor-core kernel
    PagedKv kv;
    const float *q;            // [n_q][H*D] pre-RoPE
    const float *k_new;        // [n_q][G*D] pre-RoPE (append_new only)
    const float *v_new;        // [n_q][G*D]
    float *out;                // [n_q][H*D]
    float *lse;                // optional [n_q][H], log2-domain LSE of a partial result
    const float2 *rope;        // [ctx_max][D/2] (cos, sin) as kore.cpp:1405-1410
    float *part_o;             // split scratch [n_q][G][max_splits][R][D]
    float2 *part_ml;           // split scratch [n_q][G][max_splits][R] (max, sum)
    int *err;                  // device error word
    unsigned long long wait_ns;   // limit of each bounded wait for a K/V tile (then DEV_WAIT_FULL_TIMEOUT)
    float scale_log2;          // (1/sqrt(D)) * log2(e)
    int H, n_q, split_tokens, max_splits;
    int append_new;            // 1: the token at pos comes from k_new/v_new and is appended
    int contiguous;            // 1: query i is (seq0, pos0 + i); 0: seq[i], pos[i]
    int prefetch_ok;           // 1: the preceding kernel in the stream wrote no KV of this layer,
                               //    so KV tiles may be fetched before waiting for it
    int prefetch_stages;       // with prefetch_ok: ring stages per warp fetched before the wait
    int l2_inputs;             // with prefetch_ok: the CTA's q, new k/v and RoPE row asked into L2 first
                               //    (the rest right after it)
    int l2_prefetch_tokens;    // with prefetch_ok: positions of each split (from its start) that
                               //    are asked into L2 before the wait, so that HBM keeps streaming
                               //    while the preceding kernels finish
    int seq0, pos0;
    // A KV-split decode step (n_q = 1) with its exchange in the same launch:
    // the grid's first max_splits * G CTAs decode, each counting its arrival
    // per query head in x_arrivals after its partial is written; the last H
    // CTAs (one per query head) wait for their head's splits, merge them and
    // exchange over peer memory (exchange.cuh), writing x_out.
    int fused_exchange;
    int x_ranks;
    float *x_own;                  // this rank's exchange buffer
    float *x_peers[kMaxRanksDecode];
    size_t x_epoch_off;
    float *x_out;                  // merged output [H*D]
    int *x_arrivals;               // [H] splits arrived per query head; reset by the head's exchange CTA
    int seq[kMaxBatch];
    int pos[kMaxBatch];
};

struct AppendParams {
    PagedKv kv;
    const float *k;            // [n][G*D] pre-RoPE
    const float *v;            // [n][G*D]
    const float2 *rope;
    int *err;
    int seq, pos0, n;
};

constexpr int kMaxRanks = kMaxRanksDecode;

// One prefill chunk of one layer (attn_prefill.cu).
struct PrefillParams {
    PagedKv kv;                // the layer (unsharded)
    void *split;               // K/V operand tiles: [G][tiles][tile bytes]
    int tiles;                 // capacity of `split` per KV head, in tiles of prefill_tile_keys() keys
    const float *q;            // [n][H*D] pre-RoPE
    float *out;                // [n][H*D]
    const float2 *rope;
    int *err;
    float scale_log2;
    int seq, pos0, n, H, n_rep;
    // work list (prefill_plan): one int4 per CTA = {query head, query tile,
    // key tiles t0 | t1 << 16, split slot * 2 + part or -1}
    const int4 *items;
    float *part;               // [split slots][2 parts][kRows][D + 1]: a split half's O / l and LSE
    int *counters;             // [split slots]: halves done; reset to 0 by the merging half
    int n_items;
};

// Query slots of a rank's exchange buffer: one decode step uses one, a
// prefill chunk on a KV-split context is exchanged in pieces of this many.
constexpr int kExchangeQueries = 64;

// Positions of query `pos` that a shard holds (as PagedKv's page split) and
// the number of splits its decode runs over them (at least 1): the count the
// decode kernel, its split merge and the exchange all derive the same way.
__host__ __device__ inline int shard_count_below(int limit, int P, int NS, int rank) {
    const int F = limit / P, rem = limit - F * P;
    const int nfull_local = F > rank ? (F - rank + NS - 1) / NS : 0;
    return nfull_local * P + ((F % NS == rank) ? rem : 0);
}

// One layer's cross-GPU exchange of KV-sharded decode partials (peer_exchange.cu),
// for n_q consecutive queries (positions pos0 + i).
// Exchange buffer of each rank: (value, epoch) words [2 parities][n_ranks]
// [kExchangeQueries][H][D + 1] u64 at 0, the epochs [kExchangeQueries][H] u32
// at epoch_off; all zero at creation.
struct ExchangeParams {
    const float *local;            // this rank's partials: outputs [kExchangeQueries][H*D], then
                                   //   log2-domain LSEs [kExchangeQueries][H] (queries with one split)
    const float *part_o;           // or their splits, merged here (decode split scratch)
    const float2 *part_ml;
    int max_splits, split_tokens, n_rep;
    int pos0, append_new, P;       // the queries' positions and how the decode counted them
    float *own;                    // this rank's exchange buffer
    float *peers[kMaxRanks];       // every rank's exchange buffer as mapped here (own included)
    size_t epoch_off;              // per-(query, head) epochs in `own`
    float *out;                    // merged outputs [n_q][H*D]
    int *err;
    unsigned long long wait_ns;    // limit of the wait for a peer's partial (then DEV_PEER_TIMEOUT)
    int n_ranks, rank, H, D, n_q;
};

// Launch helpers (attn_decode.cu, kv_append.cu). Return cudaGetLastError().
// Decode kernel, followed (when grid_x > 1 and merge) by the split-merge kernel.
cudaError_t launch_attn_decode(const DecodeParams &p, int n_rep, int grid_x, cudaStream_t s, bool merge = true);
int decode_ctas_per_sm(int head_dim, int n_rep);
int decode_tile_tokens();
int decode_tc_tile_tokens();   // tokens per tile of the tensor-core decode (split lengths are multiples)
int decode_split_pages_max();
size_t decode_smem_bytes(int head_dim);
cudaError_t launch_kv_append(const AppendParams &p, cudaStream_t s);
void set_ctxless_error(const char *msg);
// A context's limits for the session server: positions per sequence,
// sequences, the uploaded model's vocabulary (0 without a model), device.
bool ctx_limits(const kore_cuda_ctx *c, int *ctx_max, int *max_seqs, int *n_vocab, int *device);
// The CUDA context current on this thread (the device's primary context
// unless the caller made another one current), as an opaque key; 0 if none.
uintptr_t current_cuda_context();
// Sets a kernel's dynamic shared memory limit once per CUDA context (the
// attribute belongs to the kernel as loaded in one context). Thread-safe.
cudaError_t ensure_smem_limit(const void *kernel, int bytes);
bool encode_kv_map(const float *base, size_t rows, TmaDesc *out);   // rows of 128 floats as a TMA tensor map
size_t prefill_tile_bytes(int head_dim);
// bytes of one split slot of PrefillParams::part
size_t prefill_slot_bytes(int head_dim);
// Bytes from one block of an uploaded matrix to the next. Q4_K blocks are
// stored as GGUF has them (144 bytes, a multiple of 16); each 210-byte Q6_K
// block is followed by 2 zero bytes, so that every block, and every 32-bit
// word a product lane reads from it, is 4-byte aligned (the block's bytes are
// GGUF's, unchanged).
constexpr int kQ4Stride = 144, kQ6Stride = 212;
__host__ __device__ constexpr int block_stride(int type) { return type == 12 ? kQ4Stride : kQ6Stride; }

// One weight matrix of a product launch: rows of uploaded blocks (type 12 =
// Q4_K, 14 = Q6_K, block_stride apart), out[r] = row r . x (+ bias[r]). The
// buffer holding w extends at least 16 bytes past the matrix.
struct QSeg {
    const uint8_t *w;
    const float *bias;
    float *out;
    int type, rows;
};
// What a product launch does with its input vector and its rows (proj.cu).
enum QInMode : int {
    QIN_QUANT = 0,     // quantise x to Q8_K
    QIN_RMSNORM = 1,   // quantise RMSNorm(x) * norm_w (kore.cpp:1367-1372)
};
enum QOutMode : int {
    QOUT_STORE = 0,      // out[r] = row (+ bias[r])
    QOUT_RESIDUAL = 1,   // out[r] = resid[r] + row (the residual add; out may be resid)
    QOUT_SWIGLU = 2,     // paired segments: seg[0].out[i] = SwiGLU(seg 0 row i, seg 1 row i)
    QOUT_ARGMAX = 3,     // out[r] = row, and *argmax = max over rows of the (value, first row) key
};
// Products of up to three matrices with one fp32 vector x [cols] (16-byte
// aligned), quantised to Q8_K inside the kernel; `grid` CTAs, one per SM.
// stages and row_slot are what qmatvec_config gives for cols and the largest
// block size of the segments; err receives DEV_WAIT_FULL_TIMEOUT if a weight
// copy never lands.
struct QMatvecParams {
    QSeg seg[3];
    int n_seg;
    int cols;
    int pair_segments;            // 1: group i = row i of seg 0 and of seg 1 (equal row counts)
    int in_mode, out_mode;
    int stages, row_slot;
    const float *x;
    const float *norm_w;          // QIN_RMSNORM weight [cols], 16-byte aligned
    float eps;                    // QIN_RMSNORM epsilon
    int rms_sequential;           // QIN_RMSNORM: always sum the squares in kore's order (launch_qmatvec sets it)
    const float *resid;           // QOUT_RESIDUAL
    unsigned long long *argmax;   // QOUT_ARGMAX: orderable (value << 32 | ~row) key, zeroed beforehand
    int *err;
    unsigned long long exp_tab[32];   // QOUT_SWIGLU: bits(2^(i/32)) - (i << 47), from the host's exp2
};
constexpr size_t kQmatvecMaxSmem = 227 * 1024;
// Ring stages per warp and bytes per row slot for a launch over cols with
// the given largest block size; returns the dynamic shared memory it needs.
size_t qmatvec_config(int cols, int max_block_bytes, int *stages, int *row_slot);
cudaError_t launch_qmatvec(const QMatvecParams &p, int grid, cudaStream_t s);
#ifdef KORE_TRACE
int proj_trace_read(void *host, unsigned max_recs, unsigned *n_recs);   // trace build only
int proj_trace_reset();
#endif

// The embedding rows of n_tokens tokens (step.cu): row z of x =
// get_row(table, token z) (kore.cpp:384-407) for table type 0 (F32), 1 (F16),
// 30 (BF16), 12 (Q4_K) or 14 (Q6_K); the tokens come from token_dev [n_tokens]
// when set, else the one `token`; also clears *key (the argmax key the
// step's logits product fills).
struct EmbedParams {
    const uint8_t *table;
    size_t row_bytes;
    int type, n_vocab, n_embd, token, n_tokens;
    const int *token_dev;
    float *x;
    unsigned long long *key;
    int *err;
};
cudaError_t launch_embed(const EmbedParams &p, cudaStream_t s);
// kore's matmul_batch_float (kore.cpp:783-845) on B tokens (batch_proj.cu):
// out[b * out_stride + r] = the fused multiply-add chain over the columns of
// the dequantised row r of seg[0] and x[b] (+ bias, or added to resid at the
// same place); with pair, seg[0].out[b * out_stride + i] = SwiGLU of gate row
// i (seg 0) and up row i (seg 1).
struct BatchMatmulParams {
    QSeg seg[2];
    int pair;
    int cols, B;
    const float *x;          // [B][cols]
    int out_mode;            // QOUT_STORE or QOUT_RESIDUAL (ignored with pair)
    const float *resid;
    int out_stride;
    unsigned long long exp_tab[32];
};
cudaError_t launch_batch_matmul(const BatchMatmulParams &p, cudaStream_t s);
// out[row] = kore's rmsnorm of x[row] times w, for `rows` rows of n values.
cudaError_t launch_rmsnorm_rows(const float *x, const float *w, float *out, int rows, int n, float eps, cudaStream_t s);
// token = the index in an argmax key (-1 for an empty key), after the
// preceding kernel (programmatic dependency).
cudaError_t launch_token(const unsigned long long *key, int *token, cudaStream_t s);

// Work list of a prefill chunk (pos0, n) over H heads on num_sms SMs: one
// item per (query head, 128-row query tile), the heaviest ones possibly split
// in two key ranges, in the dispatch order that finishes first by a replay of
// the in-order CTA dispatch. Returns the number of split slots used.
int prefill_plan(int pos0, int n, int H, int num_sms, std::vector<int4> &items);
int prefill_tile_keys();
cudaError_t launch_prefill(const PrefillParams &p, cudaStream_t s);
cudaError_t launch_peer_exchange(const ExchangeParams &p, cudaStream_t s);
// Merges n_parts partials of n_q queries each (part r: outputs [n_q][H*D]
// then LSEs [n_q][H], parts one after another) into out [n_q][H*D].
cudaError_t launch_lse_merge(const float *parts, int n_parts, int n_q, int H, int D, float *out, cudaStream_t s);

}  // namespace kore
