// capi.cu — the C ABI of include/kore_cuda.h: context, paged KV pool, RoPE
// tables, staging of host buffers, and the launch decisions (split sizing).
//
// Host-side restatements of reference arithmetic in this file:
//   inv_freq  kore.cpp:1337-1339  (float)pow((double)rope_base, -2.0*i/head_dim)
//   angles    kore.cpp:1405-1410  (float)cos/sin((double)pos * inv_freq[i])
// They are computed once per context for every position below ctx_max, so the
// device rotates with exactly the tables kore would build for that position.

#include "../../include/kore_cuda.h"
#include "attn.cuh"
#include "common.cuh"

#include <cuda.h>   // CUtensorMap and its enums (the encoder is resolved at run time)

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

using namespace kore;

struct kore_cuda_ctx {
    kore_cuda_cfg cfg{};
    int H = 0, G = 0, D = 0, R = 0, kvd = 0, P = 0, NS = 1, rank = 0;
    int pages_per_seq = 0;      // local page-table stride
    int n_pages = 0;
    int num_sms = 148;
    // L2 budget of the decode's early fetch (KORE_CUDA_L2_PREFETCH_MB). Off by
    // default: on B200 it measured slower at 32 and 64 MB, on one GPU and on
    // two (the prefetched lines did not outlive their wait)
    long long l2_prefetch_bytes = 0;
    // limit of the decode and exchange kernels' bounded waits (kore_cuda_set_wait_limit)
    unsigned long long wait_ns = kWaitNs;
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    float *kv = nullptr;        // [n_layer][2][n_pages][G][P][D]
    size_t layer_floats = 0;
    long long v_off = 0;
    // the pool as rows of D = 128 floats for the tensor-core decode's TMA
    // boxes (32 floats x 16 rows, 128-byte swizzle). KORE_CUDA_TC_DECODE=1
    // runs single queries on the tensor-core kernel: measured no faster
    // (both kernels stream at the HBM limit) and its split-bf16 products
    // round more (~1e-6 relative), which flipped a near-tie greedy token of
    // the 3B parity model, so the CUDA-core kernel is the default
    kore::TmaDesc kv_map{};
    bool kv_map_ok = false;
    bool tc_decode = false;
    // single-query host-buffer decode returns through mapped memory and a
    // polled flag (KORE_CUDA_RET_MAPPED=0: copy back and synchronise)
    bool ret_mapped = true;
    int *pt_d = nullptr;
    std::vector<int> pt_h;      // [max_seqs][pages_per_seq]
    std::vector<int> free_pages;
    std::vector<int> seq_alloc; // local pages held per sequence
    std::vector<int> seq_len;   // [max_seqs][n_layer] positions held
    float2 *rope_d = nullptr;   // [ctx_max][D/2]
    float *part_o = nullptr;
    float2 *part_ml = nullptr;
    size_t part_slots = 0;      // (query, kv head, split) slots of split scratch
    int *err_d = nullptr;
    float *dev_stage = nullptr;
    size_t dev_stage_floats = 0;
    float *host_stage = nullptr;        // pinned, mapped into the device's address space
    const float *host_stage_dev = nullptr;   // its device address (null: copies go through the copy engine)
    // Return buffer of the single-query host-buffer decode (pinned, mapped):
    // word 0 the sequence number of the last finished call, word 1 its device
    // error word, from byte kRetPad the output, written in place by the kernels
    unsigned *host_ret = nullptr;
    void *host_ret_dev = nullptr;
    size_t host_ret_floats = 0;
    unsigned ret_seq = 0;
    size_t host_stage_floats = 0;
    int *host_err = nullptr;
    int last_kv_layer = -1;     // layer whose KV the most recent kernel of this context wrote
    // cross-GPU exchange of KV-sharded partials (peer_exchange.cu)
    float *xbuf = nullptr;      // this rank's exchange buffer, shared with the peers over CUDA IPC
    size_t x_epoch_off = 0, x_local_off = 0, x_bytes = 0;
    // whether the decode after a sharded decode may fetch KV while the peer
    // exchange still runs (KORE_CUDA_SHARD_PREFETCH=0 turns it off)
    bool shard_prefetch = true;
    bool hold_prefetch = false;   // set: the next decode waits before its first KV fetch
    // KV-split decode: the exchange in the decode's own launch (KORE_CUDA_FUSED_EXCHANGE=0 turns it off)
    bool fused_exchange = true;
    // one GPU: the split merge of a single-query decode in the decode's own
    // launch (KORE_CUDA_FUSED_MERGE=0 launches split_merge_kernel instead)
    bool fused_merge = true;
    int *x_arrivals = nullptr;    // [H] arrivals per query head of a fused launch
    int prefetch_stages = 3;      // ring stages fetched early (KORE_CUDA_PREFETCH_STAGES)
    bool l2_inputs = true;        // the decode's q / new token / RoPE row asked into L2 first (KORE_CUDA_L2_INPUTS)
    int shard_ctas = 0;           // decode CTAs aimed at on a KV-split context (KORE_CUDA_SHARD_CTAS; 0: 2 per SM)
    int decode_ctas = 0;          // decode CTAs aimed at otherwise (KORE_CUDA_DECODE_CTAS; 0: 2 per SM)
    // batched decode: split-length factor chosen for the last batch shape
    long long split_key[3] = {-1, -1, -1};
    double split_f = 1.0;
    float *peers[kMaxRanks] = {};
    bool peers_open = false;
    // prefill: K/V operand tiles of the current chunk's layer (attn_prefill.cu)
    void *split = nullptr;
    int split_tiles = 0;        // capacity per KV head, in tiles of prefill_tile_keys() positions
    // prefill work list of the last chunk shape (prefill_plan), its split
    // halves' slots and arrival counters
    int pf_pos0 = -1, pf_n = -1, pf_items_n = 0;
    int4 *pf_items = nullptr;
    size_t pf_items_cap = 0;
    float *pf_part = nullptr;
    int *pf_counters = nullptr;
    int pf_slots_cap = 0;
    // attention-block projections (proj.cu): per layer wq | wk | wv | wo in
    // GGUF blocks, each 256-byte aligned with padding behind, and bq | bk | bv
    struct LayerProj {
        uint8_t *w = nullptr;
        float *bias = nullptr;
        bool has_bias = false;
        int type[4] = {0, 0, 0, 0};
        int rows[4] = {0, 0, 0, 0};
        size_t off[4] = {0, 0, 0, 0};
    };
    std::vector<LayerProj> proj;
    float *blk = nullptr;       // q [H*D] | k [kvd] | v [kvd] | att [H*D]
    // the rest of the model for the device-resident decode step
    // (kore_cuda_set_model): embedding table, per-layer norms and
    // feed-forward weights, output norm and logits matrix, step buffers
    struct LayerFfn {
        float *norms = nullptr;   // attn_norm [E] | ffn_norm [E]
        uint8_t *w = nullptr;     // w_gate | w_up | w_down, 256-byte aligned, padded
        int type[3] = {0, 0, 0};
        size_t off[3] = {0, 0, 0};
    };
    struct Model {
        bool ready = false;
        int n_ff = 0, n_vocab = 0, tok_type = 0, out_type = 0;
        float eps = 0.f;
        size_t tok_row_bytes = 0;
        uint8_t *tok = nullptr;
        float *out_norm = nullptr;
        uint8_t *out_w = nullptr;
        std::vector<LayerFfn> layers;
        float *x = nullptr;       // residual stream [E]
        float *act = nullptr;     // SwiGLU output [n_ff]
        float *logits = nullptr;  // [n_vocab]
        unsigned long long *key = nullptr;   // argmax key of the logits
        int *token = nullptr;     // [2]: a step's input and output token (device-side steps)
        unsigned long long exp_tab[32] = {};
        // forward_batch buffers for up to pf_cap tokens: x, normed x, q, k, v,
        // attention output, SwiGLU output, token ids
        int pf_cap = 0;
        float *bx = nullptr, *bxb = nullptr, *bq = nullptr, *bk = nullptr, *bv = nullptr, *batt = nullptr,
              *bact = nullptr;
        int *btok = nullptr;
    } model;
    std::string msg;
};

namespace {

thread_local std::string g_create_msg = "no error";

}  // namespace

namespace kore {
bool ctx_limits(const kore_cuda_ctx *c, int *ctx_max, int *max_seqs, int *n_vocab, int *device) {
    if (!c) return false;
    *ctx_max = c->cfg.ctx_max;
    *max_seqs = c->cfg.max_seqs;
    *n_vocab = c->model.ready ? c->model.n_vocab : 0;
    *device = c->cfg.device;
    return true;
}

// Message for calls that have no context (read with kore_cuda_last_error(NULL)).
void set_ctxless_error(const char *msg) { g_create_msg = msg; }

uintptr_t current_cuda_context() {
    // the driver's cuCtxGetCurrent, resolved once through the runtime (the
    // library links the static runtime only)
    using get_current_fn = int (*)(void **);
    static get_current_fn fn = []() -> get_current_fn {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        return reinterpret_cast<get_current_fn>(f);
    }();
    void *c = nullptr;
    if (!fn || fn(&c) != 0) return 0;
    return reinterpret_cast<uintptr_t>(c);
}

// Encodes `rows` rows of 128 floats at `base` as a 2-D TMA tensor map with
// boxes of 32 floats x 16 rows and the 128-byte swizzle (the tensor-core
// decode's K/V tiles). The driver's encoder is resolved at run time; false
// when it or the encoding is unavailable (the CUDA-core decode is used then).
bool encode_kv_map(const float *base, size_t rows, TmaDesc *out) {
    using encode_fn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    static encode_fn fn = []() -> encode_fn {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        return reinterpret_cast<encode_fn>(f);
    }();
    static_assert(sizeof(CUtensorMap) == sizeof(TmaDesc), "tensor map size");
    if (!fn || !base || rows == 0 || rows >= (1ull << 31) || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
    const cuuint64_t dims[2] = {128, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {128 * sizeof(float)};
    const cuuint32_t box[2] = {32, 16};
    const cuuint32_t estr[2] = {1, 1};
    CUtensorMap m;
    if (fn(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    memcpy(out, &m, sizeof m);
    return true;
}

cudaError_t ensure_smem_limit(const void *kernel, int bytes) {
    static std::mutex mu;
    static std::vector<std::pair<const void *, uintptr_t>> done;
    int dev = 0;
    if (cudaError_t e = cudaGetDevice(&dev)) return e;   // makes the device's primary context current if none is
    const uintptr_t ctx = current_cuda_context();
    std::lock_guard<std::mutex> lk(mu);
    for (const auto &d : done)
        if (d.first == kernel && d.second == ctx && ctx != 0) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess && ctx != 0) done.emplace_back(kernel, ctx);
    return e;
}
}  // namespace kore

namespace {

int fail(kore_cuda_ctx *c, int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (c) c->msg = buf;
    else g_create_msg = buf;
    return code;
}

#define CK(call)                                                                                   \
    do {                                                                                           \
        cudaError_t e_ = (call);                                                                   \
        if (e_ != cudaSuccess)                                                                     \
            return fail(c, e_ == cudaErrorMemoryAllocation ? KORE_CUDA_ENOMEM : KORE_CUDA_ECUDA,    \
                        "%s: %s", #call, cudaGetErrorString(e_));                                  \
    } while (0)

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) == cudaSuccess && prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

constexpr size_t kPartSlots = 8192;

// Local pages (held by this shard) among global pages [0, gpages).
int local_pages(const kore_cuda_ctx *c, int gpages) {
    return gpages > c->rank ? (gpages - c->rank + c->NS - 1) / c->NS : 0;
}

// Cached positions below `limit` held by this shard (same formula as the kernel).
int local_count(const kore_cuda_ctx *c, int limit) {
    const int F = limit / c->P, rem = limit - F * c->P;
    return local_pages(c, F) * c->P + ((F % c->NS == c->rank) ? rem : 0);
}

PagedKv layer_kv(const kore_cuda_ctx *c, int layer) {
    PagedKv kv;
    kv.k = c->kv + (size_t)layer * c->layer_floats;
    kv.v_off = c->v_off;
    kv.page_table = c->pt_d;
    kv.pt_stride = c->pages_per_seq;
    kv.P = c->P;
    kv.G = c->G;
    kv.D = c->D;
    kv.n_pages = c->n_pages;
    kv.shard_rank = c->rank;
    kv.shard_count = c->NS;
    return kv;
}

int check_seq_layer(kore_cuda_ctx *c, int seq, int layer) {
    if (seq < 0 || seq >= c->cfg.max_seqs) return fail(c, KORE_CUDA_ERANGE, "seq %d outside [0, %d)", seq, c->cfg.max_seqs);
    if (layer < 0 || layer >= c->cfg.n_layer)
        return fail(c, KORE_CUDA_ERANGE, "layer %d outside [0, %d)", layer, c->cfg.n_layer);
    return KORE_CUDA_OK;
}

// Positions [pos0, pos0+n) may be written when pos0 does not leave a hole
// below it and the range stays inside the context (kore.cpp:1400, :1490).
int check_range(kore_cuda_ctx *c, int seq, int layer, int pos0, int n) {
    if (int rc = check_seq_layer(c, seq, layer)) return rc;
    if (n <= 0) return fail(c, KORE_CUDA_EINVAL, "n = %d must be positive", n);
    if (pos0 < 0 || (long long)pos0 + n > c->cfg.ctx_max)
        return fail(c, KORE_CUDA_ERANGE, "positions [%d, %lld) outside the context of %d", pos0,
                    (long long)pos0 + n, c->cfg.ctx_max);
    const int len = c->seq_len[(size_t)seq * c->cfg.n_layer + layer];
    if (pos0 > len)
        return fail(c, KORE_CUDA_ESTATE, "seq %d layer %d holds %d positions; cannot write at %d", seq, layer, len, pos0);
    return KORE_CUDA_OK;
}

// Makes sure every page holding positions below `end` is allocated.
int ensure_pages(kore_cuda_ctx *c, int seq, int end) {
    const int need = local_pages(c, (end + c->P - 1) / c->P);
    const int have = c->seq_alloc[seq];
    if (need <= have) return KORE_CUDA_OK;
    if ((size_t)(need - have) > c->free_pages.size())
        return fail(c, KORE_CUDA_ENOMEM, "KV page pool exhausted (%d pages per layer)", c->n_pages);
    int *row = c->pt_h.data() + (size_t)seq * c->pages_per_seq;
    for (int j = have; j < need; ++j) {
        row[j] = c->free_pages.back();
        c->free_pages.pop_back();
    }
    c->seq_alloc[seq] = need;
    CK(cudaMemcpyAsync(c->pt_d + (size_t)seq * c->pages_per_seq + have, row + have, (size_t)(need - have) * sizeof(int),
                       cudaMemcpyHostToDevice, c->stream));
    return KORE_CUDA_OK;
}

void note_len(kore_cuda_ctx *c, int seq, int layer, int end) {
    int &len = c->seq_len[(size_t)seq * c->cfg.n_layer + layer];
    len = std::max(len, end);
}

constexpr size_t kRetPad = 256;

// The return buffer for `floats` outputs; false when the host memory cannot
// be mapped (the call then copies its output back instead).
bool grow_ret(kore_cuda_ctx *c, size_t floats) {
    if (c->host_ret_dev && floats <= c->host_ret_floats) return true;
    if (c->host_ret) cudaFreeHost(c->host_ret);
    c->host_ret = nullptr;
    c->host_ret_dev = nullptr;
    c->host_ret_floats = 0;
    void *h = nullptr, *d = nullptr;
    if (cudaHostAlloc(&h, kRetPad + floats * sizeof(float), cudaHostAllocMapped) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    memset(h, 0, kRetPad);
    if (cudaHostGetDevicePointer(&d, h, 0) != cudaSuccess) {
        cudaGetLastError();
        cudaFreeHost(h);
        return false;
    }
    c->host_ret = static_cast<unsigned *>(h);
    c->host_ret_dev = d;
    c->host_ret_floats = floats;
    return true;
}

// Last kernel of a host-buffer call (after every other kernel of the call, in
// stream order): the call's device error word, then its sequence number, into
// the mapped return buffer the host polls.
__global__ void ret_done_kernel(const int *err, unsigned *ret, unsigned seq) {
    if (threadIdx.x == 0) {
        const int e = *reinterpret_cast<const volatile int *>(err);
        reinterpret_cast<volatile unsigned *>(ret)[1] = (unsigned)e;
        __threadfence_system();
        reinterpret_cast<volatile unsigned *>(ret)[0] = seq;
    }
}

int grow_stage(kore_cuda_ctx *c, size_t floats) {
    if (floats > c->dev_stage_floats) {
        if (c->dev_stage) cudaFree(c->dev_stage);
        c->dev_stage = nullptr;
        c->dev_stage_floats = 0;
        CK(cudaMalloc(&c->dev_stage, floats * sizeof(float)));
        c->dev_stage_floats = floats;
    }
    if (floats > c->host_stage_floats) {
        if (c->host_stage) cudaFreeHost(c->host_stage);
        c->host_stage = nullptr;
        c->host_stage_dev = nullptr;
        c->host_stage_floats = 0;
        CK(cudaHostAlloc(reinterpret_cast<void **>(&c->host_stage), floats * sizeof(float), cudaHostAllocMapped));
        c->host_stage_floats = floats;
        void *d = nullptr;
        if (cudaHostGetDevicePointer(&d, c->host_stage, 0) == cudaSuccess) c->host_stage_dev = static_cast<const float *>(d);
        else cudaGetLastError();   // not mapped: stage_in uses the copy engine
    }
    return KORE_CUDA_OK;
}

// Copies a small host-path input (q/k/v of a decode step, xb of an attention
// block) from the mapped pinned staging into device memory. As one kernel
// launched with a programmatic dependency that lets the next kernel start at
// once, the decode (or projection) after it fetches its first K/V tiles (or
// weights) while these reads cross the host link; it reads the inputs only
// after its dependency wait. The kernel itself waits for its predecessor
// before writing, so every kernel before it has completed by the time that
// wait returns, as after a copy-engine copy.
__global__ void stage_in_kernel(const float4 *__restrict__ src, float4 *__restrict__ dst, int n4) {
    grid_dep_launch();
    grid_dep_wait();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) dst[i] = src[i];
}

// The first `floats` of the host staging (16-byte multiple) to the device
// staging, on the context's stream.
int stage_in(kore_cuda_ctx *c, size_t floats) {
    const size_t bytes = floats * sizeof(float);
    if (!c->host_stage_dev || bytes % 16 || bytes > ((size_t)1 << 20)) {
        CK(cudaMemcpyAsync(c->dev_stage, c->host_stage, bytes, cudaMemcpyHostToDevice, c->stream));
        return KORE_CUDA_OK;
    }
    const int n4 = (int)(bytes / 16);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)std::min(64, (n4 + 1023) / 1024));
    cfg.blockDim = dim3(256);
    cfg.stream = c->stream;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    CK(cudaLaunchKernelEx(&cfg, stage_in_kernel, reinterpret_cast<const float4 *>(c->host_stage_dev),
                          reinterpret_cast<float4 *>(c->dev_stage), n4));
    return KORE_CUDA_OK;
}

// Reads and clears the device error word (stream-ordered, then synchronises).
// Waits for the stream after `extra` bytes following the device error word
// (kErrPad on) were queued for copying back with it; reports a device error.
constexpr size_t kErrPad = 256;   // bytes from the device error word to the decode output behind it

const char *device_error_text(int e) {
    switch (e) {
        case DEV_WAIT_FULL_TIMEOUT: return "bounded wait for a K/V tile or weight copy expired";
        case DEV_WAIT_EMPTY_TIMEOUT: return "bounded wait for a free stage expired";
        case DEV_BAD_PAGE: return "page table entry outside the pool";
        case DEV_PEER_TIMEOUT: return "a peer GPU's partial did not arrive within the wait limit";
        case DEV_BAD_TOKEN: return "token id outside the vocabulary";
        default: return "unknown device error code";
    }
}

int finish(kore_cuda_ctx *c, size_t extra = 0) {
    CK(cudaMemcpyAsync(c->host_err, c->err_d, extra ? kErrPad + extra : sizeof(int), cudaMemcpyDeviceToHost,
                       c->stream));
    CK(cudaStreamSynchronize(c->stream));
    const int e = *c->host_err;
    if (e != DEV_OK) {
        CK(cudaMemsetAsync(c->err_d, 0, sizeof(int), c->stream));
        // a prefill that gave up may have left a split half's arrival counted,
        // a fused exchange that gave up its head's arrivals
        if (c->pf_counters) CK(cudaMemsetAsync(c->pf_counters, 0, c->pf_slots_cap * sizeof(int), c->stream));
        if (c->x_arrivals) CK(cudaMemsetAsync(c->x_arrivals, 0, (size_t)c->H * sizeof(int), c->stream));
        CK(cudaStreamSynchronize(c->stream));
        return fail(c, KORE_CUDA_EDEVICE, "device error %d (%s)", e, device_error_text(e));
    }
    return KORE_CUDA_OK;
}

// Waits for the host-buffer call with sequence number `seq` by polling the
// mapped return buffer (no copy back, no stream synchronisation); the stream
// is queried now and then, so a failed launch or a lost flag ends in finish(),
// which reports the CUDA or device error. A device error word read back with
// the flag also goes through finish(), which clears it.
int wait_ret(kore_cuda_ctx *c, unsigned seq) {
    volatile unsigned *f = c->host_ret;
    uint64_t idle_polls = 0;
    for (uint64_t it = 1;; ++it) {
        if (f[0] == seq) break;
        if ((it & 4095) == 0 || idle_polls) {
            if (!idle_polls) {
                const cudaError_t q = cudaStreamQuery(c->stream);
                if (q != cudaErrorNotReady && q != cudaSuccess) return finish(c);
                if (q == cudaSuccess) idle_polls = 1;   // the flag's write is on its way
            } else if (++idle_polls > ((uint64_t)1 << 24)) {
                return finish(c);
            }
        }
#if defined(__x86_64__)
        __builtin_ia32_pause();
#endif
    }
    std::atomic_thread_fence(std::memory_order_acquire);
    if (f[1] != 0) return finish(c);
    return KORE_CUDA_OK;
}

int run_append(kore_cuda_ctx *c, int seq, int layer, int pos0, int n, const float *k, const float *v) {
    AppendParams ap;
    ap.kv = layer_kv(c, layer);
    ap.k = k;
    ap.v = v;
    ap.rope = c->rope_d;
    ap.err = c->err_d;
    ap.seq = seq;
    ap.pos0 = pos0;
    ap.n = n;
    CK(launch_kv_append(ap, c->stream));
    c->last_kv_layer = layer;
    return KORE_CUDA_OK;
}

// Launches the decode kernel for n_q queries. `contiguous` queries are
// (seq0, pos0 + i); otherwise seqs[i], poss[i] (host arrays, n_q <= kMaxBatch).
int run_decode(kore_cuda_ctx *c, int layer, int n_q, bool contiguous, int seq0, int pos0, const int *seqs,
               const int *poss, const float *q, const float *k, const float *v, float *out, float *lse,
               bool append_new, bool launch_merge = true, int *grid_out = nullptr, int *st_out = nullptr,
               float *fused_out = nullptr) {
    if (n_q <= 0) return fail(c, KORE_CUDA_EINVAL, "no queries");
    if (!contiguous && n_q > kMaxBatch)
        return fail(c, KORE_CUDA_EINVAL, "decode batch of %d exceeds %d sequences per call", n_q, kMaxBatch);
    if (n_q > 65535) return fail(c, KORE_CUDA_EINVAL, "%d queries exceed one launch", n_q);
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15)
        return fail(c, KORE_CUDA_EINVAL, "q, k and v must be 16-byte aligned device buffers");
    DecodeParams p;
    memset(&p, 0, sizeof p);
    p.kv = layer_kv(c, layer);
    p.q = q;
    p.k_new = k;
    p.v_new = v;
    p.out = out;
    p.lse = lse;
    p.rope = c->rope_d;
    p.part_o = c->part_o;
    p.part_ml = c->part_ml;
    p.err = c->err_d;
    p.wait_ns = c->wait_ns;
    p.scale_log2 = (1.0f / std::sqrt((float)c->D)) * 1.4426950408889634f;
    p.H = c->H;
    p.n_q = n_q;
    p.append_new = append_new ? 1 : 0;
    p.contiguous = contiguous ? 1 : 0;
    p.seq0 = seq0;
    p.pos0 = pos0;
    long long total = 0;
    int max_count = 0;
    std::vector<int> counts;
    if (!contiguous) counts.resize((size_t)n_q);
    for (int i = 0; i < n_q; ++i) {
        const int ps = contiguous ? pos0 + i : poss[i];
        if (!contiguous) {
            p.seq[i] = seqs[i];
            p.pos[i] = ps;
        }
        const int cnt = local_count(c, append_new ? ps : ps + 1);
        if (!contiguous) counts[(size_t)i] = cnt;
        total += cnt;
        max_count = std::max(max_count, cnt);
    }
    // one query at D = 128 on one GPU runs the tensor-core kernel when asked
    // (16-token tiles, one CTA per SM)
    const bool use_tc = c->tc_decode && c->kv_map_ok && c->D == 128 && n_q == 1 && contiguous && c->NS == 1;
    const int TT = use_tc ? decode_tc_tile_tokens() : decode_tile_tokens();
    // CTAs to aim for: two per SM, unless set otherwise (KORE_CUDA_DECODE_CTAS;
    // KORE_CUDA_SHARD_CTAS on a KV-split context), trading CTA count for
    // longer splits
    const long long target = c->NS > 1 && c->shard_ctas > 0 ? c->shard_ctas
                             : c->decode_ctas > 0           ? c->decode_ctas
                                                            : (long long)c->num_sms * (use_tc ? 1 : decode_ctas_per_sm(c->D, c->R));
    long long st = (total * c->G + target - 1) / target;
    st = std::max<long long>(st, 4 * TT);
    st = std::max<long long>(st, (max_count + kMaxSplits - 1) / kMaxSplits);
    int grid_x;
    if (n_q > kMaxBatch) {
        st = std::max(max_count, TT);   // one split per query: no scratch
    } else if (!contiguous && n_q > 1) {
        // A batch of ragged sequences: the split length decides how the CTAs
        // (one per split, KV head and sequence, dispatched split-fastest in
        // launch order) pack onto the SMs; a count just above a whole number
        // of waves leaves most SMs idle for one more CTA. A few lengths are
        // scored by replaying that in-order dispatch onto `target` slots,
        // each CTA costing its positions plus a fixed start-up cost, and
        // the one that finishes first is kept.
        const long long st_cap_b = std::max<long long>((long long)(decode_split_pages_max() - 1) * c->P / TT * TT, TT);
        const long long ovh = 32 * TT;
        std::vector<long long> slots;
        auto makespan = [&](long long s) {
            slots.assign((size_t)target, 0);
            std::make_heap(slots.begin(), slots.end(), std::greater<long long>());
            long long end = 0;
            for (int i = 0; i < n_q; ++i) {
                const long long n = counts[(size_t)i];
                const long long ns = std::max<long long>(1, (n + s - 1) / s);
                for (int g = 0; g < c->G; ++g)
                    for (long long k = 0; k < ns; ++k) {
                        std::pop_heap(slots.begin(), slots.end(), std::greater<long long>());
                        const long long t = slots.back() + std::min(s, n - k * s) + ovh;
                        slots.back() = t;
                        std::push_heap(slots.begin(), slots.end(), std::greater<long long>());
                        end = std::max(end, t);
                    }
            }
            return end;
        };
        auto length = [&](double f) {
            const long long s = (long long)(st * f);
            return std::min<long long>(std::max<long long>((s + TT - 1) / TT * TT, TT), st_cap_b);
        };
        // the choice moves slowly as the sequences grow: it is kept until the
        // batch size, or the total or largest count in 1024-position buckets,
        // changes
        const long long key[3] = {n_q, total >> 10, max_count >> 10};
        if (key[0] != c->split_key[0] || key[1] != c->split_key[1] || key[2] != c->split_key[2]) {
            double best_f = 1.0;
            long long best_t = -1;
            for (int k = 0; k <= 26; ++k) {
                const double f = k < 26 ? 1.0 + 0.05 * k : 3.0;
                const long long t = makespan(length(f));
                if (best_t < 0 || t < best_t) {
                    best_t = t;
                    best_f = f;
                }
            }
            c->split_f = best_f;
            for (int i = 0; i < 3; ++i) c->split_key[i] = key[i];
        }
        st = length(c->split_f);
    }
    for (;;) {
        st = (st + TT - 1) / TT * TT;
        grid_x = std::max(1, (int)((max_count + st - 1) / st));
        if (grid_x == 1 || (size_t)n_q * c->G * grid_x <= c->part_slots) break;
        st *= 2;
    }
    // a split may span at most decode_split_pages_max() pages
    const long long st_cap = (long long)(decode_split_pages_max() - 1) * c->P / TT * TT;
    if (st > st_cap) {
        st = st_cap;
        grid_x = std::max(1, (int)((max_count + st - 1) / st));
        if (n_q > kMaxBatch && grid_x > 1)
            return fail(c, KORE_CUDA_EINVAL, "prefill of %d tokens over %d positions exceeds one launch", n_q, max_count);
        if ((size_t)n_q * c->G * grid_x > c->part_slots)
            return fail(c, KORE_CUDA_EINVAL, "decode batch too large for the split scratch");
    }
    if (grid_x > kMaxSplits) return fail(c, KORE_CUDA_EINVAL, "too many splits for one decode launch");
    p.split_tokens = (int)st;
    p.max_splits = grid_x;
    if (use_tc) {
        p.tc = 1;
        p.tm_k = c->kv_map;
        p.tm_v = c->kv_map;
        p.k_row0 = (long long)((size_t)layer * c->layer_floats / 128);
        p.v_row0 = p.k_row0 + c->v_off / 128;
    }
    if (fused_out) {   // the exchange CTAs join this launch (peer_exchange.cu's protocol)
        p.fused_exchange = 1;
        p.x_ranks = c->NS;
        p.x_own = c->xbuf;
        for (int r = 0; r < c->NS; ++r) p.x_peers[r] = c->peers[r];
        p.x_epoch_off = c->x_epoch_off;
        p.x_out = fused_out;
        p.x_arrivals = c->x_arrivals;
    } else if (c->fused_merge && c->NS == 1 && n_q == 1 && contiguous && launch_merge && grid_x > 1) {
        // one GPU: the heads' merge CTAs join this launch instead of split_merge_kernel
        p.fused_exchange = 1;
        p.x_ranks = 1;
        p.x_arrivals = c->x_arrivals;
    }
    p.prefetch_ok = !c->hold_prefetch && c->last_kv_layer != layer;
    p.prefetch_stages = c->prefetch_stages;
    p.l2_inputs = c->l2_inputs ? 1 : 0;
    c->hold_prefetch = false;
    if (p.prefetch_ok && c->l2_prefetch_bytes > 0) {
        // L2 budget of the early fetch over all CTAs of the launch (a part of
        // the 126 MB L2, so that the prefetched lines outlive their wait)
        const long long per_token = (long long)n_q * c->G * grid_x * 2 * c->D * 4;
        p.l2_prefetch_tokens = (int)std::min<long long>(st, c->l2_prefetch_bytes / per_token / TT * TT);
    }
    CK(launch_attn_decode(p, c->R, grid_x, c->stream, launch_merge));
    if (grid_out) *grid_out = grid_x;
    if (st_out) *st_out = (int)st;
    // the decode (and its split merge, which lets the next kernel start at
    // once) may still run when the next kernel starts: it wrote this layer's KV
    c->last_kv_layer = append_new ? layer : -1;
    return KORE_CUDA_OK;
}

}  // namespace

extern "C" {

void kore_cuda_cfg_default(kore_cuda_cfg *cfg, int n_layer, int n_head, int n_head_kv, int head_dim, int ctx_max) {
    memset(cfg, 0, sizeof *cfg);
    cfg->n_layer = n_layer;
    cfg->n_head = n_head;
    cfg->n_head_kv = n_head_kv;
    cfg->head_dim = head_dim;
    cfg->ctx_max = ctx_max;
    cfg->max_seqs = 1;
    cfg->page_tokens = 256;
    cfg->rope_base = 1e6f;
    cfg->shard_count = 1;
}

const char *kore_cuda_last_error(const kore_cuda_ctx *c) { return c ? c->msg.c_str() : g_create_msg.c_str(); }

void kore_cuda_destroy(kore_cuda_ctx *c) {
    if (!c) return;
    {
        DeviceGuard dg(c->cfg.device);
        if (c->stream) cudaStreamSynchronize(c->stream);
        for (int r = 0; r < kMaxRanks; ++r)
            if (c->peers[r] && c->peers[r] != c->xbuf) cudaIpcCloseMemHandle(c->peers[r]);
        cudaFree(c->xbuf);
        cudaFree(c->x_arrivals);
        cudaFree(c->split);
        cudaFree(c->pf_items);
        cudaFree(c->pf_part);
        cudaFree(c->pf_counters);
        for (auto &lp : c->proj) {
            cudaFree(lp.w);
            cudaFree(lp.bias);
        }
        for (auto &lf : c->model.layers) {
            cudaFree(lf.norms);
            cudaFree(lf.w);
        }
        cudaFree(c->model.tok);
        cudaFree(c->model.out_norm);
        cudaFree(c->model.out_w);
        cudaFree(c->model.x);
        cudaFree(c->model.act);
        cudaFree(c->model.logits);
        cudaFree(c->model.key);
        cudaFree(c->model.token);
        for (void *b : {(void *)c->model.bx, (void *)c->model.bxb, (void *)c->model.bq, (void *)c->model.bk,
                        (void *)c->model.bv, (void *)c->model.batt, (void *)c->model.bact, (void *)c->model.btok})
            cudaFree(b);
        cudaFree(c->blk);
        cudaFree(c->kv);
        cudaFree(c->pt_d);
        cudaFree(c->rope_d);
        cudaFree(c->part_o);
        cudaFree(c->part_ml);
        cudaFree(c->err_d);
        cudaFree(c->dev_stage);
        if (c->host_stage) cudaFreeHost(c->host_stage);
        if (c->host_err) cudaFreeHost(c->host_err);
        if (c->host_ret) cudaFreeHost(c->host_ret);
        if (c->own_stream && c->stream) cudaStreamDestroy(c->stream);
    }
    delete c;
}

int kore_cuda_create(kore_cuda_ctx **out, const kore_cuda_cfg *cfg) {
    kore_cuda_ctx *c = nullptr;
    if (!out || !cfg) return fail(c, KORE_CUDA_EINVAL, "null argument");
    *out = nullptr;
    const kore_cuda_cfg &f = *cfg;
    if (f.n_layer <= 0 || f.n_head <= 0 || f.n_head_kv <= 0 || f.n_head % f.n_head_kv)
        return fail(c, KORE_CUDA_EINVAL, "bad head geometry (n_layer %d, n_head %d, n_head_kv %d)", f.n_layer,
                    f.n_head, f.n_head_kv);
    if (f.n_head / f.n_head_kv > 8) return fail(c, KORE_CUDA_EINVAL, "n_head/n_head_kv = %d > 8", f.n_head / f.n_head_kv);
    if (f.head_dim != 64 && f.head_dim != 128) return fail(c, KORE_CUDA_EINVAL, "head_dim %d not 64 or 128", f.head_dim);
    if (f.ctx_max <= 0 || f.max_seqs <= 0) return fail(c, KORE_CUDA_EINVAL, "ctx_max and max_seqs must be positive");
    if (!(f.rope_base > 0)) return fail(c, KORE_CUDA_EINVAL, "rope_base must be positive");
    const int P = f.page_tokens ? f.page_tokens : 256;
    if (P % 64 || P > 4096) return fail(c, KORE_CUDA_EINVAL, "page_tokens %d not a multiple of 64 up to 4096", P);
    const int NS = f.shard_count > 1 ? f.shard_count : 1;
    if (f.shard_rank < 0 || f.shard_rank >= NS) return fail(c, KORE_CUDA_EINVAL, "shard_rank %d outside [0, %d)", f.shard_rank, NS);

    c = new kore_cuda_ctx;
    c->cfg = f;
    c->cfg.page_tokens = P;
    c->cfg.shard_count = NS;
    c->H = f.n_head;
    c->G = f.n_head_kv;
    c->D = f.head_dim;
    c->R = f.n_head / f.n_head_kv;
    c->kvd = c->G * c->D;
    c->P = P;
    c->NS = NS;
    c->rank = f.shard_rank;
    c->pages_per_seq = std::max(1, local_pages(c, (f.ctx_max + P - 1) / P));
    c->n_pages = f.n_pages > 0 ? f.n_pages : f.max_seqs * c->pages_per_seq;
    c->pt_h.assign((size_t)f.max_seqs * c->pages_per_seq, -1);
    c->seq_alloc.assign((size_t)f.max_seqs, 0);
    c->seq_len.assign((size_t)f.max_seqs * f.n_layer, 0);
    for (int i = c->n_pages - 1; i >= 0; --i) c->free_pages.push_back(i);
    c->cfg.inv_freq = nullptr;

    auto bail = [&](int rc) {
        g_create_msg = c->msg;
        kore_cuda_destroy(c);
        return rc;
    };
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || f.device < 0 || f.device >= ndev)
        return bail(fail(c, KORE_CUDA_ECUDA, "CUDA device %d not available (%d visible)", f.device, ndev));
    DeviceGuard dg(f.device);
#define CKB(call)                                                                                  \
    do {                                                                                           \
        int rc_ = [&]() -> int { CK(call); return 0; }();                                          \
        if (rc_) return bail(rc_);                                                                 \
    } while (0)
    CKB(cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, f.device));
    if (const char *mb = getenv("KORE_CUDA_L2_PREFETCH_MB")) c->l2_prefetch_bytes = std::max(0ll, atoll(mb)) << 20;
    if (const char *sp = getenv("KORE_CUDA_SHARD_PREFETCH")) c->shard_prefetch = atoi(sp) != 0;
    if (const char *ps = getenv("KORE_CUDA_PREFETCH_STAGES")) c->prefetch_stages = std::max(0, atoi(ps));
    if (const char *li = getenv("KORE_CUDA_L2_INPUTS")) c->l2_inputs = atoi(li) != 0;
    if (const char *sc = getenv("KORE_CUDA_SHARD_CTAS")) c->shard_ctas = std::max(0, atoi(sc));
    if (const char *dc = getenv("KORE_CUDA_DECODE_CTAS")) c->decode_ctas = std::max(0, atoi(dc));
    if (const char *fx = getenv("KORE_CUDA_FUSED_EXCHANGE")) c->fused_exchange = atoi(fx) != 0;
    if (const char *fm = getenv("KORE_CUDA_FUSED_MERGE")) c->fused_merge = atoi(fm) != 0;
    if (const char *tc = getenv("KORE_CUDA_TC_DECODE")) c->tc_decode = atoi(tc) != 0;
    if (const char *rm = getenv("KORE_CUDA_RET_MAPPED")) c->ret_mapped = atoi(rm) != 0;
    CKB(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    c->own_stream = true;

    c->layer_floats = (size_t)2 * c->n_pages * c->G * P * c->D;
    c->v_off = (long long)c->n_pages * c->G * P * c->D;
    CKB(cudaMalloc(&c->kv, c->layer_floats * f.n_layer * sizeof(float)));
    CKB(cudaMemsetAsync(c->kv, 0, c->layer_floats * f.n_layer * sizeof(float), c->stream));
    if (c->D == 128) c->kv_map_ok = encode_kv_map(c->kv, c->layer_floats * f.n_layer / 128, &c->kv_map);
    CKB(cudaMalloc(&c->pt_d, c->pt_h.size() * sizeof(int)));
    CKB(cudaMemsetAsync(c->pt_d, 0xff, c->pt_h.size() * sizeof(int), c->stream));

    // RoPE tables for every position, as kore builds them per call
    const int half = c->D / 2;
    std::vector<float> inv((size_t)half);
    for (int i = 0; i < half; i++)
        inv[(size_t)i] = f.inv_freq ? f.inv_freq[i] : (float)std::pow((double)f.rope_base, -2.0 * i / c->D);
    std::vector<float2> tab((size_t)f.ctx_max * half);
    for (int pos = 0; pos < f.ctx_max; ++pos)
        for (int i = 0; i < half; i++) {
            const double a = (double)pos * inv[(size_t)i];
            tab[(size_t)pos * half + i] = make_float2((float)std::cos(a), (float)std::sin(a));
        }
    CKB(cudaMalloc(&c->rope_d, tab.size() * sizeof(float2)));
    CKB(cudaMemcpyAsync(c->rope_d, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice, c->stream));

    c->part_slots = kPartSlots;
    CKB(cudaMalloc(&c->part_o, c->part_slots * c->R * c->D * sizeof(float)));
    CKB(cudaMalloc(&c->part_ml, c->part_slots * c->R * sizeof(float2)));
    CKB(cudaMalloc(&c->x_arrivals, (size_t)c->H * sizeof(int)));
    CKB(cudaMemsetAsync(c->x_arrivals, 0, (size_t)c->H * sizeof(int), c->stream));
    // the device error word heads a buffer that also receives one sequence's
    // decode output, so that the host-buffer decode fetches both with one copy
    const size_t err_bytes = kErrPad + (size_t)c->H * c->D * sizeof(float);
    CKB(cudaMalloc(&c->err_d, err_bytes));
    CKB(cudaMemsetAsync(c->err_d, 0, sizeof(int), c->stream));
    CKB(cudaMallocHost(&c->host_err, err_bytes));
    CKB(cudaStreamSynchronize(c->stream));
#undef CKB
    c->msg = "no error";
    *out = c;
    return KORE_CUDA_OK;
}

int kore_cuda_seq_reset(kore_cuda_ctx *c, int seq) {
    if (!c) return KORE_CUDA_EINVAL;
    if (seq < 0 || seq >= c->cfg.max_seqs) return fail(c, KORE_CUDA_ERANGE, "seq %d outside [0, %d)", seq, c->cfg.max_seqs);
    int *row = c->pt_h.data() + (size_t)seq * c->pages_per_seq;
    for (int j = c->seq_alloc[seq] - 1; j >= 0; --j) {
        c->free_pages.push_back(row[j]);
        row[j] = -1;
    }
    c->seq_alloc[seq] = 0;
    for (int l = 0; l < c->cfg.n_layer; ++l) c->seq_len[(size_t)seq * c->cfg.n_layer + l] = 0;
    DeviceGuard dg(c->cfg.device);
    CK(cudaMemcpyAsync(c->pt_d + (size_t)seq * c->pages_per_seq, row, (size_t)c->pages_per_seq * sizeof(int),
                       cudaMemcpyHostToDevice, c->stream));
    return KORE_CUDA_OK;
}

int kore_cuda_seq_truncate(kore_cuda_ctx *c, int seq, int n) {
    if (!c) return KORE_CUDA_EINVAL;
    if (seq < 0 || seq >= c->cfg.max_seqs) return fail(c, KORE_CUDA_ERANGE, "seq %d outside [0, %d)", seq, c->cfg.max_seqs);
    if (n < 0) return fail(c, KORE_CUDA_EINVAL, "n = %d is negative", n);
    for (int l = 0; l < c->cfg.n_layer; ++l) {
        int &len = c->seq_len[(size_t)seq * c->cfg.n_layer + l];
        len = std::min(len, n);
    }
    // pages wholly past the kept positions go back to the pool
    const int keep = local_pages(c, (n + c->P - 1) / c->P);
    int *row = c->pt_h.data() + (size_t)seq * c->pages_per_seq;
    if (c->seq_alloc[seq] <= keep) return KORE_CUDA_OK;
    for (int j = c->seq_alloc[seq] - 1; j >= keep; --j) {
        c->free_pages.push_back(row[j]);
        row[j] = -1;
    }
    const int had = c->seq_alloc[seq];
    c->seq_alloc[seq] = keep;
    DeviceGuard dg(c->cfg.device);
    CK(cudaMemcpyAsync(c->pt_d + (size_t)seq * c->pages_per_seq + keep, row + keep, (size_t)(had - keep) * sizeof(int),
                       cudaMemcpyHostToDevice, c->stream));
    return KORE_CUDA_OK;
}

int kore_cuda_seq_len(const kore_cuda_ctx *c, int seq, int layer) {
    if (!c || seq < 0 || seq >= c->cfg.max_seqs || layer < 0 || layer >= c->cfg.n_layer) return KORE_CUDA_ERANGE;
    return c->seq_len[(size_t)seq * c->cfg.n_layer + layer];
}

int kore_cuda_kv_append_dev(kore_cuda_ctx *c, int seq, int layer, int pos0, int n, const float *k, const float *v) {
    if (!c) return KORE_CUDA_EINVAL;
    if (!k || !v) return fail(c, KORE_CUDA_EINVAL, "null k or v");
    if (int rc = check_range(c, seq, layer, pos0, n)) return rc;
    DeviceGuard dg(c->cfg.device);
    if (int rc = ensure_pages(c, seq, pos0 + n)) return rc;
    if (int rc = run_append(c, seq, layer, pos0, n, k, v)) return rc;
    note_len(c, seq, layer, pos0 + n);
    return KORE_CUDA_OK;
}

int kore_cuda_kv_append(kore_cuda_ctx *c, int seq, int layer, int pos0, int n, const float *k, const float *v) {
    if (!c) return KORE_CUDA_EINVAL;
    if (!k || !v) return fail(c, KORE_CUDA_EINVAL, "null k or v");
    if (int rc = check_range(c, seq, layer, pos0, n)) return rc;
    DeviceGuard dg(c->cfg.device);
    const size_t nk = (size_t)n * c->kvd;
    if (int rc = grow_stage(c, 2 * nk)) return rc;
    memcpy(c->host_stage, k, nk * sizeof(float));
    memcpy(c->host_stage + nk, v, nk * sizeof(float));
    CK(cudaMemcpyAsync(c->dev_stage, c->host_stage, 2 * nk * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    if (int rc = kore_cuda_kv_append_dev(c, seq, layer, pos0, n, c->dev_stage, c->dev_stage + nk)) return rc;
    return finish(c);
}

static int prefill_sharded(kore_cuda_ctx *c, int seq, int layer, int pos0, int n, const float *q, const float *k,
                           const float *v, float *out);

int kore_cuda_attn_prefill_dev(kore_cuda_ctx *c, int seq, int layer, int pos0, int n, const float *q, const float *k,
                               const float *v, float *out) {
    if (!c) return KORE_CUDA_EINVAL;
    if (!q || !k || !v || !out) return fail(c, KORE_CUDA_EINVAL, "null q, k, v or out");
    if (int rc = check_range(c, seq, layer, pos0, n)) return rc;
    DeviceGuard dg(c->cfg.device);
    if (c->NS > 1) {
        if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 15)
            return fail(c, KORE_CUDA_EINVAL, "q and out must be 16-byte aligned device buffers");
        return prefill_sharded(c, seq, layer, pos0, n, q, k, v, out);
    }
    if (int rc = ensure_pages(c, seq, pos0 + n)) return rc;
    if (int rc = run_append(c, seq, layer, pos0, n, k, v)) return rc;
    note_len(c, seq, layer, pos0 + n);
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 15)
        return fail(c, KORE_CUDA_EINVAL, "q and out must be 16-byte aligned device buffers");
    const int tk = prefill_tile_keys();
    if (!c->split) {   // operand tiles for a whole context, allocated on the first prefill
        const int tiles = (c->cfg.ctx_max + tk - 1) / tk;
        CK(cudaMalloc(&c->split, (size_t)c->G * tiles * prefill_tile_bytes(c->D)));
        c->split_tiles = tiles;
    }
    if (pos0 != c->pf_pos0 || n != c->pf_n) {
        // a new chunk shape: plan its work list; the kernels still queued may
        // read the old one, so the stream is drained before it is replaced
        std::vector<int4> items;
        const int slots = prefill_plan(pos0, n, c->H, c->num_sms, items);
        CK(cudaStreamSynchronize(c->stream));
        if (items.size() > c->pf_items_cap) {
            cudaFree(c->pf_items);
            c->pf_items = nullptr;
            c->pf_items_cap = 0;
            CK(cudaMalloc(&c->pf_items, items.size() * sizeof(int4)));
            c->pf_items_cap = items.size();
        }
        if (slots > c->pf_slots_cap) {
            cudaFree(c->pf_part);
            cudaFree(c->pf_counters);
            c->pf_part = nullptr;
            c->pf_counters = nullptr;
            c->pf_slots_cap = 0;
            CK(cudaMalloc(&c->pf_part, (size_t)slots * prefill_slot_bytes(c->D)));
            CK(cudaMalloc(&c->pf_counters, (size_t)slots * sizeof(int)));
            CK(cudaMemset(c->pf_counters, 0, (size_t)slots * sizeof(int)));
            c->pf_slots_cap = slots;
        }
        CK(cudaMemcpy(c->pf_items, items.data(), items.size() * sizeof(int4), cudaMemcpyHostToDevice));
        c->pf_items_n = (int)items.size();
        c->pf_pos0 = pos0;
        c->pf_n = n;
    }
    PrefillParams pp;
    memset(&pp, 0, sizeof pp);
    pp.items = c->pf_items;
    pp.n_items = c->pf_items_n;
    pp.part = c->pf_part;
    pp.counters = c->pf_counters;
    pp.kv = layer_kv(c, layer);
    pp.split = c->split;
    pp.tiles = c->split_tiles;
    pp.q = q;
    pp.out = out;
    pp.rope = c->rope_d;
    pp.err = c->err_d;
    pp.scale_log2 = (1.0f / std::sqrt((float)c->D)) * 1.4426950408889634f;
    pp.seq = seq;
    pp.pos0 = pos0;
    pp.n = n;
    pp.H = c->H;
    pp.n_rep = c->R;
    CK(launch_prefill(pp, c->stream));
    c->last_kv_layer = -1;   // the prefill kernels write no KV and end before their successor starts
    return KORE_CUDA_OK;
}

int kore_cuda_attn_prefill(kore_cuda_ctx *c, int seq, int layer, int pos0, int n, const float *q, const float *k,
                           const float *v, float *out) {
    if (!c) return KORE_CUDA_EINVAL;
    if (!q || !k || !v || !out) return fail(c, KORE_CUDA_EINVAL, "null q, k, v or out");
    if (int rc = check_range(c, seq, layer, pos0, n)) return rc;
    DeviceGuard dg(c->cfg.device);
    const size_t nq = (size_t)n * c->H * c->D, nk = (size_t)n * c->kvd;
    if (int rc = grow_stage(c, 2 * nq + 2 * nk)) return rc;
    float *hs = c->host_stage, *ds = c->dev_stage;
    memcpy(hs, q, nq * sizeof(float));
    memcpy(hs + nq, k, nk * sizeof(float));
    memcpy(hs + nq + nk, v, nk * sizeof(float));
    CK(cudaMemcpyAsync(ds, hs, (nq + 2 * nk) * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    float *dout = ds + nq + 2 * nk;
    if (int rc = kore_cuda_attn_prefill_dev(c, seq, layer, pos0, n, ds, ds + nq, ds + nq + nk, dout)) return rc;
    CK(cudaMemcpyAsync(hs + nq + 2 * nk, dout, nq * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    if (int rc = finish(c)) return rc;
    memcpy(out, hs + nq + 2 * nk, nq * sizeof(float));
    return KORE_CUDA_OK;
}

int kore_cuda_attn_decode_batch_dev(kore_cuda_ctx *c, int layer, int n_seq, const int *seq_ids, const int *pos,
                                    const float *q, const float *k, const float *v, float *out) {
    if (!c) return KORE_CUDA_EINVAL;
    if (!seq_ids || !pos || !q || !k || !v || !out) return fail(c, KORE_CUDA_EINVAL, "null argument");
    if (n_seq <= 0 || n_seq > kMaxBatch) return fail(c, KORE_CUDA_EINVAL, "n_seq %d outside [1, %d]", n_seq, kMaxBatch);
    for (int i = 0; i < n_seq; ++i) {
        if (int rc = check_range(c, seq_ids[i], layer, pos[i], 1)) return rc;
        for (int j = 0; j < i; ++j)
            if (seq_ids[j] == seq_ids[i]) return fail(c, KORE_CUDA_EINVAL, "sequence %d appears twice", seq_ids[i]);
    }
    DeviceGuard dg(c->cfg.device);
    for (int i = 0; i < n_seq; ++i)
        if (int rc = ensure_pages(c, seq_ids[i], pos[i] + 1)) return rc;
    if (int rc = run_decode(c, layer, n_seq, false, 0, 0, seq_ids, pos, q, k, v, out, nullptr, true)) return rc;
    for (int i = 0; i < n_seq; ++i) note_len(c, seq_ids[i], layer, pos[i] + 1);
    return KORE_CUDA_OK;
}

int kore_cuda_attn_decode_dev(kore_cuda_ctx *c, int seq, int layer, int pos, const float *q, const float *k,
                              const float *v, float *out) {
    if (!c) return KORE_CUDA_EINVAL;
    if (!q || !k || !v || !out) return fail(c, KORE_CUDA_EINVAL, "null q, k, v or out");
    if (int rc = check_range(c, seq, layer, pos, 1)) return rc;
    DeviceGuard dg(c->cfg.device);
    if (int rc = ensure_pages(c, seq, pos + 1)) return rc;
    if (int rc = run_decode(c, layer, 1, true, seq, pos, nullptr, nullptr, q, k, v, out, nullptr, true)) return rc;
    note_len(c, seq, layer, pos + 1);
    return KORE_CUDA_OK;
}

int kore_cuda_attn_decode_partial_dev(kore_cuda_ctx *c, int seq, int layer, int pos, const float *q, const float *k,
                                      const float *v, float *part) {
    if (!c) return KORE_CUDA_EINVAL;
    if (!q || !k || !v || !part) return fail(c, KORE_CUDA_EINVAL, "null q, k, v or part");
    if (int rc = check_range(c, seq, layer, pos, 1)) return rc;
    DeviceGuard dg(c->cfg.device);
    if (int rc = ensure_pages(c, seq, pos + 1)) return rc;
    float *lse = part + (size_t)c->H * c->D;
    if (int rc = run_decode(c, layer, 1, true, seq, pos, nullptr, nullptr, q, k, v, part, lse, true)) return rc;
    note_len(c, seq, layer, pos + 1);
    return KORE_CUDA_OK;
}

int kore_cuda_lse_merge_dev(kore_cuda_ctx *c, int n_parts, const float *parts, float *out) {
    if (!c) return KORE_CUDA_EINVAL;
    if (!parts || !out || n_parts <= 0) return fail(c, KORE_CUDA_EINVAL, "bad merge arguments");
    DeviceGuard dg(c->cfg.device);
    CK(launch_lse_merge(parts, n_parts, 1, c->H, c->D, out, c->stream));
    return KORE_CUDA_OK;
}

static size_t align256(size_t b) { return (b + 255) / 256 * 256; }

int kore_cuda_peer_handle(kore_cuda_ctx *c, void *handle) {
    if (!c || !handle) return KORE_CUDA_EINVAL;
    if (c->NS < 2 || c->NS > kMaxRanks)
        return fail(c, KORE_CUDA_EINVAL, "peer exchange needs 2..%d shards (context has %d)", kMaxRanks, c->NS);
    DeviceGuard dg(c->cfg.device);
    if (!c->xbuf) {
        // [2 parity sets][rank][query slot][head][head_dim + 1] (value, epoch)
        // words, the per-(query slot, head) epochs, this rank's own partials
        const size_t Q = kExchangeQueries;
        const size_t PF = Q * ((size_t)c->H * c->D + c->H);
        c->x_epoch_off = align256(2 * (size_t)c->NS * Q * c->H * (c->D + 1) * sizeof(unsigned long long));
        c->x_local_off = c->x_epoch_off + align256(Q * c->H * sizeof(unsigned));
        c->x_bytes = c->x_local_off + align256(PF * sizeof(float));
        CK(cudaMalloc(&c->xbuf, c->x_bytes));
        CK(cudaMemset(c->xbuf, 0, c->x_bytes));
        CK(cudaDeviceSynchronize());
    }
    cudaIpcMemHandle_t h;
    CK(cudaIpcGetMemHandle(&h, c->xbuf));
    static_assert(sizeof(h) == KORE_CUDA_PEER_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof h);
    return KORE_CUDA_OK;
}

int kore_cuda_peer_open(kore_cuda_ctx *c, const void *handles) {
    if (!c || !handles) return KORE_CUDA_EINVAL;
    if (!c->xbuf) return fail(c, KORE_CUDA_ESTATE, "call kore_cuda_peer_handle first");
    DeviceGuard dg(c->cfg.device);
    for (int r = 0; r < c->NS; ++r) {
        if (r == c->rank) {
            c->peers[r] = c->xbuf;
            continue;
        }
        if (c->peers[r]) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const char *>(handles) + (size_t)r * KORE_CUDA_PEER_HANDLE_BYTES, sizeof h);
        void *ptr = nullptr;
        CK(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
        c->peers[r] = static_cast<float *>(ptr);
    }
    c->peers_open = true;
    return KORE_CUDA_OK;
}

// One exchange (peer_exchange.cu) of n_q consecutive queries' partials left
// by run_decode (grid_x splits, not merged) in the local slots.
static int launch_exchange(kore_cuda_ctx *c, int n_q, int pos0, bool append_new, int grid_x, int split_tokens,
                           float *out) {
    ExchangeParams xp;
    memset(&xp, 0, sizeof xp);
    xp.local = reinterpret_cast<float *>(reinterpret_cast<char *>(c->xbuf) + c->x_local_off);
    xp.part_o = c->part_o;
    xp.part_ml = c->part_ml;
    xp.max_splits = grid_x;
    xp.split_tokens = split_tokens;
    xp.n_rep = c->R;
    xp.pos0 = pos0;
    xp.append_new = append_new ? 1 : 0;
    xp.P = c->P;
    xp.own = c->xbuf;
    for (int r = 0; r < c->NS; ++r) xp.peers[r] = c->peers[r];
    xp.epoch_off = c->x_epoch_off;
    xp.out = out;
    xp.err = c->err_d;
    xp.wait_ns = c->wait_ns;
    xp.n_ranks = c->NS;
    xp.rank = c->rank;
    xp.H = c->H;
    xp.D = c->D;
    xp.n_q = n_q;
    CK(launch_peer_exchange(xp, c->stream));
    return KORE_CUDA_OK;
}

int kore_cuda_attn_decode_sharded_dev(kore_cuda_ctx *c, int seq, int layer, int pos, const float *q, const float *k,
                                      const float *v, float *out) {
    if (!c) return KORE_CUDA_EINVAL;
    if (!q || !k || !v || !out) return fail(c, KORE_CUDA_EINVAL, "null q, k, v or out");
    if (!c->peers_open) return fail(c, KORE_CUDA_ESTATE, "peer exchange not set up (kore_cuda_peer_open)");
    if (int rc = check_range(c, seq, layer, pos, 1)) return rc;
    DeviceGuard dg(c->cfg.device);
    if (int rc = ensure_pages(c, seq, pos + 1)) return rc;
    float *local = reinterpret_cast<float *>(reinterpret_cast<char *>(c->xbuf) + c->x_local_off);
    int grid_x = 1, st = 0;   // the splits are merged by the exchange itself
    if (int rc = run_decode(c, layer, 1, true, seq, pos, nullptr, nullptr, q, k, v, local,
                            local + (size_t)kExchangeQueries * c->H * c->D, true, false, &grid_x, &st,
                            c->fused_exchange ? out : nullptr))
        return rc;
    note_len(c, seq, layer, pos + 1);
    if (!c->fused_exchange)
        if (int rc = launch_exchange(c, 1, pos, true, grid_x, st, out)) return rc;
    c->last_kv_layer = layer;   // the decode may still run when the next kernel starts
    c->hold_prefetch = !c->shard_prefetch;
    return KORE_CUDA_OK;
}

// A prefill chunk on a KV-split context: every rank stores the chunk's rows
// of the pages it holds, attends the chunk's queries over its own positions
// (the split decode kernel, one query per position, causal by its count) and
// the exchange merges the ranks' partials, kExchangeQueries queries at a time.
static int prefill_sharded(kore_cuda_ctx *c, int seq, int layer, int pos0, int n, const float *q, const float *k,
                           const float *v, float *out) {
    if (!c->peers_open)
        return fail(c, KORE_CUDA_ESTATE, "a KV-split context needs kore_cuda_peer_open before a prefill");
    if (int rc = ensure_pages(c, seq, pos0 + n)) return rc;
    if (int rc = run_append(c, seq, layer, pos0, n, k, v)) return rc;
    note_len(c, seq, layer, pos0 + n);
    float *local = reinterpret_cast<float *>(reinterpret_cast<char *>(c->xbuf) + c->x_local_off);
    for (int z0 = 0; z0 < n; z0 += kExchangeQueries) {
        const int m = std::min(kExchangeQueries, n - z0);
        const float *qz = q + (size_t)z0 * c->H * c->D;
        int grid_x = 1, st = 0;
        if (int rc = run_decode(c, layer, m, true, seq, pos0 + z0, nullptr, nullptr, qz, qz, qz, local,
                                local + (size_t)kExchangeQueries * c->H * c->D, false, false, &grid_x, &st))
            return rc;
        if (int rc = launch_exchange(c, m, pos0 + z0, false, grid_x, st, out + (size_t)z0 * c->H * c->D)) return rc;
    }
    c->last_kv_layer = layer;
    c->hold_prefetch = !c->shard_prefetch;
    return KORE_CUDA_OK;
}

int kore_cuda_attn_prefill_partial_dev(kore_cuda_ctx *c, int seq, int layer, int pos0, int n, const float *q,
                                       const float *k, const float *v, float *part) {
    if (!c) return KORE_CUDA_EINVAL;
    if (!q || !k || !v || !part) return fail(c, KORE_CUDA_EINVAL, "null q, k, v or part");
    if (int rc = check_range(c, seq, layer, pos0, n)) return rc;
    if (n > kMaxBatch) return fail(c, KORE_CUDA_EINVAL, "a partial prefill takes at most %d queries", kMaxBatch);
    DeviceGuard dg(c->cfg.device);
    if (int rc = ensure_pages(c, seq, pos0 + n)) return rc;
    if (int rc = run_append(c, seq, layer, pos0, n, k, v)) return rc;
    note_len(c, seq, layer, pos0 + n);
    if (int rc = run_decode(c, layer, n, true, seq, pos0, nullptr, nullptr, q, q, q, part,
                            part + (size_t)n * c->H * c->D, false))
        return rc;
    return KORE_CUDA_OK;
}

int kore_cuda_lse_merge_batch_dev(kore_cuda_ctx *c, int n_parts, int n_q, const float *parts, float *out) {
    if (!c) return KORE_CUDA_EINVAL;
    if (!parts || !out || n_parts <= 0 || n_q <= 0) return fail(c, KORE_CUDA_EINVAL, "bad merge arguments");
    DeviceGuard dg(c->cfg.device);
    CK(launch_lse_merge(parts, n_parts, n_q, c->H, c->D, out, c->stream));
    return KORE_CUDA_OK;
}

static int decode_host(kore_cuda_ctx *c, int n_seq, const float *q, const float *k, const float *v, float *out,
                       const int *seq_ids, const int *pos, int layer, bool batch, bool sharded = false) {
    DeviceGuard dg(c->cfg.device);
    const size_t nq = (size_t)n_seq * c->H * c->D, nk = (size_t)n_seq * c->kvd;
    if (int rc = grow_stage(c, 2 * nq + 2 * nk)) return rc;
    float *hs = c->host_stage, *ds = c->dev_stage;
    memcpy(hs, q, nq * sizeof(float));
    memcpy(hs + nq, k, nk * sizeof(float));
    memcpy(hs + nq + nk, v, nk * sizeof(float));
    if (int rc = stage_in(c, nq + 2 * nk)) return rc;
    if (!batch && c->ret_mapped && grow_ret(c, nq)) {
        // one sequence: the kernels write the output into the mapped return
        // buffer, a last one-thread kernel the error word and the call's
        // sequence number, which the host polls
        float *hout = reinterpret_cast<float *>(reinterpret_cast<char *>(c->host_ret_dev) + kRetPad);
        if (int rc = sharded ? kore_cuda_attn_decode_sharded_dev(c, seq_ids[0], layer, pos[0], ds, ds + nq, ds + nq + nk, hout)
                             : kore_cuda_attn_decode_dev(c, seq_ids[0], layer, pos[0], ds, ds + nq, ds + nq + nk, hout))
            return rc;
        if (++c->ret_seq == 0) ++c->ret_seq;
        ret_done_kernel<<<1, 32, 0, c->stream>>>(c->err_d, static_cast<unsigned *>(c->host_ret_dev), c->ret_seq);
        CK(cudaGetLastError());
        if (int rc = wait_ret(c, c->ret_seq)) return rc;
        memcpy(out, reinterpret_cast<const char *>(c->host_ret) + kRetPad, nq * sizeof(float));
        return KORE_CUDA_OK;
    }
    if (!batch) {
        // one sequence: the output lands right behind the error word and both
        // come back in one copy
        float *dout = reinterpret_cast<float *>(reinterpret_cast<char *>(c->err_d) + kErrPad);
        if (int rc = sharded ? kore_cuda_attn_decode_sharded_dev(c, seq_ids[0], layer, pos[0], ds, ds + nq, ds + nq + nk, dout)
                             : kore_cuda_attn_decode_dev(c, seq_ids[0], layer, pos[0], ds, ds + nq, ds + nq + nk, dout))
            return rc;
        if (int rc2 = finish(c, nq * sizeof(float))) return rc2;
        memcpy(out, reinterpret_cast<const char *>(c->host_err) + kErrPad, nq * sizeof(float));
        return KORE_CUDA_OK;
    }
    float *dout = ds + nq + 2 * nk;
    if (int rc = kore_cuda_attn_decode_batch_dev(c, layer, n_seq, seq_ids, pos, ds, ds + nq, ds + nq + nk, dout))
        return rc;
    CK(cudaMemcpyAsync(hs + nq + 2 * nk, dout, nq * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    if (int rc2 = finish(c)) return rc2;
    memcpy(out, hs + nq + 2 * nk, nq * sizeof(float));
    return KORE_CUDA_OK;
}

int kore_cuda_attn_decode(kore_cuda_ctx *c, int seq, int layer, int pos, const float *q, const float *k,
                          const float *v, float *out) {
    if (!c) return KORE_CUDA_EINVAL;
    if (!q || !k || !v || !out) return fail(c, KORE_CUDA_EINVAL, "null q, k, v or out");
    if (int rc = check_range(c, seq, layer, pos, 1)) return rc;
    return decode_host(c, 1, q, k, v, out, &seq, &pos, layer, false);
}

int kore_cuda_attn_decode_sharded(kore_cuda_ctx *c, int seq, int layer, int pos, const float *q, const float *k,
                                  const float *v, float *out) {
    if (!c) return KORE_CUDA_EINVAL;
    if (!q || !k || !v || !out) return fail(c, KORE_CUDA_EINVAL, "null q, k, v or out");
    if (!c->peers_open) return fail(c, KORE_CUDA_ESTATE, "peer exchange not set up (kore_cuda_peer_open)");
    if (int rc = check_range(c, seq, layer, pos, 1)) return rc;
    return decode_host(c, 1, q, k, v, out, &seq, &pos, layer, false, true);
}

int kore_cuda_attn_decode_batch(kore_cuda_ctx *c, int layer, int n_seq, const int *seq_ids, const int *pos,
                                const float *q, const float *k, const float *v, float *out) {
    if (!c) return KORE_CUDA_EINVAL;
    if (!seq_ids || !pos || !q || !k || !v || !out) return fail(c, KORE_CUDA_EINVAL, "null argument");
    if (n_seq <= 0 || n_seq > kMaxBatch) return fail(c, KORE_CUDA_EINVAL, "n_seq %d outside [1, %d]", n_seq, kMaxBatch);
    return decode_host(c, n_seq, q, k, v, out, seq_ids, pos, layer, true);
}

// ---------------------------------------------------------------- attention block projections

// GGUF bytes of a matrix (the host layout) and bytes of its uploaded copy
// (Q6_K blocks block_stride apart).
static size_t qmat_bytes(int type, int rows, int cols) {
    return (size_t)rows * (size_t)(cols / 256) * (type == KORE_CUDA_Q4_K ? 144 : 210);
}
static size_t qmat_dev_bytes(int type, int rows, int cols) {
    return (size_t)rows * (size_t)(cols / 256) * block_stride(type);
}

// Copies a GGUF matrix to the device in the uploaded layout: Q4_K as is, Q6_K
// with 2 zero bytes behind every 210-byte block (through a host buffer of one
// slice of rows at a time).
static cudaError_t upload_qmat(uint8_t *dst, const kore_cuda_qmat &m) {
    if (m.type == KORE_CUDA_Q4_K)
        return cudaMemcpy(dst, m.data, qmat_bytes(m.type, m.rows, m.cols), cudaMemcpyHostToDevice);
    const size_t nblk = (size_t)m.rows * (m.cols / 256), per = (size_t)1 << 16;
    std::vector<uint8_t> buf(per * kQ6Stride, 0);
    const uint8_t *src = static_cast<const uint8_t *>(m.data);
    for (size_t b0 = 0; b0 < nblk; b0 += per) {
        const size_t n = std::min(per, nblk - b0);
        for (size_t b = 0; b < n; ++b) memcpy(buf.data() + b * kQ6Stride, src + (b0 + b) * 210, 210);
        if (cudaError_t e = cudaMemcpy(dst + b0 * kQ6Stride, buf.data(), n * kQ6Stride, cudaMemcpyHostToDevice))
            return e;
    }
    return cudaSuccess;
}

static int check_qmat(kore_cuda_ctx *c, const kore_cuda_qmat *m, const char *name, int rows, int cols) {
    if (!m || !m->data) return fail(c, KORE_CUDA_EINVAL, "%s: null matrix or data", name);
    if (m->type != KORE_CUDA_Q4_K && m->type != KORE_CUDA_Q6_K)
        return fail(c, KORE_CUDA_EINVAL, "%s: type %d is neither Q4_K (12) nor Q6_K (14)", name, m->type);
    if (m->rows != rows || m->cols != cols)
        return fail(c, KORE_CUDA_EINVAL, "%s is %d x %d, expected %d x %d", name, m->rows, m->cols, rows, cols);
    return KORE_CUDA_OK;
}

// A layer's uploaded projections, or null. The matrix types are set last by
// kore_cuda_set_attn_weights, so an upload that failed part-way is not one.
static const kore_cuda_ctx::LayerProj *layer_proj(kore_cuda_ctx *c, int layer) {
    if (layer < 0 || layer >= (int)c->proj.size()) return nullptr;
    const kore_cuda_ctx::LayerProj &lp = c->proj[(size_t)layer];
    return lp.w && lp.type[0] && lp.type[3] ? &lp : nullptr;
}

// One product launch whose segments, vectors and modes are filled in: the
// ring shape for its widest block, the error word, then the launch.
static int launch_products(kore_cuda_ctx *c, QMatvecParams &mp) {
    int bb = 0;
    for (int i = 0; i < mp.n_seg; ++i) bb = std::max(bb, block_stride(mp.seg[i].type));
    if (qmatvec_config(mp.cols, bb, &mp.stages, &mp.row_slot) > kQmatvecMaxSmem)
        return fail(c, KORE_CUDA_EINVAL, "a product over %d columns does not fit in shared memory", mp.cols);
    mp.err = c->err_d;
    CK(launch_qmatvec(mp, c->num_sms, c->stream));
    return KORE_CUDA_OK;
}

// One product launch over up to three of a layer's matrices (which: 0 wq,
// 1 wk, 2 wv, 3 wo) with the fp32 vector x (quantised in the kernel, after
// an RMSNorm with norm_w when given), results to outs (plus the biases of
// wq/wk/wv), or added to `resid` when given.
static int launch_proj(kore_cuda_ctx *c, const kore_cuda_ctx::LayerProj &lp, const int *which, int n, const float *x,
                       float *const *outs, const float *norm_w = nullptr, float eps = 0.f,
                       const float *resid = nullptr) {
    const int E = c->H * c->D;
    QMatvecParams mp;
    memset(&mp, 0, sizeof mp);
    mp.x = x;
    mp.cols = E;
    for (int i = 0; i < n; ++i) {
        const int w = which[i];
        QSeg &g = mp.seg[i];
        g.w = lp.w + lp.off[w];
        g.type = lp.type[w];
        g.rows = lp.rows[w];
        g.out = outs[i];
        g.bias = (w < 3 && lp.has_bias) ? lp.bias + (w == 0 ? 0 : (w == 1 ? E : E + c->kvd)) : nullptr;
    }
    mp.n_seg = n;
    mp.in_mode = norm_w ? QIN_RMSNORM : QIN_QUANT;
    mp.norm_w = norm_w;
    mp.eps = eps;
    mp.out_mode = resid ? QOUT_RESIDUAL : QOUT_STORE;
    mp.resid = resid;
    return launch_products(c, mp);
}

int kore_cuda_set_attn_weights(kore_cuda_ctx *c, int layer, const kore_cuda_qmat *wq, const kore_cuda_qmat *wk,
                               const kore_cuda_qmat *wv, const kore_cuda_qmat *wo, const float *bq, const float *bk,
                               const float *bv) {
    if (!c) return KORE_CUDA_EINVAL;
    if (layer < 0 || layer >= c->cfg.n_layer)
        return fail(c, KORE_CUDA_ERANGE, "layer %d outside [0, %d)", layer, c->cfg.n_layer);
    const int E = c->H * c->D;
    if (E % 256) return fail(c, KORE_CUDA_EINVAL, "n_embd = %d is not a multiple of 256", E);
    if ((bq == nullptr) != (bk == nullptr) || (bq == nullptr) != (bv == nullptr))
        return fail(c, KORE_CUDA_EINVAL, "bq, bk and bv must be all given or all NULL");
    const kore_cuda_qmat *m[4] = {wq, wk, wv, wo};
    const int rows[4] = {E, c->kvd, c->kvd, E};
    const char *names[4] = {"wq", "wk", "wv", "wo"};
    for (int i = 0; i < 4; ++i)
        if (int rc = check_qmat(c, m[i], names[i], rows[i], E)) return rc;
    if (qmatvec_config(E, kQ6Stride, nullptr, nullptr) > kQmatvecMaxSmem)
        return fail(c, KORE_CUDA_EINVAL, "n_embd = %d: a product launch's staging exceeds shared memory", E);
    DeviceGuard dg(c->cfg.device);
    if (c->proj.empty()) c->proj.resize((size_t)c->cfg.n_layer);
    auto &lp = c->proj[(size_t)layer];
    // kernels still queued may read this layer's previous weights
    CK(cudaStreamSynchronize(c->stream));
    cudaFree(lp.w);
    cudaFree(lp.bias);
    lp = kore_cuda_ctx::LayerProj();
    size_t off[4], total = 0;
    for (int i = 0; i < 4; ++i) {
        off[i] = total;
        total += align256(qmat_dev_bytes(m[i]->type, rows[i], E) + 16);   // the product kernel reads past a row's end
    }
    uint8_t *w = nullptr;
    CK(cudaMalloc(&w, total));
    lp.w = w;
    for (int i = 0; i < 4; ++i) CK(upload_qmat(w + off[i], *m[i]));
    if (bq) {
        float *b = nullptr;
        CK(cudaMalloc(&b, (size_t)(E + 2 * c->kvd) * sizeof(float)));
        lp.bias = b;
        CK(cudaMemcpy(b, bq, (size_t)E * sizeof(float), cudaMemcpyHostToDevice));
        CK(cudaMemcpy(b + E, bk, (size_t)c->kvd * sizeof(float), cudaMemcpyHostToDevice));
        CK(cudaMemcpy(b + E + c->kvd, bv, (size_t)c->kvd * sizeof(float), cudaMemcpyHostToDevice));
        lp.has_bias = true;
    }
    if (!c->blk) {
        CK(cudaMalloc(&c->blk, (size_t)(2 * E + 2 * c->kvd) * sizeof(float)));
    }
    for (int i = 0; i < 4; ++i) {
        lp.type[i] = m[i]->type;
        lp.rows[i] = rows[i];
        lp.off[i] = off[i];
    }
    return KORE_CUDA_OK;
}

int kore_cuda_qmatvec(kore_cuda_ctx *c, int layer, int which, const float *x, float *out) {
    if (!c) return KORE_CUDA_EINVAL;
    if (!x || !out) return fail(c, KORE_CUDA_EINVAL, "null x or out");
    if (which < 0 || which > 3) return fail(c, KORE_CUDA_EINVAL, "which = %d is not 0 (wq), 1 (wk), 2 (wv) or 3 (wo)", which);
    const kore_cuda_ctx::LayerProj *lp = layer_proj(c, layer);
    if (!lp) return fail(c, KORE_CUDA_ESTATE, "no attention weights for layer %d (kore_cuda_set_attn_weights)", layer);
    DeviceGuard dg(c->cfg.device);
    const int E = c->H * c->D, rows = lp->rows[which];
    if (int rc = grow_stage(c, (size_t)E + rows)) return rc;
    float *hs = c->host_stage, *ds = c->dev_stage;
    memcpy(hs, x, (size_t)E * sizeof(float));
    CK(cudaMemcpyAsync(ds, hs, (size_t)E * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    float *od = ds + E;
    if (int rc = launch_proj(c, *lp, &which, 1, ds, &od)) return rc;
    CK(cudaMemcpyAsync(hs + E, od, (size_t)rows * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    if (int rc = finish(c)) return rc;
    memcpy(out, hs + E, (size_t)rows * sizeof(float));
    return KORE_CUDA_OK;
}

int kore_cuda_attn_block_decode_dev(kore_cuda_ctx *c, int seq, int layer, int pos, const float *xb, float *o) {
    if (!c) return KORE_CUDA_EINVAL;
    if (!xb || !o) return fail(c, KORE_CUDA_EINVAL, "null xb or o");
    if ((reinterpret_cast<uintptr_t>(xb) | reinterpret_cast<uintptr_t>(o)) & 15)
        return fail(c, KORE_CUDA_EINVAL, "xb and o must be 16-byte aligned device buffers");
    if (int rc = check_range(c, seq, layer, pos, 1)) return rc;
    const kore_cuda_ctx::LayerProj *lp = layer_proj(c, layer);
    if (!lp) return fail(c, KORE_CUDA_ESTATE, "no attention weights for layer %d (kore_cuda_set_attn_weights)", layer);
    if (c->NS > 1 && !c->peers_open)
        return fail(c, KORE_CUDA_ESTATE, "a KV-split context needs kore_cuda_peer_open before the attention block");
    DeviceGuard dg(c->cfg.device);
    const int E = c->H * c->D;
    float *q = c->blk, *k = q + E, *v = k + c->kvd, *att = v + c->kvd;
    const int qkv[3] = {0, 1, 2};
    float *const outs[3] = {q, k, v};
    if (int rc = launch_proj(c, *lp, qkv, 3, xb, outs)) return rc;
    if (int rc = c->NS > 1 ? kore_cuda_attn_decode_sharded_dev(c, seq, layer, pos, q, k, v, att)
                           : kore_cuda_attn_decode_dev(c, seq, layer, pos, q, k, v, att))
        return rc;
    const int wo = 3;
    return launch_proj(c, *lp, &wo, 1, att, &o);
}

int kore_cuda_attn_block_decode(kore_cuda_ctx *c, int seq, int layer, int pos, const float *xb, float *o) {
    if (!c) return KORE_CUDA_EINVAL;
    if (!xb || !o) return fail(c, KORE_CUDA_EINVAL, "null xb or o");
    DeviceGuard dg(c->cfg.device);
    const int E = c->H * c->D;
    if (int rc = grow_stage(c, (size_t)E)) return rc;
    memcpy(c->host_stage, xb, (size_t)E * sizeof(float));
    if (int rc = stage_in(c, (size_t)E)) return rc;
    if (c->ret_mapped && grow_ret(c, (size_t)E)) {
        // the Wo product writes into the mapped return buffer; the host polls
        // the call's sequence number (as the host-buffer decode)
        float *hout = reinterpret_cast<float *>(reinterpret_cast<char *>(c->host_ret_dev) + kRetPad);
        if (int rc = kore_cuda_attn_block_decode_dev(c, seq, layer, pos, c->dev_stage, hout)) return rc;
        if (++c->ret_seq == 0) ++c->ret_seq;
        ret_done_kernel<<<1, 32, 0, c->stream>>>(c->err_d, static_cast<unsigned *>(c->host_ret_dev), c->ret_seq);
        CK(cudaGetLastError());
        if (int rc = wait_ret(c, c->ret_seq)) return rc;
        memcpy(o, reinterpret_cast<const char *>(c->host_ret) + kRetPad, (size_t)E * sizeof(float));
        return KORE_CUDA_OK;
    }
    // the output lands right behind the error word and both come back in one copy
    float *dout = reinterpret_cast<float *>(reinterpret_cast<char *>(c->err_d) + kErrPad);
    if (int rc = kore_cuda_attn_block_decode_dev(c, seq, layer, pos, c->dev_stage, dout)) return rc;
    if (int rc = finish(c, (size_t)E * sizeof(float))) return rc;
    memcpy(o, reinterpret_cast<const char *>(c->host_err) + kErrPad, (size_t)E * sizeof(float));
    return KORE_CUDA_OK;
}

// ---------------------------------------------------------------- the whole decode step on the device

static size_t row_bytes_of(int type, int cols) {
    switch (type) {
        case KORE_CUDA_F32: return (size_t)cols * 4;
        case KORE_CUDA_F16:
        case KORE_CUDA_BF16: return (size_t)cols * 2;
        case KORE_CUDA_Q4_K: return (size_t)(cols / 256) * 144;
        case KORE_CUDA_Q6_K: return (size_t)(cols / 256) * 210;
        default: return 0;
    }
}

int kore_cuda_set_model(kore_cuda_ctx *c, const kore_cuda_model *m) {
    if (!c) return KORE_CUDA_EINVAL;
    if (!m || !m->layers || !m->out_norm || !m->tok_embd.data || !m->out_w.data)
        return fail(c, KORE_CUDA_EINVAL, "null model, layers, out_norm, tok_embd or out_w");
    const int E = c->H * c->D, FF = m->n_ff, V = m->n_vocab;
    if (E % 256 || FF <= 0 || FF % 256 || V <= 0)
        return fail(c, KORE_CUDA_EINVAL, "n_embd %d and n_ff %d must be multiples of 256 (kore.cpp:1283), n_vocab %d > 0",
                    E, FF, V);
    if (!(m->rms_eps >= 0.f)) return fail(c, KORE_CUDA_EINVAL, "rms_eps must be non-negative");
    const kore_cuda_qmat &te = m->tok_embd;
    if (row_bytes_of(te.type, E) == 0 || ((te.type == KORE_CUDA_Q4_K || te.type == KORE_CUDA_Q6_K) && E % 256))
        return fail(c, KORE_CUDA_EINVAL, "tok_embd: type %d is none of F32, F16, BF16, Q4_K, Q6_K", te.type);
    if (te.rows != V || te.cols != E)
        return fail(c, KORE_CUDA_EINVAL, "tok_embd is %d x %d, expected %d x %d", te.rows, te.cols, V, E);
    if (int rc = check_qmat(c, &m->out_w, "output", V, E)) return rc;
    for (int l = 0; l < c->cfg.n_layer; ++l) {
        const kore_cuda_layer_weights &L = m->layers[l];
        if (!L.attn_norm || !L.ffn_norm) return fail(c, KORE_CUDA_EINVAL, "layer %d: null norm weights", l);
        if (int rc = check_qmat(c, &L.w_gate, "ffn_gate", FF, E)) return rc;
        if (int rc = check_qmat(c, &L.w_up, "ffn_up", FF, E)) return rc;
        if (int rc = check_qmat(c, &L.w_down, "ffn_down", E, FF)) return rc;
    }
    if (qmatvec_config(FF, kQ6Stride, nullptr, nullptr) > kQmatvecMaxSmem)
        return fail(c, KORE_CUDA_EINVAL, "n_ff = %d: the down product's input does not fit in shared memory", FF);
    DeviceGuard dg(c->cfg.device);
    CK(cudaStreamSynchronize(c->stream));
    auto &M = c->model;
    M.ready = false;
    for (int l = 0; l < c->cfg.n_layer; ++l) {
        const kore_cuda_layer_weights &L = m->layers[l];
        if (int rc = kore_cuda_set_attn_weights(c, l, &L.wq, &L.wk, &L.wv, &L.wo, L.bq, L.bk, L.bv)) return rc;
    }
    M.layers.resize((size_t)c->cfg.n_layer);
    for (int l = 0; l < c->cfg.n_layer; ++l) {
        const kore_cuda_layer_weights &L = m->layers[l];
        auto &lf = M.layers[(size_t)l];
        cudaFree(lf.norms);
        cudaFree(lf.w);
        lf = kore_cuda_ctx::LayerFfn();
        CK(cudaMalloc(&lf.norms, (size_t)2 * E * sizeof(float)));
        CK(cudaMemcpy(lf.norms, L.attn_norm, (size_t)E * sizeof(float), cudaMemcpyHostToDevice));
        CK(cudaMemcpy(lf.norms + E, L.ffn_norm, (size_t)E * sizeof(float), cudaMemcpyHostToDevice));
        const kore_cuda_qmat *w[3] = {&L.w_gate, &L.w_up, &L.w_down};
        size_t total = 0;
        for (int i = 0; i < 3; ++i) {
            lf.off[i] = total;
            total += align256(qmat_dev_bytes(w[i]->type, w[i]->rows, w[i]->cols) + 16);   // the product kernel reads past a row's end
        }
        CK(cudaMalloc(&lf.w, total));
        for (int i = 0; i < 3; ++i) {
            CK(upload_qmat(lf.w + lf.off[i], *w[i]));
            lf.type[i] = w[i]->type;
        }
    }
    cudaFree(M.tok);
    cudaFree(M.out_norm);
    cudaFree(M.out_w);
    M.tok = nullptr;
    M.out_norm = nullptr;
    M.out_w = nullptr;
    M.tok_row_bytes = row_bytes_of(te.type, E);
    CK(cudaMalloc(&M.tok, (size_t)V * M.tok_row_bytes));
    CK(cudaMemcpy(M.tok, te.data, (size_t)V * M.tok_row_bytes, cudaMemcpyHostToDevice));
    CK(cudaMalloc(&M.out_norm, (size_t)E * sizeof(float)));
    CK(cudaMemcpy(M.out_norm, m->out_norm, (size_t)E * sizeof(float), cudaMemcpyHostToDevice));
    CK(cudaMalloc(&M.out_w, align256(qmat_dev_bytes(m->out_w.type, V, E) + 16)));
    CK(upload_qmat(M.out_w, m->out_w));
    if (M.n_vocab != V || !M.logits) {
        cudaFree(M.logits);
        M.logits = nullptr;
        CK(cudaMalloc(&M.logits, (size_t)V * sizeof(float)));
    }
    if (M.n_ff != FF || !M.act) {
        cudaFree(M.act);
        M.act = nullptr;
        CK(cudaMalloc(&M.act, (size_t)FF * sizeof(float)));
    }
    if (!M.x) CK(cudaMalloc(&M.x, (size_t)E * sizeof(float)));
    if (!M.key) CK(cudaMalloc(&M.key, sizeof(unsigned long long)));
    if (!M.token) CK(cudaMalloc(&M.token, 2 * sizeof(int)));
    // 2^(i/32) as the C library's exp2 rounds it, exponent bits taken out:
    // the table of the expf that kore's SwiGLU calls (proj.cu, kore_expf)
    for (int i = 0; i < 32; ++i) {
        const double t = std::exp2((double)i / 32.0);
        unsigned long long b;
        memcpy(&b, &t, sizeof b);
        M.exp_tab[i] = b - ((unsigned long long)i << 47);
    }
    M.n_ff = FF;
    M.n_vocab = V;
    M.eps = m->rms_eps;
    M.tok_type = te.type;
    M.out_type = m->out_w.type;
    M.ready = true;
    return KORE_CUDA_OK;
}

// kore's forward() for one token (kore.cpp:1397-1480) and the greedy choice
// of sample_token (kore.cpp:1601-1603), every step on the device:
//   embedding row of the token                        embed_kernel
//   per layer: RMSNorm + Q8_K + Wq/Wk/Wv + biases      qmatvec (RMSNORM in, STORE out)
//              RoPE, append, attention                 attn_decode (+ split merge or peer exchange)
//              Q8_K(att) + Wo + residual add           qmatvec (QUANT in, RESIDUAL out)
//              RMSNorm + Q8_K + gate/up + SwiGLU        qmatvec (RMSNORM in, paired, SWIGLU out)
//              Q8_K + down + residual add              qmatvec (QUANT in, RESIDUAL out)
//   RMSNorm + Q8_K + output matrix + argmax            qmatvec (RMSNORM in, ARGMAX out)
//   the token from the argmax key                     token_kernel
static int run_step(kore_cuda_ctx *c, int seq, int token, const int *token_dev, int pos, int *next_dev,
                    float *logits_dev) {
    auto &M = c->model;
    const int E = c->H * c->D, FF = M.n_ff, NL = c->cfg.n_layer;
    float *q = c->blk, *k = q + E, *v = k + c->kvd, *att = v + c->kvd;
    EmbedParams ep;
    memset(&ep, 0, sizeof ep);
    ep.table = M.tok;
    ep.row_bytes = M.tok_row_bytes;
    ep.type = M.tok_type;
    ep.n_vocab = M.n_vocab;
    ep.n_embd = E;
    ep.token = token;
    ep.n_tokens = 1;
    ep.token_dev = token_dev;
    ep.x = M.x;
    ep.key = M.key;
    ep.err = c->err_d;
    CK(launch_embed(ep, c->stream));
    c->last_kv_layer = -1;
    for (int l = 0; l < NL; ++l) {
        const kore_cuda_ctx::LayerProj &lp = c->proj[(size_t)l];
        const kore_cuda_ctx::LayerFfn &lf = M.layers[(size_t)l];
        const int qkv[3] = {0, 1, 2};
        float *const outs[3] = {q, k, v};
        if (int rc = launch_proj(c, lp, qkv, 3, M.x, outs, lf.norms, M.eps)) return rc;
        if (int rc = c->NS > 1 ? kore_cuda_attn_decode_sharded_dev(c, seq, l, pos, q, k, v, att)
                               : kore_cuda_attn_decode_dev(c, seq, l, pos, q, k, v, att))
            return rc;
        const int wo = 3;
        float *const xo[1] = {M.x};
        if (int rc = launch_proj(c, lp, &wo, 1, att, xo, nullptr, 0.f, M.x)) return rc;
        QMatvecParams mp;
        memset(&mp, 0, sizeof mp);
        mp.n_seg = 2;
        mp.cols = E;
        mp.seg[0] = QSeg{lf.w + lf.off[0], nullptr, M.act, lf.type[0], FF};
        mp.seg[1] = QSeg{lf.w + lf.off[1], nullptr, M.act, lf.type[1], FF};
        mp.pair_segments = 1;
        mp.in_mode = QIN_RMSNORM;
        mp.x = M.x;
        mp.norm_w = lf.norms + E;
        mp.eps = M.eps;
        mp.out_mode = QOUT_SWIGLU;
        memcpy(mp.exp_tab, M.exp_tab, sizeof mp.exp_tab);
        if (int rc = launch_products(c, mp)) return rc;
        memset(&mp, 0, sizeof mp);
        mp.n_seg = 1;
        mp.cols = FF;
        mp.seg[0] = QSeg{lf.w + lf.off[2], nullptr, M.x, lf.type[2], E};
        mp.in_mode = QIN_QUANT;
        mp.x = M.act;
        mp.out_mode = QOUT_RESIDUAL;
        mp.resid = M.x;
        if (int rc = launch_products(c, mp)) return rc;
    }
    QMatvecParams mp;
    memset(&mp, 0, sizeof mp);
    mp.n_seg = 1;
    mp.cols = E;
    mp.seg[0] = QSeg{M.out_w, nullptr, logits_dev ? logits_dev : M.logits, M.out_type, M.n_vocab};
    mp.in_mode = QIN_RMSNORM;
    mp.x = M.x;
    mp.norm_w = M.out_norm;
    mp.eps = M.eps;
    mp.out_mode = QOUT_ARGMAX;
    mp.argmax = M.key;
    if (int rc = launch_products(c, mp)) return rc;
    CK(launch_token(M.key, next_dev, c->stream));
    return KORE_CUDA_OK;
}

static int check_step(kore_cuda_ctx *c, int seq, int pos) {
    if (!c->model.ready || c->proj.size() != (size_t)c->cfg.n_layer)
        return fail(c, KORE_CUDA_ESTATE, "no model on the device (kore_cuda_set_model)");
    for (int l = 0; l < c->cfg.n_layer; ++l) {
        if (int rc = check_range(c, seq, l, pos, 1)) return rc;
        if (!layer_proj(c, l)) return fail(c, KORE_CUDA_ESTATE, "layer %d has no attention weights", l);
    }
    if (c->NS > 1 && !c->peers_open)
        return fail(c, KORE_CUDA_ESTATE, "a KV-split context needs kore_cuda_peer_open before a decode step");
    return KORE_CUDA_OK;
}

int kore_cuda_decode_step_dev(kore_cuda_ctx *c, int seq, const int *token, int pos, int *next_token, float *logits) {
    if (!c) return KORE_CUDA_EINVAL;
    if (!token || !next_token) return fail(c, KORE_CUDA_EINVAL, "null token or next_token");
    if (int rc = check_step(c, seq, pos)) return rc;
    DeviceGuard dg(c->cfg.device);
    return run_step(c, seq, 0, token, pos, next_token, logits);
}

int kore_cuda_decode_step(kore_cuda_ctx *c, int seq, int token, int pos, int *next_token, float *logits) {
    if (!c) return KORE_CUDA_EINVAL;
    if (!next_token) return fail(c, KORE_CUDA_EINVAL, "null next_token");
    if (int rc = check_step(c, seq, pos)) return rc;
    if (token < 0 || token >= c->model.n_vocab)   // forward() returns false (kore.cpp:1400)
        return fail(c, KORE_CUDA_ERANGE, "token %d outside the vocabulary of %d", token, c->model.n_vocab);
    DeviceGuard dg(c->cfg.device);
    // the next token lands right behind the error word and both come back in one copy
    int *dnext = reinterpret_cast<int *>(reinterpret_cast<char *>(c->err_d) + kErrPad);
    if (int rc = run_step(c, seq, token, nullptr, pos, dnext, nullptr)) return rc;
    if (logits)
        CK(cudaMemcpyAsync(logits, c->model.logits, (size_t)c->model.n_vocab * sizeof(float), cudaMemcpyDeviceToHost,
                           c->stream));
    if (int rc = finish(c, sizeof(int))) return rc;
    memcpy(next_token, reinterpret_cast<const char *>(c->host_err) + kErrPad, sizeof(int));
    return KORE_CUDA_OK;
}

// ---------------------------------------------------------------- the whole prefill on the device

static int grow_prefill(kore_cuda_ctx *c, int n) {
    auto &M = c->model;
    if (n <= M.pf_cap) return KORE_CUDA_OK;
    float **fb[7] = {&M.bx, &M.bxb, &M.bq, &M.bk, &M.bv, &M.batt, &M.bact};
    for (float **b : fb) {
        cudaFree(*b);
        *b = nullptr;
    }
    cudaFree(M.btok);
    M.btok = nullptr;
    M.pf_cap = 0;
    const int cap = (n + 63) / 64 * 64;
    const size_t E = (size_t)c->H * c->D, kvd = (size_t)c->kvd, FF = (size_t)M.n_ff;
    const size_t floats[7] = {E, E, E, kvd, kvd, E, FF};
    for (int i = 0; i < 7; ++i) CK(cudaMalloc(fb[i], floats[i] * cap * sizeof(float)));
    CK(cudaMalloc(&M.btok, (size_t)cap * sizeof(int)));
    M.pf_cap = cap;
    return KORE_CUDA_OK;
}

static int launch_bmm(kore_cuda_ctx *c, const uint8_t *w, int type, int rows, int cols, int B, const float *x,
                      float *out, const float *bias, const float *resid) {
    BatchMatmulParams bp;
    memset(&bp, 0, sizeof bp);
    bp.seg[0] = QSeg{w, bias, out, type, rows};
    bp.cols = cols;
    bp.B = B;
    bp.x = x;
    bp.out_mode = resid ? QOUT_RESIDUAL : QOUT_STORE;
    bp.resid = resid;
    bp.out_stride = rows;
    CK(launch_batch_matmul(bp, c->stream));
    return KORE_CUDA_OK;
}

// kore's matmul_batch_float (kore.cpp:783-845) of B host rows with one of
// layer's uploaded matrices (0 wq, 1 wk, 2 wv, 3 wo, 4 ffn_gate, 5 ffn_up,
// 6 ffn_down; 4-6 need kore_cuda_set_model): out [B][rows] host.
int kore_cuda_matmul_batch(kore_cuda_ctx *c, int layer, int which, int B, const float *x, float *out) {
    if (!c) return KORE_CUDA_EINVAL;
    if (!x || !out || B <= 0) return fail(c, KORE_CUDA_EINVAL, "null x or out, or B <= 0");
    if (which < 0 || which > 6) return fail(c, KORE_CUDA_EINVAL, "which = %d outside 0..6", which);
    const kore_cuda_ctx::LayerProj *lp = layer_proj(c, layer);
    if (!lp) return fail(c, KORE_CUDA_ESTATE, "no attention weights for layer %d", layer);
    if (which > 3 && (!c->model.ready || layer >= (int)c->model.layers.size()))
        return fail(c, KORE_CUDA_ESTATE, "no feed-forward weights (kore_cuda_set_model)");
    const int E = c->H * c->D, FF = c->model.n_ff;
    const uint8_t *w;
    int type, rows, cols;
    if (which < 4) {
        w = lp->w + lp->off[which];
        type = lp->type[which];
        rows = lp->rows[which];
        cols = E;
    } else {
        const auto &lf = c->model.layers[(size_t)layer];
        w = lf.w + lf.off[which - 4];
        type = lf.type[which - 4];
        rows = which == 6 ? E : FF;
        cols = which == 6 ? FF : E;
    }
    DeviceGuard dg(c->cfg.device);
    const size_t nx = (size_t)B * cols, no = (size_t)B * rows;
    if (int rc = grow_stage(c, nx + no)) return rc;
    CK(cudaMemcpyAsync(c->dev_stage, x, nx * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    if (int rc = launch_bmm(c, w, type, rows, cols, B, c->dev_stage, c->dev_stage + nx, nullptr, nullptr)) return rc;
    CK(cudaMemcpyAsync(out, c->dev_stage + nx, no * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    return finish(c);
}

// kore's forward_batch() (kore.cpp:1486-1598) for n prompt tokens at pos0..,
// every step on the device, then the greedy next token (the argmax of the
// last token's logits, kore.cpp:1594-1597 and :1601-1603):
//   embedding rows                                      embed_kernel
//   per layer: RMSNorm rows                             rmsnorm_rows_kernel
//              Wq/Wk/Wv float products + biases          batch_matmul_kernel (kore's FMA chains)
//              RoPE, append, causal attention            the prefill path (kore_cuda_attn_prefill_dev)
//              Wo product + residual add                batch_matmul_kernel
//              RMSNorm rows, gate/up + SwiGLU            rmsnorm_rows_kernel, batch_matmul_kernel (paired)
//              down product + residual add              batch_matmul_kernel
//   last row: RMSNorm + Q8_K + output matrix + argmax    qmatvec (as the decode step)
// Unlike kore, n is not limited to its 64-token chunk: every product column
// and every attention row is independent of the chunk it is computed in.
int kore_cuda_prefill(kore_cuda_ctx *c, int seq, const int *tokens, int n, int pos0, int *next_token, float *logits) {
    if (!c) return KORE_CUDA_EINVAL;
    if (!tokens || !next_token || n <= 0) return fail(c, KORE_CUDA_EINVAL, "null tokens or next_token, or n <= 0");
    if (!c->model.ready || c->proj.size() != (size_t)c->cfg.n_layer)
        return fail(c, KORE_CUDA_ESTATE, "no model on the device (kore_cuda_set_model)");
    if (c->NS > 1 && !c->peers_open)
        return fail(c, KORE_CUDA_ESTATE, "a KV-split context needs kore_cuda_peer_open before a prefill");
    for (int l = 0; l < c->cfg.n_layer; ++l)
        if (int rc = check_range(c, seq, l, pos0, n)) return rc;
    auto &M = c->model;
    for (int z = 0; z < n; ++z)   // forward_batch returns false (kore.cpp:1496)
        if (tokens[z] < 0 || tokens[z] >= M.n_vocab)
            return fail(c, KORE_CUDA_ERANGE, "token %d (row %d) outside the vocabulary of %d", tokens[z], z, M.n_vocab);
    DeviceGuard dg(c->cfg.device);
    if (int rc = grow_prefill(c, n)) return rc;
    const int E = c->H * c->D, FF = M.n_ff, kvd = c->kvd;
    CK(cudaMemcpyAsync(M.btok, tokens, (size_t)n * sizeof(int), cudaMemcpyHostToDevice, c->stream));
    EmbedParams ep;
    memset(&ep, 0, sizeof ep);
    ep.table = M.tok;
    ep.row_bytes = M.tok_row_bytes;
    ep.type = M.tok_type;
    ep.n_vocab = M.n_vocab;
    ep.n_embd = E;
    ep.n_tokens = n;
    ep.token_dev = M.btok;
    ep.x = M.bx;
    ep.key = M.key;
    ep.err = c->err_d;
    CK(launch_embed(ep, c->stream));
    for (int l = 0; l < c->cfg.n_layer; ++l) {
        const kore_cuda_ctx::LayerProj &lp = c->proj[(size_t)l];
        const kore_cuda_ctx::LayerFfn &lf = M.layers[(size_t)l];
        const float *bias = lp.has_bias ? lp.bias : nullptr;
        CK(launch_rmsnorm_rows(M.bx, lf.norms, M.bxb, n, E, M.eps, c->stream));
        if (int rc = launch_bmm(c, lp.w + lp.off[0], lp.type[0], E, E, n, M.bxb, M.bq, bias, nullptr)) return rc;
        if (int rc = launch_bmm(c, lp.w + lp.off[1], lp.type[1], kvd, E, n, M.bxb, M.bk, bias ? bias + E : nullptr,
                                nullptr))
            return rc;
        if (int rc = launch_bmm(c, lp.w + lp.off[2], lp.type[2], kvd, E, n, M.bxb, M.bv,
                                bias ? bias + E + kvd : nullptr, nullptr))
            return rc;
        if (int rc = kore_cuda_attn_prefill_dev(c, seq, l, pos0, n, M.bq, M.bk, M.bv, M.batt)) return rc;
        if (int rc = launch_bmm(c, lp.w + lp.off[3], lp.type[3], E, E, n, M.batt, M.bx, nullptr, M.bx)) return rc;
        CK(launch_rmsnorm_rows(M.bx, lf.norms + E, M.bxb, n, E, M.eps, c->stream));
        BatchMatmulParams bp;
        memset(&bp, 0, sizeof bp);
        bp.seg[0] = QSeg{lf.w + lf.off[0], nullptr, M.bact, lf.type[0], FF};
        bp.seg[1] = QSeg{lf.w + lf.off[1], nullptr, M.bact, lf.type[1], FF};
        bp.pair = 1;
        bp.cols = E;
        bp.B = n;
        bp.x = M.bxb;
        bp.out_stride = FF;
        memcpy(bp.exp_tab, M.exp_tab, sizeof bp.exp_tab);
        CK(launch_batch_matmul(bp, c->stream));
        if (int rc = launch_bmm(c, lf.w + lf.off[2], lf.type[2], E, FF, n, M.bact, M.bx, nullptr, M.bx)) return rc;
    }
    QMatvecParams mp;
    memset(&mp, 0, sizeof mp);
    mp.n_seg = 1;
    mp.cols = E;
    mp.seg[0] = QSeg{M.out_w, nullptr, M.logits, M.out_type, M.n_vocab};
    mp.in_mode = QIN_RMSNORM;
    mp.x = M.bx + (size_t)(n - 1) * E;
    mp.norm_w = M.out_norm;
    mp.eps = M.eps;
    mp.out_mode = QOUT_ARGMAX;
    mp.argmax = M.key;
    if (int rc = launch_products(c, mp)) return rc;
    int *dnext = reinterpret_cast<int *>(reinterpret_cast<char *>(c->err_d) + kErrPad);
    CK(launch_token(M.key, dnext, c->stream));
    if (logits)
        CK(cudaMemcpyAsync(logits, M.logits, (size_t)M.n_vocab * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    if (int rc = finish(c, sizeof(int))) return rc;
    memcpy(next_token, reinterpret_cast<const char *>(c->host_err) + kErrPad, sizeof(int));
    return KORE_CUDA_OK;
}

int kore_cuda_kv_read(kore_cuda_ctx *c, int seq, int layer, int pos0, int n, float *k_out, float *v_out) {
    if (!c) return KORE_CUDA_EINVAL;
    if (!k_out || !v_out) return fail(c, KORE_CUDA_EINVAL, "null output");
    if (int rc = check_seq_layer(c, seq, layer)) return rc;
    const int len = c->seq_len[(size_t)seq * c->cfg.n_layer + layer];
    if (n <= 0 || pos0 < 0 || pos0 + n > len)
        return fail(c, KORE_CUDA_ERANGE, "positions [%d, %d) outside the %d held", pos0, pos0 + n, len);
    DeviceGuard dg(c->cfg.device);
    CK(cudaStreamSynchronize(c->stream));
    const int *row = c->pt_h.data() + (size_t)seq * c->pages_per_seq;
    const size_t D = c->D;
    for (int z = 0; z < n; ++z) {
        const int pos = pos0 + z, gp = pos / c->P;
        if (gp % c->NS != c->rank) continue;
        const int ph = row[gp / c->NS];
        for (int g = 0; g < c->G; ++g) {
            const float *src = c->kv + (size_t)layer * c->layer_floats + (((size_t)ph * c->G + g) * c->P + (pos - gp * c->P)) * D;
            CK(cudaMemcpyAsync(k_out + ((size_t)z * c->G + g) * D, src, D * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
            CK(cudaMemcpyAsync(v_out + ((size_t)z * c->G + g) * D, src + c->v_off, D * sizeof(float),
                               cudaMemcpyDeviceToHost, c->stream));
        }
    }
    CK(cudaStreamSynchronize(c->stream));
    return KORE_CUDA_OK;
}

int kore_cuda_set_wait_limit(kore_cuda_ctx *c, unsigned long long nanoseconds) {
    if (!c) return KORE_CUDA_EINVAL;
    c->wait_ns = nanoseconds ? nanoseconds : kWaitNs;
    return KORE_CUDA_OK;
}

int kore_cuda_sync(kore_cuda_ctx *c) {
    if (!c) return KORE_CUDA_EINVAL;
    DeviceGuard dg(c->cfg.device);
    return finish(c);
}

void *kore_cuda_stream(kore_cuda_ctx *c) { return c ? (void *)c->stream : nullptr; }

int kore_cuda_set_stream(kore_cuda_ctx *c, void *stream) {
    if (!c) return KORE_CUDA_EINVAL;
    DeviceGuard dg(c->cfg.device);
    CK(cudaStreamSynchronize(c->stream));
    if (c->own_stream) cudaStreamDestroy(c->stream);
    c->stream = (cudaStream_t)stream;
    c->own_stream = false;
    c->last_kv_layer = -1;   // the old stream was drained above: nothing of ours is in flight
    return KORE_CUDA_OK;
}

}  // extern "C"
