/*
 * kore_cuda.h — C ABI of the B200 attention path for kore (BJZR/kore).
 *
 * kore has no attention function: its attention is inlined in forward()
 * (decode, kore.cpp:1424-1455) and forward_batch() (prefill,
 * kore.cpp:1535-1563), reading and writing the fp32 KV cache
 * Engine::kcache/vcache (kore.cpp:1260, allocated at :1344-1345). The entry
 * points below replace exactly those regions. Their inputs are what kore holds
 * at the start of each region: the bias-added, PRE-RoPE q, k and v
 * (e.q/e.k/e.v, or the e.bq/e.bk/e.bv rows); their output is what the region
 * leaves in e.att / e.batt ([tokens][n_head*head_dim], head-major within a
 * token), which kore then feeds to the Wo projection (kore.cpp:1456, :1566).
 *
 * The KV cache moves into the context: it is device-resident, fp32 as in the
 * reference, paged (page_tokens positions per page, one page table per
 * sequence shared by all layers) so that several sequences share one pool.
 *
 * Conventions
 *  - Every function returns KORE_CUDA_OK (0) or a negative KORE_CUDA_E* code
 *    and leaves a message for kore_cuda_last_error(); none aborts or exits.
 *    kore maps a non-zero return to `return false` from forward() /
 *    forward_batch(), as it does for a bad token or position
 *    (kore.cpp:1400, :1490).
 *  - Host-pointer entry points copy their inputs to the device, run on the
 *    context's stream, copy the output back and return once it is valid.
 *  - *_dev entry points take device pointers (q, k, v 16-byte aligned, as
 *    any cudaMalloc'd row of n_head*head_dim floats is), are ordered on the
 *    context's stream and return without synchronising; kore_cuda_sync()
 *    waits and reports any error raised on the device since the last check.
 *  - A context is not re-entrant: one host thread at a time (kore calls
 *    attention from its main thread, or from the HTTP handler under the
 *    session mutex, kore.cpp:2600).
 */
#ifndef KORE_CUDA_H
#define KORE_CUDA_H

#ifdef __cplusplus
extern "C" {
#endif

#define KORE_CUDA_ABI_VERSION 1

enum kore_cuda_status {
    KORE_CUDA_OK = 0,
    KORE_CUDA_EINVAL = -1,   /* bad argument: shape, null pointer, unsupported head_dim */
    KORE_CUDA_ERANGE = -2,   /* seq / layer / position outside the limits (kore.cpp:1400, :1490) */
    KORE_CUDA_ENOMEM = -3,   /* device memory or KV pages exhausted */
    KORE_CUDA_ECUDA = -4,    /* a CUDA runtime call failed */
    KORE_CUDA_ESTATE = -5,   /* out-of-order call, e.g. attending at pos with rows missing below it */
    KORE_CUDA_EDEVICE = -6,  /* a kernel reported an error (bounded wait expired, bad page) */
    KORE_CUDA_ENCCL = -7     /* a cross-GPU exchange failed */
};

typedef struct kore_cuda_ctx kore_cuda_ctx;

typedef struct kore_cuda_cfg {
    int n_layer;            /* hp.n_layer */
    int n_head;             /* hp.n_head, H */
    int n_head_kv;          /* hp.n_head_kv, G; H % G == 0, H/G <= 8 */
    int head_dim;           /* e.head_dim, d: 64 or 128 */
    int ctx_max;            /* e.ctx: positions per sequence (kore.cpp:1291) */
    int max_seqs;           /* sequences sharing the page pool; kore's single session uses 1 */
    int page_tokens;        /* positions per KV page, a multiple of 64; 0 selects 256 */
    int n_pages;            /* pages per layer in the pool; 0 selects max_seqs*ceil(ctx_max/page_tokens) */
    float rope_base;        /* hp.rope_base (kore.cpp:230) */
    const float *inv_freq;  /* optional host [head_dim/2], e.inv_freq; NULL builds it as kore.cpp:1339 */
    int device;             /* CUDA device ordinal */
    int shard_rank;         /* KV-sequence split over GPUs: this context holds the positions of */
    int shard_count;        /*   every page j with j % shard_count == shard_rank; 0/1 = unsplit */
} kore_cuda_cfg;

/* Fills *cfg with defaults for the given geometry (page_tokens 256, one
 * sequence, rope_base 1e6, device 0, unsplit). */
void kore_cuda_cfg_default(kore_cuda_cfg *cfg, int n_layer, int n_head, int n_head_kv,
                           int head_dim, int ctx_max);

/* Creates a context: KV page pool for all layers, RoPE angle tables for
 * positions [0, ctx_max) built on the host exactly as kore.cpp:1405-1410
 * builds them, a stream and staging buffers. Replaces the KV allocation of
 * engine_init (kore.cpp:1344-1345). */
int kore_cuda_create(kore_cuda_ctx **out, const kore_cuda_cfg *cfg);
void kore_cuda_destroy(kore_cuda_ctx *ctx);

/* Message for the last failed call on ctx (or on a failed create when ctx is
 * NULL). Never NULL. */
const char *kore_cuda_last_error(const kore_cuda_ctx *ctx);

/* Drops a sequence's pages: kore starting a new conversation, or about to
 * re-prefill from position 0 (condense, kore.cpp:1790-1796). */
int kore_cuda_seq_reset(kore_cuda_ctx *ctx, int seq);

/* Number of positions of (seq, layer) currently held, i.e. the next position
 * that may be appended. */
int kore_cuda_seq_len(const kore_cuda_ctx *ctx, int seq, int layer);

/* Keeps the first n positions of a sequence in every layer and gives the
 * pages wholly past them back to the pool: a conversation rebuilt shorter
 * (condense, kore.cpp:1760-1799) then appends from n. kore itself only
 * overwrites from position 0 and leaves the stale rows, which its attention
 * never reads again (kore.cpp:1763-1765); dropping them frees the pages. */
int kore_cuda_seq_truncate(kore_cuda_ctx *ctx, int seq, int n);

/*
 * RoPE + append of n tokens at positions pos0..pos0+n-1 of (seq, layer):
 * k is rotated with the tables of its position and stored, v is stored as
 * is (kore.cpp:1425, :1429-1430 for one token; :1534-1538 per batch row).
 *   k, v: [n][n_head_kv*head_dim], bias-added, pre-RoPE
 * pos0 may not exceed the current length (no holes); rows at and past pos0
 * are overwritten.
 */
int kore_cuda_kv_append(kore_cuda_ctx *ctx, int seq, int layer, int pos0, int n,
                        const float *k, const float *v);
int kore_cuda_kv_append_dev(kore_cuda_ctx *ctx, int seq, int layer, int pos0, int n,
                            const float *k, const float *v);

/*
 * Prefill chunk, replacing kore.cpp:1527-1563: appends k/v for positions
 * pos0..pos0+n-1 (as kore_cuda_kv_append), then causal grouped-query
 * attention of the n queries (RoPE'd at their positions) over positions
 * 0..pos0+z for query row z.
 *   q: [n][n_head*head_dim], k, v: [n][n_head_kv*head_dim]   (pre-RoPE)
 *   out: [n][n_head*head_dim]                                 (e.batt rows)
 * n is not limited to kore's 64-token batch (KORE_BMAX, kore.cpp:690). On a
 * context with shard_count > 1 (after kore_cuda_peer_open; every rank makes
 * the same call) each rank stores the rows of its own pages, attends the
 * queries over its own positions, and the partials are merged over NVLink
 * peer memory as the sharded decode merges them; every rank gets all of out.
 */
int kore_cuda_attn_prefill(kore_cuda_ctx *ctx, int seq, int layer, int pos0, int n,
                           const float *q, const float *k, const float *v, float *out);
int kore_cuda_attn_prefill_dev(kore_cuda_ctx *ctx, int seq, int layer, int pos0, int n,
                               const float *q, const float *k, const float *v, float *out);

/*
 * Decode step, replacing kore.cpp:1424-1455 for one layer: RoPE of q and k
 * at `pos`, append of k/v at `pos`, attention of the n_head queries over
 * positions 0..pos.
 *   q: [n_head*head_dim], k, v: [n_head_kv*head_dim]   (pre-RoPE)
 *   out: [n_head*head_dim]                             (e.att)
 */
int kore_cuda_attn_decode(kore_cuda_ctx *ctx, int seq, int layer, int pos,
                          const float *q, const float *k, const float *v, float *out);
int kore_cuda_attn_decode_dev(kore_cuda_ctx *ctx, int seq, int layer, int pos,
                              const float *q, const float *k, const float *v, float *out);

/*
 * Decode step for n_seq sequences at once (one token each, own positions):
 * the batched form of kore_cuda_attn_decode over the shared page pool.
 *   seq_ids, pos: host arrays [n_seq]
 *   q: [n_seq][n_head*head_dim], k, v: [n_seq][n_head_kv*head_dim], out like q
 */
int kore_cuda_attn_decode_batch(kore_cuda_ctx *ctx, int layer, int n_seq, const int *seq_ids,
                                const int *pos, const float *q, const float *k, const float *v,
                                float *out);
int kore_cuda_attn_decode_batch_dev(kore_cuda_ctx *ctx, int layer, int n_seq, const int *seq_ids,
                                    const int *pos, const float *q, const float *k, const float *v,
                                    float *out);

/*
 * The attention block with its quantised projections on the GPU.
 *
 * kore's decode step wraps the attention region in four projections
 * (kore.cpp:1418-1423 and :1456-1457): the normed hidden state xb is
 * quantised to Q8_K (quantize_row_q8_K, kore.cpp:422-447), multiplied by Wq,
 * Wk and Wv (GGUF Q4_K or Q6_K blocks, matvec_mt, kore.cpp:649-682) and
 * bias-added, the attention runs, and its output is quantised again and
 * multiplied by Wo. With the weights uploaded once, the whole block runs on
 * the device: the host passes xb and gets Wo*att back, instead of moving
 * q, k, v and att across PCIe around every attention call.
 *
 * Results equal kore's own bit for bit: the Q8_K quantisation exactly, the
 * products in the lane and summation order of kore's AVX2 kernels
 * (kore.cpp:540-640, the ones kore runs on every AVX2/FMA CPU), the bias add
 * as kore.cpp:1422-1423.
 */
#define KORE_CUDA_Q4_K 12   /* GGUF tensor type ids (kore.cpp:161) */
#define KORE_CUDA_Q6_K 14

typedef struct kore_cuda_qmat {
    int type;           /* KORE_CUDA_Q4_K (144-byte blocks) or KORE_CUDA_Q6_K (210-byte blocks) */
    int rows;           /* output values */
    int cols;           /* input values, a multiple of 256 */
    const void *data;   /* host, rows * cols/256 blocks in GGUF order (Tensor::data, kore.cpp:168) */
} kore_cuda_qmat;

/* Uploads one layer's attention projections (Layer::wq/wk/wv/wo, bq/bk/bv,
 * kore.cpp:1246-1249) into device memory, replacing any earlier upload:
 *   wq [n_head*head_dim x n_embd], wk, wv [n_head_kv*head_dim x n_embd],
 *   wo [n_embd x n_head*head_dim], with n_embd = n_head*head_dim a multiple of
 *   256 (engine_init's own condition, kore.cpp:1283);
 *   bq [n_head*head_dim], bk, bv [n_head_kv*head_dim] fp32 host arrays, or
 *   NULL for none. Synchronous. */
int kore_cuda_set_attn_weights(kore_cuda_ctx *ctx, int layer, const kore_cuda_qmat *wq,
                               const kore_cuda_qmat *wk, const kore_cuda_qmat *wv,
                               const kore_cuda_qmat *wo, const float *bq, const float *bk,
                               const float *bv);

/* kore's mv() with quant() (kore.cpp:1388-1394) for one uploaded matrix of
 * `layer` (which: 0 = wq, 1 = wk, 2 = wv, 3 = wo): out = W * quantize(x),
 * plus the matrix's bias for wq/wk/wv. x [cols] and out [rows] are host
 * arrays. */
int kore_cuda_qmatvec(kore_cuda_ctx *ctx, int layer, int which, const float *x, float *out);

/* One decode step of the attention block, kore.cpp:1419-1457 from the
 * quantisation of xb to o = Wo * att: q/k/v projections + biases, RoPE,
 * append of k/v at pos, attention over positions 0..pos (as
 * kore_cuda_attn_decode), the quantisation of att and Wo.
 *   xb: [n_embd] (kore's e.xb after the attention rmsnorm)
 *   o:  [n_embd] (kore's e.o, before the residual add)
 * On a context with shard_count > 1 the attention is the peer-exchange split
 * (kore_cuda_attn_decode_sharded_dev; kore_cuda_peer_open first) and every
 * rank computes the projections. The _dev form takes 16-byte aligned device
 * pointers and is stream-ordered. */
int kore_cuda_attn_block_decode(kore_cuda_ctx *ctx, int seq, int layer, int pos, const float *xb,
                                float *o);
int kore_cuda_attn_block_decode_dev(kore_cuda_ctx *ctx, int seq, int layer, int pos,
                                    const float *xb, float *o);

/*
 * The whole decode step on the GPU.
 *
 * kore's forward() (kore.cpp:1397-1480) for one token and its greedy choice
 * (sample_token at temperature 0, kore.cpp:1601-1603), all on the device:
 * the token's embedding row (get_row, kore.cpp:384-407), per layer the
 * attention block above with its RMSNorm (kore.cpp:1367-1372) and residual
 * add, the SwiGLU feed-forward (kore.cpp:1460-1471) with its RMSNorm and
 * residual add, then the output RMSNorm, the logits (kore.cpp:1474-1478) and
 * their argmax (the first index of the largest logit). With the weights
 * uploaded once (kore_cuda_set_model), a step moves a token id in and a token
 * id out, instead of crossing PCIe around every layer.
 *
 * Arithmetic is kore's own in every step but the attention (which is within
 * the attention tolerance, as kore_cuda_attn_decode): the Q8_K quantisations
 * and the Q4_K / Q6_K products bit for bit (as kore_cuda_qmatvec), the
 * RMSNorm with kore's double-precision sum of squares, the SwiGLU with the
 * C library's expf as kore calls it, the residual adds and the embedding
 * dequantisation with kore's rounding. A step at position 0 (one key: the
 * attention is exact too) therefore gives kore's logits bit for bit.
 */
#define KORE_CUDA_F32 0     /* GGUF tensor type ids of the embedding tables get_row reads */
#define KORE_CUDA_F16 1
#define KORE_CUDA_BF16 30

typedef struct kore_cuda_layer_weights {
    kore_cuda_qmat wq, wk, wv, wo;    /* as kore_cuda_set_attn_weights (Layer::wq.., kore.cpp:1246-1249) */
    const float *bq, *bk, *bv;        /* host, or all NULL */
    const float *attn_norm;           /* host [n_embd] (Layer::attn_norm) */
    const float *ffn_norm;            /* host [n_embd] (Layer::ffn_norm) */
    kore_cuda_qmat w_gate, w_up;      /* [n_ff x n_embd], Q4_K or Q6_K */
    kore_cuda_qmat w_down;            /* [n_embd x n_ff], Q4_K or Q6_K */
} kore_cuda_layer_weights;

typedef struct kore_cuda_model {
    int n_ff;                         /* hp.n_ff, a multiple of 256 */
    int n_vocab;                      /* rows of tok_embd and out_w */
    float rms_eps;                    /* hp.rms_eps */
    kore_cuda_qmat tok_embd;          /* [n_vocab x n_embd]: type F32, F16, BF16, Q4_K or Q6_K */
    const float *out_norm;            /* host [n_embd] (Engine::out_norm) */
    kore_cuda_qmat out_w;             /* [n_vocab x n_embd], Q4_K or Q6_K (Engine::out_w) */
    const kore_cuda_layer_weights *layers;   /* [n_layer] */
} kore_cuda_model;

/* Uploads the whole model (every layer's attention projections as
 * kore_cuda_set_attn_weights does, norms, feed-forward weights, embedding
 * table, output norm and matrix), replacing any earlier upload. Synchronous. */
int kore_cuda_set_model(kore_cuda_ctx *ctx, const kore_cuda_model *model);

/* One decode step of sequence `seq`: `token` at `pos` through every layer
 * (appending its k/v at pos in every layer's cache), then the greedy next
 * token into *next_token; logits [n_vocab] (host, optional) receives the
 * logits as kore's e.logits. Returns KORE_CUDA_ERANGE for a token outside the
 * vocabulary or a bad position, as forward() returns false (kore.cpp:1400).
 * On a context with shard_count > 1 every rank makes the same calls. */
int kore_cuda_decode_step(kore_cuda_ctx *ctx, int seq, int token, int pos, int *next_token, float *logits);
/* The same, stream-ordered: token and next_token are device ints (they may be
 * the same int, so that steps chain on the device), logits an optional device
 * [n_vocab]. A token outside the vocabulary is reported by kore_cuda_sync. */
int kore_cuda_decode_step_dev(kore_cuda_ctx *ctx, int seq, const int *token, int pos, int *next_token,
                              float *logits);

/* kore's forward_batch() (kore.cpp:1486-1598) for n prompt tokens at
 * positions pos0..pos0+n-1 of sequence `seq`, on the device: the float
 * projections of its prefill (matmul_batch_float, kore.cpp:783-845: each
 * weight block dequantised to fp32, one fused multiply-add per column in
 * column order; bit for bit kore's), the biases, RoPE, the cache append, the
 * causal attention (as kore_cuda_attn_prefill), the residual adds, the
 * SwiGLU feed-forward and, for the last token, the logits (optional host
 * logits [n_vocab]) and the greedy next token (*next_token) as kore's
 * prefill() leaves them for gen_step (kore.cpp:1720-1750). n is not limited
 * to kore's 64-token chunk (KORE_BMAX, kore.cpp:690): chunking changes no
 * value. Returns KORE_CUDA_ERANGE for a token outside the vocabulary. */
int kore_cuda_prefill(kore_cuda_ctx *ctx, int seq, const int *tokens, int n, int pos0, int *next_token,
                      float *logits);

/* kore's matmul_batch_float (kore.cpp:783-845), the float product of its
 * prefill, of B host rows x [B][cols] with one uploaded matrix of `layer`
 * (which: 0 wq, 1 wk, 2 wv, 3 wo, 4 ffn_gate, 5 ffn_up, 6 ffn_down; 4-6 after
 * kore_cuda_set_model): out [B][rows] host, bit for bit kore's (no bias). */
int kore_cuda_matmul_batch(kore_cuda_ctx *ctx, int layer, int which, int B, const float *x, float *out);

/*
 * Many chat sessions over one context (the model uploaded with
 * kore_cuda_set_model): kore's ChatSession, prefill(), gen_step() and
 * condense() (kore.cpp:1674-1799) with every session a sequence of the
 * shared page pool (cfg.max_seqs sessions at most).
 *  - open: admits a session (a free sequence slot, emptied); close: retires
 *    it and frees its pages.
 *  - submit: a turn's token ids, appended after the session's conversation
 *    at the next step (kore's prefill(), with its length check: the turn must
 *    leave room in the context); max_new bounds the tokens generated for it
 *    (0: until eos/bos or a full context).
 *  - step: one round: every submitted turn is prefilled on the device
 *    (kore_cuda_prefill), then every generating session takes one greedy
 *    gen_step: the token sampled from its last logits is reported, and
 *    unless it is eos/bos or the context is full it is appended and run
 *    through the whole model (kore_cuda_decode_step_dev). The sessions'
 *    steps are queued back to back with their tokens kept on the device;
 *    the host reads the next tokens back once per round. events receives
 *    one entry per session that was generating.
 *  - condense: rebuilds a session's cache from position 0 over the token ids
 *    given (kore's re-prefill of {system + summary} + recent tail,
 *    kore.cpp:1786-1797); the session stops generating until its next turn.
 * Not re-entrant: one host thread at a time, as the context.
 */
typedef struct kore_cuda_server kore_cuda_server;

enum kore_cuda_event_status {
    KORE_CUDA_EV_TOKEN = 0,   /* token generated and appended */
    KORE_CUDA_EV_END = 1,     /* eos or bos sampled (not appended): the session stops generating */
    KORE_CUDA_EV_FULL = 2,    /* the context is full (token not appended): the session stops */
    KORE_CUDA_EV_LIMIT = 3    /* token generated and appended; the turn's max_new is reached */
};

typedef struct kore_cuda_event {
    int session;
    int token;
    int status;               /* kore_cuda_event_status */
} kore_cuda_event;

int kore_cuda_server_create(kore_cuda_server **out, kore_cuda_ctx *ctx, int eos_token, int bos_token);
void kore_cuda_server_destroy(kore_cuda_server *srv);
const char *kore_cuda_server_last_error(const kore_cuda_server *srv);
int kore_cuda_server_open(kore_cuda_server *srv, int *session);
int kore_cuda_server_close(kore_cuda_server *srv, int session);
int kore_cuda_server_submit(kore_cuda_server *srv, int session, const int *ids, int n, int max_new);
int kore_cuda_server_step(kore_cuda_server *srv, kore_cuda_event *events, int max_events, int *n_events);
int kore_cuda_server_condense(kore_cuda_server *srv, int session, const int *ids, int n);
/* The session's conversation (every token in its cache): copies up to cap
 * ids and returns the length, or KORE_CUDA_ERANGE for a session not open. */
int kore_cuda_server_history(const kore_cuda_server *srv, int session, int *ids, int cap);

/*
 * KV-sequence split over GPUs (cfg.shard_count > 1). Each context holds the
 * positions of every page j with j % shard_count == shard_rank; a decode step
 * then runs in two parts:
 *   kore_cuda_attn_decode_partial_dev: this shard's share of the decode at
 *     pos (the owner of pos also appends k/v there). `part` receives the
 *     packed partial [n_head*head_dim outputs normalised by this shard's own
 *     softmax sum][n_head log2-domain log-sum-exp values], -inf where the
 *     shard holds none of positions 0..pos.
 *   kore_cuda_lse_merge_dev: merges n_parts packed partials (laid out one
 *     after another, as an all-gather leaves them) into out [n_head*head_dim].
 * The merge is kore's single softmax (kore.cpp:1437-1454) regrouped by shard.
 * Device pointers; stream-ordered.
 */
int kore_cuda_attn_decode_partial_dev(kore_cuda_ctx *ctx, int seq, int layer, int pos,
                                      const float *q, const float *k, const float *v, float *part);
int kore_cuda_lse_merge_dev(kore_cuda_ctx *ctx, int n_parts, const float *parts, float *out);
/* The same for a prefill chunk (kore.cpp:1527-1563): the owner of each of
 * positions pos0..pos0+n-1 appends its k/v, and `part` receives this shard's
 * causal partial of the n queries, outputs [n][n_head*head_dim] then
 * log2-domain LSEs [n][n_head] (n <= 256). kore_cuda_lse_merge_batch_dev
 * merges n_parts such partials of n_q queries (one after another) into out
 * [n_q][n_head*head_dim]. */
int kore_cuda_attn_prefill_partial_dev(kore_cuda_ctx *ctx, int seq, int layer, int pos0, int n,
                                       const float *q, const float *k, const float *v, float *part);
int kore_cuda_lse_merge_batch_dev(kore_cuda_ctx *ctx, int n_parts, int n_q, const float *parts, float *out);

/*
 * The same split with the exchange done by this library over NVLink peer
 * memory instead of by the caller. Each rank exports its exchange buffer
 * (kore_cuda_peer_handle: a CUDA IPC handle of KORE_CUDA_PEER_HANDLE_BYTES),
 * the caller passes all ranks' handles, in rank order, to every rank
 * (kore_cuda_peer_open), and then kore_cuda_attn_decode_sharded_dev runs one
 * layer's decode step on every rank and leaves the full merged output
 * [n_head*head_dim] on every rank: the partial, a push of it into every
 * peer's memory with a flag, a bounded wait (2 s, then KORE_CUDA_EDEVICE from
 * kore_cuda_sync) for the peers' partials, and the merge. Every rank must make
 * the same sequence of calls. One process per GPU; shard_count <= 8.
 */
#define KORE_CUDA_PEER_HANDLE_BYTES 64
int kore_cuda_peer_handle(kore_cuda_ctx *ctx, void *handle);
int kore_cuda_peer_open(kore_cuda_ctx *ctx, const void *handles);
int kore_cuda_attn_decode_sharded_dev(kore_cuda_ctx *ctx, int seq, int layer, int pos,
                                      const float *q, const float *k, const float *v, float *out);
/* The same with kore's host buffers (as kore_cuda_attn_decode): q/k/v in,
 * the merged output back, on every rank. */
int kore_cuda_attn_decode_sharded(kore_cuda_ctx *ctx, int seq, int layer, int pos,
                                  const float *q, const float *k, const float *v, float *out);

/* Copies positions pos0..pos0+n-1 of (seq, layer) back to the host in kore's
 * row layout, k_out/v_out [n][n_head_kv*head_dim] (post-RoPE keys), so that a
 * caller can compare with or restore Engine::kcache/vcache. */
int kore_cuda_kv_read(kore_cuda_ctx *ctx, int seq, int layer, int pos0, int n,
                      float *k_out, float *v_out);

/* Waits for the context's stream; returns KORE_CUDA_EDEVICE if a kernel
 * raised its error flag since the last check. */
int kore_cuda_sync(kore_cuda_ctx *ctx);

/* Limit of every bounded wait inside the decode and peer-exchange kernels of
 * this context (a K/V tile copy, a peer GPU's partial), in nanoseconds of the
 * GPU's global timer; 0 restores the default of 2 s. A kernel whose wait runs
 * out records the failure, waits for its own copies still in flight and
 * returns; the next kore_cuda_sync (or host-buffer call) reports
 * KORE_CUDA_EDEVICE with a message naming the wait, and the context stays
 * usable. kore has no counterpart (its attention cannot wait on anything):
 * this is the failure detection of the multi-GPU split, where a rank that
 * died or fell behind would otherwise leave its peers waiting. */
int kore_cuda_set_wait_limit(kore_cuda_ctx *ctx, unsigned long long nanoseconds);

/* The context's stream (a cudaStream_t) and a way to replace it with the
 * caller's (for interop with an engine that already owns a stream). */
void *kore_cuda_stream(kore_cuda_ctx *ctx);
int kore_cuda_set_stream(kore_cuda_ctx *ctx, void *stream);

/*
 * Decode for callers that cannot allocate GPU memory.
 *
 * No counterpart in the reference: kore has no GPU code, and this entry point
 * is an addition of this library. Some hosts own all device memory themselves
 * and forbid allocations once they run: an inference server that carves
 * every buffer out of its own pre-reserved pool (so that a stray cudaMalloc
 * cannot fragment memory or stall its other streams), or a plugin whose host
 * hands it device buffers and a stream but no permission to allocate. Such a
 * caller cannot create a context (kore_cuda_create allocates the KV pool,
 * the RoPE tables and split scratch). Here it lays the paged KV cache out
 * itself, in a context's layout (kore_cuda_kv_view), and passes every input
 * and output; the call allocates nothing. The KV-split scratch it needs is a
 * fixed array inside the library, KORE_CUDA_NOALLOC_SCRATCH_BYTES on every
 * GPU that loads the library, held until the process exits.
 *
 *  - The first call on a device looks up the array's device address (a
 *    one-time set-up done with that device current, repeated for each CUDA
 *    context the caller makes current on it); make that first call before any
 *    stream capture. The address belongs to the context it was looked up in:
 *    after cudaDeviceReset, reload the library before calling again.
 *  - All calls on a device share the one array and it keeps the last call's
 *    contents, so calls that overlap on the GPU (on different streams, or from
 *    host threads without ordering) race and corrupt each other's results:
 *    serialise them. Nothing in it has to start at zero: a call writes every
 *    slot it later reads.
 *  - A geometry whose split scratch would exceed the array is refused with
 *    KORE_CUDA_EINVAL and a message (kore_cuda_last_error(NULL)).
 */
#define KORE_CUDA_NOALLOC_SCRATCH_BYTES (2359296)   /* 2.25 MiB */

typedef struct kore_cuda_kv_view {
    float *k_pages;         /* device [n_pages][n_head_kv][page_tokens][head_dim], post-RoPE keys */
    float *v_pages;         /* device, same layout, values */
    const int *page_table;  /* device [n_table]: physical page of logical page j */
    int n_table;
    int n_pages;
    int page_tokens;        /* a multiple of 64 */
    int n_head, n_head_kv, head_dim;   /* as in kore_cuda_cfg */
    const float *rope_cs;   /* device [n_rope][head_dim/2][2]: (cos, sin) per position, kore.cpp:1405-1410 */
    int n_rope;
} kore_cuda_kv_view;

/* One decode step of the sequence described by kv: RoPE of q and k at pos,
 * append of k/v at pos (written into kv's pages), attention over positions
 * 0..pos, output to out [n_head*head_dim]. q, k, v, out and dev_status are
 * device pointers; dev_status (optional, zeroed by the caller) receives the
 * first failure a kernel meets: 3 for a page id outside the pool, 1 for a
 * K/V tile copy that did not land within 2 s. Ordered on `stream` (a
 * cudaStream_t; NULL for the default stream); returns without synchronising.
 * Every input (pages, page table, q/k/v, RoPE table) may be written by the
 * kernel just before on the stream, even one that lets its dependents start
 * early: this call reads nothing before that kernel has completed. */
int kore_cuda_attn_decode_noalloc(const kore_cuda_kv_view *kv, int pos, const float *q, const float *k,
                                  const float *v, float *out, int *dev_status, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* KORE_CUDA_H */
