// server.cu — many chat sessions over one context: kore's ChatSession,
// prefill(), gen_step() and condense() (kore.cpp:1674-1799) on the device.
//
// kore serves one conversation at a time: a ChatSession holds the engine (its
// KV cache), the token history `conv` and a `generating` flag; prefill()
// appends a turn's ids to the cache with forward_batch and leaves the logits
// of its last token; gen_step() samples from the logits, stops on eos/bos or a
// full context, else appends the token and runs forward() for the next
// logits; condense() rebuilds the cache from position 0 over a shorter
// history. Here every session is a sequence of one context's shared page
// pool, with the whole model on the device (kore_cuda_set_model):
//   * a submitted turn is prefilled with kore_cuda_prefill at the session's
//     current length (kore's prefill(), same length check);
//   * one round (kore_cuda_server_step) prefills every submitted turn and
//     then advances every generating session by one gen_step: the token
//     sampled from its last logits is checked (eos/bos, full context, the
//     turn's token limit), appended and run through the model with
//     kore_cuda_decode_step_dev. The next tokens stay on the device: the
//     sessions' steps are queued back to back on the context's stream, each
//     reading its token from and writing its next token to the session's
//     device slot, and the host reads all next tokens back with one copy
//     and one synchronisation per round;
//   * close frees a session's pages for the next one (the pool is shared);
//   * condense rebuilds a session's cache from position 0 over the history
//     the caller passes (kore's condense after its summary, kore.cpp:1786-
//     1797): the stale positions beyond it are dropped first.
// Greedy sampling only (kore's temp <= 0 path, sample_token kore.cpp:1601-
// 1603); the sampling at a temperature is host-side randomness and stays
// kore's.

#include "../../include/kore_cuda.h"
#include "attn.cuh"

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

struct kore_cuda_server {
    struct Session {
        bool open = false, generating = false;
        std::vector<int> conv;      // every token in the session's cache, in order
        std::vector<int> pending;   // a submitted turn, prefilled at the next round
        int max_new = 0, emitted = 0;
    };
    kore_cuda_ctx *ctx = nullptr;
    int eos = -1, bos = -1;
    int n_seq = 0, ctx_max = 0, n_vocab = 0, device = 0;
    std::vector<Session> s;
    int *next_dev = nullptr;    // [n_seq] each session's next token, on the device
    int *next_host = nullptr;   // [n_seq] pinned copy, read back once per round
    std::string msg = "no error";
};

namespace {

thread_local std::string g_server_msg = "no error";

int sfail(kore_cuda_server *v, int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (v) v->msg = buf;
    else g_server_msg = buf;
    return code;
}

// A context call failed: its message becomes the server's.
int from_ctx(kore_cuda_server *v, int rc) {
    v->msg = std::string("context: ") + kore_cuda_last_error(v->ctx);
    return rc;
}

int check_session(kore_cuda_server *v, int session) {
    if (session < 0 || session >= v->n_seq || !v->s[(size_t)session].open)
        return sfail(v, KORE_CUDA_ERANGE, "session %d is not open", session);
    return KORE_CUDA_OK;
}

}  // namespace

extern "C" {

const char *kore_cuda_server_last_error(const kore_cuda_server *v) {
    return v ? v->msg.c_str() : g_server_msg.c_str();
}

int kore_cuda_server_create(kore_cuda_server **out, kore_cuda_ctx *ctx, int eos_token, int bos_token) {
    if (!out || !ctx) return sfail(nullptr, KORE_CUDA_EINVAL, "null argument");
    *out = nullptr;
    int ctx_max = 0, max_seqs = 0, n_vocab = 0, device = 0;
    if (!kore::ctx_limits(ctx, &ctx_max, &max_seqs, &n_vocab, &device) || n_vocab <= 0)
        return sfail(nullptr, KORE_CUDA_ESTATE, "the context has no model (kore_cuda_set_model first)");
    auto *v = new kore_cuda_server;
    v->ctx = ctx;
    v->eos = eos_token;
    v->bos = bos_token;
    v->n_seq = max_seqs;
    v->ctx_max = ctx_max;
    v->n_vocab = n_vocab;
    v->device = device;
    v->s.resize((size_t)max_seqs);
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    cudaError_t e = cudaMalloc(&v->next_dev, (size_t)max_seqs * sizeof(int));
    if (e == cudaSuccess) e = cudaMallocHost(&v->next_host, (size_t)max_seqs * sizeof(int));
    if (prev >= 0) cudaSetDevice(prev);
    if (e != cudaSuccess) {
        kore_cuda_server_destroy(v);
        return sfail(nullptr, KORE_CUDA_ENOMEM, "server buffers: %s", cudaGetErrorString(e));
    }
    *out = v;
    return KORE_CUDA_OK;
}

void kore_cuda_server_destroy(kore_cuda_server *v) {
    if (!v) return;
    if (v->ctx) kore_cuda_sync(v->ctx);
    cudaFree(v->next_dev);
    if (v->next_host) cudaFreeHost(v->next_host);
    delete v;
}

int kore_cuda_server_open(kore_cuda_server *v, int *session) {
    if (!v || !session) return sfail(v, KORE_CUDA_EINVAL, "null argument");
    for (int i = 0; i < v->n_seq; ++i) {
        auto &S = v->s[(size_t)i];
        if (S.open) continue;
        if (int rc = kore_cuda_seq_reset(v->ctx, i)) return from_ctx(v, rc);   // a new conversation
        S = kore_cuda_server::Session();
        S.open = true;
        *session = i;
        return KORE_CUDA_OK;
    }
    return sfail(v, KORE_CUDA_ENOMEM, "all %d sessions are open", v->n_seq);
}

int kore_cuda_server_close(kore_cuda_server *v, int session) {
    if (!v) return KORE_CUDA_EINVAL;
    if (int rc = check_session(v, session)) return rc;
    if (int rc = kore_cuda_seq_reset(v->ctx, session)) return from_ctx(v, rc);   // its pages back to the pool
    v->s[(size_t)session] = kore_cuda_server::Session();
    return KORE_CUDA_OK;
}

int kore_cuda_server_submit(kore_cuda_server *v, int session, const int *ids, int n, int max_new) {
    if (!v) return KORE_CUDA_EINVAL;
    if (int rc = check_session(v, session)) return rc;
    if (!ids || n <= 0) return sfail(v, KORE_CUDA_EINVAL, "empty turn");
    auto &S = v->s[(size_t)session];
    if (!S.pending.empty()) return sfail(v, KORE_CUDA_ESTATE, "session %d already has a turn waiting", session);
    // kore's prefill(): the turn must leave room in the context (kore.cpp:1722)
    if ((long long)S.conv.size() + n >= v->ctx_max)
        return sfail(v, KORE_CUDA_ERANGE, "turn of %d tokens after %zu does not fit the context of %d", n, S.conv.size(),
                     v->ctx_max);
    for (int i = 0; i < n; ++i)
        if (ids[i] < 0 || ids[i] >= v->n_vocab)
            return sfail(v, KORE_CUDA_ERANGE, "token %d outside the vocabulary of %d", ids[i], v->n_vocab);
    S.pending.assign(ids, ids + n);
    S.max_new = max_new > 0 ? max_new : 0x7fffffff;
    S.emitted = 0;
    S.generating = false;
    return KORE_CUDA_OK;
}

int kore_cuda_server_step(kore_cuda_server *v, kore_cuda_event *events, int max_events, int *n_events) {
    if (!v || !n_events || (max_events > 0 && !events)) return sfail(v, KORE_CUDA_EINVAL, "null argument");
    *n_events = 0;
    int busy = 0;
    for (const auto &S : v->s) busy += S.open && (S.generating || !S.pending.empty());
    if (busy > max_events) return sfail(v, KORE_CUDA_EINVAL, "room for %d events, %d sessions busy", max_events, busy);
    // 1. every submitted turn: kore's prefill() at the session's length
    for (int i = 0; i < v->n_seq; ++i) {
        auto &S = v->s[(size_t)i];
        if (!S.open || S.pending.empty()) continue;
        int next = -1;
        if (int rc = kore_cuda_prefill(v->ctx, i, S.pending.data(), (int)S.pending.size(), (int)S.conv.size(), &next,
                                       nullptr)) {
            S.pending.clear();
            return from_ctx(v, rc);
        }
        S.conv.insert(S.conv.end(), S.pending.begin(), S.pending.end());
        S.pending.clear();
        S.generating = true;
        v->next_host[i] = next;
    }
    // 2. one gen_step for every generating session, the steps queued back to back
    cudaStream_t st = static_cast<cudaStream_t>(kore_cuda_stream(v->ctx));
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(v->device);
    cudaError_t e = cudaMemcpyAsync(v->next_dev, v->next_host, (size_t)v->n_seq * sizeof(int), cudaMemcpyHostToDevice, st);
    int rc = e == cudaSuccess ? KORE_CUDA_OK : sfail(v, KORE_CUDA_ECUDA, "%s", cudaGetErrorString(e));
    for (int i = 0; i < v->n_seq && rc == KORE_CUDA_OK; ++i) {
        auto &S = v->s[(size_t)i];
        if (!S.open || !S.generating) continue;
        const int tok = v->next_host[i];
        kore_cuda_event &ev = events[(*n_events)++];
        ev.session = i;
        ev.token = tok;
        if (tok == v->eos || tok == v->bos) {   // kore.cpp:1746
            S.generating = false;
            ev.status = KORE_CUDA_EV_END;
            continue;
        }
        if ((int)S.conv.size() >= v->ctx_max) {   // kore.cpp:1747
            S.generating = false;
            ev.status = KORE_CUDA_EV_FULL;
            continue;
        }
        const int pos = (int)S.conv.size();
        S.conv.push_back(tok);
        S.emitted += 1;
        if (int r = kore_cuda_decode_step_dev(v->ctx, i, v->next_dev + i, pos, v->next_dev + i, nullptr)) {
            rc = from_ctx(v, r);
            break;
        }
        ev.status = S.emitted >= S.max_new ? KORE_CUDA_EV_LIMIT : KORE_CUDA_EV_TOKEN;
        if (S.emitted >= S.max_new) S.generating = false;
    }
    if (rc == KORE_CUDA_OK) {
        e = cudaMemcpyAsync(v->next_host, v->next_dev, (size_t)v->n_seq * sizeof(int), cudaMemcpyDeviceToHost, st);
        if (e != cudaSuccess) rc = sfail(v, KORE_CUDA_ECUDA, "%s", cudaGetErrorString(e));
    }
    if (prev >= 0) cudaSetDevice(prev);
    if (int r = kore_cuda_sync(v->ctx)) return rc ? rc : from_ctx(v, r);
    return rc;
}

int kore_cuda_server_condense(kore_cuda_server *v, int session, const int *ids, int n) {
    if (!v) return KORE_CUDA_EINVAL;
    if (int rc = check_session(v, session)) return rc;
    if (!ids || n <= 0 || n >= v->ctx_max) return sfail(v, KORE_CUDA_ERANGE, "history of %d tokens", n);
    auto &S = v->s[(size_t)session];
    // drop the old positions, then forward_batch from position 0 over the new
    // history (kore.cpp:1786-1797); kore leaves the session not generating
    if (int rc = kore_cuda_seq_truncate(v->ctx, session, 0)) return from_ctx(v, rc);
    int next = -1;
    if (int rc = kore_cuda_prefill(v->ctx, session, ids, n, 0, &next, nullptr)) return from_ctx(v, rc);
    S.conv.assign(ids, ids + n);
    S.pending.clear();
    S.generating = false;
    v->next_host[session] = next;
    return KORE_CUDA_OK;
}

int kore_cuda_server_history(const kore_cuda_server *v, int session, int *ids, int cap) {
    if (!v || session < 0 || session >= v->n_seq || !v->s[(size_t)session].open) return KORE_CUDA_ERANGE;
    const auto &c = v->s[(size_t)session].conv;
    for (int i = 0; i < cap && i < (int)c.size(); ++i) ids[i] = c[(size_t)i];
    return (int)c.size();
}

}  // extern "C"
