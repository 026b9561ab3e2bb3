// common.cuh — device helpers shared by the attention kernels (sm_100a).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace kore {

// Error codes a kernel can leave in the context's device error word. The
// first failure wins (atomicCAS from 0); the host reads and clears it.
enum DeviceError : int {
    DEV_OK = 0,
    DEV_WAIT_FULL_TIMEOUT = 1,    // consumer waited too long for a tile copy
    DEV_WAIT_EMPTY_TIMEOUT = 2,   // producer waited too long for a free stage
    DEV_BAD_PAGE = 3,             // page table entry outside the pool
    DEV_PEER_TIMEOUT = 4,         // a peer GPU's partial did not arrive in time
    DEV_BAD_TOKEN = 5,            // token id outside the vocabulary (device-side token)
};

__device__ __forceinline__ void raise_error(int *err, int code) {
    if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Makes initialised barriers visible to the async (bulk copy) proxy.
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

#ifdef KORE_TRACE
// Trace build only (kore_b200/build.py --trace): thread 0 of a CTA claims a
// record and stamps %globaltimer at fixed points of its kernel (TraceRec::t).
// Each translation unit that stamps holds its own buffer (KORE_TRACE_BUFFER,
// inside its anonymous namespace); kore_trace_read returns them all.
struct TraceRec {
    unsigned long long t[5];   // five stamps, entry first; their meaning is the kind's
    unsigned blk, sm, kind, tag;   // tag, pad2: the launch's shape (products), else 0
    unsigned long long pad2;
};
constexpr unsigned kTraceRecs = 1u << 16;
__device__ __forceinline__ unsigned trace_open_in(TraceRec *buf, unsigned *n, unsigned kind, unsigned tag,
                                                  unsigned long long tag2) {
    if (threadIdx.x != 0) return kTraceRecs;
    const unsigned slot = atomicAdd(n, 1u);
    if (slot < kTraceRecs) {
        unsigned sm;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
        buf[slot].t[0] = global_ns();
        buf[slot].blk = blockIdx.x | (blockIdx.y << 16);
        buf[slot].sm = sm;
        buf[slot].kind = kind;
        buf[slot].tag = tag;
        buf[slot].pad2 = tag2;
    }
    return slot;
}
__device__ __forceinline__ void trace_stamp_in(TraceRec *buf, unsigned slot, int i) {
    if (slot < kTraceRecs) buf[slot].t[i] = global_ns();
}
#define KORE_TRACE_BUFFER() \
    __device__ TraceRec g_trace[kTraceRecs]; \
    __device__ unsigned g_trace_n
#define KTRACE_OPEN(kind) const unsigned tr_slot_ = trace_open_in(g_trace, &g_trace_n, kind, 0u, 0ull)
#define KTRACE_OPEN_TAGGED(kind, tag, tag2) const unsigned tr_slot_ = trace_open_in(g_trace, &g_trace_n, kind, tag, tag2)
#define KTRACE(i) trace_stamp_in(g_trace, tr_slot_, i)
#else
#define KTRACE_OPEN(kind)
#define KTRACE_OPEN_TAGGED(kind, tag, tag2)
#define KTRACE(i)
#endif

// Bounded wait on a phase of an mbarrier: gives up after `limit_ns` of wall
// time (checked every 8 polls) or kWaitPolls polls, whichever comes first,
// records `code` in the error word and returns false. A healthy pipeline waits
// microseconds; the bound only turns a lost copy into an error the host sees.
// kWaitNs is the default limit (a context can set another one for the decode
// and exchange kernels); kDrainNs bounds the wait a kernel that gave up makes
// for its own copies still in flight before it exits.
constexpr uint64_t kWaitNs = 2000000000ull;    // 2 s
constexpr uint64_t kDrainNs = 2000000000ull;   // 2 s
constexpr uint32_t kWaitPolls = 1u << 26;

__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err, int code,
                                          uint64_t limit_ns = kWaitNs) {
    // a try_wait may suspend until the phase completes: under a limit shorter
    // than the default even the first one is timed
    const bool timed_first = limit_ns < kWaitNs;
    const uint64_t t_first = timed_first ? global_ns() : 0;
    if (mbar_try_wait(bar, parity)) {
        if (!timed_first || global_ns() - t_first <= limit_ns) return true;
        raise_error(err, code);
        return false;
    }
    const uint64_t t0 = timed_first ? t_first : global_ns();
    for (uint32_t it = 1; it < kWaitPolls; ++it) {
        // a try_wait may itself suspend until the phase completes: a wait that
        // ends after its limit counts as expired even if the copy landed
        if (mbar_try_wait(bar, parity)) {
            if (global_ns() - t0 <= limit_ns) return true;
            break;
        }
        if ((it & 7) == 0 && global_ns() - t0 > limit_ns) break;
    }
    raise_error(err, code);
    return false;
}

// Waits, bounded by kDrainNs and without recording an error, for a phase of
// an mbarrier whose bulk copy is in flight: a kernel that gave up calls this
// for every copy it issued and never consumed, so that no copy lands in the
// shared memory of a block that has exited. Returns false if even this wait
// expired (the error word already holds the first failure).
__device__ __forceinline__ bool mbar_drain(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t it = 1; it < kWaitPolls; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63) == 0 && global_ns() - t0 > kDrainNs) break;
    }
    return false;
}

// ---------------------------------------------------------------- bulk copy

// Orders this thread's earlier generic-proxy accesses of shared memory before
// later async-proxy (bulk copy) accesses: a stage that was just read is only
// then refilled.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Creates an L2 policy that marks lines as first to evict: streamed K/V are
// read exactly once per launch.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// One-dimensional bulk copy global -> this CTA's shared memory, completing on
// `bar` with a transaction count of `bytes`. Both addresses 16-byte aligned,
// bytes a multiple of 16. This is the plain (non-multicast) form.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// ---------------------------------------------------------------- dependent launch

// Programmatic dependent launch: wait until the preceding kernel in the stream
// has completed and its writes are visible (a no-op when this launch has no
// programmatic dependency), and allow the next kernel to be scheduled.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// The same copy without a cache hint (data that other CTAs will read again).
__device__ __forceinline__ void bulk_g2s_plain(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// Asks L2 to fetch [src, src + bytes) from HBM, with no destination and no
// completion to wait for (16-byte aligned address, size a multiple of 16).
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------- math

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// NEOX rotation of one element, rounded exactly as kore's rope_neox
// (kore.cpp:1379-1381): two products and their difference (or sum), each
// rounded on its own, never fused.
__device__ __forceinline__ float rope_lo(float x0, float x1, float c, float s) {
    return __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
}
__device__ __forceinline__ float rope_hi(float x0, float x1, float c, float s) {
    return __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
}

}  // namespace kore
