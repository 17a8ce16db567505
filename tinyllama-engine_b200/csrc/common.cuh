// common.cuh -- sm_100a PTX helpers shared by the attention kernels:
// mbarriers with bounded waits, 1-D bulk (TMA) copies, named barriers and the
// device error word.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define TLE_DEV __device__ __forceinline__

namespace tle {

// Device error codes recorded in g_tle_error (first writer wins).
enum : uint32_t {
    kErrNone = 0,
    kErrWaitFull = 0x101,   // consumer gave up waiting for a stage to fill
    kErrWaitEmpty = 0x102,  // producer gave up waiting for a stage to drain
    kErrWaitMma = 0x103,    // waiter gave up on a tensor-core commit
    kErrDrain = 0x104,      // exit-time wait for in-flight copies gave up
    kErrBadPage = 0x105,    // paged decode: a page id outside the pool (access skipped)
    kErrBadToken = 0x106,   // forward: a token id outside the vocabulary (zero embedding used)
    kErrGridWait = 0x108,   // persistent forward: a grid barrier wait gave up
    kErrF16Range = 0x109,   // batched prompt: a finite value beyond fp16's range became inf
    kErrBadSeq = 0x10a,     // bf16 decode: a sequence record outside its cache or max_rows (skipped)
    kErrSelfTest = 0x1ff,   // tle_selftest_wait_timeout: the planted wait expired
};

// A bounded wait gives up after this long (nanoseconds of %globaltimer).
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;  // 2 s

// Records `code` in the device error word (first writer wins).
TLE_DEV void record_error(uint32_t* word, uint32_t code) {
    if (word) atomicCAS(word, 0u, code);
}

TLE_DEV uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

TLE_DEV uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

TLE_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

TLE_DEV void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

TLE_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

// Counts `bytes` of the barrier's expected transaction as done without a
// copy (for a piece the issuer decided not to copy).
TLE_DEV void mbar_tx_complete(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.complete_tx.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

TLE_DEV void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

TLE_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
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

// Non-suspending probe of a phase (never parks the warp).
TLE_DEV bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Spin wait for short, latency-critical handoffs: test_wait probes, bounded
// by %globaltimer like mbar_wait.
TLE_DEV bool mbar_wait_spin(uint64_t* bar, uint32_t parity) {
    if (mbar_test_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (;;) {
#pragma unroll 1
        for (int i = 0; i < 64; ++i)
            if (mbar_test_wait(bar, parity)) return true;
        if (globaltimer() - t0 > kWaitTimeoutNs) return false;
    }
}

// Waits for the phase with the given parity to complete; false after
// kWaitTimeoutNs (the caller records an error and unwinds).  The first probe
// is test_wait: on an already-completed phase it costs ~10 cycles where
// try_wait costs ~110 (measured on B200); try_wait, which may park the warp,
// is only used once the phase is known to be pending.
TLE_DEV bool mbar_wait_for(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
    if (mbar_test_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (;;) {
#pragma unroll 1
        for (int i = 0; i < 32; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer() - t0 > limit_ns) return false;
    }
}
TLE_DEV bool mbar_wait(uint64_t* bar, uint32_t parity) { return mbar_wait_for(bar, parity, kWaitTimeoutNs); }

// L2 policy for data read exactly once (the KV stream).
TLE_DEV uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// 1-D bulk copy global -> shared (TMA engine), completion counted on `bar`
// in bytes.  dst, src 16-byte aligned; bytes a multiple of 16.
TLE_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// 1-D bulk copy global -> shared with the default L2 policy.
TLE_DEV void bulk_g2s_plain(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Loads of data another CTA or an earlier grid wrote, issued after the
// wait (griddepcontrol.wait, an mbarrier, an acquire fence) that makes it
// visible: L2 (.cg, never a stale L1 line) and volatile with a memory
// clobber, so the compiler cannot schedule them above that wait (the
// __ldcg/__ldg intrinsics are plain inline asm without a memory operand,
// and a const __restrict__ load may be treated as invariant and hoisted).
TLE_DEV float ld_cg(const float* p) {
    float v;
    asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
    return v;
}
TLE_DEV float4 ld_cg4(const float4* p) {
    float4 v;
    asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}
TLE_DEV int32_t ld_cg_s32(const int32_t* p) {
    int32_t v;
    asm volatile("ld.global.cg.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// 4-byte asynchronous global -> shared copy (cp.async), and an arrival on
// `bar` once this thread's earlier cp.async copies have landed.  The arrive
// form without .noinc raises the barrier's pending count when it executes,
// so issue it before the arrival that could otherwise complete the phase.
TLE_DEV void cp_async_4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// Waits until every cp.async this thread issued has landed.
TLE_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
TLE_DEV void cp_async_mbar_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Named barrier over `nthreads` threads (a multiple of 32), id 1..15.
TLE_DEV void named_bar_sync(uint32_t id, uint32_t nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace tle
