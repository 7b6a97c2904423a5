// mbarrier + 1-D bulk-copy (TMA) helpers for sm_100a, with bounded waits.
#pragma once

#include <stdint.h>

namespace fl {

// Device-wide error word: set when a bounded wait gives up (the kernel then
// stops issuing work, drains its own copies and exits). Read by the host
// after a synchronisation (fl_cuda_sync / engine calls report FL_E_TIMEOUT).
// Only gemv_tma.cu includes this header; it also reads the word back.
static __device__ int g_fl_error = 0;
constexpr int kErrMbarTimeout = 1;
constexpr long long kWaitLimit = 1ll << 24;  // try_wait rounds (each can sleep a while)

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// FL_MBAR_SUSPEND_NS > 0: try_wait carries that suspend-time hint (a waiting
// thread sleeps until the phase completes or the hint expires).
#ifndef FL_MBAR_SUSPEND_NS
#define FL_MBAR_SUSPEND_NS 0
#endif
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
#if FL_MBAR_SUSPEND_NS > 0
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"((uint32_t)FL_MBAR_SUSPEND_NS)
        : "memory");
#else
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
#endif
    return ok != 0;
}

// Bounded wait on a phase of an mbarrier. Returns false (and raises the
// device error word) when the limit is reached.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    for (long long i = 0; i < kWaitLimit; i++)
        if (mbar_try_wait(bar, parity)) return true;
    atomicOr(&g_fl_error, kErrMbarTimeout);
    return false;
}

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes).
// dst, src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

}  // namespace fl
