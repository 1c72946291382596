// bnn_sync.cuh - mbarrier and bulk-copy (TMA 1D) helpers with bounded waits.
//
// Every wait here gives up after a bounded time (and a bounded number of
// polls) and reports it, so a logic error can never leave a GPU spinning
// forever: the caller sets an error bit that the host maps to BNN_ETIMEOUT.
#pragma once

#include <cstdint>

namespace bnn {

constexpr int kStatusTimeout = 2;
// A healthy wait completes in microseconds; a wait gives up after one second
// of device time (or this many polls, whichever comes first).
constexpr uint32_t kWaitPollLimit = 1u << 26;
constexpr uint64_t kWaitNsLimit = 1000000000ull;
// Suspend-time hint of a blocking poll: a waiting warp sleeps until the phase
// completes (or this many ns pass) instead of re-issuing the poll, so waiting
// producer/consumer warps leave the issue slots to the warps doing the work.
constexpr uint32_t kSuspendHintNs = 20000u;

// The limit a wait applies, in ns. Each translation unit holds its own copy,
// kWaitNsLimit unless a test lowers the copy that BNN_Execute's kernels read
// (bnn_b200_test_wait_limit) to make a wait run out within milliseconds.
static __device__ unsigned long long g_wait_ns_limit = kWaitNsLimit;

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(kSuspendHintNs)
        : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity))
        return true;
    const uint64_t t0 = globaltimer_ns();
    const uint64_t limit = *reinterpret_cast<volatile unsigned long long*>(&g_wait_ns_limit);
    for (uint32_t i = 0; i < kWaitPollLimit; ++i) {
        if (mbar_try_wait_suspend(bar, parity))
            return true;
        if (globaltimer_ns() - t0 > limit)
            return false;
    }
    return false;
}

// Named barrier over `threads` threads (a multiple of 32); id 0 is __syncthreads.
__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// 1D bulk copy global -> shared, completion signalled on `bar` as tx bytes.
// src, dst 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

}  // namespace bnn
