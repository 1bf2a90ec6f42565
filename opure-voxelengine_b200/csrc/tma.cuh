// tma.cuh -- bulk (non-tensor) TMA copies global -> shared completing on an mbarrier,
// and a time-bounded mbarrier wait. No multicast: every copy targets this CTA only.
#pragma once

#include "common.cuh"

namespace opure {

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

// dst and src 16-byte aligned, bytes a multiple of 16; the mbarrier's transaction count
// is limited to 2^20 - 1 bytes per phase. Used for weights, which are read once per step:
// the copy is marked evict-first in L2.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(l2_evict_first())
        : "memory");
}

// bulk_load with the default L2 policy, for data that is read again later (KV rows).
__device__ __forceinline__ void bulk_load_keep(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(phase)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Waits for `phase` of the mbarrier for at most `limit_ns` (default 1 s). Returns false
// when the limit is reached; the caller then reports OPURE_ERR_DEVICE_TIMEOUT.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t phase, uint64_t limit_ns = 1000000000ull) {
    if (mbar_try_wait(bar, phase)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, phase)) return true;
        if ((i & 63u) == 0 && global_ns() - t0 > limit_ns) return false;
    }
}

// Whole-CTA wait on a weight copy. On timeout every thread learns it (the kernel must then
// skip its compute); thread 0 records the failure and waits once more, also bounded, so
// the copy is not left in flight into shared memory when the CTA exits.
__device__ __forceinline__ bool cta_wait_copy(uint64_t *bar, DeviceStatus *st, uint32_t where) {
    __shared__ int failed;
    if (threadIdx.x == 0) {
        failed = 0;
        if (!mbar_wait(bar, 0)) {
            failed = 1;
            report(st, OPURE_ERR_DEVICE_TIMEOUT, where, blockIdx.x);
            mbar_wait(bar, 0);
        }
    }
    __syncthreads();
    const bool ok = !failed;
    if (ok) {
        // Every thread observes the completed phase before reading the copied bytes.
        mbar_wait(bar, 0);
    }
    return ok;
}

}  // namespace opure
