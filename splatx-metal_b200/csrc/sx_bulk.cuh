// sx_bulk.cuh — the sm_100a bulk-copy engine (TMA, untiled form) and mbarrier helpers.
//
// Loads: cp.async.bulk global -> shared, completion counted in bytes on an mbarrier.
// Stores: cp.async.bulk shared -> global in a bulk group, waited on before the CTA retires.
// Every wait is bounded: a wait that runs out sets a bit in a device status word the host reads,
// so a stuck copy becomes an error report instead of a hung GPU.
// Addresses and sizes given to the copies are 16-byte aligned multiples of 16 bytes.
#pragma once

#include <cstdint>

namespace sx {

constexpr uint32_t kStatusBulkWaitTimeout = 1u;  // a bounded mbarrier wait gave up
constexpr int kBulkSpinLimit = 1 << 20;          // try_wait rounds before giving up

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
    // make the initialised barrier visible to the async (bulk-copy) proxy
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    uint64_t state;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 %0, [%1], %2;"
                 : "=l"(state)
                 : "r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
    (void)state;
}

// Bounded wait on the given phase parity; returns false when the limit ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_addr(bar);
    for (int it = 0; it < kBulkSpinLimit; ++it) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

// global -> shared, `bytes` (multiple of 16) accounted on `bar`.
__device__ __forceinline__ void bulk_load(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                          uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_addr(dst_smem)), "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// shared -> global in the current bulk group.
__device__ __forceinline__ void bulk_store(void* dst_gmem, const void* src_smem, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
                 ::"l"(dst_gmem), "r"(smem_addr(src_smem)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void bulk_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Waits until every committed bulk store of this thread has completed (hardware wait).
__device__ __forceinline__ void bulk_wait_all() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Orders this thread's generic-proxy shared-memory writes before later bulk-copy reads of them.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

}  // namespace sx
