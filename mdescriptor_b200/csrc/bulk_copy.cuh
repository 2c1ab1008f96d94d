// Bulk (TMA) copies from global to shared memory completed on an mbarrier,
// and a wait on that barrier with a time limit.
//
// cp.async.bulk (untiled) wants 16-byte aligned source and destination and a
// byte count that is a multiple of 16; callers guarantee both.  No multicast:
// every copy lands in the issuing CTA's own shared memory.
#pragma once

#include <cstdint>

#include <cuda_runtime.h>

namespace mdsoap {
namespace bulk {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void barrier_init(uint64_t* bar, uint32_t arrivals) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(arrivals) : "memory");
}

// Makes barrier initialisation visible to the async proxy (the copy engine).
__device__ __forceinline__ void barrier_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this CTA's earlier generic-proxy accesses to shared memory before
// later async-proxy writes (a buffer that was read is about to be refilled).
__device__ __forceinline__ void proxy_fence() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// One arrival that also announces `bytes` of transactions to come.
__device__ __forceinline__ void arrive_expect(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ bool try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits for the barrier phase with the given parity to complete; false after
// `limit_ns` nanoseconds without completion.
__device__ __forceinline__ bool wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns = 1000000000ull) {
    if (try_wait(bar, parity)) return true;
    const uint64_t start = global_ns();
    while (!try_wait(bar, parity))
        if (global_ns() - start > limit_ns) return false;
    return true;
}

}  // namespace bulk
}  // namespace mdsoap
