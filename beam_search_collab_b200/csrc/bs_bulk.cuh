// bs_bulk.cuh -- one-lane bulk copies global -> shared memory (cp.async.bulk,
// completion counted on a per-warp mbarrier) with bounded waits, shared by the
// neighbourhood-block search kernels.
#pragma once

#include <cstdint>

#include "bs_device.cuh"

namespace bsb {
namespace dev {

__device__ __forceinline__ unsigned smem_u32(const void* p) {
    return static_cast<unsigned>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* mbar) {
    asm volatile("mbarrier.init.shared.b64 [%0], 1;\n" ::"r"(smem_u32(mbar)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

// One lane: announce `bytes` of transaction and start the copy.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, unsigned bytes, uint64_t* mbar) {
    // the warp's earlier generic-proxy reads of dst are ordered before the
    // asynchronous write that follows
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    asm volatile("mbarrier.arrive.expect_tx.shared.b64 _, [%0], %1;\n" ::"r"(smem_u32(mbar)), "r"(bytes)
                 : "memory");
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(mbar))
        : "memory");
}

// Hint: bring `bytes` at src into L2 (no completion to wait for).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, unsigned bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* mbar, unsigned phase) {
    unsigned ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(mbar)), "r"(phase)
        : "memory");
    return ok != 0;
}

// Bounded wait: every lane polls at most `polls` times (each try_wait may
// itself suspend for a while); the warp agrees on the outcome.
__device__ __forceinline__ bool mbar_wait(uint64_t* mbar, unsigned phase, unsigned polls) {
    bool done = false;
    for (unsigned i = 0; i < polls && !done; ++i) done = mbar_try_wait(mbar, phase);
    return __all_sync(kFull, done);
}

}  // namespace dev
}  // namespace bsb
