// Device-side primitives shared by the VecKern-B200 kernels: shared-memory mbarriers, TMA bulk copies
// (cp.async.bulk, no multicast) and bounded waits.
//
// Every wait in these kernels is bounded by a clock64() budget. A wait that runs out sets a bit in the kernel's
// status word and the kernel unwinds instead of spinning forever; the host reports VK_ERR_DEVICE.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "vk_gen.h"

namespace vk {

constexpr int KSUB = 256;  // centroids per sub-space: one byte per sub-code
constexpr int WARP = 32;
constexpr unsigned FULL = 0xffffffffu;
constexpr int32_t SENTINEL_ID = 0x7fffffff;  // empty list slot: loses to every real (dist, id) pair

// Status-word bits written by kernels (atomicOr). ERR_DRAIN_TIMEOUT: after a wait ran out, the block also failed to
// see its own bulk copies land within a second, longer budget before exiting; such a copy may still write the
// block's shared memory, so the host treats the context as suspect.
enum : int { ERR_WAIT_TIMEOUT = 1, ERR_LAYOUT = 2, ERR_DRAIN_TIMEOUT = 4 };

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Makes mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses before later async-proxy ones.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
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

// Waits for the phase with the given parity to complete; false if `budget` SM cycles pass first.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, long long budget) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > budget) return false;
    return true;
}

// TMA bulk copy global -> this CTA's shared memory, completing `bytes` of transaction count on `bar`.
// dst and src 16-byte aligned, bytes a multiple of 16. No multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// (dist, id) strict order of the reference (include/veckern/common.hpp:19-21).
__device__ __forceinline__ bool nb_less(float da, int32_t ia, float db, int32_t ib) {
    return da < db || (da == db && ia < ib);
}

}  // namespace vk
