// Instantiation table of scan_kernel<Q, MT, ILP, S, NW>. Each Q lives in its own translation unit
// (scan_q{1,2,4,8}.cu) so nvcc compiles them in parallel.
#pragma once
#include "kernels.cuh"

namespace vk {

constexpr int kScanWarps = 8;  // NW: warps per block (256 threads)

// Returns the kernel for (mt in {16, 32, 64, 0}, ilp in {1, 2, 4}, s in {1, 2, 4}); nullptr otherwise.
template <int Q>
const void* scan_kernel_for(int mt, int ilp, int s);

#define VK_SCAN_TABLE(Q)                                                                           \
    template <>                                                                                    \
    const void* scan_kernel_for<Q>(int mt, int ilp, int s) {                                       \
        switch (mt * 100 + ilp * 10 + s) {                                                         \
            VK_SCAN_CASES_MT(Q, 16)                                                                \
            VK_SCAN_CASES_MT(Q, 32)                                                                \
            VK_SCAN_CASES_MT(Q, 64)                                                                \
            VK_SCAN_CASES_MT(Q, 0)                                                                 \
            default: return nullptr;                                                               \
        }                                                                                          \
    }
#define VK_SCAN_CASE(Q, MT, ILP, S) \
    case MT * 100 + ILP * 10 + S: return reinterpret_cast<const void*>(&scan_kernel<Q, MT, ILP, S, kScanWarps>);
#define VK_SCAN_CASES_ILP(Q, MT, ILP) VK_SCAN_CASE(Q, MT, ILP, 1) VK_SCAN_CASE(Q, MT, ILP, 2) VK_SCAN_CASE(Q, MT, ILP, 4)
#define VK_SCAN_CASES_MT(Q, MT) VK_SCAN_CASES_ILP(Q, MT, 1) VK_SCAN_CASES_ILP(Q, MT, 2) VK_SCAN_CASES_ILP(Q, MT, 4)

}  // namespace vk
