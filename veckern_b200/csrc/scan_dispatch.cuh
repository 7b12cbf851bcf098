// Instantiation table of scan_kernel<Q, MT, ILP, S, NW = scan_warps(Q, MT, H16), PRUNE, H16>. Each Q lives in its own
// translation unit (scan_q{1,2,4,8}.cu; half-precision LUTs: scan_h{4,8}.cu) so nvcc compiles them in parallel.
#pragma once
#include "kernels.cuh"

namespace vk {

// Returns the kernel for (mt in {16, 32, 64, 0}, ilp in {1, 2, 4}, s in {1, 2, 4}, prune); nullptr if there is
// none (the pruned scan exists for mt in {16, 32, 64} and ilp in {1, 2}).
template <int Q>
const void* scan_kernel_for(int mt, int ilp, int s, bool prune);
// Half-precision LUTs: Q in {4, 8}, mt in {16, 32, 64}, ilp in {1, 2}.
template <int Q>
const void* scan_kernel_h16_for(int mt, int ilp, int s, bool prune);
// IVF items: Q in {4, 8}, mt in {16, 32}, ilp in {1, 2}, fp32 LUTs.
template <int Q>
const void* scan_kernel_ivf_for(int mt, int ilp, int s, bool prune);
// 4-bit PQ: Q in {4, 8}, mt in {16, 32, 64}, ilp in {1, 2}, fp32 LUTs.
template <int Q>
const void* scan_kernel_p4_for(int mt, int ilp, int s, bool prune);

#define VK_SCAN_CASE(Q, MT, ILP, S, P)            \
    case (P) * 10000 + MT * 100 + ILP * 10 + S: \
        return reinterpret_cast<const void*>(&scan_kernel<Q, MT, ILP, S, scan_warps(Q, MT), P>);
#define VK_SCAN_CASES_S(Q, MT, ILP, P) VK_SCAN_CASE(Q, MT, ILP, 1, P) VK_SCAN_CASE(Q, MT, ILP, 2, P) VK_SCAN_CASE(Q, MT, ILP, 4, P)
#define VK_SCAN_CASES_MT(Q, MT) \
    VK_SCAN_CASES_S(Q, MT, 1, false) VK_SCAN_CASES_S(Q, MT, 2, false) VK_SCAN_CASES_S(Q, MT, 4, false)
#define VK_SCAN_CASES_MT_PRUNE(Q, MT) VK_SCAN_CASES_S(Q, MT, 1, true) VK_SCAN_CASES_S(Q, MT, 2, true)

#define VK_SCAN_TABLE(Q)                                                \
    template <>                                                         \
    const void* scan_kernel_for<Q>(int mt, int ilp, int s, bool prune) { \
        switch ((prune ? 10000 : 0) + mt * 100 + ilp * 10 + s) {        \
            VK_SCAN_CASES_MT(Q, 16)                                     \
            VK_SCAN_CASES_MT(Q, 32)                                     \
            VK_SCAN_CASES_MT(Q, 64)                                     \
            VK_SCAN_CASES_MT(Q, 0)                                      \
            VK_SCAN_CASES_MT_PRUNE(Q, 16)                               \
            VK_SCAN_CASES_MT_PRUNE(Q, 32)                               \
            VK_SCAN_CASES_MT_PRUNE(Q, 64)                               \
            default: return nullptr;                                    \
        }                                                               \
    }

#define VK_SCAN_CASE_H(Q, MT, ILP, S, P)          \
    case (P) * 10000 + MT * 100 + ILP * 10 + S: \
        return reinterpret_cast<const void*>(&scan_kernel<Q, MT, ILP, S, scan_warps(Q, MT, true), P, true>);
#define VK_SCAN_CASES_H_S(Q, MT, ILP, P) VK_SCAN_CASE_H(Q, MT, ILP, 1, P) VK_SCAN_CASE_H(Q, MT, ILP, 2, P) VK_SCAN_CASE_H(Q, MT, ILP, 4, P)
#define VK_SCAN_CASES_H_MT(Q, MT)                                                                          \
    VK_SCAN_CASES_H_S(Q, MT, 1, false) VK_SCAN_CASES_H_S(Q, MT, 2, false) VK_SCAN_CASES_H_S(Q, MT, 1, true) \
        VK_SCAN_CASES_H_S(Q, MT, 2, true)

#define VK_SCAN_TABLE_H(Q)                                                  \
    template <>                                                             \
    const void* scan_kernel_h16_for<Q>(int mt, int ilp, int s, bool prune) { \
        switch ((prune ? 10000 : 0) + mt * 100 + ilp * 10 + s) {            \
            VK_SCAN_CASES_H_MT(Q, 16)                                       \
            VK_SCAN_CASES_H_MT(Q, 32)                                       \
            VK_SCAN_CASES_H_MT(Q, 64)                                       \
            default: return nullptr;                                        \
        }                                                                   \
    }

#define VK_SCAN_CASE_I(Q, MT, ILP, S, P)          \
    case (P) * 10000 + MT * 100 + ILP * 10 + S: \
        return reinterpret_cast<const void*>(&scan_kernel<Q, MT, ILP, S, scan_warps(Q, MT), P, false, true>);
#define VK_SCAN_CASES_I_S(Q, MT, ILP, P) VK_SCAN_CASE_I(Q, MT, ILP, 1, P) VK_SCAN_CASE_I(Q, MT, ILP, 2, P) VK_SCAN_CASE_I(Q, MT, ILP, 4, P)
#define VK_SCAN_CASES_I_MT(Q, MT)                                                                          \
    VK_SCAN_CASES_I_S(Q, MT, 1, false) VK_SCAN_CASES_I_S(Q, MT, 2, false) VK_SCAN_CASES_I_S(Q, MT, 1, true) \
        VK_SCAN_CASES_I_S(Q, MT, 2, true)

#define VK_SCAN_TABLE_I(Q)                                                  \
    template <>                                                             \
    const void* scan_kernel_ivf_for<Q>(int mt, int ilp, int s, bool prune) { \
        switch ((prune ? 10000 : 0) + mt * 100 + ilp * 10 + s) {            \
            VK_SCAN_CASES_I_MT(Q, 16)                                       \
            VK_SCAN_CASES_I_MT(Q, 32)                                       \
            default: return nullptr;                                        \
        }                                                                   \
    }

#define VK_SCAN_CASE_P4(Q, MT, ILP, S, P)         \
    case (P) * 10000 + MT * 100 + ILP * 10 + S: \
        return reinterpret_cast<const void*>(&scan_kernel<Q, MT, ILP, S, scan_warps(Q, MT, false, true), P, false, false, true>);
#define VK_SCAN_CASES_P4_S(Q, MT, ILP, P) VK_SCAN_CASE_P4(Q, MT, ILP, 1, P) VK_SCAN_CASE_P4(Q, MT, ILP, 2, P) VK_SCAN_CASE_P4(Q, MT, ILP, 4, P)
#define VK_SCAN_CASES_P4_MT(Q, MT)                                                                            \
    VK_SCAN_CASES_P4_S(Q, MT, 1, false) VK_SCAN_CASES_P4_S(Q, MT, 2, false) VK_SCAN_CASES_P4_S(Q, MT, 1, true) \
        VK_SCAN_CASES_P4_S(Q, MT, 2, true)

#define VK_SCAN_TABLE_P4(Q)                                                 \
    template <>                                                             \
    const void* scan_kernel_p4_for<Q>(int mt, int ilp, int s, bool prune) { \
        switch ((prune ? 10000 : 0) + mt * 100 + ilp * 10 + s) {            \
            VK_SCAN_CASES_P4_MT(Q, 16)                                      \
            VK_SCAN_CASES_P4_MT(Q, 32)                                      \
            VK_SCAN_CASES_P4_MT(Q, 64)                                      \
            default: return nullptr;                                        \
        }                                                                   \
    }

}  // namespace vk
