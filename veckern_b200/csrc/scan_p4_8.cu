// scan_kernel instantiations for 4-bit PQ codes with Q = 8 queries per block (see scan_dispatch.cuh).
#include "scan_dispatch.cuh"

namespace vk {
VK_SCAN_TABLE_P4(8)
}  // namespace vk
