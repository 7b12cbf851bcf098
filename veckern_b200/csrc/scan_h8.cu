// scan_kernel instantiations with half-precision LUTs for Q = 8 queries per block (see scan_dispatch.cuh).
#include "scan_dispatch.cuh"

namespace vk {
VK_SCAN_TABLE_H(8)
}  // namespace vk
