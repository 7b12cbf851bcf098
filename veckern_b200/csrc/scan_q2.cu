// scan_kernel instantiations for Q = 2 queries per block (see scan_dispatch.cuh).
#include "scan_dispatch.cuh"

namespace vk {
VK_SCAN_TABLE(2)
}  // namespace vk
