// scan_kernel instantiations for Q = 1 queries per block (see scan_dispatch.cuh).
#include "scan_dispatch.cuh"

namespace vk {
VK_SCAN_TABLE(1)
}  // namespace vk
