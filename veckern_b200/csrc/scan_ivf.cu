// scan_kernel instantiations for IVF work items, Q = 4 and 8 queries per item (see scan_dispatch.cuh).
#include "scan_dispatch.cuh"

namespace vk {
VK_SCAN_TABLE_I(4)
VK_SCAN_TABLE_I(8)
}  // namespace vk
