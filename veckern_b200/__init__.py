"""VecKern-B200: flat product-quantisation search (per-query L2 LUT -> ADC scan over uint8 codes -> k-smallest
selection) on NVIDIA B200 (sm_100a), bit-identical to the reference CPU path of shivdeshpande/VecKern.

The product is the native library veckern_b200/_native/libveckern_b200.so (C ABI: include/vk_abi.h; C++ API:
include/veckern/gpu.hpp). This package is the Python host side over that ABI; it has no compute of its own.
"""
from .searcher import (NEIGHBOR_DTYPE, CoopSearch, DeviceInfo, IVFSearcher, LaunchShape, MultiPQSearcher,  # noqa
                       PQSearcher, ScanVariant, assign_lists,
                       Timings, Tuning,
                       VkError, device_info, device_result_split, empty_neighbors, is_fused, merge_topk_device,
                       neighbors_split, rerank_device, variant_name)
