// Counter-based synthetic code generator shared by host (C++) and device (CUDA) code: the same integer
// expression on both sides, so a database generated on the GPU can be re-generated row by row on the host.
//
//   key      = mix64(seed)
//   h        = mix64(key + row)                      per row
//   cluster  = (hi32(h) * clusters) >> 32            uniform over [0, clusters)
//   u        = hi32(mix64(h + (s + 1) * GOLDEN))     per (row, sub-space)
//   code     = #{c < 255 : cdf[cluster][s][c] <= u}  inverse of the cluster's categorical CDF (uint32 scale)
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define VK_HD __host__ __device__ __forceinline__
#else
#define VK_HD inline
#endif

namespace vk {

// SplitMix64 finaliser.
VK_HD uint64_t mix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

VK_HD uint32_t gen_code(uint64_t key, uint64_t row, int s, const uint32_t* cdf, int clusters, int m) {
    const uint64_t h = mix64(key + row);
    const uint32_t cl = (uint32_t)(((h >> 32) * (uint64_t)clusters) >> 32);
    const uint32_t u = (uint32_t)(mix64(h + (uint64_t)(s + 1) * 0x9E3779B97F4A7C15ull) >> 32);
    const uint32_t* t = cdf + ((uint64_t)cl * (uint64_t)m + (uint64_t)s) * 256u;
    uint32_t pos = 0;
    for (uint32_t step = 128; step; step >>= 1)
        if (pos + step <= 255 && t[pos + step - 1] <= u) pos += step;
    return pos;
}

}  // namespace vk
