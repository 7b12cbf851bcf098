#pragma once
// GPU search API (no CUDA types). Declarations match shivdeshpande/VecKern's include/veckern/gpu.hpp, so the
// reference's benchmark driver and GPU tests build unchanged against this implementation
// (libveckern_b200.so). Every fused variant runs the one sm_100a fused scan + warp top-k kernel; every unfused
// variant's distances() runs the one materialising scan. Results are bit-identical to the reference CPU path.
#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "veckern/common.hpp"
#include "veckern/pq.hpp"

namespace veckern::gpu {

// The reference's kernel history v0..v8. Here a variant only selects the reference's validation rules
// (m % 16 == 0 for SharedLutVec, FusedVec, FusedVecMQ and FusedWarp; distances() only for unfused ones).
enum class ScanVariant {
    GlobalLut,
    SharedLut,
    SharedLutVec,
    Interleaved,
    Fused,
    FusedReg,
    FusedVec,
    FusedVecMQ,
    FusedWarp,
};

const char* variant_name(ScanVariant v);
bool is_fused(ScanVariant v);

// Launch-shape overrides. 0 = automatic.
struct Tuning {
    int scan_threads = 256;     // block size of the materialising scan (multiple of 32, <= 1024)
    int blocks_per_query = 0;   // vector chunks per query group of the fused scan; 0 = wave model
    int queries_per_block = 2;  // Q: queries sharing each code fetch (1, 2, 4 or 8; capped by shared memory)
    int vectors_per_step = 4;   // 32-row groups each warp holds per pipeline step (1, 2 or 4)
};

struct DeviceInfo {
    std::string name;
    int sm_count = 0;
    double peak_bandwidth_gbs = 0.0;
    std::size_t max_smem_per_block = 0;
};

DeviceInfo device_info(int device = 0);

// Milliseconds per stage, from CUDA events, summed over query batches.
struct Timings {
    double transfer_ms = 0, lut_ms = 0, scan_ms = 0, select_ms = 0;
    double kernel_ms() const { return lut_ms + scan_ms + select_ms; }
    double total_ms() const { return transfer_ms + kernel_ms(); }
};

class PQSearcher {
public:
    // Copies centroids and row-major n x m codes to the current CUDA device once.
    PQSearcher(const ProductQuantizer& pq, const uint8_t* codes, std::size_t n);
    ~PQSearcher();
    PQSearcher(const PQSearcher&) = delete;
    PQSearcher& operator=(const PQSearcher&) = delete;

    // out: nq x k neighbors, ascending (dist, id). 1 <= k <= min(128, n).
    Timings search(const float* queries, std::size_t nq, std::size_t k, ScanVariant variant, Neighbor* out);
    // out: nq x n ADC distances. Unfused variants only.
    Timings distances(const float* queries, std::size_t nq, ScanVariant variant, float* out);

    void set_tuning(const Tuning& tuning);
    const Tuning& tuning() const;
    // Shape of the last launch: threads per block, blocks_x = vector chunks per query group, grid_y = query
    // groups, Q and ILP actually used, resident blocks per SM and waves = work items / resident blocks.
    struct LaunchShape {
        int threads = 0, blocks_x = 0, grid_y = 0, queries_per_block = 1, vectors_per_step = 1;
        int blocks_per_sm = 0;
        double waves = 0.0;
    };
    LaunchShape last_launch() const;

private:
    struct Impl;
    std::unique_ptr<Impl> impl_;
};

// Additive (no counterpart in the reference): one database split into contiguous row shards over several devices
// of this process (a device may be listed more than once); search results are identical to one PQSearcher over all
// rows. Backed by vk_multi_* of include/vk_abi.h.
class MultiPQSearcher {
public:
    MultiPQSearcher(const ProductQuantizer& pq, const uint8_t* codes, std::size_t n, const std::vector<int>& devices);
    ~MultiPQSearcher();
    MultiPQSearcher(const MultiPQSearcher&) = delete;
    MultiPQSearcher& operator=(const MultiPQSearcher&) = delete;

    // out: nq x k neighbors, ascending (dist, id), global row ids. 1 <= k <= min(128, n).
    Timings search(const float* queries, std::size_t nq, std::size_t k, Neighbor* out);
    void set_tuning(const Tuning& tuning);
    std::size_t shards() const;

private:
    struct Impl;
    std::unique_ptr<Impl> impl_;
};

}  // namespace veckern::gpu
