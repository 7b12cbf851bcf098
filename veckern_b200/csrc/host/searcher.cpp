// veckern::gpu::PQSearcher over the VecKern-B200 C ABI (include/vk_abi.h).
//
// Drop-in replacement for the reference's src/cuda/searcher.cu: same class, same validation and the same error
// convention (std::runtime_error from check() and from CUDA failures; src/cuda/searcher.cu:11-16, 430, 450-460,
// 468). All device work goes through the vk_* entry points; this file contains no kernels.
#include <cstddef>
#include <cuda_runtime_api.h>
#include <string>

#include "veckern/gpu.hpp"
#include "vk_abi.h"

namespace veckern::gpu {
namespace {

static_assert(sizeof(Neighbor) == sizeof(vk_neighbor_t), "Neighbor must keep the 8-byte (dist, id) layout");
static_assert(offsetof(Neighbor, id) == offsetof(vk_neighbor_t, id), "Neighbor must keep the (dist, id) layout");

[[noreturn]] void raise(int code, const char* what) {
    char msg[1024];
    vk_last_error(msg, sizeof(msg));
    throw std::runtime_error(std::string(what) + " failed (" + std::to_string(code) + "): " + msg);
}

void ok(int code, const char* what) {
    if (code != VK_OK) raise(code, what);
}

vk_tuning_t to_c(const Tuning& t) {
    return vk_tuning_t{t.scan_threads, t.blocks_per_query, t.queries_per_block, t.vectors_per_step, 1, VK_LUT_F32};
}

}  // namespace

const char* variant_name(ScanVariant v) {
    switch (v) {
        case ScanVariant::GlobalLut: return "v0_global_lut";
        case ScanVariant::SharedLut: return "v1_shared_lut";
        case ScanVariant::SharedLutVec: return "v2_shared_lut_vec";
        case ScanVariant::Interleaved: return "v3_interleaved";
        case ScanVariant::Fused: return "v4_fused";
        case ScanVariant::FusedReg: return "v5_fused_reg";
        case ScanVariant::FusedVec: return "v6_fused_vec";
        case ScanVariant::FusedVecMQ: return "v7_fused_vec_mq";
        case ScanVariant::FusedWarp: return "v8_fused_warp";
    }
    return "unknown";
}

bool is_fused(ScanVariant v) {
    const int i = static_cast<int>(v);
    return i >= static_cast<int>(ScanVariant::Fused) && i <= static_cast<int>(ScanVariant::FusedWarp);
}

DeviceInfo device_info(int device) {
    vk_device_info_t c{};
    ok(vk_device_info(device, &c), "vk_device_info");
    DeviceInfo info;
    info.name = c.name;
    info.sm_count = c.sm_count;
    info.peak_bandwidth_gbs = c.peak_bandwidth_gbs;
    info.max_smem_per_block = c.max_smem_per_block;
    return info;
}

struct PQSearcher::Impl {
    vk_index_t* index = nullptr;
    std::size_t n = 0;
    Tuning tuning;
    LaunchShape last;
    ~Impl() {
        if (index) vk_index_destroy(index);
    }
};

PQSearcher::PQSearcher(const ProductQuantizer& pq, const uint8_t* codes, std::size_t n)
    : impl_(std::make_unique<Impl>()) {
    check(n > 0 && n < static_cast<std::size_t>(2147483647), "n must fit in int32 ids");
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) device = 0;
    impl_->n = n;
    ok(vk_index_create(device, pq.centroids().data(), static_cast<int>(pq.m()), static_cast<int>(pq.dsub()), codes,
                       static_cast<int64_t>(n), 0, &impl_->index),
       "vk_index_create");
}

PQSearcher::~PQSearcher() = default;

void PQSearcher::set_tuning(const Tuning& t) {
    const vk_tuning_t c = to_c(t);
    ok(vk_tuning_validate(&c), "set_tuning");
    impl_->tuning = t;
}

const Tuning& PQSearcher::tuning() const { return impl_->tuning; }

PQSearcher::LaunchShape PQSearcher::last_launch() const { return impl_->last; }

Timings PQSearcher::search(const float* queries, std::size_t nq, std::size_t k, ScanVariant v, Neighbor* out) {
    check(k >= 1 && k <= 128 && k <= impl_->n, "k must be in [1, min(128, n)]");
    const vk_tuning_t c = to_c(impl_->tuning);
    vk_timings_t t{};
    vk_launch_shape_t s{};
    ok(vk_search(impl_->index, queries, static_cast<int64_t>(nq), static_cast<int>(k), static_cast<int>(v), &c,
                 reinterpret_cast<vk_neighbor_t*>(out), &t, &s),
       "search");
    if (nq > 0) impl_->last = LaunchShape{s.threads, s.blocks_x, s.grid_y, s.queries_per_block, s.vectors_per_step,
                                          s.blocks_per_sm, s.waves};
    return Timings{t.transfer_ms, t.lut_ms, t.scan_ms, t.select_ms};
}

Timings PQSearcher::distances(const float* queries, std::size_t nq, ScanVariant v, float* out) {
    check(!is_fused(v), "fused variants do not materialise distances");
    const vk_tuning_t c = to_c(impl_->tuning);
    vk_timings_t t{};
    ok(vk_distances(impl_->index, queries, static_cast<int64_t>(nq), static_cast<int>(v), &c, out, &t), "distances");
    impl_->last = LaunchShape{c.scan_threads, 0, static_cast<int>(nq), 1, 1, 0, 0.0};
    return Timings{t.transfer_ms, t.lut_ms, t.scan_ms, t.select_ms};
}

struct MultiPQSearcher::Impl {
    vk_multi_t* multi = nullptr;
    std::size_t n = 0, shards = 0;
    Tuning tuning;
    ~Impl() {
        if (multi) vk_multi_destroy(multi);
    }
};

MultiPQSearcher::MultiPQSearcher(const ProductQuantizer& pq, const uint8_t* codes, std::size_t n,
                                 const std::vector<int>& devices)
    : impl_(std::make_unique<Impl>()) {
    check(n > 0 && n < static_cast<std::size_t>(2147483647), "n must fit in int32 ids");
    check(!devices.empty(), "need at least one device");
    impl_->n = n;
    impl_->shards = devices.size();
    ok(vk_multi_create(static_cast<int>(devices.size()), devices.data(), pq.centroids().data(),
                       static_cast<int>(pq.m()), static_cast<int>(pq.dsub()), codes, static_cast<int64_t>(n),
                       &impl_->multi),
       "vk_multi_create");
}

MultiPQSearcher::~MultiPQSearcher() = default;

void MultiPQSearcher::set_tuning(const Tuning& t) {
    const vk_tuning_t c = to_c(t);
    ok(vk_tuning_validate(&c), "set_tuning");
    impl_->tuning = t;
}

std::size_t MultiPQSearcher::shards() const { return impl_->shards; }

Timings MultiPQSearcher::search(const float* queries, std::size_t nq, std::size_t k, Neighbor* out) {
    check(k >= 1 && k <= 128 && k <= impl_->n, "k must be in [1, min(128, n)]");
    const vk_tuning_t c = to_c(impl_->tuning);
    vk_timings_t t{};
    ok(vk_multi_search(impl_->multi, queries, static_cast<int64_t>(nq), static_cast<int>(k), &c,
                       reinterpret_cast<vk_neighbor_t*>(out), &t),
       "multi search");
    return Timings{t.transfer_ms, t.lut_ms, t.scan_ms, t.select_ms};
}

}  // namespace veckern::gpu
