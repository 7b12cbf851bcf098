#pragma once
// Product quantizer: d dimensions in m sub-spaces of dsub = d / m, 256 centroids each, one byte per sub-code.
// Declarations and data members match shivdeshpande/VecKern's include/veckern/pq.hpp (same order, so objects
// built by either implementation can be passed to either PQSearcher); set_centroids is an addition for
// databases whose codebooks are given rather than trained.
#include <cstdint>
#include <vector>

#include "veckern/common.hpp"

namespace veckern {

class ProductQuantizer {
public:
    ProductQuantizer(std::size_t d, std::size_t m);

    // k-means per sub-space on the first n rows of x (row-major n x d), seeded with 256 distinct training rows.
    void train(const float* x, std::size_t n, std::size_t iters = 20, uint64_t seed = 1);
    // codes: row-major n x m bytes (nearest centroid per sub-space).
    void encode(const float* x, std::size_t n, uint8_t* codes) const;
    void decode(const uint8_t* codes, std::size_t n, float* x) const;

    const float* centroid(std::size_t sub, std::size_t c) const {
        return centroids_.data() + (sub * kSubCentroids + c) * dsub_;
    }
    // [m][256][dsub] floats: the layout the GPU LUT builder reads.
    const std::vector<float>& centroids() const { return centroids_; }
    // Replaces the codebooks (m * 256 * dsub floats, same layout).
    void set_centroids(const float* c) { centroids_.assign(c, c + centroids_.size()); }

    std::size_t d() const { return d_; }
    std::size_t m() const { return m_; }
    std::size_t dsub() const { return dsub_; }

private:
    std::size_t d_, m_, dsub_;
    std::vector<float> centroids_;
};

}  // namespace veckern
