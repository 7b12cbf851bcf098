#pragma once
// Shared types of the veckern C++ API. Declarations match shivdeshpande/VecKern's include/veckern/common.hpp so
// that code written against the reference compiles unchanged (the (dist, id) order and l2sq's arithmetic are
// what make GPU and CPU results bit-comparable).
#include <chrono>
#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>

namespace veckern {

constexpr std::size_t kSubCentroids = 256;  // centroids per sub-space: a PQ sub-code is one byte

// One search result; id -1 marks padding.
struct Neighbor {
    float dist;
    int32_t id;
};

// Strict (dist, id) order: equal distances go to the lower id.
inline bool operator<(const Neighbor& a, const Neighbor& b) {
    if (a.dist != b.dist) return a.dist < b.dist;
    return a.id < b.id;
}

inline void check(bool condition, const std::string& message) {
    if (!condition) throw std::runtime_error(message);
}

// Squared L2 distance, summed in index order from 0; each product is rounded before it is added.
inline float l2sq(const float* a, const float* b, std::size_t d) {
    float acc = 0.f;
    for (std::size_t j = 0; j < d; ++j) {
        const float diff = a[j] - b[j];
        acc += diff * diff;
    }
    return acc;
}

// Wall-clock stopwatch in milliseconds.
class Timer {
public:
    Timer() : t0_(std::chrono::steady_clock::now()) {}
    double ms() const {
        return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0_).count();
    }

private:
    std::chrono::steady_clock::time_point t0_;
};

}  // namespace veckern
