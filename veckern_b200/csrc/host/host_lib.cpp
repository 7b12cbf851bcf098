// VecKern-B200 host library: product quantizer and synthetic data generators (include/vk_host.h) and the
// veckern::ProductQuantizer class (include/veckern/pq.hpp).
//
// ProductQuantizer follows the steps of the reference's src/cpu/pq.cpp:31-81 exactly: the same RNG
// (std::mt19937_64(seed)), the same draws in the same order (one std::shuffle of 0..n-1 per sub-space, one rng()
// per empty cluster), the same float sums and divisions. That is what makes the benchmark configurations'
// codebooks ("256 database sub-vectors picked with seed 1", "10 Lloyd iterations") the reference's codebooks.
// Built with -ffp-contract=off: l2sq must not be contracted to FMA.
#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <numeric>
#include <random>
#include <vector>

#include "../vk_gen.h"
#include "index_file.h"
#include "veckern/pq.hpp"
#include "vk_host.h"

namespace {

using veckern::kSubCentroids;

inline float l2(const float* a, const float* b, int d) {
    float acc = 0.f;
    for (int j = 0; j < d; ++j) {
        const float diff = a[j] - b[j];
        const float sq = diff * diff;
        acc = acc + sq;
    }
    return acc;
}

// First centroid (of ksub) with the strictly smallest distance (src/cpu/pq.cpp:11-22).
inline int nearest(const float* x, const float* cents, int dsub, int ksub = (int)kSubCentroids) {
    int best = 0;
    float best_d = FLT_MAX;
    for (int c = 0; c < ksub; ++c) {
        const float dist = l2(x, cents + (size_t)c * dsub, dsub);
        if (dist < best_d) {
            best_d = dist;
            best = c;
        }
    }
    return best;
}

// ksub = 256: the reference's trainer step for step. ksub = 16 (4-bit PQ, no counterpart in the reference): the same
// steps with 16 centroids per sub-space.
void train_impl(const float* x, size_t n, size_t d, size_t m, size_t iters, uint64_t seed, float* centroids,
                size_t ksub = kSubCentroids) {
    const size_t dsub = d / m;
    std::mt19937_64 rng(seed);
    std::vector<float> sub(n * dsub), sums(ksub * dsub);
    std::vector<size_t> perm(n), assign(n), counts(ksub);
    for (size_t s = 0; s < m; ++s) {
        for (size_t i = 0; i < n; ++i) std::memcpy(&sub[i * dsub], x + i * d + s * dsub, dsub * sizeof(float));
        float* cent = centroids + s * ksub * dsub;
        std::iota(perm.begin(), perm.end(), size_t(0));
        std::shuffle(perm.begin(), perm.end(), rng);
        for (size_t c = 0; c < ksub; ++c)
            std::memcpy(cent + c * dsub, &sub[perm[c] * dsub], dsub * sizeof(float));
        for (size_t it = 0; it < iters; ++it) {
#pragma omp parallel for schedule(static)
            for (long long i = 0; i < (long long)n; ++i)
                assign[i] = (size_t)nearest(&sub[i * dsub], cent, (int)dsub, (int)ksub);
            std::fill(sums.begin(), sums.end(), 0.f);
            std::fill(counts.begin(), counts.end(), size_t(0));
            for (size_t i = 0; i < n; ++i) {
                const size_t a = assign[i];
                ++counts[a];
                for (size_t j = 0; j < dsub; ++j) sums[a * dsub + j] += sub[i * dsub + j];
            }
            for (size_t c = 0; c < ksub; ++c) {
                if (counts[c] == 0) {  // an empty cluster takes a random training row
                    std::memcpy(cent + c * dsub, &sub[(rng() % n) * dsub], dsub * sizeof(float));
                    continue;
                }
                for (size_t j = 0; j < dsub; ++j) cent[c * dsub + j] = sums[c * dsub + j] / (float)counts[c];
            }
        }
    }
}

void encode_impl(const float* centroids, size_t d, size_t m, const float* x, size_t n, uint8_t* codes) {
    const size_t dsub = d / m;
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; ++i)
        for (size_t s = 0; s < m; ++s)
            codes[(size_t)i * m + s] =
                (uint8_t)nearest(x + (size_t)i * d + s * dsub, centroids + s * kSubCentroids * dsub, (int)dsub);
}

// 4-bit codes: nearest of 16 centroids per sub-space, sub-code s in nibble s % 2 (low first) of byte s / 2.
void encode4_impl(const float* centroids, size_t d, size_t m, const float* x, size_t n, uint8_t* codes) {
    const size_t dsub = d / m, mb = (m + 1) / 2;
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; ++i) {
        uint8_t* row = codes + (size_t)i * mb;
        std::memset(row, 0, mb);
        for (size_t s = 0; s < m; ++s) {
            const int c = nearest(x + (size_t)i * d + s * dsub, centroids + s * 16 * dsub, (int)dsub, 16);
            row[s / 2] |= (uint8_t)(c << (4 * (s % 2)));
        }
    }
}

void decode_impl(const float* centroids, size_t d, size_t m, const uint8_t* codes, size_t n, float* x) {
    const size_t dsub = d / m;
    for (size_t i = 0; i < n; ++i)
        for (size_t s = 0; s < m; ++s)
            std::memcpy(x + i * d + s * dsub, centroids + (s * kSubCentroids + codes[i * m + s]) * dsub,
                        dsub * sizeof(float));
}

// ---------------------------------------------------------------- counter-based draws
constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;

inline double unit_open(uint64_t h) { return ((double)(h >> 11) + 0.5) * (1.0 / 9007199254740992.0); }  // (0,1)
inline double unit_closed0(uint64_t h) { return (double)(h >> 11) * (1.0 / 9007199254740992.0); }       // [0,1)

inline double normal_at(uint64_t key, uint64_t idx) {
    const double u1 = unit_open(vk::mix64(key + 2 * idx));
    const double u2 = unit_closed0(vk::mix64(key + 2 * idx + 1));
    return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
}

// Sequential stream for rejection samplers: value i of stream `key`.
struct Stream {
    uint64_t key, i = 0;
    uint64_t next() { return vk::mix64(key + kGolden * ++i); }
    double uniform() { return unit_open(next()); }
    double normal() {
        const double u1 = unit_open(next()), u2 = unit_closed0(next());
        return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
    }
};

// Marsaglia-Tsang gamma sampler; shape < 1 via Gamma(a + 1) * U^(1/a).
double gamma_draw(Stream& st, double a) {
    if (a < 1.0) {
        const double g = gamma_draw(st, a + 1.0);
        return g * std::pow(st.uniform(), 1.0 / a);
    }
    const double dd = a - 1.0 / 3.0, c = 1.0 / std::sqrt(9.0 * dd);
    for (;;) {
        double x, v;
        do {
            x = st.normal();
            v = 1.0 + c * x;
        } while (v <= 0.0);
        v = v * v * v;
        const double u = st.uniform();
        if (std::log(u) < 0.5 * x * x + dd - dd * v + dd * std::log(v)) return dd * v;
    }
}

}  // namespace

// ------------------------------------------------------------------------------------------------ C++ class
namespace veckern {

ProductQuantizer::ProductQuantizer(std::size_t d, std::size_t m) : d_(d), m_(m), dsub_(m ? d / m : 0) {
    check(m > 0 && d > 0 && d % m == 0, "d must be a positive multiple of m");
    centroids_.assign(m_ * kSubCentroids * dsub_, 0.f);
}

void ProductQuantizer::train(const float* x, std::size_t n, std::size_t iters, uint64_t seed) {
    check(n >= kSubCentroids, "PQ training needs at least 256 vectors");
    train_impl(x, n, d_, m_, iters, seed, centroids_.data());
}

void ProductQuantizer::encode(const float* x, std::size_t n, uint8_t* codes) const {
    encode_impl(centroids_.data(), d_, m_, x, n, codes);
}

void ProductQuantizer::decode(const uint8_t* codes, std::size_t n, float* x) const {
    decode_impl(centroids_.data(), d_, m_, codes, n, x);
}

}  // namespace veckern

// ------------------------------------------------------------------------------------------------ C ABI
extern "C" {

int vk_host_pq_train(const float* x, int64_t n, int d, int m, int64_t iters, uint64_t seed, float* centroids) {
    if (!x || !centroids || m <= 0 || d <= 0 || d % m != 0 || n < (int64_t)kSubCentroids || iters < 0) return -1;
    train_impl(x, (size_t)n, (size_t)d, (size_t)m, (size_t)iters, seed, centroids);
    return 0;
}

int vk_host_pq_encode(const float* centroids, int d, int m, const float* x, int64_t n, uint8_t* codes) {
    if (!centroids || !x || !codes || m <= 0 || d <= 0 || d % m != 0 || n < 0) return -1;
    encode_impl(centroids, (size_t)d, (size_t)m, x, (size_t)n, codes);
    return 0;
}

int vk_host_pq4_train(const float* x, int64_t n, int d, int m, int64_t iters, uint64_t seed, float* centroids) {
    if (!x || !centroids || m <= 0 || d <= 0 || d % m != 0 || n < 16 || iters < 0) return -1;
    train_impl(x, (size_t)n, (size_t)d, (size_t)m, (size_t)iters, seed, centroids, 16);
    return 0;
}

int vk_host_pq4_encode(const float* centroids, int d, int m, const float* x, int64_t n, uint8_t* codes) {
    if (!centroids || !x || !codes || m <= 0 || d <= 0 || d % m != 0 || n < 0) return -1;
    encode4_impl(centroids, (size_t)d, (size_t)m, x, (size_t)n, codes);
    return 0;
}

int vk_host_pq_decode(const float* centroids, int d, int m, const uint8_t* codes, int64_t n, float* x) {
    if (!centroids || !x || !codes || m <= 0 || d <= 0 || d % m != 0 || n < 0) return -1;
    decode_impl(centroids, (size_t)d, (size_t)m, codes, (size_t)n, x);
    return 0;
}

// The reference's synthetic_clustered (src/cpu/io.cpp:54-69): same engine, distributions and draw order.
int vk_host_synthetic_clustered(int64_t n, int d, int64_t clusters, uint64_t seed, float* out) {
    if (n < 0 || d <= 0 || clusters <= 0 || !out) return -1;
    std::mt19937_64 rng(seed);
    std::uniform_real_distribution<float> center_dist(-1.f, 1.f);
    std::normal_distribution<float> noise(0.f, 0.15f);
    std::uniform_int_distribution<std::size_t> pick(0, (std::size_t)clusters - 1);
    std::vector<float> centers((size_t)clusters * d);
    for (auto& v : centers) v = center_dist(rng);
    for (int64_t i = 0; i < n; ++i) {
        const float* c = centers.data() + pick(rng) * (size_t)d;
        for (int j = 0; j < d; ++j) out[i * d + j] = c[j] + noise(rng);
    }
    return 0;
}

int vk_host_gen_normal(uint64_t seed, int64_t row0, int64_t rows, int d, float* out) {
    if (row0 < 0 || rows < 0 || d <= 0 || !out) return -1;
    const uint64_t key = vk::mix64(seed ^ 0x4e4f524d414c5321ull);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r)
        for (int j = 0; j < d; ++j)
            out[r * d + j] = (float)normal_at(key, (uint64_t)(row0 + r) * (uint64_t)d + (uint64_t)j);
    return 0;
}

int vk_host_gen_mixture(uint64_t mix_seed, int ncomp, float sigma, uint64_t sample_seed, int64_t row0, int64_t rows,
                        int d, float* out) {
    if (ncomp <= 0 || row0 < 0 || rows < 0 || d <= 0 || !out) return -1;
    const uint64_t kmean = vk::mix64(mix_seed ^ 0x4d49585f4d45414eull);
    const uint64_t kpick = vk::mix64(sample_seed ^ 0x4d49585f5049434bull);
    const uint64_t knoise = vk::mix64(sample_seed ^ 0x4d49585f4e4f4953ull);
    std::vector<float> means((size_t)ncomp * d);
    for (size_t e = 0; e < means.size(); ++e) means[e] = (float)(64.0 * unit_closed0(vk::mix64(kmean + e)));
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const uint64_t row = (uint64_t)(row0 + r);
        const uint64_t comp = ((vk::mix64(kpick + row) >> 32) * (uint64_t)ncomp) >> 32;
        const float* mu = means.data() + comp * d;
        for (int j = 0; j < d; ++j) {
            const double v = (double)mu[j] + (double)sigma * normal_at(knoise, row * (uint64_t)d + (uint64_t)j);
            out[r * d + j] = (float)std::min(255.0, std::max(0.0, std::nearbyint(v)));
        }
    }
    return 0;
}

int vk_host_gen_cdf(uint64_t seed, int clusters, int m, double alpha, uint32_t* cdf) {
    if (clusters <= 0 || m <= 0 || !(alpha > 0) || !cdf) return -1;
    const uint64_t key = vk::mix64(seed ^ 0x44495249434c4554ull);
#pragma omp parallel for schedule(dynamic)
    for (int64_t t = 0; t < (int64_t)clusters * m; ++t) {
        Stream st{vk::mix64(key + (uint64_t)t)};
        double g[256], sum = 0.0;
        for (int c = 0; c < 256; ++c) sum += (g[c] = gamma_draw(st, alpha));
        uint32_t* out = cdf + (size_t)t * 256;
        double cum = 0.0;
        for (int c = 0; c < 255; ++c) {
            cum += g[c] / sum;
            const double v = std::floor(cum * 4294967296.0);
            out[c] = v >= 4294967295.0 ? 4294967295u : (uint32_t)v;
        }
        out[255] = 4294967295u;
    }
    return 0;
}

int vk_host_gen_codes(uint64_t seed, const uint32_t* cdf, int clusters, int m, int64_t row0, int64_t n,
                      uint8_t* codes) {
    if (!cdf || !codes || clusters <= 0 || m <= 0 || row0 < 0 || n < 0) return -1;
    const uint64_t key = vk::mix64(seed);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < n; ++r)
        for (int s = 0; s < m; ++s)
            codes[r * m + s] = (uint8_t)vk::gen_code(key, (uint64_t)(row0 + r), s, cdf, clusters, m);
    return 0;
}

int vk_host_gen_codes_rows(uint64_t seed, const uint32_t* cdf, int clusters, int m, const int64_t* rows,
                           int64_t count, uint8_t* codes) {
    if (!cdf || !codes || !rows || clusters <= 0 || m <= 0 || count < 0) return -1;
    const uint64_t key = vk::mix64(seed);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < count; ++r)
        for (int s = 0; s < m; ++s)
            codes[r * m + s] = rows[r] < 0 ? 0 : (uint8_t)vk::gen_code(key, (uint64_t)rows[r], s, cdf, clusters, m);
    return 0;
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------ index files
namespace {
thread_local std::string g_host_error;
int host_fail(int code, const std::string& msg) {
    g_host_error = msg;
    return code;
}
}  // namespace

int vk_host_last_error(char* buf, size_t len) {
    if (!buf || len == 0) return -1;
    std::snprintf(buf, len, "%s", g_host_error.c_str());
    return 0;
}

uint32_t vk_host_crc32c(const void* data, size_t len, int hardware) { return vkio::crc32c(data, len, hardware != 0); }

int vk_host_index_write(const char* path, const float* centroids, int m, int dsub, const uint8_t* codes, int64_t n) {
    if (!path || !centroids || (!codes && n > 0) || m <= 0 || dsub <= 0 || n < 0) return host_fail(-1, "bad arguments");
    uint64_t done = 0;
    const std::string err = vkio::write_index(path, centroids, (uint32_t)m, (uint32_t)dsub, (uint64_t)n,
                                              [&](uint64_t rows, uint8_t* buf) {
                                                  std::memcpy(buf, codes + done * m, rows * m);
                                                  done += rows;
                                                  return true;
                                              });
    return err.empty() ? 0 : host_fail(-2, err);
}

int vk_host_index_info(const char* path, int64_t* n, int* d, int* m, int* dsub) {
    if (!path) return host_fail(-1, "bad arguments");
    vkio::Reader r(path);
    if (!r.ok()) return host_fail(-2, r.err);
    if (n) *n = (int64_t)r.h.n;
    if (d) *d = (int)r.h.d;
    if (m) *m = (int)r.h.m;
    if (dsub) *dsub = (int)r.h.dsub;
    return 0;
}

int vk_host_index_read(const char* path, float* centroids, int64_t first, int64_t count, uint8_t* codes, int verify) {
    if (!path || first < 0 || count < 0 || (!codes && count > 0)) return host_fail(-1, "bad arguments");
    vkio::Reader r(path);
    if (!r.ok()) return host_fail(-2, r.err);
    if (centroids) {
        const std::string err = r.centroids(centroids);
        if (!err.empty()) return host_fail(-2, err);
    }
    const std::string err = r.rows((uint64_t)first, (uint64_t)count, verify != 0,
                                   [&](uint64_t row0, uint64_t rows, const uint8_t* bytes) {
                                       std::memcpy(codes + (row0 - first) * r.h.m, bytes, rows * r.h.m);
                                       return true;
                                   });
    return err.empty() ? 0 : host_fail(err == "row range out of bounds" ? -1 : -2, err);
}
