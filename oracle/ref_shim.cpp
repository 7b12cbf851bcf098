// extern "C" shim over the reference's own CPU library — TEST INFRASTRUCTURE ONLY.
//
// oracle/Makefile compiles this file together with the reference's unmodified sources
// (src/cpu/cpu_ref.cpp, src/cpu/pq.cpp, src/cpu/io.cpp, read where they lie) into oracle/_ref/libveckern_ref.so.
// It lets Python tests and bench.py's CPU-baseline leg call the reference itself: to pin the plain-C
// restatement (oracle/vk_oracle.c), to generate the golden fixtures under tests/golden/, and to time the
// reference CPU path. Nothing in the product loads it.
#include <omp.h>

#include <cstdint>
#include <cstring>
#include <vector>

#include "veckern/cpu_ref.hpp"
#include "veckern/io.hpp"
#include "veckern/pq.hpp"

using veckern::Neighbor;
using veckern::ProductQuantizer;

namespace {
void split(const std::vector<Neighbor>& nb, float* d, int32_t* i) {
    for (std::size_t j = 0; j < nb.size(); ++j) {
        d[j] = nb[j].dist;
        i[j] = nb[j].id;
    }
}
}  // namespace

extern "C" {

// OpenMP threads for the reference's parallel loops (its CPU path, PQ training and encoding). A launcher may have
// set OMP_NUM_THREADS=1 before the process started (torchrun does); this overrides it for the calling thread.
void ref_set_threads(int n) {
    if (n > 0) omp_set_num_threads(n);
}
int ref_get_threads() { return omp_get_max_threads(); }

void* ref_pq_create(int64_t d, int64_t m) { return new ProductQuantizer(d, m); }
void ref_pq_destroy(void* pq) { delete static_cast<ProductQuantizer*>(pq); }
void ref_pq_train(void* pq, const float* x, int64_t n, int64_t iters, uint64_t seed) {
    static_cast<ProductQuantizer*>(pq)->train(x, n, iters, seed);
}
void ref_pq_encode(const void* pq, const float* x, int64_t n, uint8_t* codes) {
    static_cast<const ProductQuantizer*>(pq)->encode(x, n, codes);
}
void ref_pq_decode(const void* pq, const uint8_t* codes, int64_t n, float* x) {
    static_cast<const ProductQuantizer*>(pq)->decode(codes, n, x);
}
void ref_pq_get_centroids(const void* pq, float* out) {
    const auto& c = static_cast<const ProductQuantizer*>(pq)->centroids();
    std::memcpy(out, c.data(), c.size() * sizeof(float));
}
// The reference has no centroid setter (include/veckern/pq.hpp:30-32); configs with given centroids need one.
void ref_pq_set_centroids(void* pq, const float* in) {
    const auto& c = static_cast<ProductQuantizer*>(pq)->centroids();
    std::memcpy(const_cast<float*>(c.data()), in, c.size() * sizeof(float));
}

void ref_compute_lut(const void* pq, const float* queries, int64_t nq, float* lut) {
    veckern::compute_lut(*static_cast<const ProductQuantizer*>(pq), queries, nq, lut);
}
void ref_adc_scan(const float* lut, int64_t nq, const uint8_t* codes, int64_t n, int64_t m, float* dists) {
    veckern::adc_scan(lut, nq, codes, n, m, dists);
}
void ref_select_topk(const float* dists, int64_t nq, int64_t n, int64_t k, float* out_d, int32_t* out_i) {
    std::vector<Neighbor> out(nq * k);
    veckern::select_topk(dists, nq, n, k, out.data());
    split(out, out_d, out_i);
}
void ref_adc_search(const void* pq, const uint8_t* codes, int64_t n, const float* queries, int64_t nq, int64_t k,
                    float* out_d, int32_t* out_i) {
    std::vector<Neighbor> out(nq * k);
    veckern::adc_search(*static_cast<const ProductQuantizer*>(pq), codes, n, queries, nq, k, out.data());
    split(out, out_d, out_i);
}
void ref_exact_knn(const float* base, int64_t n, const float* queries, int64_t nq, int64_t d, int64_t k,
                   float* out_d, int32_t* out_i) {
    std::vector<Neighbor> out(nq * k);
    veckern::exact_knn(base, n, queries, nq, d, k, out.data());
    split(out, out_d, out_i);
}
void ref_rerank_exact(const float* base, int64_t d, const float* queries, int64_t nq, const int32_t* cand_ids,
                      int64_t r, int64_t k, float* out_d, int32_t* out_i) {
    std::vector<Neighbor> cand(nq * r), out(nq * k);
    for (int64_t j = 0; j < nq * r; ++j) cand[j] = {0.f, cand_ids[j]};
    veckern::rerank_exact(base, d, queries, nq, cand.data(), r, k, out.data());
    split(out, out_d, out_i);
}
void ref_topk_push_all(const float* dists, const int32_t* ids, int64_t count, int64_t k, float* out_d,
                       int32_t* out_i) {
    veckern::TopK top(k);
    for (int64_t j = 0; j < count; ++j) top.push(dists[j], ids[j]);
    std::vector<Neighbor> out(k);
    top.write(out.data());
    split(out, out_d, out_i);
}
void ref_synthetic_clustered(int64_t n, int64_t d, int64_t clusters, uint64_t seed, float* out) {
    const auto v = veckern::synthetic_clustered(n, d, clusters, seed);
    std::memcpy(out, v.data(), v.size() * sizeof(float));
}

}  // extern "C"
