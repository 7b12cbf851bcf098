/*
 * CPU oracle for the flat PQ search path — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's CPU path (shivdeshpande/VecKern, src/cpu/cpu_ref.cpp and
 * include/veckern/cpu_ref.hpp). Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
 * may load it, and only as the checker: the product path never calls it.
 *
 * Arithmetic contract (what makes results bit-comparable with the reference):
 *   - LUT entry:  acc = 0; for j < dsub: diff = q[j] - c[j]; acc = acc + diff * diff   (fp32, no FMA)
 *     (include/veckern/common.hpp:27-34, src/cpu/cpu_ref.cpp:7-14)
 *   - distance:   acc = 0; for s < m: acc = acc + lut[s][code[s]]                     (fp32, in order)
 *     (src/cpu/cpu_ref.cpp:16-27, 46-50)
 *   - selection:  the k smallest (dist, id) pairs under the strict order
 *     a < b  <=>  a.dist < b.dist || (a.dist == b.dist && a.id < b.id), ascending, padded with
 *     {+inf, -1}  (include/veckern/common.hpp:19-21, include/veckern/cpu_ref.hpp:14-40)
 * The library is compiled with -ffp-contract=off so the compiler cannot fuse diff*diff into an FMA.
 */
#ifndef VK_ORACLE_H
#define VK_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* lut: nq x m x 256, row-major.  centroids: [m][256][dsub].  queries: nq x (m*dsub). */
void vko_compute_lut(const float* centroids, int m, int dsub, const float* queries, int64_t nq, float* lut);

/* dists: nq x n.  codes: row-major n x m bytes. */
void vko_adc_scan(const float* lut, int64_t nq, const uint8_t* codes, int64_t n, int m, float* dists);

/* Row-wise top-k of an nq x n matrix; ids are column indices. */
void vko_select_topk(const float* dists, int64_t nq, int64_t n, int k, float* out_d, int32_t* out_i);

/* Fused LUT + scan + top-k per query (the reference's adc_search). threads <= 0: all cores. */
void vko_adc_search(const float* centroids, int m, int dsub, const uint8_t* codes, int64_t n,
                    const float* queries, int64_t nq, int k, float* out_d, int32_t* out_i, int threads);

/* Pushes count (dist, id) pairs, in order, through one bounded top-k and writes k results. */
void vko_topk_push_all(const float* dists, const int32_t* ids, int64_t count, int k, float* out_d,
                       int32_t* out_i);

/* Merges `lists` lists of k_in (dist, id) per query (layout [nq][lists][k_in]) into the k best. Entries with
 * id < 0 are padding and are skipped. */
void vko_merge_topk(const float* d, const int32_t* ids, int lists, int k_in, int64_t nq, int k, float* out_d,
                    int32_t* out_i);

/* Exact re-rank (src/cpu/cpu_ref.cpp:66-77): for each query, l2sq(query, base[id], d) of its r candidate ids
 * (id < 0 skipped), pushed in candidate order through one bounded top-k of k. base: n x d, queries: nq x d. */
void vko_rerank_exact(const float* base, int d, const float* queries, int64_t nq, const int32_t* cand_ids, int r,
                      int k, float* out_d, int32_t* out_i);

/* Mean |found[:k] ∩ truth[:k]| / k (src/cpu/cpu_ref.cpp:79-91). */
double vko_recall_at_k(const int32_t* found, int64_t found_stride, const int32_t* truth, int64_t truth_stride,
                       int64_t nq, int k);

/* Half-precision LUT search (the library's VK_LUT_F16 definition; see vk_oracle.c): the scaled, half-rounded
 * tables (as floats) with their per-query exponents, and the search over them. */
void vko_compute_lut_h16(const float* centroids, int m, int dsub, const float* queries, int64_t nq, float* lut,
                         int* exps);
void vko_adc_search_h16(const float* centroids, int m, int dsub, const uint8_t* codes, int64_t n,
                        const float* queries, int64_t nq, int k, float* out_d, int32_t* out_i, int threads);

/* IVF search (the library's IVF definition; see vk_oracle.c): the flat search restricted to the rows of each
 * query's nprobe nearest lists. */
void vko_ivf_search(const float* centroids, int m, int dsub, const uint8_t* codes, const int32_t* list_of, int64_t n,
                    const float* coarse, int nlist, const float* queries, int64_t nq, int nprobe, int k,
                    float* out_d, int32_t* out_i, int32_t* probes_out, int threads);

/* 4-bit PQ (the library's vk_index_create_pq4 definition; see vk_oracle.c): centroids [m][16][dsub], codes
 * n x ceil(m / 2) bytes with sub-code s in nibble s % 2 (low first) of byte s / 2; lut: nq x m x 16. */
void vko_pq4_encode(const float* centroids, int m, int dsub, const float* x, int64_t n, uint8_t* codes);
void vko_compute_lut_pq4(const float* centroids, int m, int dsub, const float* queries, int64_t nq, float* lut);
void vko_adc_search_pq4(const float* centroids, int m, int dsub, const uint8_t* codes, int64_t n,
                        const float* queries, int64_t nq, int k, float* out_d, int32_t* out_i, int threads);

/* Streaming search over codes that arrive in blocks (large configs: the codes never exist on the host at
 * once). Per query one bounded top-k; feed() must be called with ascending, non-overlapping id ranges. */
typedef struct vko_stream vko_stream;
vko_stream* vko_stream_create(const float* lut, int64_t nq, int m, int k);
void vko_stream_feed(vko_stream* s, const uint8_t* codes, int64_t count, int64_t id_base, int threads);
void vko_stream_finish(vko_stream* s, float* out_d, int32_t* out_i);
void vko_stream_destroy(vko_stream* s);

#ifdef __cplusplus
}
#endif
#endif
