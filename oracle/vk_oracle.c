/*
 * CPU oracle for the flat PQ search path — TEST INFRASTRUCTURE ONLY (see vk_oracle.h).
 * Plain-C restatement of shivdeshpande/VecKern's CPU reference; every function cites the reference lines it
 * follows. Built with -O2 -ffp-contract=off -fopenmp.
 */
#include "vk_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define KSUB 256

/* ---------------------------------------------------------------- ordering
 * include/veckern/common.hpp:19-21: a < b iff a.dist < b.dist, or equal dists and a.id < b.id. */
static inline int nb_less(float da, int32_t ia, float db, int32_t ib) {
    return da < db || (da == db && ia < ib);
}

/* ---------------------------------------------------------------- l2sq
 * include/veckern/common.hpp:27-34: sequential j, acc starts at 0, diff = a - b, acc += diff * diff. */
static inline float l2sq(const float* a, const float* b, int d) {
    float acc = 0.f;
    for (int j = 0; j < d; ++j) {
        const float diff = a[j] - b[j];
        const float sq = diff * diff; /* separate statement + -ffp-contract=off: no FMA */
        acc = acc + sq;
    }
    return acc;
}

/* ---------------------------------------------------------------- bounded top-k
 * include/veckern/cpu_ref.hpp:14-40 (TopK): a max-heap of at most k (dist, id) pairs; once full, a candidate
 * replaces the root only if it is strictly smaller; write() emits ascending order padded with {+inf, -1}. */
typedef struct {
    int k, size;
    float* d;
    int32_t* id;
} topk_t;

static void topk_init(topk_t* t, int k, float* dbuf, int32_t* ibuf) {
    t->k = k;
    t->size = 0;
    t->d = dbuf;
    t->id = ibuf;
}

static void heap_sift_down(topk_t* t, int i) {
    for (;;) {
        int l = 2 * i + 1, r = l + 1, big = i;
        if (l < t->size && nb_less(t->d[big], t->id[big], t->d[l], t->id[l])) big = l;
        if (r < t->size && nb_less(t->d[big], t->id[big], t->d[r], t->id[r])) big = r;
        if (big == i) return;
        float td = t->d[i]; t->d[i] = t->d[big]; t->d[big] = td;
        int32_t ti = t->id[i]; t->id[i] = t->id[big]; t->id[big] = ti;
        i = big;
    }
}

static inline void topk_push(topk_t* t, float dist, int32_t id) {
    if (t->size < t->k) {
        int i = t->size++;
        t->d[i] = dist;
        t->id[i] = id;
        while (i > 0) { /* sift up */
            int p = (i - 1) / 2;
            if (!nb_less(t->d[p], t->id[p], t->d[i], t->id[i])) break;
            float td = t->d[i]; t->d[i] = t->d[p]; t->d[p] = td;
            int32_t ti = t->id[i]; t->id[i] = t->id[p]; t->id[p] = ti;
            i = p;
        }
    } else if (t->k > 0 && nb_less(dist, id, t->d[0], t->id[0])) {
        t->d[0] = dist;
        t->id[0] = id;
        heap_sift_down(t, 0);
    }
}

/* Ascending output: repeatedly move the heap root (the largest) to the end. */
static void topk_write(topk_t* t, float* out_d, int32_t* out_i) {
    const int n = t->size;
    for (int end = n - 1; end > 0; --end) {
        float td = t->d[0]; t->d[0] = t->d[end]; t->d[end] = td;
        int32_t ti = t->id[0]; t->id[0] = t->id[end]; t->id[end] = ti;
        t->size = end;
        heap_sift_down(t, 0);
    }
    t->size = n;
    for (int j = 0; j < n; ++j) {
        out_d[j] = t->d[j];
        out_i[j] = t->id[j];
    }
    for (int j = n; j < t->k; ++j) {
        out_d[j] = INFINITY;
        out_i[j] = -1;
    }
}

/* ---------------------------------------------------------------- LUT
 * src/cpu/cpu_ref.cpp:7-14 (compute_lut): lut[q][s][c] = l2sq(query[q] + s*dsub, centroid(s, c), dsub). */
void vko_compute_lut(const float* centroids, int m, int dsub, const float* queries, int64_t nq, float* lut) {
    const int64_t d = (int64_t)m * dsub;
#pragma omp parallel for schedule(static)
    for (int64_t q = 0; q < nq; ++q)
        for (int s = 0; s < m; ++s)
            for (int c = 0; c < KSUB; ++c)
                lut[(q * m + s) * KSUB + c] =
                    l2sq(queries + q * d + (int64_t)s * dsub, centroids + ((int64_t)s * KSUB + c) * dsub, dsub);
}

/* ---------------------------------------------------------------- scan
 * src/cpu/cpu_ref.cpp:16-27 (adc_scan): acc = 0; acc += table[s*256 + code[s]] for s = 0..m-1. */
static inline float adc_one(const float* table, const uint8_t* code, int m) {
    float acc = 0.f;
    for (int s = 0; s < m; ++s) acc = acc + table[s * KSUB + code[s]];
    return acc;
}

void vko_adc_scan(const float* lut, int64_t nq, const uint8_t* codes, int64_t n, int m, float* dists) {
#pragma omp parallel for schedule(static)
    for (int64_t q = 0; q < nq; ++q) {
        const float* table = lut + q * m * KSUB;
        for (int64_t i = 0; i < n; ++i) dists[q * n + i] = adc_one(table, codes + i * m, m);
    }
}

/* ---------------------------------------------------------------- select
 * src/cpu/cpu_ref.cpp:29-36 (select_topk): push every column index of the row, in order. */
void vko_select_topk(const float* dists, int64_t nq, int64_t n, int k, float* out_d, int32_t* out_i) {
#pragma omp parallel
    {
        float* hd = (float*)malloc(sizeof(float) * (size_t)(k > 0 ? k : 1));
        int32_t* hi = (int32_t*)malloc(sizeof(int32_t) * (size_t)(k > 0 ? k : 1));
#pragma omp for schedule(static)
        for (int64_t q = 0; q < nq; ++q) {
            topk_t t;
            topk_init(&t, k, hd, hi);
            for (int64_t i = 0; i < n; ++i) topk_push(&t, dists[q * n + i], (int32_t)i);
            topk_write(&t, out_d + q * k, out_i + q * k);
        }
        free(hd);
        free(hi);
    }
}

/* ---------------------------------------------------------------- fused search
 * src/cpu/cpu_ref.cpp:38-54 (adc_search): per query, LUT then scan then bounded top-k, no n-wide matrix. */
void vko_adc_search(const float* centroids, int m, int dsub, const uint8_t* codes, int64_t n,
                    const float* queries, int64_t nq, int k, float* out_d, int32_t* out_i, int threads) {
#ifdef _OPENMP
    const int nt = threads > 0 ? threads : omp_get_max_threads();
#else
    const int nt = 1;
    (void)threads;
#endif
    const int64_t d = (int64_t)m * dsub;
#pragma omp parallel num_threads(nt)
    {
        float* lut = (float*)malloc(sizeof(float) * (size_t)m * KSUB);
        float* hd = (float*)malloc(sizeof(float) * (size_t)(k > 0 ? k : 1));
        int32_t* hi = (int32_t*)malloc(sizeof(int32_t) * (size_t)(k > 0 ? k : 1));
#pragma omp for schedule(dynamic)
        for (int64_t q = 0; q < nq; ++q) {
            vko_compute_lut(centroids, m, dsub, queries + q * d, 1, lut);
            topk_t t;
            topk_init(&t, k, hd, hi);
            for (int64_t i = 0; i < n; ++i) topk_push(&t, adc_one(lut, codes + i * m, m), (int32_t)i);
            topk_write(&t, out_d + q * k, out_i + q * k);
        }
        free(lut);
        free(hd);
        free(hi);
    }
}

/* ---------------------------------------------------------------- half-precision LUT search
 * Not in the reference, which lists fp16 lookup tables as a next step (README.md:219); this is the definition the
 * library's VK_LUT_F16 search implements (include/vk_abi.h, lut_precision), restated on the CPU:
 *   T = the fp32 LUT of compute_lut; M = max over (s, c) of T; e = 15 - E with M = f * 2^E, f in [0.5, 1),
 *   clamped to [-64, 64] (e = 0 when M = 0, 64 when M is subnormal); entry = half(T * 2^e), round to nearest even;
 *   distance = (fp32 sum over s = 0..m-1 of the entries, from 0, in order) * 2^-e; top-k by (distance, id). */
static int h16_exponent(float max) {
    uint32_t bits;
    memcpy(&bits, &max, sizeof(bits));
    const int ef = (int)((bits >> 23) & 0xffu);
    if (bits == 0u || ef == 255) return 0;
    if (ef == 0) return 64;
    const int e = 15 - (ef - 126);
    return e < -64 ? -64 : e > 64 ? 64 : e;
}

/* x (>= 0, < 65520) rounded to the nearest half-precision value (ties to even), returned as a float. The step
 * between halves around x is 2^(E - 10) for x in [2^E, 2^(E+1)), E >= -14, and 2^-24 below 2^-14 (subnormals);
 * x / step is exact in double, so rounding it to an integer (nearbyint: ties to even) rounds x. */
static float half_round(float x) {
    if (x == 0.f) return x;
    int ex;
    frexp((double)x, &ex); /* x = f * 2^ex, f in [0.5, 1): x in [2^(ex-1), 2^ex) */
    int E = ex - 1;
    if (E < -14) E = -14;
    const double step = ldexp(1.0, E - 10);
    return (float)(nearbyint((double)x / step) * step);
}

void vko_compute_lut_h16(const float* centroids, int m, int dsub, const float* queries, int64_t nq, float* lut,
                         int* exps) {
    vko_compute_lut(centroids, m, dsub, queries, nq, lut);
#pragma omp parallel for schedule(static)
    for (int64_t q = 0; q < nq; ++q) {
        float* t = lut + q * m * KSUB;
        float mx = 0.f;
        for (int j = 0; j < m * KSUB; ++j) mx = t[j] > mx ? t[j] : mx;
        const int e = h16_exponent(mx);
        for (int j = 0; j < m * KSUB; ++j) t[j] = half_round(ldexpf(t[j], e));
        exps[q] = e;
    }
}

void vko_adc_search_h16(const float* centroids, int m, int dsub, const uint8_t* codes, int64_t n,
                        const float* queries, int64_t nq, int k, float* out_d, int32_t* out_i, int threads) {
#ifdef _OPENMP
    const int nt = threads > 0 ? threads : omp_get_max_threads();
#else
    const int nt = 1;
    (void)threads;
#endif
    const int64_t d = (int64_t)m * dsub;
#pragma omp parallel num_threads(nt)
    {
        float* lut = (float*)malloc(sizeof(float) * (size_t)m * KSUB);
        float* hd = (float*)malloc(sizeof(float) * (size_t)(k > 0 ? k : 1));
        int32_t* hi = (int32_t*)malloc(sizeof(int32_t) * (size_t)(k > 0 ? k : 1));
#pragma omp for schedule(dynamic)
        for (int64_t q = 0; q < nq; ++q) {
            vko_compute_lut(centroids, m, dsub, queries + q * d, 1, lut);
            float mx = 0.f;
            for (int j = 0; j < m * KSUB; ++j) mx = lut[j] > mx ? lut[j] : mx;
            const int e = h16_exponent(mx);
            for (int j = 0; j < m * KSUB; ++j) lut[j] = half_round(ldexpf(lut[j], e));
            topk_t t;
            topk_init(&t, k, hd, hi);
            for (int64_t i = 0; i < n; ++i) topk_push(&t, ldexpf(adc_one(lut, codes + i * m, m), -e), (int32_t)i);
            topk_write(&t, out_d + q * k, out_i + q * k);
        }
        free(lut);
        free(hd);
        free(hi);
    }
}

/* ---------------------------------------------------------------- IVF (inverted-file) search
 * Not in the reference, which lists IVF partitioning as a next step (README.md:219); this is the definition the
 * library's IVF search implements, restated on the CPU. Rows belong to lists (list_of[i] in [0, nlist)); per query:
 *   probes = the nprobe smallest (l2sq(query, coarse[l]), l) pairs over the lists (the exact l2sq of
 *            common.hpp:27-34 over all d dimensions; ties to the lower list);
 *   result = the k smallest (ADC distance, row) pairs over the rows of the probed lists, the ADC distance being the
 *            flat search's (the same fp32 LUT, summed in sub-space order): the flat search restricted to those rows.
 * probes_out (optional, nq x nprobe): the probed lists in ascending (distance, list) order. */
void vko_ivf_search(const float* centroids, int m, int dsub, const uint8_t* codes, const int32_t* list_of, int64_t n,
                    const float* coarse, int nlist, const float* queries, int64_t nq, int nprobe, int k,
                    float* out_d, int32_t* out_i, int32_t* probes_out, int threads) {
#ifdef _OPENMP
    const int nt = threads > 0 ? threads : omp_get_max_threads();
#else
    const int nt = 1;
    (void)threads;
#endif
    const int64_t d = (int64_t)m * dsub;
#pragma omp parallel num_threads(nt)
    {
        float* lut = (float*)malloc(sizeof(float) * (size_t)m * KSUB);
        float* hd = (float*)malloc(sizeof(float) * (size_t)(k > 0 ? k : 1));
        int32_t* hi = (int32_t*)malloc(sizeof(int32_t) * (size_t)(k > 0 ? k : 1));
        float* pd = (float*)malloc(sizeof(float) * (size_t)(nprobe > 0 ? nprobe : 1));
        int32_t* pi = (int32_t*)malloc(sizeof(int32_t) * (size_t)(nprobe > 0 ? nprobe : 1));
        float* pod = (float*)malloc(sizeof(float) * (size_t)(nprobe > 0 ? nprobe : 1));
        int32_t* poi = (int32_t*)malloc(sizeof(int32_t) * (size_t)(nprobe > 0 ? nprobe : 1));
        unsigned char* probed = (unsigned char*)malloc((size_t)(nlist > 0 ? nlist : 1));
#pragma omp for schedule(dynamic)
        for (int64_t q = 0; q < nq; ++q) {
            const float* qv = queries + q * d;
            topk_t pt;
            topk_init(&pt, nprobe, pd, pi);
            for (int l = 0; l < nlist; ++l) topk_push(&pt, l2sq(qv, coarse + (int64_t)l * d, (int)d), l);
            topk_write(&pt, pod, poi);
            memset(probed, 0, (size_t)nlist);
            for (int j = 0; j < nprobe; ++j) {
                if (poi[j] >= 0) probed[poi[j]] = 1;
                if (probes_out) probes_out[q * nprobe + j] = poi[j];
            }
            vko_compute_lut(centroids, m, dsub, qv, 1, lut);
            topk_t t;
            topk_init(&t, k, hd, hi);
            for (int64_t i = 0; i < n; ++i)
                if (probed[list_of[i]]) topk_push(&t, adc_one(lut, codes + i * m, m), (int32_t)i);
            topk_write(&t, out_d + q * k, out_i + q * k);
        }
        free(lut);
        free(hd);
        free(hi);
        free(pd);
        free(pi);
        free(pod);
        free(poi);
        free(probed);
    }
}

/* ---------------------------------------------------------------- 4-bit PQ
 * Not in the reference, which lists 4-bit PQ as a next step (README.md:219); this is the definition the library's
 * 4-bit indexes (vk_index_create_pq4) implement, restated on the CPU. 16 centroids per sub-space ([m][16][dsub]);
 * sub-code s of a row sits in nibble s % 2 (low first) of byte s / 2 (ceil(m / 2) bytes per row):
 *   lut[s][c] = l2sq(query sub-vector s, centroid (s, c)) for c < 16 (the arithmetic of compute_lut);
 *   distance  = fp32 sum over s = 0..m-1 of lut[s][code_s], from 0, in order (adc_scan's order);
 *   result    = the k smallest (distance, id) pairs (TopK), ascending, padded with {+inf, -1};
 *   encoding  = the first nearest of the 16 centroids under l2sq (pq.cpp:11-22's rule). */
#define KSUB4 16

static inline uint32_t nib(const uint8_t* row, int s) { return (row[s >> 1] >> (4 * (s & 1))) & 0xfu; }

void vko_pq4_encode(const float* centroids, int m, int dsub, const float* x, int64_t n, uint8_t* codes) {
    const int64_t d = (int64_t)m * dsub, mb = (m + 1) / 2;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        uint8_t* row = codes + i * mb;
        memset(row, 0, (size_t)mb);
        for (int s = 0; s < m; ++s) {
            int best = 0;
            float best_d = 3.402823466e+38f;
            for (int c = 0; c < KSUB4; ++c) {
                const float dist = l2sq(x + i * d + (int64_t)s * dsub, centroids + ((int64_t)s * KSUB4 + c) * dsub, dsub);
                if (dist < best_d) {
                    best_d = dist;
                    best = c;
                }
            }
            row[s >> 1] |= (uint8_t)(best << (4 * (s & 1)));
        }
    }
}

void vko_compute_lut_pq4(const float* centroids, int m, int dsub, const float* queries, int64_t nq, float* lut) {
    const int64_t d = (int64_t)m * dsub;
#pragma omp parallel for schedule(static)
    for (int64_t q = 0; q < nq; ++q)
        for (int s = 0; s < m; ++s)
            for (int c = 0; c < KSUB4; ++c)
                lut[(q * m + s) * KSUB4 + c] =
                    l2sq(queries + q * d + (int64_t)s * dsub, centroids + ((int64_t)s * KSUB4 + c) * dsub, dsub);
}

void vko_adc_search_pq4(const float* centroids, int m, int dsub, const uint8_t* codes, int64_t n,
                        const float* queries, int64_t nq, int k, float* out_d, int32_t* out_i, int threads) {
#ifdef _OPENMP
    const int nt = threads > 0 ? threads : omp_get_max_threads();
#else
    const int nt = 1;
    (void)threads;
#endif
    const int64_t d = (int64_t)m * dsub, mb = (m + 1) / 2;
#pragma omp parallel num_threads(nt)
    {
        float* lut = (float*)malloc(sizeof(float) * (size_t)m * KSUB4);
        float* hd = (float*)malloc(sizeof(float) * (size_t)(k > 0 ? k : 1));
        int32_t* hi = (int32_t*)malloc(sizeof(int32_t) * (size_t)(k > 0 ? k : 1));
#pragma omp for schedule(dynamic)
        for (int64_t q = 0; q < nq; ++q) {
            vko_compute_lut_pq4(centroids, m, dsub, queries + q * d, 1, lut);
            topk_t t;
            topk_init(&t, k, hd, hi);
            for (int64_t i = 0; i < n; ++i) {
                const uint8_t* row = codes + i * mb;
                float acc = 0.f;
                for (int s = 0; s < m; ++s) acc = acc + lut[s * KSUB4 + nib(row, s)];
                topk_push(&t, acc, (int32_t)i);
            }
            topk_write(&t, out_d + q * k, out_i + q * k);
        }
        free(lut);
        free(hd);
        free(hi);
    }
}

void vko_topk_push_all(const float* dists, const int32_t* ids, int64_t count, int k, float* out_d,
                       int32_t* out_i) {
    float* hd = (float*)malloc(sizeof(float) * (size_t)(k > 0 ? k : 1));
    int32_t* hi = (int32_t*)malloc(sizeof(int32_t) * (size_t)(k > 0 ? k : 1));
    topk_t t;
    topk_init(&t, k, hd, hi);
    for (int64_t j = 0; j < count; ++j) topk_push(&t, dists[j], ids[j]);
    topk_write(&t, out_d, out_i);
    free(hd);
    free(hi);
}

/* Merge of per-shard lists: the union's k best under the same order; padding (id < 0) is skipped, as the
 * reference's select_kernel skips id < 0 candidates (src/cuda/kernels.cuh:193-195). */
void vko_merge_topk(const float* d, const int32_t* ids, int lists, int k_in, int64_t nq, int k, float* out_d,
                    int32_t* out_i) {
#pragma omp parallel
    {
        float* hd = (float*)malloc(sizeof(float) * (size_t)(k > 0 ? k : 1));
        int32_t* hi = (int32_t*)malloc(sizeof(int32_t) * (size_t)(k > 0 ? k : 1));
#pragma omp for schedule(static)
        for (int64_t q = 0; q < nq; ++q) {
            topk_t t;
            topk_init(&t, k, hd, hi);
            const int64_t base = q * (int64_t)lists * k_in;
            for (int64_t j = 0; j < (int64_t)lists * k_in; ++j)
                if (ids[base + j] >= 0) topk_push(&t, d[base + j], ids[base + j]);
            topk_write(&t, out_d + q * k, out_i + q * k);
        }
        free(hd);
        free(hi);
    }
}

/* src/cpu/cpu_ref.cpp:66-77 (rerank_exact): candidates in order, id < 0 skipped, l2sq(query, base row). */
void vko_rerank_exact(const float* base, int d, const float* queries, int64_t nq, const int32_t* cand_ids, int r,
                      int k, float* out_d, int32_t* out_i) {
#pragma omp parallel
    {
        float* hd = (float*)malloc(sizeof(float) * (size_t)(k > 0 ? k : 1));
        int32_t* hi = (int32_t*)malloc(sizeof(int32_t) * (size_t)(k > 0 ? k : 1));
#pragma omp for schedule(static)
        for (int64_t q = 0; q < nq; ++q) {
            topk_t t;
            topk_init(&t, k, hd, hi);
            for (int j = 0; j < r; ++j) {
                const int32_t id = cand_ids[q * r + j];
                if (id >= 0) topk_push(&t, l2sq(queries + q * d, base + (int64_t)id * d, d), id);
            }
            topk_write(&t, out_d + q * k, out_i + q * k);
        }
        free(hd);
        free(hi);
    }
}

/* src/cpu/cpu_ref.cpp:79-91 (recall_at_k), on id arrays. */
double vko_recall_at_k(const int32_t* found, int64_t found_stride, const int32_t* truth, int64_t truth_stride,
                       int64_t nq, int k) {
    if (nq == 0 || k == 0) return 0.0;
    double total = 0.0;
    for (int64_t q = 0; q < nq; ++q) {
        int hits = 0;
        for (int j = 0; j < k; ++j) {
            const int32_t f = found[q * found_stride + j];
            for (int t = 0; t < k; ++t)
                if (truth[q * truth_stride + t] == f) {
                    ++hits;
                    break;
                }
        }
        total += (double)hits / k;
    }
    return total / (double)nq;
}

/* ---------------------------------------------------------------- streaming search */
struct vko_stream {
    int64_t nq;
    int m, k;
    const float* lut;
    float* hd;
    int32_t* hi;
    int* size;
};

vko_stream* vko_stream_create(const float* lut, int64_t nq, int m, int k) {
    vko_stream* s = (vko_stream*)calloc(1, sizeof(vko_stream));
    s->nq = nq;
    s->m = m;
    s->k = k;
    s->lut = lut;
    s->hd = (float*)malloc(sizeof(float) * (size_t)(nq * (k > 0 ? k : 1)));
    s->hi = (int32_t*)malloc(sizeof(int32_t) * (size_t)(nq * (k > 0 ? k : 1)));
    s->size = (int*)calloc((size_t)nq, sizeof(int));
    return s;
}

void vko_stream_feed(vko_stream* s, const uint8_t* codes, int64_t count, int64_t id_base, int threads) {
#ifdef _OPENMP
    const int nt = threads > 0 ? threads : omp_get_max_threads();
#else
    const int nt = 1;
    (void)threads;
#endif
#pragma omp parallel for schedule(dynamic) num_threads(nt)
    for (int64_t q = 0; q < s->nq; ++q) {
        topk_t t;
        topk_init(&t, s->k, s->hd + q * s->k, s->hi + q * s->k);
        t.size = s->size[q];
        const float* table = s->lut + q * s->m * KSUB;
        for (int64_t i = 0; i < count; ++i)
            topk_push(&t, adc_one(table, codes + i * s->m, s->m), (int32_t)(id_base + i));
        s->size[q] = t.size;
    }
}

void vko_stream_finish(vko_stream* s, float* out_d, int32_t* out_i) {
    for (int64_t q = 0; q < s->nq; ++q) {
        topk_t t;
        topk_init(&t, s->k, s->hd + q * s->k, s->hi + q * s->k);
        t.size = s->size[q];
        topk_write(&t, out_d + q * s->k, out_i + q * s->k);
        s->size[q] = t.size;
    }
}

void vko_stream_destroy(vko_stream* s) {
    if (!s) return;
    free(s->hd);
    free(s->hi);
    free(s->size);
    free(s);
}
