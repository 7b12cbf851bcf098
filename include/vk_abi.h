/*
 * VecKern-B200 C ABI: flat PQ search (per-query L2 LUT -> ADC scan over uint8 codes -> k-smallest selection)
 * on NVIDIA B200 (sm_100a). Plain pointers and sizes only; no CUDA or C++ types cross this boundary.
 *
 * Every entry point returns an int status (VK_OK = 0, negative on error); vk_last_error() gives the message of
 * the calling thread's last failure. The C++ class veckern::gpu::PQSearcher (include/veckern/gpu.hpp) is a thin
 * wrapper over these functions that rethrows failures as std::runtime_error, which is the reference's error
 * convention (src/cuda/searcher.cu:11-16, include/veckern/common.hpp:23-25).
 *
 * Results are bit-identical to the reference CPU path (src/cpu/cpu_ref.cpp:38-54): fp32 LUT entries summed over
 * j without FMA contraction, distances summed over sub-spaces s = 0..m-1 in order, and the k smallest
 * (dist, id) pairs with ties broken by the lower id, ascending, padded with {+inf, -1}.
 * Inputs must be finite: NaN distances are never returned (the reference's heap keeps them in arbitrary order).
 *
 * Thread safety: one index may be used by one host thread at a time (as the reference's PQSearcher).
 */
#ifndef VK_ABI_H
#define VK_ABI_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    VK_OK = 0,
    VK_ERR_INVALID = -1,     /* bad argument (the reference throws std::runtime_error from check()) */
    VK_ERR_CUDA = -2,        /* a CUDA runtime call failed */
    VK_ERR_NOMEM = -3,       /* device allocation failed */
    VK_ERR_DEVICE = -4,      /* a kernel reported an error through its status word (e.g. a bounded wait ran out) */
    VK_ERR_UNSUPPORTED = -5  /* configuration this build does not implement */
};

/* Scan variants of the reference API (include/veckern/gpu.hpp:13-23). They select validation rules only: every
 * search runs the one fused B200 kernel, every distances() call the one materialising scan. */
enum {
    VK_VARIANT_GLOBAL_LUT = 0,
    VK_VARIANT_SHARED_LUT = 1,
    VK_VARIANT_SHARED_LUT_VEC = 2,
    VK_VARIANT_INTERLEAVED = 3,
    VK_VARIANT_FUSED = 4,
    VK_VARIANT_FUSED_REG = 5,
    VK_VARIANT_FUSED_VEC = 6,
    VK_VARIANT_FUSED_VEC_MQ = 7,
    VK_VARIANT_FUSED_WARP = 8
};

/* One result: the reference's veckern::Neighbor (include/veckern/common.hpp:13-16), same 8-byte layout. */
typedef struct {
    float dist;
    int32_t id;
} vk_neighbor_t;

/* Replaces gpu::DeviceInfo (include/veckern/gpu.hpp:36-41). */
typedef struct {
    char name[256];
    int sm_count;
    double peak_bandwidth_gbs;  /* 2 x memory clock x bus width */
    size_t max_smem_per_block;  /* opt-in limit */
    int clock_mhz;              /* max SM clock */
} vk_device_info_t;

/* LUT precision of a search (vk_tuning_t.lut_precision). */
enum {
    VK_LUT_F32 = 0, /* fp32 entries: results bit-identical to the reference CPU path (the default) */
    VK_LUT_F16 = 1  /* half entries, summed in fp32: an approximate search with its own exact definition (below) */
};

/* Replaces gpu::Tuning (include/veckern/gpu.hpp:29-34) with the same meaning and the same accepted values
 * (src/cuda/searcher.cu:450-460): scan_threads multiple of 32 in [32, 1024] (used by distances()),
 * blocks_per_query >= 0 (vector chunks per query group; 0 = auto), queries_per_block in {1, 2, 4, 8},
 * vectors_per_step in {1, 2, 4} (32-vector groups each warp holds in flight). Added fields:
 * early_abandon (1 = default, 0 = off): stop summing a (query, row) pair once its partial distance exceeds a
 * proven bound on the query's k-th distance (m in {16, 32, 64}); results are identical either way.
 * lut_precision: VK_LUT_F32 (default) or VK_LUT_F16, the half-precision lookup tables the reference lists as a
 * next step (README.md:219), for m in {16, 32, 64}, with 4 or 8 queries per block. Per query, T[s][c] is the fp32
 * entry of the exact path, M its largest value, e = 15 - E where M = f * 2^E with f in [0.5, 1) (clamped to
 * [-64, 64]; e = 0 when M = 0); the table holds half(T * 2^e) rounded to nearest even; a row's distance is the
 * fp32 sum of its entries in sub-space order times 2^-e, and the k smallest (distance, id) pairs are returned.
 * oracle/vk_oracle.c restates this definition on the CPU (vko_adc_search_h16). vk_distances always uses fp32. */
typedef struct {
    int scan_threads;
    int blocks_per_query;
    int queries_per_block;
    int vectors_per_step;
    int early_abandon;
    int lut_precision;
} vk_tuning_t;

/* Replaces gpu::Timings (include/veckern/gpu.hpp:46-50): milliseconds per stage from CUDA events. */
typedef struct {
    double transfer_ms, lut_ms, scan_ms, select_ms;
} vk_timings_t;

/* Replaces PQSearcher::LaunchShape (include/veckern/gpu.hpp:68-73). For the fused kernel: threads = block size,
 * blocks_x = vector chunks per query group, grid_y = query groups (ceil(nq / Q)), blocks_per_sm from the
 * occupancy API, waves = work items / resident blocks. */
typedef struct {
    int threads, blocks_x, grid_y, queries_per_block, vectors_per_step, blocks_per_sm;
    double waves;
} vk_launch_shape_t;

typedef struct vk_index vk_index_t;

/* Replaces gpu::device_info (src/cuda/searcher.cu:143-156). */
int vk_device_info(int device, vk_device_info_t* out);

/* Copies the message of this thread's last failure into buf (NUL-terminated); returns its full length. */
size_t vk_last_error(char* buf, size_t len);

/* Tuning defaults and validation (include/veckern/gpu.hpp:29-34, src/cuda/searcher.cu:450-460). */
void vk_tuning_default(vk_tuning_t* t);
int vk_tuning_validate(const vk_tuning_t* t);

/* Replaces the PQSearcher constructor (src/cuda/searcher.cu:427-444): copies centroids ([m][256][dsub] fp32) and
 * row-major n x m codes from HOST memory to `device` and builds the 16-byte-word-interleaved layout there.
 * Ids reported by searches are id_base + row (id_base + n must fit in int32, as the reference's n < INT_MAX
 * check, src/cuda/searcher.cu:430). */
int vk_index_create(int device, const float* centroids, int m, int dsub, const uint8_t* codes, int64_t n,
                    int64_t id_base, vk_index_t** out);

/* 4-bit PQ index, the 4-bit codes the reference lists as a next step (README.md:219); no counterpart in its API.
 * centroids: [m][16][dsub] fp32 (16 centroids per sub-space); codes: HOST, row-major n x (m / 2) bytes, sub-code s
 * of a row in nibble s % 2 (low nibble first) of byte s / 2; m = 16, 32 or 64 (VK_ERR_UNSUPPORTED otherwise).
 * vk_search, vk_search_device, vk_search_device_coop and vk_search_noalloc accept the index; fp32 LUTs only.
 * Definition (restated on the CPU by oracle vko_adc_search_pq4): lut[s][c] = l2sq(query sub-vector s, centroid
 * (s, c)) for c < 16 with the arithmetic of the 8-bit path; a row's distance is the fp32 sum of lut[s][code_s] over
 * s = 0..m-1 in order; the k smallest (distance, id) pairs, ties to the lower id, padded with {+inf, -1}.
 * vk_host_pq4_train / vk_host_pq4_encode (include/vk_host.h) build such codebooks and codes. The index's device
 * copy interleaves the bytes in 16-byte words (32 sub-codes each) and keeps rows in id order; vk_index_get_codes
 * returns the packed bytes. vk_distances, vk_compute_lut_device and vk_index_save reject 4-bit indexes
 * (VK_ERR_UNSUPPORTED). */
int vk_index_create_pq4(int device, const float* centroids, int m, int dsub, const uint8_t* codes, int64_t n,
                        int64_t id_base, vk_index_t** out);

/* Bits per sub-code of an index: 8 or 4. */
int vk_index_bits(const vk_index_t* index, int* nbits);

/* Same, with the row-major codes already in DEVICE memory of `device` (e.g. produced by vk_encode_device). */
int vk_index_create_from_device(int device, const float* centroids, int m, int dsub, const uint8_t* d_codes,
                                int64_t n, int64_t id_base, vk_index_t** out);

/* Synthetic code database generated directly on the device (BASELINE configs 3/4): rows
 * [row_first, row_first + n) of the generator `vk_gen_codes_host` (veckern_b200 host library) defines. cdf is
 * the host-computed [clusters][m][256] uint32 categorical table. Ids are id_base + (row - row_first). */
int vk_index_create_generated(int device, const float* centroids, int m, int dsub, uint64_t seed,
                              const uint32_t* cdf, int clusters, int64_t row_first, int64_t n, int64_t id_base,
                              vk_index_t** out);

/* Replaces ~PQSearcher. */
int vk_index_destroy(vk_index_t* index);

/* Basic facts about an index: n, m, dsub, id_base, device. Any pointer may be NULL. */
int vk_index_info(const vk_index_t* index, int64_t* n, int* m, int* dsub, int64_t* id_base, int* device);

/* Copies the index's row-major codes for rows [first, first + count) back to host memory (tests, tools). */
int vk_index_get_codes(const vk_index_t* index, int64_t first, int64_t count, uint8_t* out);

/* Single-process multi-GPU search (no counterpart in the reference, which runs on one device). The database is
 * split into ndev contiguous row shards, shard g on devices[g] (a device may be listed more than once) with global
 * ids; vk_multi_search runs every shard on its own stream, gathers the per-shard lists on devices[0] over the
 * device interconnect and merges them there: results are identical to one index over all rows. Timings:
 * scan_ms = slowest shard (LUT + scan + its lists), select_ms = cross-shard merge, transfer_ms = the rest. */
typedef struct vk_multi vk_multi_t;
int vk_multi_create(int ndev, const int* devices, const float* centroids, int m, int dsub, const uint8_t* codes,
                    int64_t n, vk_multi_t** out);
/* Each shard reads only its rows of a persisted index file (vk_index_load). */
int vk_multi_load(int ndev, const int* devices, const char* path, int verify, vk_multi_t** out);
int vk_multi_search(vk_multi_t* multi, const float* queries, int64_t nq, int k, const vk_tuning_t* tuning,
                    vk_neighbor_t* out, vk_timings_t* timings);
int vk_multi_info(const vk_multi_t* multi, int64_t* n, int* shards);
int vk_multi_destroy(vk_multi_t* multi);

/* Persisted index (no counterpart in the reference, whose io.cpp only reads TEXMEX vectors). vk_index_save writes
 * the index's centroids and its codes in row order to `path` (format in include/vk_host.h: header, centroids,
 * row-major codes, one CRC-32C per 2^20 rows). vk_index_load builds an index on `device` from rows
 * [row_first, row_first + count) of such a file (count < 0: to the end; id_base < 0: ids = file rows), reading
 * only that range, so each shard of a multi-GPU search loads its own rows; verify != 0 checks every checksum block
 * the range touches (VK_ERR_INVALID on a mismatch or a malformed file). */
int vk_index_save(const vk_index_t* index, const char* path);
int vk_index_load(int device, const char* path, int64_t row_first, int64_t count, int64_t id_base, int verify,
                  vk_index_t** out);

/* Lane placement of the device layout (no counterpart in the reference): out[j] = the row, relative to its window
 * of 64 positions, stored at position first + j, for j < count. The index stores the rows of every whole 64-row
 * window in an order chosen at build time to cut shared-memory bank conflicts of the LUT lookups; ids and results
 * are unaffected. first must be a multiple of 64 and first + count <= n rounded up to 128 (diagnostics, tests). */
int vk_index_get_placement(const vk_index_t* index, int64_t first, int64_t count, uint8_t* out);

/* Replaces PQSearcher::search (src/cuda/searcher.cu:466-520): HOST queries (nq x d fp32) in, HOST results
 * (nq x k vk_neighbor_t, ascending) out, 1 <= k <= min(128, n). Synchronous. timings/shape may be NULL.
 * `variant` only selects the reference's validation rules (m % 16 == 0 for variants 2, 6, 7, 8). */
int vk_search(vk_index_t* index, const float* queries, int64_t nq, int k, int variant, const vk_tuning_t* tuning,
              vk_neighbor_t* out, vk_timings_t* timings, vk_launch_shape_t* shape);

/* Device-resident search: DEVICE queries and results on the caller's CUDA stream (cudaStream_t passed as void*;
 * NULL = the default stream, as in the CUDA runtime). Asynchronous: vk_index_sync waits and collects the kernels'
 * status. One index's workspace serves one search at a time: searches on different streams must not overlap. */
int vk_search_device(vk_index_t* index, const float* d_queries, int64_t nq, int k, const vk_tuning_t* tuning,
                     vk_neighbor_t* d_out, void* stream);

/* Waits for the index's work on `stream` (NULL = the default stream) and reports any kernel-side error. */
int vk_index_sync(vk_index_t* index, void* stream);

/* Cooperative sharded search (no counterpart in the reference, which runs on one device). The shards of one
 * database (one index per GPU, ids offset by id_base) searched with the same queries share, while they scan, each
 * query's pruning bound: every shard's scan lowers the other shards' bounds with posted atomics into their memory
 * (over NVLink) and reads its own, so a small shard prunes with the bound of the whole database instead of its own.
 * A shard's lists then hold every pair of that shard that belongs to the merged top-k, and may miss others (padded
 * with {+inf, -1}): merge the shards' lists (vk_merge_topk_device) for the exact result, which equals one index
 * over all rows. Pairs are exchanged as (epoch, bound): all shards of a search pass the same epoch, and each new
 * search a larger one (>= 1); bounds of an older epoch are ignored. A shard's memory must outlive every search of
 * the others that uses it: synchronise all shards (e.g. a barrier after the last search) before destroying any.
 *   vk_coop_create      exchange array of nq_max queries on `device`
 *   vk_coop_ipc_handle  its VK_COOP_HANDLE_BYTES-byte handle (CUDA IPC handle, length, device), for shards in
 *                       other processes of this node
 *   vk_coop_attach_ipc  maps the other shards' arrays from their handles (the list may include its own)
 *   vk_coop_attach      the same for shards in this process (the list may include itself)
 * Shards on different GPUs need a link that carries atomics (NVLink); attaching fails with VK_ERR_UNSUPPORTED
 * otherwise. A search's nq may not exceed any attached shard's nq_max. */
#define VK_COOP_HANDLE_BYTES 80
typedef struct vk_coop vk_coop_t;
int vk_coop_create(int device, int64_t nq_max, vk_coop_t** out);
int vk_coop_ipc_handle(const vk_coop_t* coop, void* handle);
int vk_coop_attach_ipc(vk_coop_t* coop, int n, const void* handles);
int vk_coop_attach(vk_coop_t* coop, int n, vk_coop_t* const* coops);
int vk_coop_destroy(vk_coop_t* coop);
/* vk_search_device for one shard of a cooperative search (the pruned scan; with early_abandon = 0 the shard
 * neither reads nor lowers shared bounds). */
int vk_search_device_coop(vk_index_t* index, vk_coop_t* coop, uint32_t epoch, const float* d_queries, int64_t nq,
                          int k, const vk_tuning_t* tuning, vk_neighbor_t* d_out, void* stream);

/* Replaces PQSearcher::distances (src/cuda/searcher.cu:522-547): the full nq x n ADC matrix to HOST memory.
 * Rejected for the fused variants, as in the reference. */
int vk_distances(vk_index_t* index, const float* queries, int64_t nq, int variant, const vk_tuning_t* tuning,
                 float* out, vk_timings_t* timings);

/* Replaces lut_kernel (src/cuda/kernels.cuh:17-30) for direct use: lut[q][s][c] (nq x m x 256 fp32) in DEVICE
 * memory, computed on `stream` from DEVICE queries with the index's centroids. */
int vk_compute_lut_device(vk_index_t* index, const float* d_queries, int64_t nq, float* d_lut, void* stream);

/* Replaces select_kernel's role as the final reduction (src/cuda/kernels.cuh:179-202) and is the multi-GPU
 * merge: for each of nq queries, the k best of `lists` sorted candidate lists of k_in entries each, all in DEVICE
 * memory on `device`. Entry (q, list l, j) is at in[q * query_stride + l * list_stride + j]. Entries with
 * id < 0 are padding and are skipped. Output: nq x k ascending, padded with {+inf, -1}. */
int vk_merge_topk_device(int device, const vk_neighbor_t* d_in, int64_t nq, int lists, int k_in,
                         int64_t query_stride, int64_t list_stride, int k, vk_neighbor_t* d_out, void* stream);

/* Replaces rerank_exact (src/cpu/cpu_ref.cpp:66-77) on the device: for each of nq queries (DEVICE, nq x d fp32),
 * re-scores its r candidates (DEVICE, nq x r vk_neighbor_t; only the ids are read, ids < 0 are skipped) against
 * the DEVICE base vectors (n x d fp32, row = id) with the exact l2sq and keeps the k best (1 <= k <= 128),
 * ascending, padded with {+inf, -1}: identical to the reference's CPU re-rank. */
int vk_rerank_device(int device, const float* d_base, int64_t n, int d, const float* d_queries, int64_t nq,
                     const vk_neighbor_t* d_candidates, int r, int k, vk_neighbor_t* d_out, void* stream);

/* Bit-exact PQ encode on the device (nearest centroid per sub-space under the reference's l2sq, first minimum
 * wins; src/cpu/pq.cpp:11-22, 71-76): DEVICE x (n x d fp32) -> DEVICE codes (n x m). */
int vk_encode_device(int device, const float* centroids, int m, int dsub, const float* d_x, int64_t n,
                     uint8_t* d_codes, void* stream);

/* Replaces ProductQuantizer::train (src/cpu/pq.cpp:31-69) for a training set in DEVICE memory (n x d fp32,
 * n >= 256, d = m * dsub, dsub <= 128): the same std::mt19937_64 draws (one shuffle per sub-space, rng() % n per
 * empty cluster) and the same arithmetic (l2sq assignment, first minimum wins; sums in row order; sum / count),
 * so the HOST output `centroids` ([m][256][dsub] fp32) is bit-identical to the reference's. Synchronous. */
int vk_pq_train_device(int device, const float* d_x, int64_t n, int d, int m, int64_t iters, uint64_t seed,
                       float* centroids, void* stream);

/* Generates rows [row_first, row_first + n) of the synthetic code generator into DEVICE memory (row-major n x m);
 * the same integers as vk_gen_codes_host. */
int vk_gen_codes_device(int device, uint64_t seed, const uint32_t* cdf, int clusters, int m, int64_t row_first,
                        int64_t n, uint8_t* d_codes, void* stream);

/* IVF (inverted-file) search: the IVF partitioning the reference lists as a next step (README.md:219). Rows are
 * partitioned into nlist lists (list_of[i] in [0, nlist), e.g. the nearest of nlist coarse centroids:
 * vk_ivf_assign_device; vk_pq_train_device with m = 1 trains 256 such centroids); a search scans only the rows of
 * each query's nprobe nearest lists. Definition (restated on the CPU by oracle vko_ivf_search): the probed lists are
 * the nprobe smallest (l2sq(query, coarse[l]), l) pairs (the reference's exact l2sq over all d dimensions, ties to
 * the lower list), and the result is the k smallest (distance, id) pairs among their rows, distances being the flat
 * search's (the same fp32 LUT summed in sub-space order): the flat search restricted to those rows, bit for bit.
 * PQ codes are not residuals, so one LUT per query serves every list. m = 16 or 32, fp32 LUTs, 1 <= k <= 128,
 * 1 <= nprobe <= min(128, nlist); a query whose lists hold fewer than k rows is padded with {+inf, -1}.
 *   vk_ivf_create          builds the index from HOST centroids, codes (n x m, row-major), coarse centroids
 *                          (nlist x d) and list_of (n)
 *   vk_ivf_search          HOST queries and results, synchronous (timings: transfer_ms and, in scan_ms, the
 *                          whole device search)
 *   vk_ivf_search_device   DEVICE queries and results on `stream`, asynchronous (vk_ivf_sync reads the status)
 *   vk_ivf_assign_device   nearest coarse centroid of each DEVICE row (exact l2sq, first minimum wins) */
typedef struct vk_ivf vk_ivf_t;
int vk_ivf_create(int device, const float* centroids, int m, int dsub, const uint8_t* codes, int64_t n,
                  const float* coarse, int nlist, const int32_t* list_of, vk_ivf_t** out);
int vk_ivf_destroy(vk_ivf_t* ivf);
int vk_ivf_info(const vk_ivf_t* ivf, int64_t* n, int* nlist, int64_t* slots);
int vk_ivf_search(vk_ivf_t* ivf, const float* queries, int64_t nq, int k, int nprobe, const vk_tuning_t* tuning,
                  vk_neighbor_t* out, vk_timings_t* timings);
int vk_ivf_search_device(vk_ivf_t* ivf, const float* d_queries, int64_t nq, int k, int nprobe,
                         const vk_tuning_t* tuning, vk_neighbor_t* d_out, void* stream);
int vk_ivf_sync(vk_ivf_t* ivf, void* stream);
int vk_ivf_assign_device(int device, const float* d_x, int64_t n, int d, const float* d_coarse, int nlist,
                         int32_t* d_list_of, void* stream);

/* No counterpart in the reference. A device-resident search that allocates nothing, for callers that must not
 * call cudaMalloc or cudaFree: code running where an allocation would synchronise the device and stall other
 * streams (latency-bound serving threads), or under an allocator the process has handed all memory to.
 * Same inputs and output as vk_search_device (the index built beforehand, DEVICE queries, DEVICE results), but
 * the search's working memory (LUTs, per-chunk lists, pruning state) lives in one fixed array of
 * VK_NOALLOC_SCRATCH_BYTES compiled into the library, which every GPU that loads the library holds until the
 * process exits. Calls needing more than that (about nq * m KiB of LUTs plus nq * k * (chunks + 2) * 8 bytes of
 * lists) are rejected with VK_ERR_INVALID; split the queries. The array's device address is looked up when the
 * first index is created on a device, not during a search. Make one warm-up call per index and per search shape
 * (k, tuning, query count class) before serving: the CUDA runtime loads a kernel's code on its first launch (lazy
 * module loading, the CUDA 12 default), and that load may allocate device memory. Runs on `stream` (NULL = the
 * default stream) and is synchronous: it returns when the results are written and the kernels' status is read.
 * All calls share the one array, which keeps the previous call's contents (each call resets what must start at
 * zero): calls that overlap on the GPU (other host threads, other streams) race and must not be made. */
#define VK_NOALLOC_SCRATCH_BYTES ((size_t)32 << 20)
int vk_search_noalloc(vk_index_t* index, const float* d_queries, int64_t nq, int k, const vk_tuning_t* tuning,
                      vk_neighbor_t* d_out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* VK_ABI_H */
