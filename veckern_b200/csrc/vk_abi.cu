// VecKern-B200 C ABI implementation: index ownership, launch planning for the B200's 148 SMs, query batching,
// per-stage CUDA-event timing, and the error convention (int status + vk_last_error).
//
// Reference behaviour this file reproduces (shivdeshpande/VecKern):
//   PQSearcher ctor      src/cuda/searcher.cu:427-444   (copy centroids + codes to the device once)
//   search               src/cuda/searcher.cu:466-520   (k in [1, min(128, n)], batches, stage timings)
//   distances            src/cuda/searcher.cu:522-547   (nq x n matrix, 512 MB batches, unfused variants only)
//   validation           src/cuda/searcher.cu:243-249, 450-460
//   device_info          src/cuda/searcher.cu:143-156
#include <algorithm>
#include <cstdlib>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <limits>
#include <map>
#include <mutex>
#include <numeric>
#include <random>
#include <vector>
#include <string>

#include "../../include/vk_abi.h"
#include "aux_kernels.cuh"
#include "ivf_kernels.cuh"
#include "host/index_file.h"
#include "kernels.cuh"
#include "scan_dispatch.cuh"

namespace {

thread_local std::string g_error;

int fail(int code, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_error = buf;
    return code;
}

#define VK_TRY_CUDA(call)                                                                                  \
    do {                                                                                                   \
        const cudaError_t e_ = (call);                                                                     \
        if (e_ != cudaSuccess) return fail(e_ == cudaErrorMemoryAllocation ? VK_ERR_NOMEM : VK_ERR_CUDA, \
                                           "%s failed: %s", #call, cudaGetErrorString(e_));                \
    } while (0)

#define VK_TRY(call)                    \
    do {                                \
        const int r_ = (call);          \
        if (r_ != VK_OK) return r_;     \
    } while (0)

// Restores the caller's current device on scope exit.
struct DeviceGuard {
    int prev = -1;
    cudaError_t err = cudaSuccess;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) err = cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

template <typename T>
struct DevBuf {
    T* ptr = nullptr;
    size_t cap = 0;  // elements
    ~DevBuf() { release(); }
    void release() {
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        cap = 0;
    }
    // Grows (never shrinks), like the reference's DeviceBuffer::ensure (src/cuda/searcher.cu:31-37).
    int ensure(size_t count) {
        if (count <= cap) return VK_OK;
        release();
        const cudaError_t e = cudaMalloc(&ptr, std::max<size_t>(count, 1) * sizeof(T));
        if (e != cudaSuccess) {
            ptr = nullptr;
            return fail(VK_ERR_NOMEM, "cudaMalloc of %zu bytes failed: %s", count * sizeof(T), cudaGetErrorString(e));
        }
        cap = count;
        return VK_OK;
    }
};

constexpr size_t kL2WindowBytes = size_t(80) << 20;  // L2 share for one window's LUTs plus two chunks' codes
constexpr int64_t kMaxRowsPerChunk = 1 << 20;       // L2 locality: a chunk's codes stay well inside the 126 MB L2
constexpr size_t kLutBudgetBytes = size_t(1) << 30;  // LUT buffer cap per query batch
constexpr size_t kDistanceBudgetBytes = size_t(512) << 20;  // distances(): the reference's 512 MB cap
constexpr int kStagesMax = 4;

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

bool is_fused_variant(int v) { return v >= VK_VARIANT_FUSED && v <= VK_VARIANT_FUSED_WARP; }
bool needs_m16(int v) {
    return v == VK_VARIANT_SHARED_LUT_VEC || v == VK_VARIANT_FUSED_VEC || v == VK_VARIANT_FUSED_VEC_MQ ||
           v == VK_VARIANT_FUSED_WARP;
}
const char* variant_name(int v) {
    static const char* names[] = {"v0_global_lut", "v1_shared_lut", "v2_shared_lut_vec", "v3_interleaved",
                                  "v4_fused",      "v5_fused_reg",  "v6_fused_vec",      "v7_fused_vec_mq",
                                  "v8_fused_warp"};
    return v >= 0 && v <= 8 ? names[v] : "unknown";
}

const void* scan_kernel_ptr(int Q, int mt, int ilp, int s, bool prune, bool h16) {
    if (h16) {
        switch (Q) {
            case 4: return vk::scan_kernel_h16_for<4>(mt, ilp, s, prune);
            case 8: return vk::scan_kernel_h16_for<8>(mt, ilp, s, prune);
            default: return nullptr;
        }
    }
    switch (Q) {
        case 1: return vk::scan_kernel_for<1>(mt, ilp, s, prune);
        case 2: return vk::scan_kernel_for<2>(mt, ilp, s, prune);
        case 4: return vk::scan_kernel_for<4>(mt, ilp, s, prune);
        case 8: return vk::scan_kernel_for<8>(mt, ilp, s, prune);
        default: return nullptr;
    }
}

const void* lut_max_kernel_ptr(int Q) {
    return Q == 4 ? reinterpret_cast<const void*>(&vk::lut_max_kernel<4>)
                  : reinterpret_cast<const void*>(&vk::lut_max_kernel<8>);
}

const void* lut_h16_kernel_ptr(int Q) {
    return Q == 4 ? reinterpret_cast<const void*>(&vk::lut_h16_kernel<4>)
                  : reinterpret_cast<const void*>(&vk::lut_h16_kernel<8>);
}

const void* lut_kernel_ptr(int Q) {
    switch (Q) {
        case 1: return reinterpret_cast<const void*>(&vk::lut_kernel<1>);
        case 2: return reinterpret_cast<const void*>(&vk::lut_kernel<2>);
        case 4: return reinterpret_cast<const void*>(&vk::lut_kernel<4>);
        default: return reinterpret_cast<const void*>(&vk::lut_kernel<8>);
    }
}

const void* merge_kernel_ptr(int s) {
    switch (s) {
        case 1: return reinterpret_cast<const void*>(&vk::merge_kernel<1>);
        case 2: return reinterpret_cast<const void*>(&vk::merge_kernel<2>);
        default: return reinterpret_cast<const void*>(&vk::merge_kernel<4>);
    }
}

const void* merge_wide_kernel_ptr(int s) {
    switch (s) {
        case 1: return reinterpret_cast<const void*>(&vk::merge_wide_kernel<1>);
        case 2: return reinterpret_cast<const void*>(&vk::merge_wide_kernel<2>);
        default: return reinterpret_cast<const void*>(&vk::merge_wide_kernel<4>);
    }
}

int s_for_k(int k) { return k <= 32 ? 1 : k <= 64 ? 2 : 4; }

}  // namespace

// ------------------------------------------------------------------------------------------------ index
struct vk_index {
    int device = 0;
    int m = 0, dsub = 0, W = 0;
    int nbits = 8;  // bits per sub-code: 8 (256 centroids per sub-space) or 4 (16 centroids, two codes per byte)
    int mb = 0;     // code bytes per row: m (8-bit) or ceil(m / 2) (4-bit)
    int64_t n = 0, n_pad = 0, id_base = 0;
    float* centroids = nullptr;
    uint4* codes = nullptr;
    uint8_t* perm = nullptr;  // [n_pad] lane placement (place_rows_kernel)
    cudaStream_t stream = nullptr;
    DevBuf<float> queries, lut, dists;
    DevBuf<int2> part, out;
    DevBuf<uint32_t> bound;  // per-query running bound of the k-th distance (pruned scan)
    DevBuf<int2> glist;      // per-query global best-k list (pruned scan)
    DevBuf<int> glock;       // per-query try-locks of glist
    DevBuf<uint32_t> qmax;   // per-query largest LUT entry (half-precision LUTs)
    DevBuf<int> qexp;        // per-query scale exponent (half-precision LUTs)
    int* flags = nullptr;  // [0] work counter, [1] kernel status word
    cudaEvent_t ev[6] = {};
    int sm_count = 0, smem_optin = 0, clock_khz = 0;
    long long wait_budget = 0;
    // Launch set-up already done on this device: dynamic shared memory granted per kernel, and resident blocks per
    // SM per (kernel, shared memory, threads); saves two driver calls per search.
    mutable std::map<const void*, uint32_t> smem_granted;
    mutable std::map<std::pair<const void*, uint64_t>, int> resident_per_sm;

    ~vk_index() {
        DeviceGuard g(device);
        for (auto& e : ev)
            if (e) cudaEventDestroy(e);
        if (stream) cudaStreamDestroy(stream);
        if (centroids) cudaFree(centroids);
        if (codes) cudaFree(codes);
        if (perm) cudaFree(perm);
        if (flags) cudaFree(flags);
    }
};

namespace {

struct Plan {
    int Q = 1, ilp = 1, stages = kStagesMax, S = 1, mt = 0, merge_slots = 1, group_window = 1;
    bool prune = false, h16 = false, ivf = false, p4 = false;
    int threads = 0, blocks_per_sm = 0, grid = 0;
    int groups = 0, chunks = 0;
    int64_t chunk_len = 0, first_len = 0;
    uint32_t smem = 0;
    const void* fn = nullptr;
};

// Chooses Q (the requested queries per block, halved until the LUTs fit, and never more than the batch needs),
// ILP and the ring depth, then the chunk count with a wave model over the occupancy API's resident blocks:
// time ~ ceil(items / resident) * (rows per chunk + a LUT-load overhead), minimised over the chunk count.
// ivf: a plan for IVF work items (Q in {4, 8}, m in {16, 32}, ILP <= 2, fp32 LUTs; no chunking: the items are the
// (list, query batch) pairs the IVF planning kernels produce).
int plan_scan(const vk_index* ix, int64_t nq, int k, const vk_tuning_t& t, Plan& p, bool ivf = false) {
    p.S = s_for_k(k);
    p.mt = (ix->m == 16 || ix->m == 32 || ix->m == 64) ? ix->m : 0;
    // Exact early abandoning: specialised for m in {16, 32, 64}; its compaction queue holds 1 or 2 row groups.
    p.prune = t.early_abandon != 0 && p.mt != 0;
    p.h16 = t.lut_precision == VK_LUT_F16;
    p.ivf = ivf;
    p.p4 = ix->nbits == 4;
    if (p.p4 && (p.h16 || ivf))
        return fail(VK_ERR_UNSUPPORTED, "4-bit PQ indexes are searched with fp32 LUTs and without IVF lists");
    if (p.h16 && p.mt == 0)
        return fail(VK_ERR_UNSUPPORTED, "half-precision LUTs need m = 16, 32 or 64 (m = %d)", ix->m);
    if (ivf && (p.h16 || (ix->m != 16 && ix->m != 32)))
        return fail(VK_ERR_UNSUPPORTED, "IVF search supports m = 16 or 32 with fp32 LUTs (m = %d)", ix->m);
    int Q = t.queries_per_block;
    int64_t need = 1;
    while (need < nq && need < 8) need *= 2;
    Q = (int)std::min<int64_t>(Q, need);
    if (p.h16) Q = Q >= 8 ? 8 : 4;  // half LUT entries hold 4 or 8 queries
    if (ivf) Q = Q >= 8 ? 8 : 4;    // IVF items hold 4 or 8 queries
    if (p.p4) Q = Q >= 8 ? 8 : 4;   // 4-bit kernels are built for 4 or 8 queries
    const int ilp_req =
        (p.prune || p.h16 || ivf || p.p4) ? std::min(t.vectors_per_step, 2) : t.vectors_per_step;
    p.ilp = ilp_req;
    p.stages = kStagesMax;
    // warps per block as the kernel is instantiated (vk::scan_warps); the generic-m kernel uses its table size
    auto warps = [&](int q) { return vk::scan_warps(q, p.mt, p.h16, p.p4); };
    auto slots = [&](int q) { return (uint32_t)q * warps(q) * k * 8u <= 16384u ? q : 1; };  // parallel merges
    auto fits = [&](int q, int ilp, int st) {
        return vk::scan_smem_plan(q, ix->m, ix->W, ilp, warps(q), st, k, p.prune, slots(q), p.h16, p.ivf, p.p4).total <=
               (uint32_t)ix->smem_optin;
    };
    for (;;) {
        if (fits(Q, p.ilp, p.stages)) break;
        if (p.stages > 2) { --p.stages; continue; }
        if (p.ilp > 1) { p.ilp /= 2; p.stages = kStagesMax; continue; }
        if (Q > (p.h16 || p.ivf || p.p4 ? 4 : 1)) { Q /= 2; p.ilp = ilp_req; p.stages = kStagesMax; continue; }
        return fail(VK_ERR_INVALID, "LUT does not fit in shared memory (m = %d needs %u bytes, device allows %d)",
                    ix->m, vk::scan_smem_plan(p.h16 ? 4 : 1, ix->m, ix->W, 1, warps(p.h16 ? 4 : 1), 2, k, p.prune, 1,
                                              p.h16).total,
                    ix->smem_optin);
    }
    p.Q = Q;
    const int nw = warps(Q);
    p.threads = nw * 32;
    if (ivf)
        p.fn = Q == 8 ? vk::scan_kernel_ivf_for<8>(p.mt, p.ilp, p.S, p.prune)
                      : vk::scan_kernel_ivf_for<4>(p.mt, p.ilp, p.S, p.prune);
    else if (p.p4)
        p.fn = Q == 8 ? vk::scan_kernel_p4_for<8>(p.mt, p.ilp, p.S, p.prune)
                      : vk::scan_kernel_p4_for<4>(p.mt, p.ilp, p.S, p.prune);
    else
        p.fn = scan_kernel_ptr(Q, p.mt, p.ilp, p.S, p.prune, p.h16);
    if (!p.fn) return fail(VK_ERR_UNSUPPORTED, "no scan kernel for Q=%d m=%d ilp=%d", Q, ix->m, p.ilp);
    p.merge_slots = slots(Q);
    p.smem = vk::scan_smem_plan(Q, ix->m, ix->W, p.ilp, nw, p.stages, k, p.prune, p.merge_slots, p.h16, p.ivf, p.p4)
                 .total;
    auto granted = ix->smem_granted.find(p.fn);
    if (granted == ix->smem_granted.end() || granted->second < p.smem) {
        VK_TRY_CUDA(cudaFuncSetAttribute(p.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem));
        ix->smem_granted[p.fn] = p.smem;
    }
    const auto occ_key = std::make_pair(p.fn, ((uint64_t)p.smem << 16) | (uint64_t)p.threads);
    auto occ = ix->resident_per_sm.find(occ_key);
    int per_sm = 0;
    if (occ != ix->resident_per_sm.end()) {
        per_sm = occ->second;
    } else {
        VK_TRY_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, p.fn, p.threads, p.smem));
        ix->resident_per_sm[occ_key] = per_sm;
    }
    p.blocks_per_sm = std::max(per_sm, 1);
    const int64_t resident = (int64_t)p.blocks_per_sm * ix->sm_count;
    if (ivf) {  // persistent grid over the item table; the item count is known on the device only
        p.groups = 1;
        p.chunks = 1;
        p.grid = (int)resident;
        return VK_OK;
    }

    p.groups = (int)ceil_div(nq, Q);
    const int64_t tile_rows = 32 * p.ilp;
    const int64_t tiles = ix->n_pad / tile_rows;
    const int64_t max_chunks = std::max<int64_t>(1, tiles / (2 * nw));  // >= 2 tiles per warp per chunk
    // Chunk count: a wave model over the resident blocks, time ~ ceil(items / resident) * (rows per chunk + a
    // per-item overhead in rows of scan work), minimised over a range of chunk counts. The pruned scan tightens each
    // query's bound whenever one of its chunks completes, so its chunks stay between 16K and 64K rows (up to 48
    // chunks; more only when the L2 locality cap asks for it), and its per-item overhead is higher (list merge and
    // fold at every item end: about 2K rows of work, measured).
    const int64_t l2_chunks = ceil_div(ix->n_pad, kMaxRowsPerChunk);
    int64_t lo = l2_chunks, hi = l2_chunks + 8 * resident;
    double item_rows = 512.0;
    if (p.prune) {
        lo = std::max(l2_chunks, std::min<int64_t>(48, ceil_div(ix->n_pad, 65536)));
        hi = std::max(lo, std::min<int64_t>(48, ix->n_pad / 16384));
        hi = std::max(hi, ceil_div(resident, p.groups));  // few query groups: spread their rows over every SM
        item_rows = 2048.0;
    }
    lo = std::min(lo, max_chunks);
    hi = std::min(hi, max_chunks);
    int64_t chunks = lo;
    if (t.blocks_per_query > 0) {
        chunks = std::min<int64_t>(t.blocks_per_query, max_chunks);
        // the pruned m = 16 scan addresses a chunk's rows in 24 bits of its queue entries
        if (p.prune && vk::carry_queue(ix->m) && !p.p4)
            chunks = std::max<int64_t>(chunks, ceil_div(ix->n_pad, vk::CARRY_MAX_CHUNK_ROWS));
    } else {
        double best = 1e300;
        for (int64_t c = lo; c <= hi; ++c) {
            const double waves = (double)ceil_div((int64_t)p.groups * c, resident);
            const double cost = waves * ((double)ix->n_pad / c + item_rows);
            if (cost < best * 0.999) {
                best = cost;
                chunks = c;
            }
        }
    }
    p.chunk_len = ceil_div(tiles, chunks) * tile_rows;
    // Pruned scans with a planned chunk count start with a half-length chunk 0: the first wave of items runs
    // before any of a query's chunks has folded its list into the query's bound, so it is shortened
    // (measured 3-6 % faster at 250k-1M rows).
    p.first_len = p.chunk_len;
    if (p.prune && t.blocks_per_query <= 0)
        p.first_len = std::max<int64_t>(tile_rows, p.chunk_len / 2 / tile_rows * tile_rows);
    p.chunks = (int)(1 + ceil_div(std::max<int64_t>(0, ix->n_pad - p.first_len), p.chunk_len));
    // Item order: chunk-major over all query groups while their LUTs and two chunks of codes fit in the L2 share;
    // otherwise window by window of as many groups as fit (each chunk's codes then come from HBM once per window
    // instead of once per group whose LUT was evicted).
    {
        const size_t lut_group = (size_t)p.Q * ix->m * (p.p4 ? vk::KSUB4 : vk::KSUB) * (p.h16 ? 2 : 4);
        const size_t chunk_bytes = (size_t)p.chunk_len * ((size_t)ix->W * 16 + 1);
        const size_t room = kL2WindowBytes > 2 * chunk_bytes ? kL2WindowBytes - 2 * chunk_bytes : 0;
        p.group_window = (size_t)p.groups * lut_group <= room
                             ? p.groups
                             : (int)std::max<size_t>(1, std::min<size_t>(room / lut_group, (size_t)p.groups));
    }
    const int64_t items = (int64_t)p.groups * p.chunks;
    if (items > std::numeric_limits<int>::max() / 2)
        return fail(VK_ERR_UNSUPPORTED, "too many work items (%lld); search fewer queries per call", (long long)items);
    p.grid = (int)std::min<int64_t>(items, resident);
    return VK_OK;
}

int validate_tuning(const vk_tuning_t* t) {
    if (!t) return VK_OK;
    if (!(t->scan_threads >= 32 && t->scan_threads <= 1024 && t->scan_threads % 32 == 0))
        return fail(VK_ERR_INVALID, "scan_threads must be a multiple of 32 in [32, 1024]");
    if (t->blocks_per_query < 0) return fail(VK_ERR_INVALID, "blocks_per_query must be >= 0");
    if (!(t->queries_per_block == 1 || t->queries_per_block == 2 || t->queries_per_block == 4 ||
          t->queries_per_block == 8))
        return fail(VK_ERR_INVALID, "queries_per_block must be 1, 2, 4 or 8");
    if (!(t->vectors_per_step == 1 || t->vectors_per_step == 2 || t->vectors_per_step == 4))
        return fail(VK_ERR_INVALID, "vectors_per_step must be 1, 2 or 4");
    if (t->early_abandon != 0 && t->early_abandon != 1) return fail(VK_ERR_INVALID, "early_abandon must be 0 or 1");
    if (t->lut_precision != VK_LUT_F32 && t->lut_precision != VK_LUT_F16)
        return fail(VK_ERR_INVALID, "lut_precision must be VK_LUT_F32 (0) or VK_LUT_F16 (1)");
    return VK_OK;
}

int check_variant(const vk_index* ix, int variant) {
    if (variant < 0 || variant > 8) return fail(VK_ERR_INVALID, "unknown scan variant %d", variant);
    if (needs_m16(variant) && ix->m % 16 != 0)
        return fail(VK_ERR_INVALID, "%s requires m %% 16 == 0", variant_name(variant));
    if ((int64_t)ix->m * vk::KSUB * 4 > ix->smem_optin)
        return fail(VK_ERR_INVALID, "LUT does not fit in shared memory");
    return VK_OK;
}

// Device working memory of one search: from the index's buffers (run_search) or carved from the fixed array of
// vk_search_noalloc.
struct Workspace {
    void* lut = nullptr;        // groups x Q x m x 256 entries (fp32, or half for half-precision LUTs)
    int2* part = nullptr;       // [nq][chunks][k] per-item lists
    uint32_t* bound = nullptr;  // [nq] pruning bounds
    int2* glist = nullptr;      // [nq][k] pruning global lists
    int* glock = nullptr;       // [nq] try-locks
    int* flags = nullptr;       // [0] work counter, [1] status word
    uint32_t* qmax = nullptr;   // [nq] half LUTs: largest entry per query
    int* qexp = nullptr;        // [nq] half LUTs: scale exponent per query
    // cooperative sharded search (vk_search_device_coop): exchange arrays and the search's epoch
    unsigned long long* xb = nullptr;
    unsigned long long* xpeer[vk::COOP_MAX_PEERS] = {};
    int npeers = 0;
    uint32_t epoch = 0;
};

// Bytes each workspace array needs for a plan (the flags are not included).
struct WorkspaceBytes {
    size_t lut, part, bound, glist, glock, qmax, qexp;
};
WorkspaceBytes workspace_bytes(const vk_index* ix, int64_t nq, int k, const Plan& p) {
    WorkspaceBytes b;
    b.lut = (size_t)p.groups * p.Q * ix->m * (p.p4 ? vk::KSUB4 : vk::KSUB) * (p.h16 ? 2 : 4);
    b.part = (size_t)nq * p.chunks * k * sizeof(int2);
    b.bound = (size_t)nq * sizeof(uint32_t);
    b.glist = (size_t)nq * k * sizeof(int2);
    b.glock = (size_t)nq * sizeof(int);
    b.qmax = p.h16 ? (size_t)nq * sizeof(uint32_t) : 0;
    b.qexp = p.h16 ? (size_t)nq * sizeof(int) : 0;
    return b;
}

// Launches LUT (two passes for half LUTs) -> scan -> merge for one batch of device-resident queries into d_out
// (nq x k). Resets the work counter; the status word accumulates until it is read.
int launch_search(vk_index* ix, const float* d_queries, int64_t nq, int k, const Plan& p, const Workspace& w,
                  int2* d_out, cudaStream_t st, cudaEvent_t* marks) {
    // LUT
    {
        const size_t smem = (size_t)p.Q * ix->dsub * sizeof(float);
        const float* cen = ix->centroids;
        uint32_t* bound = p.prune ? w.bound : nullptr;
        int2* glist = w.glist;
        int* glock = w.glock;
        int m = ix->m, dsub = ix->dsub, kk = k;
        void* lut = w.lut;
        if (p.h16) {
            uint32_t* qmax = w.qmax;
            int* qexp = w.qexp;
            const void* fmax = lut_max_kernel_ptr(p.Q);
            const void* fh = lut_h16_kernel_ptr(p.Q);
            if (smem > 48 * 1024) {
                VK_TRY_CUDA(cudaFuncSetAttribute(fmax, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
                VK_TRY_CUDA(cudaFuncSetAttribute(fh, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            }
            VK_TRY_CUDA(cudaMemsetAsync(qmax, 0, (size_t)nq * sizeof(uint32_t), st));
            void* a0[] = {(void*)&cen, (void*)&d_queries, (void*)&nq, (void*)&m, (void*)&dsub, (void*)&qmax};
            VK_TRY_CUDA(cudaLaunchKernel(fmax, dim3(ix->m, p.groups), dim3(vk::KSUB), a0, smem, st));
            void* a1[] = {(void*)&cen,  (void*)&d_queries, (void*)&nq,    (void*)&m,     (void*)&dsub, (void*)&qmax,
                          (void*)&qexp, (void*)&lut,       (void*)&bound, (void*)&glist, (void*)&glock, (void*)&kk};
            VK_TRY_CUDA(cudaLaunchKernel(fh, dim3(ix->m, p.groups), dim3(vk::KSUB), a1, smem, st));
        } else if (p.p4) {  // 16 sub-spaces x 16 centroids per block; the group's query sub-vectors in shared memory
            const void* fn = p.Q == 8 ? reinterpret_cast<const void*>(&vk::lut4_kernel<8>)
                                      : reinterpret_cast<const void*>(&vk::lut4_kernel<4>);
            const size_t smem4 = (size_t)p.Q * 16 * ix->dsub * sizeof(float);
            if (smem4 > 48 * 1024)
                VK_TRY_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem4));
            float* lutf = static_cast<float*>(lut);
            void* args[] = {(void*)&cen, (void*)&d_queries, (void*)&nq, (void*)&m, (void*)&dsub, (void*)&lutf,
                            (void*)&bound, (void*)&glist, (void*)&glock, (void*)&kk};
            VK_TRY_CUDA(cudaLaunchKernel(fn, dim3((unsigned)ceil_div(ix->m, 16), p.groups), dim3(256), args, smem4, st));
        } else {
            const void* fn = lut_kernel_ptr(p.Q);
            if (smem > 48 * 1024)
                VK_TRY_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            void* args[] = {(void*)&cen, (void*)&d_queries, (void*)&nq, (void*)&m, (void*)&dsub, (void*)&lut,
                            (void*)&bound, (void*)&glist, (void*)&glock, (void*)&kk};
            VK_TRY_CUDA(cudaLaunchKernel(fn, dim3(ix->m, p.groups), dim3(vk::KSUB), args, smem, st));
        }
    }
    if (marks) VK_TRY_CUDA(cudaEventRecord(marks[0], st));
    // fused scan + top-k
    {
        VK_TRY_CUDA(cudaMemsetAsync(w.flags, 0, sizeof(int), st));
        vk::ScanArgs a{};
        a.codes = ix->codes;
        a.perm = ix->perm;
        a.lut = static_cast<const float*>(w.lut);
        a.part = w.part;
        a.work_counter = w.flags;
        a.status = w.flags + 1;
        a.bound = w.bound;
        a.glist = w.glist;
        a.glock = w.glock;
        a.n = ix->n;
        a.n_pad = ix->n_pad;
        a.chunk_len = p.chunk_len;
        a.first_len = p.first_len;
        a.id_base = ix->id_base;
        a.m = ix->m;
        a.W = ix->W;
        a.nq = (int)nq;
        a.groups = p.groups;
        a.chunks = p.chunks;
        a.group_window = p.group_window;
        a.k = k;
        a.stages = p.stages;
        a.merge_slots = p.merge_slots;
        a.wait_budget = ix->wait_budget;
        a.xb = w.xb;
        for (int i = 0; i < vk::COOP_MAX_PEERS; ++i) a.xpeer[i] = w.xpeer[i];
        a.npeers = w.npeers;
        a.epoch = w.epoch;
        void* args[] = {(void*)&a};
        VK_TRY_CUDA(cudaLaunchKernel(p.fn, dim3(p.grid), dim3(p.threads), args, p.smem, st));
    }
    if (marks) VK_TRY_CUDA(cudaEventRecord(marks[1], st));
    // merge of the per-chunk partial lists: one warp per query, or, when there are fewer queries than SMs and many
    // lists, one 8-warp block per query; half LUTs are scaled back to distances here
    {
        const bool wide = nq <= ix->sm_count && (int64_t)p.chunks * k >= 256;
        const void* fn = wide ? merge_wide_kernel_ptr(p.S) : merge_kernel_ptr(p.S);
        const int2* in = w.part;
        const int* qexp = p.h16 ? w.qexp : nullptr;
        int lists = p.chunks, k_in = k, kk = k;
        int64_t qstride = (int64_t)p.chunks * k, lstride = k;
        void* args[] = {(void*)&in, (void*)&nq, (void*)&lists, (void*)&k_in, (void*)&qstride, (void*)&lstride,
                        (void*)&kk, (void*)&d_out, (void*)&qexp};
        if (wide)
            VK_TRY_CUDA(cudaLaunchKernel(fn, dim3((unsigned)nq), dim3(256), args, 0, st));
        else
            VK_TRY_CUDA(cudaLaunchKernel(fn, dim3((unsigned)ceil_div(nq, 4)), dim3(128), args, 0, st));
    }
    return VK_OK;
}

// One batch of device-resident queries into d_out (nq x k), with the index's own (growing) buffers; `coop`
// (optional) carries a cooperative search's exchange arrays and epoch.
int run_search(vk_index* ix, const float* d_queries, int64_t nq, int k, const vk_tuning_t& t, int2* d_out,
               cudaStream_t st, vk_launch_shape_t* shape, cudaEvent_t* marks, const Workspace* coop = nullptr) {
    Plan p;
    VK_TRY(plan_scan(ix, nq, k, t, p));
    const WorkspaceBytes b = workspace_bytes(ix, nq, k, p);
    VK_TRY(ix->lut.ensure((b.lut + sizeof(float) - 1) / sizeof(float)));
    VK_TRY(ix->part.ensure(b.part / sizeof(int2)));
    VK_TRY(ix->bound.ensure(b.bound / sizeof(uint32_t)));
    VK_TRY(ix->glist.ensure(b.glist / sizeof(int2)));
    VK_TRY(ix->glock.ensure(b.glock / sizeof(int)));
    if (p.h16) {
        VK_TRY(ix->qmax.ensure(b.qmax / sizeof(uint32_t)));
        VK_TRY(ix->qexp.ensure(b.qexp / sizeof(int)));
    }
    Workspace w;
    w.lut = ix->lut.ptr;
    w.part = ix->part.ptr;
    w.bound = ix->bound.ptr;
    w.glist = ix->glist.ptr;
    w.glock = ix->glock.ptr;
    w.flags = ix->flags;
    w.qmax = ix->qmax.ptr;
    w.qexp = ix->qexp.ptr;
    if (coop) {
        w.xb = coop->xb;
        for (int i = 0; i < vk::COOP_MAX_PEERS; ++i) w.xpeer[i] = coop->xpeer[i];
        w.npeers = coop->npeers;
        w.epoch = coop->epoch;
    }
    VK_TRY(launch_search(ix, d_queries, nq, k, p, w, d_out, st, marks));
    if (shape) {
        shape->threads = p.threads;
        shape->blocks_x = p.chunks;
        shape->grid_y = p.groups;
        shape->queries_per_block = p.Q;
        shape->vectors_per_step = p.ilp;
        shape->blocks_per_sm = p.blocks_per_sm;
        shape->waves = (double)p.groups * p.chunks / ((double)p.blocks_per_sm * ix->sm_count);
    }
    return VK_OK;
}

int status_error(int status) {
    if (status & vk::ERR_DRAIN_TIMEOUT)
        return fail(VK_ERR_DEVICE,
                    "kernel reported status 0x%x: a bounded wait ran out and the kernel could not confirm that its "
                    "own copies had finished; treat this device's CUDA context as unusable",
                    status);
    return fail(VK_ERR_DEVICE, "kernel reported status 0x%x (a bounded wait ran out)", status);
}

int read_status(vk_index* ix, cudaStream_t st) {
    int status = 0;
    VK_TRY_CUDA(cudaMemcpyAsync(&status, ix->flags + 1, sizeof(int), cudaMemcpyDeviceToHost, st));
    VK_TRY_CUDA(cudaStreamSynchronize(st));
    if (status != 0) {
        VK_TRY_CUDA(cudaMemsetAsync(ix->flags + 1, 0, sizeof(int), st));
        VK_TRY_CUDA(cudaStreamSynchronize(st));
        return status_error(status);
    }
    return VK_OK;
}

int64_t max_query_batch(const vk_index* ix) {
    // grid.y of the LUT and distance kernels stays below 65536 and the LUT buffer within its budget
    const int64_t by_lut = std::max<int64_t>(8, (int64_t)(kLutBudgetBytes / ((size_t)ix->m * vk::KSUB * 4)));
    return std::min<int64_t>(by_lut, 65528) / 8 * 8;
}

// ------------------------------------------------------------------------------------------------ no allocation
// Working memory of vk_search_noalloc: one fixed array in the library's device image instead of the index's
// cudaMalloc'd buffers. Host code cannot use the array's name as a device address (in host code it names a
// host-side stand-in); the address is looked up per device with cudaGetSymbolAddress, the device current, when the
// first index is created on that device, and cached. Nothing on vk_search_noalloc's path calls cudaMalloc, cudaFree
// or any allocating routine.
static __device__ __align__(256) unsigned char g_noalloc_scratch[VK_NOALLOC_SCRATCH_BYTES];

std::mutex g_noalloc_mutex;
constexpr int kNoAllocMaxDevices = 64;
unsigned char* g_noalloc_addr[kNoAllocMaxDevices] = {};

// The array's device address on `device`, which must be the current device.
int noalloc_scratch_address(int device, unsigned char** out) {
    if (device < 0 || device >= kNoAllocMaxDevices) return fail(VK_ERR_UNSUPPORTED, "device %d out of range", device);
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (!g_noalloc_addr[device]) {
        void* addr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&addr, g_noalloc_scratch);
        if (e != cudaSuccess)
            return fail(VK_ERR_CUDA, "cudaGetSymbolAddress(scratch) on device %d failed: %s", device, cudaGetErrorString(e));
        g_noalloc_addr[device] = static_cast<unsigned char*>(addr);
    }
    *out = g_noalloc_addr[device];
    return VK_OK;
}

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

int create_common(int device, const float* centroids, int m, int dsub, int64_t n, int64_t id_base,
                  vk_index** out, vk_index*& ix, int nbits = 8) {
    if (!out) return fail(VK_ERR_INVALID, "out must not be NULL");
    *out = nullptr;
    if (!centroids) return fail(VK_ERR_INVALID, "centroids must not be NULL");
    if (m <= 0 || dsub <= 0) return fail(VK_ERR_INVALID, "m and dsub must be positive");
    if (n <= 0 || n >= (int64_t)std::numeric_limits<int>::max())
        return fail(VK_ERR_INVALID, "n must fit in int32 ids");
    if (id_base < 0 || id_base + n > (int64_t)std::numeric_limits<int>::max())
        return fail(VK_ERR_INVALID, "id_base + n must fit in int32 ids");
    int count = 0;
    VK_TRY_CUDA(cudaGetDeviceCount(&count));
    if (device < 0 || device >= count) return fail(VK_ERR_INVALID, "device %d does not exist", device);
    ix = new vk_index();
    ix->device = device;
    ix->m = m;
    ix->dsub = dsub;
    ix->nbits = nbits;
    ix->mb = nbits == 4 ? (m + 1) / 2 : m;
    ix->W = (ix->mb + 15) / 16;
    ix->n = n;
    ix->n_pad = ceil_div(n, 128) * 128;
    ix->id_base = id_base;
    VK_TRY_CUDA(cudaDeviceGetAttribute(&ix->sm_count, cudaDevAttrMultiProcessorCount, device));
    VK_TRY_CUDA(cudaDeviceGetAttribute(&ix->smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
    VK_TRY_CUDA(cudaDeviceGetAttribute(&ix->clock_khz, cudaDevAttrClockRate, device));
    ix->wait_budget = (long long)std::max(ix->clock_khz, 1000000) * 1000LL * 2;  // about two seconds
    VK_TRY_CUDA(cudaStreamCreateWithFlags(&ix->stream, cudaStreamNonBlocking));
    for (auto& e : ix->ev) VK_TRY_CUDA(cudaEventCreate(&e));
    VK_TRY_CUDA(cudaMalloc(&ix->flags, 4 * sizeof(int)));
    VK_TRY_CUDA(cudaMemsetAsync(ix->flags, 0, 4 * sizeof(int), ix->stream));
    const size_t cbytes = (size_t)m * (nbits == 4 ? vk::KSUB4 : vk::KSUB) * dsub * sizeof(float);
    VK_TRY_CUDA(cudaMalloc(&ix->centroids, cbytes));
    VK_TRY_CUDA(cudaMemcpyAsync(ix->centroids, centroids, cbytes, cudaMemcpyHostToDevice, ix->stream));
    VK_TRY_CUDA(cudaMalloc(&ix->codes, (size_t)ix->n_pad * ix->W * sizeof(uint4)));
    VK_TRY_CUDA(cudaMemsetAsync(ix->codes, 0, (size_t)ix->n_pad * ix->W * sizeof(uint4), ix->stream));
    VK_TRY_CUDA(cudaMalloc(&ix->perm, (size_t)ix->n_pad));
    unsigned char* scratch = nullptr;  // vk_search_noalloc's array: its address is resolved here, not at a search
    VK_TRY(noalloc_scratch_address(device, &scratch));
    return VK_OK;
}

unsigned grid_for(int64_t total, int sm_count) {
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>(ceil_div(total, 256), (int64_t)sm_count * 16));
}

// Lane placement of the rows of every 64-row window (vk::place_rows_kernel), on the index stream after the codes
// are in place. The objective follows the LUT layout the default plan picks for this m: 16-byte entries (Q >= 4)
// up to m = 32, 8-byte entries (Q = 2) beyond; its weights follow the pruned scan's phase-A depths.
cudaError_t place_rows(vk_index* ix) {
    if (ix->nbits == 4) {  // 4-bit LUT fetches never conflict (one 128-byte table per query pair): rows stay in order
        vk::identity_perm_kernel<<<grid_for(ix->n_pad, ix->sm_count), 256, 0, ix->stream>>>(ix->perm, ix->n_pad);
        return cudaGetLastError();
    }
    constexpr int kSteps = 4096;
    constexpr uint64_t kKey = 0x6c616e6570696b73ull;
    const int mt = (ix->m == 16 || ix->m == 32 || ix->m == 64) ? ix->m : 0;
    const int first = mt ? vk::prune_first(mt) : 0, last = mt ? vk::prune_last(mt) : 0;
    const uint32_t smem = ix->W > 4 ? 0u : 4 * ((vk::place_warp_smem(ix->m, ix->W) + 15u) & ~15u);  // <= 33 KB
    const int64_t windows = ix->n_pad / vk::PLACE_WINDOW;
    const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(ceil_div(windows, 4), (int64_t)ix->sm_count * 16));
    if (ix->m <= 32)
        vk::place_rows_kernel<8><<<grid, 128, smem, ix->stream>>>(ix->codes, ix->n, ix->n_pad, ix->m, ix->W, ix->perm,
                                                                   first, last, kSteps, kKey);
    else
        vk::place_rows_kernel<16><<<grid, 128, smem, ix->stream>>>(ix->codes, ix->n, ix->n_pad, ix->m, ix->W,
                                                                    ix->perm, first, last, kSteps, kKey);
    return cudaGetLastError();
}

}  // namespace

// ------------------------------------------------------------------------------------------------ C ABI
extern "C" {

size_t vk_last_error(char* buf, size_t len) {
    if (buf && len > 0) {
        const size_t n = std::min(len - 1, g_error.size());
        std::memcpy(buf, g_error.data(), n);
        buf[n] = '\0';
    }
    return g_error.size();
}

void vk_tuning_default(vk_tuning_t* t) {
    if (!t) return;
    t->scan_threads = 256;
    t->blocks_per_query = 0;
    t->queries_per_block = 2;
    t->vectors_per_step = 4;
    t->early_abandon = 1;
    t->lut_precision = VK_LUT_F32;
}

int vk_tuning_validate(const vk_tuning_t* t) {
    if (!t) return fail(VK_ERR_INVALID, "tuning must not be NULL");
    return validate_tuning(t);
}

int vk_device_info(int device, vk_device_info_t* out) {
    if (!out) return fail(VK_ERR_INVALID, "out must not be NULL");
    cudaDeviceProp prop{};
    VK_TRY_CUDA(cudaGetDeviceProperties(&prop, device));
    std::memset(out, 0, sizeof(*out));
    std::snprintf(out->name, sizeof(out->name), "%s", prop.name);
    int mem_khz = 0, bus = 0, smem = 0, clk = 0;
    VK_TRY_CUDA(cudaDeviceGetAttribute(&out->sm_count, cudaDevAttrMultiProcessorCount, device));
    VK_TRY_CUDA(cudaDeviceGetAttribute(&mem_khz, cudaDevAttrMemoryClockRate, device));
    VK_TRY_CUDA(cudaDeviceGetAttribute(&bus, cudaDevAttrGlobalMemoryBusWidth, device));
    VK_TRY_CUDA(cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
    VK_TRY_CUDA(cudaDeviceGetAttribute(&clk, cudaDevAttrClockRate, device));
    out->peak_bandwidth_gbs = 2.0 * mem_khz * 1e3 * (bus / 8.0) / 1e9;
    out->max_smem_per_block = (size_t)smem;
    out->clock_mhz = clk / 1000;
    return VK_OK;
}

}  // extern "C"

namespace {
// vk_index_create and vk_index_create_pq4: row-major codes (mb bytes per row) from HOST memory.
int index_from_host(int device, const float* centroids, int m, int dsub, const uint8_t* codes, int64_t n,
                    int64_t id_base, int nbits, vk_index_t** out) {
    if (!codes) return fail(VK_ERR_INVALID, "codes must not be NULL");
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess) return fail(VK_ERR_CUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(guard.err));
    vk_index* ix = nullptr;
    int rc = create_common(device, centroids, m, dsub, n, id_base, out, ix, nbits);
    if (rc == VK_OK) {
        // Upload row-major codes in slices through one staging buffer and interleave each slice on the device.
        const int mb = ix->mb;
        const int64_t slice = std::min<int64_t>(ceil_div(n, 32) * 32, int64_t(1) << 22);
        uint8_t* staging = nullptr;
        cudaError_t e = cudaMalloc(&staging, (size_t)slice * mb);
        for (int64_t r0 = 0; e == cudaSuccess && r0 < n; r0 += slice) {
            const int64_t cnt = std::min(slice, n - r0);
            e = cudaMemcpyAsync(staging, codes + r0 * mb, (size_t)cnt * mb, cudaMemcpyHostToDevice, ix->stream);
            if (e == cudaSuccess) {
                vk::interleave_kernel<<<grid_for(ceil_div(cnt, 32) * 32 * ix->W, ix->sm_count), 256, 0, ix->stream>>>(
                    staging, r0, cnt, n, mb, ix->W, ix->codes);
                e = cudaGetLastError();
            }
            if (e == cudaSuccess) e = cudaStreamSynchronize(ix->stream);  // staging is reused
        }
        if (staging) cudaFree(staging);
        if (e == cudaSuccess) e = place_rows(ix);
        if (e != cudaSuccess) rc = fail(VK_ERR_CUDA, "code upload failed: %s", cudaGetErrorString(e));
    }
    if (rc == VK_OK) {
        const cudaError_t e = cudaStreamSynchronize(ix->stream);
        if (e != cudaSuccess) rc = fail(VK_ERR_CUDA, "index build failed: %s", cudaGetErrorString(e));
    }
    if (rc != VK_OK) {
        delete ix;
        return rc;
    }
    *out = ix;
    return VK_OK;
}
}  // namespace

extern "C" {

int vk_index_create(int device, const float* centroids, int m, int dsub, const uint8_t* codes, int64_t n,
                    int64_t id_base, vk_index_t** out) {
    return index_from_host(device, centroids, m, dsub, codes, n, id_base, 8, out);
}

int vk_index_create_pq4(int device, const float* centroids, int m, int dsub, const uint8_t* codes, int64_t n,
                        int64_t id_base, vk_index_t** out) {
    if (out) *out = nullptr;
    if (m != 16 && m != 32 && m != 64)
        return fail(VK_ERR_UNSUPPORTED, "4-bit PQ indexes support m = 16, 32 or 64 (m = %d)", m);
    return index_from_host(device, centroids, m, dsub, codes, n, id_base, 4, out);
}

int vk_index_bits(const vk_index_t* ix, int* nbits) {
    if (!ix || !nbits) return fail(VK_ERR_INVALID, "index and nbits must not be NULL");
    *nbits = ix->nbits;
    return VK_OK;
}

int vk_index_create_from_device(int device, const float* centroids, int m, int dsub, const uint8_t* d_codes,
                                int64_t n, int64_t id_base, vk_index_t** out) {
    if (!d_codes) return fail(VK_ERR_INVALID, "codes must not be NULL");
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess) return fail(VK_ERR_CUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(guard.err));
    vk_index* ix = nullptr;
    int rc = create_common(device, centroids, m, dsub, n, id_base, out, ix);
    if (rc == VK_OK) {
        vk::interleave_kernel<<<grid_for(ix->n_pad * ix->W, ix->sm_count), 256, 0, ix->stream>>>(d_codes, 0, n, n, m,
                                                                                                   ix->W, ix->codes);
        cudaError_t e = cudaGetLastError();
        if (e == cudaSuccess) e = place_rows(ix);
        if (e == cudaSuccess) e = cudaStreamSynchronize(ix->stream);
        if (e != cudaSuccess) rc = fail(VK_ERR_CUDA, "index build failed: %s", cudaGetErrorString(e));
    }
    if (rc != VK_OK) {
        delete ix;
        return rc;
    }
    *out = ix;
    return VK_OK;
}

int vk_index_create_generated(int device, const float* centroids, int m, int dsub, uint64_t seed,
                              const uint32_t* cdf, int clusters, int64_t row_first, int64_t n, int64_t id_base,
                              vk_index_t** out) {
    if (!cdf || clusters <= 0) return fail(VK_ERR_INVALID, "cdf must not be NULL and clusters must be positive");
    if (row_first < 0) return fail(VK_ERR_INVALID, "row_first must be >= 0");
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess) return fail(VK_ERR_CUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(guard.err));
    vk_index* ix = nullptr;
    int rc = create_common(device, centroids, m, dsub, n, id_base, out, ix);
    if (rc == VK_OK) {
        uint32_t* d_cdf = nullptr;
        const size_t bytes = (size_t)clusters * m * vk::KSUB * sizeof(uint32_t);
        cudaError_t e = cudaMalloc(&d_cdf, bytes);
        if (e == cudaSuccess) e = cudaMemcpyAsync(d_cdf, cdf, bytes, cudaMemcpyHostToDevice, ix->stream);
        if (e == cudaSuccess) {
            vk::gen_interleaved_kernel<<<grid_for(ix->n_pad * ix->W, ix->sm_count), 256, 0, ix->stream>>>(
                vk::mix64(seed), d_cdf, clusters, m, ix->W, row_first, n, ix->n_pad, ix->codes);
            e = cudaGetLastError();
        }
        if (e == cudaSuccess) e = place_rows(ix);
        if (e == cudaSuccess) e = cudaStreamSynchronize(ix->stream);
        if (d_cdf) cudaFree(d_cdf);
        if (e != cudaSuccess) rc = fail(VK_ERR_CUDA, "code generation failed: %s", cudaGetErrorString(e));
    }
    if (rc != VK_OK) {
        delete ix;
        return rc;
    }
    *out = ix;
    return VK_OK;
}

int vk_index_destroy(vk_index_t* index) {
    delete index;
    return VK_OK;
}

int vk_index_info(const vk_index_t* ix, int64_t* n, int* m, int* dsub, int64_t* id_base, int* device) {
    if (!ix) return fail(VK_ERR_INVALID, "index must not be NULL");
    if (n) *n = ix->n;
    if (m) *m = ix->m;
    if (dsub) *dsub = ix->dsub;
    if (id_base) *id_base = ix->id_base;
    if (device) *device = ix->device;
    return VK_OK;
}

int vk_index_get_codes(const vk_index_t* ix, int64_t first, int64_t count, uint8_t* out) {
    if (!ix || !out) return fail(VK_ERR_INVALID, "index and out must not be NULL");
    if (first < 0 || count < 0 || first + count > ix->n) return fail(VK_ERR_INVALID, "row range out of bounds");
    if (count == 0) return VK_OK;
    DeviceGuard guard(ix->device);
    uint8_t* d = nullptr;
    VK_TRY_CUDA(cudaMalloc(&d, (size_t)count * ix->mb));
    vk::deinterleave_kernel<<<grid_for((count + 2 * vk::PLACE_WINDOW) * ix->mb, ix->sm_count), 256, 0, ix->stream>>>(
        ix->codes, ix->perm, first, count, ix->mb, ix->W, d);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, d, (size_t)count * ix->mb, cudaMemcpyDeviceToHost, ix->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ix->stream);
    cudaFree(d);
    if (e != cudaSuccess) return fail(VK_ERR_CUDA, "reading codes failed: %s", cudaGetErrorString(e));
    return VK_OK;
}

int vk_index_save(const vk_index_t* ix, const char* path) {
    if (!ix || !path) return fail(VK_ERR_INVALID, "index and path must not be NULL");
    if (ix->nbits != 8) return fail(VK_ERR_UNSUPPORTED, "index files hold 8-bit codes only");
    DeviceGuard guard(ix->device);
    std::vector<float> cent((size_t)ix->m * vk::KSUB * ix->dsub);
    VK_TRY_CUDA(cudaMemcpy(cent.data(), ix->centroids, cent.size() * sizeof(float), cudaMemcpyDeviceToHost));
    int64_t done = 0;
    int rc = VK_OK;
    const std::string err = vkio::write_index(path, cent.data(), (uint32_t)ix->m, (uint32_t)ix->dsub, (uint64_t)ix->n,
                                              [&](uint64_t rows, uint8_t* buf) {
                                                  rc = vk_index_get_codes(ix, done, (int64_t)rows, buf);
                                                  done += (int64_t)rows;
                                                  return rc == VK_OK;
                                              });
    if (rc != VK_OK) return rc;
    if (!err.empty()) return fail(VK_ERR_CUDA, "saving %s: %s", path, err.c_str());
    return VK_OK;
}

int vk_index_load(int device, const char* path, int64_t row_first, int64_t count, int64_t id_base, int verify,
                  vk_index_t** out) {
    if (!path || !out) return fail(VK_ERR_INVALID, "path and out must not be NULL");
    *out = nullptr;
    vkio::Reader rd(path);
    if (!rd.ok()) return fail(VK_ERR_INVALID, "%s: %s", path, rd.err.c_str());
    const int64_t n_file = (int64_t)rd.h.n;
    if (count < 0) count = n_file - row_first;
    if (row_first < 0 || row_first > n_file || count <= 0 || count > n_file - row_first)
        return fail(VK_ERR_INVALID, "row range [%lld, +%lld) is outside the file's %lld rows", (long long)row_first,
                    (long long)count, (long long)n_file);
    if (id_base < 0) id_base = row_first;
    std::vector<float> cent((size_t)rd.h.m * vk::KSUB * rd.h.dsub);
    std::string err = rd.centroids(cent.data());
    if (!err.empty()) return fail(VK_ERR_INVALID, "%s: %s", path, err.c_str());
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess) return fail(VK_ERR_CUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(guard.err));
    vk_index* ix = nullptr;
    int rc = create_common(device, cent.data(), (int)rd.h.m, (int)rd.h.dsub, count, id_base, out, ix);
    if (rc != VK_OK) {
        delete ix;
        return rc;
    }
    // Rows arrive in pieces of at most one checksum block; they are gathered into a staging slice (a multiple of
    // 32 rows, so every slice starts a 32-row group) and interleaved on the device slice by slice.
    const int m = ix->m;
    const int64_t slice = std::min<int64_t>(ceil_div(count, 32) * 32, int64_t(1) << 22);
    std::vector<uint8_t> host((size_t)slice * m);
    uint8_t* staging = nullptr;
    cudaError_t e = cudaMalloc(&staging, (size_t)slice * m);
    int64_t fill = 0, slice0 = 0;  // rows in the staging slice, its first row (relative to row_first)
    auto flush = [&]() {
        if (e != cudaSuccess || fill == 0) return;
        e = cudaMemcpyAsync(staging, host.data(), (size_t)fill * m, cudaMemcpyHostToDevice, ix->stream);
        if (e == cudaSuccess) {
            vk::interleave_kernel<<<grid_for(ceil_div(fill, 32) * 32 * ix->W, ix->sm_count), 256, 0, ix->stream>>>(
                staging, slice0, fill, count, m, ix->W, ix->codes);
            e = cudaGetLastError();
        }
        if (e == cudaSuccess) e = cudaStreamSynchronize(ix->stream);  // host and staging are reused
        slice0 += fill;
        fill = 0;
    };
    if (e == cudaSuccess) {
        err = rd.rows((uint64_t)row_first, (uint64_t)count, verify != 0,
                      [&](uint64_t row0, uint64_t rows, const uint8_t* bytes) {
                          uint64_t done = 0;
                          while (done < rows && e == cudaSuccess) {
                              const int64_t take = std::min<int64_t>((int64_t)(rows - done), slice - fill);
                              std::memcpy(host.data() + (size_t)fill * m, bytes + done * m, (size_t)take * m);
                              fill += take;
                              done += (uint64_t)take;
                              if (fill == slice) flush();
                          }
                          (void)row0;
                          return e == cudaSuccess;
                      });
        flush();
    }
    if (staging) cudaFree(staging);
    if (e == cudaSuccess && err.empty()) e = place_rows(ix);
    if (e == cudaSuccess && err.empty()) e = cudaStreamSynchronize(ix->stream);
    if (e != cudaSuccess || !err.empty()) {
        delete ix;
        *out = nullptr;
        if (!err.empty()) return fail(VK_ERR_INVALID, "%s: %s", path, err.c_str());
        return fail(VK_ERR_CUDA, "loading %s failed: %s", path, cudaGetErrorString(e));
    }
    *out = ix;
    return VK_OK;
}

// ------------------------------------------------------------------------------------------------ multi-GPU
}  // extern "C"

// One process, several devices: shard g of G holds rows [g * ceil(n / G), ...) as its own index with global ids.
// A search launches every shard's search on its own stream (all asynchronous, so the devices run concurrently from
// one host thread), pads each shard's lists to k when the shard has fewer than k rows, copies them over the device
// interconnect (cudaMemcpyPeerAsync) into a [shard][query][k] buffer on the first device and merges them there.
struct vk_multi {
    struct Lane {
        int device = 0;
        vk_index* index = nullptr;
        int64_t lo = 0, rows = 0;
        cudaStream_t st = nullptr;
        cudaEvent_t ev[3] = {};  // before the search, after it, after the copy to the first device
        DevBuf<float> queries;
        DevBuf<int2> res, padded;
    };
    std::vector<Lane> lanes;
    int64_t n = 0;
    int m = 0, dsub = 0;
    cudaStream_t st0 = nullptr;  // on lanes[0].device
    cudaEvent_t ev0[4] = {};
    DevBuf<int2> lists, merged;

    ~vk_multi() {
        for (auto& l : lanes) {
            DeviceGuard g(l.device);
            delete l.index;
            l.index = nullptr;
            l.queries.release();
            l.res.release();
            l.padded.release();
            for (auto& e : l.ev)
                if (e) cudaEventDestroy(e);
            if (l.st) cudaStreamDestroy(l.st);
        }
        if (!lanes.empty()) {
            DeviceGuard g(lanes[0].device);
            lists.release();
            merged.release();
            for (auto& e : ev0)
                if (e) cudaEventDestroy(e);
            if (st0) cudaStreamDestroy(st0);
        }
    }
};

namespace {

// Creates the lanes' streams and events, enables peer access to the first device; `make(lane)` builds the index.
template <class Make>
int multi_create(int ndev, const int* devices, int64_t n, vk_multi_t** out, Make&& make) {
    if (!out) return fail(VK_ERR_INVALID, "out must not be NULL");
    *out = nullptr;
    if (ndev < 1 || !devices) return fail(VK_ERR_INVALID, "need at least one device");
    const int64_t per = ceil_div(n, ndev);
    if (n <= 0 || (int64_t)(ndev - 1) * per >= n)
        return fail(VK_ERR_INVALID, "n = %lld rows leave a shard of %d empty", (long long)n, ndev);
    auto* mx = new vk_multi();
    mx->n = n;
    mx->lanes.resize(ndev);
    int rc = VK_OK;
    for (int g = 0; g < ndev && rc == VK_OK; ++g) {
        auto& l = mx->lanes[g];
        l.device = devices[g];
        l.lo = (int64_t)g * per;
        l.rows = std::min(n, l.lo + per) - l.lo;
        rc = make(l);
        if (rc != VK_OK) break;
        DeviceGuard guard(l.device);
        if (cudaStreamCreateWithFlags(&l.st, cudaStreamNonBlocking) != cudaSuccess) rc = fail(VK_ERR_CUDA, "stream");
        for (auto& e : l.ev)
            if (rc == VK_OK && cudaEventCreate(&e) != cudaSuccess) rc = fail(VK_ERR_CUDA, "event");
        if (rc == VK_OK && l.device != devices[0]) {
            int can = 0;
            cudaDeviceCanAccessPeer(&can, devices[0], l.device);
            if (can) {
                DeviceGuard g0(devices[0]);
                const cudaError_t e = cudaDeviceEnablePeerAccess(l.device, 0);
                if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled)
                    rc = fail(VK_ERR_CUDA, "peer access %d -> %d: %s", devices[0], l.device, cudaGetErrorString(e));
                cudaGetLastError();  // clear cudaErrorPeerAccessAlreadyEnabled
            }
        }
    }
    if (rc == VK_OK) {
        mx->m = mx->lanes[0].index->m;
        mx->dsub = mx->lanes[0].index->dsub;
        DeviceGuard guard(devices[0]);
        if (cudaStreamCreateWithFlags(&mx->st0, cudaStreamNonBlocking) != cudaSuccess) rc = fail(VK_ERR_CUDA, "stream");
        for (auto& e : mx->ev0)
            if (rc == VK_OK && cudaEventCreate(&e) != cudaSuccess) rc = fail(VK_ERR_CUDA, "event");
    }
    if (rc != VK_OK) {
        delete mx;
        return rc;
    }
    *out = mx;
    return VK_OK;
}

}  // namespace

extern "C" {

int vk_multi_create(int ndev, const int* devices, const float* centroids, int m, int dsub, const uint8_t* codes,
                    int64_t n, vk_multi_t** out) {
    if (!codes || !centroids) return fail(VK_ERR_INVALID, "centroids and codes must not be NULL");
    return multi_create(ndev, devices, n, out, [&](vk_multi::Lane& l) {
        return vk_index_create(l.device, centroids, m, dsub, codes + l.lo * m, l.rows, l.lo, &l.index);
    });
}

int vk_multi_load(int ndev, const int* devices, const char* path, int verify, vk_multi_t** out) {
    if (!path) return fail(VK_ERR_INVALID, "path must not be NULL");
    vkio::Reader rd(path);
    if (!rd.ok()) return fail(VK_ERR_INVALID, "%s: %s", path, rd.err.c_str());
    return multi_create(ndev, devices, (int64_t)rd.h.n, out, [&](vk_multi::Lane& l) {
        return vk_index_load(l.device, path, l.lo, l.rows, l.lo, verify, &l.index);
    });
}

int vk_multi_destroy(vk_multi_t* mx) {
    delete mx;
    return VK_OK;
}

int vk_multi_info(const vk_multi_t* mx, int64_t* n, int* shards) {
    if (!mx) return fail(VK_ERR_INVALID, "multi-GPU searcher must not be NULL");
    if (n) *n = mx->n;
    if (shards) *shards = (int)mx->lanes.size();
    return VK_OK;
}

int vk_multi_search(vk_multi_t* mx, const float* queries, int64_t nq, int k, const vk_tuning_t* tuning,
                    vk_neighbor_t* out, vk_timings_t* timings) {
    if (!mx) return fail(VK_ERR_INVALID, "multi-GPU searcher must not be NULL");
    if (k < 1 || k > 128 || (int64_t)k > mx->n) return fail(VK_ERR_INVALID, "k must be in [1, min(128, n)]");
    if (nq < 0) return fail(VK_ERR_INVALID, "nq must be >= 0");
    if (nq > 0 && (!queries || !out)) return fail(VK_ERR_INVALID, "queries and out must not be NULL");
    vk_tuning_t t;
    vk_tuning_default(&t);
    if (tuning) t = *tuning;
    VK_TRY(validate_tuning(&t));
    if (timings) *timings = vk_timings_t{};
    if (nq == 0) return VK_OK;
    const int G = (int)mx->lanes.size();
    const int d = mx->m * mx->dsub;
    int64_t batch = nq;
    for (auto& l : mx->lanes) batch = std::min(batch, max_query_batch(l.index));
    const int dev0 = mx->lanes[0].device;
    vk_timings_t acc{};
    for (int64_t q0 = 0; q0 < nq; q0 += batch) {
        const int64_t b = std::min(batch, nq - q0);
        {
            DeviceGuard g0(dev0);
            VK_TRY(mx->lists.ensure((size_t)G * b * k));
            VK_TRY(mx->merged.ensure((size_t)b * k));
            VK_TRY_CUDA(cudaEventRecord(mx->ev0[0], mx->st0));
        }
        for (int g = 0; g < G; ++g) {
            auto& l = mx->lanes[g];
            DeviceGuard guard(l.device);
            const int kg = (int)std::min<int64_t>(k, l.rows);
            VK_TRY(l.queries.ensure((size_t)b * d));
            VK_TRY(l.res.ensure((size_t)b * kg));
            VK_TRY_CUDA(cudaMemcpyAsync(l.queries.ptr, queries + q0 * d, (size_t)b * d * sizeof(float),
                                        cudaMemcpyHostToDevice, l.st));
            VK_TRY_CUDA(cudaEventRecord(l.ev[0], l.st));
            VK_TRY(run_search(l.index, l.queries.ptr, b, kg, t, l.res.ptr, l.st, nullptr, nullptr));
            VK_TRY_CUDA(cudaEventRecord(l.ev[1], l.st));
            const int2* src = l.res.ptr;
            if (kg < k) {  // a shard with fewer than k rows: pad its lists with (NaN bits, -1) = merge padding
                VK_TRY(l.padded.ensure((size_t)b * k));
                VK_TRY_CUDA(cudaMemsetAsync(l.padded.ptr, 0xFF, (size_t)b * k * sizeof(int2), l.st));
                VK_TRY_CUDA(cudaMemcpy2DAsync(l.padded.ptr, (size_t)k * sizeof(int2), l.res.ptr,
                                              (size_t)kg * sizeof(int2), (size_t)kg * sizeof(int2), (size_t)b,
                                              cudaMemcpyDeviceToDevice, l.st));
                src = l.padded.ptr;
            }
            VK_TRY_CUDA(cudaMemcpyPeerAsync(mx->lists.ptr + (size_t)g * b * k, dev0, src, l.device,
                                            (size_t)b * k * sizeof(int2), l.st));
            VK_TRY_CUDA(cudaEventRecord(l.ev[2], l.st));
        }
        DeviceGuard g0(dev0);
        for (auto& l : mx->lanes) VK_TRY_CUDA(cudaStreamWaitEvent(mx->st0, l.ev[2], 0));
        VK_TRY_CUDA(cudaEventRecord(mx->ev0[1], mx->st0));
        VK_TRY(vk_merge_topk_device(dev0, reinterpret_cast<const vk_neighbor_t*>(mx->lists.ptr), b, G, k, k, b * k,
                                    k, reinterpret_cast<vk_neighbor_t*>(mx->merged.ptr), mx->st0));
        VK_TRY_CUDA(cudaEventRecord(mx->ev0[2], mx->st0));
        VK_TRY_CUDA(cudaMemcpyAsync(out + q0 * k, mx->merged.ptr, (size_t)b * k * sizeof(int2), cudaMemcpyDeviceToHost,
                                    mx->st0));
        VK_TRY_CUDA(cudaEventRecord(mx->ev0[3], mx->st0));
        VK_TRY_CUDA(cudaEventSynchronize(mx->ev0[3]));
        float scan = 0.f, ms = 0.f;
        for (auto& l : mx->lanes) {
            DeviceGuard guard(l.device);
            VK_TRY_CUDA(cudaEventElapsedTime(&ms, l.ev[0], l.ev[1]));
            scan = std::max(scan, ms);
        }
        float gather_merge = 0.f, copy_out = 0.f, total = 0.f;
        VK_TRY_CUDA(cudaEventElapsedTime(&gather_merge, mx->ev0[1], mx->ev0[2]));
        VK_TRY_CUDA(cudaEventElapsedTime(&copy_out, mx->ev0[2], mx->ev0[3]));
        VK_TRY_CUDA(cudaEventElapsedTime(&total, mx->ev0[0], mx->ev0[3]));
        acc.scan_ms += scan;                                                  // slowest shard: LUT + scan + lists
        acc.select_ms += gather_merge;                                        // cross-shard merge on the first device
        acc.transfer_ms += std::max(0.f, total - scan - gather_merge);        // query uploads, gathers, result copy
    }
    for (auto& l : mx->lanes) {
        DeviceGuard guard(l.device);
        VK_TRY(read_status(l.index, l.st));
    }
    if (timings) *timings = acc;
    return VK_OK;
}

int vk_index_get_placement(const vk_index_t* ix, int64_t first, int64_t count, uint8_t* out) {
    if (!ix || (!out && count > 0)) return fail(VK_ERR_INVALID, "index and out must not be NULL");
    if (first < 0 || count < 0 || first % vk::PLACE_WINDOW != 0 || first + count > ix->n_pad)
        return fail(VK_ERR_INVALID, "position range out of bounds");
    if (count == 0) return VK_OK;
    DeviceGuard guard(ix->device);
    VK_TRY_CUDA(cudaMemcpyAsync(out, ix->perm + first, (size_t)count, cudaMemcpyDeviceToHost, ix->stream));
    VK_TRY_CUDA(cudaStreamSynchronize(ix->stream));
    return VK_OK;
}

int vk_search(vk_index_t* ix, const float* queries, int64_t nq, int k, int variant, const vk_tuning_t* tuning,
              vk_neighbor_t* out, vk_timings_t* timings, vk_launch_shape_t* shape) {
    if (!ix) return fail(VK_ERR_INVALID, "index must not be NULL");
    if (k < 1 || k > 128 || (int64_t)k > ix->n) return fail(VK_ERR_INVALID, "k must be in [1, min(128, n)]");
    if (nq < 0) return fail(VK_ERR_INVALID, "nq must be >= 0");
    if (nq > 0 && (!queries || !out)) return fail(VK_ERR_INVALID, "queries and out must not be NULL");
    VK_TRY(check_variant(ix, variant));
    vk_tuning_t t;
    vk_tuning_default(&t);
    if (tuning) t = *tuning;
    VK_TRY(validate_tuning(&t));
    if (timings) *timings = vk_timings_t{};
    if (nq == 0) return VK_OK;
    DeviceGuard guard(ix->device);
    if (guard.err != cudaSuccess) return fail(VK_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(guard.err));
    cudaStream_t st = ix->stream;
    const int64_t d = (int64_t)ix->m * ix->dsub;
    const int64_t batch = std::min(nq, max_query_batch(ix));
    VK_TRY(ix->queries.ensure((size_t)batch * d));
    VK_TRY(ix->out.ensure((size_t)batch * k));
    vk_timings_t acc{};
    for (int64_t q0 = 0; q0 < nq; q0 += batch) {
        const int64_t b = std::min(batch, nq - q0);
        cudaEvent_t* ev = ix->ev;
        VK_TRY_CUDA(cudaEventRecord(ev[0], st));
        VK_TRY_CUDA(cudaMemcpyAsync(ix->queries.ptr, queries + q0 * d, (size_t)b * d * sizeof(float),
                                    cudaMemcpyHostToDevice, st));
        VK_TRY_CUDA(cudaEventRecord(ev[1], st));
        cudaEvent_t marks[2] = {ev[2], ev[3]};
        VK_TRY(run_search(ix, ix->queries.ptr, b, k, t, ix->out.ptr, st, shape, marks));
        VK_TRY_CUDA(cudaEventRecord(ev[4], st));
        VK_TRY_CUDA(cudaMemcpyAsync(out + q0 * k, ix->out.ptr, (size_t)b * k * sizeof(int2), cudaMemcpyDeviceToHost,
                                    st));
        VK_TRY_CUDA(cudaEventRecord(ev[5], st));
        VK_TRY_CUDA(cudaEventSynchronize(ev[5]));
        float ms[5];
        for (int i = 0; i < 5; ++i) VK_TRY_CUDA(cudaEventElapsedTime(&ms[i], ev[i], ev[i + 1]));
        acc.transfer_ms += ms[0] + ms[4];
        acc.lut_ms += ms[1];
        acc.scan_ms += ms[2];
        acc.select_ms += ms[3];
    }
    VK_TRY(read_status(ix, st));
    if (timings) *timings = acc;
    return VK_OK;
}

int vk_search_device(vk_index_t* ix, const float* d_queries, int64_t nq, int k, const vk_tuning_t* tuning,
                     vk_neighbor_t* d_out, void* stream) {
    if (!ix) return fail(VK_ERR_INVALID, "index must not be NULL");
    if (k < 1 || k > 128 || (int64_t)k > ix->n) return fail(VK_ERR_INVALID, "k must be in [1, min(128, n)]");
    if (nq < 0) return fail(VK_ERR_INVALID, "nq must be >= 0");
    if (nq > 0 && (!d_queries || !d_out)) return fail(VK_ERR_INVALID, "queries and out must not be NULL");
    if (nq > max_query_batch(ix))
        return fail(VK_ERR_INVALID, "nq %lld exceeds the device-path batch limit %lld", (long long)nq,
                    (long long)max_query_batch(ix));
    vk_tuning_t t;
    vk_tuning_default(&t);
    if (tuning) t = *tuning;
    VK_TRY(validate_tuning(&t));
    if (nq == 0) return VK_OK;
    DeviceGuard guard(ix->device);
    if (guard.err != cudaSuccess) return fail(VK_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(guard.err));
    return run_search(ix, d_queries, nq, k, t, reinterpret_cast<int2*>(d_out), static_cast<cudaStream_t>(stream),
                      nullptr, nullptr);
}

// ------------------------------------------------------------------------------------------------ cooperative search
}  // extern "C"

struct vk_coop {
    int device = 0;
    int64_t nq_max = 0;
    int64_t nq_limit = 0;                       // the smallest nq_max of this shard and the attached ones
    unsigned long long* xb = nullptr;           // this shard's exchange array (cudaMalloc'd, zeroed)
    std::vector<unsigned long long*> peers;     // the other shards' arrays
    std::vector<void*> ipc_opened;              // of those, the ones mapped with cudaIpcOpenMemHandle
    ~vk_coop() {
        DeviceGuard g(device);
        for (void* p : ipc_opened) cudaIpcCloseMemHandle(p);
        if (xb) cudaFree(xb);
    }
};

extern "C" {

int vk_coop_create(int device, int64_t nq_max, vk_coop_t** out) {
    if (!out) return fail(VK_ERR_INVALID, "out must not be NULL");
    *out = nullptr;
    if (nq_max < 1) return fail(VK_ERR_INVALID, "nq_max must be >= 1");
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess) return fail(VK_ERR_CUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(guard.err));
    auto* c = new vk_coop();
    c->device = device;
    c->nq_max = nq_max;
    c->nq_limit = nq_max;
    cudaError_t e = cudaMalloc(&c->xb, (size_t)nq_max * sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMemset(c->xb, 0, (size_t)nq_max * sizeof(unsigned long long));
    if (e != cudaSuccess) {
        delete c;
        return fail(e == cudaErrorMemoryAllocation ? VK_ERR_NOMEM : VK_ERR_CUDA, "cooperative search buffer: %s",
                    cudaGetErrorString(e));
    }
    *out = c;
    return VK_OK;
}

// What one shard publishes for the others: its array's IPC handle, the array's length and its device ordinal.
struct CoopHandle {
    cudaIpcMemHandle_t ipc;
    int64_t nq_max;
    int32_t device;
    int32_t reserved;
};
static_assert(sizeof(CoopHandle) == VK_COOP_HANDLE_BYTES, "VK_COOP_HANDLE_BYTES");

// Posted atomics into another GPU's memory need a link that carries them natively (NVLink); refuse otherwise.
int check_peer_atomics(int dev, int peer) {
    if (dev == peer) return VK_OK;
    int atomics = 0, access = 0;
    VK_TRY_CUDA(cudaDeviceCanAccessPeer(&access, dev, peer));
    VK_TRY_CUDA(cudaDeviceGetP2PAttribute(&atomics, cudaDevP2PAttrNativeAtomicSupported, dev, peer));
    if (!access || !atomics)
        return fail(VK_ERR_UNSUPPORTED, "device %d cannot make atomic writes into device %d's memory", dev, peer);
    return VK_OK;
}

int vk_coop_ipc_handle(const vk_coop_t* c, void* handle) {
    if (!c || !handle) return fail(VK_ERR_INVALID, "coop and handle must not be NULL");
    DeviceGuard guard(c->device);
    CoopHandle h{};
    VK_TRY_CUDA(cudaIpcGetMemHandle(&h.ipc, c->xb));
    h.nq_max = c->nq_max;
    h.device = c->device;
    std::memcpy(handle, &h, sizeof(h));
    return VK_OK;
}

int vk_coop_attach_ipc(vk_coop_t* c, int n, const void* handles) {
    if (!c || (n > 0 && !handles)) return fail(VK_ERR_INVALID, "coop and handles must not be NULL");
    if (!c->peers.empty()) return fail(VK_ERR_INVALID, "this cooperative search is already attached");
    CoopHandle own;
    VK_TRY(vk_coop_ipc_handle(c, &own));
    int count = 0;
    VK_TRY_CUDA(cudaGetDeviceCount(&count));
    DeviceGuard guard(c->device);
    for (int i = 0; i < n; ++i) {
        CoopHandle h;
        std::memcpy(&h, static_cast<const unsigned char*>(handles) + (size_t)i * VK_COOP_HANDLE_BYTES, sizeof(h));
        if (std::memcmp(&h.ipc, &own.ipc, sizeof(h.ipc)) == 0) continue;  // this shard's own array
        if ((int)c->peers.size() >= vk::COOP_MAX_PEERS)
            return fail(VK_ERR_UNSUPPORTED, "at most %d other shards", vk::COOP_MAX_PEERS);
        if (h.nq_max < 1 || h.device < 0 || h.device >= count)
            return fail(VK_ERR_INVALID, "handle %d is not a cooperative search handle of this node", i);
        VK_TRY(check_peer_atomics(c->device, h.device));
        void* p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h.ipc, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return fail(VK_ERR_CUDA, "cudaIpcOpenMemHandle (shard %d): %s", i, cudaGetErrorString(e));
        c->ipc_opened.push_back(p);
        c->peers.push_back(static_cast<unsigned long long*>(p));
        c->nq_limit = std::min(c->nq_limit, h.nq_max);
    }
    return VK_OK;
}

int vk_coop_attach(vk_coop_t* c, int n, vk_coop_t* const* others) {
    if (!c || (n > 0 && !others)) return fail(VK_ERR_INVALID, "coop and others must not be NULL");
    if (!c->peers.empty()) return fail(VK_ERR_INVALID, "this cooperative search is already attached");
    for (int i = 0; i < n; ++i) {
        const vk_coop* o = others[i];
        if (!o) return fail(VK_ERR_INVALID, "shard %d is NULL", i);
        if (o == c) continue;
        if ((int)c->peers.size() >= vk::COOP_MAX_PEERS)
            return fail(VK_ERR_UNSUPPORTED, "at most %d other shards", vk::COOP_MAX_PEERS);
        if (o->device != c->device) {  // this device's kernels write into the other device's memory
            VK_TRY(check_peer_atomics(c->device, o->device));
            DeviceGuard g(c->device);
            const cudaError_t e = cudaDeviceEnablePeerAccess(o->device, 0);
            if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled)
                return fail(VK_ERR_CUDA, "peer access %d -> %d: %s", c->device, o->device, cudaGetErrorString(e));
            cudaGetLastError();
        }
        c->peers.push_back(o->xb);
        c->nq_limit = std::min(c->nq_limit, o->nq_max);
    }
    return VK_OK;
}

int vk_coop_destroy(vk_coop_t* c) {
    delete c;
    return VK_OK;
}

int vk_search_device_coop(vk_index_t* ix, vk_coop_t* c, uint32_t epoch, const float* d_queries, int64_t nq, int k,
                          const vk_tuning_t* tuning, vk_neighbor_t* d_out, void* stream) {
    if (!ix || !c) return fail(VK_ERR_INVALID, "index and coop must not be NULL");
    if (epoch == 0) return fail(VK_ERR_INVALID, "epoch must be >= 1");
    if (nq > c->nq_limit)  // every shard's array must hold nq queries
        return fail(VK_ERR_INVALID, "nq %lld exceeds the cooperative search's nq_max %lld (of this or another shard)",
                    (long long)nq, (long long)c->nq_limit);
    if (c->device != ix->device) return fail(VK_ERR_INVALID, "coop and index are on different devices");
    if (k < 1 || k > 128 || (int64_t)k > ix->n) return fail(VK_ERR_INVALID, "k must be in [1, min(128, n)]");
    if (nq < 0) return fail(VK_ERR_INVALID, "nq must be >= 0");
    if (nq > 0 && (!d_queries || !d_out)) return fail(VK_ERR_INVALID, "queries and out must not be NULL");
    if (nq > max_query_batch(ix))
        return fail(VK_ERR_INVALID, "nq %lld exceeds the device-path batch limit %lld", (long long)nq,
                    (long long)max_query_batch(ix));
    vk_tuning_t t;
    vk_tuning_default(&t);
    if (tuning) t = *tuning;
    VK_TRY(validate_tuning(&t));
    if (nq == 0) return VK_OK;
    DeviceGuard guard(ix->device);
    if (guard.err != cudaSuccess) return fail(VK_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(guard.err));
    Workspace w;
    w.xb = c->xb;
    for (size_t i = 0; i < c->peers.size(); ++i) w.xpeer[i] = c->peers[i];
    w.npeers = (int)c->peers.size();
    w.epoch = epoch;
    return run_search(ix, d_queries, nq, k, t, reinterpret_cast<int2*>(d_out), static_cast<cudaStream_t>(stream),
                      nullptr, nullptr, &w);
}

int vk_index_sync(vk_index_t* ix, void* stream) {
    if (!ix) return fail(VK_ERR_INVALID, "index must not be NULL");
    DeviceGuard guard(ix->device);
    return read_status(ix, static_cast<cudaStream_t>(stream));
}

int vk_distances(vk_index_t* ix, const float* queries, int64_t nq, int variant, const vk_tuning_t* tuning,
                 float* out, vk_timings_t* timings) {
    if (!ix) return fail(VK_ERR_INVALID, "index must not be NULL");
    if (ix->nbits != 8) return fail(VK_ERR_UNSUPPORTED, "distances() is implemented for 8-bit indexes only");
    if (variant < 0 || variant > 8) return fail(VK_ERR_INVALID, "unknown scan variant %d", variant);
    if (is_fused_variant(variant)) return fail(VK_ERR_INVALID, "fused variants do not materialise distances");
    VK_TRY(check_variant(ix, variant));
    vk_tuning_t t;
    vk_tuning_default(&t);
    if (tuning) t = *tuning;
    VK_TRY(validate_tuning(&t));
    if (timings) *timings = vk_timings_t{};
    if (nq < 0) return fail(VK_ERR_INVALID, "nq must be >= 0");
    if (nq == 0) return VK_OK;
    if (!queries || !out) return fail(VK_ERR_INVALID, "queries and out must not be NULL");
    DeviceGuard guard(ix->device);
    if (guard.err != cudaSuccess) return fail(VK_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(guard.err));
    cudaStream_t st = ix->stream;
    const int64_t d = (int64_t)ix->m * ix->dsub;
    const int64_t batch =
        std::max<int64_t>(1, std::min<int64_t>(65535, (int64_t)(kDistanceBudgetBytes / ((size_t)ix->n * 4))));
    const int64_t b0 = std::min(batch, nq);
    VK_TRY(ix->queries.ensure((size_t)b0 * d));
    VK_TRY(ix->lut.ensure((size_t)b0 * ix->m * vk::KSUB));
    VK_TRY(ix->dists.ensure((size_t)b0 * ix->n));
    const size_t lut_smem = (size_t)ix->m * vk::KSUB * sizeof(float);
    VK_TRY_CUDA(cudaFuncSetAttribute(reinterpret_cast<const void*>(&vk::dist_kernel),
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lut_smem));
    vk_timings_t acc{};
    cudaEvent_t* ev = ix->ev;
    for (int64_t q0 = 0; q0 < nq; q0 += batch) {
        const int64_t b = std::min(batch, nq - q0);
        VK_TRY_CUDA(cudaEventRecord(ev[0], st));
        VK_TRY_CUDA(cudaMemcpyAsync(ix->queries.ptr, queries + q0 * d, (size_t)b * d * sizeof(float),
                                    cudaMemcpyHostToDevice, st));
        VK_TRY_CUDA(cudaEventRecord(ev[1], st));
        vk::lut_kernel<1><<<dim3(ix->m, (unsigned)b), vk::KSUB, ix->dsub * sizeof(float), st>>>(
            ix->centroids, ix->queries.ptr, b, ix->m, ix->dsub, ix->lut.ptr, nullptr, nullptr, nullptr, 0);
        VK_TRY_CUDA(cudaGetLastError());
        VK_TRY_CUDA(cudaEventRecord(ev[2], st));
        const int threads = t.scan_threads;
        const int64_t bx = std::max<int64_t>(1, std::min<int64_t>(ceil_div(ix->n, threads),
                                                                  ceil_div(8LL * ix->sm_count, b)));
        vk::dist_kernel<<<dim3((unsigned)bx, (unsigned)b), threads, lut_smem, st>>>(ix->codes, ix->perm, ix->lut.ptr,
                                                                                    ix->n, ix->m, ix->W, ix->dists.ptr);
        VK_TRY_CUDA(cudaGetLastError());
        VK_TRY_CUDA(cudaEventRecord(ev[3], st));
        VK_TRY_CUDA(cudaMemcpyAsync(out + q0 * ix->n, ix->dists.ptr, (size_t)b * ix->n * sizeof(float),
                                    cudaMemcpyDeviceToHost, st));
        VK_TRY_CUDA(cudaEventRecord(ev[4], st));
        VK_TRY_CUDA(cudaEventSynchronize(ev[4]));
        float ms[4];
        for (int i = 0; i < 4; ++i) VK_TRY_CUDA(cudaEventElapsedTime(&ms[i], ev[i], ev[i + 1]));
        acc.transfer_ms += ms[0] + ms[3];
        acc.lut_ms += ms[1];
        acc.scan_ms += ms[2];
    }
    if (timings) *timings = acc;
    return VK_OK;
}

int vk_compute_lut_device(vk_index_t* ix, const float* d_queries, int64_t nq, float* d_lut, void* stream) {
    if (!ix) return fail(VK_ERR_INVALID, "index must not be NULL");
    if (ix->nbits != 8) return fail(VK_ERR_UNSUPPORTED, "vk_compute_lut_device is implemented for 8-bit indexes only");
    if (nq < 0) return fail(VK_ERR_INVALID, "nq must be >= 0");
    if (nq == 0) return VK_OK;
    if (!d_queries || !d_lut) return fail(VK_ERR_INVALID, "queries and lut must not be NULL");
    if (nq > 65535) return fail(VK_ERR_INVALID, "at most 65535 queries per call");
    DeviceGuard guard(ix->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    vk::lut_kernel<1><<<dim3(ix->m, (unsigned)nq), vk::KSUB, ix->dsub * sizeof(float), st>>>(
        ix->centroids, d_queries, nq, ix->m, ix->dsub, d_lut, nullptr, nullptr, nullptr, 0);
    VK_TRY_CUDA(cudaGetLastError());
    return VK_OK;
}

int vk_merge_topk_device(int device, const vk_neighbor_t* d_in, int64_t nq, int lists, int k_in,
                         int64_t query_stride, int64_t list_stride, int k, vk_neighbor_t* d_out, void* stream) {
    if (k < 1 || k > 128) return fail(VK_ERR_INVALID, "k must be in [1, 128]");
    if (nq < 0 || lists < 0 || k_in < 0) return fail(VK_ERR_INVALID, "sizes must be >= 0");
    if (nq == 0) return VK_OK;
    if (!d_in || !d_out) return fail(VK_ERR_INVALID, "in and out must not be NULL");
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess) return fail(VK_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(guard.err));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int2* in = reinterpret_cast<const int2*>(d_in);
    int2* o = reinterpret_cast<int2*>(d_out);
    switch (s_for_k(k)) {
        case 1: vk::merge_kernel<1><<<(unsigned)ceil_div(nq, 4), 128, 0, st>>>(in, nq, lists, k_in, query_stride, list_stride, k, o, nullptr); break;
        case 2: vk::merge_kernel<2><<<(unsigned)ceil_div(nq, 4), 128, 0, st>>>(in, nq, lists, k_in, query_stride, list_stride, k, o, nullptr); break;
        default: vk::merge_kernel<4><<<(unsigned)ceil_div(nq, 4), 128, 0, st>>>(in, nq, lists, k_in, query_stride, list_stride, k, o, nullptr); break;
    }
    VK_TRY_CUDA(cudaGetLastError());
    return VK_OK;
}

int vk_rerank_device(int device, const float* d_base, int64_t n, int d, const float* d_queries, int64_t nq,
                     const vk_neighbor_t* d_candidates, int r, int k, vk_neighbor_t* d_out, void* stream) {
    if (k < 1 || k > 128) return fail(VK_ERR_INVALID, "k must be in [1, 128]");
    if (n < 0 || nq < 0 || r < 0 || d <= 0) return fail(VK_ERR_INVALID, "bad sizes");
    if (nq == 0) return VK_OK;
    if (!d_base || !d_queries || !d_out || (r > 0 && !d_candidates))
        return fail(VK_ERR_INVALID, "pointers must not be NULL");
    if ((size_t)4 * d * sizeof(float) > 48 * 1024) return fail(VK_ERR_UNSUPPORTED, "d = %d is too large", d);
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess) return fail(VK_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(guard.err));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int2* c = reinterpret_cast<const int2*>(d_candidates);
    int2* o = reinterpret_cast<int2*>(d_out);
    const dim3 grid((unsigned)ceil_div(nq, 4));
    const size_t smem = (size_t)4 * d * sizeof(float);
    switch (s_for_k(k)) {
        case 1: vk::rerank_kernel<1><<<grid, 128, smem, st>>>(d_base, d, d_queries, nq, c, r, k, o); break;
        case 2: vk::rerank_kernel<2><<<grid, 128, smem, st>>>(d_base, d, d_queries, nq, c, r, k, o); break;
        default: vk::rerank_kernel<4><<<grid, 128, smem, st>>>(d_base, d, d_queries, nq, c, r, k, o); break;
    }
    VK_TRY_CUDA(cudaGetLastError());
    (void)n;
    return VK_OK;
}

int vk_encode_device(int device, const float* centroids, int m, int dsub, const float* d_x, int64_t n,
                     uint8_t* d_codes, void* stream) {
    if (!centroids || !d_x || !d_codes) return fail(VK_ERR_INVALID, "pointers must not be NULL");
    if (m <= 0 || dsub <= 0 || n < 0) return fail(VK_ERR_INVALID, "bad sizes");
    if (n == 0) return VK_OK;
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess) return fail(VK_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(guard.err));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t cbytes = (size_t)m * vk::KSUB * dsub * sizeof(float);
    float* d_cen = nullptr;
    VK_TRY_CUDA(cudaMallocAsync(&d_cen, cbytes, st));
    VK_TRY_CUDA(cudaMemcpyAsync(d_cen, centroids, cbytes, cudaMemcpyHostToDevice, st));
    const size_t smem = (size_t)vk::KSUB * dsub * sizeof(float);
    if (smem > 48 * 1024)
        VK_TRY_CUDA(cudaFuncSetAttribute(reinterpret_cast<const void*>(&vk::encode_kernel),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const dim3 egrid((unsigned)ceil_div(n, 256), m);
    switch (dsub) {
        case 1: vk::encode_kernel_t<1><<<egrid, 256, 0, st>>>(d_cen, m, d_x, n, d_codes); break;
        case 2: vk::encode_kernel_t<2><<<egrid, 256, 0, st>>>(d_cen, m, d_x, n, d_codes); break;
        case 4: vk::encode_kernel_t<4><<<egrid, 256, 0, st>>>(d_cen, m, d_x, n, d_codes); break;
        case 8: vk::encode_kernel_t<8><<<egrid, 256, 0, st>>>(d_cen, m, d_x, n, d_codes); break;
        case 16: vk::encode_kernel_t<16><<<egrid, 256, 0, st>>>(d_cen, m, d_x, n, d_codes); break;
        case 32: vk::encode_kernel_t<32><<<egrid, 256, 0, st>>>(d_cen, m, d_x, n, d_codes); break;
        default: vk::encode_kernel<<<egrid, 256, smem, st>>>(d_cen, m, dsub, d_x, n, d_codes); break;
    }
    VK_TRY_CUDA(cudaGetLastError());
    VK_TRY_CUDA(cudaFreeAsync(d_cen, st));
    return VK_OK;
}

int vk_pq_train_device(int device, const float* d_x, int64_t n, int d, int m, int64_t iters, uint64_t seed,
                       float* centroids, void* stream) {
    if (!d_x || !centroids) return fail(VK_ERR_INVALID, "pointers must not be NULL");
    if (m <= 0 || d <= 0 || d % m != 0) return fail(VK_ERR_INVALID, "d must be a positive multiple of m");
    if (n < vk::KSUB) return fail(VK_ERR_INVALID, "PQ training needs at least 256 vectors");
    if (iters < 0) return fail(VK_ERR_INVALID, "iters must be >= 0");
    const int dsub = d / m;
    if (dsub > 128) return fail(VK_ERR_UNSUPPORTED, "dsub > 128 is not supported by the device trainer");
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess) return fail(VK_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(guard.err));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t cbytes = (size_t)vk::KSUB * dsub * sizeof(float);
    DevBuf<int> assign, counts;
    DevBuf<float> cent, sums;
    DevBuf<int64_t> rows;
    VK_TRY(assign.ensure((size_t)n));
    VK_TRY(counts.ensure(vk::KSUB));
    VK_TRY(cent.ensure((size_t)vk::KSUB * dsub));
    VK_TRY(sums.ensure((size_t)vk::KSUB * dsub));
    VK_TRY(rows.ensure(vk::KSUB));
    if (cbytes > 48 * 1024)
        VK_TRY_CUDA(cudaFuncSetAttribute(reinterpret_cast<const void*>(&vk::train_assign_kernel),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cbytes));
    // The reference's draws, in its order: one generator for the whole training, one shuffle of all row indices
    // per sub-space (its first 256 entries seed the centroids), then rng() % n per empty cluster per iteration.
    std::mt19937_64 rng(seed);
    std::vector<size_t> perm((size_t)n);
    std::vector<int64_t> host_rows(vk::KSUB);
    std::vector<int> host_counts(vk::KSUB);
    const unsigned agrid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, 256), 148LL * 8));
    for (int s = 0; s < m; ++s) {
        std::iota(perm.begin(), perm.end(), (size_t)0);
        std::shuffle(perm.begin(), perm.end(), rng);
        for (int c = 0; c < vk::KSUB; ++c) host_rows[c] = (int64_t)perm[c];
        VK_TRY_CUDA(cudaMemcpyAsync(rows.ptr, host_rows.data(), vk::KSUB * sizeof(int64_t), cudaMemcpyHostToDevice, st));
        vk::train_gather_kernel<<<1, 256, 0, st>>>(d_x, d, s, dsub, rows.ptr, cent.ptr);
        VK_TRY_CUDA(cudaGetLastError());
        for (int64_t it = 0; it < iters; ++it) {
            switch (dsub) {
                case 1: vk::train_assign_kernel_t<1><<<agrid, 256, 0, st>>>(d_x, n, d, s, cent.ptr, assign.ptr); break;
                case 2: vk::train_assign_kernel_t<2><<<agrid, 256, 0, st>>>(d_x, n, d, s, cent.ptr, assign.ptr); break;
                case 4: vk::train_assign_kernel_t<4><<<agrid, 256, 0, st>>>(d_x, n, d, s, cent.ptr, assign.ptr); break;
                case 8: vk::train_assign_kernel_t<8><<<agrid, 256, 0, st>>>(d_x, n, d, s, cent.ptr, assign.ptr); break;
                case 16: vk::train_assign_kernel_t<16><<<agrid, 256, 0, st>>>(d_x, n, d, s, cent.ptr, assign.ptr); break;
                case 32: vk::train_assign_kernel_t<32><<<agrid, 256, 0, st>>>(d_x, n, d, s, cent.ptr, assign.ptr); break;
                default:
                    vk::train_assign_kernel<<<agrid, 256, cbytes, st>>>(d_x, n, d, s, dsub, cent.ptr, assign.ptr);
                    break;
            }
            VK_TRY_CUDA(cudaGetLastError());
            vk::train_sums_kernel<<<vk::KSUB / 8, 256, 0, st>>>(d_x, n, d, s, dsub, assign.ptr, sums.ptr, counts.ptr);
            VK_TRY_CUDA(cudaGetLastError());
            VK_TRY_CUDA(cudaMemcpyAsync(host_counts.data(), counts.ptr, vk::KSUB * sizeof(int), cudaMemcpyDeviceToHost,
                                        st));
            VK_TRY_CUDA(cudaStreamSynchronize(st));
            for (int c = 0; c < vk::KSUB; ++c) host_rows[c] = host_counts[c] == 0 ? (int64_t)(rng() % (uint64_t)n) : 0;
            VK_TRY_CUDA(cudaMemcpyAsync(rows.ptr, host_rows.data(), vk::KSUB * sizeof(int64_t), cudaMemcpyHostToDevice,
                                        st));
            vk::train_update_kernel<<<1, 256, 0, st>>>(d_x, d, s, dsub, sums.ptr, counts.ptr, rows.ptr, cent.ptr);
            VK_TRY_CUDA(cudaGetLastError());
        }
        VK_TRY_CUDA(cudaMemcpyAsync(centroids + (size_t)s * vk::KSUB * dsub, cent.ptr, cbytes, cudaMemcpyDeviceToHost,
                                    st));
    }
    VK_TRY_CUDA(cudaStreamSynchronize(st));
    return VK_OK;
}

int vk_gen_codes_device(int device, uint64_t seed, const uint32_t* cdf, int clusters, int m, int64_t row_first,
                        int64_t n, uint8_t* d_codes, void* stream) {
    if (!cdf || !d_codes || clusters <= 0 || m <= 0 || n < 0 || row_first < 0)
        return fail(VK_ERR_INVALID, "bad arguments");
    if (n == 0) return VK_OK;
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess) return fail(VK_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(guard.err));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t bytes = (size_t)clusters * m * vk::KSUB * sizeof(uint32_t);
    uint32_t* d_cdf = nullptr;
    VK_TRY_CUDA(cudaMallocAsync(&d_cdf, bytes, st));
    VK_TRY_CUDA(cudaMemcpyAsync(d_cdf, cdf, bytes, cudaMemcpyHostToDevice, st));
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    vk::gen_rows_kernel<<<grid_for(n * m, sms), 256, 0, st>>>(vk::mix64(seed), d_cdf, clusters, m, row_first, n,
                                                              d_codes);
    VK_TRY_CUDA(cudaGetLastError());
    VK_TRY_CUDA(cudaFreeAsync(d_cdf, st));
    return VK_OK;
}

}  // extern "C"

extern "C" int vk_search_noalloc(vk_index_t* ix, const float* d_queries, int64_t nq, int k, const vk_tuning_t* tuning,
                                 vk_neighbor_t* d_out, void* stream) {
    if (!ix) return fail(VK_ERR_INVALID, "index must not be NULL");
    if (k < 1 || k > 128 || (int64_t)k > ix->n) return fail(VK_ERR_INVALID, "k must be in [1, min(128, n)]");
    if (nq < 0) return fail(VK_ERR_INVALID, "nq must be >= 0");
    if (nq > 0 && (!d_queries || !d_out)) return fail(VK_ERR_INVALID, "queries and out must not be NULL");
    vk_tuning_t t;
    vk_tuning_default(&t);
    if (tuning) t = *tuning;
    VK_TRY(validate_tuning(&t));
    if (nq == 0) return VK_OK;
    if (nq > max_query_batch(ix))
        return fail(VK_ERR_INVALID, "nq %lld exceeds the batch limit %lld", (long long)nq, (long long)max_query_batch(ix));
    DeviceGuard guard(ix->device);
    if (guard.err != cudaSuccess) return fail(VK_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(guard.err));
    unsigned char* base = nullptr;
    VK_TRY(noalloc_scratch_address(ix->device, &base));
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    Plan p;
    VK_TRY(plan_scan(ix, nq, k, t, p));
    // Carve the array: LUTs | per-chunk lists | bounds | global lists | locks | half-LUT maxima | exponents |
    // counter + status.
    const WorkspaceBytes b = workspace_bytes(ix, nq, k, p);
    const size_t o_lut = 0;
    const size_t o_part = o_lut + align256(b.lut);
    const size_t o_bound = o_part + align256(b.part);
    const size_t o_glist = o_bound + align256(b.bound);
    const size_t o_glock = o_glist + align256(b.glist);
    const size_t o_qmax = o_glock + align256(b.glock);
    const size_t o_qexp = o_qmax + align256(b.qmax);
    const size_t o_flags = o_qexp + align256(b.qexp);
    const size_t need = o_flags + align256(2 * sizeof(int));
    if (need > VK_NOALLOC_SCRATCH_BYTES)
        return fail(VK_ERR_INVALID,
                    "this search needs %zu bytes of working memory; vk_search_noalloc has %zu (search fewer queries "
                    "per call)",
                    need, (size_t)VK_NOALLOC_SCRATCH_BYTES);
    Workspace w;
    w.lut = base + o_lut;
    w.part = reinterpret_cast<int2*>(base + o_part);
    w.bound = reinterpret_cast<uint32_t*>(base + o_bound);
    w.glist = reinterpret_cast<int2*>(base + o_glist);
    w.glock = reinterpret_cast<int*>(base + o_glock);
    w.qmax = reinterpret_cast<uint32_t*>(base + o_qmax);
    w.qexp = reinterpret_cast<int*>(base + o_qexp);
    w.flags = reinterpret_cast<int*>(base + o_flags);
    int* flags = w.flags;
    // The array keeps the previous call's contents: the status word starts at zero here, the work counter in
    // launch_search; the LUT kernels rewrite the LUTs and, for the pruned scan, reset the bounds, global lists
    // and locks.
    VK_TRY_CUDA(cudaMemsetAsync(flags + 1, 0, sizeof(int), st));
    VK_TRY(launch_search(ix, d_queries, nq, k, p, w, reinterpret_cast<int2*>(d_out), st, nullptr));
    int status = 0;
    VK_TRY_CUDA(cudaMemcpyAsync(&status, flags + 1, sizeof(int), cudaMemcpyDeviceToHost, st));
    VK_TRY_CUDA(cudaStreamSynchronize(st));
    if (status != 0) return status_error(status);
    return VK_OK;
}

// ------------------------------------------------------------------------------------------------ IVF
// An IVF index: the rows of each list in a contiguous, 64-aligned range of slots of an ordinary index (its lane
// placement then never mixes lists), the id of the row in each slot (-1 for padding), and the coarse centroids.
struct vk_ivf {
    vk_index* index = nullptr;
    int device = 0, nlist = 0, d = 0;
    int64_t n = 0;
    float* coarse = nullptr;      // [nlist][d]
    int64_t* list_off = nullptr;  // [nlist]
    int* list_rows = nullptr;     // [nlist]
    int32_t* ids = nullptr;       // [index->n_pad]
    DevBuf<float> queries;
    DevBuf<int2> out, by_list, item_pairs, part;
    DevBuf<int32_t> probes;
    DevBuf<int> counts, item_off, item_list, nitems;
    DevBuf<int64_t> pair_off;
    ~vk_ivf() {
        DeviceGuard g(device);
        queries.release();
        out.release();
        by_list.release();
        item_pairs.release();
        part.release();
        probes.release();
        counts.release();
        item_off.release();
        item_list.release();
        nitems.release();
        pair_off.release();
        if (coarse) cudaFree(coarse);
        if (list_off) cudaFree(list_off);
        if (list_rows) cudaFree(list_rows);
        if (ids) cudaFree(ids);
        delete index;
    }
};

namespace {

constexpr int kIvfMaxProbe = 128;

int64_t ivf_max_items(int64_t nq, int nprobe, int Q, int nlist) {
    return std::min<int64_t>(nq * nprobe, ceil_div(nq * nprobe, Q) + nlist);
}

// Largest query batch whose per-item LUTs stay within the LUT budget (at Q = 8, the larger case).
int64_t ivf_max_batch(const vk_ivf* ivf, int nprobe) {
    const int64_t lut_item = (int64_t)8 * ivf->index->m * vk::KSUB * 4;
    const int64_t items = std::max<int64_t>(1, std::min<int64_t>(65535, (int64_t)(kLutBudgetBytes / lut_item)) - ivf->nlist);
    return std::max<int64_t>(1, std::min<int64_t>(items * 4 / nprobe, 1 << 20));
}

// Probe selection, planning, per-item LUTs, the IVF scan and the merge of each query's nprobe lists into d_out.
int ivf_run(vk_ivf* ivf, const float* d_queries, int64_t nq, int k, int nprobe, const vk_tuning_t& t, int2* d_out,
            cudaStream_t st) {
    vk_index* ix = ivf->index;
    Plan p;
    VK_TRY(plan_scan(ix, nq, k, t, p, true));
    const int Q = p.Q, nlist = ivf->nlist;
    const int64_t pairs = nq * nprobe;
    const int64_t max_items = ivf_max_items(nq, nprobe, Q, nlist);
    if (max_items > 65535)  // one LUT block row per item (grid.y)
        return fail(VK_ERR_INVALID, "too many (query, list) pairs in one IVF batch (%lld work items)",
                    (long long)max_items);
    VK_TRY(ix->lut.ensure((size_t)max_items * Q * ix->m * vk::KSUB));
    VK_TRY(ix->bound.ensure((size_t)nq));
    VK_TRY(ix->glist.ensure((size_t)nq * k));
    VK_TRY(ix->glock.ensure((size_t)nq));
    VK_TRY(ivf->probes.ensure((size_t)pairs));
    VK_TRY(ivf->counts.ensure((size_t)2 * nlist));
    VK_TRY(ivf->pair_off.ensure((size_t)nlist + 1));
    VK_TRY(ivf->item_off.ensure((size_t)nlist + 1));
    VK_TRY(ivf->nitems.ensure(1));
    VK_TRY(ivf->by_list.ensure((size_t)pairs));
    VK_TRY(ivf->item_list.ensure((size_t)max_items));
    VK_TRY(ivf->item_pairs.ensure((size_t)max_items * Q));
    VK_TRY(ivf->part.ensure((size_t)pairs * k));
    const unsigned pgrid = grid_for(pairs, ix->sm_count);
    switch (s_for_k(nprobe)) {
        case 1: vk::ivf_probe_kernel<1><<<(unsigned)ceil_div(nq, 4), 128, 0, st>>>(d_queries, nq, ivf->d, ivf->coarse, nlist, nprobe, ivf->probes.ptr, ix->bound.ptr, ix->glist.ptr, ix->glock.ptr, k); break;
        case 2: vk::ivf_probe_kernel<2><<<(unsigned)ceil_div(nq, 4), 128, 0, st>>>(d_queries, nq, ivf->d, ivf->coarse, nlist, nprobe, ivf->probes.ptr, ix->bound.ptr, ix->glist.ptr, ix->glock.ptr, k); break;
        default: vk::ivf_probe_kernel<4><<<(unsigned)ceil_div(nq, 4), 128, 0, st>>>(d_queries, nq, ivf->d, ivf->coarse, nlist, nprobe, ivf->probes.ptr, ix->bound.ptr, ix->glist.ptr, ix->glock.ptr, k); break;
    }
    VK_TRY_CUDA(cudaGetLastError());
    VK_TRY_CUDA(cudaMemsetAsync(ivf->counts.ptr, 0, (size_t)2 * nlist * sizeof(int), st));
    vk::ivf_count_kernel<<<pgrid, 256, 0, st>>>(ivf->probes.ptr, pairs, ivf->counts.ptr);
    vk::ivf_plan_kernel<<<1, 1024, 0, st>>>(ivf->counts.ptr, nlist, Q, ivf->pair_off.ptr, ivf->item_off.ptr,
                                           ivf->nitems.ptr);
    vk::ivf_fill_kernel<<<pgrid, 256, 0, st>>>(ivf->probes.ptr, nq, nprobe, ivf->pair_off.ptr, ivf->counts.ptr + nlist,
                                              ivf->by_list.ptr);
    vk::ivf_items_kernel<<<(unsigned)std::min<int64_t>(nlist, (int64_t)ix->sm_count * 8), 256, 0, st>>>(
        ivf->pair_off.ptr, ivf->item_off.ptr, nlist, Q, ivf->by_list.ptr, ivf->item_list.ptr, ivf->item_pairs.ptr);
    VK_TRY_CUDA(cudaGetLastError());
    {
        const size_t smem = (size_t)Q * ix->dsub * sizeof(float);
        const void* fn = Q == 8 ? reinterpret_cast<const void*>(&vk::ivf_lut_kernel<8>)
                                : reinterpret_cast<const void*>(&vk::ivf_lut_kernel<4>);
        if (smem > 48 * 1024) VK_TRY_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        const float* cen = ix->centroids;
        const int2* pp = ivf->item_pairs.ptr;
        const int* ni = ivf->nitems.ptr;
        float* lut = ix->lut.ptr;
        int m = ix->m, dsub = ix->dsub;
        void* args[] = {(void*)&cen, (void*)&d_queries, (void*)&nq, (void*)&m, (void*)&dsub, (void*)&pp, (void*)&ni,
                        (void*)&lut};
        VK_TRY_CUDA(cudaLaunchKernel(fn, dim3(ix->m, (unsigned)max_items), dim3(vk::KSUB), args, smem, st));
    }
    {
        VK_TRY_CUDA(cudaMemsetAsync(ix->flags, 0, sizeof(int), st));
        vk::ScanArgs a{};
        a.codes = ix->codes;
        a.perm = ix->perm;
        a.lut = ix->lut.ptr;
        a.part = ivf->part.ptr;
        a.work_counter = ix->flags;
        a.status = ix->flags + 1;
        a.bound = ix->bound.ptr;
        a.glist = ix->glist.ptr;
        a.glock = ix->glock.ptr;
        a.n = ix->n;
        a.n_pad = ix->n_pad;
        a.chunk_len = ix->n_pad;
        a.first_len = ix->n_pad;
        a.id_base = 0;
        a.m = ix->m;
        a.W = ix->W;
        a.nq = (int)nq;
        a.groups = 1;
        a.group_window = 1;
        a.chunks = 1;
        a.k = k;
        a.stages = p.stages;
        a.merge_slots = p.merge_slots;
        a.wait_budget = ix->wait_budget;
        a.ivf_item_list = ivf->item_list.ptr;
        a.ivf_item_pairs = ivf->item_pairs.ptr;
        a.ivf_list_off = ivf->list_off;
        a.ivf_list_rows = ivf->list_rows;
        a.ivf_ids = ivf->ids;
        a.ivf_nitems = ivf->nitems.ptr;
        a.nprobe = nprobe;
        void* args[] = {(void*)&a};
        VK_TRY_CUDA(cudaLaunchKernel(p.fn, dim3(p.grid), dim3(p.threads), args, p.smem, st));
    }
    {
        const bool wide = nq <= ix->sm_count && (int64_t)nprobe * k >= 256;
        const void* fn = wide ? merge_wide_kernel_ptr(p.S) : merge_kernel_ptr(p.S);
        const int2* in = ivf->part.ptr;
        const int* qexp = nullptr;
        int lists = nprobe, k_in = k, kk = k;
        int64_t qstride = (int64_t)nprobe * k, lstride = k;
        void* args[] = {(void*)&in, (void*)&nq, (void*)&lists, (void*)&k_in, (void*)&qstride, (void*)&lstride,
                        (void*)&kk, (void*)&d_out, (void*)&qexp};
        if (wide)
            VK_TRY_CUDA(cudaLaunchKernel(fn, dim3((unsigned)nq), dim3(256), args, 0, st));
        else
            VK_TRY_CUDA(cudaLaunchKernel(fn, dim3((unsigned)ceil_div(nq, 4)), dim3(128), args, 0, st));
    }
    return VK_OK;
}

int ivf_check(const vk_ivf* ivf, int64_t nq, int k, int nprobe) {
    if (!ivf) return fail(VK_ERR_INVALID, "IVF index must not be NULL");
    if (k < 1 || k > 128) return fail(VK_ERR_INVALID, "k must be in [1, 128]");
    if (nprobe < 1 || nprobe > std::min(kIvfMaxProbe, ivf->nlist))
        return fail(VK_ERR_INVALID, "nprobe must be in [1, min(128, nlist)]");
    if (nq < 0) return fail(VK_ERR_INVALID, "nq must be >= 0");
    return VK_OK;
}

}  // namespace

extern "C" {

int vk_ivf_create(int device, const float* centroids, int m, int dsub, const uint8_t* codes, int64_t n,
                  const float* coarse, int nlist, const int32_t* list_of, vk_ivf_t** out) {
    if (!out) return fail(VK_ERR_INVALID, "out must not be NULL");
    *out = nullptr;
    if (!centroids || !codes || !coarse || !list_of) return fail(VK_ERR_INVALID, "pointers must not be NULL");
    if (m <= 0 || dsub <= 0 || n <= 0 || nlist <= 0) return fail(VK_ERR_INVALID, "bad sizes");
    if (n >= (int64_t)std::numeric_limits<int>::max()) return fail(VK_ERR_INVALID, "n must fit in int32 ids");
    std::vector<int64_t> cnt((size_t)nlist, 0);
    for (int64_t i = 0; i < n; ++i) {
        if (list_of[i] < 0 || list_of[i] >= nlist) return fail(VK_ERR_INVALID, "row %lld has list %d outside [0, %d)",
                                                                (long long)i, list_of[i], nlist);
        ++cnt[(size_t)list_of[i]];
    }
    // 64-aligned list ranges, rows in id order within a list, padding slots with id -1
    std::vector<int64_t> off((size_t)nlist);
    std::vector<int> rows((size_t)nlist);
    int64_t slots = 0;
    for (int l = 0; l < nlist; ++l) {
        off[(size_t)l] = slots;
        rows[(size_t)l] = (int)(ceil_div(cnt[(size_t)l], vk::PLACE_WINDOW) * vk::PLACE_WINDOW);
        slots += rows[(size_t)l];
    }
    if (slots >= (int64_t)std::numeric_limits<int>::max() - 128) return fail(VK_ERR_INVALID, "too many rows");
    const int64_t slots_alloc = std::max<int64_t>(slots, vk::PLACE_WINDOW);  // an index needs at least one row
    std::vector<uint8_t> slot_codes((size_t)slots_alloc * m, 0);
    std::vector<int32_t> slot_ids((size_t)ceil_div(slots_alloc, 128) * 128, -1);
    std::vector<int64_t> fill((size_t)nlist, 0);
    for (int64_t i = 0; i < n; ++i) {
        const int l = list_of[i];
        const int64_t pos = off[(size_t)l] + fill[(size_t)l]++;
        std::memcpy(slot_codes.data() + pos * m, codes + i * m, (size_t)m);
        slot_ids[(size_t)pos] = (int32_t)i;
    }
    auto* ivf = new vk_ivf();
    ivf->device = device;
    ivf->nlist = nlist;
    ivf->d = m * dsub;
    ivf->n = n;
    int rc = vk_index_create(device, centroids, m, dsub, slot_codes.data(), slots_alloc, 0, &ivf->index);
    if (rc == VK_OK) {
        DeviceGuard guard(device);
        cudaError_t e = cudaMalloc(&ivf->coarse, (size_t)nlist * ivf->d * sizeof(float));
        if (e == cudaSuccess) e = cudaMalloc(&ivf->list_off, (size_t)nlist * sizeof(int64_t));
        if (e == cudaSuccess) e = cudaMalloc(&ivf->list_rows, (size_t)nlist * sizeof(int));
        if (e == cudaSuccess) e = cudaMalloc(&ivf->ids, (size_t)ivf->index->n_pad * sizeof(int32_t));
        if (e == cudaSuccess)
            e = cudaMemcpy(ivf->coarse, coarse, (size_t)nlist * ivf->d * sizeof(float), cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(ivf->list_off, off.data(), (size_t)nlist * sizeof(int64_t), cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(ivf->list_rows, rows.data(), (size_t)nlist * sizeof(int), cudaMemcpyHostToDevice);
        if (e == cudaSuccess)
            e = cudaMemcpy(ivf->ids, slot_ids.data(), (size_t)ivf->index->n_pad * sizeof(int32_t), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) rc = fail(VK_ERR_CUDA, "IVF index build: %s", cudaGetErrorString(e));
    }
    if (rc != VK_OK) {
        delete ivf;
        return rc;
    }
    *out = ivf;
    return VK_OK;
}

int vk_ivf_destroy(vk_ivf_t* ivf) {
    delete ivf;
    return VK_OK;
}

int vk_ivf_info(const vk_ivf_t* ivf, int64_t* n, int* nlist, int64_t* slots) {
    if (!ivf) return fail(VK_ERR_INVALID, "IVF index must not be NULL");
    if (n) *n = ivf->n;
    if (nlist) *nlist = ivf->nlist;
    if (slots) *slots = ivf->index->n;
    return VK_OK;
}

int vk_ivf_search_device(vk_ivf_t* ivf, const float* d_queries, int64_t nq, int k, int nprobe,
                         const vk_tuning_t* tuning, vk_neighbor_t* d_out, void* stream) {
    VK_TRY(ivf_check(ivf, nq, k, nprobe));
    if (nq > 0 && (!d_queries || !d_out)) return fail(VK_ERR_INVALID, "queries and out must not be NULL");
    if (nq > ivf_max_batch(ivf, nprobe))
        return fail(VK_ERR_INVALID, "nq %lld exceeds the IVF batch limit %lld for nprobe %d", (long long)nq,
                    (long long)ivf_max_batch(ivf, nprobe), nprobe);
    vk_tuning_t t;
    vk_tuning_default(&t);
    if (tuning) t = *tuning;
    VK_TRY(validate_tuning(&t));
    if (nq == 0) return VK_OK;
    DeviceGuard guard(ivf->device);
    if (guard.err != cudaSuccess) return fail(VK_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(guard.err));
    return ivf_run(ivf, d_queries, nq, k, nprobe, t, reinterpret_cast<int2*>(d_out), static_cast<cudaStream_t>(stream));
}

int vk_ivf_search(vk_ivf_t* ivf, const float* queries, int64_t nq, int k, int nprobe, const vk_tuning_t* tuning,
                  vk_neighbor_t* out, vk_timings_t* timings) {
    VK_TRY(ivf_check(ivf, nq, k, nprobe));
    if (nq > 0 && (!queries || !out)) return fail(VK_ERR_INVALID, "queries and out must not be NULL");
    vk_tuning_t t;
    vk_tuning_default(&t);
    if (tuning) t = *tuning;
    VK_TRY(validate_tuning(&t));
    if (timings) *timings = vk_timings_t{};
    if (nq == 0) return VK_OK;
    DeviceGuard guard(ivf->device);
    if (guard.err != cudaSuccess) return fail(VK_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(guard.err));
    vk_index* ix = ivf->index;
    cudaStream_t st = ix->stream;
    const int64_t batch = std::min(nq, ivf_max_batch(ivf, nprobe));
    VK_TRY(ivf->queries.ensure((size_t)batch * ivf->d));
    VK_TRY(ivf->out.ensure((size_t)batch * k));
    vk_timings_t acc{};
    cudaEvent_t* ev = ix->ev;
    for (int64_t q0 = 0; q0 < nq; q0 += batch) {
        const int64_t b = std::min(batch, nq - q0);
        VK_TRY_CUDA(cudaEventRecord(ev[0], st));
        VK_TRY_CUDA(cudaMemcpyAsync(ivf->queries.ptr, queries + q0 * ivf->d, (size_t)b * ivf->d * sizeof(float),
                                    cudaMemcpyHostToDevice, st));
        VK_TRY_CUDA(cudaEventRecord(ev[1], st));
        VK_TRY(ivf_run(ivf, ivf->queries.ptr, b, k, nprobe, t, ivf->out.ptr, st));
        VK_TRY_CUDA(cudaEventRecord(ev[2], st));
        VK_TRY_CUDA(cudaMemcpyAsync(out + q0 * k, ivf->out.ptr, (size_t)b * k * sizeof(int2), cudaMemcpyDeviceToHost, st));
        VK_TRY_CUDA(cudaEventRecord(ev[3], st));
        VK_TRY_CUDA(cudaEventSynchronize(ev[3]));
        float ms[3];
        for (int i = 0; i < 3; ++i) VK_TRY_CUDA(cudaEventElapsedTime(&ms[i], ev[i], ev[i + 1]));
        acc.transfer_ms += ms[0] + ms[2];
        acc.scan_ms += ms[1];
    }
    VK_TRY(read_status(ix, st));
    if (timings) *timings = acc;
    return VK_OK;
}

int vk_ivf_sync(vk_ivf_t* ivf, void* stream) {
    if (!ivf) return fail(VK_ERR_INVALID, "IVF index must not be NULL");
    DeviceGuard guard(ivf->device);
    return read_status(ivf->index, static_cast<cudaStream_t>(stream));
}

int vk_ivf_assign_device(int device, const float* d_x, int64_t n, int d, const float* d_coarse, int nlist,
                         int32_t* d_list_of, void* stream) {
    if (!d_x || !d_coarse || !d_list_of) return fail(VK_ERR_INVALID, "pointers must not be NULL");
    if (n < 0 || d <= 0 || nlist <= 0) return fail(VK_ERR_INVALID, "bad sizes");
    if (n == 0) return VK_OK;
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess) return fail(VK_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(guard.err));
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    vk::ivf_assign_kernel<<<grid_for(n, sms), 256, 0, static_cast<cudaStream_t>(stream)>>>(d_x, n, d, d_coarse, nlist,
                                                                                          d_list_of);
    VK_TRY_CUDA(cudaGetLastError());
    return VK_OK;
}

}  // extern "C"
