// VecKern-B200 kernels (sm_100a). Host dispatch lives in vk_abi.cu.
//
// Data layouts in HBM
//   centroids  [m][256][dsub] fp32 (the reference's layout, include/veckern/pq.hpp:20-24)
//   codes      16-byte-word interleaved per 32 vectors: uint4 word ((g * W + w) * 32 + l) holds sub-codes
//              16w .. 16w+15 of vector 32g + l, W = ceil(m / 16), sub-codes >= m and rows >= n are zero; rows
//              padded to a multiple of 128. A warp reading word w of its 32 vectors reads 512 contiguous bytes.
//   LUT        per query group of Q queries, contiguous, already in the shared-memory layout of the scan:
//              Q = 1: [s][c]; Q = 2: [s][c][2]; Q = 4: [s][c][4]; Q = 8: two [s][c][4] tables (queries 0-3, 4-7).
//              One code byte then fetches all Q queries' entries with one LDS.32/64/128 (two LDS.128 for Q = 8).
//              Half-precision LUTs (Q = 4 or 8): [s][c][Q] halves, one LDS.64 / LDS.128 per code byte.
//              4-bit PQ (16 centroids per sub-space, Q = 4 or 8): [s][q / 2][c] float2 pairs: one sub-space table
//              of two queries is 16 entries x 8 bytes = 128 bytes, one per bank pair, so a warp's LDS.64 into it
//              never conflicts (2 wavefronts for 32 rows x 2 queries).
//   4-bit codes sub-code s of a row in nibble s % 2 (low first) of byte s / 2; the bytes interleaved in 16-byte
//              words as above (32 sub-codes per word).
//   partials   [query][chunk][k] (dist, id) lists, merged by merge_kernel.
#pragma once
#include <cfloat>
#include <cstdint>
#include <cuda_fp16.h>

#include "vk_device.cuh"
#include "warp_topk.cuh"

namespace vk {

// ------------------------------------------------------------------------------------------------ LUT builder
// Block (s, g) of 256 threads: thread c computes centroid c of sub-space s for the Q queries of group g.
// Arithmetic of the reference's l2sq (include/veckern/common.hpp:27-34): diff = q - c, acc += diff * diff in
// j order, each operation rounded on its own (__fsub_rn / __fmul_rn / __fadd_rn: no FMA contraction).
// Padded query slots (index >= nq) get 0. `bound` (optional): the pruned scan's per-query bounds, reset to +inf.
// `pairs` (IVF): the group's queries are pairs[g * Q + qq].x (-1: padding) instead of g * Q + qq.
template <int Q>
__device__ __forceinline__ void lut_entries(const float* __restrict__ centroids, const float* __restrict__ queries,
                                            int64_t nq, int m, int dsub, uint32_t* __restrict__ bound,
                                            int2* __restrict__ glist, int* __restrict__ glock, int k, float* acc,
                                            const int2* __restrict__ pairs = nullptr) {
    extern __shared__ float qsub[];  // [Q][dsub]
    const int s = blockIdx.x, g = blockIdx.y, c = threadIdx.x;
    const int64_t d = (int64_t)m * dsub;
    auto query_of = [&](int qq) -> int64_t {
        const int64_t qi = pairs ? (int64_t)pairs[(int64_t)g * Q + qq].x : (int64_t)g * Q + qq;
        return qi >= 0 && qi < nq ? qi : -1;
    };
    for (int t = threadIdx.x; t < Q * dsub; t += blockDim.x) {
        const int qq = t / dsub, j = t - qq * dsub;
        const int64_t qi = query_of(qq);
        qsub[t] = qi >= 0 ? queries[qi * d + (int64_t)s * dsub + j] : 0.f;
    }
    if (bound && s == 0) {  // reset the pruned scan's per-query state: bound +inf, empty global list, lock free
        for (int t = c; t < Q * k; t += blockDim.x) {
            const int64_t qi = (int64_t)g * Q + t / k;
            if (qi < nq) glist[qi * k + t % k] = make_int2(0x7f800000, SENTINEL_ID);
        }
        if (c < Q && (int64_t)g * Q + c < nq) {
            bound[(int64_t)g * Q + c] = 0x7f800000u;
            glock[(int64_t)g * Q + c] = 0;
        }
    }
    __syncthreads();
    const float* cen = centroids + ((int64_t)s * KSUB + c) * dsub;
#pragma unroll
    for (int qq = 0; qq < Q; ++qq) acc[qq] = 0.f;
    for (int j = 0; j < dsub; ++j) {
        const float cj = cen[j];
#pragma unroll
        for (int qq = 0; qq < Q; ++qq) {
            const float diff = __fsub_rn(qsub[qq * dsub + j], cj);
            acc[qq] = __fadd_rn(acc[qq], __fmul_rn(diff, diff));
        }
    }
#pragma unroll
    for (int qq = 0; qq < Q; ++qq)
        if (query_of(qq) < 0) acc[qq] = 0.f;
}

// grid (m, groups), block 256: the fp32 LUT of each query group in the scan layout.
template <int Q>
__global__ void __launch_bounds__(256) lut_kernel(const float* __restrict__ centroids,
                                                  const float* __restrict__ queries, int64_t nq, int m, int dsub,
                                                  float* __restrict__ lut, uint32_t* __restrict__ bound,
                                                  int2* __restrict__ glist, int* __restrict__ glock, int k) {
    const int s = blockIdx.x, g = blockIdx.y, c = threadIdx.x;
    float acc[Q];
    lut_entries<Q>(centroids, queries, nq, m, dsub, bound, glist, glock, k, acc);
    float* out = lut + (int64_t)g * Q * m * KSUB;
    const int e = s * KSUB + c;
    if constexpr (Q == 1) {
        out[e] = acc[0];
    } else if constexpr (Q == 2) {
        reinterpret_cast<float2*>(out)[e] = make_float2(acc[0], acc[1]);
    } else if constexpr (Q == 4) {
        reinterpret_cast<float4*>(out)[e] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    } else {
        reinterpret_cast<float4*>(out)[e] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        reinterpret_cast<float4*>(out)[m * KSUB + e] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
}

// grid (m, max items), block 256: the fp32 LUT of each IVF work item (the queries of its pair slots), in the scan
// layout; blocks past the item count (known only on the device) return at once.
template <int Q>
__global__ void __launch_bounds__(256) ivf_lut_kernel(const float* __restrict__ centroids,
                                                      const float* __restrict__ queries, int64_t nq, int m, int dsub,
                                                      const int2* __restrict__ pairs, const int* __restrict__ nitems,
                                                      float* __restrict__ lut) {
    const int s = blockIdx.x, g = blockIdx.y, c = threadIdx.x;
    if (g >= __ldg(nitems)) return;  // block-uniform
    float acc[Q];
    lut_entries<Q>(centroids, queries, nq, m, dsub, nullptr, nullptr, nullptr, 0, acc, pairs);
    float* out = lut + (int64_t)g * Q * m * KSUB;
    const int e = s * KSUB + c;
    if constexpr (Q == 4) {
        reinterpret_cast<float4*>(out)[e] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    } else {
        static_assert(Q == 8, "IVF items hold 4 or 8 queries");
        reinterpret_cast<float4*>(out)[e] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        reinterpret_cast<float4*>(out)[m * KSUB + e] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
}

// ---- 4-bit PQ: 16 centroids per sub-space, centroids [m][16][dsub]
constexpr int KSUB4 = 16;

// grid (ceil(m / 16), groups), block 256: thread t computes centroid t % 16 of sub-space 16 * blockIdx.x + t / 16
// for the Q queries of group g, with the arithmetic of lut_entries, and writes the scan layout [s][q / 2][c] of
// float2 pairs. Blocks with blockIdx.x == 0 reset the pruned scan's per-query state (bound, global list, lock).
template <int Q>
__global__ void __launch_bounds__(256) lut4_kernel(const float* __restrict__ centroids,
                                                   const float* __restrict__ queries, int64_t nq, int m, int dsub,
                                                   float* __restrict__ lut, uint32_t* __restrict__ bound,
                                                   int2* __restrict__ glist, int* __restrict__ glock, int k) {
    static_assert(Q % 2 == 0, "4-bit LUT entries hold query pairs");
    extern __shared__ float qsub4[];  // [Q][16][dsub]: the group's query sub-vectors of the block's 16 sub-spaces
    const int s0 = blockIdx.x * 16, g = blockIdx.y;
    const int ns = min(16, m - s0);
    const int64_t d = (int64_t)m * dsub;
    for (int t = threadIdx.x; t < Q * ns * dsub; t += blockDim.x) {
        const int qq = t / (ns * dsub), r = t - qq * ns * dsub;
        const int64_t qi = (int64_t)g * Q + qq;
        qsub4[qq * 16 * dsub + r] = qi < nq ? queries[qi * d + (int64_t)s0 * dsub + r] : 0.f;
    }
    if (bound && blockIdx.x == 0) {
        for (int t = threadIdx.x; t < Q * k; t += blockDim.x) {
            const int64_t qi = (int64_t)g * Q + t / k;
            if (qi < nq) glist[qi * k + t % k] = make_int2(0x7f800000, SENTINEL_ID);
        }
        if (threadIdx.x < Q && (int64_t)g * Q + threadIdx.x < nq) {
            bound[(int64_t)g * Q + threadIdx.x] = 0x7f800000u;
            glock[(int64_t)g * Q + threadIdx.x] = 0;
        }
    }
    __syncthreads();
    const int sl = threadIdx.x >> 4, c = threadIdx.x & 15, s = s0 + sl;
    if (sl >= ns) return;
    const float* cen = centroids + ((int64_t)s * KSUB4 + c) * dsub;
    float acc[Q];
#pragma unroll
    for (int qq = 0; qq < Q; ++qq) acc[qq] = 0.f;
    for (int j = 0; j < dsub; ++j) {
        const float cj = cen[j];
#pragma unroll
        for (int qq = 0; qq < Q; ++qq) {
            const float diff = __fsub_rn(qsub4[(qq * 16 + sl) * dsub + j], cj);
            acc[qq] = __fadd_rn(acc[qq], __fmul_rn(diff, diff));
        }
    }
    float2* out = reinterpret_cast<float2*>(lut + (int64_t)g * Q * m * KSUB4);
#pragma unroll
    for (int qp = 0; qp < Q / 2; ++qp) {
        const bool v0 = (int64_t)g * Q + 2 * qp < nq, v1 = (int64_t)g * Q + 2 * qp + 1 < nq;
        out[((int64_t)s * (Q / 2) + qp) * KSUB4 + c] = make_float2(v0 ? acc[2 * qp] : 0.f, v1 ? acc[2 * qp + 1] : 0.f);
    }
}

// ---- half-precision LUTs (lut_precision = VK_LUT_F16)
// Per query: T[s][c] = the fp32 entry above; M = max over (s, c) of T; e = the power of two that puts M in
// [2^14, 2^15) (lut_h16_exponent); entry = T * 2^e rounded to half (round to nearest even). The scan sums the
// halves in fp32 in sub-space order exactly as the fp32 path sums fp32 entries, and reports sum * 2^-e: both
// scalings are exact, so ordering by the scaled sums is ordering by the reported distances.
// Exponent of the per-query scale from the bits of the query's largest entry (entries are >= +0).
__host__ __device__ inline int lut_h16_exponent(uint32_t max_bits) {
    const int ef = (int)((max_bits >> 23) & 0xffu);
    if (max_bits == 0u || ef == 255) return 0;  // all entries zero (or not finite: outside the input contract)
    if (ef == 0) return 64;                     // subnormal maximum: the largest scale
    const int e = 15 - (ef - 126);              // M = f * 2^(ef - 126), f in [0.5, 1)
    return e < -64 ? -64 : e > 64 ? 64 : e;
}
// 2^e as a float, for |e| <= 64 (exact).
__device__ __forceinline__ float exp2_int(int e) { return __int_as_float((int)((uint32_t)(127 + e) << 23)); }

// Pass 0: each query's largest entry, as float bits (atomicMax on the bits orders non-negative floats); qmax
// zeroed before the launch.
template <int Q>
__global__ void __launch_bounds__(256) lut_max_kernel(const float* __restrict__ centroids,
                                                      const float* __restrict__ queries, int64_t nq, int m, int dsub,
                                                      uint32_t* __restrict__ qmax) {
    __shared__ uint32_t red[Q];
    const int g = blockIdx.y;
    if (threadIdx.x < Q) red[threadIdx.x] = 0u;
    float acc[Q];
    lut_entries<Q>(centroids, queries, nq, m, dsub, nullptr, nullptr, nullptr, 0, acc);
#pragma unroll
    for (int qq = 0; qq < Q; ++qq) {
        const uint32_t w = __reduce_max_sync(FULL, __float_as_uint(acc[qq]));
        if ((threadIdx.x & (WARP - 1)) == 0) atomicMax(red + qq, w);
    }
    __syncthreads();
    if (threadIdx.x < Q && (int64_t)g * Q + threadIdx.x < nq) atomicMax(qmax + (int64_t)g * Q + threadIdx.x, red[threadIdx.x]);
}

// Pass 1: the scaled half entries in the scan layout [s][c][Q] (Q = 4 or 8); blocks of sub-space 0 also store
// each query's exponent and reset the pruned scan's state.
template <int Q>
__global__ void __launch_bounds__(256) lut_h16_kernel(const float* __restrict__ centroids,
                                                      const float* __restrict__ queries, int64_t nq, int m, int dsub,
                                                      const uint32_t* __restrict__ qmax, int* __restrict__ qexp,
                                                      __half* __restrict__ lut, uint32_t* __restrict__ bound,
                                                      int2* __restrict__ glist, int* __restrict__ glock, int k) {
    static_assert(Q == 4 || Q == 8, "half LUTs are built for 4 or 8 queries per group");
    const int s = blockIdx.x, g = blockIdx.y, c = threadIdx.x;
    float acc[Q];
    lut_entries<Q>(centroids, queries, nq, m, dsub, bound, glist, glock, k, acc);
    __half h[Q];
#pragma unroll
    for (int qq = 0; qq < Q; ++qq) {
        const int64_t qi = (int64_t)g * Q + qq;
        const int e = qi < nq ? lut_h16_exponent(qmax[qi]) : 0;
        if (s == 0 && c == 0 && qi < nq) qexp[qi] = e;
        h[qq] = __float2half_rn(__fmul_rn(acc[qq], exp2_int(e)));
    }
    __half* out = lut + ((int64_t)g * m * KSUB + (int64_t)s * KSUB + c) * Q;
    if constexpr (Q == 4) {
        uint2 v;
        v.x = (uint32_t)__half_as_ushort(h[0]) | ((uint32_t)__half_as_ushort(h[1]) << 16);
        v.y = (uint32_t)__half_as_ushort(h[2]) | ((uint32_t)__half_as_ushort(h[3]) << 16);
        *reinterpret_cast<uint2*>(out) = v;
    } else {
        uint4 v;
        v.x = (uint32_t)__half_as_ushort(h[0]) | ((uint32_t)__half_as_ushort(h[1]) << 16);
        v.y = (uint32_t)__half_as_ushort(h[2]) | ((uint32_t)__half_as_ushort(h[3]) << 16);
        v.z = (uint32_t)__half_as_ushort(h[4]) | ((uint32_t)__half_as_ushort(h[5]) << 16);
        v.w = (uint32_t)__half_as_ushort(h[6]) | ((uint32_t)__half_as_ushort(h[7]) << 16);
        *reinterpret_cast<uint4*>(out) = v;
    }
}

// ------------------------------------------------------------------------------------------------ fused scan
constexpr int COOP_MAX_PEERS = 15;  // shards of one cooperative search, besides this one

struct ScanArgs {
    const uint4* codes;  // interleaved layout, n_pad rows
    const uint8_t* perm; // [n_pad] lane placement: position p holds row (p & ~63) + perm[p]
    const float* lut;    // groups x (Q * m * 256), scan layout
    int2* part;          // [nq][chunks][k] partial lists (dist bits, id)
    int* work_counter;   // dynamic work-item counter, zero before launch
    int* status;         // kernel status word (ERR_* bits)
    uint32_t* bound;     // [nq] float bits: running upper bound of each query's k-th distance (pruned scan)
    int2* glist;         // [nq][k] best (dist, id) pairs of the chunks merged so far (pruned scan)
    int* glock;          // [nq] try-locks of glist (0 = free)
    int64_t n, n_pad;    // valid rows, padded rows (multiple of 128)
    int64_t chunk_len;   // rows per chunk, a multiple of 32 * ILP
    int64_t first_len;   // rows of chunk 0 (a multiple of 32 * ILP, <= chunk_len); chunk c > 0 starts at
                         // first_len + (c - 1) * chunk_len
    int64_t id_base;     // global id = id_base + row
    int m, W, nq, groups, chunks, k, stages;
    int group_window;       // flat search: items run window by window of this many query groups, chunk-major inside
                            // a window, so that the window's LUTs and the current chunk's codes stay in L2 together
    int merge_slots;        // 1 or Q (see scan_smem_plan)
    long long wait_budget;  // SM cycles a bounded wait may take
    // Cooperative sharded search (pruned scan): xb = this shard's exchange array, xpeer = the other shards'
    // (peer or IPC-mapped device memory); entries (epoch << 32) | ~bound_bits, so atomicMax keeps the newest
    // search's smallest bound; a stale epoch reads as +inf. npeers = 0 and xb = nullptr: no exchange.
    unsigned long long* xb;
    unsigned long long* xpeer[COOP_MAX_PEERS];
    int npeers;
    uint32_t epoch;
    // IVF search (scan_kernel with IVF = true): work items come from an item table instead of (chunk, group).
    const int* ivf_item_list;      // [items] the list an item scans
    const int2* ivf_item_pairs;    // [items][Q] (query, probe slot) of the item's queries; (-1, -1) pads
    const int64_t* ivf_list_off;   // [nlist] first position of each list (a multiple of 64)
    const int* ivf_list_rows;      // [nlist] positions of each list (a multiple of 64)
    const int32_t* ivf_ids;        // [n_pad] id of the row in each position's slot, -1 for padding
    const int* ivf_nitems;         // number of items (written by the planning kernels)
    int nprobe;
};

// Bound of query qi from the other shards of a cooperative search (+inf bits when there is none yet), in two steps
// so that a caller can issue the load early and combine it later: coop_load reads the exchange entry (0 without an
// exchange), coop_decode turns it into float bits.
__device__ __forceinline__ unsigned long long coop_load(const ScanArgs& a, int64_t qi) {
    return a.xb ? __ldcg(a.xb + qi) : 0ull;
}
__device__ __forceinline__ uint32_t coop_decode(const ScanArgs& a, unsigned long long v) {
    return a.xb && (uint32_t)(v >> 32) == a.epoch ? 0xffffffffu - (uint32_t)v : 0x7f800000u;
}
__device__ __forceinline__ uint32_t coop_bound(const ScanArgs& a, int64_t qi) { return coop_decode(a, coop_load(a, qi)); }
// Offers a lowered bound of query qi to the other shards (posted system-scope atomics over NVLink). The loop stays
// rolled: unrolled at every publishing site it made the scan kernel's code a fifth larger (instruction-cache misses
// in the per-tile loop).
__device__ __forceinline__ void coop_publish(const ScanArgs& a, int64_t qi, uint32_t bits) {
    const unsigned long long v = ((unsigned long long)a.epoch << 32) | (unsigned long long)(0xffffffffu - bits);
#pragma unroll 1
    for (int p = 0; p < a.npeers; ++p) atomicMax_system(a.xpeer[p] + qi, v);
}

// Shared-memory plan of scan_kernel; host and device compute it with the same function. merge_slots: how many
// queries' warp lists the item-end merge stages at once (1 or Q).
struct ScanSmem {
    uint32_t lut, stage, scratch, queue, ring, bars, flags, total, tile_bytes, stage_bytes, lut_bytes;
};
// Pruned scan at m = 16: a (row, query) pair that survives phase A is queued together with its partial sum and its
// remaining sub-codes (16 bytes), in a per-warp queue that persists across the item's tiles, so that phase B runs in
// full batches of 32 pairs and the tile's stage buffer is released as soon as its survivors are queued. A tile with
// more than CARRY_QWIDE survivors is finished with the Q-wide lookups instead (it always fits: full batches leave
// fewer than 32 entries queued between tiles). Other m keep a per-tile queue of row indices into the stage buffer.
constexpr int CARRY_CAP = 96;
constexpr int CARRY_QWIDE = CARRY_CAP - 32;
constexpr int CARRY_DEPTH0 = 8;  // queued pairs resume at sub-space 8 + 2 * (their 2-bit depth field)
__host__ __device__ constexpr bool carry_queue(int m) { return m == 16; }
// Rows of a pruned chunk, relative to its first 64-row window: 24 bits of a queue entry (with the query, 3 bits,
// and the phase-A depth, 2 bits).
constexpr int64_t CARRY_MAX_CHUNK_ROWS = int64_t(1) << 23;

// p4: 4-bit PQ (16-entry sub-space tables, W words of 32 sub-codes per row, no carry queue).
__host__ __device__ inline ScanSmem scan_smem_plan(int Q, int m, int W, int ilp, int nw, int stages, int k,
                                                   bool prune, int merge_slots, bool h16, bool ivf = false,
                                                   bool p4 = false) {
    auto up = [](uint32_t x, uint32_t a) { return (x + a - 1) / a * a; };
    ScanSmem p;
    p.lut_bytes = (uint32_t)Q * m * (p4 ? KSUB4 : KSUB) * (h16 ? 2u : 4u);
    p.tile_bytes = (uint32_t)ilp * W * 512u;
    // codes, then the tile's placement bytes, then (IVF) the ids of the tile's 64-row window
    p.stage_bytes = p.tile_bytes + (uint32_t)ilp * 32u + (ivf ? 256u : 0u);
    p.lut = 0;
    p.stage = up(p.lut_bytes, 128);
    p.scratch = up(p.stage + (uint32_t)nw * stages * p.stage_bytes, 128);
    p.queue = up(p.scratch + (uint32_t)merge_slots * nw * k * 8u, 16);
    // m = 16: the carry queue (CARRY_CAP 16-byte entries per warp); other m: at most half a tile's (row, query)
    // pairs, 8 bytes each (with more survivors the tile is finished in full)
    const uint32_t queue_bytes = !prune ? 0u : carry_queue(m) && !p4 ? (uint32_t)nw * CARRY_CAP * 16u
                                                                     : (uint32_t)nw * 16u * ilp * Q * 8u;
    p.ring = up(p.queue + queue_bytes, 16);
    p.bars = up(p.ring + (uint32_t)nw * stages * 4u, 16);
    p.flags = p.bars + (uint32_t)(nw * stages + 1) * 8u;
    p.total = up(p.flags + 16 + 64, 128);  // s_item, s_abort, s_tile; the item's (query, probe slot) pairs
    return p;
}

// Depth of phase A in the pruned scan: sub-spaces computed for every row before the rows are tested against the
// bounds. A tile is first tested at prune_first(m); while more than 1/PRUNE_DEEPEN of its (row, query) pairs
// survive, phase A goes two sub-spaces deeper, up to prune_last(m): below that share, finishing the survivors one
// pair per lane costs less than two more Q-wide sub-spaces of every row. Survival curves of partial sums differ
// between data sets (on the clustered SIFT-shaped mixture at m = 16, 0.15% of the pairs survive 8 sub-spaces; on
// the Dirichlet-generated codes 72% survive 8, 20% survive 10 and 1.3% survive 12), hence the per-tile choice.
// Lane placement: within each window of PLACE_WINDOW rows (whole windows below n only), the index stores rows in
// an order chosen at build time so that the rows one quarter-warp serves in a 16-byte LUT fetch fall into different
// shared-memory bank groups as often as possible (place_rows_kernel). perm[p] gives the row of position p within
// its window; ids, and so results, are those of the rows.
constexpr int PLACE_WINDOW = 64;

// 4-bit codes (p4) carry half the bits per sub-space: their first vote comes after half of the sub-spaces (at config 1
// with m = 32, first votes after 12 / 16 / 20 sub-spaces measured 4.18 / 3.36 / 3.50 ms).
__host__ __device__ constexpr int prune_first(int m, bool p4 = false) {
    return p4 ? m / 2 : m <= 16 ? 8 : m <= 32 ? 12 : 24;
}
__host__ __device__ constexpr int prune_last(int m, bool p4 = false) {
    return p4 ? m / 2 + (m <= 16 ? 4 : 8) : m <= 16 ? 12 : m <= 32 ? 16 : 28;
}
constexpr int PRUNE_DEEPEN = 8;

// Adds the 2 halves of a 32-bit word to acc[0], acc[1]: the mixed-precision add of sm_100 (add.rn.f32.f16)
// converts the half exactly to fp32 and rounds the sum once, so each is __fadd_rn(acc, __half2float(h)) in one
// instruction instead of a conversion and an add.
__device__ __forceinline__ float add_f32_f16(float acc, unsigned short h) {
    float r;
    asm("add.rn.f32.f16 %0, %1, %2;" : "=f"(r) : "h"(h), "f"(acc));
    return r;
}
__device__ __forceinline__ void add_half2(uint32_t w, float* acc) {
    acc[0] = add_f32_f16(acc[0], (unsigned short)(w & 0xffffu));
    acc[1] = add_f32_f16(acc[1], (unsigned short)(w >> 16));
}

// One sub-space lookup for Q queries: acc[q] += LUT_q[s][c], rounded per add, in s order.
template <int Q, bool H16>
__device__ __forceinline__ void lookup_add(const unsigned char* lut_smem, int mtab, int s, uint32_t c,
                                           float* acc) {
    const uint32_t e = (uint32_t)s * KSUB + c;
    if constexpr (H16) {
        static_assert(Q == 4 || Q == 8, "half LUTs hold 4 or 8 queries per entry");
        if constexpr (Q == 4) {
            const uint2 v = reinterpret_cast<const uint2*>(lut_smem)[e];
            add_half2(v.x, acc);
            add_half2(v.y, acc + 2);
        } else {
            const uint4 v = reinterpret_cast<const uint4*>(lut_smem)[e];
            add_half2(v.x, acc);
            add_half2(v.y, acc + 2);
            add_half2(v.z, acc + 4);
            add_half2(v.w, acc + 6);
        }
    } else if constexpr (Q == 1) {
        acc[0] = __fadd_rn(acc[0], reinterpret_cast<const float*>(lut_smem)[e]);
    } else if constexpr (Q == 2) {
        const float2 v = reinterpret_cast<const float2*>(lut_smem)[e];
        acc[0] = __fadd_rn(acc[0], v.x);
        acc[1] = __fadd_rn(acc[1], v.y);
    } else if constexpr (Q == 4) {
        const float4 v = reinterpret_cast<const float4*>(lut_smem)[e];
        acc[0] = __fadd_rn(acc[0], v.x);
        acc[1] = __fadd_rn(acc[1], v.y);
        acc[2] = __fadd_rn(acc[2], v.z);
        acc[3] = __fadd_rn(acc[3], v.w);
    } else {
        const float4 v = reinterpret_cast<const float4*>(lut_smem)[e];
        const float4 u = reinterpret_cast<const float4*>(lut_smem)[(uint32_t)mtab * KSUB + e];
        acc[0] = __fadd_rn(acc[0], v.x);
        acc[1] = __fadd_rn(acc[1], v.y);
        acc[2] = __fadd_rn(acc[2], v.z);
        acc[3] = __fadd_rn(acc[3], v.w);
        acc[4] = __fadd_rn(acc[4], u.x);
        acc[5] = __fadd_rn(acc[5], u.y);
        acc[6] = __fadd_rn(acc[6], u.z);
        acc[7] = __fadd_rn(acc[7], u.w);
    }
}

// Byte offset of query q's entry (s = 0, c = 0) in the group's LUT, the stride between c entries, and the offset of
// entry (s, c) from the query's base (P4: 4-bit PQ's [s][q / 2][c] float2 tables).
template <int Q, bool H16, bool P4 = false>
__device__ __forceinline__ uint32_t lut_query_base(int q, int mtab) {
    if constexpr (P4) return (uint32_t)(q >> 1) * 128u + (uint32_t)(q & 1) * 4u;
    else if constexpr (H16) return (uint32_t)q * 2u;
    else if constexpr (Q >= 4) return (uint32_t)(q >> 2) * (uint32_t)mtab * KSUB * 16u + (uint32_t)(q & 3) * 4u;
    else return (uint32_t)q * 4u;
}
template <int Q, bool H16, bool P4 = false>
__host__ __device__ constexpr uint32_t lut_entry_bytes() {
    return P4 ? 8u : H16 ? (uint32_t)Q * 2u : Q >= 4 ? 16u : (uint32_t)Q * 4u;
}
template <int Q, bool H16, bool P4 = false>
__device__ __forceinline__ uint32_t lut_pos(int s, uint32_t c) {
    if constexpr (P4) return (uint32_t)s * (uint32_t)(Q * 64) + c * 8u;
    else return ((uint32_t)s * KSUB + c) * lut_entry_bytes<Q, H16>();
}
// One query's entry at byte address p of the shared LUT, as fp32.
template <bool H16>
__device__ __forceinline__ float lut_value(const unsigned char* p) {
    if constexpr (H16) return __half2float(*reinterpret_cast<const __half*>(p));
    else return *reinterpret_cast<const float*>(p);
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, int b) {
    return b < 4 ? v.x : b < 8 ? v.y : b < 12 ? v.z : v.w;
}

__device__ __forceinline__ uint32_t code_byte(const uint4& v, int b) { return (word_of(v, b) >> (8 * (b & 3))) & 0xffu; }

// 4-bit codes: sub-code j (0..31) of a 16-byte word, and 8 times it (the byte offset of its float2 LUT entry).
__device__ __forceinline__ uint32_t code_nib(const uint4& v, int j) { return (word_of(v, j >> 1) >> (4 * (j & 7))) & 0xfu; }
__device__ __forceinline__ uint32_t code_nib8(const uint4& v, int j) {
    const uint32_t w = word_of(v, j >> 1);
    const int sh = 4 * (j & 7);
    return sh >= 3 ? (w >> (sh - 3)) & 0x78u : (w << 3) & 0x78u;
}

// 4-bit PQ: one sub-space lookup for Q queries, Q / 2 conflict-free LDS.64 from the [s][q / 2][c] float2 tables
// (c8 = 8 * code); acc[q] += LUT_q[s][c], rounded per add, in s order.
template <int Q>
__device__ __forceinline__ void lookup_add4(const unsigned char* lut_smem, int s, uint32_t c8, float* acc) {
    const unsigned char* p = lut_smem + (uint32_t)s * (uint32_t)(Q * 64) + c8;
#pragma unroll
    for (int qp = 0; qp < Q / 2; ++qp) {
        const float2 v = *reinterpret_cast<const float2*>(p + qp * 128);
        acc[2 * qp] = __fadd_rn(acc[2 * qp], v.x);
        acc[2 * qp + 1] = __fadd_rn(acc[2 * qp + 1], v.y);
    }
}

// Persistent fused scan + top-k. Work item = (vector chunk, query group), handed out by an atomic counter in
// chunk-major order, so the blocks running at one time share the same chunk of codes through L2.
//   per item:  (group changed) TMA bulk copy of the group's Q LUTs into shared memory;
//              warps take the chunk's 32*ILP-row tiles from a block counter and stream each through a private
//              ring of `stages` shared buffers filled by TMA bulk copies (lane 0 issues, one mbarrier per slot),
//              compute Q distances per row with strictly ordered fp32 adds, and offer them to one WarpTopK per
//              query; at the end the NW warp lists of each query are merged into the item's partial list.
// PRUNE (exact early abandoning): partial sums only grow (every LUT entry is >= +0 and fp32 round-to-nearest
//   addition is monotone), so a (query, row) pair whose partial sum already exceeds an upper bound T_q of the
//   query's k-th distance cannot be in the result. T_q = min(the warp list's k-th distance, a per-query global
//   bound: the k-th distance of a global list into which every finished item folds its own list). Phase A
//   computes sub-spaces [0, SA) of every row for all Q queries (LDS.128 lookups); when at most half of the
//   (row, query) pairs survive, the survivors are compacted (ballot + popc) into a per-warp shared-memory queue
//   and finished 32 at a time, each lane dropping out as soon as its sum exceeds T_q; otherwise the whole tile
//   is finished with the Q-wide lookups. Results are unchanged.
// MT: m when it is 16, 32 or 64 (fully unrolled sub-space loop), 0 for any other m.
// Block shape: two blocks of 8 warps share an SM when the group's fp32 LUT is at most 80 KB; a larger LUT leaves room
// for one block, which then has 16 warps. Either way 16 warps per SM, registers capped at 128.
// Half-precision LUTs always take 16-warp blocks: two 8-warp blocks with their own 64 KB LUTs, rings and queues do
// not fit one SM's shared memory together, which left one 8-warp block per SM (measured: 12.5 % warps active).
// 4-bit PQ LUTs (at most 8 queries x 64 sub-spaces x 16 entries x 4 bytes = 32 KB) always take two 8-warp blocks.
__host__ __device__ constexpr int scan_warps(int Q, int MT, bool H16 = false, bool P4 = false) {
    return P4 || (!H16 && Q * (MT ? MT : 16) * KSUB * 4 <= 80 * 1024) ? 8 : 16;
}
template <int Q, int MT, bool H16, bool P4>
constexpr int scan_min_blocks() { return scan_warps(Q, MT, H16, P4) == 8 ? 2 : 1; }

// H16: half-precision LUT entries (Q = 4 or 8, m = 16, 32 or 64), summed in fp32 like the fp32 entries.
// IVF: items are (list, up to Q queries probing it) from the IVF item table; ids come from the index's id array.
// P4: 4-bit PQ codes (16 centroids per sub-space, 32 sub-codes per 16-byte word) and their float2-pair LUTs.
template <int Q, int MT, int ILP, int S, int NW, bool PRUNE, bool H16 = false, bool IVF = false, bool P4 = false>
__global__ void __launch_bounds__(NW * 32, scan_min_blocks<Q, MT, H16, P4>()) scan_kernel(const ScanArgs a) {
    static_assert(!IVF || (ILP <= 2 && !H16), "IVF items start on 64-row windows; fp32 LUTs");
    static_assert(!H16 || (MT != 0 && (Q == 4 || Q == 8)), "half LUTs: m = 16, 32, 64 and 4 or 8 queries");
    static_assert(!P4 || (MT != 0 && (Q == 4 || Q == 8) && !H16 && !IVF), "4-bit PQ: m = 16, 32, 64, Q = 4 or 8");
    static_assert(!PRUNE || MT != 0, "the pruned scan is specialised for m = 16, 32, 64");
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr int SPW = P4 ? 32 : 16;  // sub-codes per 16-byte word
    constexpr int W_T = MT ? (MT + SPW - 1) / SPW : 0;
    constexpr int SA = prune_first(MT, P4), SAX = prune_last(MT, P4);
    constexpr bool CARRY = carry_queue(MT) && !P4;
    static_assert(!PRUNE || (SA % 2 == 0 && SAX % 2 == 0 && SAX >= SA && SAX < MT),
                  "phase A stops at even sub-spaces: phase B fetches sub-spaces in pairs inside one 16-byte word");
    const int m = MT ? MT : a.m;
    const int W = MT ? W_T : a.W;
    const ScanSmem plan = scan_smem_plan(Q, m, W, ILP, NW, a.stages, a.k, PRUNE, a.merge_slots, H16, IVF, P4);
    unsigned char* lut_smem = smem + plan.lut;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + plan.bars);
    uint64_t* lut_bar = bars + NW * a.stages;
    int* s_item = reinterpret_cast<int*>(smem + plan.flags);
    int* s_abort = s_item + 1;
    int* s_tile = s_item + 2;
    int2* s_pairs = reinterpret_cast<int2*>(smem + plan.flags + 16);  // IVF: the item's (query, probe slot) pairs
    int2* scratch = reinterpret_cast<int2*>(smem + plan.scratch);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t* my_bars = bars + warp * a.stages;
    unsigned char* my_stages = smem + plan.stage + (uint32_t)warp * a.stages * plan.stage_bytes;
    int2* my_queue = reinterpret_cast<int2*>(smem + plan.queue) + warp * (16 * ILP * Q);
    int* my_ring = reinterpret_cast<int*>(smem + plan.ring) + warp * a.stages;  // tile held by each slot, -1: none

    if (threadIdx.x == 0) {
        for (int i = 0; i < NW * a.stages + 1; ++i) mbar_init(bars + i, 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    const int items = IVF ? __ldg(a.ivf_nitems) : a.groups * a.chunks;
    const int64_t tile_rows = 32 * ILP;
    uint32_t issued = 0, consumed = 0, lut_phase = 0;  // issued: lane 0 only
    uint32_t lut_pending = ~0u;  // thread 0: parity of a LUT copy not yet seen complete (~0u: none)
    int cur_g = -1;

    for (;;) {
        if (threadIdx.x == 0) {
            *s_item = atomicAdd(a.work_counter, 1);
            *s_tile = 0;
        }
        if constexpr (IVF) {
            __syncthreads();  // s_item is visible
            const int it = *s_item;
            if (threadIdx.x < Q) s_pairs[threadIdx.x] = it < items ? a.ivf_item_pairs[(int64_t)it * Q + threadIdx.x]
                                                                   : make_int2(-1, -1);
        }
        __syncthreads();  // (A) previous item finished by every warp; the LUT may be replaced
        const int item = *s_item;
        if (item >= items || *s_abort) break;
        // flat: (chunk, query group); IVF: the item's list, and its own LUT (g = item)
        int chunk = 0, g = item;
        if constexpr (!IVF) {  // window of group_window groups, then chunk, then group (group_window = groups: chunk-major)
            const int per_win = a.group_window * a.chunks;
            const int win = item / per_win, r = item - win * per_win;
            const int g0 = win * a.group_window, gw = min(a.group_window, a.groups - g0);
            chunk = r / gw;
            g = g0 + (r - chunk * gw);
        }
        const int list = IVF ? a.ivf_item_list[item] : 0;
        // global index of the item's query q (-1: padding); IVF: the probe slot its list is for that query
        auto qidx = [&](int q) -> int64_t {
            if constexpr (IVF) return s_pairs[q].x;
            else return (int64_t)g * Q + q < a.nq ? (int64_t)g * Q + q : -1;
        };

        if (IVF || g != cur_g) {
            if (threadIdx.x == 0) {
                fence_proxy_async_smem();
                const unsigned char* src =
                    reinterpret_cast<const unsigned char*>(a.lut) + (int64_t)g * plan.lut_bytes;
                mbar_arrive_expect_tx(lut_bar, plan.lut_bytes);
                for (uint32_t off = 0; off < plan.lut_bytes; off += 32768u) {
                    const uint32_t len = min(32768u, plan.lut_bytes - off);
                    bulk_g2s(lut_smem + off, src + off, len, lut_bar);
                }
                lut_pending = lut_phase;
            }
            // Vote, so that the warp's lanes take the same path even if only some of them ran out of time.
            if (!__all_sync(FULL, mbar_wait_bounded(lut_bar, lut_phase, a.wait_budget))) {
                if (lane == 0) atomicOr(a.status, ERR_WAIT_TIMEOUT);
                *s_abort = 1;
            } else if (threadIdx.x == 0) {
                lut_pending = ~0u;
            }
            lut_phase ^= 1u;
            cur_g = g;
        }

        WarpTopK<S> top[Q];
        float known[Q];  // PRUNE: this warp's view of the global bounds (padded query slots: -1, prune all)
#pragma unroll
        for (int q = 0; q < Q; ++q) {
            top[q].init();
            if constexpr (PRUNE) {
                const int64_t qi = qidx(q);
                known[q] = qi >= 0 ? __uint_as_float(min(__ldcg(a.bound + qi), coop_bound(a, qi))) : -1.f;
            }
        }

        const int64_t row_begin = IVF ? a.ivf_list_off[list]
                                      : chunk == 0 ? 0 : a.first_len + (int64_t)(chunk - 1) * a.chunk_len;
        const int64_t row_end = IVF ? row_begin + a.ivf_list_rows[list]
                                    : min(a.first_len + (int64_t)chunk * a.chunk_len, a.n_pad);
        const int64_t t_begin = row_begin / tile_rows;
        const int ntiles = (int)(row_end / tile_rows - t_begin);

        // Carry queue (PRUNE, m = 16): entry = {partial sum bits, rel | q << 24 | (depth - SA) / 2 << 27, sub-codes
        // depth..15 as 8 bytes (sub-code `depth` lowest)}, rel = row - the chunk's first 64-row window, so that the
        // row's id is carry_id0 + rel; qcnt is warp-uniform.
        int qcnt = 0;
        const int32_t carry_id0 = (int32_t)(a.id_base + (row_begin & ~(int64_t)(PLACE_WINDOW - 1)));
        int4* my_carry = reinterpret_cast<int4*>(smem + plan.queue) + warp * CARRY_CAP;
        // Finishes entries [start, start + count) (count <= 32), one pair per lane, two sub-spaces per step, each
        // lane dropping out as soon as its sum exceeds its query's bound; offers the completed pairs.
        auto carry_batch = [&](int start, int count) {
            __syncwarp();  // entries written by other lanes are visible
            const bool in = lane < count;
            const int4 ent = in ? my_carry[start + lane] : make_int4(0, 0, 0, 0);
            float x = __int_as_float(ent.x);
            const uint32_t meta = (uint32_t)ent.y;
            const int q = (int)((meta >> 24) & 7u);
            int s = CARRY_DEPTH0 + 2 * (int)(meta >> 27);
            uint32_t lo = (uint32_t)ent.z, hi = (uint32_t)ent.w;
            // the query's bound now: min(the warp's view of its global bound, the warp list's k-th distance)
            float bq = fminf(known[0], top[0].thr_d);
#pragma unroll
            for (int qq = 1; qq < Q; ++qq)
                if (q == qq) bq = fminf(known[qq], top[qq].thr_d);
            const unsigned char* lq = lut_smem + lut_query_base<Q, H16, P4>(q, MT);
            bool live = in && !(x > bq);  // the bound may have dropped since the pair was queued
#pragma unroll
            for (int t = 0; t < (MT - SA) / 2; ++t) {
                const bool go = live && s < MT;
                if (!__any_sync(FULL, go)) break;
                if (go) {
                    const uint32_t c0 = lo & 0xffu, c1 = (lo >> 8) & 0xffu;
                    lo = __funnelshift_r(lo, hi, 16);
                    hi >>= 16;
                    const float v0 = lut_value<H16>(lq + lut_pos<Q, H16, P4>(s, c0));
                    const float v1 = lut_value<H16>(lq + lut_pos<Q, H16, P4>(s + 1, c1));
                    x = __fadd_rn(x, v0);
                    live = !(x > bq);
                    x = __fadd_rn(x, v1);
                    live = live && !(x > bq);
                    s += 2;
                }
            }
            if (__any_sync(FULL, live)) {  // usually every pair of the batch was abandoned
                const int32_t id = IVF ? (in ? __ldg(a.ivf_ids + (row_begin & ~(int64_t)(PLACE_WINDOW - 1)) +
                                                     (int64_t)(meta & 0xffffffu))
                                             : -1)
                                       : carry_id0 + (int32_t)(meta & 0xffffffu);
#pragma unroll
                for (int qq = 0; qq < Q; ++qq) {
                    if (__any_sync(FULL, live && q == qq)) top[qq].offer(x, id, live && q == qq, a.k);
                }
            }
        };
        // Runs the queue's full batches (all = true: every entry, at the end of the item).
        auto carry_drain = [&](bool all) {
            while (qcnt >= 32 || (all && qcnt > 0)) {
                const int take = min(qcnt, 32);
                qcnt -= take;
                carry_batch(qcnt, take);
            }
        };

        // lane 0: take the chunk's next tile (if any) into the next ring slot
        auto refill = [&]() {
            const uint32_t slot = issued % (uint32_t)a.stages;
            const int t = atomicAdd(s_tile, 1);
            if (t < ntiles) {
                my_ring[slot] = t;
                fence_proxy_async_smem();
                unsigned char* dst = my_stages + slot * plan.stage_bytes;
                mbar_arrive_expect_tx(my_bars + slot, plan.stage_bytes);
                bulk_g2s(dst, a.codes + (t_begin + t) * tile_rows * W, plan.tile_bytes, my_bars + slot);
                bulk_g2s(dst + plan.tile_bytes, a.perm + (t_begin + t) * tile_rows, (uint32_t)tile_rows, my_bars + slot);
                if constexpr (IVF)  // the ids of the tile's 64-row window (1 KB-aligned source: 16-byte rule holds)
                    bulk_g2s(dst + plan.tile_bytes + (uint32_t)tile_rows,
                             a.ivf_ids + (((t_begin + t) * tile_rows) & ~(int64_t)(PLACE_WINDOW - 1)), 256u,
                             my_bars + slot);
                ++issued;
            } else {
                my_ring[slot] = -1;
            }
        };
        bool warp_abort = __any_sync(FULL, *s_abort != 0);
        if (lane == 0 && !warp_abort)
            for (int j = 0; j < a.stages; ++j) {  // fill the ring; stop at the first slot marked empty
                const uint32_t before = issued;
                refill();
                if (issued == before) break;
            }
        // fin: the chunk has no tiles left. The carry queue is drained at one place, the top of this loop: full
        // batches after each tile, every entry once the tiles are done (one inlined copy of the batch code and its
        // Q top-k offers instead of two keeps the kernel's instruction footprint down).
        bool fin = false;
        while (!warp_abort) {
            if constexpr (PRUNE && CARRY) carry_drain(fin);
            if (fin) break;
            __syncwarp();  // ring entries written by lane 0 are visible
            const uint32_t slot = consumed % (uint32_t)a.stages;
            const int tile = my_ring[slot];
            if (tile < 0 || consumed == __shfl_sync(FULL, issued, 0)) {
                fin = true;
                continue;
            }
            const uint32_t parity = (consumed / (uint32_t)a.stages) & 1u;
            if (!__all_sync(FULL, mbar_wait_bounded(my_bars + slot, parity, a.wait_budget))) {
                if (lane == 0) atomicOr(a.status, ERR_WAIT_TIMEOUT);
                *s_abort = 1;
                warp_abort = true;
                break;
            }
            ++consumed;
            const uint4* st = reinterpret_cast<const uint4*>(my_stages + slot * plan.stage_bytes);
            const uint8_t* st_perm = my_stages + slot * plan.stage_bytes + plan.tile_bytes;
            const int64_t tile_row0 = (t_begin + tile) * tile_rows;
            // global id of the row at tile position r (lane placement within 64-row windows)
            auto row_id = [&](int r) {
                if constexpr (IVF) {  // the slot's id from the window's ids staged with the tile (-1: padding)
                    return reinterpret_cast<const int32_t*>(st_perm + tile_rows)[st_perm[r]];
                } else {
                    return (int32_t)(a.id_base + ((tile_row0 + r) & ~(int64_t)(PLACE_WINDOW - 1)) + st_perm[r]);
                }
            };
            // rows past n (flat) or padding slots of a list (IVF) are computed but never offered
            auto row_valid = [&](int r) {
                if constexpr (IVF) return row_id(r) >= 0;
                else return tile_row0 + r < a.n;
            };

            if constexpr (!PRUNE) {
                float acc[ILP][Q];
#pragma unroll
                for (int u = 0; u < ILP; ++u)
#pragma unroll
                    for (int q = 0; q < Q; ++q) acc[u][q] = 0.f;

#pragma unroll
                for (int w = 0; w < (MT ? W_T : 1); ++w) {
                    // generic m: a run-time loop over words; MT: the unrolled loop above with W_T words
                    for (int wr = 0; wr < (MT ? 1 : W); ++wr) {
                        const int ww = MT ? w : wr;
                        uint4 cv[ILP];
#pragma unroll
                        for (int u = 0; u < ILP; ++u) cv[u] = st[(u * W + ww) * 32 + lane];
#pragma unroll
                        for (int b = 0; b < SPW; ++b) {
                            const int s = ww * SPW + b;
                            if ((!MT || P4) && s >= m) break;  // P4: MT = 16 fills half a word
#pragma unroll
                            for (int u = 0; u < ILP; ++u) {
                                if constexpr (P4) lookup_add4<Q>(lut_smem, s, code_nib8(cv[u], b), acc[u]);
                                else lookup_add<Q, H16>(lut_smem, m, s, code_byte(cv[u], b), acc[u]);
                            }
                        }
                    }
                }
                int32_t ids[ILP];
                bool valid[ILP];
#pragma unroll
                for (int u = 0; u < ILP; ++u) {  // both read the stage slot (IVF), so before it is refilled
                    ids[u] = row_id(u * 32 + lane);
                    valid[u] = row_valid(u * 32 + lane);
                }
                __syncwarp();  // every lane has consumed the slot (codes, placement bytes, ids)
                if (lane == 0) refill();

                bool any = false;
#pragma unroll
                for (int u = 0; u < ILP; ++u) {
#pragma unroll
                    for (int q = 0; q < Q; ++q) any |= valid[u] && top[q].admits(acc[u][q], ids[u]);
                }
                if (__any_sync(FULL, any)) {
                    // 8-bit codes: one offer per row group (4 % faster here than offer_n at config 1); 4-bit codes:
                    // offer_n (8 % faster for them)
                    if constexpr (P4) {
                        static_for<Q>([&](auto qc) {
                            constexpr int q = decltype(qc)::value;
                            float x[ILP];
#pragma unroll
                            for (int u = 0; u < ILP; ++u) x[u] = acc[u][q];
                            top[q].offer_n(x, ids, valid, a.k);
                        });
                    } else {
#pragma unroll
                        for (int u = 0; u < ILP; ++u)
#pragma unroll
                            for (int q = 0; q < Q; ++q) top[q].offer(acc[u][q], ids[u], valid[u], a.k);
                    }
                }
            } else {
                // The query group's global bounds, loaded now (lane q: query q) so that the L2 latency hides
                // behind phase A; other warps and blocks keep lowering them.
                // (the other shards' bounds of a cooperative search are read at item start only, and this shard's
                // lowered bounds are offered to them at item end: no per-tile cost)
                uint32_t gbits = 0x7f800000u;
                if (lane < Q) {
                    const int64_t qi = qidx(lane);
                    if (qi >= 0) gbits = __ldcg(a.bound + qi);
                }
                // ---- phase A: sub-spaces [0, SA) of every row, all Q queries per fetch
                float acc[ILP][Q];
#pragma unroll
                for (int u = 0; u < ILP; ++u)
#pragma unroll
                    for (int q = 0; q < Q; ++q) acc[u][q] = 0.f;
                uint4 cv[ILP];
                auto phase_a = [&](auto sc) {  // one sub-space (a compile-time constant) of every row
                    constexpr int s = decltype(sc)::value;
                    if constexpr (s % SPW == 0) {
#pragma unroll
                        for (int u = 0; u < ILP; ++u) cv[u] = st[(u * W_T + s / SPW) * 32 + lane];
                    }
#pragma unroll
                    for (int u = 0; u < ILP; ++u) {
                        if constexpr (P4) lookup_add4<Q>(lut_smem, s, code_nib8(cv[u], s % SPW), acc[u]);
                        else lookup_add<Q, H16>(lut_smem, MT, s, code_byte(cv[u], s % 16), acc[u]);
                    }
                };
                static_for<SA>(phase_a);
                const float gb = __uint_as_float(gbits);  // the load has landed by now
                float bnd[Q];
#pragma unroll
                for (int q = 0; q < Q; ++q) {
                    known[q] = fminf(known[q], __shfl_sync(FULL, gb, q));  // padded slots keep -1
                    bnd[q] = fminf(known[q], top[q].thr_d);
                }
                // ---- surviving (row, query) pairs: this lane's pair (u, q) is alive while its partial sum is not
                // above the query's bound (recomputed where needed rather than kept as ballots: registers)
                auto alive = [&](int u, int q) {
                    return row_valid(u * 32 + lane) && !(acc[u][q] > bnd[q]);
                };
                int total = 0;
                auto vote = [&]() {
                    total = 0;
#pragma unroll
                    for (int u = 0; u < ILP; ++u)
#pragma unroll
                        for (int q = 0; q < Q; ++q) total += __popc(__ballot_sync(FULL, alive(u, q)));
                };
                vote();
                // ---- deeper phase A while many pairs survive (warp-uniform: total comes from ballots)
                int dep = SA;
                static_for<(SAX - SA) / 2>([&](auto e) {
                    constexpr int s0 = SA + 2 * decltype(e)::value;
                    if (dep == s0 && total * PRUNE_DEEPEN > 32 * ILP * Q) {
                        phase_a(Int<s0>{});
                        phase_a(Int<s0 + 1>{});
                        dep = s0 + 2;
                        vote();
                    }
                });
                // Finishes every row with the Q-wide lookups of the full scan (called only at dep == SAX) and
                // offers the surviving pairs.
                auto finish_qwide = [&]() {
                    static_for<MT - SAX>([&](auto e) { phase_a(Int<SAX + decltype(e)::value>{}); });
                    bool any = false;
                    int32_t ids[ILP];
#pragma unroll
                    for (int u = 0; u < ILP; ++u) {
                        ids[u] = row_id(u * 32 + lane);
#pragma unroll
                        for (int q = 0; q < Q; ++q) any |= alive(u, q) && top[q].admits(acc[u][q], ids[u]);
                    }
                    if (__any_sync(FULL, any)) {
                        static_for<Q>([&](auto qc) {
                            constexpr int q = decltype(qc)::value;
                            float x[ILP];
                            bool v[ILP];
#pragma unroll
                            for (int u = 0; u < ILP; ++u) {
                                x[u] = acc[u][q];
                                v[u] = alive(u, q);
                            }
                            top[q].offer_n(x, ids, v, a.k);
                        });
                    }
                };
                if constexpr (CARRY) {
                    static_assert(CARRY_QWIDE * PRUNE_DEEPEN >= 32 * ILP * Q,
                                  "a tile with more than CARRY_QWIDE survivors must have been deepened to SAX");
                    if (total > CARRY_QWIDE) {
                        finish_qwide();
                    } else if (total > 0) {
                        // Queue the survivors: first (partial sum, tile row | q << 24) while the sums are in
                        // registers, then, entry per lane, each row's remaining sub-codes (dep .. 15 of its 16-byte
                        // word) and its chunk-relative row from the stage slot, which keeps the sums' live range short.
                        const unsigned lt = (1u << lane) - 1u;
                        const int first = qcnt;
#pragma unroll
                        for (int u = 0; u < ILP; ++u)
#pragma unroll
                            for (int q = 0; q < Q; ++q) {
                                const unsigned mk = __ballot_sync(FULL, alive(u, q));
                                if (mk != 0) {  // uniform: most (row group, query) ballots are empty
                                    if ((mk >> lane) & 1u)
                                        reinterpret_cast<int2*>(my_carry + qcnt + __popc(mk & lt))[0] =
                                            make_int2(__float_as_int(acc[u][q]), (u * 32 + lane) | (q << 24));
                                    qcnt += __popc(mk);
                                }
                            }
                        __syncwarp();
                        // entries hold the codes of sub-spaces d0 .. 15 (8 bytes at most): a pair voted at a depth
                        // below CARRY_DEPTH0 first gets its sub-spaces dep .. CARRY_DEPTH0 - 1 added here
                        const int d0 = dep > CARRY_DEPTH0 ? dep : CARRY_DEPTH0;
                        const uint32_t dsel = (uint32_t)(d0 - CARRY_DEPTH0) / 2u;
                        // the chunk's first window starts row_begin % 64 rows before it (windows are 64-aligned)
                        const uint32_t tile_rel = (uint32_t)(row_begin & (PLACE_WINDOW - 1)) + (uint32_t)tile * (uint32_t)tile_rows;
                        for (int e = first + lane; e < qcnt; e += 32) {
                            uint32_t* ent = reinterpret_cast<uint32_t*>(my_carry + e);
                            const uint32_t y = ent[1];
                            const uint32_t r = y & 0xffffu;
                            float x = __uint_as_float(ent[0]);
                            uint32_t lo, hi;
                            if constexpr (SA < CARRY_DEPTH0) {
                                const uint4 w = st[r];  // the row's 16 sub-codes
                                if (dep < CARRY_DEPTH0) {  // warp-uniform
                                    const unsigned char* lq = lut_smem + lut_query_base<Q, H16>((int)(y >> 24), MT);
                                    for (int sb = dep; sb < CARRY_DEPTH0; ++sb)
                                        x = __fadd_rn(x, lut_value<H16>(lq + lut_pos<Q, H16>(sb, code_byte(w, sb))));
                                }
                                lo = d0 == 8 ? w.z : d0 == 10 ? __funnelshift_r(w.z, w.w, 16) : w.w;
                                hi = d0 == 8 ? w.w : d0 == 10 ? w.w >> 16 : 0u;
                            } else {  // phase A never stops before CARRY_DEPTH0: only bytes 8..15 are needed
                                const uint2 zw = reinterpret_cast<const uint2*>(st + r)[1];
                                lo = d0 == 8 ? zw.x : d0 == 10 ? __funnelshift_r(zw.x, zw.y, 16) : zw.y;
                                hi = d0 == 8 ? zw.y : d0 == 10 ? zw.y >> 16 : 0u;
                            }
                            const uint32_t rel = ((tile_rel + r) & ~(uint32_t)(PLACE_WINDOW - 1)) + st_perm[r];
                            reinterpret_cast<uint4*>(ent)[0] =
                                make_uint4(__float_as_uint(x), rel | (y & (7u << 24)) | (dsel << 27), lo, hi);
                        }
                    }
                    __syncwarp();  // the stage slot is free: queued pairs carry their codes
                    if (lane == 0) refill();
                } else {
                int cnt = 0;
                if (2 * total > 32 * ILP * Q) {
                    // Most pairs survive (no tight bound yet), which the deepening above leaves possible only at
                    // dep == SAX: finishing every row with the Q-wide lookups of the full scan is cheaper than
                    // finishing pairs one query per lane.
                    finish_qwide();
                } else {
                    const unsigned lt = (1u << lane) - 1u;
#pragma unroll
                    for (int u = 0; u < ILP; ++u)
#pragma unroll
                        for (int q = 0; q < Q; ++q) {
                            const unsigned mk = __ballot_sync(FULL, alive(u, q));
                            if (mk != 0) {  // uniform: most (row group, query) ballots are empty
                                if ((mk >> lane) & 1u)
                                    my_queue[cnt + __popc(mk & lt)] =
                                        make_int2(__float_as_int(acc[u][q]), (u * 32 + lane) | (q << 16));
                                cnt += __popc(mk);
                            }
                        }
                }
                __syncwarp();
                // ---- phase B: finish the queued pairs 32 at a time from sub-space D = dep, two sub-spaces per step,
                // each lane dropping out as soon as its sum exceeds its query's bound. One copy per depth, so that
                // every sub-space index stays a compile-time constant.
                // One copy of the batch loop and its Q top-k offers; only the lookups are specialised per depth D
                // (every sub-space index a compile-time constant).
                for (int base = 0; base < cnt; base += 32) {
                    const int e = base + lane;
                    bool live = e < cnt;
                    const int2 ent = live ? my_queue[e] : make_int2(0, 0);
                    float x = __int_as_float(ent.x);
                    const int r = ent.y & 0xffff, q = ent.y >> 16;
                    float bq = bnd[0];
#pragma unroll
                    for (int qq = 1; qq < Q; ++qq)
                        if (q == qq) bq = bnd[qq];
                    const unsigned char* lq = lut_smem + lut_query_base<Q, H16, P4>(q, MT);
                    const uint4* rowp = st + (r >> 5) * W_T * 32 + (r & 31);
                    static_for<(SAX - SA) / 2 + 1>([&](auto dc) {
                        constexpr int D = SA + 2 * decltype(dc)::value;
                        if (dep != D) return;
                        uint4 cw = make_uint4(0, 0, 0, 0);
#pragma unroll
                        for (int s = D; s < MT; s += 2) {
                            if (s == D || s % SPW == 0) {
                                if (!__any_sync(FULL, live)) break;
                                if (live) cw = rowp[(s / SPW) * 32];
                            } else if ((s - D) % 4 == 0 && !__any_sync(FULL, live)) {
                                break;
                            }
                            if (live) {
                                const uint32_t c0 = P4 ? code_nib(cw, s % SPW) : code_byte(cw, s % 16);
                                const uint32_t c1 = P4 ? code_nib(cw, (s + 1) % SPW) : code_byte(cw, (s + 1) % 16);
                                const float v0 = lut_value<H16>(lq + lut_pos<Q, H16, P4>(s, c0));
                                const float v1 = lut_value<H16>(lq + lut_pos<Q, H16, P4>(s + 1, c1));
                                x = __fadd_rn(x, v0);
                                live = !(x > bq);
                                x = __fadd_rn(x, v1);
                                live = live && !(x > bq);
                            }
                        }
                    });
                    const int32_t id = row_id(r);
                    if (__any_sync(FULL, live)) {  // usually every pair of the batch was abandoned
#pragma unroll
                        for (int qq = 0; qq < Q; ++qq) {
                            if (__any_sync(FULL, live && q == qq)) {
                                top[qq].offer(x, id, live && q == qq, a.k);
                                bnd[qq] = fminf(bnd[qq], top[qq].thr_d);
                            }
                        }
                    }
                }
                __syncwarp();  // the queue and the stage slot are free again
                if (lane == 0) refill();
                }
                // Publish improved list thresholds as global bounds for the other warps and blocks.
#pragma unroll
                for (int q = 0; q < Q; ++q) {
                    if (top[q].thr_d < known[q]) {  // never for padded slots (known -1)
                        if (lane == 0) {
                            const int64_t qi = qidx(q);
                            atomicMin(a.bound + qi, __float_as_uint(top[q].thr_d));
                        }
                        known[q] = top[q].thr_d;
                    }
                }
            }
        }
        if constexpr (PRUNE && CARRY) qcnt = 0;  // drained at the loop's end, or abandoned on a timeout
        if (warp_abort && lane == 0) {
            // Let this warp's copies still in flight land before the block can exit.
            while (consumed < issued) {
                const uint32_t slot = consumed % (uint32_t)a.stages;
                if (!mbar_wait_bounded(my_bars + slot, (consumed / (uint32_t)a.stages) & 1u, 4 * a.wait_budget))
                    atomicOr(a.status, ERR_DRAIN_TIMEOUT);
                ++consumed;
            }
        }
        consumed = __shfl_sync(FULL, consumed, 0);

        __syncthreads();  // (B) all warps finished the item's tiles; s_abort is stable
        if (*s_abort) continue;  // uniform: the next (A) exits the loop
        // Merge the NW warp lists of each query into the item's partial list: merge_slots queries at a time,
        // query q0 + j merged by warp j. qi: the query's global index, ql: its slot in the item.
        auto merge_and_publish = [&](int64_t qi, int ql, const int2* slot_lists, float kb) {
            WarpTopK<S> mt;
            mt.init();
            // Pairs above kb (an upper bound of the query's final k-th distance) cannot be in the result, so they
            // are left out of the item's list: fewer insertions, same final merge.
            const int total = NW * a.k;
            for (int j0 = 0; j0 < total; j0 += 32) {
                const int j = j0 + lane;
                const int2 e = j < total ? slot_lists[j] : make_int2(0x7f800000, SENTINEL_ID);
                mt.offer(__int_as_float(e.x), e.y, j < total && !(__int_as_float(e.x) > kb), a.k);
            }
            // this item's own list: [query][chunk][k] (flat), [query][probe slot][k] (IVF)
            if constexpr (IVF) mt.store(a.part + (qi * a.nprobe + s_pairs[ql].y) * a.k, a.k);
            else mt.store(a.part + (qi * a.chunks + chunk) * a.k, a.k);
            if constexpr (PRUNE) {
                // Fold the item's list into the query's global list of the best pairs seen so far, whose k-th
                // distance bounds the query for every other warp. Chunks cover disjoint rows, so the union has
                // no duplicates. If another block holds the lock the fold is skipped: only the bound gets
                // weaker, never wrong. kb is an upper bound of the query's bound (this warp's last view): when
                // the item's best pair is not below it, the fold cannot lower the bound (fewer than k pairs of
                // the union lie below it) and is skipped, which late in a scan is nearly every item.
                const bool useful = __shfl_sync(FULL, mt.d[0], 0) < kb;
                int got = 0;
                if (lane == 0 && useful) got = atomicCAS(a.glock + qi, 0, 1) == 0;
                if (__shfl_sync(FULL, got, 0)) {
                    __threadfence();
                    int2* gl = a.glist + qi * a.k;
                    for (int j0 = 0; j0 < a.k; j0 += 32) {
                        const int j = j0 + lane;
                        const int2 e = j < a.k ? __ldcg(gl + j) : make_int2(0x7f800000, SENTINEL_ID);
                        mt.offer(__int_as_float(e.x), e.y, j < a.k, a.k);
                    }
                    mt.store(gl, a.k);
                    __threadfence();
                    __syncwarp();
                    if (lane == 0) atomicExch(a.glock + qi, 0);
                }
                if (lane == 0) {
                    const bool lower = mt.thr_i != SENTINEL_ID && mt.thr_d < kb;
                    if (lower) atomicMin(a.bound + qi, __float_as_uint(mt.thr_d));
                    // Cooperative search: offer the other shards this shard's bound of the query as it stands now
                    // (the warps lowered it per tile too), once per item.
                    if (a.npeers > 0) {
                        uint32_t b = __ldcg(a.bound + qi);
                        if (lower) b = min(b, __float_as_uint(mt.thr_d));
                        if (b != 0x7f800000u) coop_publish(a, qi, b);
                    }
                }
            }
        };
        // merge_slots queries at a time (Q, or 1 when Q lists per warp do not fit the scratch), query q0 + j merged
        // by warp j: one call site for merge_and_publish (its code is large and runs once per item).
        for (int q0 = 0; q0 < Q; q0 += a.merge_slots) {
            static_for<Q>([&](auto qc) {
                constexpr int q = decltype(qc)::value;
                if (q >= q0 && q < q0 + a.merge_slots) top[q].store(scratch + ((q - q0) * NW + warp) * a.k, a.k);
            });
            __syncthreads();
            const int ql = q0 + warp;
            const int64_t qi = warp < a.merge_slots && ql < Q ? qidx(ql) : -1;
            float kb = __int_as_float(0x7f800000);
            if constexpr (PRUNE) {
                static_for<Q>([&](auto qc) {
                    if (ql == decltype(qc)::value) kb = known[decltype(qc)::value];
                });
            }
            if (qi >= 0) merge_and_publish(qi, ql, scratch + warp * NW * a.k, kb);
            __syncthreads();
        }
    }
    // A LUT copy whose wait ran out may still be in flight: it must land before the block's shared memory is
    // released.
    if (threadIdx.x == 0 && lut_pending != ~0u && !mbar_wait_bounded(lut_bar, lut_pending, 4 * a.wait_budget))
        atomicOr(a.status, ERR_DRAIN_TIMEOUT);
}

// ------------------------------------------------------------------------------------------------ merge
// One warp per query: the k best of `lists` sorted lists of k_in entries (entry (q, l, j) at
// in[q * qstride + l * lstride + j]); entries with id < 0 are padding. Output ascending, empty slots {+inf, -1}
// (the reference's host fix-up, src/cuda/searcher.cu:514-517).
// qexp (optional): per-query exponents of half-precision LUTs; distances are scaled by 2^-qexp[q] on output.
template <int S>
__global__ void __launch_bounds__(128) merge_kernel(const int2* __restrict__ in, int64_t nq, int lists, int k_in,
                                                    int64_t qstride, int64_t lstride, int k,
                                                    int2* __restrict__ out, const int* __restrict__ qexp) {
    const int lane = threadIdx.x & 31;
    const int64_t q = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (q >= nq) return;  // warp-uniform
    WarpTopK<S> top;
    top.init();
    const int64_t total = (int64_t)lists * k_in;
    const int2* base = in + q * qstride;
    for (int64_t j0 = 0; j0 < total; j0 += 32) {
        const int64_t j = j0 + lane;
        int2 e = make_int2(0x7f800000, SENTINEL_ID);
        if (j < total) {
            const int64_t l = j / k_in, i = j - l * k_in;
            e = base[l * lstride + i];
        }
        top.offer(__int_as_float(e.x), e.y, j < total && e.y >= 0, k);
    }
    const float scale = qexp ? exp2_int(-qexp[q]) : 1.f;
#pragma unroll
    for (int r = 0; r < S; ++r) {
        const int e = r * 32 + lane;
        if (e < k) {
            const bool pad = top.id[r] == SENTINEL_ID;
            out[q * k + e] = pad ? make_int2(0x7f800000, -1)
                                 : make_int2(__float_as_int(qexp ? __fmul_rn(top.d[r], scale) : top.d[r]), top.id[r]);
        }
    }
}

// Few queries (the latency case): one block of 8 warps per query. Warp w keeps the k best of candidates
// w * 32 + lane, w * 32 + 256 + lane, ...; warp 0 then merges the 8 lists. The k smallest of distinct (dist, id)
// pairs do not depend on the merge order, so the result equals merge_kernel's.
template <int S>
__global__ void __launch_bounds__(256) merge_wide_kernel(const int2* __restrict__ in, int64_t nq, int lists, int k_in,
                                                         int64_t qstride, int64_t lstride, int k,
                                                         int2* __restrict__ out, const int* __restrict__ qexp) {
    constexpr int NWM = 8;
    __shared__ int2 part[NWM * 32 * S];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t q = blockIdx.x;
    if (q >= nq) return;  // block-uniform
    const int2* base = in + q * qstride;
    const int64_t total = (int64_t)lists * k_in;
    WarpTopK<S> top;
    top.init();
    for (int64_t j0 = (int64_t)warp * 32; j0 < total; j0 += NWM * 32) {
        const int64_t j = j0 + lane;
        int2 e = make_int2(0x7f800000, SENTINEL_ID);
        if (j < total) {
            const int64_t l = j / k_in, i = j - l * k_in;
            e = base[l * lstride + i];
        }
        top.offer(__int_as_float(e.x), e.y, j < total && e.y >= 0, k);
    }
    top.store(part + warp * k, k);
    __syncthreads();
    if (warp != 0) return;
    WarpTopK<S> fin;
    fin.init();
    for (int j0 = 0; j0 < NWM * k; j0 += 32) {
        const int j = j0 + lane;
        const int2 e = j < NWM * k ? part[j] : make_int2(0x7f800000, SENTINEL_ID);
        fin.offer(__int_as_float(e.x), e.y, j < NWM * k, k);
    }
    const float scale = qexp ? exp2_int(-qexp[q]) : 1.f;
#pragma unroll
    for (int r = 0; r < S; ++r) {
        const int e = r * 32 + lane;
        if (e < k) {
            const bool pad = fin.id[r] == SENTINEL_ID;
            out[q * k + e] = pad ? make_int2(0x7f800000, -1)
                                 : make_int2(__float_as_int(qexp ? __fmul_rn(fin.d[r], scale) : fin.d[r]), fin.id[r]);
        }
    }
}

}  // namespace vk
