// Auxiliary VecKern-B200 kernels (non-template): materialising scan for distances(), code layout transforms,
// the synthetic code generator and PQ encoding. Included only by vk_abi.cu.
#pragma once
#include <cfloat>
#include <cstdint>

#include "kernels.cuh"

namespace vk {

// ------------------------------------------------------------------------------------------------ distances
// Materialising ADC scan for PQSearcher::distances (src/cuda/searcher.cu:522-547): grid (bx, nq_batch),
// block T; the query's [s][c] LUT in shared memory; dists[q][i] for every row i < n, same add order.
__global__ void dist_kernel(const uint4* __restrict__ codes, const float* __restrict__ lut, int64_t n, int m,
                            int W, float* __restrict__ out) {
    extern __shared__ float slut[];
    const float* src = lut + (int64_t)blockIdx.y * m * KSUB;
    for (int t = threadIdx.x; t < m * KSUB; t += blockDim.x) slut[t] = src[t];
    __syncthreads();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const uint4* row = codes + (i >> 5) * W * 32 + (i & 31);
        float acc = 0.f;
        for (int w = 0; w < W; ++w) {
            const uint4 v = row[w * 32];
#pragma unroll
            for (int b = 0; b < 16; ++b) {
                const int s = w * 16 + b;
                if (s >= m) break;
                const uint32_t c = (word_of(v, b) >> (8 * (b & 3))) & 0xffu;
                acc = __fadd_rn(acc, slut[s * KSUB + c]);
            }
        }
        out[(int64_t)blockIdx.y * n + i] = acc;
    }
}

// ------------------------------------------------------------------------------------------------ layouts
// Row-major codes of rows [row0, row0 + cnt) (row0 a multiple of 32) -> the interleaved words of the 32-row
// groups covering them; one thread per output uint4. Rows >= n are left untouched (the buffer is zeroed first).
__global__ void interleave_kernel(const uint8_t* __restrict__ rows, int64_t row0, int64_t cnt, int64_t n, int m,
                                  int W, uint4* __restrict__ out) {
    const int64_t g0 = row0 >> 5, ngroups = (cnt + 31) >> 5;
    const int64_t total = ngroups * W * 32;
    for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < total; o += (int64_t)gridDim.x * blockDim.x) {
        const int64_t l = o & 31, w = (o >> 5) % W, g = g0 + (o >> 5) / W;
        const int64_t i = g * 32 + l;
        if (i >= n) continue;
        uint32_t word[4] = {0, 0, 0, 0};
        if (i - row0 < cnt) {
            const uint8_t* src = rows + (i - row0) * m;
            for (int b = 0; b < 16; ++b) {
                const int s = (int)w * 16 + b;
                if (s < m) word[b >> 2] |= (uint32_t)src[s] << (8 * (b & 3));
            }
        }
        out[(g * W + w) * 32 + l] = make_uint4(word[0], word[1], word[2], word[3]);
    }
}

// Inverse of interleave_kernel for rows [first, first + count): row-major output (tests and tools).
__global__ void deinterleave_kernel(const uint4* __restrict__ codes, int64_t first, int64_t count, int m, int W,
                                    uint8_t* __restrict__ out) {
    const int64_t total = count * m;
    for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < total; o += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = o / m, s = o - r * m;
        const int64_t i = first + r;
        const uint4 v = codes[((i >> 5) * W + (s >> 4)) * 32 + (i & 31)];
        out[o] = (uint8_t)((word_of(v, (int)(s & 15)) >> (8 * (s & 3))) & 0xffu);
    }
}

// ------------------------------------------------------------------------------------------------ generator
// Synthetic code generator (BASELINE configs 3/4): gen_code in vk_gen.h, identical on host and device.
// Generated codes written straight into the interleaved layout; rows >= n are zero.
__global__ void gen_interleaved_kernel(uint64_t key, const uint32_t* __restrict__ cdf, int clusters, int m, int W,
                                       int64_t row_first, int64_t n, int64_t n_pad, uint4* __restrict__ out) {
    const int64_t total = n_pad * W;
    for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < total; o += (int64_t)gridDim.x * blockDim.x) {
        const int64_t l = o & 31, w = (o >> 5) % W, g = (o >> 5) / W;
        const int64_t i = g * 32 + l;
        uint32_t word[4] = {0, 0, 0, 0};
        if (i < n) {
            for (int b = 0; b < 16; ++b) {
                const int s = (int)w * 16 + b;
                if (s < m) word[b >> 2] |= gen_code(key, (uint64_t)(row_first + i), s, cdf, clusters, m) << (8 * (b & 3));
            }
        }
        out[o] = make_uint4(word[0], word[1], word[2], word[3]);
    }
}

__global__ void gen_rows_kernel(uint64_t key, const uint32_t* __restrict__ cdf, int clusters, int m,
                                int64_t row_first, int64_t n, uint8_t* __restrict__ out) {
    const int64_t total = n * m;
    for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < total; o += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = o / m;
        const int s = (int)(o - r * m);
        out[o] = (uint8_t)gen_code(key, (uint64_t)(row_first + r), s, cdf, clusters, m);
    }
}

// ------------------------------------------------------------------------------------------------ encode
// Nearest centroid per (row, sub-space) under the reference's l2sq, strict < so the first minimum wins
// (src/cpu/pq.cpp:11-22, 71-76). grid (ceil(n / 256), m), block 256; sub-space centroids in shared memory.
__global__ void __launch_bounds__(256) encode_kernel(const float* __restrict__ centroids, int m, int dsub,
                                                     const float* __restrict__ x, int64_t n,
                                                     uint8_t* __restrict__ codes) {
    extern __shared__ float scen[];  // [256][dsub]
    const int s = blockIdx.y;
    for (int t = threadIdx.x; t < KSUB * dsub; t += blockDim.x) scen[t] = centroids[(int64_t)s * KSUB * dsub + t];
    __syncthreads();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float* xs = x + i * ((int64_t)m * dsub) + (int64_t)s * dsub;
    int best = 0;
    float best_d = FLT_MAX;
    for (int c = 0; c < KSUB; ++c) {
        float acc = 0.f;
        for (int j = 0; j < dsub; ++j) {
            const float diff = __fsub_rn(xs[j], scen[c * dsub + j]);
            acc = __fadd_rn(acc, __fmul_rn(diff, diff));
        }
        if (acc < best_d) {
            best_d = acc;
            best = c;
        }
    }
    codes[i * m + s] = (uint8_t)best;
}

// ------------------------------------------------------------------------------------------------ re-rank
// Exact re-rank (the reference's rerank_exact, src/cpu/cpu_ref.cpp:66-77): one warp per query; lane l re-scores
// candidates l, l + 32, ... with l2sq(query, base row) summed over j in order, each operation rounded on its own
// (diff = q - b, acc += diff * diff; no FMA), and the warp keeps the k best (dist, id) in candidate order through
// WarpTopK (same admission rule as the reference's heap, so duplicates and ties come out identically).
// Candidate ids < 0 are skipped. The query row is staged in shared memory (block: 4 warps, 4 queries).
template <int S>
__global__ void __launch_bounds__(128) rerank_kernel(const float* __restrict__ base, int d,
                                                     const float* __restrict__ queries, int64_t nq,
                                                     const int2* __restrict__ cand, int r, int k,
                                                     int2* __restrict__ out) {
    extern __shared__ float sq[];  // [4][d]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t q = (int64_t)blockIdx.x * 4 + warp;
    float* my_q = sq + warp * d;
    if (q < nq)
        for (int j = lane; j < d; j += 32) my_q[j] = queries[q * d + j];
    __syncwarp();
    if (q >= nq) return;  // warp-uniform
    WarpTopK<S> top;
    top.init();
    for (int j0 = 0; j0 < r; j0 += 32) {
        const int j = j0 + lane;
        const int id = j < r ? cand[q * r + j].y : -1;
        float acc = 0.f;
        if (id >= 0) {
            const float* b = base + (int64_t)id * d;
            for (int t = 0; t < d; ++t) {
                const float diff = __fsub_rn(my_q[t], b[t]);
                acc = __fadd_rn(acc, __fmul_rn(diff, diff));
            }
        }
        // candidates are pushed in candidate order: offer the 32 of this round one lane at a time, so ties and
        // duplicates meet the list in the same order as the reference's loop
        for (int src = 0; src < 32; ++src) {
            const float x = __shfl_sync(FULL, acc, src);
            const int xi = __shfl_sync(FULL, id, src);
            if (xi >= 0 && top.admits(x, xi)) top.insert(x, xi, k);
        }
    }
    static_for<S>([&](auto rr) {
        const int e = rr * 32 + lane;
        if (e < k) {
            const bool pad = top.id[rr] == SENTINEL_ID;
            out[q * k + e] = pad ? make_int2(0x7f800000, -1) : make_int2(__float_as_int(top.d[rr]), top.id[rr]);
        }
    });
}

}  // namespace vk
