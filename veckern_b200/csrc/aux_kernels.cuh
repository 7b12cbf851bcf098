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
__global__ void dist_kernel(const uint4* __restrict__ codes, const uint8_t* __restrict__ perm,
                            const float* __restrict__ lut, int64_t n, int m, int W, float* __restrict__ out) {
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
        out[(int64_t)blockIdx.y * n + (i & ~(int64_t)(PLACE_WINDOW - 1)) + perm[i]] = acc;  // column = row id
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

// Identity lane placement (4-bit indexes): position p holds row p.
__global__ void identity_perm_kernel(uint8_t* __restrict__ perm, int64_t n_pad) {
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < n_pad; p += (int64_t)gridDim.x * blockDim.x)
        perm[p] = (uint8_t)(p & (PLACE_WINDOW - 1));
}

// Inverse of interleave_kernel + place_rows_kernel for rows [first, first + count): row-major output (tests and
// tools). One thread per (position, sub-space) of the placement windows covering the rows.
__global__ void deinterleave_kernel(const uint4* __restrict__ codes, const uint8_t* __restrict__ perm, int64_t first,
                                    int64_t count, int m, int W, uint8_t* __restrict__ out) {
    const int64_t p0 = first & ~(int64_t)(PLACE_WINDOW - 1);
    const int64_t total = ((first + count + PLACE_WINDOW - 1) / PLACE_WINDOW * PLACE_WINDOW - p0) * m;
    for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < total; o += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = p0 + o / m, s = o % m;
        const int64_t row = (i & ~(int64_t)(PLACE_WINDOW - 1)) + perm[i];
        if (row < first || row >= first + count) continue;
        const uint4 v = codes[((i >> 5) * W + (s >> 4)) * 32 + (i & 31)];
        out[(row - first) * m + s] = (uint8_t)((word_of(v, (int)(s & 15)) >> (8 * (s & 3))) & 0xffu);
    }
}

// ------------------------------------------------------------------------------------------------ lane placement
// Index build: reorders the rows of every whole window of PLACE_WINDOW rows (all positions < n; other windows and
// m > 64 keep the identity) and records the order in perm. A warp's LUT fetch is served in phases of P lanes, P
// bank groups each (P = 8: 16-byte entries, Q >= 4 layouts; P = 16: 8-byte entries, Q = 2): entry c of a sub-space
// table lies in group c mod P. The cost of a placement is the sum over sub-spaces (weight w_s) and phases of the
// largest number of the phase's rows whose codes share a group, i.e. the fetch's wavefronts when no two of those
// rows hold the same code. Hill climbing: `steps` swaps of two positions in different phases, drawn from a
// per-window xorshift sequence seeded by a counter-based hash (deterministic layout), each kept when it does not
// raise the cost. Weights follow the pruned scan: w = 20 for s < first_depth (phase A of every row), 6 for
// s < last_depth, 1 beyond.
// One warp per window; lane l keeps the counts of sub-spaces l and l + 32.
__host__ __device__ constexpr uint32_t place_warp_smem(int m, int W) { return (uint32_t)(PLACE_WINDOW * W * 16 + PLACE_WINDOW * m + PLACE_WINDOW); }

template <int P>
__device__ __forceinline__ uint32_t max_byte(const uint32_t (&w)[P / 4]) {
    uint32_t t = w[0];
#pragma unroll
    for (int i = 1; i < P / 4; ++i) t = __vmaxu4(t, w[i]);
    t = __vmaxu4(t, t >> 16);
    t = __vmaxu4(t, t >> 8);
    return t & 0xffu;
}

template <int P>
__global__ void __launch_bounds__(128) place_rows_kernel(uint4* __restrict__ codes, int64_t n, int64_t n_pad, int m,
                                                         int W, uint8_t* __restrict__ perm, int first_depth,
                                                         int last_depth, int steps, uint64_t key) {
    static_assert(PLACE_WINDOW == 64 && (P == 8 || P == 16), "two positions per lane, phases of 8 or 16 lanes");
    constexpr int PH = PLACE_WINDOW / P;  // phases per window
    extern __shared__ __align__(16) unsigned char place_smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, wpb = blockDim.x >> 5;
    const uint32_t per_warp = (place_warp_smem(m, W) + 15u) & ~15u;
    unsigned char* mine = place_smem + warp * per_warp;
    uint4* words = reinterpret_cast<uint4*>(mine);                  // [64][W]: the window's rows, in row order
    const unsigned char* row_codes = mine;                          // row r, sub-space s at r * W * 16 + s
    unsigned char* cnt = mine + PLACE_WINDOW * W * 16;              // [PH][m][P]
    unsigned char* order = cnt + PLACE_WINDOW * m;                  // [64]: row at each position
    const int64_t windows = n_pad / PLACE_WINDOW;
    for (int64_t win = (int64_t)blockIdx.x * wpb + warp; win < windows; win += (int64_t)gridDim.x * wpb) {
        const int64_t p0 = win * PLACE_WINDOW;
        if (p0 + PLACE_WINDOW > n || W > 4) {
            perm[p0 + lane] = (uint8_t)lane;
            perm[p0 + 32 + lane] = (uint8_t)(32 + lane);
            continue;
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int p = h * 32 + lane;
            const int64_t i = p0 + p;
            for (int w = 0; w < W; ++w) words[p * W + w] = codes[((i >> 5) * W + w) * 32 + (i & 31)];
            order[p] = (uint8_t)p;
        }
        for (int t = lane; t < PLACE_WINDOW * m; t += 32) cnt[t] = 0;
        __syncwarp();
        for (int h = 0; h < 2; ++h) {
            const int s = lane + 32 * h;
            if (s < m)
                for (int p = 0; p < PLACE_WINDOW; ++p)
                    ++cnt[((p / P) * m + s) * P + (row_codes[p * W * 16 + s] & (P - 1))];
        }
        __syncwarp();
        uint32_t rs = (uint32_t)mix64(key ^ (uint64_t)win) | 1u;  // xorshift32 state, seeded per window
        for (int it = 0; it < steps; ++it) {
            rs ^= rs << 13;
            rs ^= rs >> 17;
            rs ^= rs << 5;
            const int i = (int)(rs & 63u), j = (int)((rs >> 6) & 63u);
            const int pa = i / P, pb = j / P;
            if (pa == pb) continue;  // uniform: every lane draws the same pair
            const int ri = order[i], rj = order[j];
            int delta = 0;
            uint32_t na[2][P / 4], nb[2][P / 4];
            bool moved[2] = {false, false};
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int s = lane + 32 * h;
                if (s >= m) continue;
                const int ci = row_codes[ri * W * 16 + s] & (P - 1), cj = row_codes[rj * W * 16 + s] & (P - 1);
                if (ci == cj) continue;
                const uint32_t* ca = reinterpret_cast<const uint32_t*>(cnt + (pa * m + s) * P);
                const uint32_t* cb = reinterpret_cast<const uint32_t*>(cnt + (pb * m + s) * P);
#pragma unroll
                for (int e = 0; e < P / 4; ++e) {
                    na[h][e] = ca[e];
                    nb[h][e] = cb[e];
                }
                const int before = (int)max_byte<P>(na[h]) + (int)max_byte<P>(nb[h]);
                // row ri moves from phase pa to pb, row rj the other way
                na[h][ci >> 2] -= 1u << (8 * (ci & 3));
                na[h][cj >> 2] += 1u << (8 * (cj & 3));
                nb[h][cj >> 2] -= 1u << (8 * (cj & 3));
                nb[h][ci >> 2] += 1u << (8 * (ci & 3));
                const int after = (int)max_byte<P>(na[h]) + (int)max_byte<P>(nb[h]);
                const int wgt = s < first_depth ? 20 : s < last_depth ? 6 : 1;
                delta += wgt * (after - before);
                moved[h] = true;
            }
            delta = __reduce_add_sync(FULL, delta);
            if (delta <= 0) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    if (!moved[h]) continue;
                    const int s = lane + 32 * h;
                    uint32_t* ca = reinterpret_cast<uint32_t*>(cnt + (pa * m + s) * P);
                    uint32_t* cb = reinterpret_cast<uint32_t*>(cnt + (pb * m + s) * P);
#pragma unroll
                    for (int e = 0; e < P / 4; ++e) {
                        ca[e] = na[h][e];
                        cb[e] = nb[h][e];
                    }
                }
                if (lane == 0) {
                    order[i] = (uint8_t)rj;
                    order[j] = (uint8_t)ri;
                }
            }
            __syncwarp();
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int p = h * 32 + lane;
            const int r = order[p];
            const int64_t i = p0 + p;
            for (int w = 0; w < W; ++w) codes[((i >> 5) * W + w) * 32 + (i & 31)] = words[r * W + w];
            perm[i] = (uint8_t)r;
        }
        __syncwarp();  // the warp's shared buffers are reused by its next window
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

// ------------------------------------------------------------------------------------------------ PQ training
// Lloyd iterations of ProductQuantizer::train (src/cpu/pq.cpp:31-69) for one sub-space s, bit-identical to it:
// the assignment is the encoder's nearest centroid (strict <, first minimum wins, from FLT_MAX; pq.cpp:11-22) and
// each centroid's sums are accumulated in row order from +0 (pq.cpp:55-58), then divided by the count as a float
// (pq.cpp:64). The host drives the loop and the std::mt19937_64 draws (shuffle, empty-cluster reseeds).

// cent[c] = sub-vector s of row rows[c], c < 256 (the initial centroids: the first 256 rows of the shuffle).
__global__ void train_gather_kernel(const float* __restrict__ x, int d, int s, int dsub,
                                    const int64_t* __restrict__ rows, float* __restrict__ cent) {
    for (int t = threadIdx.x; t < KSUB * dsub; t += blockDim.x) {
        const int c = t / dsub, j = t - c * dsub;
        cent[t] = x[rows[c] * d + (int64_t)s * dsub + j];
    }
}

// assign[i] = nearest centroid of row i's sub-vector s; the 256 centroids in shared memory.
__global__ void __launch_bounds__(256) train_assign_kernel(const float* __restrict__ x, int64_t n, int d, int s,
                                                           int dsub, const float* __restrict__ cent,
                                                           int* __restrict__ assign) {
    extern __shared__ float tcen[];  // [256][dsub]
    for (int t = threadIdx.x; t < KSUB * dsub; t += blockDim.x) tcen[t] = cent[t];
    __syncthreads();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float* v = x + i * d + (int64_t)s * dsub;
        int best = 0;
        float best_dist = FLT_MAX;
        for (int c = 0; c < KSUB; ++c) {
            float acc = 0.f;
            for (int j = 0; j < dsub; ++j) {
                const float diff = __fsub_rn(v[j], tcen[c * dsub + j]);
                acc = __fadd_rn(acc, __fmul_rn(diff, diff));
            }
            if (acc < best_dist) {
                best_dist = acc;
                best = c;
            }
        }
        assign[i] = best;
    }
}

// One warp per centroid c: sums[c] = sub-vectors of the rows assigned to c, added in row order; counts[c].
// Lane l holds components l, l + 32, ... (dsub <= 128).
__global__ void __launch_bounds__(256) train_sums_kernel(const float* __restrict__ x, int64_t n, int d, int s, int dsub,
                                                         const int* __restrict__ assign, float* __restrict__ sums,
                                                         int* __restrict__ counts) {
    const int lane = threadIdx.x & 31;
    const int c = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (c >= KSUB) return;  // warp-uniform
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int count = 0;
    for (int64_t i0 = 0; i0 < n; i0 += 128) {  // four 32-row groups per step: their loads are in flight together
        int a[4];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const int64_t i = i0 + 32 * g + lane;
            a[g] = i < n ? assign[i] : -1;
        }
#pragma unroll
        for (int g = 0; g < 4; ++g) {  // groups in row order, rows within a group in order
            unsigned mask = __ballot_sync(FULL, a[g] == c);
            count += __popc(mask);
            while (mask) {
                const int64_t row = i0 + 32 * g + __ffs(mask) - 1;
                mask &= mask - 1;
                const float* v = x + row * d + (int64_t)s * dsub;
#pragma unroll
                for (int r = 0; r < 4; ++r)
                    if (lane + 32 * r < dsub) acc[r] = __fadd_rn(acc[r], v[lane + 32 * r]);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r)
        if (lane + 32 * r < dsub) sums[c * dsub + lane + 32 * r] = acc[r];
    if (lane == 0) counts[c] = count;
}

// cent[c] = sums[c] / counts[c], or sub-vector s of row reseed[c] for an empty cluster (pq.cpp:60-66).
__global__ void train_update_kernel(const float* __restrict__ x, int d, int s, int dsub, const float* __restrict__ sums,
                                    const int* __restrict__ counts, const int64_t* __restrict__ reseed,
                                    float* __restrict__ cent) {
    for (int t = threadIdx.x; t < KSUB * dsub; t += blockDim.x) {
        const int c = t / dsub, j = t - c * dsub;
        cent[t] = counts[c] == 0 ? x[reseed[c] * d + (int64_t)s * dsub + j]
                                 : __fdiv_rn(sums[t], (float)counts[c]);
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

// Shape-specialised versions of encode_kernel / train_assign_kernel for dsub in {1, 2, 4, 8, 16, 32}: the row's
// sub-vector in registers, four centroids' distances computed side by side (each summed over j in order, every
// operation rounded on its own), then compared in centroid order, so the first minimum still wins.
template <int DSUB>
__device__ __forceinline__ int nearest_centroid(const float (&v)[DSUB], const float* __restrict__ cen) {
    int best = 0;
    float best_d = FLT_MAX;
    for (int c = 0; c < KSUB; c += 4) {
        float acc[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            acc[t] = 0.f;
#pragma unroll
            for (int j = 0; j < DSUB; ++j) {
                const float diff = __fsub_rn(v[j], cen[(c + t) * DSUB + j]);
                acc[t] = __fadd_rn(acc[t], __fmul_rn(diff, diff));
            }
        }
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            if (acc[t] < best_d) {
                best_d = acc[t];
                best = c + t;
            }
        }
    }
    return best;
}

template <int DSUB>
__global__ void __launch_bounds__(256) encode_kernel_t(const float* __restrict__ centroids, int m,
                                                       const float* __restrict__ x, int64_t n,
                                                       uint8_t* __restrict__ codes) {
    __shared__ float scen[KSUB * DSUB];
    const int s = blockIdx.y;
    for (int t = threadIdx.x; t < KSUB * DSUB; t += blockDim.x) scen[t] = centroids[(int64_t)s * KSUB * DSUB + t];
    __syncthreads();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float* xs = x + i * ((int64_t)m * DSUB) + (int64_t)s * DSUB;
    float v[DSUB];
#pragma unroll
    for (int j = 0; j < DSUB; ++j) v[j] = xs[j];
    codes[i * m + s] = (uint8_t)nearest_centroid<DSUB>(v, scen);
}

template <int DSUB>
__global__ void __launch_bounds__(256) train_assign_kernel_t(const float* __restrict__ x, int64_t n, int d, int s,
                                                             const float* __restrict__ cent, int* __restrict__ assign) {
    __shared__ float tcen[KSUB * DSUB];
    for (int t = threadIdx.x; t < KSUB * DSUB; t += blockDim.x) tcen[t] = cent[t];
    __syncthreads();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float* xs = x + i * d + (int64_t)s * DSUB;
        float v[DSUB];
#pragma unroll
        for (int j = 0; j < DSUB; ++j) v[j] = xs[j];
        assign[i] = nearest_centroid<DSUB>(v, tcen);
    }
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
