// IVF (inverted-file) search planning kernels (sm_100a). The scan itself is scan_kernel with IVF = true.
//
// An IVF index keeps the PQ codes of each list in a contiguous range of positions, padded to a multiple of 64 (the
// lane-placement window), with the id of every slot (-1 for padding). A search:
//   ivf_probe_kernel   per query: the nprobe lists with the smallest exact l2sq(query, coarse centroid), ties to the
//                      lower list (WarpTopK), ascending; resets the query's pruning state
//   ivf_count_kernel   queries per list
//   ivf_plan_kernel    prefix sums: each list's first (query, probe) pair and first work item; the item count
//   ivf_fill_kernel    the (query, probe slot) pairs grouped by list
//   ivf_items_kernel   work items: (list, up to Q pairs); the last item of a list is padded with (-1, -1)
// then ivf_lut_kernel (one LUT per item, in the scan layout), scan_kernel<..., IVF> and merge_kernel over the
// [query][probe slot][k] lists. Pairs land in a list in an order set by atomics; a query's result does not depend
// on which items its pairs share (the k smallest (distance, id) pairs of the rows it scans are unique).
#pragma once
#include <cfloat>
#include <cstdint>

#include "vk_device.cuh"
#include "warp_topk.cuh"

namespace vk {

// One warp per query (4 per block). Lane l computes l2sq(query, coarse[j]) for lists j = l, l + 32, ... with the
// reference's l2sq arithmetic (common.hpp:27-34: sequential dimensions, separately rounded operations).
template <int S>
__global__ void __launch_bounds__(128) ivf_probe_kernel(const float* __restrict__ queries, int64_t nq, int d,
                                                        const float* __restrict__ coarse, int nlist, int nprobe,
                                                        int32_t* __restrict__ probes, uint32_t* __restrict__ bound,
                                                        int2* __restrict__ glist, int* __restrict__ glock, int k) {
    const int lane = threadIdx.x & 31;
    const int64_t q = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
    if (q >= nq) return;  // warp-uniform
    const float* qv = queries + q * d;
    WarpTopK<S> top;
    top.init();
    for (int j0 = 0; j0 < nlist; j0 += 32) {
        const int j = j0 + lane;
        float acc = 0.f;
        if (j < nlist) {
            const float* cv = coarse + (int64_t)j * d;
            for (int t = 0; t < d; ++t) {
                const float diff = __fsub_rn(__ldg(qv + t), __ldg(cv + t));
                acc = __fadd_rn(acc, __fmul_rn(diff, diff));
            }
        }
        top.offer(acc, j, j < nlist, nprobe);
    }
    static_for<S>([&](auto r) {
        const int e = r * 32 + lane;
        if (e < nprobe) probes[q * nprobe + e] = top.id[r] == SENTINEL_ID ? -1 : top.id[r];
    });
    // the pruned scan's per-query state: bound +inf, empty global list, lock free
    for (int t = lane; t < k; t += 32) glist[q * k + t] = make_int2(0x7f800000, SENTINEL_ID);
    if (lane == 0) {
        bound[q] = 0x7f800000u;
        glock[q] = 0;
    }
}

__global__ void ivf_count_kernel(const int32_t* __restrict__ probes, int64_t pairs, int* __restrict__ cnt) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < pairs; i += (int64_t)gridDim.x * blockDim.x) {
        const int l = probes[i];
        if (l >= 0) atomicAdd(cnt + l, 1);
    }
}

// One block of 1024 threads: pair_off[l] = pairs of lists < l, item_off[l] = items of lists < l (ceil(cnt / Q)
// each), both with their totals at [nlist]; *nitems = the item total.
__global__ void __launch_bounds__(1024) ivf_plan_kernel(const int* __restrict__ cnt, int nlist, int Q,
                                                        int64_t* __restrict__ pair_off, int* __restrict__ item_off,
                                                        int* __restrict__ nitems) {
    __shared__ int64_t sp[1024];
    __shared__ int si[1024];
    const int per = (nlist + 1023) / 1024;
    const int a0 = min(nlist, (int)threadIdx.x * per), a1 = min(nlist, a0 + per);
    int64_t p = 0;
    int it = 0;
    for (int l = a0; l < a1; ++l) {
        p += cnt[l];
        it += (cnt[l] + Q - 1) / Q;
    }
    sp[threadIdx.x] = p;
    si[threadIdx.x] = it;
    __syncthreads();
    if (threadIdx.x == 0) {  // exclusive scan of the 1024 segment sums
        int64_t ps = 0;
        int is = 0;
        for (int t = 0; t < 1024; ++t) {
            const int64_t x = sp[t];
            const int y = si[t];
            sp[t] = ps;
            si[t] = is;
            ps += x;
            is += y;
        }
        pair_off[nlist] = ps;
        item_off[nlist] = is;
        *nitems = is;
    }
    __syncthreads();
    p = sp[threadIdx.x];
    it = si[threadIdx.x];
    for (int l = a0; l < a1; ++l) {
        pair_off[l] = p;
        item_off[l] = it;
        p += cnt[l];
        it += (cnt[l] + Q - 1) / Q;
    }
}

__global__ void ivf_fill_kernel(const int32_t* __restrict__ probes, int64_t nq, int nprobe,
                                const int64_t* __restrict__ pair_off, int* __restrict__ fill,
                                int2* __restrict__ by_list) {
    const int64_t pairs = nq * nprobe;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < pairs; i += (int64_t)gridDim.x * blockDim.x) {
        const int l = probes[i];
        if (l < 0) continue;
        const int slot = atomicAdd(fill + l, 1);
        by_list[pair_off[l] + slot] = make_int2((int)(i / nprobe), (int)(i % nprobe));
    }
}

// Blocks stride over the lists; the threads of a block fill the Q pair slots of the list's items.
__global__ void ivf_items_kernel(const int64_t* __restrict__ pair_off, const int* __restrict__ item_off, int nlist,
                                 int Q, const int2* __restrict__ by_list, int* __restrict__ item_list,
                                 int2* __restrict__ item_pairs) {
    for (int l = blockIdx.x; l < nlist; l += gridDim.x) {
        const int64_t p0 = pair_off[l], p1 = pair_off[l + 1];
        const int i0 = item_off[l], i1 = item_off[l + 1];
        for (int64_t t = threadIdx.x; t < (int64_t)(i1 - i0) * Q; t += blockDim.x) {
            const int64_t item = i0 + t / Q;
            const int64_t p = p0 + t;
            item_pairs[item * Q + t % Q] = p < p1 ? by_list[p] : make_int2(-1, -1);
            if (t % Q == 0) item_list[item] = l;
        }
    }
}

// Nearest coarse centroid of each row (exact l2sq, the first minimum wins, as the reference's nearest_centroid,
// pq.cpp:11-22): one thread per row, centroids read through the cache (every thread of a warp reads the same one).
__global__ void ivf_assign_kernel(const float* __restrict__ x, int64_t n, int d, const float* __restrict__ coarse,
                                  int nlist, int32_t* __restrict__ out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float* xv = x + i * d;
        float best = FLT_MAX;
        int bi = 0;
        for (int l = 0; l < nlist; ++l) {
            const float* cv = coarse + (int64_t)l * d;
            float acc = 0.f;
            for (int t = 0; t < d; ++t) {
                const float diff = __fsub_rn(xv[t], __ldg(cv + t));
                acc = __fadd_rn(acc, __fmul_rn(diff, diff));
            }
            if (acc < best) {
                best = acc;
                bi = l;
            }
        }
        out[i] = bi;
    }
}

}  // namespace vk
