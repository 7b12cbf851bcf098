// Warp-cooperative bounded top-k: one sorted list of k (dist, id) pairs per warp, entry e held by lane e % 32 in
// register e / 32 (S = ceil(k / 32) registers per lane). Same contract as the reference's WarpTopK
// (src/cuda/kernels.cuh:392-466): k smallest under the (dist, id) order; here k is a run-time value <= 32 * S.
//
// Insertion of an admitted candidate: one ballot per register counts the entries below it (its position p),
// then every entry at or after p moves up by one (shfl_up within a register, lane 31 of register r carrying into
// lane 0 of register r + 1) and slot p takes the candidate. Entries past k - 1 are never read as results; they
// only ever hold values that are not below the current threshold, so they never disturb the position count.
#pragma once
#include "vk_device.cuh"

namespace vk {

// Compile-time loop: f(Int<i>) for i = 0 .. N-1. Arrays indexed by i keep constant indices (and stay in registers)
// however large the loop body gets, where `#pragma unroll` is only a request (nvcc left the k = 100 lists' loops
// rolled and moved the lists to local memory).
template <int I>
struct Int {
    static constexpr int value = I;
    __host__ __device__ constexpr operator int() const { return I; }
};
template <int I, int N, class F>
__device__ __forceinline__ void static_for_impl(F&& f) {
    if constexpr (I < N) {
        f(Int<I>{});
        static_for_impl<I + 1, N>(f);
    }
}
template <int N, class F>
__device__ __forceinline__ void static_for(F&& f) {
    static_for_impl<0, N>(f);
}

template <int S>
struct WarpTopK {
    float d[S];
    int32_t id[S];
    float thr_d;  // entry k - 1 (warp-uniform): the admission threshold
    int32_t thr_i;

    __device__ __forceinline__ void init() {
        static_for<S>([&](auto r) {
            d[r] = __int_as_float(0x7f800000);  // +inf
            id[r] = SENTINEL_ID;
        });
        thr_d = __int_as_float(0x7f800000);
        thr_i = SENTINEL_ID;
    }

    __device__ __forceinline__ bool admits(float x, int32_t xi) const { return nb_less(x, xi, thr_d, thr_i); }

    // All 32 lanes call with the same (x, xi), which admits() accepted.
    __device__ __forceinline__ void insert(float x, int32_t xi, int k) {
        const int lane = threadIdx.x & (WARP - 1);
        int pos = 0;
        static_for<S>([&](auto r) { pos += __popc(__ballot_sync(FULL, nb_less(d[r], id[r], x, xi))); });
        float carry_d = x;
        int32_t carry_i = xi;
        static_for<S>([&](auto r) {
            float up_d = __shfl_up_sync(FULL, d[r], 1);
            int32_t up_i = __shfl_up_sync(FULL, id[r], 1);
            const float last_d = __shfl_sync(FULL, d[r], WARP - 1);
            const int32_t last_i = __shfl_sync(FULL, id[r], WARP - 1);
            if (lane == 0) {
                up_d = carry_d;
                up_i = carry_i;
            }
            const int e = r * WARP + lane;
            if (e == pos) {
                d[r] = x;
                id[r] = xi;
            } else if (e > pos) {
                d[r] = up_d;
                id[r] = up_i;
            }
            carry_d = last_d;
            carry_i = last_i;
        });
        const int t = k - 1;
        float td = d[0];
        int32_t ti = id[0];
        static_for<S>([&](auto r) {
            if (r > 0 && (t >> 5) == r) {
                td = d[r];
                ti = id[r];
            }
        });
        thr_d = __shfl_sync(FULL, td, t & (WARP - 1));
        thr_i = __shfl_sync(FULL, ti, t & (WARP - 1));
    }

    // One candidate per lane; admitted ones are inserted one at a time (rare once the list has filled).
    __device__ __forceinline__ void offer(float x, int32_t xi, bool valid, int k) {
        unsigned mask = __ballot_sync(FULL, valid && admits(x, xi));
        while (mask) {
            const int src = __ffs(mask) - 1;
            mask &= mask - 1;
            const float cx = __shfl_sync(FULL, x, src);
            const int32_t ci = __shfl_sync(FULL, xi, src);
            if (admits(cx, ci)) insert(cx, ci, k);  // the threshold may have dropped since the ballot
        }
    }

    // N candidates per lane (x[u], xi[u], valid[u]), e.g. the rows of N 32-row groups: one ballot per group, then
    // the admitted candidates inserted one at a time from one loop. Equivalent to N offer() calls (the k smallest of
    // distinct (dist, id) pairs do not depend on the order they arrive in), with one copy of the insertion code
    // instead of N where it is inlined.
    template <int N>
    __device__ __forceinline__ void offer_n(const float (&x)[N], const int32_t (&xi)[N], const bool (&valid)[N],
                                            int k) {
        unsigned mask[N];
        static_for<N>([&](auto u) { mask[u] = __ballot_sync(FULL, valid[u] && admits(x[u], xi[u])); });
        for (;;) {
            int uu = -1;
            unsigned mm = 0u;
            static_for<N>([&](auto c) {
                if (uu < 0 && mask[c] != 0u) {
                    uu = c;
                    mm = mask[c];
                }
            });
            if (uu < 0) break;  // warp-uniform: the masks come from ballots
            const int src = __ffs(mm) - 1;
            float v = x[0];
            int32_t vi = xi[0];
            static_for<N>([&](auto c) {
                if (c == uu) {
                    mask[c] &= mask[c] - 1u;
                    v = x[c];
                    vi = xi[c];
                }
            });
            const float cx = __shfl_sync(FULL, v, src);
            const int32_t ci = __shfl_sync(FULL, vi, src);
            if (admits(cx, ci)) insert(cx, ci, k);  // the threshold may have dropped since the ballot
        }
    }

    // Writes entries 0 .. k-1 (ascending) as (dist, id) pairs.
    __device__ __forceinline__ void store(int2* out, int k) const {
        const int lane = threadIdx.x & (WARP - 1);
        static_for<S>([&](auto r) {
            const int e = r * WARP + lane;
            if (e < k) out[e] = make_int2(__float_as_int(d[r]), id[r]);
        });
    }
};

}  // namespace vk
