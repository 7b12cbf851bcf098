// extern "C" shim over the reference's own GPU library — BENCHMARK COMPARISON ONLY, never product code.
//
// oracle/Makefile (target refgpu) compiles this file with the reference's unmodified src/cuda/searcher.cu (+
// kernels.cuh) for sm_100a and its CPU sources (read where they lie) into oracle/_ref/libveckern_refgpu.so. It lets
// bench.py's reference arm run the reference's final kernel (ScanVariant::FusedWarp, "v8") on the same centroids,
// codes and queries as this repository's search, through the reference's own veckern::gpu::PQSearcher, with the
// tuning grid the reference's campaign sweeps (scripts/run_all.sh:87-91: queries_per_block x ilp) and its timing
// convention (bench/bench_main.cpp:191-214: one warm-up search, then the median of `reps` searches' stage times).
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

#include "veckern/gpu.hpp"
#include "veckern/pq.hpp"

namespace {
std::string g_err;

double median(std::vector<double> v) {
    std::sort(v.begin(), v.end());
    return v.empty() ? 0.0 : v[v.size() / 2];
}
}  // namespace

extern "C" {

const char* refgpu_last_error() { return g_err.c_str(); }

// For tuning point p (queries_per_block qs[p], vectors_per_step ilps[p], the reference's other defaults) writes
// out[p * 10 + 0..9] = {total_ms, transfer_ms, lut_ms, scan_ms, select_ms (medians), threads, blocks_x, grid_y,
// queries_per_block, vectors_per_step (the launch the reference reports)}. The first point's last result goes to
// out_d / out_i (nq x k). Returns 0, or -1 with refgpu_last_error() set.
int refgpu_sweep(const float* centroids, int64_t d, int64_t m, const uint8_t* codes, int64_t n, const float* queries,
                 int64_t nq, int64_t k, const int* qs, const int* ilps, int points, int reps, double* out,
                 float* out_d, int32_t* out_i) {
    try {
        veckern::ProductQuantizer pq((std::size_t)d, (std::size_t)m);
        const auto& c = pq.centroids();  // the reference has no setter; configs with given centroids need one
        std::memcpy(const_cast<float*>(c.data()), centroids, c.size() * sizeof(float));
        veckern::gpu::PQSearcher s(pq, codes, (std::size_t)n);
        std::vector<veckern::Neighbor> res((std::size_t)(nq * k));
        for (int p = 0; p < points; ++p) {
            veckern::gpu::Tuning t;
            t.queries_per_block = qs[p];
            t.vectors_per_step = ilps[p];
            s.set_tuning(t);
            const auto v = veckern::gpu::ScanVariant::FusedWarp;
            s.search(queries, (std::size_t)nq, (std::size_t)k, v, res.data());  // warm-up (and layout build)
            std::vector<double> total, xfer, lut, scan, sel;
            for (int r = 0; r < reps; ++r) {
                const auto tm = s.search(queries, (std::size_t)nq, (std::size_t)k, v, res.data());
                total.push_back(tm.total_ms());
                xfer.push_back(tm.transfer_ms);
                lut.push_back(tm.lut_ms);
                scan.push_back(tm.scan_ms);
                sel.push_back(tm.select_ms);
            }
            const auto sh = s.last_launch();
            double* o = out + (std::size_t)p * 10;
            o[0] = median(total);
            o[1] = median(xfer);
            o[2] = median(lut);
            o[3] = median(scan);
            o[4] = median(sel);
            o[5] = sh.threads;
            o[6] = sh.blocks_x;
            o[7] = sh.grid_y;
            o[8] = sh.queries_per_block;
            o[9] = sh.vectors_per_step;
            if (p == 0)
                for (std::size_t j = 0; j < res.size(); ++j) {
                    out_d[j] = res[j].dist;
                    out_i[j] = res[j].id;
                }
        }
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

}  // extern "C"
