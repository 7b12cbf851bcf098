// Drives veckern::gpu::PQSearcher — the C++ class the reference's callers link (include/veckern/gpu.hpp) — over
// inputs written by tests/test_dropin_gpu.py, and writes the results back for a bit-exact comparison with the CPU
// oracle. Built by that test with g++ against include/ and the in-tree libraries.
//
//   searcher_check <dir>: reads dir/meta.txt ("n m dsub nq k"), centroids.f32 ([m][256][dsub]), codes.u8 ([n][m]),
//   queries.f32 ([nq][m*dsub]); writes out_default.bin (the reference's default Tuning) and out_q8.bin
//   (queries_per_block 8, vectors_per_step 2), each nq*k (float dist, int32 id) pairs, and shape.txt with the
//   default search's LaunchShape.
#include <cstdio>
#include <exception>
#include <fstream>
#include <string>
#include <vector>

#include "veckern/gpu.hpp"
#include "veckern/pq.hpp"

namespace {
template <class T>
std::vector<T> read_all(const std::string& path, std::size_t count) {
    std::vector<T> v(count);
    std::ifstream f(path, std::ios::binary);
    f.read(reinterpret_cast<char*>(v.data()), static_cast<std::streamsize>(count * sizeof(T)));
    if (!f) throw std::runtime_error("cannot read " + path);
    return v;
}

void write_all(const std::string& path, const std::vector<veckern::Neighbor>& v) {
    std::ofstream f(path, std::ios::binary);
    f.write(reinterpret_cast<const char*>(v.data()), static_cast<std::streamsize>(v.size() * sizeof(v[0])));
    if (!f) throw std::runtime_error("cannot write " + path);
}
}  // namespace

int main(int argc, char** argv) {
    if (argc != 2) {
        std::fprintf(stderr, "usage: %s <dir>\n", argv[0]);
        return 2;
    }
    try {
        const std::string dir = argv[1];
        std::size_t n = 0, m = 0, dsub = 0, nq = 0, k = 0;
        {
            std::ifstream meta(dir + "/meta.txt");
            meta >> n >> m >> dsub >> nq >> k;
            if (!meta) throw std::runtime_error("bad meta.txt");
        }
        const auto cent = read_all<float>(dir + "/centroids.f32", m * 256 * dsub);
        const auto codes = read_all<uint8_t>(dir + "/codes.u8", n * m);
        const auto queries = read_all<float>(dir + "/queries.f32", nq * m * dsub);
        veckern::ProductQuantizer pq(m * dsub, m);
        pq.set_centroids(cent.data());
        veckern::gpu::PQSearcher searcher(pq, codes.data(), n);
        std::vector<veckern::Neighbor> out(nq * k);
        searcher.search(queries.data(), nq, k, veckern::gpu::ScanVariant::FusedWarp, out.data());
        write_all(dir + "/out_default.bin", out);
        const auto sh = searcher.last_launch();
        std::ofstream(dir + "/shape.txt") << sh.threads << " " << sh.blocks_x << " " << sh.grid_y << " "
                                          << sh.queries_per_block << " " << sh.vectors_per_step << "\n";
        veckern::gpu::Tuning t;
        t.queries_per_block = 8;
        t.vectors_per_step = 2;
        searcher.set_tuning(t);
        searcher.search(queries.data(), nq, k, veckern::gpu::ScanVariant::FusedWarp, out.data());
        write_all(dir + "/out_q8.bin", out);
        return 0;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 1;
    }
}
