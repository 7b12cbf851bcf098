/*
 * VecKern-B200 host library (libveckern_b200_host.so): the input side of the search path, on the CPU.
 *
 *  - Product quantizer training / encoding / decoding on raw arrays: the algorithm of the reference's
 *    ProductQuantizer (src/cpu/pq.cpp:31-81): per sub-space, 256 rows picked by std::shuffle with
 *    std::mt19937_64(seed), then `iters` Lloyd iterations; encode = first nearest centroid under l2sq.
 *    The C++ class veckern::ProductQuantizer (include/veckern/pq.hpp) is implemented in the same library.
 *  - synthetic_clustered: the reference's Gaussian-blob generator used by its test fixtures (src/cpu/io.cpp:54-69).
 *  - Generators of the benchmark configurations (counter-based, any row range independently):
 *    i.i.d. N(0,1) rows, the 1,000-component integer mixture, Dirichlet(alpha) categorical tables and the
 *    cluster/categorical code generator shared with the device (vk_index_create_generated).
 * All functions return 0 on success and a negative value on bad arguments.
 */
#ifndef VK_HOST_H
#define VK_HOST_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

int vk_host_pq_train(const float* x, int64_t n, int d, int m, int64_t iters, uint64_t seed, float* centroids);
int vk_host_pq_encode(const float* centroids, int d, int m, const float* x, int64_t n, uint8_t* codes);
int vk_host_pq_decode(const float* centroids, int d, int m, const uint8_t* codes, int64_t n, float* x);

/* 4-bit PQ (no counterpart in the reference, which lists 4-bit codes as a next step, README.md:219): the same
 * trainer with 16 centroids per sub-space (n >= 16; centroids [m][16][dsub]), and the encoder that packs the first
 * nearest of the 16 centroids of sub-space s into nibble s % 2 (low first) of byte s / 2 (n x ceil(m / 2) bytes). */
int vk_host_pq4_train(const float* x, int64_t n, int d, int m, int64_t iters, uint64_t seed, float* centroids);
int vk_host_pq4_encode(const float* centroids, int d, int m, const float* x, int64_t n, uint8_t* codes);

int vk_host_synthetic_clustered(int64_t n, int d, int64_t clusters, uint64_t seed, float* out);

/* rows [row0, row0 + rows) of d i.i.d. N(0,1) values (Box-Muller on two 53-bit uniforms per value) */
int vk_host_gen_normal(uint64_t seed, int64_t row0, int64_t rows, int d, float* out);

/* rows [row0, row0 + rows) of the integer Gaussian mixture: `ncomp` component means uniform on [0, 64]^d drawn
 * from mix_seed; each row picks a component and adds N(0, sigma^2) noise from sample_seed; values are rounded
 * (ties to even) and clipped to [0, 255]. */
int vk_host_gen_mixture(uint64_t mix_seed, int ncomp, float sigma, uint64_t sample_seed, int64_t row0, int64_t rows,
                        int d, float* out);

/* [clusters][m][256] uint32 categorical tables: weights ~ Dirichlet(alpha) per (cluster, sub-space), stored as
 * cumulative thresholds floor(2^32 * sum_{j<=c} w_j) (entry 255 = 2^32 - 1). */
int vk_host_gen_cdf(uint64_t seed, int clusters, int m, double alpha, uint32_t* cdf);

/* rows [row0, row0 + n) of the generated code database (row-major n x m) */
int vk_host_gen_codes(uint64_t seed, const uint32_t* cdf, int clusters, int m, int64_t row0, int64_t n,
                      uint8_t* codes);

/* the listed rows (count of them, any order) of the generated code database (row-major count x m) */
int vk_host_gen_codes_rows(uint64_t seed, const uint32_t* cdf, int clusters, int m, const int64_t* rows,
                           int64_t count, uint8_t* codes);

/* ---- persisted index files (no counterpart in the reference, whose io.cpp only reads TEXMEX vectors) ----
 * Format: 128-byte header ("VKPQIDX1", n, d, m, dsub, section offsets, CRC-32C of header and centroids), the
 * centroids [m][256][dsub] fp32, the codes [n][m] uint8 row-major (4096-byte aligned), and one CRC-32C per block of
 * 2^20 rows. Return 0, -1 for bad arguments, -2 for I/O or format errors (vk_host_last_error has the message). */
int vk_host_last_error(char* buf, size_t len);

/* CRC-32C (Castagnoli) of len bytes; hardware = 0 forces the portable table path. */
uint32_t vk_host_crc32c(const void* data, size_t len, int hardware);

/* Writes centroids [m][256][dsub] and codes [n][m] to `path`. */
int vk_host_index_write(const char* path, const float* centroids, int m, int dsub, const uint8_t* codes, int64_t n);

/* Shape of the index in `path`; any pointer may be NULL. */
int vk_host_index_info(const char* path, int64_t* n, int* d, int* m, int* dsub);

/* Reads the centroids (if `centroids` is not NULL) and the codes of rows [first, first + count) of `path`. With
 * verify != 0 every checksum block the range touches is read whole and checked. */
int vk_host_index_read(const char* path, float* centroids, int64_t first, int64_t count, uint8_t* codes, int verify);

#ifdef __cplusplus
}
#endif
#endif
