// Persisted PQ index file (".vkpq"): codebooks + row-major codes, readable by row range so that every shard of a
// multi-GPU search loads only its own rows. The reference has no index format (its io.cpp reads TEXMEX vectors only).
//
// Layout (little-endian):
//   [0, 128)          header
//       0  char[8]  magic "VKPQIDX1"
//       8  u32      version (1)
//      12  u32      header bytes (128)
//      16  u64      n (rows)
//      24  u32      d
//      28  u32      m
//      32  u32      dsub (d / m)
//      36  u32      centroids per sub-space (256)
//      40  u64      offset of the centroids: [m][256][dsub] fp32
//      48  u64      offset of the codes: [n][m] uint8, row-major
//      56  u64      rows per checksum block (B)
//      64  u64      offset of the block checksums: ceil(n / B) x u32, CRC-32C of each block's code bytes
//      72  u32      CRC-32C of the centroid bytes
//      76  u32      CRC-32C of header bytes [0, 76)
//      80  zero up to 128
//   centroids, codes (4096-byte aligned), block checksums.
//
// CRC-32C (Castagnoli, reflected polynomial 0x82F63B78, initial value and final xor 0xFFFFFFFF): the SSE 4.2
// crc32 instruction where the CPU has it, a byte-wise table otherwise (identical results).
#pragma once
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#if defined(__x86_64__)
#include <nmmintrin.h>
#endif

namespace vkio {

constexpr char kMagic[8] = {'V', 'K', 'P', 'Q', 'I', 'D', 'X', '1'};
constexpr uint32_t kVersion = 1;
constexpr uint32_t kHeaderBytes = 128;
constexpr uint64_t kBlockRows = 1u << 20;
constexpr uint64_t kAlign = 4096;

struct Header {
    uint64_t n = 0;
    uint32_t d = 0, m = 0, dsub = 0, ksub = 256;
    uint64_t centroids_off = 0, codes_off = 0, block_rows = kBlockRows, crc_off = 0;
    uint32_t centroids_crc = 0, header_crc = 0;
};

struct Crc32cTable {
    uint32_t t[256];
    Crc32cTable() {
        for (uint32_t i = 0; i < 256; ++i) {
            uint32_t c = i;
            for (int k = 0; k < 8; ++k) c = (c >> 1) ^ (0x82F63B78u & (0u - (c & 1u)));
            t[i] = c;
        }
    }
};

inline uint32_t crc32c_table_update(uint32_t crc, const uint8_t* p, size_t len) {
    static const Crc32cTable table;  // thread-safe one-time initialisation
    for (size_t i = 0; i < len; ++i) crc = table.t[(crc ^ p[i]) & 0xffu] ^ (crc >> 8);
    return crc;
}

#if defined(__x86_64__)
__attribute__((target("sse4.2"))) inline uint32_t crc32c_hw_update(uint32_t crc, const uint8_t* p, size_t len) {
    uint64_t c = crc;
    while (len >= 8) {
        uint64_t v;
        std::memcpy(&v, p, 8);
        c = _mm_crc32_u64(c, v);
        p += 8;
        len -= 8;
    }
    uint32_t c32 = (uint32_t)c;
    while (len--) c32 = _mm_crc32_u8(c32, *p++);
    return c32;
}
inline bool have_hw_crc() {
    static const int has = __builtin_cpu_supports("sse4.2") ? 1 : 0;
    return has != 0;
}
#endif

// CRC-32C of [p, p + len); `hw` = false forces the table path (tests compare the two).
inline uint32_t crc32c(const void* data, size_t len, bool hw = true) {
    const uint8_t* p = static_cast<const uint8_t*>(data);
#if defined(__x86_64__)
    if (hw && have_hw_crc()) return crc32c_hw_update(0xFFFFFFFFu, p, len) ^ 0xFFFFFFFFu;
#endif
    (void)hw;
    return crc32c_table_update(0xFFFFFFFFu, p, len) ^ 0xFFFFFFFFu;
}

inline void put32(uint8_t* b, size_t off, uint32_t v) { std::memcpy(b + off, &v, 4); }
inline void put64(uint8_t* b, size_t off, uint64_t v) { std::memcpy(b + off, &v, 8); }
inline uint32_t get32(const uint8_t* b, size_t off) {
    uint32_t v;
    std::memcpy(&v, b + off, 4);
    return v;
}
inline uint64_t get64(const uint8_t* b, size_t off) {
    uint64_t v;
    std::memcpy(&v, b + off, 8);
    return v;
}

inline uint64_t align_up(uint64_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

inline void encode_header(const Header& h, uint8_t* b) {
    std::memset(b, 0, kHeaderBytes);
    std::memcpy(b, kMagic, 8);
    put32(b, 8, kVersion);
    put32(b, 12, kHeaderBytes);
    put64(b, 16, h.n);
    put32(b, 24, h.d);
    put32(b, 28, h.m);
    put32(b, 32, h.dsub);
    put32(b, 36, h.ksub);
    put64(b, 40, h.centroids_off);
    put64(b, 48, h.codes_off);
    put64(b, 56, h.block_rows);
    put64(b, 64, h.crc_off);
    put32(b, 72, h.centroids_crc);
    put32(b, 76, crc32c(b, 76));
}

// Returns an empty string or what is wrong with the header.
inline std::string decode_header(const uint8_t* b, uint64_t file_bytes, Header& h) {
    if (std::memcmp(b, kMagic, 8) != 0) return "not a VecKern-B200 index file (bad magic)";
    if (get32(b, 8) != kVersion) return "unsupported index file version " + std::to_string(get32(b, 8));
    if (get32(b, 12) != kHeaderBytes) return "bad header size";
    if (get32(b, 76) != crc32c(b, 76)) return "header checksum mismatch";
    h.n = get64(b, 16);
    h.d = get32(b, 24);
    h.m = get32(b, 28);
    h.dsub = get32(b, 32);
    h.ksub = get32(b, 36);
    h.centroids_off = get64(b, 40);
    h.codes_off = get64(b, 48);
    h.block_rows = get64(b, 56);
    h.crc_off = get64(b, 64);
    h.centroids_crc = get32(b, 72);
    h.header_crc = get32(b, 76);
    // Bound every field before any arithmetic on it, so that no product or sum below can wrap: a header whose own
    // checksum is right may still have been written with nonsense values.
    if (h.m == 0 || h.m > 4096 || h.dsub == 0 || h.dsub > 4096 || h.n >= (uint64_t(1) << 31) ||
        (uint64_t)h.d != (uint64_t)h.m * h.dsub || h.ksub != 256 || h.block_rows == 0 ||
        h.block_rows > (uint64_t(1) << 31))
        return "inconsistent shape in header";
    if (h.centroids_off > file_bytes || h.codes_off > file_bytes || h.crc_off > file_bytes)
        return "file truncated or section offsets out of range";
    const uint64_t cbytes = (uint64_t)h.m * 256u * h.dsub * 4u;  // < 2^35
    const uint64_t code_bytes = h.n * h.m;                          // < 2^43
    const uint64_t blocks = (h.n + h.block_rows - 1) / h.block_rows;
    // every offset is at most file_bytes (< 2^63), every size below 2^44: the sums cannot wrap
    if (h.centroids_off < kHeaderBytes || h.centroids_off + cbytes > h.codes_off ||
        h.codes_off + code_bytes > h.crc_off || h.crc_off + blocks * 4u > file_bytes)
        return "file truncated or section offsets out of range";
    return "";
}

inline Header make_header(uint64_t n, uint32_t m, uint32_t dsub) {
    Header h;
    h.n = n;
    h.m = m;
    h.dsub = dsub;
    h.d = m * dsub;
    h.centroids_off = kHeaderBytes;
    h.codes_off = align_up(h.centroids_off + (uint64_t)m * 256u * dsub * 4u);
    h.crc_off = align_up(h.codes_off + n * m);
    return h;
}

struct File {
    FILE* f = nullptr;
    explicit File(const char* path, const char* mode) : f(std::fopen(path, mode)) {}
    ~File() {
        if (f) std::fclose(f);
    }
    bool seek(uint64_t off) { return fseeko(f, (off_t)off, SEEK_SET) == 0; }
    bool read(void* p, size_t n) { return std::fread(p, 1, n, f) == n; }
    bool write(const void* p, size_t n) { return std::fwrite(p, 1, n, f) == n; }
    uint64_t size() {
        if (fseeko(f, 0, SEEK_END) != 0) return 0;
        return (uint64_t)ftello(f);
    }
};

// Streams an index file out: header + centroids, then codes in row order through `next(rows, buf)`, which fills
// `buf` with the next `rows` rows (row-major, m bytes each) and returns false on failure.
template <class NextRows>
inline std::string write_index(const char* path, const float* centroids, uint32_t m, uint32_t dsub, uint64_t n,
                               NextRows&& next) {
    File out(path, "wb");
    if (!out.f) return std::string("cannot create ") + path;
    Header h = make_header(n, m, dsub);
    const size_t cbytes = (size_t)m * 256u * dsub * 4u;
    h.centroids_crc = crc32c(centroids, cbytes);
    uint8_t hb[kHeaderBytes];
    encode_header(h, hb);
    std::vector<uint8_t> pad(kAlign, 0);
    if (!out.write(hb, kHeaderBytes) || !out.write(centroids, cbytes)) return "write failed";
    if (!out.write(pad.data(), h.codes_off - (h.centroids_off + cbytes))) return "write failed";
    std::vector<uint32_t> crcs;
    std::vector<uint8_t> buf;
    for (uint64_t r0 = 0; r0 < n; r0 += h.block_rows) {
        const uint64_t rows = std::min<uint64_t>(h.block_rows, n - r0);
        buf.resize(rows * m);
        if (!next(rows, buf.data())) return "reading the codes to write failed";
        crcs.push_back(crc32c(buf.data(), buf.size()));
        if (!out.write(buf.data(), buf.size())) return "write failed";
    }
    if (!out.write(pad.data(), h.crc_off - (h.codes_off + n * m))) return "write failed";
    if (!crcs.empty() && !out.write(crcs.data(), crcs.size() * 4)) return "write failed";
    if (std::fflush(out.f) != 0) return "write failed";
    return "";
}

struct Reader {
    File in;
    Header h;
    std::string err;
    std::vector<uint32_t> crcs;
    explicit Reader(const char* path) : in(path, "rb") {
        if (!in.f) {
            err = std::string("cannot open ") + path;
            return;
        }
        const uint64_t bytes = in.size();
        uint8_t hb[kHeaderBytes];
        if (bytes < kHeaderBytes || !in.seek(0) || !in.read(hb, kHeaderBytes)) {
            err = "file truncated (no header)";
            return;
        }
        err = decode_header(hb, bytes, h);
        if (!err.empty()) return;
        crcs.resize((h.n + h.block_rows - 1) / h.block_rows);
        if (!crcs.empty() && (!in.seek(h.crc_off) || !in.read(crcs.data(), crcs.size() * 4))) err = "read failed";
    }
    bool ok() const { return err.empty(); }

    std::string centroids(float* out) {
        const size_t cbytes = (size_t)h.m * 256u * h.dsub * 4u;
        if (!in.seek(h.centroids_off) || !in.read(out, cbytes)) return "read failed";
        if (crc32c(out, cbytes) != h.centroids_crc) return "centroid checksum mismatch";
        return "";
    }

    // Rows [first, first + count) into `emit(row0, rows, bytes)` in pieces of at most one checksum block. With
    // `verify`, every block the range touches is read whole and checked against its stored checksum.
    template <class Emit>
    std::string rows(uint64_t first, uint64_t count, bool verify, Emit&& emit) {
        if (first > h.n || count > h.n - first) return "row range out of bounds";
        std::vector<uint8_t> buf;
        uint64_t r = first;
        const uint64_t end = first + count;
        while (r < end) {
            const uint64_t blk = r / h.block_rows;
            const uint64_t b0 = blk * h.block_rows, b1 = std::min(h.n, b0 + h.block_rows);
            const uint64_t lo = verify ? b0 : r, hi = verify ? b1 : std::min(end, b1);
            buf.resize((hi - lo) * h.m);
            if (!in.seek(h.codes_off + lo * h.m) || !in.read(buf.data(), buf.size())) return "read failed";
            if (verify && crc32c(buf.data(), buf.size()) != crcs[blk])
                return "code checksum mismatch in rows " + std::to_string(b0) + ".." + std::to_string(b1 - 1);
            const uint64_t take_hi = std::min(end, b1);
            if (!emit(r, take_hi - r, buf.data() + (r - lo) * h.m)) return "consumer failed";
            r = take_hi;
        }
        return "";
    }
};

}  // namespace vkio
