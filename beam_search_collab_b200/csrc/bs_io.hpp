// bs_io.hpp -- readers for the reference's file formats (host, C++17).
//
//   graph.bin  int32 n, int32 degree, uint32[n*degree]      (include/cpu_graph.hpp:125-144)
//   *.fvecs    per row: int32 d, d x float32                   (include/data_loader.hpp:9-26)
//   *.ivecs    per row: int32 d, d x int32                     (include/data_loader.hpp:28-45)
//   codebook   uint32 entry, n rows of (dim + wpp*deg + 3*deg + deg) 4-byte
//              slots [raw vector | codes | factors | neighbour ids], then
//              float32 signs[padded_dim]                        (include/rabitq.hpp:49-97)
//
// The byte layouts are those of the reference; unlike the reference readers
// these validate sizes and report errors instead of reading past the end.
#pragma once

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

namespace bsb {
namespace io {

struct FileCloser {
    void operator()(std::FILE* f) const {
        if (f) std::fclose(f);
    }
};

inline bool file_size(std::FILE* f, uint64_t& size) {
    if (std::fseek(f, 0, SEEK_END) != 0) return false;
    const long s = std::ftell(f);
    if (s < 0) return false;
    size = static_cast<uint64_t>(s);
    return std::fseek(f, 0, SEEK_SET) == 0;
}

inline bool read_graph(const std::string& path, uint64_t& n, int32_t& degree,
                       std::vector<uint32_t>& edges, std::string& err) {
    std::FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) { err = "Cannot open graph file: " + path; return false; }
    FileCloser close;
    uint64_t size = 0;
    int32_t hdr[2] = {0, 0};
    if (!file_size(f, size) || std::fread(hdr, sizeof(int32_t), 2, f) != 2) {
        close(f); err = "Cannot read graph header: " + path; return false;
    }
    if (hdr[0] < 0 || hdr[1] <= 0) { close(f); err = "Invalid graph header in: " + path; return false; }
    n = static_cast<uint64_t>(hdr[0]);
    degree = hdr[1];
    const uint64_t count = n * static_cast<uint64_t>(degree);
    if (size < 8 + count * 4) { close(f); err = "Truncated graph file: " + path; return false; }
    edges.resize(count);
    if (count && std::fread(edges.data(), sizeof(uint32_t), count, f) != count) {
        close(f); err = "Short read in graph file: " + path; return false;
    }
    close(f);
    return true;
}

// Reads rows of [int32 d][d x 4-byte payload]; T is float or int32_t.
template <typename T>
inline bool read_vecs(const std::string& path, uint64_t& n, int32_t& d, std::vector<T>& out,
                      std::string& err) {
    std::FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) { err = "Cannot open " + path; return false; }
    FileCloser close;
    uint64_t size = 0;
    int32_t dim = 0;
    if (!file_size(f, size)) { close(f); err = "Cannot stat " + path; return false; }
    if (size == 0) { close(f); n = 0; d = 0; out.clear(); return true; }
    if (std::fread(&dim, sizeof(int32_t), 1, f) != 1 || dim <= 0) {
        close(f); err = "Invalid vecs header in: " + path; return false;
    }
    const uint64_t stride = 4ull * (static_cast<uint64_t>(dim) + 1);
    if (size % stride != 0) { close(f); err = "Corrupt vecs file (size not a multiple of the row): " + path; return false; }
    n = size / stride;
    d = dim;
    out.resize(n * static_cast<uint64_t>(dim));
    std::fseek(f, 0, SEEK_SET);
    std::vector<int32_t> row(static_cast<size_t>(dim) + 1);
    for (uint64_t i = 0; i < n; ++i) {
        if (std::fread(row.data(), 4, row.size(), f) != row.size()) {
            close(f); err = "Short read in: " + path; return false;
        }
        if (row[0] != dim) { close(f); err = "Inconsistent row dimension in: " + path; return false; }
        std::memcpy(out.data() + i * static_cast<uint64_t>(dim), row.data() + 1, 4ull * dim);
    }
    close(f);
    return true;
}

inline int32_t padded_dim_of(int32_t dim) {
    int32_t p = 1;
    while (p < dim) p <<= 1;
    return p;
}

struct Codebook {
    uint32_t entry = 0xffffffffu;
    int32_t padded_dim = 0;
    std::vector<uint32_t> codes;    // [n][degree][wpp]
    std::vector<float> factors;     // [n][3][degree]
    std::vector<float> signs;       // [padded_dim]
};

inline bool read_codebook(const std::string& path, uint64_t n, int32_t dim, int32_t degree,
                          Codebook& cb, std::string& err) {
    std::FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) { err = "Cannot open codebook: " + path; return false; }
    FileCloser close;
    const int32_t pdim = padded_dim_of(dim);
    const uint64_t wpp = static_cast<uint64_t>(pdim) / 32;
    const uint64_t deg = static_cast<uint64_t>(degree);
    const uint64_t code_off = static_cast<uint64_t>(dim);
    const uint64_t factor_off = code_off + wpp * deg;
    const uint64_t row = factor_off + 4 * deg;
    uint64_t size = 0;
    if (!file_size(f, size)) { close(f); err = "Cannot stat codebook: " + path; return false; }
    const uint64_t need = 4 + n * row * 4 + static_cast<uint64_t>(pdim) * 4;
    if (size < need) { close(f); err = "Truncated codebook (or dim/degree mismatch): " + path; return false; }
    if (std::fread(&cb.entry, 4, 1, f) != 1) { close(f); err = "Cannot read codebook header: " + path; return false; }
    cb.padded_dim = pdim;
    cb.codes.resize(n * deg * wpp);
    cb.factors.resize(n * 3 * deg);
    cb.signs.resize(static_cast<size_t>(pdim));
    std::vector<uint32_t> buf(row);
    for (uint64_t i = 0; i < n; ++i) {
        if (std::fread(buf.data(), 4, row, f) != row) { close(f); err = "Short read in codebook: " + path; return false; }
        std::memcpy(cb.codes.data() + i * deg * wpp, buf.data() + code_off, 4 * deg * wpp);
        std::memcpy(cb.factors.data() + i * 3 * deg, buf.data() + factor_off, 4 * 3 * deg);
    }
    if (std::fread(cb.signs.data(), 4, static_cast<size_t>(pdim), f) != static_cast<size_t>(pdim)) {
        close(f); err = "Short read of codebook signs: " + path; return false;
    }
    close(f);
    return true;
}

}  // namespace io
}  // namespace bsb
