// bs_load.cu -- the device side of the file loaders: the reference's files
// are streamed to the GPU as they lie on disk (memory-mapped, copied through
// page-locked staging buffers with asynchronous copies, so the next chunk is
// read from disk while the GPU takes apart the previous one) and taken apart
// on the GPU:
//
//   base .fvecs   rows [int32 d | d x f32]  -> [n][row_stride] f32 rows, the
//                 header of every row checked, the values scanned (all
//                 integers? range? positions of -0.0) for the byte copy
//                 (include/data_loader.hpp:9-26)
//   codebook.bin  rows [raw vector | codes | factors | neighbour ids] ->
//                 codes [n][deg][wpp] and factors [n][3][deg]
//                 (include/rabitq.hpp:49-97)
//
// graph.bin's payload is already the device layout; it is copied as it is.
#include <cfloat>
#include <cmath>
#include <cstdint>

#include "bs_internal.h"

namespace bsb {

namespace {

__device__ __forceinline__ uint32_t ford(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void k_fvecs_rows(const uint32_t* __restrict__ raw, uint64_t rows, uint64_t first_row, uint32_t dim,
                             uint32_t row_stride, float* __restrict__ out, LoadScan* scan) {
    const uint64_t in_stride = static_cast<uint64_t>(dim) + 1;
    const uint64_t total = rows * row_stride;
    bool all_int = true, bad = false;
    uint32_t lo = 0xffffffffu, hi = 0u;
    for (uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
         t += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t r = t / row_stride;
        const uint32_t d = static_cast<uint32_t>(t - r * row_stride);
        const uint32_t* row = raw + r * in_stride;
        if (d == 0 && row[0] != dim) bad = true;
        float v = 0.0f;
        if (d < dim) {
            v = __uint_as_float(row[1 + d]);
            all_int = all_int && (v == rintf(v));
            if (v == v) {
                const uint32_t o = ford(v == 0.0f ? 0.0f : v);
                lo = o < lo ? o : lo;
                hi = o > hi ? o : hi;
            }
            if (__float_as_uint(v) == 0x80000000u) {
                const unsigned long long at = atomicAdd(&scan->neg_zero_count, 1ull);
                if (at < scan->neg_zero_cap) scan->neg_zero_pos[at] = (first_row + r) * dim + d;
            }
        }
        out[(first_row + r) * row_stride + d] = v;
    }
    if (bad) atomicOr(&scan->bad_rows, 1u);
    if (!all_int) atomicAnd(&scan->all_int, 0u);
    if (lo != 0xffffffffu) atomicMin(&scan->min_ord, lo);
    if (hi != 0u) atomicMax(&scan->max_ord, hi);
}

__global__ void k_rows_to_u8(const float* __restrict__ in, uint64_t n, uint32_t dim, uint32_t row_stride,
                             uint32_t row_bytes, uint8_t* __restrict__ out) {
    const uint64_t total = n * row_bytes;
    for (uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
         t += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t r = t / row_bytes;
        const uint32_t d = static_cast<uint32_t>(t - r * row_bytes);
        out[t] = d < dim ? static_cast<uint8_t>(in[r * row_stride + d]) : 0u;
    }
}

__global__ void k_codebook_rows(const uint32_t* __restrict__ raw, uint64_t rows, uint64_t first_row, uint32_t dim,
                                uint32_t deg, uint32_t wpp, uint32_t* __restrict__ codes, float* __restrict__ factors) {
    const uint64_t in_row = static_cast<uint64_t>(dim) + static_cast<uint64_t>(wpp) * deg + 4ull * deg;
    const uint64_t cw = static_cast<uint64_t>(deg) * wpp, fw = 3ull * deg;
    const uint64_t total = rows * (cw + fw);
    for (uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
         t += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t r = t / (cw + fw);
        const uint64_t j = t - r * (cw + fw);
        const uint32_t* row = raw + r * in_row;
        if (j < cw) codes[(first_row + r) * cw + j] = row[dim + j];
        else factors[(first_row + r) * fw + (j - cw)] = __uint_as_float(row[dim + cw + (j - cw)]);
    }
}

unsigned grid_for(uint64_t items) {
    const uint64_t b = (items + 255) / 256;
    return static_cast<unsigned>(b < 65535ull * 16 ? (b ? b : 1) : 65535ull * 16);
}

}  // namespace

cudaError_t load_fvecs_chunk(const uint32_t* raw, uint64_t rows, uint64_t first_row, uint32_t dim, uint32_t row_stride,
                             float* out, LoadScan* scan, cudaStream_t stream) {
    k_fvecs_rows<<<grid_for(rows * row_stride), 256, 0, stream>>>(raw, rows, first_row, dim, row_stride, out, scan);
    return cudaGetLastError();
}

cudaError_t rows_to_u8(const float* in, uint64_t n, uint32_t dim, uint32_t row_stride, uint32_t row_bytes, uint8_t* out,
                       cudaStream_t stream) {
    k_rows_to_u8<<<grid_for(n * row_bytes), 256, 0, stream>>>(in, n, dim, row_stride, row_bytes, out);
    return cudaGetLastError();
}

cudaError_t load_codebook_chunk(const uint32_t* raw, uint64_t rows, uint64_t first_row, uint32_t dim, uint32_t deg,
                                uint32_t wpp, uint32_t* codes, float* factors, cudaStream_t stream) {
    const uint64_t items = rows * (static_cast<uint64_t>(deg) * wpp + 3ull * deg);
    k_codebook_rows<<<grid_for(items), 256, 0, stream>>>(raw, rows, first_row, dim, deg, wpp, codes, factors);
    return cudaGetLastError();
}

}  // namespace bsb
