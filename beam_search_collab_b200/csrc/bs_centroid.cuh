// bs_centroid.cuh -- per-dimension sequential folds over all rows, in row
// order, for the two centroids of the path: the search entry point's float
// centroid (sum of row[d] * (1/n) in fp32, src/gpu_cli.cu:55-83) and the
// codebook medoid's double centroid (sum of row[d] in double, then / n,
// src/build_rabitq.cpp:59-70).
//
// Each dimension's fold is a chain in row order by definition, so the work
// splits by dimension: one block per 32-byte slice of the rows (8 f32 or 32
// u8 dimensions).  All of the block's threads stream the slice's rows through
// shared memory in double-buffered cp.async tiles; one thread per dimension
// folds each tile's rows in order -- the same operations in the same order as
// a single thread walking every row, so the same bits.
#pragma once

#include <cstdint>

#include "bs_device.cuh"

namespace bsb {

// c = c + x * inv, each operation rounded (entry point)
struct FoldF32 {
    float inv;
    __device__ __forceinline__ float operator()(float c, float x) const { return __fadd_rn(c, __fmul_rn(x, inv)); }
    __device__ __forceinline__ float finish(float c) const { return c; }
};

// c = c + (double)x, then c / n (medoid)
struct FoldF64 {
    double n;
    __device__ __forceinline__ double operator()(double c, float x) const {
        return __dadd_rn(c, static_cast<double>(x));
    }
    __device__ __forceinline__ double finish(double c) const { return __ddiv_rn(c, n); }
};

constexpr uint32_t kSliceBytes = 32;
constexpr uint32_t kSliceThreads = 256;

// grid = ceil(row_bytes / 32) blocks of kSliceThreads; rows row_bytes apart
// (a multiple of 16), vecs 16-byte aligned; shared memory 2 * tile_rows * 32.
template <typename T, typename Acc, typename Fold>
__global__ void __launch_bounds__(kSliceThreads)
    k_centroid_sliced(const T* __restrict__ vecs, uint64_t n, uint32_t dim, uint32_t row_bytes, uint32_t tile_rows,
                      Fold fold, Acc* __restrict__ out) {
    extern __shared__ __align__(16) unsigned char slice_tiles[];
    const uint32_t off = blockIdx.x * kSliceBytes;
    const uint32_t sb = row_bytes - off < kSliceBytes ? row_bytes - off : kSliceBytes;   // 16 or 32
    const uint32_t pieces_row = sb / 16u;
    const uint32_t tile_bytes = tile_rows * kSliceBytes;
    const unsigned char* src = reinterpret_cast<const unsigned char*>(vecs) + off;
    const uint64_t ntiles = (n + tile_rows - 1) / tile_rows;
    auto load = [&](uint64_t t) {
        if (t < ntiles) {
            const uint64_t r0 = t * tile_rows;
            const uint32_t rows = static_cast<uint32_t>(n - r0 < tile_rows ? n - r0 : tile_rows);
            unsigned char* dst = slice_tiles + (t & 1u) * tile_bytes;
            for (uint32_t i = threadIdx.x; i < rows * pieces_row; i += blockDim.x) {
                const uint32_t r = i / pieces_row, p = i - r * pieces_row;
                dev::cp_async16(dst + 16u * i, src + (r0 + r) * row_bytes + 16u * p);
            }
        }
        asm volatile("cp.async.commit_group;\n" ::: "memory");
    };
    const uint32_t per_row = sb / static_cast<uint32_t>(sizeof(T));   // elements of the slice
    const uint32_t d = off / static_cast<uint32_t>(sizeof(T)) + threadIdx.x;
    const bool mine = threadIdx.x < per_row && d < dim;
    Acc c = Acc(0);
    load(0);
    for (uint64_t t = 0; t < ntiles; ++t) {
        load(t + 1);
        asm volatile("cp.async.wait_group 1;\n" ::: "memory");
        __syncthreads();
        if (mine) {
            const uint32_t rows = static_cast<uint32_t>(n - t * tile_rows < tile_rows ? n - t * tile_rows : tile_rows);
            const T* tile = reinterpret_cast<const T*>(slice_tiles + (t & 1u) * tile_bytes);
#pragma unroll 8
            for (uint32_t r = 0; r < rows; ++r) c = fold(c, static_cast<float>(tile[r * per_row + threadIdx.x]));
        }
        __syncthreads();   // this buffer is refilled by the next iteration's load
    }
    if (mine) out[d] = fold.finish(c);
}

// Launches k_centroid_sliced; false when the rows do not meet its alignment
// (the caller then uses its plain kernel).
template <typename T, typename Acc, typename Fold>
inline bool launch_centroid_sliced(const T* vecs, uint64_t n, uint32_t dim, uint32_t row_bytes, Fold fold, Acc* out,
                                   cudaStream_t stream, cudaError_t& err) {
    if (row_bytes % 16u != 0 || (reinterpret_cast<uintptr_t>(vecs) & 15u) != 0 || n == 0) return false;
    const uint64_t want = (48u * 1024u) / kSliceBytes;
    const uint32_t tile_rows = static_cast<uint32_t>(want < n ? want : n);
    const size_t smem = 2ull * tile_rows * kSliceBytes;
    err = cudaFuncSetAttribute(k_centroid_sliced<T, Acc, Fold>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(smem));
    if (err != cudaSuccess) return true;
    const unsigned grid = (row_bytes + kSliceBytes - 1) / kSliceBytes;
    k_centroid_sliced<T, Acc, Fold><<<grid, kSliceThreads, smem, stream>>>(vecs, n, dim, row_bytes, tile_rows, fold,
                                                                            out);
    err = cudaGetLastError();
    return true;
}

}  // namespace bsb
