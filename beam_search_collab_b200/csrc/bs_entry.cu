// bs_entry.cu -- search entry point on the GPU.
//
// Same rule and the same fp32 arithmetic as the reference host function
// compute_entry_point (src/gpu_cli.cu:55-83 == src/cpu_cli.cpp:35-62):
//   inv = 1/n;  centroid[d] = sum over rows i = 0..n-1 (in order) of row_i[d]*inv
//   entry = first row with the smallest sequential squared distance to it.
// The centroid sum is a sequential fold per dimension, so one thread owns
// one dimension and walks the rows in order (bs_centroid.cuh: one block per
// 32-byte slice of the rows, streamed through shared memory); the
// per-row distances are independent, one thread per row, folded over d in
// order; the argmin packs (distance, row) into one 64-bit key so that
// atomicMin keeps the smallest distance and, among equals, the first row.
// Rows are f32, or u8 when the index stores an exact byte copy (converted to
// float exactly before any arithmetic).
#include <cfloat>
#include <cstdint>

#include "bs_centroid.cuh"
#include "bs_device.cuh"
#include "bs_internal.h"

namespace bsb {
namespace {

__device__ __forceinline__ float load_elem(const float* p) { return __ldg(p); }
__device__ __forceinline__ float load_elem(const uint8_t* p) { return static_cast<float>(__ldg(p)); }

template <typename T>
__global__ void k_centroid(const T* __restrict__ vecs, uint64_t n, uint32_t dim, uint32_t row_stride,
                           float inv, float* __restrict__ centroid) {
    const uint32_t d = blockIdx.x * blockDim.x + threadIdx.x;
    if (d >= dim) return;
    float c = 0.0f;
    const T* p = vecs + d;
    uint64_t i = 0;
    for (; i + 8 <= n; i += 8) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = load_elem(p + (i + j) * row_stride);
#pragma unroll
        for (int j = 0; j < 8; ++j) c = __fadd_rn(c, __fmul_rn(v[j], inv));
    }
    for (; i < n; ++i) c = __fadd_rn(c, __fmul_rn(load_elem(p + i * row_stride), inv));
    centroid[d] = c;
}

template <typename T>
__global__ void k_nearest(const T* __restrict__ vecs, uint64_t n, uint32_t dim, uint32_t row_stride,
                          const float* __restrict__ centroid, unsigned long long* __restrict__ best) {
    extern __shared__ float c_sm[];
    for (uint32_t d = threadIdx.x; d < dim; d += blockDim.x) c_sm[d] = centroid[d];
    __syncthreads();
    unsigned long long mine = ~0ull;
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const T* row = vecs + i * row_stride;
        float s = 0.0f;
        for (uint32_t d = 0; d < dim; ++d) {
            const float t = __fsub_rn(load_elem(row + d), c_sm[d]);
            s = __fadd_rn(s, __fmul_rn(t, t));
        }
        const unsigned long long key =
            (static_cast<unsigned long long>(dev::f2ord(s)) << 32) | static_cast<unsigned long long>(i);
        mine = mine < key ? mine : key;
    }
    // warp min then one atomic per warp
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(dev::kFull, mine, o);
        mine = mine < other ? mine : other;
    }
    if ((threadIdx.x & 31) == 0) atomicMin(best, mine);
}

__global__ void k_finish(const unsigned long long* best, uint32_t* out) {
    *out = static_cast<uint32_t>(*best & 0xffffffffull);
}

template <typename T>
cudaError_t entry_impl(const T* vecs, uint64_t n, uint32_t dim, uint32_t row_stride, uint32_t* d_result,
                       float* d_scratch, cudaStream_t stream) {
    if (n == 0 || dim == 0) return cudaErrorInvalidValue;
    if (n > 0xffffffffull) return cudaErrorInvalidValue;
    unsigned long long* best = reinterpret_cast<unsigned long long*>(d_scratch);
    float* centroid = reinterpret_cast<float*>(reinterpret_cast<char*>(d_scratch) + 8);
    cudaError_t e = cudaMemsetAsync(best, 0xff, sizeof(unsigned long long), stream);
    if (e != cudaSuccess) return e;
    const float inv = 1.0f / static_cast<float>(n);
    const uint32_t row_bytes = row_stride * static_cast<uint32_t>(sizeof(T));
    if (launch_centroid_sliced<T, float, FoldF32>(vecs, n, dim, row_bytes, FoldF32{inv}, centroid, stream, e)) {
        if (e != cudaSuccess) return e;
    } else {
        k_centroid<T><<<(dim + 127) / 128, 128, 0, stream>>>(vecs, n, dim, row_stride, inv, centroid);
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const uint64_t blocks64 = (n + 255) / 256;
    const unsigned blocks = static_cast<unsigned>(blocks64 < 4096 ? blocks64 : 4096);
    k_nearest<T><<<blocks, 256, dim * sizeof(float), stream>>>(vecs, n, dim, row_stride, centroid, best);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    k_finish<<<1, 1, 0, stream>>>(best, d_result);
    return cudaGetLastError();
}

}  // namespace

size_t entry_point_scratch_bytes(uint64_t /*n*/, uint32_t dim) {
    return 8 + ((static_cast<size_t>(dim) * 4 + 7) & ~static_cast<size_t>(7));
}

cudaError_t compute_entry_point(const float* vecs, uint64_t n, uint32_t dim, uint32_t row_stride,
                                uint32_t* d_result, float* d_scratch, cudaStream_t stream) {
    return entry_impl<float>(vecs, n, dim, row_stride, d_result, d_scratch, stream);
}

cudaError_t compute_entry_point_u8(const uint8_t* vecs8, uint64_t n, uint32_t dim, uint32_t row_bytes,
                                   uint32_t* d_result, float* d_scratch, cudaStream_t stream) {
    return entry_impl<uint8_t>(vecs8, n, dim, row_bytes, d_result, d_scratch, stream);
}

}  // namespace bsb
