// bs_codebook.cu -- RaBitQ codebook builder on the GPU.
//
// Same rule and the same arithmetic as the reference builder
// (src/build_rabitq.cpp), over the index's device-resident rows and graph:
//   * medoid (find_medoid, :59-99): centroid[d] = (sum over rows in order of
//     row[d] in double) / n; entry = first row with the smallest double
//     sequential squared distance to it;
//   * per edge (u, v) (:170-258): rotate both rows (sign flip, then the
//     Walsh-Hadamard butterfly network of wht_inplace, :19-30), residual =
//     v_rot - u_rot over the first dim components, sqr_r / fac_x0 / fac_x1 as
//     sequential fp32 folds, one code bit per component (residual > 0), and
//     the two long-double factors at x87 precision (bs_x87.hpp).
// Every fp32 operation is a separately rounded intrinsic (no contraction), in
// the reference's order, so the codes and factors are bit-identical to the
// reference's output.
//
// Layout: one warp per node.  The warp rotates the node's row into shared
// memory, then up to 32 neighbour rows (k_quantize_edges_reg: each row's
// butterfly network in registers across the lanes; k_quantize_edges, for
// padded_dim above 1024: each lane runs the network of its own row in shared
// memory), rows at an odd pitch so that the lanes hit distinct banks, and each
// lane folds one edge.
#include <cfloat>
#include <cstdint>

#include "bs_centroid.cuh"
#include "bs_device.cuh"
#include "bs_internal.h"
#include "bs_x87.hpp"

namespace bsb {
namespace {

__device__ __forceinline__ float elem(const float* p) { return __ldg(p); }
__device__ __forceinline__ float elem(const uint8_t* p) { return static_cast<float>(__ldg(p)); }

// In-place butterfly network over the n (power of two) floats x[0..n): stage
// len = 1, 2, ..., n/2 maps (a, b) at (i + j, i + j + len) to (a + b, a - b)
// -- wht_inplace of the reference, one thread.
__device__ __forceinline__ void wht_seq(float* x, uint32_t n) {
    for (uint32_t len = 1; len < n; len <<= 1)
        for (uint32_t i = 0; i < n; i += len << 1)
            for (uint32_t j = 0; j < len; ++j) {
                const float a = x[i + j], b = x[i + j + len];
                x[i + j] = __fadd_rn(a, b);
                x[i + j + len] = __fsub_rn(a, b);
            }
}

// The same network over one row by the whole warp: the pairs of a stage are
// disjoint, so any schedule of them gives the same bits.
__device__ __forceinline__ void wht_warp(float* x, uint32_t n, unsigned lane) {
    for (uint32_t len = 1; len < n; len <<= 1) {
        for (uint32_t t = lane; t < n / 2u; t += 32u) {
            const uint32_t i = (t / len) * (len << 1) + (t % len);
            const float a = x[i], b = x[i + len];
            x[i] = __fadd_rn(a, b);
            x[i + len] = __fsub_rn(a, b);
        }
        __syncwarp();
    }
}

template <typename T>
__global__ void __launch_bounds__(128) k_quantize_edges(CodebookArgs a, const T* __restrict__ vecs) {
    extern __shared__ __align__(16) float cb_smem[];
    const unsigned lane = threadIdx.x & 31u;
    const uint32_t pdim = a.pdim, dim = a.dim, deg = a.degree, wpp = pdim / 32u;
    const uint32_t pitch = pdim + 1u;
    float* urot = cb_smem + static_cast<size_t>(threadIdx.x >> 5) * a.smem_floats_per_warp;
    float* rows = urot + pdim;
    const uint64_t warp = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = (static_cast<uint64_t>(gridDim.x) * blockDim.x) >> 5;
    const float fac_norm = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(dim)));

    for (uint64_t u = warp; u < a.n; u += nwarps) {
        const T* urow = vecs + u * a.row_stride;
        for (uint32_t d = lane; d < pdim; d += 32u)
            urot[d] = d < dim ? __fmul_rn(elem(urow + d), a.signs[d]) : 0.0f;
        __syncwarp();
        wht_warp(urot, pdim, lane);

        for (uint32_t b0 = 0; b0 < deg; b0 += a.batch_rows) {
            const uint32_t nb = deg - b0 < a.batch_rows ? deg - b0 : a.batch_rows;
            // rotate-in: row r of the batch = signs * neighbour (zeros past dim)
            for (uint32_t r = 0; r < nb; ++r) {
                const uint32_t v = a.adj[u * deg + b0 + r];
                if (v >= a.n) continue;
                const T* vrow = vecs + static_cast<uint64_t>(v) * a.row_stride;
                float* dst = rows + r * pitch;
                for (uint32_t d = lane; d < pdim; d += 32u)
                    dst[d] = d < dim ? __fmul_rn(elem(vrow + d), a.signs[d]) : 0.0f;
            }
            __syncwarp();
            if (lane < nb) {
                const uint32_t i = b0 + lane;
                const uint32_t v = a.adj[u * deg + i];
                uint32_t* codes = a.codes + (u * deg + i) * wpp;
                float* fac = a.factors + u * 3u * deg;
                if (v >= a.n) {
                    // no neighbour (UINT32_MAX in graph.bin; ids past the
                    // graph are treated the same): empty code, triple_x = FLT_MAX
                    for (uint32_t w = 0; w < wpp; ++w) codes[w] = 0u;
                    fac[i] = FLT_MAX;
                    fac[deg + i] = 0.0f;
                    fac[2u * deg + i] = 0.0f;
                } else {
                    float* x = rows + lane * pitch;
                    // own row, own butterfly network: the pitch pdim + 1
                    // puts the 32 lanes' elements in 32 different banks
                    wht_seq(x, pdim);
                    float sqr_r = 0.0f;
                    for (uint32_t d = 0; d < dim; ++d) {
                        const float res = __fsub_rn(x[d], urot[d]);
                        sqr_r = __fadd_rn(sqr_r, __fmul_rn(res, res));
                    }
                    const float r_norm = __fadd_rn(__fsqrt_rn(sqr_r), 1e-10f);
                    float fac_x0 = 0.0f, fac_x1 = 0.0f;
                    int bin_sum = 0;
                    for (uint32_t w = 0; w < wpp; ++w) {
                        uint32_t word = 0;
                        const uint32_t dend = (w + 1u) * 32u < dim ? (w + 1u) * 32u : dim;
                        for (uint32_t d = w * 32u; d < dend; ++d) {
                            const float res = __fsub_rn(x[d], urot[d]);
                            const bool pos = res > 0.0f;
                            word |= (pos ? 1u : 0u) << (d & 31u);
                            const float sv = pos ? 1.0f : -1.0f;
                            fac_x0 = __fadd_rn(fac_x0, __fmul_rn(__fmul_rn(res, sv), fac_norm));
                            fac_x1 = __fadd_rn(fac_x1, __fmul_rn(urot[d], sv));
                        }
                        bin_sum += __popc(word);
                        codes[w] = word;
                    }
                    fac_x0 = __fdiv_rn(fac_x0, r_norm);
                    fac_x1 = __fmul_rn(fac_x1, fac_norm);
                    float triple, dq;
                    x87::edge_factors(r_norm, fac_x0, fac_x1, fac_norm, triple, dq);
                    fac[i] = triple;
                    fac[deg + i] = dq;
                    fac[2u * deg + i] = __fmul_rn(dq, static_cast<float>(2 * bin_sum - static_cast<int>(dim)));
                }
            }
            __syncwarp();   // the batch rows are rewritten next
        }
    }
}

// The network over one row of pdim = 32 * EPL components held in registers,
// component lane + 32 k in x[k]: stages len = 1..16 pair lane with lane ^ len
// (shuffles), stages len = 32, 64, ... pair x[k] with x[k | len / 32] in the
// lane.  Stages run in the network's order and each element gets the same
// operation as in wht_inplace (the lower one a + b, the upper one a - b), so
// the bits are the same.
template <int EPL>
__device__ __forceinline__ void wht_lanes(float (&x)[EPL], unsigned lane) {
#pragma unroll
    for (int len = 1; len < 32; len <<= 1) {
        const bool upper = (lane & static_cast<unsigned>(len)) != 0u;
#pragma unroll
        for (int k = 0; k < EPL; ++k) {
            const float p = __shfl_xor_sync(dev::kFull, x[k], len);
            x[k] = upper ? __fsub_rn(p, x[k]) : __fadd_rn(x[k], p);
        }
    }
#pragma unroll
    for (int m = 1; m < EPL; m <<= 1)
#pragma unroll
        for (int k = 0; k < EPL; ++k)
            if (!(k & m)) {
                const float a = x[k], b = x[k | m];
                x[k] = __fadd_rn(a, b);
                x[k | m] = __fsub_rn(a, b);
            }
}

// signs * row (components past dim are +0.0, as the reference's rotate_vector)
template <typename T, int EPL>
__device__ __forceinline__ void load_rotated(const T* row, uint32_t dim, const float (&sg)[EPL], unsigned lane,
                                             float (&x)[EPL]) {
#pragma unroll
    for (int k = 0; k < EPL; ++k) {
        const uint32_t d = lane + 32u * static_cast<uint32_t>(k);
        x[k] = d < dim ? __fmul_rn(elem(row + d), sg[k]) : 0.0f;
    }
}

// k_quantize_edges with the butterfly networks in registers (pdim <= 1024,
// 32 rows per batch): the warp rotates two neighbour rows at a time and
// stores them at the odd pitch; each lane then folds its edge in one pass
// (sqr_r, the code bits, fac_x0 and fac_x1 are independent sequential folds).
template <typename T, int EPL>
__global__ void __launch_bounds__(128) k_quantize_edges_reg(CodebookArgs a, const T* __restrict__ vecs) {
    extern __shared__ __align__(16) float cb_smem[];
    constexpr uint32_t pdim = 32u * EPL, wpp = EPL, pitch = pdim + 1u;
    const unsigned lane = threadIdx.x & 31u;
    const uint32_t dim = a.dim, deg = a.degree;
    float* urot = cb_smem + static_cast<size_t>(threadIdx.x >> 5) * a.smem_floats_per_warp;
    float* rows = urot + pdim;
    const uint64_t warp = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = (static_cast<uint64_t>(gridDim.x) * blockDim.x) >> 5;
    const float fac_norm = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(dim)));
    float sg[EPL];
#pragma unroll
    for (int k = 0; k < EPL; ++k) sg[k] = a.signs[lane + 32u * k];

    for (uint64_t u = warp; u < a.n; u += nwarps) {
        {
            float x[EPL];
            load_rotated<T, EPL>(vecs + u * a.row_stride, dim, sg, lane, x);
            wht_lanes<EPL>(x, lane);
#pragma unroll
            for (int k = 0; k < EPL; ++k) urot[lane + 32u * k] = x[k];
        }
        const uint32_t* arow = a.adj + u * deg;
        for (uint32_t b0 = 0; b0 < deg; b0 += 32u) {
            const uint32_t nb = deg - b0 < 32u ? deg - b0 : 32u;
            const uint32_t myv = lane < nb ? arow[b0 + lane] : 0xffffffffu;
            for (uint32_t r = 0; r < nb; r += 2) {
                const uint32_t v0 = __shfl_sync(dev::kFull, myv, static_cast<int>(r));
                const uint32_t v1 = __shfl_sync(dev::kFull, myv, static_cast<int>((r + 1u) & 31u));
                const bool has1 = r + 1u < nb;
                float x0[EPL], x1[EPL];
                if (v0 < a.n) load_rotated<T, EPL>(vecs + static_cast<uint64_t>(v0) * a.row_stride, dim, sg, lane, x0);
                if (has1 && v1 < a.n)
                    load_rotated<T, EPL>(vecs + static_cast<uint64_t>(v1) * a.row_stride, dim, sg, lane, x1);
                if (v0 < a.n) {
                    wht_lanes<EPL>(x0, lane);
#pragma unroll
                    for (int k = 0; k < EPL; ++k) rows[r * pitch + lane + 32u * k] = x0[k];
                }
                if (has1 && v1 < a.n) {
                    wht_lanes<EPL>(x1, lane);
#pragma unroll
                    for (int k = 0; k < EPL; ++k) rows[(r + 1u) * pitch + lane + 32u * k] = x1[k];
                }
            }
            __syncwarp();
            if (lane < nb) {
                const uint32_t i = b0 + lane;
                uint32_t* codes = a.codes + (u * deg + i) * wpp;
                float* fac = a.factors + u * 3u * deg;
                if (myv >= a.n) {
                    for (uint32_t w = 0; w < wpp; ++w) codes[w] = 0u;
                    fac[i] = FLT_MAX;
                    fac[deg + i] = 0.0f;
                    fac[2u * deg + i] = 0.0f;
                } else {
                    const float* x = rows + lane * pitch;
                    float sqr_r = 0.0f, fac_x0 = 0.0f, fac_x1 = 0.0f;
                    int bin_sum = 0;
                    for (uint32_t w = 0; w < wpp; ++w) {
                        uint32_t word = 0;
                        const uint32_t dend = (w + 1u) * 32u < dim ? (w + 1u) * 32u : dim;
#pragma unroll 4
                        for (uint32_t d = w * 32u; d < dend; ++d) {
                            const float ud = urot[d];
                            const float res = __fsub_rn(x[d], ud);
                            sqr_r = __fadd_rn(sqr_r, __fmul_rn(res, res));
                            const bool pos = res > 0.0f;
                            word |= (pos ? 1u : 0u) << (d & 31u);
                            const float sv = pos ? 1.0f : -1.0f;
                            fac_x0 = __fadd_rn(fac_x0, __fmul_rn(__fmul_rn(res, sv), fac_norm));
                            fac_x1 = __fadd_rn(fac_x1, __fmul_rn(ud, sv));
                        }
                        bin_sum += __popc(word);
                        codes[w] = word;
                    }
                    const float r_norm = __fadd_rn(__fsqrt_rn(sqr_r), 1e-10f);
                    fac_x0 = __fdiv_rn(fac_x0, r_norm);
                    fac_x1 = __fmul_rn(fac_x1, fac_norm);
                    float triple, dq;
                    x87::edge_factors(r_norm, fac_x0, fac_x1, fac_norm, triple, dq);
                    fac[i] = triple;
                    fac[deg + i] = dq;
                    fac[2u * deg + i] = __fmul_rn(dq, static_cast<float>(2 * bin_sum - static_cast<int>(dim)));
                }
            }
            __syncwarp();   // the batch rows are rewritten next
        }
    }
}

// --- medoid -----------------------------------------------------------------

__device__ __forceinline__ bool medoid_less(double a, uint32_t ia, double b, uint32_t ib) {
    return a < b || (a == b && ia < ib);
}

// per-block (distance, first row) of the smallest double sequential distance
template <typename T>
__global__ void __launch_bounds__(256) k_medoid_nearest(const T* __restrict__ vecs, uint64_t n, uint32_t dim,
                                                        uint32_t row_stride, const double* __restrict__ centroid,
                                                        double* __restrict__ bdist, uint32_t* __restrict__ bidx) {
    extern __shared__ double c_sm[];
    __shared__ double wd[8];
    __shared__ uint32_t wi[8];
    for (uint32_t d = threadIdx.x; d < dim; d += blockDim.x) c_sm[d] = centroid[d];
    __syncthreads();
    double best = DBL_MAX;
    uint32_t bi = 0xffffffffu;
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const T* row = vecs + i * row_stride;
        double s = 0.0;
        for (uint32_t d = 0; d < dim; ++d) {
            const double t = __dsub_rn(static_cast<double>(elem(row + d)), c_sm[d]);
            s = __dadd_rn(s, __dmul_rn(t, t));
        }
        if (medoid_less(s, static_cast<uint32_t>(i), best, bi)) {
            best = s;
            bi = static_cast<uint32_t>(i);
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const double od = __shfl_xor_sync(dev::kFull, best, o);
        const uint32_t oi = __shfl_xor_sync(dev::kFull, bi, o);
        if (medoid_less(od, oi, best, bi)) {
            best = od;
            bi = oi;
        }
    }
    const unsigned w = threadIdx.x >> 5;
    if ((threadIdx.x & 31u) == 0) {
        wd[w] = best;
        wi[w] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (unsigned k = 1; k < blockDim.x / 32u; ++k)
            if (medoid_less(wd[k], wi[k], best, bi)) {
                best = wd[k];
                bi = wi[k];
            }
        bdist[blockIdx.x] = best;
        bidx[blockIdx.x] = bi;
    }
}

__global__ void k_medoid_finish(const double* bdist, const uint32_t* bidx, uint32_t blocks, uint32_t* out) {
    double best = DBL_MAX;
    uint32_t bi = 0xffffffffu;
    for (uint32_t k = 0; k < blocks; ++k)
        if (medoid_less(bdist[k], bidx[k], best, bi)) {
            best = bdist[k];
            bi = bidx[k];
        }
    // no row below DBL_MAX (all distances NaN or huge): row 0, as the reference
    *out = bi == 0xffffffffu ? 0u : bi;
}

// --- codebook.bin rows --------------------------------------------------------

// Rows [first, first + count) in the reference file layout
// (src/build_rabitq.cpp:152-159): raw vector (dim f32), codes (wpp * deg u32),
// factors (3 * deg f32), neighbour ids (deg u32), 4-byte slots.
template <typename T>
__global__ void k_pack_rows(CodebookArgs a, const T* __restrict__ vecs, uint64_t first, uint64_t count,
                            uint32_t* __restrict__ out) {
    const unsigned lane = threadIdx.x & 31u;
    const uint64_t warp = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = (static_cast<uint64_t>(gridDim.x) * blockDim.x) >> 5;
    const uint32_t deg = a.degree, wpp = a.pdim / 32u;
    const uint64_t row_slots = static_cast<uint64_t>(a.dim) + wpp * deg + 4ull * deg;
    for (uint64_t k = warp; k < count; k += nwarps) {
        const uint64_t u = first + k;
        uint32_t* row = out + k * row_slots;
        const T* src = vecs + u * a.row_stride;
        for (uint32_t d = lane; d < a.dim; d += 32u) row[d] = __float_as_uint(elem(src + d));
        uint32_t* c = row + a.dim;
        const uint32_t* cs = a.codes + u * deg * wpp;
        for (uint32_t w = lane; w < wpp * deg; w += 32u) c[w] = cs[w];
        uint32_t* f = c + wpp * deg;
        const float* fs = a.factors + u * 3u * deg;
        for (uint32_t w = lane; w < 3u * deg; w += 32u) f[w] = __float_as_uint(fs[w]);
        uint32_t* ids = f + 3u * deg;
        for (uint32_t w = lane; w < deg; w += 32u) ids[w] = a.adj[u * deg + w];
    }
}

template <typename T>
cudaError_t medoid_impl(const T* vecs, uint64_t n, uint32_t dim, uint32_t row_stride, uint32_t* d_result,
                        void* d_scratch, cudaStream_t stream) {
    double* centroid = reinterpret_cast<double*>(d_scratch);
    const uint32_t blocks = kMedoidBlocks;
    double* bdist = centroid + ((dim + 1u) & ~1u);
    uint32_t* bidx = reinterpret_cast<uint32_t*>(bdist + blocks);
    const uint32_t row_bytes = row_stride * static_cast<uint32_t>(sizeof(T));
    cudaError_t e = cudaSuccess;
    if (!launch_centroid_sliced<T, double, FoldF64>(vecs, n, dim, row_bytes, FoldF64{static_cast<double>(n)}, centroid,
                                                    stream, e))
        return cudaErrorInvalidValue;
    if (e != cudaSuccess) return e;
    const size_t csm = static_cast<size_t>(dim) * sizeof(double);
    if (csm > 48u * 1024u) {
        e = cudaFuncSetAttribute(k_medoid_nearest<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(csm));
        if (e != cudaSuccess) return e;
    }
    k_medoid_nearest<T><<<blocks, 256, csm, stream>>>(vecs, n, dim, row_stride, centroid, bdist, bidx);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    k_medoid_finish<<<1, 1, 0, stream>>>(bdist, bidx, blocks, d_result);
    return cudaGetLastError();
}

template <typename T, int EPL>
cudaError_t quantize_reg_impl(const CodebookArgs& a0, const T* vecs, size_t smem_optin, int num_sms,
                              cudaStream_t stream) {
    CodebookArgs a = a0;
    const size_t floats = a.pdim + 32u * (a.pdim + 1u);
    a.batch_rows = 32;
    a.smem_floats_per_warp = static_cast<uint32_t>((floats + 3u) & ~static_cast<size_t>(3));
    const size_t per_warp = static_cast<size_t>(a.smem_floats_per_warp) * 4u;
    int warps = static_cast<int>(smem_optin / per_warp);
    if (warps > 4) warps = 4;
    if (warps < 1) return cudaErrorInvalidValue;
    const size_t smem = per_warp * static_cast<size_t>(warps);
    auto fn = k_quantize_edges_reg<T, EPL>;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, 32 * warps, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    const uint64_t want = (a.n + warps - 1) / warps;
    const uint64_t cap = static_cast<uint64_t>(per_sm) * num_sms;
    const unsigned grid = static_cast<unsigned>(want < cap ? want : cap);
    fn<<<grid, 32 * warps, smem, stream>>>(a, vecs);
    return cudaGetLastError();
}

template <typename T>
cudaError_t quantize_impl(const CodebookArgs& a0, const T* vecs, size_t smem_optin, int num_sms, cudaStream_t stream) {
    // registers hold the butterfly networks up to pdim 1024 (32 rows per
    // batch must fit the shared memory); the generic kernel otherwise
    if ((a0.pdim + 32u * (a0.pdim + 1u)) * 4u <= smem_optin) {
        switch (a0.pdim) {
            case 32: return quantize_reg_impl<T, 1>(a0, vecs, smem_optin, num_sms, stream);
            case 64: return quantize_reg_impl<T, 2>(a0, vecs, smem_optin, num_sms, stream);
            case 128: return quantize_reg_impl<T, 4>(a0, vecs, smem_optin, num_sms, stream);
            case 256: return quantize_reg_impl<T, 8>(a0, vecs, smem_optin, num_sms, stream);
            case 512: return quantize_reg_impl<T, 16>(a0, vecs, smem_optin, num_sms, stream);
            case 1024: return quantize_reg_impl<T, 32>(a0, vecs, smem_optin, num_sms, stream);
            default: break;
        }
    }
    CodebookArgs a = a0;
    const size_t row_floats = a.pdim + 1u;
    // rows per batch: up to 32, within the opt-in shared memory of one warp
    size_t rows = 32;
    while (rows > 1 && (a.pdim + rows * row_floats) * 4u > smem_optin) --rows;
    if ((a.pdim + rows * row_floats) * 4u > smem_optin) return cudaErrorInvalidValue;
    a.batch_rows = static_cast<uint32_t>(rows);
    a.smem_floats_per_warp = static_cast<uint32_t>((a.pdim + rows * row_floats + 3u) & ~static_cast<size_t>(3));
    const size_t per_warp = static_cast<size_t>(a.smem_floats_per_warp) * 4u;
    int warps = static_cast<int>(smem_optin / per_warp);
    if (warps > 4) warps = 4;
    if (warps < 1) warps = 1;
    const size_t smem = per_warp * static_cast<size_t>(warps);
    cudaError_t e = cudaFuncSetAttribute(k_quantize_edges<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_quantize_edges<T>, 32 * warps, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    const uint64_t want = (a.n + warps - 1) / warps;
    const uint64_t cap = static_cast<uint64_t>(per_sm) * num_sms;
    const unsigned grid = static_cast<unsigned>(want < cap ? want : cap);
    k_quantize_edges<T><<<grid, 32 * warps, smem, stream>>>(a, vecs);
    return cudaGetLastError();
}

}  // namespace

size_t medoid_scratch_bytes(uint32_t dim) {
    return (static_cast<size_t>((dim + 1u) & ~1u) + kMedoidBlocks) * sizeof(double) + kMedoidBlocks * sizeof(uint32_t);
}

cudaError_t compute_medoid(const CodebookArgs& a, uint32_t* d_result, void* d_scratch, cudaStream_t stream) {
    if (a.n == 0 || a.dim == 0 || a.n > 0xffffffffull) return cudaErrorInvalidValue;
    return a.vecs8 ? medoid_impl<uint8_t>(a.vecs8, a.n, a.dim, a.row_stride, d_result, d_scratch, stream)
                   : medoid_impl<float>(a.vecs, a.n, a.dim, a.row_stride, d_result, d_scratch, stream);
}

cudaError_t quantize_edges(const CodebookArgs& a, size_t smem_optin, int num_sms, cudaStream_t stream) {
    if (a.n == 0) return cudaSuccess;
    if (a.pdim < 32u || (a.pdim & (a.pdim - 1u)) != 0 || a.pdim < a.dim) return cudaErrorInvalidValue;
    return a.vecs8 ? quantize_impl<uint8_t>(a, a.vecs8, smem_optin, num_sms, stream)
                   : quantize_impl<float>(a, a.vecs, smem_optin, num_sms, stream);
}

cudaError_t pack_codebook_rows(const CodebookArgs& a, uint64_t first, uint64_t count, uint32_t* out, int num_sms,
                               cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    const uint64_t want = (count + 7) / 8;
    const uint64_t cap = static_cast<uint64_t>(num_sms) * 8u;
    const unsigned grid = static_cast<unsigned>(want < cap ? want : cap);
    if (a.vecs8) k_pack_rows<uint8_t><<<grid, 256, 0, stream>>>(a, a.vecs8, first, count, out);
    else k_pack_rows<float><<<grid, 256, 0, stream>>>(a, a.vecs, first, count, out);
    return cudaGetLastError();
}

}  // namespace bsb
