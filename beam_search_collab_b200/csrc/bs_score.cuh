// bs_score.cuh -- exact L2 distances of a list of candidate rows, shared by
// the L2 search kernels and the RaBitQ rerank.
#pragma once

#include "bs_device.cuh"
#include "bs_internal.h"

namespace bsb {
namespace dev {

// Whole-warp test of the integer-exact condition for the query in smem:
// every value an integer in [qlo, qhi].  The host derives that range from the
// base vectors' own range so that every |q_d - x_d| <= B with
// dim * B^2 <= 2^24: every product and partial sum is then an exactly
// representable integer and the summation order cannot change a bit.
__device__ __forceinline__ bool query_integer_exact(const float* qsm, uint32_t dim, float qlo,
                                                    float qhi) {
    bool ok = qlo <= qhi;
    for (uint32_t d = threadIdx.x & 31u; d < dim; d += 32) {
        const float v = qsm[d];
        ok = ok && (v == rintf(v)) && (v >= qlo) && (v <= qhi);
    }
    return __all_sync(kFull, ok);
}

// Distances of the m rows cids[0..m) into cdist[0..m), in the reference's
// sequential order.  Rows are staged into shared memory with coalesced
// 16-byte cp.async, then lane i folds row i.  Ends with __syncwarp.
__device__ __forceinline__ void score_rows_seq(const SearchParams& p, uint32_t m,
                                               const uint32_t* cids, float* cdist,
                                               const float* qsm, float* stage, unsigned lane) {
    const uint32_t chunks = p.row_stride >> 2;
    for (uint32_t c0 = 0; c0 < m; c0 += p.stage_rows) {
        const uint32_t nrows = min(p.stage_rows, m - c0);
        const uint32_t total = nrows * chunks;
        for (uint32_t t = lane; t < total; t += 32) {
            const uint32_t r = t / chunks;
            const uint32_t ch = t - r * chunks;
            const float* src = p.vecs + static_cast<size_t>(cids[c0 + r]) * p.row_stride + ch * 4;
            cp_async16(stage + r * p.stage_pitch + ch * 4, src);
        }
        cp_async_wait_all();
        __syncwarp();
        if (lane < nrows) cdist[c0 + lane] = l2_seq(qsm, stage + lane * p.stage_pitch, p.dim);
        __syncwarp();
    }
}

// Same order without staging: lane i reads row i straight from global
// memory.  Used by the integer-exact kernels for a query that does not meet
// the integer condition (those kernels carry no staging area).
__device__ __forceinline__ void score_rows_seq_direct(const SearchParams& p, uint32_t m,
                                                      const uint32_t* cids, float* cdist,
                                                      const float* qsm, unsigned lane) {
    for (uint32_t c0 = 0; c0 < m; c0 += 32) {
        const uint32_t s = c0 + lane;
        if (s < m) cdist[s] = l2_seq(qsm, p.vecs + static_cast<size_t>(cids[s]) * p.row_stride, p.dim);
    }
    __syncwarp();
}

// Integer-exact data: 4 teams of 8 lanes, one row per team at a time, 16-byte
// loads straight from HBM, fma and a shuffle tree (exact for these values).
__device__ __forceinline__ void score_rows_team(const SearchParams& p, uint32_t m,
                                                const uint32_t* cids, float* cdist,
                                                const float* qsm, unsigned lane) {
    const unsigned team = lane >> 3, tl = lane & 7u;
    for (uint32_t s0 = 0; s0 < m; s0 += 16) {
        const float* rp[4];
        bool ok[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t s = s0 + team + 4u * j;
            ok[j] = s < m;
            rp[j] = p.vecs + static_cast<size_t>(cids[ok[j] ? s : 0]) * p.row_stride;
        }
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
        for (uint32_t d = tl * 4; d < p.row_stride; d += 32) {
            const float4 qv = *reinterpret_cast<const float4*>(qsm + d);
            float4 v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) v[j] = ok[j] ? ldg_stream4(rp[j] + d) : qv;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float t;
                t = qv.x - v[j].x; acc[j] = fmaf(t, t, acc[j]);
                t = qv.y - v[j].y; acc[j] = fmaf(t, t, acc[j]);
                t = qv.z - v[j].z; acc[j] = fmaf(t, t, acc[j]);
                t = qv.w - v[j].w; acc[j] = fmaf(t, t, acc[j]);
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            acc[j] += __shfl_xor_sync(kFull, acc[j], 4);
            acc[j] += __shfl_xor_sync(kFull, acc[j], 2);
            acc[j] += __shfl_xor_sync(kFull, acc[j], 1);
        }
        if (tl == 0) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (ok[j]) cdist[s0 + team + 4u * j] = acc[j];
        }
    }
    __syncwarp();
}

// Dispatch on the compile-time distance mode and the per-query flag.
template <int DM>
__device__ __forceinline__ void score_rows(const SearchParams& p, uint32_t m, const uint32_t* cids,
                                           float* cdist, const float* qsm, float* stage,
                                           unsigned lane, bool team_ok) {
    if (DM == kSeq) {
        score_rows_seq(p, m, cids, cdist, qsm, stage, lane);
    } else if (team_ok) {
        score_rows_team(p, m, cids, cdist, qsm, lane);
    } else {
        score_rows_seq_direct(p, m, cids, cdist, qsm, lane);
    }
}

}  // namespace dev
}  // namespace bsb
