// bs_nb.cuh -- distances from the query to the rows of a neighbourhood
// block (the expanded node's adjacency row followed by its neighbours' rows,
// laid out by k_build_nb in bs_search_nb.cu), shared by the warp-per-query
// and the block-per-query kernels over that layout.
#pragma once

#include <cstdint>

#include "bs_device.cuh"
#include "bs_internal.h"
#include "bs_score.cuh"

namespace bsb {
namespace dev {

// ------------------------------------------------------------- scoring

// Position of 16-byte chunk c of neighbour row s inside a block of u8 rows
// (nch chunks per row): the chunks of each group of 8 are rotated by s, so
// the 8 lanes of one shared-memory phase, reading chunk c of 8 consecutive
// rows, touch 8 different bank groups.
__device__ __forceinline__ uint32_t nb_chunk_pos(uint32_t c, uint32_t s, uint32_t nch) {
    const uint32_t g0 = c & ~7u;
    const uint32_t g = nch - g0 < 8u ? nch - g0 : 8u;
    return g0 + (c - g0 + s) % g;
}

__device__ __forceinline__ void dp4a_chunk(const uint4 v, const uint4 q, unsigned& xx, unsigned& qx) {
    xx = __dp4a(v.x, v.x, xx); qx = __dp4a(q.x, v.x, qx);
    xx = __dp4a(v.y, v.y, xx); qx = __dp4a(q.y, v.y, qx);
    xx = __dp4a(v.z, v.z, xx); qx = __dp4a(q.z, v.z, qx);
    xx = __dp4a(v.w, v.w, xx); qx = __dp4a(q.w, v.w, qx);
}

__device__ __forceinline__ float seq_step(float acc, float q, float x) {
    const float t = __fsub_rn(q, x);
    return __fadd_rn(acc, __fmul_rn(t, t));
}

// Distance from the query to neighbour row s of the block, computed by the
// calling lane alone.
//   kU8, integer query : sum (q-x)^2 = sum x^2 - 2 sum q.x + sum q^2 over the
//                        bytes with __dp4a -- exact integers, hence the
//                        reference's fp32 value (the host only selects this
//                        path when dim * 255^2 fits 24 bits)
//   kTeam, integer data: fused multiply-add; every partial sum is an exact
//                        integer, so any order gives the reference's bits
//   otherwise          : the reference's sequential fold, d = 0..dim-1, each
//                        operation rounded separately
//                        (include/cpu_search_base.hpp:29-37); the zero pad
//                        lanes add +0 and change nothing
template <int DM>
__device__ __forceinline__ float block_row_dist(const SearchParams& p, const unsigned char* rows, uint32_t s,
                                                const float* qsm, const unsigned char* qb, uint32_t qq,
                                                bool team_ok) {
    const unsigned char* row = rows + static_cast<size_t>(s) * p.nb_pitch;
    if (DM == kU8) {
        const uint32_t nch = p.row_bytes / 16u;
        if (team_ok) {
            unsigned xx = 0u, qx = 0u;
            if ((nch & 7u) == 0u) {
                for (uint32_t g0 = 0; g0 < nch; g0 += 8u) {
#pragma unroll 4
                    for (uint32_t t = 0; t < 8u; ++t) {
                        const uint4 v = *reinterpret_cast<const uint4*>(row + (g0 + ((s + t) & 7u)) * 16u);
                        const uint4 q = *reinterpret_cast<const uint4*>(qb + (g0 + t) * 16u);
                        dp4a_chunk(v, q, xx, qx);
                    }
                }
            } else {
                for (uint32_t c = 0; c < nch; ++c) {
                    const uint4 v = *reinterpret_cast<const uint4*>(row + nb_chunk_pos(c, s, nch) * 16u);
                    const uint4 q = *reinterpret_cast<const uint4*>(qb + c * 16u);
                    dp4a_chunk(v, q, xx, qx);
                }
            }
            return static_cast<float>(xx - 2u * qx + qq);
        }
        float acc = 0.0f;
        for (uint32_t c = 0; c < nch; ++c) {
            const unsigned char* chunk = row + nb_chunk_pos(c, s, nch) * 16u;
            const uint32_t d0 = c * 16u;
            const uint32_t n = p.dim - d0 < 16u ? p.dim - d0 : 16u;
            for (uint32_t k = 0; k < n; ++k) acc = seq_step(acc, qsm[d0 + k], static_cast<float>(chunk[k]));
        }
        return acc;
    }
    const float4* r4 = reinterpret_cast<const float4*>(row);
    const float4* q4 = reinterpret_cast<const float4*>(qsm);
    const uint32_t units = p.row_stride / 4u;
    float acc = 0.0f;
    if (DM == kTeam && team_ok) {
        for (uint32_t u = 0; u < units; ++u) {
            const float4 v = r4[u], q = q4[u];
            float t;
            t = q.x - v.x; acc = fmaf(t, t, acc);
            t = q.y - v.y; acc = fmaf(t, t, acc);
            t = q.z - v.z; acc = fmaf(t, t, acc);
            t = q.w - v.w; acc = fmaf(t, t, acc);
        }
        return acc;
    }
    for (uint32_t u = 0; u < units; ++u) {
        const float4 v = r4[u], q = q4[u];
        acc = seq_step(acc, q.x, v.x);
        acc = seq_step(acc, q.y, v.y);
        acc = seq_step(acc, q.z, v.z);
        acc = seq_step(acc, q.w, v.w);
    }
    return acc;
}

// Exact distance of one node straight from the gather layout (the entry).
template <int DM>
__device__ __forceinline__ void score_direct(const SearchParams& p, uint32_t m, const uint32_t* cids,
                                             float* cdist, const float* qsm, const uint32_t* q8,
                                             unsigned lane, bool team_ok) {
    if (DM == kU8) {
        if (team_ok) score_rows_u8(p, m, cids, cdist, q8, lane);
        else score_rows_u8_seq(p, m, cids, cdist, qsm, lane);
    } else if (DM == kTeam && team_ok) {
        score_rows_team(p, m, cids, cdist, qsm, lane);
    } else {
        score_rows_seq_direct(p, m, cids, cdist, qsm, lane);
    }
}

}  // namespace dev
}  // namespace bsb
