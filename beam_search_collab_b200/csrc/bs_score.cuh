// bs_score.cuh -- exact L2 distances of a list of candidate rows, shared by
// the L2 search kernels and the RaBitQ rerank.
#pragma once

#include "bs_device.cuh"
#include "bs_internal.h"

namespace bsb {
namespace dev {

// Where query qi is read from: the caller's pinned host buffer through its
// device mapping (plain loads, once per query, over the bus), else the
// device array.
__device__ __forceinline__ const float* query_src(const SearchParams& p, uint32_t qi) {
    return (p.queries_src != nullptr ? p.queries_src : p.queries) + static_cast<size_t>(qi) * p.dim;
}

// A query row read from host memory mapped into the device (page-locked
// buffers used in place) into its device slot: every load of a thread is
// issued before its stores, so the row crosses the bus in one round trip
// (16-byte loads when the row allows them) instead of one per 32 elements.
__device__ __forceinline__ void copy_query_row(float* __restrict__ slot, const float* __restrict__ q, uint32_t dim,
                                               unsigned t, unsigned nt) {
    if ((dim & 3u) == 0u && ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(slot)) & 15u) == 0u) {
        const float4* q4 = reinterpret_cast<const float4*>(q);
        float4* s4 = reinterpret_cast<float4*>(slot);
        const uint32_t n4 = dim / 4u;
        for (uint32_t b = 0; b < n4; b += 4u * nt) {
            float4 v[4];
#pragma unroll
            for (uint32_t j = 0; j < 4u; ++j) {
                const uint32_t i = b + j * nt + t;
                if (i < n4) v[j] = q4[i];
            }
#pragma unroll
            for (uint32_t j = 0; j < 4u; ++j) {
                const uint32_t i = b + j * nt + t;
                if (i < n4) s4[i] = v[j];
            }
        }
        return;
    }
    for (uint32_t d = t; d < dim; d += nt) slot[d] = q[d];
}

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

// Wide rows (the 960-d C4 rows are 3.84 KB): the same sequential order, with
// the rows streamed through a ring of S chunks of kRingCh dimensions of up to
// 32 rows -- every lane folds its own row while the next S-1 chunks are in
// flight -- so a warp holds S * 32 * kRingPitch floats of shared memory
// instead of whole rows.  Each lane keeps its running sum in a register
// across chunks and adds the elements d = 0..row_stride-1 in order with
// separately rounded operations: the reference's bits (the zero pad of the
// stored rows and of the query adds +0).  S (p.stage_ring) is chosen by the
// planner: the deepest ring that still keeps every query of the launch
// resident (more bytes in flight per SM without a second wave).
constexpr uint32_t kRingCh = 32;       // dimensions per chunk
constexpr uint32_t kRingStages = 4;    // the default (and the builders') ring
constexpr uint32_t kRingPitch = 36;    // floats per staged row chunk: 9 16-byte units, odd
constexpr uint32_t kRingStageFloats = 32u * kRingPitch;
constexpr uint32_t kRingFloats = kRingStages * kRingStageFloats;

// Sequential fold of one staged row chunk (n4 groups of 4 dimensions from d0)
// into acc; full chunks are unrolled so that the shared-memory loads run
// ahead of the dependent additions.
__device__ __forceinline__ float fold_chunk(float acc, const float* x, const float* qsm, uint32_t d0, uint32_t n4) {
    if (n4 == kRingCh / 4u) {
        float4 v[kRingCh / 4u];
#pragma unroll
        for (uint32_t j = 0; j < kRingCh / 4u; ++j) v[j] = *reinterpret_cast<const float4*>(x + 4u * j);
#pragma unroll
        for (uint32_t j = 0; j < kRingCh / 4u; ++j) {
            const float4 q = *reinterpret_cast<const float4*>(qsm + d0 + 4u * j);
            float t;
            t = __fsub_rn(q.x, v[j].x); acc = __fadd_rn(acc, __fmul_rn(t, t));
            t = __fsub_rn(q.y, v[j].y); acc = __fadd_rn(acc, __fmul_rn(t, t));
            t = __fsub_rn(q.z, v[j].z); acc = __fadd_rn(acc, __fmul_rn(t, t));
            t = __fsub_rn(q.w, v[j].w); acc = __fadd_rn(acc, __fmul_rn(t, t));
        }
        return acc;
    }
    for (uint32_t j = 0; j < n4; ++j) {
        const float4 v = *reinterpret_cast<const float4*>(x + 4u * j);
        const float4 q = *reinterpret_cast<const float4*>(qsm + d0 + 4u * j);
        float t;
        t = __fsub_rn(q.x, v.x); acc = __fadd_rn(acc, __fmul_rn(t, t));
        t = __fsub_rn(q.y, v.y); acc = __fadd_rn(acc, __fmul_rn(t, t));
        t = __fsub_rn(q.z, v.z); acc = __fadd_rn(acc, __fmul_rn(t, t));
        t = __fsub_rn(q.w, v.w); acc = __fadd_rn(acc, __fmul_rn(t, t));
    }
    return acc;
}

template <uint32_t S>
__device__ __forceinline__ void score_rows_seq_ring_s(const SearchParams& p, uint32_t m, const uint32_t* cids,
                                                      float* cdist, const float* qsm, float* ring,
                                                      unsigned lane) {
    const uint32_t nch = (p.row_stride + kRingCh - 1) / kRingCh;
    const uint32_t part = lane & 7u;     // 16-byte piece of a row chunk this lane copies
    for (uint32_t g0 = 0; g0 < m; g0 += 32) {
        const uint32_t rows = min(32u, m - g0);
        // one commit group per chunk (empty past the last one), so that
        // wait_group S-1 always means "chunk c has landed"
        auto issue = [&](uint32_t c) {
            if (c < nch) {
                const uint32_t d = c * kRingCh + part * 4u;
                float* st = ring + (c % S) * kRingStageFloats + part * 4u;
                if (d < p.row_stride)
                    for (uint32_t r = lane >> 3; r < rows; r += 4)
                        cp_async16(st + r * kRingPitch, p.vecs + static_cast<size_t>(cids[g0 + r]) * p.row_stride + d);
            }
            asm volatile("cp.async.commit_group;\n" ::: "memory");
        };
        for (uint32_t c = 0; c + 1 < S; ++c) issue(c);
        float acc = 0.0f;
        for (uint32_t c = 0; c < nch; ++c) {
            issue(c + S - 1);
            asm volatile("cp.async.wait_group %0;\n" ::"n"(S - 1) : "memory");
            __syncwarp();
            if (lane < rows) {
                const uint32_t d0 = c * kRingCh;
                acc = fold_chunk(acc, ring + (c % S) * kRingStageFloats + lane * kRingPitch, qsm, d0,
                                 min(kRingCh, p.row_stride - d0) / 4u);
            }
            __syncwarp();   // this stage is refilled by the next iteration's issue
        }
        if (lane < rows) cdist[g0 + lane] = acc;
        asm volatile("cp.async.wait_group 0;\n" ::: "memory");
        __syncwarp();
    }
}

__device__ __forceinline__ void score_rows_seq_ring(const SearchParams& p, uint32_t m, const uint32_t* cids,
                                                    float* cdist, const float* qsm, float* ring,
                                                    unsigned lane) {
    switch (p.stage_ring) {
        case 5: score_rows_seq_ring_s<5>(p, m, cids, cdist, qsm, ring, lane); break;
        case 6: score_rows_seq_ring_s<6>(p, m, cids, cdist, qsm, ring, lane); break;
        case 8: score_rows_seq_ring_s<8>(p, m, cids, cdist, qsm, ring, lane); break;
        default: score_rows_seq_ring_s<kRingStages>(p, m, cids, cdist, qsm, ring, lane); break;
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

__device__ __forceinline__ uint4 ldg_stream_u4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// u8 rows and a query of integers in [0,255]: 4 teams of 8 lanes, up to 8
// rows per team in flight (one 16-byte load per lane and row when the row is
// at most 128 bytes) and dp4a integer dot products.  With dim * 255^2 <= 2^24
// (checked on the host) the integer sum is the reference's fp32 result.
// sum(q - x)^2 = sum q^2 + sum x^2 - 2 sum q*x over the bytes, each term an
// exact integer: two dp4a per 4 dimensions.  qq = sum q^2 of the query.
template <int SLOTS>
__device__ __forceinline__ void score_rows_u8_slots(const SearchParams& p, uint32_t m, const uint32_t* cids,
                                                    float* cdist, const uint32_t* q8, unsigned qq,
                                                    unsigned lane) {
    const unsigned team = lane >> 3, tl = lane & 7u;
    const unsigned char* qb = reinterpret_cast<const unsigned char*>(q8);
    for (uint32_t s0 = 0; s0 < m; s0 += 4u * SLOTS) {
        unsigned xx[SLOTS], qx[SLOTS];
#pragma unroll
        for (int j = 0; j < SLOTS; ++j) { xx[j] = 0u; qx[j] = 0u; }
        for (uint32_t off = tl * 16u; off < p.row_bytes; off += 128u) {
            const uint4 q = *reinterpret_cast<const uint4*>(qb + off);
            uint4 v[SLOTS];
#pragma unroll
            for (int j = 0; j < SLOTS; ++j) {
                const uint32_t s = s0 + team + 4u * j;
                v[j] = s < m ? ldg_stream_u4(p.vecs8 + static_cast<size_t>(cids[s]) * p.row_bytes + off)
                             : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int j = 0; j < SLOTS; ++j) {
                xx[j] = __dp4a(v[j].x, v[j].x, xx[j]);
                qx[j] = __dp4a(q.x, v[j].x, qx[j]);
                xx[j] = __dp4a(v[j].y, v[j].y, xx[j]);
                qx[j] = __dp4a(q.y, v[j].y, qx[j]);
                xx[j] = __dp4a(v[j].z, v[j].z, xx[j]);
                qx[j] = __dp4a(q.z, v[j].z, qx[j]);
                xx[j] = __dp4a(v[j].w, v[j].w, xx[j]);
                qx[j] = __dp4a(q.w, v[j].w, qx[j]);
            }
        }
        unsigned acc[SLOTS];
#pragma unroll
        for (int j = 0; j < SLOTS; ++j) acc[j] = xx[j] - 2u * qx[j];   // mod 2^32; qq added below
#pragma unroll
        for (int j = 0; j < SLOTS; ++j) {
            acc[j] += __shfl_xor_sync(kFull, acc[j], 4);
            acc[j] += __shfl_xor_sync(kFull, acc[j], 2);
            acc[j] += __shfl_xor_sync(kFull, acc[j], 1);
        }
        if (tl == 0) {
#pragma unroll
            for (int j = 0; j < SLOTS; ++j) {
                const uint32_t s = s0 + team + 4u * j;
                if (s < m) cdist[s] = static_cast<float>(acc[j] + qq);
            }
        }
    }
    __syncwarp();
}

// up to 1, 4 or 8 rows per team (rows in flight per lane) by list length
__device__ __forceinline__ void score_rows_u8(const SearchParams& p, uint32_t m, const uint32_t* cids,
                                              float* cdist, const uint32_t* q8, unsigned lane) {
    const unsigned qq = q8[p.row_bytes / 4u];   // sum of q^2, stored after the packed bytes
    if (m <= 4) score_rows_u8_slots<1>(p, m, cids, cdist, q8, qq, lane);
    else if (m <= 16) score_rows_u8_slots<4>(p, m, cids, cdist, q8, qq, lane);
    else score_rows_u8_slots<8>(p, m, cids, cdist, q8, qq, lane);
}

// u8 rows and any query: lane i folds row i in the reference order, each
// byte converted to float exactly.
__device__ __forceinline__ float l2_seq_u8(const float* __restrict__ q, const uint8_t* __restrict__ x,
                                           uint32_t dim) {
    float s = 0.0f;
    uint32_t d = 0;
    for (; d + 16 <= dim; d += 16) {
        const uint4 w = ldg_stream_u4(x + d);
        const unsigned words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const float xv = static_cast<float>((words[k >> 2] >> (8 * (k & 3))) & 0xffu);
            const float t = __fsub_rn(q[d + k], xv);
            s = __fadd_rn(s, __fmul_rn(t, t));
        }
    }
    for (; d < dim; ++d) {
        const float t = __fsub_rn(q[d], static_cast<float>(x[d]));
        s = __fadd_rn(s, __fmul_rn(t, t));
    }
    return s;
}

__device__ __forceinline__ void score_rows_u8_seq(const SearchParams& p, uint32_t m, const uint32_t* cids,
                                                  float* cdist, const float* qsm, unsigned lane) {
    for (uint32_t c0 = 0; c0 < m; c0 += 32) {
        const uint32_t s = c0 + lane;
        if (s < m) cdist[s] = l2_seq_u8(qsm, p.vecs8 + static_cast<size_t>(cids[s]) * p.row_bytes, p.dim);
    }
    __syncwarp();
}

// kU8: the query packed as bytes into q8 (row_bytes, zero pad) followed by
// the word sum q^2, for a query that passed query_integer_exact with a range
// inside [0,255].
__device__ __forceinline__ void pack_query_u8(const float* qsm, uint32_t dim, uint32_t row_bytes,
                                              uint32_t* q8, unsigned lane) {
    unsigned qq = 0;
    for (uint32_t w = lane; w < row_bytes / 4u; w += 32) {
        unsigned v = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t d = 4u * w + k;
            const unsigned b = d < dim ? static_cast<unsigned>(qsm[d]) & 0xffu : 0u;
            v |= b << (8 * k);
        }
        q8[w] = v;
        qq = __dp4a(v, v, qq);
    }
    for (int o = 16; o > 0; o >>= 1) qq += __shfl_xor_sync(kFull, qq, o);
    if (lane == 0) q8[row_bytes / 4u] = qq;
    __syncwarp();
}

// Dispatch on the compile-time distance mode and the per-query flag.
template <int DM>
__device__ __forceinline__ void score_rows(const SearchParams& p, uint32_t m, const uint32_t* cids,
                                           float* cdist, const float* qsm, const uint32_t* q8,
                                           float* stage, unsigned lane, bool team_ok) {
    if (DM == kSeq) {
        if (p.stage_ring) score_rows_seq_ring(p, m, cids, cdist, qsm, stage, lane);
        else score_rows_seq(p, m, cids, cdist, qsm, stage, lane);
    } else if (DM == kTeam) {
        if (team_ok) score_rows_team(p, m, cids, cdist, qsm, lane);
        else score_rows_seq_direct(p, m, cids, cdist, qsm, lane);
    } else {
        if (team_ok) score_rows_u8(p, m, cids, cdist, q8, lane);
        else score_rows_u8_seq(p, m, cids, cdist, qsm, lane);
    }
}

// Key of the beam's last admissible position (topk-1); kEmptyKey while the
// beam is not full.  A candidate at or above it can never enter the beam.
template <int RX>
__device__ __forceinline__ uint64_t beam_bound(const uint64_t (&beam)[RX], uint32_t topk) {
    const uint32_t pos = (topk < 32u * RX ? topk : 32u * RX) - 1u;
    const int reg = static_cast<int>(pos >> 5);
    uint64_t mine = kEmptyKey;
#pragma unroll
    for (int r = 0; r < RX; ++r)
        if (r == reg) mine = beam[r];
    return __shfl_sync(kFull, mine, static_cast<int>(pos & 31u));
}

}  // namespace dev
}  // namespace bsb
