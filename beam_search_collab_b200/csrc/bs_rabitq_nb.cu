// bs_rabitq_nb.cu -- the RaBitQ beam search (mode rabitq) over node blocks.
//
// Same results as bs_rabitq.cu, i.e. the reference CPU search
// CPURabitqSearch::search (include/cpu_search_rabitq.hpp:28-150):
//
//   query   : q*signs, Walsh-Hadamard transform over padded_dim, 6-bit
//             quantisation q_d = lroundf((x - low) * (1/w) + 0.5), w = (high-low)/63
//   seed    : the entry point with its exact L2 distance
//   expand  : the smallest unexpanded entry p; exact L2 of p; every neighbour
//             i not seen before (marked when pushed, never forgotten) gets
//             the estimate ((tx_i + exact_p) + (fdq_i*w)*ip) + fvq_i*low with
//             ip = 2*raw - sum_q, raw = sum_{d: bit_d(i)=1} q_d (exact integer)
//   finish  : exact L2 for every beam entry, re-sort by (dist, id), K best.
//
// Memory path: everything one expansion reads depends only on the expanded
// node, so every node owns one contiguous block in HBM,
//
//   [ adjacency row | neighbour codes [deg][wpp] | factors [3][deg] | own row ]
//
// (C3: 256 + 1,024 + 768 + 384 = 2,432 B) and an expansion is ONE bulk copy
// into shared memory, with the likely next block prefetched into L2 (the
// layout of the reference's codebook.bin rows, include/rabitq.hpp:61-64,
// regrouped).  The visited set must never forget (an estimate depends on the
// parent that reaches a node first), so it is a bitmap over the node ids per
// resident warp in global memory: one atomicOr per neighbour both tests and
// sets its bit (the returned word says whether it was new), and the ids a
// query sets are logged so that the words are cleared when it ends -- no
// per-query clearing of a whole table.  The exact distance of the expanded
// node folds its own row from the block (products on all lanes, the
// reference's sequential sum on one) while the atomics are in flight.
//
// Estimator, integer part: the 7 bit-planes of the quantised query
// (q_d <= 64) and raw = sum_b popc(plane_b & code) << b, or (rq_lut) a
// per-query table of 4-dimension group sums indexed by the code's nibbles.
#include <cfloat>
#include <cstdio>

#include "bs_bulk.cuh"
#include "bs_device.cuh"
#include "bs_internal.h"
#include "bs_score.cuh"

namespace bsb {

using namespace dev;

namespace {

constexpr int kPlanes = 7;   // quantised query values are 1..64

// Test-and-set of node c's bit: true when it was not set before.
__device__ __forceinline__ bool visit(uint32_t* bits, uint32_t c) {
    const uint32_t m = 1u << (c & 31u);
    return (atomicOr(bits + (c >> 5), m) & m) == 0u;
}

// Clears the bitmap words of the ids this query set (or the whole bitmap when
// the log overflowed) and orders the clearing before the next query's atomics.
__device__ __forceinline__ void clear_visited(const SearchParams& p, uint32_t* bits, const uint32_t* log,
                                              uint32_t logged, unsigned lane) {
    __syncwarp();
    if (logged <= p.vis_log_cap) {
        for (uint32_t i = lane; i < logged; i += 32) bits[log[i] >> 5] = 0u;
    } else {
        uint4* b4 = reinterpret_cast<uint4*>(bits);
        for (uint32_t i = lane; i < p.vis_words / 4u; i += 32) b4[i] = make_uint4(0u, 0u, 0u, 0u);
    }
    __threadfence();
    __syncwarp();
}

// Exact squared distance from the query to the expanded node's own row in the
// block, in the reference's order (include/cpu_search_rabitq.hpp:60-68).
//   kSeq / fractional queries: every lane squares its differences in place,
//     one lane adds them in order d = 0..dim-1 (separately rounded
//     operations, the zero pad adds +0)
//   kTeam / kU8 with an integer query: exact integers, any order
template <int DM>
__device__ __forceinline__ float block_exact(const SearchParams& p, unsigned char* row, const float* qsm,
                                             const uint32_t* q8, bool team_ok, unsigned lane) {
    if (DM == kU8 && team_ok) {
        unsigned acc = 0u;
        const uint32_t* x = reinterpret_cast<const uint32_t*>(row);
        for (uint32_t w = lane; w < p.row_bytes / 4u; w += 32) {
            const unsigned d = __vabsdiffu4(q8[w], x[w]);
            acc = __dp4a(d, d, acc);
        }
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(kFull, acc, o);
        return static_cast<float>(acc);
    }
    if (DM == kU8) {
        float e0 = 0.0f;
        if (lane == 0)
            for (uint32_t d = 0; d < p.dim; ++d) {
                const float t = __fsub_rn(qsm[d], static_cast<float>(row[d]));
                e0 = __fadd_rn(e0, __fmul_rn(t, t));
            }
        return __shfl_sync(kFull, e0, 0);
    }
    float* x = reinterpret_cast<float*>(row);
    if (DM == kTeam && team_ok) {
        float acc = 0.0f;
        for (uint32_t d = lane; d < p.row_stride; d += 32) {
            const float t = qsm[d] - x[d];
            acc = fmaf(t, t, acc);
        }
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(kFull, acc, o);
        return acc;
    }
    for (uint32_t d = lane; d < p.row_stride; d += 32) {
        const float t = __fsub_rn(qsm[d], x[d]);
        x[d] = __fmul_rn(t, t);
    }
    __syncwarp();
    float e0 = 0.0f;
    if (lane == 0) {
        const float4* x4 = reinterpret_cast<const float4*>(x);
        for (uint32_t u = 0; u < p.row_stride / 4u; ++u) {
            const float4 v = x4[u];
            e0 = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(e0, v.x), v.y), v.z), v.w);
        }
    }
    // these generic writes precede the next bulk copy into the buffer
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    return __shfl_sync(kFull, e0, 0);
}

// raw = sum of q_d over the set bits of one neighbour's code.
template <int EM>
__device__ __forceinline__ uint32_t raw_sum(const uint32_t* code, uint32_t wpp, const uint32_t* est_tab) {
    uint32_t raw = 0;
    if (EM == 0) {
        // bit-planes: est_tab = [wd][8] words (planes 0..6, pad)
        for (uint32_t wd = 0; wd < wpp; ++wd) {
            const uint32_t cw = code[wd];
            const uint4 a = *reinterpret_cast<const uint4*>(est_tab + 8u * wd);
            const uint4 b = *reinterpret_cast<const uint4*>(est_tab + 8u * wd + 4u);
            raw += static_cast<uint32_t>(__popc(a.x & cw));
            raw += static_cast<uint32_t>(__popc(a.y & cw)) << 1;
            raw += static_cast<uint32_t>(__popc(a.z & cw)) << 2;
            raw += static_cast<uint32_t>(__popc(a.w & cw)) << 3;
            raw += static_cast<uint32_t>(__popc(b.x & cw)) << 4;
            raw += static_cast<uint32_t>(__popc(b.y & cw)) << 5;
            raw += static_cast<uint32_t>(__popc(b.z & cw)) << 6;
        }
    } else {
        // nibble table: est_tab = u16 [pdim/4][16], entry = sum of q_d over
        // the set bits of the nibble in its group of 4 dimensions
        const uint16_t* lut = reinterpret_cast<const uint16_t*>(est_tab);
        for (uint32_t wd = 0; wd < wpp; ++wd) {
            const uint32_t cw = code[wd];
            const uint16_t* t = lut + 128u * wd;
#pragma unroll
            for (uint32_t k = 0; k < 8u; ++k) raw += t[16u * k + ((cw >> (4u * k)) & 15u)];
        }
    }
    return raw;
}

// Resident blocks of 4 warps per SM the register budget is fitted to (6:
// 85 registers a thread) for beams up to 256 entries.
#ifndef BS_RQ_MIN_BLOCKS
#define BS_RQ_MIN_BLOCKS 6
#endif

template <int RX, int RY, int DM, int EM>
__global__ void __launch_bounds__(128, (RX <= 8 ? BS_RQ_MIN_BLOCKS : 4)) k_search_rq_nb(const SearchParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const unsigned lane = threadIdx.x & 31u;
    unsigned char* ws = smem_raw + static_cast<size_t>(threadIdx.x >> 5) * p.smem_per_warp;
    float* qsm = reinterpret_cast<float*>(ws);
    uint32_t* q8 = reinterpret_cast<uint32_t*>(ws + p.off_q8);
    uint32_t* est_tab = reinterpret_cast<uint32_t*>(ws + p.off_est);
    uint32_t* cids = reinterpret_cast<uint32_t*>(ws + p.off_cids);
    float* cdist = reinterpret_cast<float*>(ws + p.off_cdist);
    uint64_t* ckeys = reinterpret_cast<uint64_t*>(ws + p.off_keys);
    uint64_t* mbar = reinterpret_cast<uint64_t*>(ws + p.off_mbar);
    unsigned char* blk = ws + p.off_block;
    const uint32_t* blk_adj = reinterpret_cast<const uint32_t*>(blk);
    const uint32_t* blk_codes = reinterpret_cast<const uint32_t*>(blk + p.rq_off_codes);
    const float* blk_fac = reinterpret_cast<const float*>(blk + p.rq_off_fac);
    unsigned char* blk_row = blk + p.rq_off_row;

    const uint32_t deg = p.degree;
    const uint32_t wpp = p.wpp;
    const uint32_t pdim = p.pdim;
    const unsigned lt_mask = (1u << lane) - 1u;
    const size_t gwarp = static_cast<size_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    uint32_t* vbits = p.vis + gwarp * (static_cast<size_t>(p.vis_words) + p.vis_log_cap);
    uint32_t* vlog = vbits + p.vis_words;
    unsigned phase = 0;
    if (lane == 0) mbar_init(mbar);
    __syncwarp();

    for (;;) {
        unsigned qi = 0;
        if (lane == 0) qi = atomicAdd(&p.counters->next_query, 1u);
        qi = __shfl_sync(kFull, qi, 0);
        if (qi >= p.nq) break;

        const float* q = query_src(p, qi);
        for (uint32_t d = lane; d < p.row_stride; d += 32) qsm[d] = d < p.dim ? q[d] : 0.0f;
        __syncwarp();
        const bool team_ok = DM != kSeq && query_integer_exact(qsm, p.dim, p.team_qlo, p.team_qhi);
        if (DM != kSeq && !team_ok && lane == 0) atomicAdd(&p.counters->team_fallbacks, 1u);
        if (DM == kU8 && team_ok) pack_query_u8(qsm, p.dim, p.row_bytes, q8, lane);

        // ---- rotate + quantise (include/cpu_search_rabitq.hpp:34-57); the
        // rotated query and its quantised bytes live in the block buffer
        float* qrot = reinterpret_cast<float*>(blk);
        unsigned char* qq = blk + pdim * 4u;
        for (uint32_t d = lane; d < pdim; d += 32)
            qrot[d] = d < p.dim ? __fmul_rn(qsm[d], __ldg(p.signs + d)) : 0.0f;
        __syncwarp();
        for (uint32_t len = 1; len < pdim; len <<= 1) {
            for (uint32_t pi = lane; pi < (pdim >> 1); pi += 32) {
                const uint32_t b = pi / len, j = pi - b * len;
                const uint32_t i1 = b * (len << 1) + j, i2 = i1 + len;
                const float u = qrot[i1], v = qrot[i2];
                qrot[i1] = __fadd_rn(u, v);
                qrot[i2] = __fsub_rn(u, v);
            }
            __syncwarp();
        }
        float lo = FLT_MAX, hi = -FLT_MAX;
        for (uint32_t d = lane; d < pdim; d += 32) {
            lo = fminf(lo, qrot[d]);
            hi = fmaxf(hi, qrot[d]);
        }
        for (int o = 16; o > 0; o >>= 1) {
            lo = fminf(lo, __shfl_xor_sync(kFull, lo, o));
            hi = fmaxf(hi, __shfl_xor_sync(kFull, hi, o));
        }
        const float w = __fdiv_rn(__fsub_rn(hi, lo), 63.0f);
        const float inv_w = __fdiv_rn(1.0f, w);
        int32_t sum_q = 0;
        for (uint32_t wd = 0; wd < wpp; ++wd) {
            const float t = __fadd_rn(__fmul_rn(__fsub_rn(qrot[wd * 32 + lane], lo), inv_w), 0.5f);
            // lroundf of NaN (w == 0) is the integer indefinite on the
            // reference's x86 host, which truncates to 0 as uint8_t
            const uint32_t v = (t == t) ? (static_cast<uint32_t>(lroundf(t)) & 0xffu) : 0u;
            sum_q += static_cast<int32_t>(v);
            if (EM == 0) {
#pragma unroll
                for (int b = 0; b < kPlanes; ++b) {
                    const unsigned word = __ballot_sync(kFull, (v >> b) & 1u);
                    if (lane == 0) est_tab[8 * wd + b] = word;
                }
            } else {
                qq[wd * 32 + lane] = static_cast<unsigned char>(v);
            }
        }
        for (int o = 16; o > 0; o >>= 1) sum_q += __shfl_xor_sync(kFull, sum_q, o);
        if (EM == 1) {
            __syncwarp();
            uint16_t* lut = reinterpret_cast<uint16_t*>(est_tab);
            for (uint32_t e = lane; e < pdim * 4u; e += 32) {
                const uint32_t g = e >> 4, nib = e & 15u;
                uint32_t s = 0;
#pragma unroll
                for (uint32_t j = 0; j < 4u; ++j)
                    if ((nib >> j) & 1u) s += qq[4u * g + j];
                lut[e] = static_cast<uint16_t>(s);
            }
        }
        __syncwarp();

        // ---- seed: the entry's row into the block buffer's row slot, then
        // the same fold as for an expanded node
        {
            const uint32_t words = (DM == kU8 ? p.row_bytes : p.row_stride * 4u) / 4u;
            const uint32_t* src = DM == kU8 ? reinterpret_cast<const uint32_t*>(p.vecs8 + static_cast<size_t>(p.entry) * p.row_bytes)
                                            : reinterpret_cast<const uint32_t*>(p.vecs + static_cast<size_t>(p.entry) * p.row_stride);
            uint32_t* dst = reinterpret_cast<uint32_t*>(blk_row);
            for (uint32_t i = lane; i < words; i += 32) dst[i] = src[i];
            __syncwarp();
        }
        const float entry_d = block_exact<DM>(p, blk_row, qsm, q8, team_ok, lane);
        uint64_t beam[RX];
#pragma unroll
        for (int r = 0; r < RX; ++r) beam[r] = kEmptyKey;
        uint32_t logged = 1;
        if (lane == 0) {
            beam[0] = make_key(entry_d, p.entry);
            visit(vbits, p.entry);
            vlog[0] = p.entry;
        }
        uint32_t E = 0, D = 1, EST = 0;
        // generic accesses of the block buffer are done before the first copy
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        __syncwarp();

        for (int iter = 0; iter < p.max_iterations; ++iter) {
            uint32_t cur, nxt;
            if (!beam_pick_next<RX>(beam, lane, cur, nxt)) break;
            ++E;
            __syncwarp();   // earlier reads of the block are done

            if (lane == 0) {
                bulk_load(blk, p.rq_nb + static_cast<size_t>(cur) * p.rq_stride, p.rq_stride, mbar);
                if (nxt != kNoNode) bulk_prefetch_l2(p.rq_nb + static_cast<size_t>(nxt) * p.rq_stride, p.rq_stride);
            }
            if (!mbar_wait(mbar, phase, p.wait_polls)) {
                // wait (bounded again) for the copy in flight, leave the
                // visited bitmap clean, report, and stop this warp
                const bool landed = mbar_wait(mbar, phase, kDefaultWaitPolls);
                clear_visited(p, vbits, vlog, logged, lane);
                if (lane == 0) report_errors(p, kErrWaitTimeout | (landed ? 0u : kErrCopyPending));
                return;
            }
            phase ^= 1u;

            // test-and-set every neighbour's bit; the returned words are
            // first needed after the own-row fold and the estimates, which
            // are computed for every neighbour meanwhile
            uint32_t c[RY], old[RY];
#pragma unroll
            for (int r = 0; r < RY; ++r) {
                const uint32_t pos = static_cast<uint32_t>(r) * 32u + lane;
                c[r] = pos < deg ? blk_adj[pos] : kNoNode;
                old[r] = c[r] < p.n ? atomicOr(vbits + (c[r] >> 5), 1u << (c[r] & 31u)) : ~0u;
            }
            // exact distance of the expanded node (include/cpu_search_rabitq.hpp:130)
            const float exact = block_exact<DM>(p, blk_row, qsm, q8, team_ok, lane);
            ++D;

            float est[RY];
#pragma unroll
            for (int r = 0; r < RY; ++r) {
                // include/cpu_search_rabitq.hpp:72-97
                const uint32_t pos = static_cast<uint32_t>(r) * 32u + lane;
                est[r] = FLT_MAX;
                const float tx = pos < deg ? blk_fac[pos] : FLT_MAX;
                if (tx != FLT_MAX) {
                    const float fdq = blk_fac[deg + pos];
                    const float fvq = blk_fac[2u * deg + pos];
                    const uint32_t raw = raw_sum<EM>(blk_codes + pos * wpp, wpp, est_tab);
                    const float ip = static_cast<float>((static_cast<int32_t>(raw) << 1) - sum_q);
                    const float e = __fadd_rn(__fadd_rn(__fadd_rn(tx, exact), __fmul_rn(__fmul_rn(fdq, w), ip)),
                                              __fmul_rn(fvq, lo));
                    est[r] = isfinite(e) ? e : FLT_MAX;
                }
            }

            // the neighbours whose bit was new: log them, keep their estimates
            uint64_t k[RY];
            bool keep[RY];
            const uint64_t bound = beam_bound<RX>(beam, p.topk);
#pragma unroll
            for (int r = 0; r < RY; ++r) {
                const bool fresh = (old[r] & (1u << (c[r] & 31u))) == 0u;
                const unsigned b = __ballot_sync(kFull, fresh);
                if (fresh) {
                    const uint32_t at = logged + __popc(b & lt_mask);
                    if (at < p.vis_log_cap) vlog[at] = c[r];
                }
                logged += __popc(b);
                EST += __popc(b);
                k[r] = fresh ? make_key(est[r], c[r]) : kEmptyKey;
                keep[r] = k[r] < bound;
            }

            unsigned cnt = 0;
#pragma unroll
            for (int r = 0; r < RY; ++r) {
                const unsigned b = __ballot_sync(kFull, keep[r]);
                if (keep[r]) ckeys[cnt + __popc(b & lt_mask)] = k[r];
                cnt += __popc(b);
            }
            if (cnt) {
                __syncwarp();
                beam_merge_compact_wide<RX, RY>(beam, ckeys, cnt, lane, p.topk);
            }
        }

        // ---- exact rerank of the whole beam (include/cpu_search_rabitq.hpp:144-146);
        // the block buffer stages rows
        __syncwarp();
        uint32_t rr = 0;
#pragma unroll
        for (int r = 0; r < RX; ++r) {
            const bool v = beam[r] != kEmptyKey;
            if (v) cids[r * 32 + lane] = key_id(beam[r]);
            rr += __popc(__ballot_sync(kFull, v));                 // valid entries form a prefix
        }
        __syncwarp();
        if (rr) score_rows<DM>(p, rr, cids, cdist, qsm, q8, reinterpret_cast<float*>(blk), lane, team_ok);
#pragma unroll
        for (int r = 0; r < RX; ++r)
            if (beam[r] != kEmptyKey) beam[r] = make_key(cdist[r * 32 + lane], key_id(beam[r]));
        sort_rt<RX, 32u * RX>(beam, lane);

        uint32_t* oid = p.out_ids + static_cast<size_t>(qi) * p.K;
        float* odist = p.out_dists ? p.out_dists + static_cast<size_t>(qi) * p.K : nullptr;
#pragma unroll
        for (int r = 0; r < RX; ++r) {
            const uint32_t pos = static_cast<uint32_t>(r) * 32u + lane;
            if (pos < p.K) {
                const bool v = beam[r] != kEmptyKey;
                oid[pos] = v ? key_id(beam[r]) : kNoNode;
                if (odist) odist[pos] = v ? key_dist(beam[r]) : FLT_MAX;
            }
        }
        for (uint32_t pos = 32u * RX + lane; pos < p.K; pos += 32) {
            oid[pos] = kNoNode;
            if (odist) odist[pos] = FLT_MAX;
        }
        if (lane == 0) {
            atomicAdd(&p.counters->expansions, static_cast<unsigned long long>(E));
            atomicAdd(&p.counters->distances, static_cast<unsigned long long>(D));
            atomicAdd(&p.counters->estimates, static_cast<unsigned long long>(EST));
            atomicAdd(&p.counters->rerank, static_cast<unsigned long long>(rr));
            if (p.q_stats) {
                p.q_stats[2 * static_cast<size_t>(qi)] = E;
                p.q_stats[2 * static_cast<size_t>(qi) + 1] = D;
            }
        }
        clear_visited(p, vbits, vlog, logged, lane);
        // the block buffer is written by generic stores (query setup) next
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        __syncwarp();
    }
}

// One warp per node: [adjacency (a repeated id -> kNoNode) | codes | factors
// | own row], from the gather layout.
__global__ void k_build_rq_blocks(const SearchParams p, unsigned char* __restrict__ out) {
    const unsigned lane = threadIdx.x & 31u;
    const uint64_t warp = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = (static_cast<uint64_t>(gridDim.x) * blockDim.x) >> 5;
    const uint32_t deg = p.degree;
    const bool u8 = p.vecs8 != nullptr;
    const uint32_t row_words = (u8 ? p.row_bytes : p.row_stride * 4u) / 4u;
    for (uint64_t v = warp; v < p.n; v += nwarps) {
        unsigned char* dst = out + v * p.rq_stride;
        const uint32_t* arow = p.adj + v * deg;
        uint32_t* dadj = reinterpret_cast<uint32_t*>(dst);
        for (uint32_t i = lane; i < p.rq_off_codes / 4u; i += 32) {
            uint32_t a = kNoNode;
            if (i < deg) {
                a = arow[i];
                for (uint32_t j = 0; j < i; ++j)
                    if (arow[j] == a) { a = kNoNode; break; }
            }
            dadj[i] = a;
        }
        const uint32_t* csrc = p.codes + v * deg * p.wpp;
        uint32_t* dcodes = reinterpret_cast<uint32_t*>(dst + p.rq_off_codes);
        for (uint32_t i = lane; i < deg * p.wpp; i += 32) dcodes[i] = csrc[i];
        const float* fsrc = p.factors + v * 3u * deg;
        float* dfac = reinterpret_cast<float*>(dst + p.rq_off_fac);
        for (uint32_t i = lane; i < (p.rq_off_row - p.rq_off_fac) / 4u; i += 32) dfac[i] = i < 3u * deg ? fsrc[i] : 0.0f;
        const uint32_t* rsrc = u8 ? reinterpret_cast<const uint32_t*>(p.vecs8 + v * p.row_bytes)
                                  : reinterpret_cast<const uint32_t*>(p.vecs + v * p.row_stride);
        uint32_t* drow = reinterpret_cast<uint32_t*>(dst + p.rq_off_row);
        for (uint32_t i = lane; i < (p.rq_stride - p.rq_off_row) / 4u; i += 32) drow[i] = i < row_words ? rsrc[i] : 0u;
    }
}

using KernelFn = void (*)(SearchParams);

template <int RX, int RY, int EM>
KernelFn pick_rqnb(int dm) {
    if (dm == kSeq) return k_search_rq_nb<RX, RY, kSeq, EM>;
    if (dm == kU8) return k_search_rq_nb<RX, RY, kU8, EM>;
    return k_search_rq_nb<RX, RY, kTeam, EM>;
}

template <int EM>
KernelFn select_rqnb_em(int regx, int regy, int dm) {
    if (regy == 1) {
        switch (regx) {
            case 1: return pick_rqnb<1, 1, EM>(dm);
            case 2: return pick_rqnb<2, 1, EM>(dm);
            case 4: return pick_rqnb<4, 1, EM>(dm);
            case 8: return pick_rqnb<8, 1, EM>(dm);
            case 16: return pick_rqnb<16, 1, EM>(dm);
        }
    } else if (regy == 2) {
        switch (regx) {
            case 2: return pick_rqnb<2, 2, EM>(dm);
            case 4: return pick_rqnb<4, 2, EM>(dm);
            case 8: return pick_rqnb<8, 2, EM>(dm);
            case 16: return pick_rqnb<16, 2, EM>(dm);
        }
    }
    return nullptr;
}

KernelFn select_rqnb(const SearchParams& p, const LaunchShape& s) {
    return p.rq_lut ? select_rqnb_em<1>(s.regx, s.regy, s.dmode) : select_rqnb_em<0>(s.regx, s.regy, s.dmode);
}

uint32_t a16(uint32_t x) { return (x + 15u) & ~15u; }

cudaError_t occupancy(const SearchParams& p, const LaunchShape& shape, KernelFn& fn, int& per_sm) {
    fn = select_rqnb(p, shape);
    if (!fn) return cudaErrorInvalidValue;
    const int threads = 32 * shape.warps_per_block;
    const size_t smem = static_cast<size_t>(shape.smem_per_warp) * shape.warps_per_block;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, smem);
    if (e != cudaSuccess) return e;
    return per_sm < 1 ? cudaErrorInvalidConfiguration : cudaSuccess;
}

}  // namespace

cudaError_t plan_search_rq_nb(SearchParams& p, LaunchShape& shape, size_t max_smem_optin, char* why,
                              size_t why_len) {
    auto fail = [&](const char* msg) {
        if (why && why_len) std::snprintf(why, why_len, "%s", msg);
        return cudaErrorInvalidValue;
    };
    if (p.degree == 0 || p.degree > 64) return fail("RaBitQ blocks support graph degree 1..64");
    shape.regy = p.degree <= 32 ? 1 : 2;
    if (p.topk == 0 || p.topk > 512) return fail("topk_size must be in 1..512");
    uint32_t cap = 32;
    while (cap < p.topk) cap <<= 1;
    shape.regx = static_cast<int>(cap / 32);
    if (shape.regx < shape.regy) shape.regx = shape.regy;
    if (p.wpp == 0 || p.pdim != 32u * p.wpp) return fail("RaBitQ needs padded_dim >= 32");
    // staging for the seed and the rerank (score_rows), in the block buffer
    const uint32_t units = p.row_stride / 4u;
    p.stage_pitch = (units % 2u == 0u) ? p.row_stride + 4u : p.row_stride + 8u;
    p.stage_ring = 0;
    uint32_t buf = a16(p.rq_stride);
    buf = buf > p.pdim * 5u ? buf : a16(p.pdim * 5u);           // rotated query + quantised bytes
    if (shape.dmode == kSeq) {
        if (p.row_stride * 4u > 1024u) {
            p.stage_ring = kRingStages;
            p.stage_rows = 0;
            buf = buf > kRingFloats * 4u ? buf : kRingFloats * 4u;
        } else {
            const uint32_t row_bytes = p.stage_pitch * 4u;
            uint32_t rows = buf / row_bytes;
            if (rows < 4u) {
                rows = 4u;
                buf = a16(4u * row_bytes);
            }
            p.stage_rows = rows > 32u ? 32u : rows;
        }
    } else {
        p.stage_rows = 0;
    }
    uint32_t off = a16(p.row_stride * 4u);                          // f32 query
    p.off_q8 = off;
    if (shape.dmode == kU8) off = a16(off + p.row_bytes + 4u);
    p.off_est = off;
    off = a16(off + (p.rq_lut ? p.pdim * 8u : p.wpp * 32u));       // nibble table or bit-planes
    p.off_cids = off;                                               // the final beam's ids
    off = a16(off + 32u * static_cast<uint32_t>(shape.regx) * 4u);
    p.off_cdist = off;
    off = a16(off + 32u * static_cast<uint32_t>(shape.regx) * 4u);
    p.off_keys = off;
    off = a16(off + 32u * static_cast<uint32_t>(shape.regy) * 8u);
    p.off_mbar = off;
    off = a16(off + 8u);
    p.off_block = off;
    off = a16(off + buf);
    p.off_filter = 0;
    p.filter_words = 0;
    p.smem_per_warp = off;
    shape.smem_per_warp = off;
    if (static_cast<size_t>(off) * shape.warps_per_block > max_smem_optin)
        return fail("shared memory per block exceeds the device limit");
    return cudaSuccess;
}

cudaError_t rq_nb_capacity_warps(const SearchParams& p, const LaunchShape& shape, int num_sms, uint64_t& warps) {
    KernelFn fn;
    int per_sm = 0;
    const cudaError_t e = occupancy(p, shape, fn, per_sm);
    warps = static_cast<uint64_t>(per_sm) * static_cast<uint64_t>(num_sms) * shape.warps_per_block;
    return e;
}

cudaError_t launch_search_rq_nb(const SearchParams& p, const LaunchShape& shape, int num_sms, cudaStream_t stream) {
    KernelFn fn;
    int per_sm = 0;
    cudaError_t e = occupancy(p, shape, fn, per_sm);
    if (e != cudaSuccess) return e;
    unsigned grid = persistent_blocks(p.nq, shape.warps_per_block, per_sm, num_sms);
    const unsigned arena_blocks = p.vis_warps / static_cast<uint32_t>(shape.warps_per_block);
    if (grid > arena_blocks) grid = arena_blocks;
    if (grid == 0) return p.nq ? cudaErrorInvalidConfiguration : cudaSuccess;
    const size_t smem = static_cast<size_t>(shape.smem_per_warp) * shape.warps_per_block;
    fn<<<grid, 32 * shape.warps_per_block, smem, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t build_rabitq_blocks(const SearchParams& p, unsigned char* out, cudaStream_t stream) {
    const uint64_t blocks64 = (p.n + 7) / 8;
    const unsigned blocks = static_cast<unsigned>(blocks64 < 65535ull * 8 ? blocks64 : 65535ull * 8);
    k_build_rq_blocks<<<blocks, 256, 0, stream>>>(p, out);
    return cudaGetLastError();
}

}  // namespace bsb
