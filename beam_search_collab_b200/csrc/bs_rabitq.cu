// bs_rabitq.cu -- persistent warp-per-query RaBitQ beam search (mode rabitq).
//
// Replaces kernel_rabitq_search (src/gpu_cli.cu:121-136) and its visitor
// GPURabitqSearch::search (include/gpu_search_rabitq.cuh:191-340) with the
// semantics of the reference CPU search CPURabitqSearch::search
// (include/cpu_search_rabitq.hpp:28-150):
//
//   query   : q*signs, Walsh-Hadamard transform over padded_dim, 6-bit
//             quantisation q_d = lroundf((x - low) * (1/w) + 0.5), w=(high-low)/63
//   seed    : the entry point with its exact L2 distance
//   expand  : the smallest unexpanded entry p; exact L2 of p; every unvisited
//             neighbour i (visited marked when pushed) gets the estimate
//             tx_i + exact_p + fdq_i*w*ip + fvq_i*low,
//             ip = 2*sum_{d: bit_d(i)=1} q_d - sum_d q_d   (integer part exact)
//   finish  : exact L2 for every beam entry, re-sort by (dist, id), K best.
//
// The integer part uses the query's quantised values as 7 bit-planes
// (q_d <= 64) held in shared memory: raw = sum_b popc(plane_b & code) << b,
// i.e. an AND/POPC per 32 dimensions and bit, accumulated in integers.
// Per expansion every load (adjacency row, codes, factors, parent vector)
// depends only on the expanded node, so all of them are in flight together.
#include <cfloat>
#include <cstdio>

#include "bs_device.cuh"
#include "bs_internal.h"
#include "bs_score.cuh"

namespace bsb {

using namespace dev;

namespace {

constexpr int kPlanes = 7;   // quantised query values are 1..64

template <int RX, int RY, int DM>
__global__ void __launch_bounds__(128, (RX <= 8 ? 5 : 2)) k_search_rabitq(const SearchParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const unsigned lane = threadIdx.x & 31u;
    unsigned char* ws = smem_raw + static_cast<size_t>(threadIdx.x >> 5) * p.smem_per_warp;
    float* qsm = reinterpret_cast<float*>(ws);
    uint32_t* filt = reinterpret_cast<uint32_t*>(ws + p.off_filter);
    uint32_t* cids = reinterpret_cast<uint32_t*>(ws + p.off_cids);
    float* cdist = reinterpret_cast<float*>(ws + p.off_cdist);
    float* stage = reinterpret_cast<float*>(ws + p.off_stage);
    uint32_t* q8 = reinterpret_cast<uint32_t*>(ws + p.off_q8);
    uint64_t* ckeys = reinterpret_cast<uint64_t*>(ws + p.off_keys);
    // rotated query (pdim floats) and bit-planes (kPlanes * wpp words) follow
    // the candidate arrays; the host reserves them in off_stage's front.
    float* qrot = reinterpret_cast<float*>(ws + p.off_stage - p.pdim * 4u - kPlanes * p.wpp * 4u);
    uint32_t* planes = reinterpret_cast<uint32_t*>(ws + p.off_stage - kPlanes * p.wpp * 4u);

    const uint32_t deg = p.degree;
    const uint32_t wpp = p.wpp;
    const uint32_t pdim = p.pdim;
    const uint32_t fmask = p.filter_slots - 1u;
    const uint32_t fshift = 32u - static_cast<uint32_t>(__popc(fmask));
    const unsigned lt_mask = (1u << lane) - 1u;
    unsigned err = 0;
    const size_t gwarp = static_cast<size_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    uint32_t* gtab = p.spill + gwarp * p.spill_slots;
    const uint32_t gmask = p.spill_slots - 1u;
    const uint32_t gshift = 32u - static_cast<uint32_t>(__popc(gmask));

    for (;;) {
        unsigned qi = 0;
        if (lane == 0) qi = atomicAdd(&p.counters->next_query, 1u);
        qi = __shfl_sync(kFull, qi, 0);
        if (qi >= p.nq) break;

        const float* q = query_src(p, qi);
        for (uint32_t d = lane; d < p.row_stride; d += 32) qsm[d] = d < p.dim ? q[d] : 0.0f;
        for (uint32_t i = lane; i < p.filter_words; i += 32) filt[i] = kNoNode;
        __syncwarp();
        const bool team_ok = DM != kSeq && query_integer_exact(qsm, p.dim, p.team_qlo, p.team_qhi);
        if (DM != kSeq && !team_ok && lane == 0) atomicAdd(&p.counters->team_fallbacks, 1u);
        if (DM == kU8 && team_ok) pack_query_u8(qsm, p.dim, p.row_bytes, q8, lane);

        // ---- rotate + quantise (include/cpu_search_rabitq.hpp:34-57)
        for (uint32_t d = lane; d < pdim; d += 32)
            qrot[d] = d < p.dim ? __fmul_rn(qsm[d], __ldg(p.signs + d)) : 0.0f;
        __syncwarp();
        for (uint32_t len = 1; len < pdim; len <<= 1) {
            for (uint32_t pi = lane; pi < (pdim >> 1); pi += 32) {
                const uint32_t blk = pi / len, j = pi - blk * len;
                const uint32_t i1 = blk * (len << 1) + j, i2 = i1 + len;
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
#pragma unroll
            for (int b = 0; b < kPlanes; ++b) {
                const unsigned word = __ballot_sync(kFull, (v >> b) & 1u);
                if (lane == 0) planes[b * wpp + wd] = word;
            }
        }
        for (int o = 16; o > 0; o >>= 1) sum_q += __shfl_xor_sync(kFull, sum_q, o);
        if (lane == 0) cids[0] = p.entry;
        __syncwarp();

        // ---- seed
        score_rows<DM>(p, 1, cids, cdist, qsm, q8, stage, lane, team_ok);
        uint64_t beam[RX];
#pragma unroll
        for (int r = 0; r < RX; ++r) beam[r] = kEmptyKey;
        if (lane == 0) {
            beam[0] = make_key(cdist[0], p.entry);
            hash_insert(filt, fmask, fshift, p.entry, err);
        }
        uint32_t filled = 1, gfilled = 0;
        bool spilled = false;
        uint32_t E = 0, D = 1, EST = 0;
        __syncwarp();

        for (int iter = 0; iter < p.max_iterations; ++iter) {
            uint32_t cur;
            if (!beam_pick<RX>(beam, lane, cur)) break;
            ++E;
            __syncwarp();

            // every load below depends only on `cur`
            if (DM == kSeq) {
                const float* src = p.vecs + static_cast<size_t>(cur) * p.row_stride;
                for (uint32_t ch = lane; ch < (p.row_stride >> 2); ch += 32)
                    cp_async16(stage + ch * 4, src + ch * 4);
                asm volatile("cp.async.commit_group;\n" ::: "memory");
            }
            uint32_t c[RY];
            float tx[RY], fdq[RY], fvq[RY];
            // codes of up to 128 padded dimensions ride along with the
            // adjacency row (one round trip per expansion); wider codes are
            // read after the visited test
            uint4 code4[RY];
            const bool code_early = wpp <= 4u;
            const uint32_t* row = p.adj + static_cast<size_t>(cur) * deg;
            const float* fac = p.factors + static_cast<size_t>(cur) * 3u * deg;
#pragma unroll
            for (int r = 0; r < RY; ++r) {
                const uint32_t pos = static_cast<uint32_t>(r) * 32u + lane;
                const bool in = pos < deg;
                c[r] = in ? ldg_u32(row + pos) : kNoNode;
                tx[r] = in ? __ldg(fac + pos) : FLT_MAX;
                fdq[r] = in ? __ldg(fac + deg + pos) : 0.0f;
                fvq[r] = in ? __ldg(fac + 2 * deg + pos) : 0.0f;
                code4[r] = make_uint4(0u, 0u, 0u, 0u);
                if (in && code_early) {
                    const uint32_t* code = p.codes + (static_cast<size_t>(cur) * deg + pos) * wpp;
                    code4[r].x = ldg_u32(code);
                    if (wpp > 1u) code4[r].y = ldg_u32(code + 1);
                    if (wpp > 2u) code4[r].z = ldg_u32(code + 2);
                    if (wpp > 3u) code4[r].w = ldg_u32(code + 3);
                }
            }

            // exact distance of the expanded node (include/cpu_search_rabitq.hpp:130)
            float exact;
            if (DM == kSeq) {
                asm volatile("cp.async.wait_group 0;\n" ::: "memory");
                __syncwarp();
                float e0 = 0.0f;
                if (lane == 0) e0 = l2_seq(qsm, stage, p.dim);
                exact = __shfl_sync(kFull, e0, 0);
            } else {
                if (lane == 0) cids[0] = cur;
                __syncwarp();
                score_rows<DM>(p, 1, cids, cdist, qsm, q8, stage, lane, team_ok);
                exact = cdist[0];
                __syncwarp();   // cids/cdist are rewritten by the compaction below
            }
            ++D;

            // visited set: marked when pushed and never forgotten
            // (include/cpu_search_rabitq.hpp:131-135).  An estimate depends on
            // the parent, so a forgotten node could come back with a smaller
            // value; the set is therefore exact: the shared-memory table
            // first, then this warp's table in global memory once it is full.
            if (!spilled && filled + deg > p.filter_limit) {
                spilled = true;
                for (uint32_t i = lane; i < p.spill_slots; i += 32) gtab[i] = kNoNode;
                __syncwarp();
            }
            if (spilled && gfilled + deg > (p.spill_slots / 4u) * 3u) err |= kErrSpillFull;
            bool fresh[RY];
            float est[RY];
#pragma unroll
            for (int r = 0; r < RY; ++r) {
                if (!spilled)
                    fresh[r] = c[r] < p.n && hash_insert(filt, fmask, fshift, c[r], err) != 0;
                else
                    fresh[r] = c[r] < p.n && !hash_contains(filt, fmask, fshift, c[r]) &&
                               hash_insert(gtab, gmask, gshift, c[r], err) != 0;
                est[r] = FLT_MAX;
                if (fresh[r] && tx[r] != FLT_MAX) {
                    // include/cpu_search_rabitq.hpp:72-97
                    const uint32_t pos = static_cast<uint32_t>(r) * 32u + lane;
                    const uint32_t* code = p.codes + (static_cast<size_t>(cur) * deg + pos) * wpp;
                    uint32_t raw = 0;
                    for (uint32_t wd = 0; wd < wpp; ++wd) {
                        uint32_t cw;
                        if (code_early)
                            cw = wd == 0 ? code4[r].x : wd == 1 ? code4[r].y : wd == 2 ? code4[r].z : code4[r].w;
                        else
                            cw = ldg_u32(code + wd);
#pragma unroll
                        for (int b = 0; b < kPlanes; ++b)
                            raw += static_cast<uint32_t>(__popc(planes[b * wpp + wd] & cw)) << b;
                    }
                    const float ip = static_cast<float>((static_cast<int32_t>(raw) << 1) - sum_q);
                    const float e = __fadd_rn(__fadd_rn(__fadd_rn(tx[r], exact),
                                                        __fmul_rn(__fmul_rn(fdq[r], w), ip)),
                                              __fmul_rn(fvq[r], lo));
                    est[r] = isfinite(e) ? e : FLT_MAX;
                }
            }

            uint32_t m = 0;
#pragma unroll
            for (int r = 0; r < RY; ++r) {
                const unsigned b = __ballot_sync(kFull, fresh[r]);
                if (fresh[r]) {
                    const uint32_t at = m + __popc(b & lt_mask);
                    cids[at] = c[r];
                    cdist[at] = est[r];
                }
                m += __popc(b);
            }
            __syncwarp();
            if (m) {
                if (spilled) gfilled += m; else filled += m;
                EST += m;
                const uint64_t bound = beam_bound<RX>(beam, p.topk);
                unsigned cnt = 0;
#pragma unroll
                for (int r = 0; r < RY; ++r) {
                    const uint32_t s = static_cast<uint32_t>(r) * 32u + lane;
                    const uint64_t k = s < m ? make_key(cdist[s], cids[s]) : kEmptyKey;
                    const bool keep = k < bound;
                    const unsigned b = __ballot_sync(kFull, keep);
                    if (keep) ckeys[cnt + __popc(b & lt_mask)] = k;
                    cnt += __popc(b);
                }
                if (cnt) {
                    __syncwarp();
                    beam_merge_compact<RX, RY>(beam, ckeys, cnt, lane, p.topk);
                }
            }
        }

        // ---- exact rerank of the whole beam (include/cpu_search_rabitq.hpp:144-146)
        uint32_t rr = 0;
#pragma unroll
        for (int r = 0; r < RX; ++r) {
            const bool v = beam[r] != kEmptyKey;
            const uint32_t cnt = __popc(__ballot_sync(kFull, v));   // valid entries form a prefix
            if (cnt) {
                __syncwarp();
                if (v) cids[lane] = key_id(beam[r]);
                __syncwarp();
                score_rows<DM>(p, cnt, cids, cdist, qsm, q8, stage, lane, team_ok);
                if (v) beam[r] = make_key(cdist[lane], key_id(beam[r]));
                rr += cnt;
            }
        }
        sort_asc<RX>(beam, lane);

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
        __syncwarp();
    }
    if (lane == 0 && err) report_errors(p, err);
}

using KernelFn = void (*)(SearchParams);

template <int RX, int RY>
KernelFn pick_rq(int dm) {
    if (dm == kSeq) return k_search_rabitq<RX, RY, kSeq>;
    if (dm == kU8) return k_search_rabitq<RX, RY, kU8>;
    return k_search_rabitq<RX, RY, kTeam>;
}

KernelFn select_rq(int regx, int regy, int dm) {
    if (regy == 1) {
        switch (regx) {
            case 1: return pick_rq<1, 1>(dm);
            case 2: return pick_rq<2, 1>(dm);
            case 4: return pick_rq<4, 1>(dm);
            case 8: return pick_rq<8, 1>(dm);
            case 16: return pick_rq<16, 1>(dm);
        }
    } else if (regy == 2) {
        switch (regx) {
            case 2: return pick_rq<2, 2>(dm);
            case 4: return pick_rq<4, 2>(dm);
            case 8: return pick_rq<8, 2>(dm);
            case 16: return pick_rq<16, 2>(dm);
        }
    }
    return nullptr;
}

// Persistent grid: at most the resident capacity, at least one warp per query.
cudaError_t rabitq_grid(const SearchParams& p, const LaunchShape& shape, int num_sms, KernelFn& fn,
                        unsigned& grid) {
    fn = select_rq(shape.regx, shape.regy, shape.dmode);
    if (!fn) return cudaErrorInvalidValue;
    const int threads = 32 * shape.warps_per_block;
    const size_t smem = static_cast<size_t>(shape.smem_per_warp) * shape.warps_per_block;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    grid = persistent_blocks(p.nq, shape.warps_per_block, per_sm, num_sms);
    return cudaSuccess;
}

}  // namespace

cudaError_t rabitq_grid_warps(const SearchParams& p, const LaunchShape& shape, int num_sms,
                              uint64_t& warps) {
    KernelFn fn;
    unsigned grid = 0;
    const cudaError_t e = rabitq_grid(p, shape, num_sms, fn, grid);
    warps = static_cast<uint64_t>(grid) * shape.warps_per_block;
    return e;
}

cudaError_t launch_search_rabitq(const SearchParams& p, const LaunchShape& shape, int num_sms,
                                 cudaStream_t stream) {
    KernelFn fn;
    unsigned grid = 0;
    const cudaError_t e = rabitq_grid(p, shape, num_sms, fn, grid);
    if (e != cudaSuccess) return e;
    if (grid == 0) return cudaSuccess;
    const size_t smem = static_cast<size_t>(shape.smem_per_warp) * shape.warps_per_block;
    fn<<<grid, 32 * shape.warps_per_block, smem, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace bsb
