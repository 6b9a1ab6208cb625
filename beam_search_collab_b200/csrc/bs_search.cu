// bs_search.cu -- persistent warp-per-query beam search with exact L2
// distances (modes base, warp1..8, bwarp1..8).
//
// Replaces the reference kernels kernel_warp_search / kernel_base_search
// (src/gpu_cli.cu:87-119) and their visitors GPUWarpSearch::search
// (include/gpu_search_warp.cuh:123-238) and GPUBaseSearch::search
// (include/gpu_search_base.cuh:121-247), with the semantics of the reference
// CPU search CPUBaseSearch::search (include/cpu_search_base.hpp:22-82):
//
//   beam   = the topk_size best (dist, id) entries pushed so far
//   loop   : expand the smallest unexpanded entry, push every unvisited
//            neighbour with its exact distance, keep the best topk_size
//   stop   : no unexpanded entry, or max_iterations expansions
//   output : the K best entries, 0xffffffff past the end of the beam
//
// One warp owns one query at a time and pulls the next query index from a
// global counter when it finishes (persistent grid sized to the resident
// capacity of the GPU).  Per warp state: the beam (registers), the query and
// the visited filter (shared memory), and a staging area for candidate rows.
#include <cfloat>
#include <cstdio>
#include <cstring>

#include "bs_device.cuh"
#include "bs_internal.h"
#include "bs_score.cuh"

namespace bsb {

using namespace dev;

namespace {

template <int RX, int RY, int DM, int FM>
__global__ void __launch_bounds__(256) k_search_l2(const SearchParams p) {
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

    const uint32_t deg = p.degree;
    const uint32_t fmask = p.filter_slots - 1u;
    const uint32_t fshift = 32u - static_cast<uint32_t>(__popc(fmask));
    const unsigned lt_mask = (1u << lane) - 1u;
    unsigned err = 0;
    for (;;) {
        unsigned qi = 0;
        if (lane == 0) qi = atomicAdd(&p.counters->next_query, 1u);
        qi = __shfl_sync(kFull, qi, 0);
        if (qi >= p.nq) break;

        // query -> shared memory (zero pad up to the stored row width)
        const float* q = query_src(p, qi);
        for (uint32_t d = lane; d < p.row_stride; d += 32) qsm[d] = d < p.dim ? q[d] : 0.0f;
        for (uint32_t i = lane; i < p.filter_words; i += 32) filt[i] = (FM == kHash) ? kNoNode : 0u;
        if (lane == 0) cids[0] = p.entry;
        __syncwarp();
        const bool team_ok = DM != kSeq && query_integer_exact(qsm, p.dim, p.team_qlo, p.team_qhi);
        if (DM != kSeq && !team_ok && lane == 0) atomicAdd(&p.counters->team_fallbacks, 1u);
        if (DM == kU8 && team_ok) pack_query_u8(qsm, p.dim, p.row_bytes, q8, lane);

        // seed: the entry point with its exact distance
        score_rows<DM>(p, 1, cids, cdist, qsm, q8, stage, lane, team_ok);
        uint64_t beam[RX];
#pragma unroll
        for (int r = 0; r < RX; ++r) beam[r] = kEmptyKey;
        if (lane == 0) {
            beam[0] = make_key(cdist[0], p.entry);
            if (FM == kHash) hash_insert(filt, fmask, fshift, p.entry, err);
            else bloom_set(filt, fmask, p.entry);
        }
        uint32_t filled = 1;           // entries in the hash table
        uint32_t E = 0, D = 1;
        __syncwarp();

        for (int iter = 0; iter < p.max_iterations; ++iter) {
            uint32_t cur, nxt;
            if (!beam_pick_next<RX>(beam, lane, cur, nxt)) break;
            ++E;
            __syncwarp();   // previous round's cids/cdist reads are done

            uint32_t c[RY];
            bool fresh[RY];
            const uint32_t* row = p.adj + static_cast<size_t>(cur) * deg;
            // the adjacency row the next expansion reads unless a better
            // candidate turns up: start it towards L2 now
            if (lane == 0 && nxt != kNoNode)
                asm volatile("prefetch.global.L2 [%0];\n" ::"l"(p.adj + static_cast<size_t>(nxt) * deg));
#pragma unroll
            for (int r = 0; r < RY; ++r) {
                const uint32_t pos = static_cast<uint32_t>(r) * 32u + lane;
                c[r] = pos < deg ? ldg_u32(row + pos) : kNoNode;
            }

            if (FM == kHash) {
                if (filled + deg > p.filter_limit) {
                    // Forget everything but the beam.  Any node that left the
                    // beam is worse than all current entries, so seeing it
                    // again can never change the beam: results stay exact.
                    for (uint32_t i = lane; i < p.filter_words; i += 32) filt[i] = kNoNode;
                    __syncwarp();
                    uint32_t cnt = 0;
#pragma unroll
                    for (int r = 0; r < RX; ++r) {
                        const bool v = beam[r] != kEmptyKey;
                        if (v) hash_insert(filt, fmask, fshift, key_id(beam[r]), err);
                        cnt += __popc(__ballot_sync(kFull, v));
                    }
                    filled = cnt;
                    __syncwarp();
                }
#pragma unroll
                for (int r = 0; r < RY; ++r)
                    fresh[r] = c[r] < p.n && hash_insert(filt, fmask, fshift, c[r], err) != 0;
            } else {
                // Bloom: presence against the filter as it was before this
                // expansion; repeated ids in one row count once.
#pragma unroll
                for (int r = 0; r < RY; ++r) cids[static_cast<uint32_t>(r) * 32u + lane] = c[r];
                __syncwarp();
                bool valid[RY], present[RY];
#pragma unroll
                for (int r = 0; r < RY; ++r) {
                    const uint32_t pos = static_cast<uint32_t>(r) * 32u + lane;
                    bool v = c[r] < p.n;
                    for (uint32_t j = 0; j < pos && v; ++j) v = cids[j] != c[r];
                    valid[r] = v;
                    present[r] = v ? bloom_test(filt, fmask, c[r]) : true;
                }
                __syncwarp();
#pragma unroll
                for (int r = 0; r < RY; ++r) {
                    if (valid[r]) bloom_set(filt, fmask, c[r]);
                    fresh[r] = valid[r] && !present[r];
                }
                __syncwarp();
            }

            // compact the unvisited neighbours into cids[0..m)
            uint32_t m = 0;
#pragma unroll
            for (int r = 0; r < RY; ++r) {
                const unsigned b = __ballot_sync(kFull, fresh[r]);
                if (fresh[r]) cids[m + __popc(b & lt_mask)] = c[r];
                m += __popc(b);
            }
            __syncwarp();

            if (m) {
                filled += m;
                D += m;
                score_rows<DM>(p, m, cids, cdist, qsm, q8, stage, lane, team_ok);
                // candidates at or above the full beam's last key cannot enter
                // it; the others are compacted and merged (none: no merge)
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
                    // wide beams: lane stages as loops and only the beam's
                    // affected suffix merged (same result, a fraction of the
                    // code and of the stages)
                    if (RX >= 8) beam_merge_compact_wide<RX, RY>(beam, ckeys, cnt, lane, p.topk);
                    else beam_merge_compact<RX, RY>(beam, ckeys, cnt, lane, p.topk);
                }
            }

            if (FM == kBloom && p.reset_interval > 0 && (iter + 1) % p.reset_interval == 0) {
                // include/gpu_search_warp.cuh:171-178: forget, re-add the beam
                __syncwarp();
                for (uint32_t i = lane; i < p.filter_words; i += 32) filt[i] = 0u;
                __syncwarp();
#pragma unroll
                for (int r = 0; r < RX; ++r)
                    if (beam[r] != kEmptyKey) bloom_set(filt, fmask, key_id(beam[r]));
                __syncwarp();
            }
        }

        // the K best, 0xffffffff / FLT_MAX past the end of the beam
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
KernelFn pick_l2(int dm, int fm) {
    if (dm == kSeq) return fm == kHash ? k_search_l2<RX, RY, kSeq, kHash> : k_search_l2<RX, RY, kSeq, kBloom>;
    if (dm == kU8) return fm == kHash ? k_search_l2<RX, RY, kU8, kHash> : k_search_l2<RX, RY, kU8, kBloom>;
    return fm == kHash ? k_search_l2<RX, RY, kTeam, kHash> : k_search_l2<RX, RY, kTeam, kBloom>;
}

KernelFn select_l2(int regx, int regy, int dm, int fm) {
    if (regy == 1) {
        switch (regx) {
            case 1: return pick_l2<1, 1>(dm, fm);
            case 2: return pick_l2<2, 1>(dm, fm);
            case 4: return pick_l2<4, 1>(dm, fm);
            case 8: return pick_l2<8, 1>(dm, fm);
            case 16: return pick_l2<16, 1>(dm, fm);
        }
    } else if (regy == 2) {
        switch (regx) {
            case 2: return pick_l2<2, 2>(dm, fm);
            case 4: return pick_l2<4, 2>(dm, fm);
            case 8: return pick_l2<8, 2>(dm, fm);
            case 16: return pick_l2<16, 2>(dm, fm);
        }
    }
    return nullptr;
}

inline uint32_t pow2_at_least(uint64_t v) {
    uint64_t p = 1;
    while (p < v) p <<= 1;
    return static_cast<uint32_t>(p);
}
inline uint32_t align16(uint32_t v) { return (v + 15u) & ~15u; }

}  // namespace

cudaError_t plan_search(SearchParams& p, LaunchShape& shape, size_t max_smem_optin, char* why,
                        size_t why_len) {
    auto fail = [&](const char* msg) {
        if (why && why_len) std::snprintf(why, why_len, "%s", msg);
        return cudaErrorInvalidValue;
    };
    if (p.degree == 0) return fail("graph degree is zero");
    if (p.degree <= 32) shape.regy = 1;
    else if (p.degree <= 64) shape.regy = 2;
    else return fail("graph degree above 64 is not supported by this build");
    if (p.topk == 0) return fail("topk_size must be positive");
    if (p.topk > 512) return fail("topk_size above 512 is not supported by this build");
    const uint32_t cap = pow2_at_least(p.topk < 32 ? 32 : p.topk);
    shape.regx = static_cast<int>(cap / 32);
    if (shape.regx < shape.regy) shape.regx = shape.regy;

    // visited filter
    if (p.codes != nullptr) {
        // RaBitQ: exact, never-reset set -- a shared-memory table of
        // filter_capacity slots (<= 3/4 load) that spills into a per-warp
        // global table sized for every insert max_iterations expansions make.
        const uint64_t need = (static_cast<uint64_t>(p.topk) + 2ull * p.degree) * 4ull / 3ull + 1;
        const uint32_t slots = pow2_at_least(p.filter_slots > need ? p.filter_slots : need);
        p.filter_slots = slots;
        p.filter_limit = slots / 4u * 3u;
        p.filter_words = slots;
        const uint64_t inserts = 1ull + static_cast<uint64_t>(p.max_iterations > 0 ? p.max_iterations : 0) * p.degree;
        uint64_t gs = pow2_at_least(inserts * 4ull / 3ull + 1ull);
        if (gs < 1024u) gs = 1024u;
        if (gs > 65536u) gs = 65536u;
        p.spill_slots = static_cast<uint32_t>(gs);
    } else if (shape.fmode == kHash) {
        // Room for the beam plus several rows between resets, at <= 3/4 load.
        const uint64_t need = (static_cast<uint64_t>(p.topk) + 4ull * p.degree) * 4ull / 3ull + 1;
        // With neighbourhood blocks the table only holds ids that passed
        // into the beam, so it is sized to the beam instead of
        // filter_capacity (more resident warps).
#ifndef BS_NB_TABLE_FACTOR
#define BS_NB_TABLE_FACTOR 4     // block-layout table: slots >= factor * (topk + degree)
#endif
#ifndef BS_NB_TABLE_LOAD
#define BS_NB_TABLE_LOAD 4       // ... rebuilt from the beam at 1/load of its slots
#endif
        const uint64_t want = p.nb != nullptr ? BS_NB_TABLE_FACTOR * (static_cast<uint64_t>(p.topk) + p.degree)
                                              : (p.filter_slots > need ? p.filter_slots : need);
        const uint32_t slots = pow2_at_least(want);
        p.filter_slots = slots < 64 ? 64 : slots;
        p.filter_limit = p.nb != nullptr ? p.filter_slots / BS_NB_TABLE_LOAD : p.filter_slots / 4u * 3u;
        p.filter_words = p.filter_slots;
    } else {
        const uint32_t bits = pow2_at_least(p.filter_slots < 32 ? 32 : p.filter_slots);
        p.filter_slots = bits;
        p.filter_limit = 0;
        p.filter_words = bits / 32u;
    }

    // stored rows are padded to a multiple of 4 floats; staged rows get an
    // odd number of 16-byte units per pitch so that 8 lanes reading 16 bytes
    // at the same offset of 8 different rows hit 8 different bank groups.
    const uint32_t units = p.row_stride / 4u;
    p.stage_pitch = (units % 2u == 0u) ? p.row_stride + 4u : p.row_stride + 8u;
    const uint32_t cand = 32u * static_cast<uint32_t>(shape.regy);

    const bool blocks = p.nb != nullptr && p.codes == nullptr;
    // the f32 query (the block kernel keeps it in global memory for byte rows)
    uint32_t off = (blocks && shape.dmode == kU8) ? 0u : align16(p.row_stride * 4u);
    p.off_q8 = off;
    if (shape.dmode == kU8) off = align16(off + p.row_bytes + 4u);   // bytes + sum q^2
    p.off_filter = off;
    off = align16(off + p.filter_words * 4u);
    if (!blocks) {
        p.off_cids = off;
        off = align16(off + cand * 4u);
        p.off_cdist = off;
        off = align16(off + cand * 4u);
    }
    p.off_keys = off;
    off = align16(off + cand * 8u);
    if (p.codes != nullptr) {
        // RaBitQ: rotated query and the 7 bit-planes sit right below the
        // staging area (the kernel addresses them from off_stage down).
        if (p.wpp == 0 || p.pdim != 32u * p.wpp) return fail("RaBitQ needs padded_dim >= 32");
        off = align16(off + p.pdim * 4u + 7u * p.wpp * 4u);
    }
    p.off_stage = off;
    if (blocks) {
        // neighbourhood blocks: the mbarrier and one block copy replace the
        // staging area; the entry's id and distance (the only users of
        // cids/cdist) sit in the block buffer before its first copy
        p.off_mbar = off;
        off = align16(off + 8u);
        p.off_block = off;
        p.off_cids = off;
        p.off_cdist = off + 16u;
        off = align16(off + (p.nb_stride > 32u ? p.nb_stride : 32u));
        p.stage_rows = 0;
    } else if (shape.dmode == kSeq) {
        const uint32_t row_bytes = p.stage_pitch * 4u;
        // up to 32 rows per round, within ~48 KB per warp
        uint32_t rows = (48u * 1024u) / row_bytes;
        if (rows > 32u) rows = 32u;
        // RaBitQ stages one parent row per expansion and the final rerank
        // only: a few rows leave the shared memory to resident warps (C3:
        // 3 -> 4 blocks of 4 warps per SM, +4% queries/s)
        if (p.codes != nullptr && rows > 8u) rows = 8u;
        if (rows > cand) rows = cand;
        if (rows < 1u) rows = 1u;
        p.stage_rows = rows;
        p.stage_ring = 0;
        if (p.codes == nullptr && row_bytes > 1024u) {
            // wide rows (C4: 3.84 KB): whole-row staging held 12 rows per warp
            // (one 4-warp block per SM, 12 of 32 lanes folding); a ring of row
            // chunks keeps all 32 lanes folding in 18 KB per warp
            // tens of KB per warp: one warp per block, so that the SM's shared
            // memory holds as many warps (queries) as fit, not whole blocks.
            // Ring depth: the deepest of 4/5/6/8 chunks at which the launch's
            // queries still all fit on the SMs at once (a second wave would
            // cost more than the extra bytes in flight gain); 4 when they do
            // not fit anyway.
            shape.warps_per_block = 1;
            p.stage_ring = dev::kRingStages;
            p.stage_rows = 0;
            if (p.sm_count > 0 && p.nq > 0) {
                constexpr uint64_t kSmemPerSm = 233472;   // B200: 228 KB per SM, 1 KB reserved per block
                const uint64_t per_sm = (static_cast<uint64_t>(p.nq) + p.sm_count - 1) / p.sm_count;
                const uint32_t depths[3] = {8u, 6u, 5u};
                for (uint32_t s : depths) {
                    const uint64_t need = align16(off + s * dev::kRingStageFloats * 4u) + 1024u;
                    if (need <= max_smem_optin + 1024u && per_sm <= 32u && per_sm * need <= kSmemPerSm) {
                        p.stage_ring = s;
                        break;
                    }
                }
            }
            off = align16(off + p.stage_ring * dev::kRingStageFloats * 4u);
        } else {
            off = align16(off + rows * row_bytes);
        }
    } else {
        p.stage_rows = 0;
    }
    p.smem_per_warp = off;
    shape.smem_per_warp = off;
    const size_t total = static_cast<size_t>(off) * static_cast<size_t>(shape.warps_per_block);
    if (total > max_smem_optin) return fail("shared memory per block exceeds the device limit");
    return cudaSuccess;
}

cudaError_t launch_search(const SearchParams& p, const LaunchShape& shape, int num_sms,
                          cudaStream_t stream) {
    KernelFn fn = select_l2(shape.regx, shape.regy, shape.dmode, shape.fmode);
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
    const unsigned grid = persistent_blocks(p.nq, shape.warps_per_block, per_sm, num_sms);
    if (grid == 0) return cudaSuccess;
    fn<<<grid, threads, smem, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace bsb
