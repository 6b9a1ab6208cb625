// bs_search_nb.cu -- the exact L2 beam search (modes base, warp1..8,
// bwarp1..8) over neighbourhood blocks.
//
// Same results as bs_search.cu (the reference CPU search,
// include/cpu_search_base.hpp:22-82); the memory path and the order of the
// work differ.  The gather layout needs two dependent round trips per
// expansion -- the node's adjacency row, then the rows of its unvisited
// neighbours.  Here every node owns one contiguous block in HBM:
//
//     [ adjacency row (degree u32, padded to 16 B) | row of neighbour 0 | ... ]
//
// so an expansion is ONE bulk copy (cp.async.bulk global->shared, completion
// counted on a per-warp mbarrier) of the expanded node's block.  With every
// neighbour row already in shared memory, lane i scores row i outright, and
// the exact visited set is consulted only by the candidates whose key beats
// the beam's T-th key:
//
//   * a node seen before that is not in the beam has a key at or above the
//     current T-th key -- it left the beam, or never entered it, while T
//     better keys were present, and the T-th key never rises -- so the
//     bound drops it, as the reference's visited set would;
//   * a candidate below the bound that was seen before is therefore in the
//     beam, and the table (every id that ever passed into the beam; rebuilt
//     from the beam when full) finds it.
//
// The Bloom modes keep the reference's filter in front of the merge (its
// false positives skip nodes).  Repeated ids inside one adjacency row are
// replaced by "no node" when the blocks are built: the reference skips a
// repeat because the first occurrence marked it visited.
//
// The blocks trade capacity for latency (C2: 4.2 KB per node, 4.2 GB for 1M
// nodes); the host builds them only when they fit the device comfortably.
#include <cfloat>
#include <cstdio>

#include "bs_device.cuh"
#include "bs_internal.h"
#include "bs_score.cuh"
#include "bs_bulk.cuh"
#include "bs_nb.cuh"

namespace bsb {

using namespace dev;

namespace {

template <int RX, int RY, int DM, int FM>
#ifdef BS_NB_MAXNREG
__global__ void __maxnreg__(BS_NB_MAXNREG) k_search_nb(const SearchParams p) {
#else
__global__ void __launch_bounds__(256) k_search_nb(const SearchParams p) {
#endif
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const unsigned lane = threadIdx.x & 31u;
    unsigned char* ws = smem_raw + static_cast<size_t>(threadIdx.x >> 5) * p.smem_per_warp;
    float* qsm = reinterpret_cast<float*>(ws);
    uint32_t* q8 = reinterpret_cast<uint32_t*>(ws + p.off_q8);
    const unsigned char* qb = ws + p.off_q8;
    uint32_t* filt = reinterpret_cast<uint32_t*>(ws + p.off_filter);
    uint32_t* cids = reinterpret_cast<uint32_t*>(ws + p.off_cids);
    float* cdist = reinterpret_cast<float*>(ws + p.off_cdist);
    uint64_t* ckeys = reinterpret_cast<uint64_t*>(ws + p.off_keys);
    uint64_t* mbar = reinterpret_cast<uint64_t*>(ws + p.off_mbar);
    unsigned char* blk = ws + p.off_block;
    const uint32_t* blk_adj = reinterpret_cast<const uint32_t*>(blk);
    const unsigned char* blk_rows = blk + p.nb_adj_bytes;

    const uint32_t deg = p.degree;
    const uint32_t fmask = p.filter_slots - 1u;
    const uint32_t fshift = 32u - static_cast<uint32_t>(__popc(fmask));
    const unsigned lt_mask = (1u << lane) - 1u;
    unsigned err = 0;
    unsigned phase = 0;
    if (lane == 0) mbar_init(mbar);
    __syncwarp();

    for (;;) {
        unsigned qi = 0;
        if (lane == 0) qi = atomicAdd(&p.counters->next_query, 1u);
        qi = __shfl_sync(kFull, qi, 0);
        if (qi >= p.nq) break;

        // byte rows read the f32 query from global memory (packing, and the
        // rare sequential fallback); the others keep it in shared memory
        const float* q = query_src(p, qi);
        if (DM == kU8 && p.queries_src != nullptr) {
            // read over the bus once, into this query's device slot
            float* slot = const_cast<float*>(p.queries) + static_cast<size_t>(qi) * p.dim;
            copy_query_row(slot, q, p.dim, lane, 32u);
            __syncwarp();
            q = slot;
        }
        const float* qv = DM == kU8 ? q : qsm;
        if (DM != kU8)
            for (uint32_t d = lane; d < p.row_stride; d += 32) qsm[d] = d < p.dim ? q[d] : 0.0f;
        for (uint32_t i = lane; i < p.filter_words; i += 32) filt[i] = (FM == kHash) ? kNoNode : 0u;
        if (lane == 0) cids[0] = p.entry;
        __syncwarp();
        const bool team_ok = DM != kSeq && query_integer_exact(qv, p.dim, p.team_qlo, p.team_qhi);
        if (DM != kSeq && !team_ok && lane == 0) atomicAdd(&p.counters->team_fallbacks, 1u);
        if (DM == kU8 && team_ok) pack_query_u8(qv, p.dim, p.row_bytes, q8, lane);
        const uint32_t qq = (DM == kU8 && team_ok) ? q8[p.row_bytes / 4u] : 0u;

        score_direct<DM>(p, 1, cids, cdist, qv, q8, lane, team_ok);
        uint64_t beam[RX];
#pragma unroll
        for (int r = 0; r < RX; ++r) beam[r] = kEmptyKey;
        if (lane == 0) {
            beam[0] = make_key(cdist[0], p.entry);
            if (FM == kHash) hash_insert(filt, fmask, fshift, p.entry, err);
            else bloom_set(filt, fmask, p.entry);
        }
        uint32_t filled = 1;
        uint32_t E = 0, D = 1;
        // cids/cdist of the entry live in the block buffer: order these
        // generic accesses before the first bulk copy overwrites them
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        __syncwarp();

        for (int iter = 0; iter < p.max_iterations; ++iter) {
            uint32_t cur, nxt;
            if (!beam_pick_next<RX>(beam, lane, cur, nxt)) break;
            ++E;
            __syncwarp();   // earlier reads of the block and of ckeys are done

            if (lane == 0) {
                bulk_load(blk, p.nb + static_cast<size_t>(cur) * p.nb_stride, p.nb_stride, mbar);
                // the block the next expansion takes unless a better
                // candidate turns up: start it towards L2 now
                if (nxt != kNoNode) bulk_prefetch_l2(p.nb + static_cast<size_t>(nxt) * p.nb_stride, p.nb_stride);
            }
            if (!mbar_wait(mbar, phase, p.wait_polls)) {
                // wait (bounded again) for the copy in flight to land before
                // leaving, so that no copy outlives the warp; the host reads
                // the flag and reports BS_ERR_KERNEL
                const bool landed = mbar_wait(mbar, phase, kDefaultWaitPolls);
                if (lane == 0) report_errors(p, err | kErrWaitTimeout | (landed ? 0u : kErrCopyPending));
                return;
            }
            phase ^= 1u;

            uint32_t c[RY];
            bool live[RY];
#pragma unroll
            for (int r = 0; r < RY; ++r) {
                const uint32_t pos = static_cast<uint32_t>(r) * 32u + lane;
                c[r] = pos < deg ? blk_adj[pos] : kNoNode;
                live[r] = c[r] < p.n;
            }
            if (FM == kBloom) {
                // reference order: every child tested against the filter as it
                // was before this expansion, then every child set
                bool present[RY];
#pragma unroll
                for (int r = 0; r < RY; ++r) present[r] = live[r] && bloom_test(filt, fmask, c[r]);
                __syncwarp();
#pragma unroll
                for (int r = 0; r < RY; ++r) {
                    if (live[r]) bloom_set(filt, fmask, c[r]);
                    live[r] = live[r] && !present[r];
                }
            }

            // one row per lane, straight from the block
            uint64_t k[RY];
            bool keep[RY];
            const uint64_t bound = beam_bound<RX>(beam, p.topk);
            uint32_t nkeep = 0;
#pragma unroll
            for (int r = 0; r < RY; ++r) {
                float d = 0.0f;
                if (live[r])
                    d = block_row_dist<DM>(p, blk_rows, static_cast<uint32_t>(r) * 32u + lane, qv, qb, qq, team_ok);
                k[r] = live[r] ? make_key(d, c[r]) : kEmptyKey;
                D += __popc(__ballot_sync(kFull, live[r]));
                keep[r] = k[r] < bound;
                nkeep += __popc(__ballot_sync(kFull, keep[r]));
            }

            if (FM == kHash && nkeep) {
                if (filled + nkeep > p.filter_limit) {
                    // keep only the beam's ids: every other id seen so far is
                    // at or above the bound for good
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
                    if (keep[r]) keep[r] = hash_insert(filt, fmask, fshift, c[r], err) != 0;
            }

            unsigned cnt = 0;
#pragma unroll
            for (int r = 0; r < RY; ++r) {
                const unsigned b = __ballot_sync(kFull, keep[r]);
                if (keep[r]) ckeys[cnt + __popc(b & lt_mask)] = k[r];
                cnt += __popc(b);
            }
            if (cnt) {
                filled += cnt;
                __syncwarp();
                if (RX >= 8) beam_merge_compact_wide<RX, RY>(beam, ckeys, cnt, lane, p.topk);
                else beam_merge_compact<RX, RY>(beam, ckeys, cnt, lane, p.topk);
            }

            if (FM == kBloom && p.reset_interval > 0 && (iter + 1) % p.reset_interval == 0) {
                __syncwarp();
                for (uint32_t i = lane; i < p.filter_words; i += 32) filt[i] = 0u;
                __syncwarp();
#pragma unroll
                for (int r = 0; r < RX; ++r)
                    if (beam[r] != kEmptyKey) bloom_set(filt, fmask, key_id(beam[r]));
                __syncwarp();
            }
        }

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

// One warp per node: the node's adjacency row (a repeated id replaced by
// kNoNode), then each neighbour's row (zeros for an id outside the graph),
// 16 bytes per lane per step; u8 rows with their chunks rotated
// (nb_chunk_pos).  Degree <= 64.
__global__ void k_build_nb(const SearchParams p, unsigned char* __restrict__ out) {
    const unsigned lane = threadIdx.x & 31u;
    const uint64_t warp = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = (static_cast<uint64_t>(gridDim.x) * blockDim.x) >> 5;
    const bool u8 = p.vecs8 != nullptr;
    const uint32_t src_bytes = u8 ? p.row_bytes : p.row_stride * 4u;
    const uint32_t nch = src_bytes / 16u;
    const uint32_t chunks = p.nb_pitch / 16u;
    const uint32_t deg = p.degree;
    for (uint64_t v = warp; v < p.n; v += nwarps) {
        unsigned char* dst = out + v * p.nb_stride;
        const uint32_t* arow = p.adj + v * deg;
        const uint32_t a0 = lane < deg ? arow[lane] : kNoNode;
        const uint32_t a1 = lane + 32u < deg ? arow[lane + 32u] : kNoNode;
        bool dup0 = false, dup1 = false;
        for (uint32_t j = 0; j < deg; ++j) {
            const uint32_t a = __shfl_sync(kFull, j < 32u ? a0 : a1, static_cast<int>(j & 31u));
            dup0 |= j < lane && a == a0;
            dup1 |= j < lane + 32u && a == a1;
        }
        uint32_t* dadj = reinterpret_cast<uint32_t*>(dst);
        const uint32_t words = p.nb_adj_bytes / 4u;
        if (lane < words) dadj[lane] = dup0 ? kNoNode : a0;
        if (lane + 32u < words) dadj[lane + 32u] = dup1 ? kNoNode : a1;
        const uint32_t total = deg * chunks;
        for (uint32_t t = lane; t < total; t += 32) {
            const uint32_t i = t / chunks, ch = t - i * chunks;
            const uint32_t child = arow[i];
            uint4 val = make_uint4(0u, 0u, 0u, 0u);
            if (child < p.n && ch < nch) {
                const unsigned char* src = u8 ? p.vecs8 + static_cast<size_t>(child) * p.row_bytes
                                              : reinterpret_cast<const unsigned char*>(
                                                    p.vecs + static_cast<size_t>(child) * p.row_stride);
                val = *reinterpret_cast<const uint4*>(src + ch * 16u);
            }
            const uint32_t at = (u8 && ch < nch) ? nb_chunk_pos(ch, i, nch) : ch;
            *reinterpret_cast<uint4*>(dst + p.nb_adj_bytes + static_cast<size_t>(i) * p.nb_pitch + at * 16u) = val;
        }
    }
}

using KernelFn = void (*)(SearchParams);

template <int RX, int RY>
KernelFn pick_nb(int dm, int fm) {
    if (dm == kSeq) return fm == kHash ? k_search_nb<RX, RY, kSeq, kHash> : k_search_nb<RX, RY, kSeq, kBloom>;
    if (dm == kU8) return fm == kHash ? k_search_nb<RX, RY, kU8, kHash> : k_search_nb<RX, RY, kU8, kBloom>;
    return fm == kHash ? k_search_nb<RX, RY, kTeam, kHash> : k_search_nb<RX, RY, kTeam, kBloom>;
}

KernelFn select_nb(int regx, int regy, int dm, int fm) {
    if (regy == 1) {
        switch (regx) {
            case 1: return pick_nb<1, 1>(dm, fm);
            case 2: return pick_nb<2, 1>(dm, fm);
            case 4: return pick_nb<4, 1>(dm, fm);
            case 8: return pick_nb<8, 1>(dm, fm);
            case 16: return pick_nb<16, 1>(dm, fm);
        }
    } else if (regy == 2) {
        switch (regx) {
            case 2: return pick_nb<2, 2>(dm, fm);
            case 4: return pick_nb<4, 2>(dm, fm);
            case 8: return pick_nb<8, 2>(dm, fm);
            case 16: return pick_nb<16, 2>(dm, fm);
        }
    }
    return nullptr;
}

}  // namespace

cudaError_t launch_search_nb(const SearchParams& p, const LaunchShape& shape, int num_sms, cudaStream_t stream) {
    KernelFn fn = select_nb(shape.regx, shape.regy, shape.dmode, shape.fmode);
    if (!fn) return cudaErrorInvalidValue;
    const int threads = 32 * shape.warps_per_block;
    const size_t smem = static_cast<size_t>(shape.smem_per_warp) * shape.warps_per_block;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
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

cudaError_t build_neighbourhood_blocks(const SearchParams& p, unsigned char* out, cudaStream_t stream) {
    if (p.degree > 64u) return cudaErrorInvalidValue;
    const uint64_t warps = p.n;
    const uint64_t blocks64 = (warps + 7) / 8;
    const unsigned blocks = static_cast<unsigned>(blocks64 < 65535ull * 8 ? blocks64 : 65535ull * 8);
    k_build_nb<<<blocks, 256, 0, stream>>>(p, out);
    return cudaGetLastError();
}

}  // namespace bsb
