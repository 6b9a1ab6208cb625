// bs_search_bq.cu -- mode "base": the exact L2 beam search with one thread
// block per query over the neighbourhood blocks.
//
// The reference's base mode runs one block of threads per query and lets its
// warps split the neighbour distances (include/gpu_search_base.cuh:121-247,
// launched by src/gpu_cli.cu:236-284).  Same results as every other exact
// mode here (the reference CPU search, include/cpu_search_base.hpp:22-82);
// the block's extra warps shorten one query's chain of expansions instead of
// serving more queries, which pays when a GPU has fewer queries than resident
// warps (small batches, a fixed batch split over many GPUs):
//
//   * warp 0 owns the beam (registers), the visited table and the merge, as
//     the warp-per-query kernel does;
//   * two block buffers: while expansion i is scored, the block of the entry
//     the next pick takes if nothing better turns up is already being copied
//     into the other buffer (one bulk copy), so a correct guess finds its
//     block in shared memory; a wrong guess costs one copy and the right
//     block is copied then;
//   * every thread scores: byte rows with integer queries split each row over
//     NW consecutive threads (exact integer sums, any order gives the same
//     value), the sequential fold keeps one thread per row (its order).
//
// Control per expansion: warp 0 picks and starts copies, a block barrier
// publishes the buffer, all threads wait for it (bounded) and score, a second
// barrier hands the distances to warp 0.
#include <cfloat>
#include <cstdio>
#include <cstdlib>

#include "bs_bulk.cuh"
#include "bs_device.cuh"
#include "bs_internal.h"
#include "bs_nb.cuh"
#include "bs_score.cuh"

namespace bsb {

using namespace dev;

namespace {

struct BqCtl {
    uint32_t qi;        // the block's query
    uint32_t state;     // 0: expand, 1: query done, 2: a wait gave up
    uint32_t buf;       // buffer holding this expansion's block
    uint32_t phase;     // parity the buffer's copy completes with
    uint32_t pending;   // the copy has not been waited for yet
    uint32_t team_ok;   // the query takes the integer-exact path
};

// Distances of the rows of one block into dsm[0..degree), by all 32*NW
// threads of the block.
template <int DM, int NW, int RY>
__device__ __forceinline__ void bq_score(const SearchParams& p, const unsigned char* rows, const float* qv,
                                         const unsigned char* qb, uint32_t qq, bool team_ok, float* dsm,
                                         unsigned tid) {
    if (DM == kU8 && team_ok) {
        const uint32_t nch = p.row_bytes / 16u;
        const uint32_t part = tid % NW;
#pragma unroll
        for (int g = 0; g < RY; ++g) {
            const uint32_t s = tid / NW + 32u * static_cast<uint32_t>(g);
            unsigned xx = 0u, qx = 0u;
            if (s < p.degree) {
                const unsigned char* row = rows + static_cast<size_t>(s) * p.nb_pitch;
                if ((nch & 7u) == 0u) {
                    // the row's chunks sit rotated by s within each group of 8
                    // (nb_chunk_pos); thread `part` reads the physical chunks
                    // part, part+NW, ... starting at a row-dependent one, so
                    // the 8 threads of a shared-memory phase (8/NW rows) read
                    // 8 different chunk positions, and pairs each with the
                    // query chunk it holds
                    for (uint32_t g0 = 0; g0 < nch; g0 += 8u) {
#pragma unroll
                        for (uint32_t i = 0; i < 8u / NW; ++i) {
                            const uint32_t pl = part + NW * ((i + s) & (8u / NW - 1u));
                            const uint32_t c = (pl - s) & 7u;
                            const uint4 v = *reinterpret_cast<const uint4*>(row + (g0 + pl) * 16u);
                            const uint4 q = *reinterpret_cast<const uint4*>(qb + (g0 + c) * 16u);
                            dp4a_chunk(v, q, xx, qx);
                        }
                    }
                } else {
                    for (uint32_t c = part; c < nch; c += NW) {
                        const uint4 v = *reinterpret_cast<const uint4*>(row + nb_chunk_pos(c, s, nch) * 16u);
                        const uint4 q = *reinterpret_cast<const uint4*>(qb + c * 16u);
                        dp4a_chunk(v, q, xx, qx);
                    }
                }
            }
            // sum x^2 - 2 sum q.x over the row's parts (mod 2^32, exact once
            // sum q^2 is added: the true value is below 2^24)
            unsigned t = xx - 2u * qx;
#pragma unroll
            for (int o = NW / 2; o > 0; o >>= 1) t += __shfl_xor_sync(kFull, t, o);
            if (part == 0u && s < p.degree) dsm[s] = static_cast<float>(t + qq);
        }
        return;
    }
    // one thread per row: the sequential fold (its order), or the integer
    // paths of non-byte rows
    for (uint32_t s = tid; s < p.degree; s += 32u * NW)
        dsm[s] = block_row_dist<DM>(p, rows, s, qv, qb, qq, team_ok);
}

template <int RX, int RY, int DM, int NW>
__global__ void __launch_bounds__(32 * NW, (RX >= 8 ? 16 : 32) / NW) k_search_bq(const SearchParams p) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const unsigned tid = threadIdx.x;
    const unsigned lane = tid & 31u;
    const bool w0 = tid < 32u;
    float* qsm = reinterpret_cast<float*>(smem_raw);
    uint32_t* q8 = reinterpret_cast<uint32_t*>(smem_raw + p.off_q8);
    const unsigned char* qb = smem_raw + p.off_q8;
    uint32_t* filt = reinterpret_cast<uint32_t*>(smem_raw + p.off_filter);
    uint64_t* ckeys = reinterpret_cast<uint64_t*>(smem_raw + p.off_keys);
    float* dsm = reinterpret_cast<float*>(smem_raw + p.off_cdist);
    uint32_t* cids = reinterpret_cast<uint32_t*>(smem_raw + p.off_cids);
    BqCtl* ctl = reinterpret_cast<BqCtl*>(smem_raw + p.off_stage);
    uint64_t* mbar = reinterpret_cast<uint64_t*>(smem_raw + p.off_mbar);   // [2]
    unsigned char* blk0 = smem_raw + p.off_block;
    const uint32_t bpitch = bq_buffer_pitch(p.nb_stride);

    const uint32_t deg = p.degree;
    const uint32_t fmask = p.filter_slots - 1u;
    const uint32_t fshift = 32u - static_cast<uint32_t>(__popc(fmask));
    const unsigned lt_mask = (1u << lane) - 1u;
    unsigned err = 0;
    // warp 0's record of the two buffers: the node whose block was last
    // copied into each, the parity its copy completes with, and whether that
    // copy is still to be waited for
    uint32_t bnode0 = kNoNode, bnode1 = kNoNode;
    unsigned bph0 = 0u, bph1 = 0u;
    bool bpend0 = false, bpend1 = false;
    if (tid == 0) {
        mbar_init(&mbar[0]);
        mbar_init(&mbar[1]);
    }
    __syncthreads();

    for (;;) {
        if (tid == 0) ctl->qi = atomicAdd(&p.counters->next_query, 1u);
        __syncthreads();
        const unsigned qi = ctl->qi;
        if (qi >= p.nq) break;

        const float* q = query_src(p, qi);
        if (DM == kU8 && p.queries_src != nullptr) {
            // read over the bus once, into this query's device slot
            float* slot = const_cast<float*>(p.queries) + static_cast<size_t>(qi) * p.dim;
            copy_query_row(slot, q, p.dim, tid, 32u * NW);
            q = slot;
        }
        const float* qv = DM == kU8 ? q : qsm;
        if (DM != kU8)
            for (uint32_t d = tid; d < p.row_stride; d += 32u * NW) qsm[d] = d < p.dim ? q[d] : 0.0f;
        for (uint32_t i = tid; i < p.filter_words; i += 32u * NW) filt[i] = kNoNode;
        __syncthreads();

        uint64_t beam[RX];
#pragma unroll
        for (int r = 0; r < RX; ++r) beam[r] = kEmptyKey;
        uint32_t filled = 1, E = 0, D = 1;
        if (w0) {
            const bool team_ok = DM != kSeq && query_integer_exact(qv, p.dim, p.team_qlo, p.team_qhi);
            if (DM != kSeq && !team_ok && lane == 0) atomicAdd(&p.counters->team_fallbacks, 1u);
            if (DM == kU8 && team_ok) pack_query_u8(qv, p.dim, p.row_bytes, q8, lane);
            if (lane == 0) cids[0] = p.entry;
            __syncwarp();
            score_direct<DM>(p, 1, cids, dsm, qv, q8, lane, team_ok);
            if (lane == 0) {
                beam[0] = make_key(dsm[0], p.entry);
                hash_insert(filt, fmask, fshift, p.entry, err);
                ctl->team_ok = team_ok ? 1u : 0u;
            }
        }
        __syncthreads();
        const bool team_ok = ctl->team_ok != 0u;
        const uint32_t qq = (DM == kU8 && team_ok) ? q8[p.row_bytes / 4u] : 0u;

        for (int iter = 0;; ++iter) {
            if (w0) {
                uint32_t cur = kNoNode, nxt = kNoNode;
                const bool go = iter < p.max_iterations && beam_pick_next<RX>(beam, lane, cur, nxt);
                unsigned state = go ? 0u : 1u, cb = 0u;
                if (go) {
                    ++E;
                    if (bnode0 == cur) cb = 0u;
                    else if (bnode1 == cur) cb = 1u;
                    else {
                        // at most one copy is pending here (the last guess);
                        // the other buffer's block was waited for and read
                        cb = bpend0 ? 1u : 0u;
                        if (lane == 0)
                            bulk_load(blk0 + cb * bpitch, p.nb + static_cast<size_t>(cur) * p.nb_stride, p.nb_stride,
                                      &mbar[cb]);
                        if (cb) { bnode1 = cur; bpend1 = true; } else { bnode0 = cur; bpend0 = true; }
                    }
                    // the guess for the next expansion, into the other buffer
                    const unsigned ob = cb ^ 1u;
                    const uint32_t onode = ob ? bnode1 : bnode0;
                    if (nxt != kNoNode && onode != nxt) {
                        bool ready = true;
                        if (ob ? bpend1 : bpend0) {
                            // a wrong guess still in flight: let it land first
                            ready = mbar_wait(&mbar[ob], ob ? bph1 : bph0, p.wait_polls);
                            if (ready) {
                                if (ob) { bph1 ^= 1u; bpend1 = false; } else { bph0 ^= 1u; bpend0 = false; }
                            } else {
                                err |= kErrWaitTimeout;
                                state = 2u;
                            }
                        }
                        if (ready) {
                            if (lane == 0)
                                bulk_load(blk0 + ob * bpitch, p.nb + static_cast<size_t>(nxt) * p.nb_stride,
                                          p.nb_stride, &mbar[ob]);
                            if (ob) { bnode1 = nxt; bpend1 = true; } else { bnode0 = nxt; bpend0 = true; }
                        }
                    }
                }
                if (lane == 0) {
                    ctl->state = state;
                    ctl->buf = cb;
                    ctl->phase = cb ? bph1 : bph0;
                    ctl->pending = (cb ? bpend1 : bpend0) ? 1u : 0u;
                }
            }
            __syncthreads();
            const unsigned state = ctl->state;
            const unsigned cb = ctl->buf;
            bool ok = state != 2u;
            if (state == 0u && ctl->pending) ok = mbar_wait(&mbar[cb], ctl->phase, p.wait_polls);
            if (__syncthreads_or(!ok)) {
                // a wait gave up: wait (bounded again) for the copies in
                // flight so that none outlives the block, report, leave
                if (w0) {
                    bool landed = true;
                    if (bpend0) landed = mbar_wait(&mbar[0], bph0, kDefaultWaitPolls) && landed;
                    if (bpend1) landed = mbar_wait(&mbar[1], bph1, kDefaultWaitPolls) && landed;
                    if (lane == 0) report_errors(p, err | kErrWaitTimeout | (landed ? 0u : kErrCopyPending));
                }
                return;
            }
            if (state != 0u) break;

            const unsigned char* blk = blk0 + cb * bpitch;
            bq_score<DM, NW, RY>(p, blk + p.nb_adj_bytes, qv, qb, qq, team_ok, dsm, tid);
            __syncthreads();
            if (!w0) continue;   // the next barrier orders warp 0's merge before the next scoring

            if (cb) { if (bpend1) { bph1 ^= 1u; bpend1 = false; } }
            else if (bpend0) { bph0 ^= 1u; bpend0 = false; }
            const uint32_t* blk_adj = reinterpret_cast<const uint32_t*>(blk);
            uint64_t k[RY];
            bool keep[RY];
            uint32_t c[RY];
            const uint64_t bound = beam_bound<RX>(beam, p.topk);
            uint32_t nkeep = 0;
#pragma unroll
            for (int r = 0; r < RY; ++r) {
                const uint32_t pos = static_cast<uint32_t>(r) * 32u + lane;
                c[r] = pos < deg ? blk_adj[pos] : kNoNode;
                const bool live = c[r] < p.n;
                k[r] = live ? make_key(dsm[pos], c[r]) : kEmptyKey;
                D += __popc(__ballot_sync(kFull, live));
                keep[r] = k[r] < bound;
                nkeep += __popc(__ballot_sync(kFull, keep[r]));
            }
            if (nkeep) {
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
        }

        if (w0) {
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
        }
    }
    // a guess may still be in flight: it lands before the block leaves
    if (w0) {
        bool landed = true;
        if (bpend0) landed = mbar_wait(&mbar[0], bph0, kDefaultWaitPolls) && landed;
        if (bpend1) landed = mbar_wait(&mbar[1], bph1, kDefaultWaitPolls) && landed;
        if (!landed) err |= kErrWaitTimeout | kErrCopyPending;
        if (lane == 0 && err) report_errors(p, err);
    }
}

using KernelFn = void (*)(SearchParams);

template <int RX, int RY, int NW>
KernelFn pick_bq(int dm) {
    if (dm == kSeq) return k_search_bq<RX, RY, kSeq, NW>;
    if (dm == kU8) return k_search_bq<RX, RY, kU8, NW>;
    return k_search_bq<RX, RY, kTeam, NW>;
}

template <int NW>
KernelFn select_bq_nw(int regx, int regy, int dm) {
    if (regy == 1) {
        switch (regx) {
            case 1: return pick_bq<1, 1, NW>(dm);
            case 2: return pick_bq<2, 1, NW>(dm);
            case 4: return pick_bq<4, 1, NW>(dm);
            case 8: return pick_bq<8, 1, NW>(dm);
            case 16: return pick_bq<16, 1, NW>(dm);
        }
    } else if (regy == 2) {
        switch (regx) {
            case 2: return pick_bq<2, 2, NW>(dm);
            case 4: return pick_bq<4, 2, NW>(dm);
            case 8: return pick_bq<8, 2, NW>(dm);
            case 16: return pick_bq<16, 2, NW>(dm);
        }
    }
    return nullptr;
}

KernelFn select_bq(int regx, int regy, int dm, int nw) {
    return nw == 2 ? select_bq_nw<2>(regx, regy, dm) : select_bq_nw<4>(regx, regy, dm);
}

inline uint32_t a16(uint32_t v) { return (v + 15u) & ~15u; }

}  // namespace

cudaError_t plan_search_bq(SearchParams& p, LaunchShape& shape, size_t max_smem_optin, char* why,
                           size_t why_len) {
    auto fail = [&](const char* msg) {
        if (why && why_len) std::snprintf(why, why_len, "%s", msg);
        return cudaErrorInvalidValue;
    };
    if (p.nb == nullptr || p.codes != nullptr || shape.fmode != kHash)
        return fail("block-per-query search needs neighbourhood blocks and the exact table");
    if (p.degree == 0) return fail("graph degree is zero");
    if (p.degree <= 32) shape.regy = 1;
    else if (p.degree <= 64) shape.regy = 2;
    else return fail("graph degree above 64 is not supported by this build");
    if (p.topk == 0) return fail("topk_size must be positive");
    if (p.topk > 512) return fail("topk_size above 512 is not supported by this build");
    uint32_t cap = 32;
    while (cap < p.topk) cap <<= 1;
    shape.regx = static_cast<int>(cap / 32);
    if (shape.regx < shape.regy) shape.regx = shape.regy;
    // the exact table holds the ids that passed into the beam (as in the
    // warp-per-query block kernel): >= 4 * (topk + degree) slots, rebuilt
    // from the beam at a quarter load
    uint32_t slots = 64;
    while (slots < 4u * (p.topk + p.degree)) slots <<= 1;
    p.filter_slots = slots;
    p.filter_limit = slots / 4u;
    p.filter_words = slots;
    const uint32_t cand = 32u * static_cast<uint32_t>(shape.regy);
    uint32_t off = shape.dmode == kU8 ? 0u : a16(p.row_stride * 4u);   // f32 query (non-byte rows)
    p.off_q8 = off;
    if (shape.dmode == kU8) off = a16(off + p.row_bytes + 4u);          // packed query + sum q^2
    p.off_filter = off;
    off = a16(off + p.filter_words * 4u);
    p.off_keys = off;
    off = a16(off + cand * 8u);
    p.off_cdist = off;
    off = a16(off + cand * 4u);
    p.off_cids = off;
    off = a16(off + 16u);
    p.off_stage = off;                      // control words
    off = a16(off + static_cast<uint32_t>(sizeof(BqCtl)));
    p.off_mbar = off;
    off = a16(off + 16u);
    off = (off + 127u) & ~127u;
    p.off_block = off;
    off += 2u * bq_buffer_pitch(p.nb_stride);
    p.stage_rows = 0;
    p.stage_ring = 0;
    p.smem_per_warp = off;                  // per block (one query)
    shape.smem_per_warp = off;
    int nw = (p.sm_count > 0 && p.nq > 8ull * p.sm_count) ? 2 : 4;
    if (const char* e = std::getenv("BSEARCH_BQ_WARPS")) {
        const int v = std::atoi(e);
        if (v == 2 || v == 4) nw = v;
    }
    shape.warps_per_block = nw;
    shape.block_query = 1;
    if (off > max_smem_optin) return fail("shared memory per block exceeds the device limit");
    return cudaSuccess;
}

cudaError_t launch_search_bq(const SearchParams& p, const LaunchShape& shape, int num_sms, cudaStream_t stream) {
    KernelFn fn = select_bq(shape.regx, shape.regy, shape.dmode, shape.warps_per_block);
    if (!fn) return cudaErrorInvalidValue;
    const int threads = 32 * shape.warps_per_block;
    const size_t smem = shape.smem_per_warp;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    // one query per block at a time: the grid is the resident capacity in
    // blocks, or one block per query
    const unsigned grid = persistent_blocks(p.nq, 1, per_sm, num_sms);
    if (grid == 0) return cudaSuccess;
    fn<<<grid, threads, smem, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace bsb
