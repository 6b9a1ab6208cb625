// bs_graph_build.cu -- the reference Vamana graph builder (src/build_graph.cpp:
// 255-397) on the GPU, producing the same graph.bin.
//
// The reference inserts the nodes in a seeded random order in batches
// (start = 1; each batch doubles, capped at 2% of n).  Inside a batch every
// target is independent -- it searches the graph of the earlier batches,
// which the batch never changes -- so the batch maps to one warp per target:
//
//   search  (:312-333): greedy beam search of width L from order[0]; every
//           node the search expands joins the target's candidate pool; the
//           neighbours of an expanded node are visited in list order and
//           pushed one after another, each only while the beam has room or
//           its distance is below the beam's tail (strict, by distance:
//           BeamQueue, :44-96), which is an order-dependent rule for ties,
//           so the pushes stay sequential per warp;
//   prune   (:142-198): sort the pool by (distance, id), drop the target and
//           repeats, and if more than R remain run the robust prune, alpha
//           1 then alpha: a candidate is dropped when alpha * d(kept, c) <= d(c);
//   reverse (:352-356): every new edge src -> dst appends (d, src) to dst's
//           list, in batch order then list order (a stable sort of the
//           batch's edges by destination), and lists longer than R are
//           pruned again (:357-363);
//   finish  (:372-381): every list sorted, repeats dropped, the first R ids
//           written, missing slots 0.
//
// Distances are the reference's sequential fp32 sums (or exact integer sums
// for integer rows, the same values), so the lists, their order and hence
// the file are the reference's.
#include <cfloat>
#include <cstdio>

#include <cub/device/device_radix_sort.cuh>

#include "bs_device.cuh"
#include "bs_internal.h"
#include "bs_score.cuh"

namespace bsb {

using namespace dev;

namespace {

// Candidate key: ord(dist) << 32 | id, ordered as the reference's (distance,
// id) pairs (src/build_graph.cpp:148-151).
__device__ __forceinline__ unsigned long long pkey(float d, uint32_t id) {
    return (static_cast<unsigned long long>(f2ord(d)) << 32) | id;
}

__device__ __forceinline__ bool gb_visit(uint32_t* bits, uint32_t c) {
    const uint32_t m = 1u << (c & 31u);
    return (atomicOr(bits + (c >> 5), m) & m) == 0u;
}

__device__ __forceinline__ void gb_clear(const GraphBuildArgs& a, uint32_t* bits, const uint32_t* log,
                                         uint32_t logged, unsigned lane) {
    __syncwarp();
    if (logged <= a.vis_log_cap) {
        for (uint32_t i = lane; i < logged; i += 32) bits[log[i] >> 5] = 0u;
    } else {
        uint4* b4 = reinterpret_cast<uint4*>(bits);
        for (uint32_t i = lane; i < a.vis_words / 4u; i += 32) b4[i] = make_uint4(0u, 0u, 0u, 0u);
    }
    __threadfence();
    __syncwarp();
}

// Loads node u's row as the "query" of the distance helpers: f32 into qsm
// (zero pad to row_stride), and for byte rows its packed bytes + sum of
// squares into q8.  Returns whether the integer-exact paths may be used.
template <int DM>
__device__ __forceinline__ bool load_row_as_query(const SearchParams& sp, uint32_t u, float* qsm, uint32_t* q8,
                                                  unsigned lane) {
    if (DM == kU8) {
        const uint8_t* r = sp.vecs8 + static_cast<size_t>(u) * sp.row_bytes;
        for (uint32_t d = lane; d < sp.row_stride; d += 32) qsm[d] = d < sp.dim ? static_cast<float>(r[d]) : 0.0f;
    } else {
        const float* r = sp.vecs + static_cast<size_t>(u) * sp.row_stride;
        for (uint32_t d = lane; d < sp.row_stride; d += 32) qsm[d] = r[d];
    }
    __syncwarp();
    const bool team_ok = DM != kSeq && query_integer_exact(qsm, sp.dim, sp.team_qlo, sp.team_qhi);
    if (DM == kU8 && team_ok) pack_query_u8(qsm, sp.dim, sp.row_bytes, q8, lane);
    return team_ok;
}

// ------------------------------------------------------------- search

template <int RX, int DM>
__global__ void __launch_bounds__(128) k_gb_search(const GraphBuildArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const SearchParams& sp = a.sp;
    const unsigned lane = threadIdx.x & 31u;
    unsigned char* ws = smem_raw + static_cast<size_t>(threadIdx.x >> 5) * sp.smem_per_warp;
    float* qsm = reinterpret_cast<float*>(ws);
    uint32_t* q8 = reinterpret_cast<uint32_t*>(ws + sp.off_q8);
    uint32_t* cids = reinterpret_cast<uint32_t*>(ws + sp.off_cids);
    float* cdist = reinterpret_cast<float*>(ws + sp.off_cdist);
    float* stage = reinterpret_cast<float*>(ws + sp.off_stage);
    const unsigned lt_mask = (1u << lane) - 1u;
    const uint64_t gwarp = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = (static_cast<uint64_t>(gridDim.x) * blockDim.x) >> 5;
    uint32_t* vbits = a.vis + gwarp * (static_cast<uint64_t>(a.vis_words) + a.vis_log_cap);
    uint32_t* vlog = vbits + a.vis_words;
    const uint32_t L = a.L;
    const uint32_t entry = a.order[0];
    unsigned err = 0;

    for (uint64_t slot = gwarp; slot < a.count; slot += nwarps) {
        const uint32_t target = a.order[a.start + slot];
        const bool team_ok = load_row_as_query<DM>(sp, target, qsm, q8, lane);
        if (lane == 0) cids[0] = entry;
        __syncwarp();
        score_rows<DM>(sp, 1, cids, cdist, qsm, q8, stage, lane, team_ok);
        uint64_t beam[RX];
#pragma unroll
        for (int r = 0; r < RX; ++r) beam[r] = kEmptyKey;
        if (lane == 0) {
            beam[0] = make_key(cdist[0], entry);
            gb_visit(vbits, entry);
            vlog[0] = entry;
        }
        uint32_t size = 1, logged = 1, pooled = 0;
        unsigned long long* pool = a.pool + slot * a.pool_cap;
        __syncwarp();

        for (;;) {
            uint32_t cur;
            if (!beam_pick<RX>(beam, lane, cur)) break;
            // the expanded entry joins the pool (its key without the mark)
            if (pooled >= a.pool_cap) { err |= kErrPoolFull; break; }
            {
                uint64_t mine = 0;
                const uint64_t want = static_cast<uint64_t>(cur) << 1;
#pragma unroll
                for (int r = 0; r < RX; ++r)
                    if ((beam[r] & 0xffffffffull & ~1ull) == want && beam[r] != kEmptyKey) mine = beam[r];
                const unsigned has = __ballot_sync(kFull, mine != 0);
                const uint64_t k = __shfl_sync(kFull, mine, __ffs(has) - 1);
                if (lane == 0) pool[pooled] = (k & 0xffffffff00000000ull) | cur;
            }
            ++pooled;
            __syncwarp();   // earlier reads of cids / cdist are done

            // cur's list in order; a node is new when its bit was clear
            const uint32_t cnt = a.nbr_cnt[cur];
            uint32_t m = 0;
            for (uint32_t b0 = 0; b0 < cnt; b0 += 32) {
                const uint32_t pos = b0 + lane;
                uint32_t nb = kNoNode;
                bool fresh = false;
                if (pos < cnt) {
                    nb = a.nbr_ids[static_cast<size_t>(cur) * a.degree + pos];
                    fresh = gb_visit(vbits, nb);
                }
                const unsigned bm = __ballot_sync(kFull, fresh);
                if (fresh) {
                    const uint32_t at = m + __popc(bm & lt_mask);
                    cids[at] = nb;
                    if (logged + at < a.vis_log_cap) vlog[logged + at] = nb;
                }
                m += __popc(bm);
            }
            logged += m;
            __syncwarp();
            if (m == 0) continue;
            score_rows<DM>(sp, m, cids, cdist, qsm, q8, stage, lane, team_ok);

            // pushes in list order (BeamQueue::push, src/build_graph.cpp:48-62,
            // 326-330): a key enters
            // while the beam is not full or its distance is below the tail's
            // distance; the tail only falls, so a key at or above the tail
            // before the first push cannot enter later either
            const uint64_t tail0 = beam_bound<RX>(beam, L);
            for (uint32_t j0 = 0; j0 < m; j0 += 32) {
                const uint32_t j = j0 + lane;
                uint64_t kj = kEmptyKey;
                if (j < m) kj = make_key(cdist[j], cids[j]);
                unsigned cand = __ballot_sync(kFull, j < m && (size < L || (kj >> 32) < (tail0 >> 32)));
                while (cand) {
                    const int src = __ffs(cand) - 1;
                    cand &= cand - 1u;
                    const uint64_t k = __shfl_sync(kFull, kj, src);
                    bool enter = size < L;
                    if (!enter) {
                        const uint64_t tail = beam_bound<RX>(beam, L);
                        enter = (k >> 32) < (tail >> 32);
                    }
                    if (enter) {
                        beam_insert1<RX>(beam, lane, k, L);
                        size = size < L ? size + 1 : L;
                    }
                }
            }
        }
        if (lane == 0) a.pool_cnt[slot] = pooled;
        gb_clear(a, vbits, vlog, logged, lane);
    }
    if (lane == 0 && err) atomicOr(a.err, err);
}

// ------------------------------------------------------------- prune

// Shared memory of a prune warp: the candidate keys (ord(dist) << 32 | id,
// sorted in place), a flag per candidate (kept in pass 1), the candidate row
// being tested, the kept ids.
struct PruneSmem {
    unsigned long long* keys;
    unsigned char* kept_flag;
    float* crow;
    uint32_t* crow8;
    uint32_t* kept_ids;
    float* kept_dist;
    uint32_t* krow8;     // byte rows of the kept candidates (null: read from global memory)
};

// Byte rows of the kept candidates are cached in shared memory when they take
// at most this many bytes (degree x row bytes): every domination test then
// reads them there instead of from L2.
constexpr uint32_t kKeptRowCacheBytes = 8192;

__host__ __device__ inline uint32_t kept_row_cache_bytes(const GraphBuildArgs& a) {
    const uint32_t b = a.degree * a.sp.row_bytes;
    return (a.sp.vecs8 != nullptr && b <= kKeptRowCacheBytes) ? b : 0u;
}

__device__ __forceinline__ void warp_sort_keys(unsigned long long* k, uint32_t P, unsigned lane) {
    for (uint32_t size = 2; size <= P; size <<= 1) {
        for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
            for (uint32_t i = lane; i < P; i += 32) {
                const uint32_t j = i ^ stride;
                if (j > i) {
                    const unsigned long long x = k[i], y = k[j];
                    const bool asc = (i & size) == 0;
                    if ((x > y) == asc) { k[i] = y; k[j] = x; }
                }
            }
            __syncwarp();
        }
    }
}

// d(kept row, candidate row) by one lane, the reference's value; byte rows
// come from krow (the kept row cached in shared memory) when it is given.
template <int DM>
__device__ __forceinline__ float pair_dist(const SearchParams& sp, uint32_t kept, const float* crow,
                                           const uint32_t* crow8, bool int_ok, const uint32_t* krow) {
    if (DM == kU8 && int_ok) {
        const uint32_t* x = krow ? krow
                                 : reinterpret_cast<const uint32_t*>(sp.vecs8 + static_cast<size_t>(kept) * sp.row_bytes);
        unsigned acc = 0u;
        for (uint32_t w = 0; w < sp.row_bytes / 4u; ++w) {
            const unsigned d = __vabsdiffu4(x[w], crow8[w]);
            acc = __dp4a(d, d, acc);
        }
        return static_cast<float>(acc);
    }
    if (DM == kU8) {
        const uint8_t* x = krow ? reinterpret_cast<const uint8_t*>(krow) : sp.vecs8 + static_cast<size_t>(kept) * sp.row_bytes;
        float s = 0.0f;
        for (uint32_t d = 0; d < sp.dim; ++d) {
            const float t = __fsub_rn(static_cast<float>(x[d]), crow[d]);
            s = __fadd_rn(s, __fmul_rn(t, t));
        }
        return s;
    }
    const float* x = sp.vecs + static_cast<size_t>(kept) * sp.row_stride;
    if (DM == kTeam && int_ok) {
        float s = 0.0f;
        for (uint32_t d = 0; d < sp.row_stride; ++d) {
            const float t = x[d] - crow[d];
            s = fmaf(t, t, s);
        }
        return s;
    }
    return l2_seq(x, crow, sp.dim);
}

// Sorts the c candidate keys of node u, drops u and repeats, and writes u's
// list: the unique candidates when at most R remain, else the robust prune's
// choice (src/build_graph.cpp:142-198).  Ends with __syncwarp.
template <int DM>
__device__ void prune_and_store(const GraphBuildArgs& a, uint32_t u, uint32_t c, const PruneSmem& s, unsigned lane) {
    const SearchParams& sp = a.sp;
    const unsigned lt_mask = (1u << lane) - 1u;
    uint32_t P = 32;
    while (P < c) P <<= 1;
    for (uint32_t i = c + lane; i < P; i += 32) s.keys[i] = kEmptyKey;
    __syncwarp();
    warp_sort_keys(s.keys, P, lane);
    // unique: not u, not the id before it in sorted order
    uint32_t nu = 0;
    for (uint32_t i0 = 0; i0 < c; i0 += 32) {
        const uint32_t i = i0 + lane;
        bool keep = false;
        if (i < c) {
            const uint32_t id = static_cast<uint32_t>(s.keys[i]);
            keep = id != u && (i == 0 || static_cast<uint32_t>(s.keys[i - 1]) != id);
            s.kept_flag[i] = keep ? 1 : 0;
        }
        nu += __popc(__ballot_sync(kFull, keep));
    }
    __syncwarp();
    uint32_t* ids = a.nbr_ids + static_cast<size_t>(u) * a.degree;
    float* dists = a.nbr_dist + static_cast<size_t>(u) * a.degree;
    if (nu <= a.degree) {
        uint32_t at = 0;
        for (uint32_t i0 = 0; i0 < c; i0 += 32) {
            const uint32_t i = i0 + lane;
            const bool keep = i < c && s.kept_flag[i];
            const unsigned bm = __ballot_sync(kFull, keep);
            if (keep) {
                const uint32_t pos = at + __popc(bm & lt_mask);
                ids[pos] = static_cast<uint32_t>(s.keys[i]);
                dists[pos] = key_dist(s.keys[i]);   // ord(dist) in the high word
            }
            at += __popc(bm);
        }
        if (lane == 0) a.nbr_cnt[u] = nu;
        __syncwarp();
        return;
    }
    // robust prune; kept_flag now marks the candidates kept in pass 1
    for (uint32_t i = lane; i < c; i += 32) s.kept_flag[i] = s.kept_flag[i] ? 2 : 0;   // 2: unique, not kept
    __syncwarp();
    uint32_t kn = 0;
    bool int_ok = false;
    for (int pass = 0; pass < 2 && kn < a.degree; ++pass) {
        const float alpha = pass == 0 ? 1.0f : a.alpha;
        for (uint32_t i = 0; i < c && kn < a.degree; ++i) {
            const unsigned char f = s.kept_flag[i];
            if (f != 2) continue;                 // a repeat, or kept in pass 1 (dominated by itself)
            const uint32_t node = static_cast<uint32_t>(s.keys[i]);
            const float dist = key_dist(s.keys[i]);
            // the candidate's row, for every lane
            __syncwarp();
            if (DM == kU8) {
                const uint8_t* r = sp.vecs8 + static_cast<size_t>(node) * sp.row_bytes;
                for (uint32_t w = lane; w < sp.row_bytes / 4u; w += 32)
                    s.crow8[w] = reinterpret_cast<const uint32_t*>(r)[w];
                for (uint32_t d = lane; d < sp.row_stride; d += 32) s.crow[d] = d < sp.dim ? static_cast<float>(r[d]) : 0.0f;
            } else {
                const float* r = sp.vecs + static_cast<size_t>(node) * sp.row_stride;
                for (uint32_t d = lane; d < sp.row_stride; d += 32) s.crow[d] = r[d];
            }
            __syncwarp();
            int_ok = DM != kSeq && query_integer_exact(s.crow, sp.dim, sp.team_qlo, sp.team_qhi);
            bool dom = false;
            const uint32_t words = sp.row_bytes / 4u;
            for (uint32_t k = lane; k < kn; k += 32) {
                const float dk = pair_dist<DM>(sp, s.kept_ids[k], s.crow, s.crow8, int_ok,
                                               s.krow8 ? s.krow8 + k * words : nullptr);
                dom = dom || (__fmul_rn(alpha, dk) <= dist);
            }
            if (!__any_sync(kFull, dom)) {
                if (lane == 0) {
                    s.kept_ids[kn] = node;
                    s.kept_dist[kn] = dist;
                    s.kept_flag[i] = 1;
                }
                if (s.krow8)
                    for (uint32_t w = lane; w < words; w += 32) s.krow8[kn * words + w] = s.crow8[w];
                ++kn;
                __syncwarp();
            }
        }
    }
    for (uint32_t k = lane; k < kn; k += 32) {
        ids[k] = s.kept_ids[k];
        dists[k] = s.kept_dist[k];
    }
    if (lane == 0) a.nbr_cnt[u] = kn;
    __syncwarp();
}

// job kinds of k_gb_prune
enum PruneJob : int { kJobTargets = 0, kJobReverse = 1, kJobFinish = 2 };

template <int DM, int JOB>
__global__ void __launch_bounds__(32) k_gb_prune(const GraphBuildArgs a, unsigned long long njobs) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const unsigned lane = threadIdx.x & 31u;
    PruneSmem s;
    unsigned char* p = smem_raw;
    s.keys = reinterpret_cast<unsigned long long*>(p);
    p += static_cast<size_t>(a.prune_cap) * 8u;
    s.crow = reinterpret_cast<float*>(p);
    p += a.sp.row_stride * 4u;
    s.crow8 = reinterpret_cast<uint32_t*>(p);
    p += (a.sp.row_bytes + 15u) & ~15u;
    s.kept_ids = reinterpret_cast<uint32_t*>(p);
    p += 64u * 4u;
    s.kept_dist = reinterpret_cast<float*>(p);
    p += 64u * 4u;
    s.kept_flag = p;
    p += (a.prune_cap + 15u) & ~15u;
    s.krow8 = kept_row_cache_bytes(a) ? reinterpret_cast<uint32_t*>(p) : nullptr;
    unsigned err = 0;
    uint32_t segs = 0;
    if (JOB == kJobReverse) segs = a.ovf_pass ? *a.ovf_count : *a.seg_count;
    const unsigned long long jobs = JOB == kJobReverse ? segs : njobs;
    for (unsigned long long it = blockIdx.x; it < jobs; it += gridDim.x) {
        const unsigned long long job = (JOB == kJobReverse && a.ovf_pass) ? a.ovf_jobs[it] : it;
        uint32_t u, c = 0;
        if (JOB == kJobTargets) {
            u = a.order[a.start + job];
            c = a.pool_cnt[job];
            if (c > a.prune_cap) { err |= kErrPruneFull; continue; }
            const unsigned long long* pool = a.pool + job * a.pool_cap;
            for (uint32_t i = lane; i < c; i += 32) s.keys[i] = pool[i];
        } else if (JOB == kJobFinish) {
            u = static_cast<uint32_t>(job);
            c = a.nbr_cnt[u];
            for (uint32_t i = lane; i < c; i += 32)
                s.keys[i] = pkey(a.nbr_dist[static_cast<size_t>(u) * a.degree + i],
                                 a.nbr_ids[static_cast<size_t>(u) * a.degree + i]);
        } else {
            // a run of the sorted reverse edges with one destination
            const uint32_t b = a.seg_start[job];
            u = a.rev_dst[b];
            uint32_t e = b + 1;
            for (;;) {
                const uint32_t q = e + lane;
                const bool other = q >= a.count * a.degree || a.rev_dst[q] != u;
                const unsigned bm = __ballot_sync(kFull, other);
                if (bm) { e += __ffs(bm) - 1; break; }
                e += 32;
            }
            const uint32_t have = a.nbr_cnt[u], k = e - b;
            uint32_t* ids = a.nbr_ids + static_cast<size_t>(u) * a.degree;
            float* dists = a.nbr_dist + static_cast<size_t>(u) * a.degree;
            if (have + k <= a.degree) {
                // appended in batch order, then list order (src/build_graph.cpp:352-356)
                for (uint32_t j = lane; j < k; j += 32) {
                    const uint32_t t = a.rev_t[b + j];
                    const uint32_t slot = t / a.degree, pos = t - slot * a.degree;
                    const uint32_t src = a.order[a.start + slot];
                    ids[have + j] = src;
                    dists[have + j] = a.nbr_dist[static_cast<size_t>(src) * a.degree + pos];
                }
                if (lane == 0) a.nbr_cnt[u] = have + k;
                __syncwarp();
                continue;
            }
            c = have + k;
            if (c > a.prune_cap) {
                // too many for this launch's shared memory: to the second
                // launch's list (prunes of different nodes are independent)
                if (!a.ovf_pass && a.ovf_jobs) {
                    uint32_t at = 0;
                    if (lane == 0) at = atomicAdd(a.ovf_count, 1u);
                    at = __shfl_sync(kFull, at, 0);
                    if (at < a.ovf_cap) {
                        if (lane == 0) a.ovf_jobs[at] = static_cast<uint32_t>(job);
                    } else {
                        err |= kErrPruneFull;
                    }
                } else {
                    err |= kErrPruneFull;
                }
                continue;
            }
            for (uint32_t i = lane; i < have; i += 32) s.keys[i] = pkey(dists[i], ids[i]);
            for (uint32_t j = lane; j < k; j += 32) {
                const uint32_t t = a.rev_t[b + j];
                const uint32_t slot = t / a.degree, pos = t - slot * a.degree;
                const uint32_t src = a.order[a.start + slot];
                s.keys[have + j] = pkey(a.nbr_dist[static_cast<size_t>(src) * a.degree + pos], src);
            }
        }
        __syncwarp();
        prune_and_store<DM>(a, u, c, s, lane);
    }
    if (lane == 0 && err) atomicOr(a.err, err);
}

// (slot, position) of every new edge -> (destination, slot * degree + position)
__global__ void k_gb_rev_tuples(const GraphBuildArgs a, uint32_t* keys, uint32_t* vals) {
    const uint64_t total = a.count * a.degree;
    for (uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
         t += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t slot = t / a.degree, pos = t - slot * a.degree;
        const uint32_t src = a.order[a.start + slot];
        const bool ok = pos < a.nbr_cnt[src];
        keys[t] = ok ? a.nbr_ids[static_cast<size_t>(src) * a.degree + pos] : 0xffffffffu;
        vals[t] = static_cast<uint32_t>(t);
    }
}

__global__ void k_gb_segments(const GraphBuildArgs a) {
    const uint64_t total = a.count * a.degree;
    for (uint64_t t = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
         t += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint32_t k = a.rev_dst[t];
        if (k != 0xffffffffu && (t == 0 || a.rev_dst[t - 1] != k)) {
            const uint32_t at = atomicAdd(a.seg_count, 1u);
            a.seg_start[at] = static_cast<uint32_t>(t);
        }
    }
}

using SearchFn = void (*)(GraphBuildArgs);

template <int RX>
SearchFn pick_gb(int dm) {
    if (dm == kSeq) return k_gb_search<RX, kSeq>;
    if (dm == kU8) return k_gb_search<RX, kU8>;
    return k_gb_search<RX, kTeam>;
}

SearchFn select_gb(uint32_t L, int dm) {
    if (L <= 32) return pick_gb<1>(dm);
    if (L <= 64) return pick_gb<2>(dm);
    if (L <= 128) return pick_gb<4>(dm);
    if (L <= 256) return pick_gb<8>(dm);
    if (L <= 512) return pick_gb<16>(dm);
    return nullptr;
}

template <int JOB>
using PruneFn = void (*)(GraphBuildArgs, unsigned long long);

template <int JOB>
PruneFn<JOB> select_prune(int dm) {
    if (dm == kSeq) return k_gb_prune<kSeq, JOB>;
    if (dm == kU8) return k_gb_prune<kU8, JOB>;
    return k_gb_prune<kTeam, JOB>;
}

size_t prune_smem(const GraphBuildArgs& a) {
    return static_cast<size_t>(a.prune_cap) * 8u + ((a.prune_cap + 15u) & ~15u) + a.sp.row_stride * 4u +
           ((a.sp.row_bytes + 15u) & ~15u) + 512u + kept_row_cache_bytes(a);
}

int dm_of(const GraphBuildArgs& a) {
    return a.sp.vecs8 ? kU8 : (a.sp.team_qlo <= a.sp.team_qhi ? kTeam : kSeq);
}

template <int JOB>
cudaError_t launch_prune(const GraphBuildArgs& a, unsigned long long jobs, int num_sms, cudaStream_t stream) {
    PruneFn<JOB> fn = select_prune<JOB>(dm_of(a));
    const size_t smem = prune_smem(a);
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, 32, smem);
    if (e != cudaSuccess) return e;
    const unsigned long long cap = static_cast<unsigned long long>(per_sm > 0 ? per_sm : 1) * num_sms;
    unsigned grid = static_cast<unsigned>(jobs < cap ? (jobs ? jobs : 1) : cap);
    if (JOB == kJobReverse) grid = static_cast<unsigned>(cap);   // the job count is on the device
    fn<<<grid, 32, smem, stream>>>(a, jobs);
    return cudaGetLastError();
}

}  // namespace

// Per-warp shared memory of the build search (the query row, candidate ids
// and distances, staging for sequential folds), like the gather search's.
cudaError_t plan_graph_build(GraphBuildArgs& a, size_t smem_optin) {
    SearchParams& p = a.sp;
    const uint32_t units = p.row_stride / 4u;
    p.stage_pitch = (units % 2u == 0u) ? p.row_stride + 4u : p.row_stride + 8u;
    auto a16 = [](uint32_t x) { return (x + 15u) & ~15u; };
    uint32_t off = a16(p.row_stride * 4u);
    p.off_q8 = off;
    if (p.vecs8) off = a16(off + p.row_bytes + 4u);
    p.off_cids = off;
    off = a16(off + 64u * 4u);
    p.off_cdist = off;
    off = a16(off + 64u * 4u);
    p.off_stage = off;
    p.stage_ring = 0;
    p.stage_rows = 0;
    if (!p.vecs8 && !(p.team_qlo <= p.team_qhi)) {
        const uint32_t row_bytes = p.stage_pitch * 4u;
        if (row_bytes > 1024u) {
            p.stage_ring = dev::kRingStages;
            off = a16(off + dev::kRingFloats * 4u);
        } else {
            uint32_t rows = (24u * 1024u) / row_bytes;
            rows = rows > 32u ? 32u : (rows < 1u ? 1u : rows);
            p.stage_rows = rows;
            off = a16(off + rows * row_bytes);
        }
    } else if (p.vecs8) {
        // a fractional query never occurs (the rows are the queries), but
        // the sequential byte fold needs no staging anyway
    }
    p.smem_per_warp = off;
    if (static_cast<size_t>(off) * 4u > smem_optin) return cudaErrorInvalidValue;
    a.prune_cap = 4096;
    if (prune_smem(a) > smem_optin) return cudaErrorInvalidValue;
    return cudaSuccess;
}

size_t graph_build_sort_bytes(uint64_t items) {
    size_t bytes = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, bytes, static_cast<const uint32_t*>(nullptr), static_cast<uint32_t*>(nullptr),
                                    static_cast<const uint32_t*>(nullptr), static_cast<uint32_t*>(nullptr),
                                    static_cast<int>(items));
    return bytes;
}

uint32_t graph_build_search_warps(const GraphBuildArgs& a, int num_sms, size_t smem_optin) {
    SearchFn fn = select_gb(a.L, dm_of(a));
    if (!fn) return 0;
    const size_t smem = static_cast<size_t>(a.sp.smem_per_warp) * 4u;
    if (smem > smem_optin) return 0;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
        return 0;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, 128, smem) != cudaSuccess) return 0;
    return static_cast<uint32_t>(per_sm) * static_cast<uint32_t>(num_sms) * 4u;
}

cudaError_t graph_build_batch(GraphBuildArgs& a, size_t smem_optin, int num_sms, void* sort_tmp, size_t sort_tmp_bytes,
                              uint32_t* rev_keys_in, uint32_t* rev_vals_in, uint32_t* rev_keys_out,
                              uint32_t* rev_vals_out, cudaStream_t stream) {
    SearchFn fn = select_gb(a.L, dm_of(a));
    if (!fn) return cudaErrorInvalidValue;
    // 1. searches: one warp per target
    const uint64_t warps = a.count < a.vis_warps ? a.count : a.vis_warps;
    const unsigned blocks = static_cast<unsigned>((warps + 3) / 4);
    const size_t smem = static_cast<size_t>(a.sp.smem_per_warp) * 4u;
    fn<<<blocks, 128, smem, stream>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    // 2. the targets' lists
    {
        // a target's pool holds at most pool_cap expanded nodes: room for
        // exactly that many candidates (smaller shared memory, more prunes
        // per SM than the general 4,096)
        GraphBuildArgs t = a;
        uint32_t cap = 64;
        while (cap < a.pool_cap) cap <<= 1;
        if (cap < t.prune_cap) t.prune_cap = cap;
        if ((e = launch_prune<kJobTargets>(t, a.count, num_sms, stream)) != cudaSuccess) return e;
    }
    // 3. reverse edges, stably sorted by destination
    const uint64_t items = a.count * a.degree;
    const unsigned tb = static_cast<unsigned>(std::min<uint64_t>((items + 255) / 256, 65535ull * 8));
    k_gb_rev_tuples<<<tb, 256, 0, stream>>>(a, rev_keys_in, rev_vals_in);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    size_t tmp = sort_tmp_bytes;
    e = cub::DeviceRadixSort::SortPairs(sort_tmp, tmp, rev_keys_in, rev_keys_out, rev_vals_in, rev_vals_out,
                                        static_cast<int>(items), 0, 32, stream);
    if (e != cudaSuccess) return e;
    a.rev_dst = rev_keys_out;
    a.rev_t = rev_vals_out;
    if ((e = cudaMemsetAsync(a.seg_count, 0, 4, stream)) != cudaSuccess) return e;
    k_gb_segments<<<tb, 256, 0, stream>>>(a);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    // 4. append, or prune the lists that grow past the degree; then the
    // prunes too large for the first launch, with the large candidate array
    if (a.ovf_jobs && (e = cudaMemsetAsync(a.ovf_count, 0, 4, stream)) != cudaSuccess) return e;
    {
        GraphBuildArgs first = a;
        if (a.rev_prune_cap && a.rev_prune_cap < a.prune_cap) first.prune_cap = a.rev_prune_cap;
        if ((e = launch_prune<kJobReverse>(first, 0, num_sms, stream)) != cudaSuccess) return e;
    }
    if (!a.ovf_jobs) return cudaSuccess;
    GraphBuildArgs big = a;
    big.prune_cap = kGraphBigPruneCap;
    big.ovf_pass = 1;
    if (prune_smem(big) > smem_optin) return cudaSuccess;   // the first launch flagged them already
    return launch_prune<kJobReverse>(big, 0, num_sms, stream);
}

cudaError_t graph_build_finish(GraphBuildArgs& a, size_t smem_optin, int num_sms, cudaStream_t stream) {
    (void)smem_optin;
    // a final list holds at most degree ids
    GraphBuildArgs f = a;
    uint32_t cap = 64;
    while (cap < a.degree) cap <<= 1;
    if (cap < f.prune_cap) f.prune_cap = cap;
    return launch_prune<kJobFinish>(f, a.sp.n, num_sms, stream);
}

}  // namespace bsb
