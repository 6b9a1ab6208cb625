// bs_internal.h -- launch-level structures shared by the C ABI (bs_capi.cu)
// and the search kernels (bs_search.cu).  Not part of the public ABI.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cstdlib>
#include <cuda_runtime.h>

namespace bsb {

// Distance evaluation order.
//   kSeq : one lane per candidate row, fp32 sum over d = 0..dim-1 with each
//          multiply and add rounded separately -- the order of the reference
//          CPU search (include/cpu_search_base.hpp:29-37), so distances are
//          bit-identical to cpu_cli for any data.
//   kTeam: eight lanes per row, coalesced 16-byte loads and a shuffle tree.
//          Chosen only when every base and query value is an integer small
//          enough that all partial sums are exact in fp32, in which case any
//          order gives the same bits.
//   kU8  : rows stored as u8 (every base value an integer in [0,255]; the
//          copy is exact).  Integer queries in range: |q-x| per byte with
//          __vabsdiffu4 and sums of squares with __dp4a, 8 lanes per row --
//          exact integers, hence the reference's fp32 bits whenever
//          dim * 255^2 <= 2^24.  Other queries: the sequential fold of the
//          converted bytes (exact conversion, reference order).
enum DistMode : int { kSeq = 0, kTeam = 1, kU8 = 2 };

// Visited filter.
//   kHash : exact set in shared memory; cleared and refilled from the beam when
//           its load would pass a bound.  Never drops an unvisited node, so
//           results equal the reference cpu_cli (warpN and base modes).
//   kBloom: Bloom filter with the reference's three hashes
//           (include/filter_bloom.cuh:25-38), reset every reset_interval
//           expansions (bwarpN modes).  False positives skip nodes.
enum FilterMode : int { kHash = 0, kBloom = 1 };

// Counters in the per-launch device scratch block.
struct DevCounters {
    unsigned long long expansions;
    unsigned long long distances;
    unsigned long long estimates;
    unsigned long long rerank;
    unsigned int next_query;     // persistent-kernel work queue
    unsigned int error_flags;    // ErrorFlag bits
    unsigned int team_fallbacks; // queries that left the integer-exact path
    unsigned int pad;
};

enum ErrorFlag : unsigned int {
    kErrProbeBound = 1u,     // a visited-table probe ran the whole table
    kErrSpillFull = 2u,      // a query overflowed its RaBitQ spill table
    kErrWaitTimeout = 4u,    // a bulk-copy wait hit its iteration bound
    kErrCopyPending = 8u,    // ... and the copy in flight did not land either
};

// Polls of a bulk-copy wait before it gives up (each mbarrier.try_wait may
// itself suspend the warp for a while).  BSEARCH_WAIT_POLLS overrides it for
// the first wait of an expansion: a test sets 0 to drive the timeout path.
constexpr unsigned kDefaultWaitPolls = 1u << 22;

// Everything a search launch needs, passed by value.
struct SearchParams {
    // index (device pointers)
    const float* vecs;          // [n][row_stride] f32, pad lanes zero (null in kU8)
    const uint8_t* vecs8;       // [n][row_bytes] u8, pad bytes zero (kU8 only)
    uint32_t row_bytes;         // dim rounded up to 16
    const uint32_t* adj;        // [n][degree] u32
    // neighbourhood blocks (null: gather layout): per node, its adjacency row
    // (nb_adj_bytes; repeated ids replaced by 0xffffffff) then the rows of its
    // degree neighbours, nb_pitch bytes apart (u8 rows: 16-byte chunks
    // rotated per row); nb_stride bytes per node, all multiples of 16
    const unsigned char* nb;
    uint32_t nb_stride;
    uint32_t nb_adj_bytes;
    uint32_t nb_pitch;
    uint32_t off_block;         // per-warp copy of one block
    uint32_t off_mbar;          // per-warp mbarrier (8 bytes)
    uint64_t n;
    uint32_t dim;
    uint32_t row_stride;        // floats per stored row (dim rounded up to 4)
    uint32_t degree;
    // RaBitQ (device pointers, null unless mode rabitq)
    const uint32_t* codes;      // [n][degree][wpp]
    const float* factors;       // [n][3][degree]
    const float* signs;         // [pdim]
    uint32_t pdim;
    uint32_t wpp;
    // queries
    const float* queries;       // [nq][dim] (stride dim)
    // the caller's pinned host queries through their device mapping: read
    // once per query over the bus (then `queries` is a device slot array the
    // kernel may fill), or null when `queries` already holds them
    const float* queries_src;
    uint32_t nq;
    // search config
    uint32_t topk;              // beam size T (topk_size)
    uint32_t K;
    uint32_t entry;
    int32_t max_iterations;
    // visited filter
    uint32_t filter_slots;      // hash: table slots (pow2); bloom: bits (pow2)
    uint32_t filter_limit;      // hash: reset when entries + degree would exceed
    int32_t reset_interval;     // bloom reset period in expansions
    // RaBitQ exact visited set, second level: one table of spill_slots u32 per
    // resident warp in global memory, used once the shared table is full
    uint32_t* spill;
    uint32_t spill_slots;
    // integer-exact distance path (kTeam): a query uses it only when all its
    // values are integers in [team_qlo, team_qhi] (empty range: never)
    float team_qlo;
    float team_qhi;
    // staging
    uint32_t stage_rows;        // rows staged per round in kSeq mode
    uint32_t stage_pitch;       // floats between staged rows (odd multiple of 4)
    uint32_t stage_ring;        // kSeq wide rows: chunks in the ring of row chunks (0: no ring; 4, 5, 6
                                // or 8, bs_score.cuh)
    uint32_t sm_count;          // the device's SMs (the planner sizes the ring so that nq warps stay resident)
    // per-warp shared-memory carve-up (bytes)
    uint32_t smem_per_warp;
    uint32_t off_q8;            // kU8: the query as packed u8 (row_bytes)
    uint32_t off_filter;
    uint32_t off_cids;
    uint32_t off_cdist;
    uint32_t off_keys;          // compacted candidate keys for the merge (u64)
    uint32_t off_stage;
    uint32_t filter_words;      // u32 words of the filter table
    // outputs
    uint32_t* out_ids;          // [nq][K]
    float* out_dists;           // [nq][K] or null
    uint32_t* q_stats;          // [nq][2] (expansions, distances) or null
    DevCounters* counters;
    // the index's error word: every kernel ORs its error bits into it too, so
    // a caller of an asynchronous search can collect them later
    unsigned int* sticky_err;
    uint32_t wait_polls;        // first bounded wait of an expansion (polls)
    // RaBitQ node blocks (null: the gather kernel): per node, its adjacency
    // row (repeats -> 0xffffffff), its neighbours' codes [degree][wpp], its
    // factors [3][degree] and its own row as stored, rq_stride bytes per node
    const unsigned char* rq_nb;
    uint32_t rq_stride;
    uint32_t rq_off_codes;
    uint32_t rq_off_fac;
    uint32_t rq_off_row;
    uint32_t rq_lut;            // 1: estimator through a per-query nibble table
    uint32_t off_est;           // per-warp bit-planes or nibble table
    // RaBitQ visited sets: per resident warp, a bitmap of vis_words words over
    // the node ids, then a log of vis_log_cap ids set by the current query
    // (cleared word by word when the query ends); all zero between queries
    uint32_t* vis;
    uint32_t vis_words;
    uint32_t vis_log_cap;
    uint32_t vis_warps;         // warps the visited arena holds (grid cap)
};

#ifdef __CUDACC__
// One lane reports a warp's error bits: to the call's counters and to the
// index's error word.
__device__ __forceinline__ void report_errors(const SearchParams& p, unsigned err) {
    atomicOr(&p.counters->error_flags, err);
    if (p.sticky_err) atomicOr(p.sticky_err, err);
}
#endif

// Blocks of a persistent search launch: every warp pulls queries from the
// call's counter until none is left, so the grid is the resident capacity
// (or one warp per query when there are fewer queries).  Measured on the
// 1M x 128 workload (10,000 queries, 4,736 resident warps): fewer warps that
// keep the load level over three equal waves are slower (3,334 warps: 0.633
// ms against 0.591 ms), the per-query latency at lower load does not fall
// enough to pay for the idle slots.  BSEARCH_ACTIVE_WARPS (> 0) caps the
// warps, for such measurements.
inline unsigned persistent_blocks(uint64_t nq, int warps_per_block, int per_sm, int num_sms) {
    const uint64_t wpb = static_cast<uint64_t>(warps_per_block);
    const uint64_t cap = static_cast<uint64_t>(per_sm) * static_cast<uint64_t>(num_sms) * wpb;
    uint64_t warps = nq < cap ? nq : cap;
    if (const char* e = std::getenv("BSEARCH_ACTIVE_WARPS")) {
        const uint64_t v = std::strtoull(e, nullptr, 10);
        if (v > 0 && v < warps) warps = v;
    }
    return static_cast<unsigned>((warps + wpb - 1) / wpb);
}

struct LaunchShape {
    int regx;                   // beam registers per lane (beam capacity 32*regx)
    int regy;                   // candidate registers per lane (degree <= 32*regy)
    DistMode dmode;
    FilterMode fmode;
    int warps_per_block;
    size_t smem_per_warp;
    int block_query;            // 1: one thread block per query (mode base; bs_search_bq.cu)
};

// Bytes between the two block buffers of the block-per-query kernel.
#ifdef __CUDACC__
__host__ __device__
#endif
inline constexpr uint32_t bq_buffer_pitch(uint32_t nb_stride) { return (nb_stride + 127u) & ~127u; }

// Host launchers implemented in bs_search.cu.  Return cudaSuccess or the
// launch error; shape.smem_per_warp is filled by plan_search.
// Fills the regx/regy/smem fields of `shape` and the filter / staging /
// shared-memory fields of `p` from the search configuration.  On an
// unsupported configuration returns cudaErrorInvalidValue with a reason.
cudaError_t plan_search(SearchParams& p, LaunchShape& shape, size_t max_smem_optin, char* why,
                        size_t why_len);
cudaError_t launch_search(const SearchParams& p, const LaunchShape& shape, int num_sms,
                          cudaStream_t stream);
cudaError_t launch_search_rabitq(const SearchParams& p, const LaunchShape& shape, int num_sms,
                                 cudaStream_t stream);
// Neighbourhood-block variant of launch_search (p.nb set; bs_search_nb.cu).
cudaError_t launch_search_nb(const SearchParams& p, const LaunchShape& shape, int num_sms,
                             cudaStream_t stream);
// Block-per-query variant over the neighbourhood blocks (mode base;
// bs_search_bq.cu): its own shared-memory carve-up (per block, in
// shape.smem_per_warp) and launch.  BSEARCH_BQ_WARPS=2|4 fixes the warps per
// query (default: 4 when the launch's queries fit the GPU at 8 blocks per
// SM, else 2).
cudaError_t plan_search_bq(SearchParams& p, LaunchShape& shape, size_t max_smem_optin, char* why,
                           size_t why_len);
cudaError_t launch_search_bq(const SearchParams& p, const LaunchShape& shape, int num_sms, cudaStream_t stream);
// Builds the neighbourhood blocks from the gather layout (bs_search_nb.cu).
cudaError_t build_neighbourhood_blocks(const SearchParams& p, unsigned char* out, cudaStream_t stream);

// RaBitQ over node blocks (bs_rabitq_nb.cu): plan (shared-memory carve-up),
// resident warps of the planned launch (sizes the visited arena), launch, and
// the block builder (from the gather layout: adj, codes, factors, rows).
cudaError_t plan_search_rq_nb(SearchParams& p, LaunchShape& shape, size_t max_smem_optin, char* why,
                              size_t why_len);
cudaError_t rq_nb_capacity_warps(const SearchParams& p, const LaunchShape& shape, int num_sms, uint64_t& warps);
cudaError_t launch_search_rq_nb(const SearchParams& p, const LaunchShape& shape, int num_sms, cudaStream_t stream);
cudaError_t build_rabitq_blocks(const SearchParams& p, unsigned char* out, cudaStream_t stream);

// Resident warps of the RaBitQ launch for `shape` (sizes the spill tables).
cudaError_t rabitq_grid_warps(const SearchParams& p, const LaunchShape& shape, int num_sms,
                              uint64_t& warps);

// Vamana graph builder (bs_graph_build.cu): the reference build_graph's
// batch loop on the GPU over the index's rows.
struct GraphBuildArgs {
    SearchParams sp;             // rows, dims, staging and distance-path fields (score_rows)
    uint32_t degree;             // out-degree R
    uint32_t L;                  // build beam width
    float alpha;
    const uint32_t* order;       // [n] insertion order (the reference's shuffle)
    uint32_t* nbr_ids;           // [n][degree] current lists
    float* nbr_dist;             // [n][degree] their stored distances
    uint32_t* nbr_cnt;           // [n] list lengths
    uint64_t start, count;       // batch: order[start, start + count)
    unsigned long long* pool;    // [count][pool_cap] expanded (ord(dist) << 32 | node), expansion order
    uint32_t* pool_cnt;          // [count]
    uint32_t pool_cap;
    uint32_t* vis;               // per warp: bitmap over the nodes, then a log
    uint32_t vis_words, vis_log_cap, vis_warps;
    // reverse edges of the batch, sorted by destination (stable)
    const uint32_t* rev_dst;     // [count * degree], 0xffffffff past the valid ones
    const uint32_t* rev_t;       // slot * degree + position in the slot's list
    uint32_t* seg_start;         // segment starts in the sorted arrays
    uint32_t* seg_count;         // [1] number of segments
    uint32_t prune_cap;          // candidates a prune holds (shared memory)
    unsigned int* err;           // error bits (kErrPoolFull, kErrPruneFull)
    // reverse-edge prunes with more candidates than prune_cap (a node that
    // receives thousands of reverse edges in one batch) are listed here and
    // run by a second launch with kGraphBigPruneCap candidates
    uint32_t* ovf_jobs;          // [ovf_cap] segment indices
    uint32_t* ovf_count;         // [1]
    uint32_t ovf_cap;
    uint32_t ovf_pass;           // 1: this launch runs the listed segments
    uint32_t rev_prune_cap;      // first reverse launch's candidate array (0: prune_cap; tests set it small)
};
constexpr uint32_t kGraphBigPruneCap = 16384;
constexpr unsigned kErrPoolFull = 16u;    // a build search expanded more than pool_cap nodes
constexpr unsigned kErrPruneFull = 32u;   // a prune had more than prune_cap candidates

cudaError_t plan_graph_build(GraphBuildArgs& a, size_t smem_optin);
cudaError_t graph_build_batch(GraphBuildArgs& a, size_t smem_optin, int num_sms, void* sort_tmp, size_t sort_tmp_bytes,
                              uint32_t* rev_keys_in, uint32_t* rev_vals_in, uint32_t* rev_keys_out,
                              uint32_t* rev_vals_out, cudaStream_t stream);
cudaError_t graph_build_finish(GraphBuildArgs& a, size_t smem_optin, int num_sms, cudaStream_t stream);
size_t graph_build_sort_bytes(uint64_t items);
uint32_t graph_build_search_warps(const GraphBuildArgs& a, int num_sms, size_t smem_optin);

// File loaders, device side (bs_load.cu).
struct LoadScan {
    unsigned int all_int;            // 1 until a value that is not an integer is seen
    unsigned int bad_rows;           // 1: a row's header differs from the dimension
    unsigned int min_ord, max_ord;   // ordered-int encodings of the smallest / largest value
    unsigned long long neg_zero_count;
    unsigned long long neg_zero_cap;
    unsigned long long* neg_zero_pos;  // flat positions of -0.0 values (unordered)
};
cudaError_t load_fvecs_chunk(const uint32_t* raw, uint64_t rows, uint64_t first_row, uint32_t dim, uint32_t row_stride,
                             float* out, LoadScan* scan, cudaStream_t stream);
cudaError_t rows_to_u8(const float* in, uint64_t n, uint32_t dim, uint32_t row_stride, uint32_t row_bytes, uint8_t* out,
                       cudaStream_t stream);
cudaError_t load_codebook_chunk(const uint32_t* raw, uint64_t rows, uint64_t first_row, uint32_t dim, uint32_t deg,
                                uint32_t wpp, uint32_t* codes, float* factors, cudaStream_t stream);

// Exact brute-force k nearest rows (bs_ground_truth.cu).
struct GroundTruthArgs {
    SearchParams sp;             // rows, dims, integer-exact range
    const float* queries;        // [nq][dim] (device)
    uint32_t nq, k, kcap;        // kcap: power of two >= k, >= 32
    uint32_t splits;             // row ranges searched apart, then merged
    uint32_t smem_per_warp, warps_per_block, off_qb, off_qq, off_lists;
    float* part_d;               // [splits][nq][k]
    uint32_t* part_i;
    uint32_t* out_ids;           // [nq][k]
    float* out_dists;            // [nq][k] or null
};
cudaError_t plan_ground_truth(GroundTruthArgs& a, size_t smem_optin, int num_sms);
cudaError_t launch_ground_truth(const GroundTruthArgs& a, int num_sms, cudaStream_t stream);

// Merge of per-shard result lists (bs_merge.cu).
constexpr uint32_t kMaxShards = 32;
struct MergeArgs {
    const float* dists;          // [shards][nq][K], each list ascending
    const uint32_t* ids;         // [shards][nq][K], shard-local ids, 0xffffffff = none
    uint32_t shards, nq, K, K_out;
    uint32_t offsets[kMaxShards];  // global id = local id + offsets[shard]
    uint32_t* out_ids;           // [nq][K_out]
    float* out_dists;            // [nq][K_out] or null
};
cudaError_t launch_merge_shards(const MergeArgs& a, int num_sms, cudaStream_t stream);

// RaBitQ codebook builder (bs_codebook.cu).
constexpr uint32_t kMedoidBlocks = 1184;
struct CodebookArgs {
    const float* vecs;           // [n][row_stride] f32, or null
    const uint8_t* vecs8;        // [n][row_stride] u8 (exact byte copy), or null
    uint32_t row_stride;         // elements per stored row
    const uint32_t* adj;         // [n][degree]
    uint64_t n;
    uint32_t dim, degree, pdim;  // pdim: next power of two >= dim, >= 32
    const float* signs;          // [pdim] (device)
    uint32_t* codes;             // [n][degree][pdim/32]
    float* factors;              // [n][3][degree]
    uint32_t batch_rows;         // set by the launcher
    uint32_t smem_floats_per_warp;
};
size_t medoid_scratch_bytes(uint32_t dim);
cudaError_t compute_medoid(const CodebookArgs& a, uint32_t* d_result, void* d_scratch, cudaStream_t stream);
cudaError_t quantize_edges(const CodebookArgs& a, size_t smem_optin, int num_sms, cudaStream_t stream);
// rows [first, first + count) in the codebook.bin row layout into out (device)
cudaError_t pack_codebook_rows(const CodebookArgs& a, uint64_t first, uint64_t count, uint32_t* out, int num_sms,
                               cudaStream_t stream);

// Entry point (bs_entry.cu): centroid-nearest row, reference arithmetic, over
// f32 rows (vecs) or exact u8 rows (vecs8, row stride in bytes).
cudaError_t compute_entry_point(const float* vecs, uint64_t n, uint32_t dim, uint32_t row_stride,
                                uint32_t* d_result, float* d_scratch, cudaStream_t stream);
cudaError_t compute_entry_point_u8(const uint8_t* vecs8, uint64_t n, uint32_t dim, uint32_t row_bytes,
                                   uint32_t* d_result, float* d_scratch, cudaStream_t stream);
size_t entry_point_scratch_bytes(uint64_t n, uint32_t dim);

}  // namespace bsb
