/*
 * bsearch.h -- C ABI of the B200 graph beam-search library
 * (libbsearch_b200.so).  Plain C types only: pointers, sizes, status codes.
 *
 * The reference (SophiaSun18/beam_search_collab) has no library boundary: its
 * gpu_cli main() builds device copies of the graph and codebook and calls
 * templated launchers directly.  Each entry point below names the reference
 * piece it replaces (reference-relative file:line), so a host program written
 * against the reference structure can bind this library one to one.
 *
 * Threading: an index is bound to one CUDA device.  bs_search may run
 * concurrently on different streams; each call uses its own scratch.
 * Errors: every call returns a bs_status; bs_last_error() gives the message
 * of the calling thread's last failure.  The library never exits the process.
 */
#ifndef BSEARCH_H
#define BSEARCH_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define BS_API __attribute__((visibility("default")))
#else
#define BS_API
#endif

#define BS_NO_NODE 0xFFFFFFFFu

typedef enum bs_status {
    BS_OK = 0,
    BS_ERR_INVALID_ARGUMENT = 1, /* bad pointer, size, mode or config        */
    BS_ERR_UNSUPPORTED = 2,      /* valid but outside this build's limits     */
    BS_ERR_IO = 3,               /* file missing, short or malformed          */
    BS_ERR_OUT_OF_MEMORY = 4,    /* host or device allocation failed          */
    BS_ERR_CUDA = 5,             /* CUDA runtime error                        */
    BS_ERR_KERNEL = 6            /* a kernel reported an internal error flag  */
} bs_status;

typedef struct bs_index bs_index;

/* Host-resident graph: num_nodes rows of dim floats and of degree node ids
 * (the CPUGraph fields of reference include/cpu_graph.hpp:24-28). */
typedef struct bs_graph_desc {
    uint64_t num_nodes;
    int32_t dim;
    int32_t degree;
    const float* vectors;     /* [num_nodes][dim]    */
    const uint32_t* edges;    /* [num_nodes][degree]; NULL: no graph yet (for
                                 bs_index_build_graph)                        */
} bs_graph_desc;

/* Host-resident RaBitQ data (CPURabitqData, reference include/rabitq.hpp:25-35).
 * padded_dim = next power of two >= dim; words_per_plane = padded_dim/32. */
typedef struct bs_rabitq_desc {
    uint32_t entry_point;     /* BS_NO_NODE: none stored                      */
    int32_t padded_dim;
    const uint32_t* codes;    /* [num_nodes][degree][padded_dim/32]            */
    const float* factors;     /* [num_nodes][3][degree] triple_x|factor_dq|factor_vq */
    const float* signs;       /* [padded_dim]                                 */
} bs_rabitq_desc;

/* Search configuration: the "search" object of the reference JSON config
 * (src/gpu_cli.cu:414-452).  mode is one of "base", "warp1", "warp2",
 * "warp4", "warp8", "bwarp1", "bwarp2", "bwarp4", "bwarp8", "rabitq". */
typedef struct bs_search_params {
    const char* mode;
    int32_t K;
    uint32_t topk_size;
    uint32_t filter_capacity;
    int32_t max_iterations;
    int32_t reset_interval;
    uint32_t entry_point;     /* BS_NO_NODE: the index's default entry        */
} bs_search_params;

typedef struct bs_stats {
    uint64_t expansions;      /* nodes expanded, all queries                  */
    uint64_t distances;       /* exact L2 distances computed                  */
    uint64_t estimates;       /* RaBitQ estimates computed                    */
    uint64_t rerank;          /* exact distances in the RaBitQ final rerank   */
    uint32_t error_flags;     /* kernel-side error bits (0 = none)            */
    uint32_t entry_point;     /* entry node the search used                   */
    uint32_t integer_exact;   /* 1: integer-exact distance path was used       */
    uint32_t row_bytes;       /* bytes per base row as stored on the device   */
    uint32_t block_bytes;     /* bytes per node block copied per expansion
                                 (neighbourhood block, or the RaBitQ node
                                 block; 0: the gather layout was used)       */
    uint32_t warps_per_query; /* warps that worked on each query: 1 for the
                                 warp-per-query kernels, 2 or 4 for mode base
                                 over neighbourhood blocks (one thread block
                                 per query)                                  */
} bs_stats;

/* Fills the reference defaults: mode "base", K 100, topk_size 256,
 * filter_capacity 1024, max_iterations 1024, reset_interval 16
 * (src/gpu_cli.cu:415-452). */
BS_API void bs_search_params_default(bs_search_params* p);

/* Replaces GPUGraph::GPUGraph(const CPUGraph&) (include/gpu_graph.cuh:126-141):
 * copies vectors and edges to `device`.  The caller keeps its host arrays. */
BS_API bs_status bs_index_create(const bs_graph_desc* desc, int device, bs_index** out);

/* Replaces CPUGraph::load (include/cpu_graph.hpp:125-173) + GPUGraph: reads
 * graph.bin (int32 n, int32 degree, uint32[n*degree]) and base .fvecs. */
BS_API bs_status bs_index_load(const char* graph_bin, const char* base_fvecs, int device,
                               bs_index** out);

/* Replaces GPURabitq::GPURabitq(const CPURabitqData&) (include/rabitq.cuh:84-104). */
BS_API bs_status bs_index_attach_rabitq(bs_index* index, const bs_rabitq_desc* desc);

/* Replaces load_rabitq_codebook (include/rabitq.hpp:49-97) + GPURabitq. */
BS_API bs_status bs_index_load_codebook(bs_index* index, const char* codebook_path);

/* Replaces the reference codebook builder (src/build_rabitq.cpp:120-285),
 * on the GPU over the index's own rows and graph: sign table from
 * std::mt19937_64(seed) as build_rabitq -seed, medoid entry point, per-edge
 * codes and factors with the same arithmetic (bit-identical).  The result is
 * attached to the index as bs_index_load_codebook would attach it; when
 * out_path is non-NULL it is also written there in the codebook.bin format,
 * byte-identical to the reference tool's file.  entry_out (nullable)
 * receives the medoid.  Needs padded_dim >= 32 (dim > 16). */
BS_API bs_status bs_index_build_codebook(bs_index* index, uint32_t seed, const char* out_path,
                                         uint32_t* entry_out);

BS_API bs_status bs_index_info(const bs_index* index, uint64_t* num_nodes, int32_t* dim,
                               int32_t* degree);

/* Parameters of the graph builder (the reference build_graph's options,
 * src/build_graph.cpp:22-31; --metric ip is not supported). */
typedef struct bs_graph_build_params {
    int32_t beam_width;       /* build beam width L (reference default 128)  */
    float alpha;              /* pruning alpha >= 1 (reference default 2.0)  */
    uint32_t seed;            /* insertion-order shuffle seed (default 1234) */
} bs_graph_build_params;

/* Replaces the reference Vamana builder build_graph (src/build_graph.cpp:
 * 255-397), on the GPU over the index's own rows: the same insertion order
 * (std::mt19937(seed) + std::shuffle from the same standard library), batch
 * schedule, greedy searches, robust prune and reverse edges, so the result is
 * the reference's graph.bin.  The index's degree is the out-degree R (<= 64);
 * create the index with edges == NULL.  The new adjacency replaces the
 * index's; a codebook and the neighbourhood blocks built for the old one are
 * dropped.  edges_out (host, nullable) receives [num_nodes][degree]. */
BS_API bs_status bs_index_build_graph(bs_index* index, const bs_graph_build_params* params, uint32_t* edges_out);

/* Replaces compute_entry_point (src/gpu_cli.cu:55-83): row nearest to the
 * float centroid, same arithmetic, computed on the GPU and cached. */
BS_API bs_status bs_index_entry_point(bs_index* index, uint32_t* entry);

/* The codebook's stored entry (medoid), BS_NO_NODE when absent or when no
 * codebook is attached (reference src/gpu_cli.cu:436-437). */
BS_API bs_status bs_index_rabitq_entry(const bs_index* index, uint32_t* entry);

/* Replaces the ground-truth files the reference reads (src/gpu_cli.cu:379-381,
 * made offline by script/unpack.py): the exact k nearest rows of every query
 * by brute force over all the index's rows, ordered by (distance, id), with
 * the search's own distances (the reference's sequential fp32 sums, or exact
 * integer sums for byte rows and integer queries).  k <= 256.  queries
 * [nq][dim], ids [nq][k] and dists [nq][k] (nullable) may be host or device
 * pointers; with any host buffer the call returns when the results are in
 * place, otherwise it is asynchronous on `stream`. */
BS_API bs_status bs_ground_truth(bs_index* index, const float* queries, uint32_t nq, uint32_t k, uint32_t* ids,
                                 float* dists, void* stream);

/* No counterpart in the reference.  Builds the device layout the exact and
 * Bloom modes search fastest on (one contiguous neighbourhood block per node:
 * its adjacency row and its neighbours' rows, one bulk copy per expansion;
 * C2: 4.2 KB per node), when it fits in 40% of the free device memory.
 * bs_search does this on its first exact or Bloom search; call it at set-up
 * to take that cost out of the first search, or before bs_search_no_alloc,
 * which never builds it (until then it searches the plain layout, with the
 * same results).  A RaBitQ-only index never needs it.  "rabitq" checks that
 * a codebook is attached (its node blocks are built when it is attached). */
BS_API bs_status bs_index_prepare(bs_index* index, const char* mode);

/* No counterpart in the reference, whose kernels have no error channel.
 * Every search kernel on this index also ORs its error bits (the ones
 * bs_search reports as BS_ERR_KERNEL) into a word held by the index, so that a
 * caller of asynchronous searches -- bs_search with device buffers and no
 * stats, or bs_search_no_alloc -- can collect them later: this call copies
 * the word to *flags and clears it, ordered after the work already queued on
 * `stream`, and synchronises `stream`.  Bits: 1 a visited-table probe ran the
 * whole table, 2 a RaBitQ visited table overflowed, 4 a block copy's wait
 * gave up, 8 that copy never landed.  0 means no kernel reported an error. */
BS_API bs_status bs_index_take_errors(bs_index* index, void* stream, uint32_t* flags);

BS_API void bs_index_destroy(bs_index* index);

/* Replaces run_base / run_warp / run_rabitq and their kernels
 * (src/gpu_cli.cu:87-349): searches nq queries ([nq][dim] floats), writes
 * ids [nq][K] (BS_NO_NODE past the end of the beam) and, when `dists` is not
 * NULL, the matching squared L2 distances.  `queries`, `ids` and `dists` may
 * each be host or device pointers.  Pageable host buffers are copied inside
 * the call; page-locked host buffers mapped into the index's device (e.g.
 * cudaHostAlloc / cudaMallocHost on that device) are read and written in
 * place by the search kernel, so their transfers overlap the search.  With
 * any host buffer the call returns only when the results are in place.  With device
 * buffers only and stats == NULL the call is asynchronous on `stream`
 * (a cudaStream_t; NULL = legacy default stream). */
BS_API bs_status bs_search(bs_index* index, const bs_search_params* params, const float* queries,
                           uint32_t nq, uint32_t* ids, float* dists, bs_stats* stats,
                           void* stream);

/* No counterpart in the reference.  The same search as bs_search for the
 * exact and Bloom modes (every mode but "rabitq"), for callers that cannot
 * allocate device memory while they run -- a process that reserves the GPU's
 * memory at start-up and forbids later allocations (fixed-budget serving, a
 * plugin inside a runtime that owns all device memory), or a loop where an
 * allocation's possible blocking or failure is not acceptable.  It calls no
 * cudaMalloc/cudaFree or allocating routine: the kernel's scratch (work
 * counter, statistics, error flags; the centroid when the entry point is
 * first computed) lives in one 16 KiB file-scope device array that every GPU
 * loading the library holds until the process exits.
 *   - queries, ids and dists (NULL allowed) must be device pointers;
 *   - nq <= 2^31; "rabitq" is rejected (its never-forgetting visited sets
 *     need a bitmap over all node ids per resident warp, far more than the
 *     fixed scratch), as is computing the entry point for dim > 4028 (pass
 *     entry_point or call bs_index_entry_point first);
 *   - it searches the layout the index already has: the neighbourhood blocks
 *     once bs_index_prepare (or an exact or Bloom bs_search) built them, else
 *     the plain layout, with the same results;
 *   - the first call on a device looks up the array's device address, and if
 *     neither entry_point nor a cached entry is available it computes the
 *     entry point and synchronises `stream`; make that first call before any
 *     stream capture;
 *   - all calls share the one array, which keeps the last call's contents
 *     (the counters are cleared at the start of every call): calls that
 *     overlap on the GPU race, so serialise them (one stream, or events);
 *   - asynchronous on `stream`; no statistics are returned (kernel error
 *     bits reach the index's error word: bs_index_take_errors). */
BS_API bs_status bs_search_no_alloc(bs_index* index, const bs_search_params* params, const float* queries,
                                    uint32_t nq, uint32_t* ids, float* dists, void* stream);

/* No counterpart in the reference, which searches one index on one GPU: the
 * merge step of a sharded index (one shard per GPU, each with its own graph
 * over its own rows; every query searched on every shard).  Input: the
 * shards' result lists gathered into dists[shards][nq][K] and
 * ids[shards][nq][K] (shard-local ids, BS_NO_NODE past the end, each list
 * ascending by (distance, id) as bs_search returns it), device pointers on
 * the current device.  Output: out_ids[nq][K_out] (and out_dists when not
 * NULL), the K_out smallest (distance, global id) entries over all shards,
 * global id = local id + id_offsets[shard] (a host array of `shards` values;
 * global ids must stay below 0xffffffff), BS_NO_NODE / FLT_MAX past the end.
 * shards <= 32, K_out <= shards * K.  Asynchronous on `stream`. */
BS_API bs_status bs_merge_shards(const float* dists, const uint32_t* ids, uint32_t shards, uint32_t nq,
                                 uint32_t K, const uint32_t* id_offsets, uint32_t K_out, uint32_t* out_ids,
                                 float* out_dists, void* stream);

/* Device buffers on the index's device (for callers that stage queries once
 * and search many times, like the reference CLI's timed loop,
 * src/gpu_cli.cu:400-421). */
BS_API bs_status bs_device_alloc(const bs_index* index, size_t bytes, void** dptr);
BS_API bs_status bs_device_free(const bs_index* index, void* dptr);
BS_API bs_status bs_copy_to_device(const bs_index* index, void* dst, const void* src, size_t bytes);
BS_API bs_status bs_copy_to_host(const bs_index* index, void* dst, const void* src, size_t bytes);
BS_API bs_status bs_device_fill(const bs_index* index, void* dptr, int byte_value, size_t bytes);
BS_API bs_status bs_synchronize(const bs_index* index, void* stream);

BS_API const char* bs_last_error(void);
BS_API const char* bs_version(void);

#ifdef __cplusplus
}
#endif
#endif /* BSEARCH_H */
