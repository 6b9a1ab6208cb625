/*
 * bs_oracle.h -- CPU restatement of the reference beam search, used ONLY as a
 * test / benchmark checker.  Nothing in the product links this library.
 *
 * Every function cites the reference file:line it restates (paths relative to
 * the reference project root).  Arithmetic is plain fp32 in the reference's
 * evaluation order with FMA contraction disabled, so results are bit-identical
 * to the reference cpu_cli built for baseline x86-64.
 */
#ifndef BS_ORACLE_H
#define BS_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    uint64_t expansions;     /* nodes expanded (E)                               */
    uint64_t distances;      /* exact L2 distances computed (D), entry included   */
    uint64_t estimates;      /* RaBitQ estimates computed                         */
    uint64_t rerank;         /* exact distances in the final RaBitQ rerank (T)    */
} orc_stats;

/* src/cpu_cli.cpp:35-62 (== src/gpu_cli.cu:55-83): float centroid, first
 * row with the smallest squared distance to it. */
uint32_t orc_entry_point(const float* base, uint64_t n, int dim);

/* Sequential fp32 squared L2 (include/cpu_search_base.hpp:29-37). */
float orc_l2(const float* a, const float* b, int dim);

/* include/cpu_search_base.hpp:22-82 -- CPUBaseSearch::search.
 * out_dists may be NULL.  Returns 0, or -1 on allocation failure. */
int orc_search_base(const float* base, uint64_t n, int dim,
                    const uint32_t* edges, int degree,
                    const float* query, int topk_size, uint32_t entry,
                    int max_iterations, int K,
                    uint32_t* out_ids, float* out_dists, orc_stats* st);

/* Same beam search with the Bloom visited filter of the bwarpN modes
 * (hashes of include/filter_bloom.cuh:25-38; batch semantics per expansion,
 * reset + beam reinsert every reset_interval expansions). */
int orc_search_bloom(const float* base, uint64_t n, int dim,
                     const uint32_t* edges, int degree,
                     const float* query, int topk_size, uint32_t entry,
                     int max_iterations, int K,
                     uint32_t filter_bits, int reset_interval,
                     uint32_t* out_ids, float* out_dists, orc_stats* st);

/* include/cpu_search_rabitq.hpp:34-57 -- rotate (signs, WHT), 6-bit query
 * quantizer with lroundf(x*inv_w + 0.5) (values 1..64).  q_out has pdim bytes. */
void orc_rabitq_quantize(const float* query, int dim, const float* signs, int pdim,
                         uint8_t* q_out, float* low, float* width, int32_t* sum_q);

/* include/cpu_search_rabitq.hpp:72-97 -- integer part of the estimator:
 * sum of q_d over dims whose code bit is set. */
uint32_t orc_rabitq_raw(const uint8_t* quant, const uint32_t* code, int pdim);

/* include/cpu_search_rabitq.hpp:28-150 -- CPURabitqSearch::search.
 * codes: [n][degree][wpp] u32, factors: [n][3][degree] f32, signs: [pdim]. */
int orc_search_rabitq(const float* base, uint64_t n, int dim,
                      const uint32_t* edges, int degree,
                      const uint32_t* codes, const float* factors,
                      const float* signs, int pdim,
                      const float* query, int topk_size, uint32_t entry,
                      int max_iterations, int K,
                      uint32_t* out_ids, float* out_dists, orc_stats* st);

/* Batch drivers over nq queries with nthreads POSIX threads (0 = 1).
 * mode 0 = base, 1 = bloom, 2 = rabitq.  stats (if non-NULL) are summed. */
typedef struct {
    const float* base; uint64_t n; int dim;
    const uint32_t* edges; int degree;
    const uint32_t* codes; const float* factors; const float* signs; int pdim;
    int topk_size; uint32_t entry; int max_iterations; int K;
    uint32_t filter_bits; int reset_interval;
    int mode;
} orc_batch_cfg;

int orc_search_batch(const orc_batch_cfg* cfg, const float* queries, uint64_t nq,
                     uint32_t* out_ids, float* out_dists, orc_stats* st, int nthreads);

/* src/cpu_cli.cpp:18-33: unique predictions found anywhere in the gt row,
 * divided by nq*K. */
double orc_recall_cpu(const uint32_t* pred, const int32_t* gt, uint64_t nq, int K, int gt_k);
/* src/gpu_cli.cu:28-51: skips -1, counts duplicates, divides by nq*min(K,gt_k). */
double orc_recall_gpu(const uint32_t* pred, const int32_t* gt, uint64_t nq, int K, int gt_k,
                      uint64_t* duplicates);

#ifdef __cplusplus
}
#endif
#endif
