/*
 * CPU oracle for the FT.SEARCH KNN hot path of Pion — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of Pion's open vector reference (Mojo), used by tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg as the checker.  It is
 * never linked into, loaded by, or called from the product library
 * (pion_b200/libpion_vector_b200.so), which has no CPU fallback.
 *
 * Parity status: UNPINNED against the reference's own outputs.  The reference
 * path is Mojo (the .mojo files under src/vector/reference/) and no Mojo toolchain exists here, and
 * the reference stores no golden vectors (its differential tests generate data
 * with Mojo's RNG).  Each function below cites the reference file:line it restates;
 * the restatement is cross-checked against an independent numpy restatement and
 * against the reference tests' invariants (tests/test_oracle.py).
 *
 * Floating-point conventions followed (x86-64-v2, the `pixi run build-open`
 * target, pixi.toml:93): no FMA contraction (src/vector/fma_mad.mojo:21-22 lowers
 * fma_mad to a*b+c there), SSE float width 4, SIMD reduce_add as a halving tree
 * (lanes [0..w/2) + [w/2..w), recursively).
 */
#ifndef PION_ORACLE_H
#define PION_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- product-key-memory routines used as FLAT INT8 inner product ---------- */
void orc_pkm_quantize_rows_i8(const float *src, int64_t n_rows, int64_t d, int64_t d_pad,
                              int8_t *dst, float *dst_scale);
void orc_pkm_scores_i8(const int8_t *keys, int64_t s_rows, int64_t d_pad, const float *row_scale,
                       const int8_t *q, const float *q_scale, int64_t nq, float *dst);
void orc_pkm_scores_f32(const float *keys, int64_t s_rows, int64_t d_pad, const float *q,
                        int64_t nq, float *dst);
void orc_pkm_rescore_f32(const float *keys, int64_t d_pad, const float *q, const int32_t *idx,
                         int64_t cnt, float *dst);
void orc_pkm_sort_desc(float *val, int32_t *idx, int64_t n);
int64_t orc_pkm_topk_max(const float *scores, int64_t n, int64_t k, int32_t *out_idx,
                         float *out_val);
int64_t orc_pkm_combine_topk(const float *s0, const int32_t *i0, int64_t k0, const float *s1,
                             const int32_t *i1, int64_t k1, int64_t s_cols, int64_t k,
                             int32_t *out_id, float *out_score);

/* Batched FLAT INT8 IP KNN = pkm_scores_i8 + pkm_topk_max per query, streamed
 * (identical results, no score matrix).  Output per query: k (idx, val), descending. */
void orc_flat_i8_knn(const int8_t *keys, int64_t n, int64_t d_pad, const float *row_scale,
                     const int8_t *q, const float *q_scale, int64_t nq, int64_t k,
                     int32_t *out_idx, float *out_val, int nthreads);

/* ---- exact FP32 rows (FLAT FP32 path) ------------------------------------ */
float orc_dot_f32_4chain(const float *q, const float *v, int64_t dim);
float orc_l2sq_f32_4chain(const float *a, const float *b, int64_t dim);
void orc_l2_normalize_fp32(const float *src, float *dst, int64_t dim);
void orc_exact_query_normalize(const float *query, float *q, int64_t dim, int cosine);
int64_t orc_exact_knn(const float *rows, int64_t n, int64_t dim, const float *query, int64_t k,
                      int cosine, int64_t *ids, float *scores);
void orc_exact_knn_batch(const float *rows, int64_t n, int64_t dim, const float *queries,
                         int64_t nq, int64_t k, int cosine, int64_t *ids, float *scores,
                         int nthreads);

/* ---- binary quantisation + FP32 rerank ---------------------------------- */
void orc_bq_pack_signs(const float *rows, int64_t n, int64_t dim, uint64_t *codes);
int64_t orc_hamming(const uint64_t *a, const uint64_t *b, int64_t words);
void orc_bq_knn_batch(const uint64_t *codes, const float *rows, int64_t n, int64_t dim,
                      const float *queries, int64_t nq, int64_t shortlist, int64_t k,
                      int64_t *ids, float *scores, int32_t *short_ids, int32_t *short_dist,
                      int nthreads);

/* ---- HNSW INT8 search (hnsw_oracle.c) ----------------------------------- */
/* A graph in the reference's compact level-0 layout plus its upper levels
 * (src/vector/hnsw.mojo:2761-2990, src/vector/beam_view.mojo:11-26). */
typedef struct orc_hnsw_layout {
    int64_t num_nodes, dim, M, entry_point, max_level;
    float global_min, global_max;
    int32_t metric, reserved;
    const int8_t *compact_buffer;
    int64_t compact_stride, compact_hdr;
    const uint32_t *l0_compact, *l0_slots, *node_slot;
    const int32_t *node_ids;
    const uint8_t *deleted;
    const int8_t *node_level;
    const int64_t *upper_offset;
    const uint32_t *upper_links;
    int64_t upper_rows;
} orc_hnsw_layout;

/* search_fp32_scored at dim 1536 (src/vector/hnsw.mojo:4136-4521) per query:
 * out_ids/out_dist [nq x k] (node_ids, pool distances; -1 / +inf past the pool),
 * stats3 += {level-0 evaluations, expansions, upper-level evaluations}.
 * Returns 0, or -1 on a layout the restatement cannot follow. */
int orc_hnsw_search(const orc_hnsw_layout *L, const float *queries, int64_t nq, int64_t k,
                    int64_t ef, int32_t *out_ids, float *out_dist, int64_t *stats3, int nthreads);
int orc_hnsw_search_ft(const orc_hnsw_layout *L, const float *queries, int64_t nq, int64_t k,
                    int64_t ef, int32_t *out_ids, float *out_dist, int64_t *stats3, int nthreads);
/* The query codes of _quantize_query_to_int8 (hnsw.mojo:657-680) after the search's
 * normalisation: codes [nq x dim]. */
void orc_hnsw_query_codes(const orc_hnsw_layout *L, const float *queries, int64_t nq,
                          int8_t *codes);

/* metric_scores (src/vector/hnsw.mojo:4523-4651) for INT8 codes: scores in/out. */
void orc_hnsw_metric_scores(const orc_hnsw_layout *L, const float *queries, int64_t nq,
                            int64_t k, const int32_t *ids, float *scores);

/* The GPU brute-force slot scan for one query (src/ffi/metal_compute.metal:19-78 and
 * pion_metal_search_topk_w, src/ffi/metal_wrap.m:495-580): entries in the order the
 * worst-replace loop leaves them.  Returns min(k, num_vectors). */
int64_t orc_slot_scan_topk(const orc_hnsw_layout *L, const int8_t *q, float qn,
                           int64_t num_vectors, int64_t k, int32_t *out_slots, float *out_d);
/* search_gpu_brute_force (src/vector/hnsw.mojo:3916-3992); rerank: FP32 rows by slot or
 * NULL. */
void orc_hnsw_brute_force(const orc_hnsw_layout *L, const float *rerank, const float *queries,
                          int64_t nq, int64_t k, int32_t *out_ids, float *out_scores,
                          int32_t *out_found);

/* beam_search_1536_ref from a caller-seeded pool (pion_v_beam_1536's contract). */
int64_t orc_hnsw_beam_pool(const orc_hnsw_layout *L, const int8_t *q, float qn, int64_t ef,
                           const float *init_d, const uint32_t *init_id, int64_t n_init,
                           int64_t cursor, float *out_d, uint32_t *out_id);

/* ---- internal: dynamic parallel-for over [0, n) with per-thread zeroed scratch */
typedef void (*orc_item_fn)(void *ctx, int64_t item, void *scratch);
void orc_parallel_for(int64_t n, int nthreads, size_t scratch_bytes, orc_item_fn fn, void *ctx);

/* ---- sharded merge ------------------------------------------------------- */
int64_t orc_shard_merge_asc(const int64_t *ids, const float *scores, int64_t n_all, int64_t k,
                            int64_t *out_ids, float *out_scores);

/* ----------------------------------------------- block-quantised HNSW (quant_oracle.c) */
#define ORC_QUANT_POLAR 0 /* INT4, stride 868 */
#define ORC_QUANT_NANO 1  /* INT2, stride 484 */
#define ORC_QUANT_TURBO 2 /* INT3 + QJL, stride 676 */

typedef struct orc_quant_layout {
    int32_t kind, metric;
    int64_t num_nodes, M, entry_point, max_level;
    const int8_t *compact; /* num_nodes x stride, slot order, header 0 */
    int64_t stride;
    const uint32_t *l0_compact, *l0_slots, *node_slot;
    const int32_t *node_ids;
    const uint8_t *deleted;
    const int8_t *node_level;
    const int64_t *upper_offset;
    const uint32_t *upper_links; /* rows of (1 + M) */
    const uint64_t *qjl;         /* num_nodes x 24, by node (TurboQuant) */
    const float *qjl_res_norms;  /* by node */
    const uint64_t *qjl_random_signs; /* 24 words */
    float qjl_lambda;
    const float *rerank;         /* num_nodes x 1536 FP32 rows by node, or NULL */
} orc_quant_layout;

uint16_t orc_f32_to_f16(float f);
float orc_f16_to_f32(uint16_t h);
int64_t orc_quant_stride(int kind);
void orc_quant_block(int kind, const float *src, int8_t *dst);
float orc_quant_dot(int kind, const int8_t *qc, const float *qs, const int8_t *v);
float orc_query_block_int8(const float *q, int8_t *codes, float *scales);
void orc_qjl_random_signs(uint64_t *out24);
float orc_qjl_signs(const float *residual, const uint64_t *rs, uint64_t *dst24);
float orc_turbo_qjl_row(const float *src, const int8_t *slot, const uint64_t *rs, uint64_t *dst24);
/* search_fp32_scored's block-quant branch per query: ids (external) / scores [nq x k],
 * out_n [nq] results per query.  0, or -1 on allocation failure. */
void orc_metric_scores_f32(const int32_t *node_ids, int64_t n, int metric, const float *rows,
                           const float *queries, int64_t nq, int64_t k, const int32_t *ids,
                           float *scores);
int orc_quant_beam_heaps(const orc_quant_layout *L, const int8_t *qc, const float *qs,
                         float qn, const uint64_t *qsig, float qres, int64_t ef, float *cand_d,
                         int64_t *cand_id, int64_t *cand_n, int64_t cand_cap,
                         int64_t *cand_total, float *res_d, int64_t *res_id, int64_t *res_n,
                         float *worst);
int orc_quant_search(const orc_quant_layout *L, const float *queries, int64_t nq, int64_t k,
                     int64_t ef, int32_t *out_ids, float *out_scores, int64_t *out_n,
                     int nthreads);

#ifdef __cplusplus
}
#endif

#endif
