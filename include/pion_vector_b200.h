/*
 * pion_vector_b200 — B200 (sm_100a) implementation of Pion's FT.SEARCH KNN hot
 * path behind a plain C ABI.
 *
 * Two groups of entry points:
 *
 *  1. The symbols Pion's engine already binds from libpion_vector
 *     (vendor/pion-vector/<platform>/MANIFEST; call sites
 *     src/vector/vector_abi.mojo:33-99 and src/vector/pkm_kernels.mojo:102-259),
 *     with the same names, argument order and meaning.  Mojo `Int` is int64_t and
 *     every pointer is a HOST pointer into engine-owned buffers; the library copies
 *     what it needs to the GPU, computes there and copies the results back.  These
 *     have no error channel in the reference; here they print a message to stderr
 *     and leave the output untouched on failure (the engine ignores their return
 *     values, src/vector/vector_abi.mojo:33-47).
 *
 *  2. New batched entry points (pion_v_b200_*) for a device-resident index:
 *     registration copies an index to the GPU once, and each query call scores a
 *     whole batch.  They return int status codes like the reference's CUDA shim
 *     (0 ok, negative error; src/ffi/cuda_kernels.cu:1330-1346) and keep the
 *     message for pion_v_b200_last_error().
 *
 * Threading: every pion_v_b200_ctx owns a CUDA stream, scratch buffers and an
 * error slot; one context per engine worker thread (the reference calls one query
 * per worker pthread, doc/architecture.md:26-36).  Registered indexes are read-only
 * and may be shared by every context on the same device.  The pion_v_* group uses
 * one context per calling thread, created on first use on device 0 (or the device
 * named by PION_B200_DEVICE).
 *
 * Ordering and ties: descending-score results (inner product) are ordered by
 * (score desc, id asc); ascending-distance results (cosine distance) by
 * (score asc, id asc).  The selected set equals the reference's whenever no two
 * candidates tie at the k-th place.
 */
#ifndef PION_VECTOR_B200_H
#define PION_VECTOR_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ status codes -- */
#define PION_B200_OK 0
#define PION_B200_EINVAL (-1)   /* bad argument (null pointer, negative size)      */
#define PION_B200_ENOMEM (-2)   /* device allocation failed                        */
#define PION_B200_ESHAPE (-3)   /* unsupported shape (dim, k, batch)               */
#define PION_B200_ENODEV (-4)   /* no usable sm_100 device                         */
#define PION_B200_ECUDA (-10)   /* CUDA launch or copy failure                     */
#define PION_B200_ETIMEOUT (-11) /* a bounded device-side wait ran out             */
#define PION_B200_EABI (-12)    /* view struct / ABI version mismatch              */

/* Where a buffer argument lives. */
#define PION_B200_MEM_HOST 0          /* host memory: copied to/from the GPU per call */
#define PION_B200_MEM_DEVICE 1        /* device memory: used in place, no copies      */
#define PION_B200_MEM_DEVICE_BORROW 2 /* registration only: keep the caller's device
                                         pointer (no copy); caller keeps it alive     */

/* Same value as VECTOR_ABI_VERSION (src/vector/vector_abi.mojo:29). */
#define PION_B200_ABI_VERSION 1

typedef struct pion_b200_ctx pion_b200_ctx;
typedef struct pion_b200_index pion_b200_index;

/* ==================================================================== group 1 */

/* src/vector/vector_abi.mojo:82-92 (vector_lib_abi / vector_abi_ok): the engine
 * refuses to start unless this equals its VECTOR_ABI_VERSION. */
int64_t pion_v_abi_version(void);

/* src/vector/vector_abi.mojo:59-79 (vector_isa): 1 = AVX-512 VNNI, 0 = x86-64-v2 in
 * the reference; this library reports 100 = CUDA sm_100a. */
int64_t pion_v_isa(void);

/* src/vector/pkm_kernels.mojo:88-105 -> ref_pkm_scores_f32
 * (src/vector/reference/pkm_ref.mojo:22-31): dst[t*s_rows + r] = <q[t], keys[r]>. */
void pion_v_pkm_scores_f32(const float *keys, int64_t s_rows, int64_t d_pad, const float *q,
                           int64_t nq, float *dst);

/* src/vector/pkm_kernels.mojo:108-126 -> ref_pkm_rescore_f32
 * (src/vector/reference/pkm_ref.mojo:34-44): dst[t] = <q, keys[idx[t]]>. */
void pion_v_pkm_rescore_f32(const float *keys, int64_t d_pad, const float *q,
                            const int32_t *idx, int64_t cnt, float *dst);

/* src/vector/pkm_kernels.mojo:129-150 -> ref_pkm_scores_i8
 * (src/vector/reference/pkm_ref.mojo:47-61):
 * dst[t*s_rows + r] = (f32(dot_i32(q[t], keys[r])) * row_scale[r]) * q_scale[t],
 * bit-identical to the reference. */
void pion_v_pkm_scores_i8(const int8_t *keys, int64_t s_rows, int64_t d_pad,
                          const float *row_scale, const int8_t *q, const float *q_scale,
                          int64_t nq, float *dst);

/* src/vector/pkm_kernels.mojo:213-236 -> ref_pkm_topk_max
 * (src/vector/reference/pkm_ref.mojo:110-130): top-k largest of scores[0:n],
 * written descending; returns min(k, n).  Same ids, values and order as the
 * reference's bounded min-heap, ties included. */
int64_t pion_v_pkm_topk_max(const float *scores, int64_t n, int64_t k, int32_t *out_idx,
                            float *out_val);

/* src/vector/pkm_kernels.mojo:199-210 -> ref_pkm_sort_desc
 * (src/vector/reference/pkm_ref.mojo:92-107): in-place min-heapsort (descending),
 * same order as the reference for equal values. */
void pion_v_pkm_sort_desc(float *val, int32_t *idx, int64_t n);

/* src/vector/pkm_kernels.mojo:238-266 -> ref_pkm_combine_topk
 * (src/vector/reference/pkm_ref.mojo:133-160). */
int64_t pion_v_pkm_combine_topk(const float *s0, const int32_t *i0, int64_t k0,
                                const float *s1, const int32_t *i1, int64_t k1, int64_t s_cols,
                                int64_t k, int32_t *out_id, float *out_score);

/* ==================================================================== group 2 */

/* Context lifecycle.  `device` < 0 picks PION_B200_DEVICE or 0.  `worker_id` is
 * recorded for messages only. */
int pion_v_b200_init(int device, int worker_id, pion_b200_ctx **out_ctx);
int pion_v_b200_shutdown(pion_b200_ctx *ctx);
/* Run this context's work on an existing CUDA stream (cudaStream_t), e.g. a
 * framework's current stream; NULL restores the context's own stream (pass
 * cudaStreamLegacy for the legacy default stream). */
int pion_v_b200_set_stream(pion_b200_ctx *ctx, void *cuda_stream);
/* Waits for the context's stream and returns the first error any device-side wait
 * recorded since the last call (PION_B200_ETIMEOUT), else 0. */
int pion_v_b200_sync(pion_b200_ctx *ctx);
/* Message of the last failing call on this context ("" if none). */
const char *pion_v_b200_last_error(const pion_b200_ctx *ctx);
/* Pre-size per-call scratch so that query calls up to these sizes allocate nothing. */
int pion_v_b200_reserve(pion_b200_ctx *ctx, int64_t max_nq, int64_t max_k);
/* Number of kernels this context has launched (for accounting in benchmarks). */
int64_t pion_v_b200_launch_count(const pion_b200_ctx *ctx);
/* Scoring-kernel timing for benchmarks: while enabled, the context records a CUDA
 * event pair on its stream around every launch of a scoring kernel (the
 * tensor-core or scan kernel that reads the index).  Enabling clears the record. */
int pion_v_b200_timing_enable(pion_b200_ctx *ctx, int enable);
/* Waits for the stream; returns the summed duration (ms) and count of the recorded
 * scoring-kernel launches. */
int pion_v_b200_timing_read(pion_b200_ctx *ctx, double *total_ms, int64_t *count);

/* FLAT INT8 inner product: rows int8[n_rows x dim]
 * (dim % 16 == 0, dim <= 16384) with a per-row fp32 scale, the output of
 * pkm_quantize_rows_i8 (src/vector/pkm_kernels.mojo:152-191).  Result ids are
 * id_base + row. */
int pion_v_b200_register_flat_i8(pion_b200_ctx *ctx, const int8_t *rows, const float *row_scale,
                                 int64_t n_rows, int64_t dim, int64_t id_base, int mem,
                                 pion_b200_index **out_index);

/* Batched FLAT INT8 IP KNN = ref_pkm_scores_i8 + ref_pkm_topk_max per query
 * (src/vector/reference/pkm_ref.mojo:47-61, :110-130) with no score matrix:
 * q int8[nq x dim], q_scale[nq] -> out_ids/out_scores [nq x k], (score desc, id asc);
 * k <= 64.  Rows past n_rows pad with id -1 and score -inf.  `mem` says where q,
 * q_scale and the outputs live. */
int pion_v_b200_flat_i8_knn(pion_b200_ctx *ctx, const pion_b200_index *index, const int8_t *q,
                            const float *q_scale, int64_t nq, int64_t k, int32_t *out_ids,
                            float *out_scores, int mem);

/* FLAT INT8 inner-product KNN that allocates no device memory.  It has no
 * counterpart in the reference.  It is for callers that cannot call cudaMalloc
 * while serving a query: an engine whose device memory is all reserved by its own
 * allocator, or a query thread that must not take cudaMalloc's device-wide
 * synchronisation.  Same selection and ordering as pion_v_b200_flat_i8_knn, but
 * every pointer is DEVICE memory and no index is registered (rows and row_scale are
 * read in place).  Its scratch is one static 8 MiB device array per GPU that loads
 * the library, held until the process exits; a call whose scratch (a 256-byte status
 * word, 4 * ceil(n_rows / 256) bytes of tile maxima and 8 * nq * lists * k bytes of
 * candidate lists, each part rounded up to 256; lists <= 128 for a batch, <= 4 * SMs
 * for one query) exceeds it returns PION_B200_ESHAPE.  The first call on
 * a device looks up the array's device address (cudaGetSymbolAddress); make that
 * first call before any stream capture.  All calls on a device share the array and
 * it keeps the last call's contents, so calls that overlap on the GPU race.  Runs on
 * `cuda_stream` (NULL: the legacy default stream) and returns once the results are
 * written: 0, or the device-side status (PION_B200_ETIMEOUT). */
int pion_v_b200_flat_i8_knn_static(const int8_t *rows, const float *row_scale, int64_t n_rows,
                                   int64_t dim, const int8_t *q, const float *q_scale, int64_t nq,
                                   int64_t k, int32_t *out_ids, float *out_scores,
                                   void *cuda_stream);

/* FLAT FP32 cosine: rows fp32[n_rows x dim].  With
 * `normalize` != 0 every row is unit-normalised on the GPU as
 * l2_normalize_fp32 does at COSINE ingest (src/vector/kernels.mojo:318-357). */
int pion_v_b200_register_flat_f32(pion_b200_ctx *ctx, const float *rows, int64_t n_rows,
                                  int64_t dim, int64_t id_base, int normalize, int mem,
                                  pion_b200_index **out_index);

/* Batched exact_knn under COSINE (src/commands/vector.mojo:1228-1365): the query is
 * normalised as exact_knn does, score = 1 - dot_f32_4chain(q^, row)
 * (src/vector/fp32_scan.mojo:17-38), k smallest by (score asc, id asc); k <= 64. */
int pion_v_b200_flat_f32_knn(pion_b200_ctx *ctx, const pion_b200_index *index, const float *q,
                             int64_t nq, int64_t k, int32_t *out_ids, float *out_scores, int mem);

/* Binary-quantised FLAT with FP32 rerank: keeps the
 * fp32 rows (normalised like register_flat_f32) and builds 1 sign bit per dimension,
 * bit b of word w = (x[64w + b] > 0) (src/vector/kernels.mojo:1711-1720). */
int pion_v_b200_register_bq(pion_b200_ctx *ctx, const float *rows, int64_t n_rows, int64_t dim,
                            int64_t id_base, int normalize, int mem, pion_b200_index **out_index);

/* Hamming shortlist of `shortlist` codes by (distance, id), Hamming = popcount of
 * XOR (src/vector/reference/quant_dots.mojo:95-100), then exact cosine rerank as
 * _exact_rescore (src/commands/vector.mojo:1413-1456), stable by score; the first k
 * are returned (score asc).  shortlist <= 256, k <= shortlist. */
int pion_v_b200_bq_rerank_knn(pion_b200_ctx *ctx, const pion_b200_index *index, const float *q,
                              int64_t nq, int64_t shortlist, int64_t k, int32_t *out_ids,
                              float *out_scores, int mem);

/* Release a registered index (and its device copies). */
int pion_v_b200_index_free(pion_b200_index *index);

/* Rows held by an index. */
int64_t pion_v_b200_index_rows(const pion_b200_index *index);

/* pkm_quantize_rows_i8 (src/vector/pkm_kernels.mojo:152-191) on the GPU, bit-identical:
 * src fp32[n_rows x d_pad] (first d columns used) -> dst int8[n_rows x d_pad], dst_scale. */
int pion_v_b200_quantize_rows_i8(pion_b200_ctx *ctx, const float *src, int64_t n_rows,
                                 int64_t d, int64_t d_pad, int8_t *dst, float *dst_scale,
                                 int mem);

/* l2_normalize_fp32 (src/vector/kernels.mojo:318-357) of every row, bit-identical. */
int pion_v_b200_l2_normalize_rows(pion_b200_ctx *ctx, const float *src, int64_t n_rows,
                                  int64_t dim, float *dst, int mem);

/* Shard merge for a row-sharded index: n_lists candidate lists per query, each of
 * k (score, id) pairs already ordered -> the k best per query (the selection rule
 * of src/commands/vector.mojo:4394-4436, with ids breaking ties).  Flags:
 * PION_B200_MERGE_DESC orders by (score desc, id asc), else (score asc, id asc);
 * PION_B200_MERGE_LISTS_MAJOR reads the input as [n_lists][nq][k] (the layout of an
 * all-gather of per-shard results) instead of [nq][n_lists][k]. */
#define PION_B200_MERGE_DESC 1
#define PION_B200_MERGE_LISTS_MAJOR 2
int pion_v_b200_merge_topk(pion_b200_ctx *ctx, const float *cand_scores, const int32_t *cand_ids,
                           int64_t nq, int64_t n_lists, int64_t k, int flags,
                           float *out_scores, int32_t *out_ids, int mem);

#ifdef __cplusplus
}
#endif
#endif /* PION_VECTOR_B200_H */
