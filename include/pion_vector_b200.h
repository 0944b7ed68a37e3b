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
/* Or'ed into `mem` of pion_v_b200_flat_i8_knn with PION_B200_MEM_DEVICE: out_scores
 * receives nq x k interleaved 8-byte (f32 score, i32 id) pairs (8-byte aligned) -- the
 * layout one row shard exchanges with the others -- and out_ids is ignored. */
#define PION_B200_OUT_PAIRS 0x100

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

/* src/common/heap.mojo:133-160: LinearPool's fields, in order (entries are 8-byte
 * (f32 dist, u32 id) pairs, bit 31 of id = expanded). */
typedef struct pion_linear_pool {
    void *entries;
    int64_t capacity;
    int64_t size;
    int64_t cursor;
    int64_t ef;
} pion_linear_pool;

/* src/vector/beam_view.mojo:11-26: BeamView1536's fields, in order. */
typedef struct pion_beam_view_1536 {
    pion_linear_pool *pool;
    int64_t ef;
    float query_norm_sq;
    float query_prefix_norm_sq;
    const int8_t *query_int8;
    const uint32_t *l0_compact;
    const uint32_t *l0_slots;
    int64_t num_nodes;
    const uint8_t *deleted;
    uint16_t *visited;
    uint16_t cur_epoch;
    const int8_t *compact_buffer;
    int64_t compact_stride;
    int64_t compact_hdr;
    const void *nodes;
} pion_beam_view_1536;

/* src/vector/vector_abi.mojo:31-36 (beam_search_1536) -> beam_search_1536_ref
 * (src/vector/reference/beam_1536.mojo:85-135): the level-0 beam of one query, on the GPU.
 * Reads the view's pool (as search_fp32_scored seeds it: the start node, marked visited),
 * runs the beam and writes the pool back entry for entry (ids with their expanded bit,
 * distances, size; cursor = size), exactly as the reference would leave it.  The graph
 * (l0_compact, l0_slots, compact_buffer) is copied to the GPU on the first call for those
 * buffers and reused while the same pointers and sizes come back; call
 * pion_v_b200_beam_forget after changing them in place.  The visited array is not
 * written (the engine starts a new epoch per query).  Returns 0, or a negative code with
 * a message on stderr. */
int64_t pion_v_beam_1536(pion_beam_view_1536 *view);

/* src/common/heap.mojo:6-30, 48-56, 237-241: HeapNode (f32 distance, Int id), and the
 * List[HeapNode] MinHeap and MaxHeap keep (the Mojo List's fields: data, length,
 * capacity), MaxHeap's cached worst distance after it. */
typedef struct pion_heap_node {
    float distance;
    int32_t pad;
    int64_t id;
} pion_heap_node;

typedef struct pion_heap_list {
    pion_heap_node *data;
    int64_t len;
    int64_t capacity;
} pion_heap_list;

typedef struct pion_min_heap {
    pion_heap_list data;
} pion_min_heap;

typedef struct pion_max_heap {
    pion_heap_list data;
    float cached_worst;
    int32_t pad;
} pion_max_heap;

/* src/vector/quant_beam_view.mojo:22-47: QuantBeamView1536's fields, in order. */
typedef struct pion_quant_beam_view_1536 {
    int64_t kind; /* 0 PolarQuant INT4, 1 NanoQuant INT2, 2 TurboQuant INT3 + QJL */
    int64_t ef;
    pion_min_heap *candidates;
    pion_max_heap *results;
    const int8_t *query_block_int8;   /* 1536 codes          */
    const float *query_block_scales;  /* 48 block scales     */
    float query_block_norm;
    const uint32_t *l0_compact;
    const uint32_t *l0_slots;
    int64_t num_nodes;
    const uint8_t *deleted;
    uint16_t *visited;
    uint16_t cur_epoch;
    const int8_t *compact_buffer;
    int64_t compact_stride;
    int64_t compact_hdr;
    const void *nodes;
    const uint64_t *qjl_buffer;       /* num_nodes x 24, by node */
    const float *qjl_res_norms;       /* num_nodes, by node      */
    const uint64_t *qjl_query_signs;  /* 24                      */
    float qjl_query_res_norm;
    float qjl_lambda;
} pion_quant_beam_view_1536;

/* src/vector/vector_abi.mojo:40-46 (quant_beam_search_1536) -> quant_beam_search_1536_ref
 * (src/vector/reference/quant_beams_1536.mojo:20-81): the level-0 beam of one query over
 * the block-quantised slots, on the GPU.  Starts from the view's heaps (as the block-quant
 * branches of search_fp32_scored seed them: the start node in both, marked visited; the
 * nodes in the heaps count as visited), runs the beam over MinHeap / MaxHeap exactly as
 * the reference does, and writes both heaps back array for array (the results heap and
 * its cached worst in full; the candidates heap up to its List's capacity, a prefix of a
 * binary heap being a heap: the engine clears it before its next use and a C library
 * cannot grow a Mojo List).  The graph (l0_compact, l0_slots, the slots at compact_buffer
 * + slot * compact_stride + compact_hdr, the QJL rows) is copied to the GPU on the first
 * call for those buffers and reused while the same pointers and sizes come back
 * (pion_v_b200_beam_forget drops it).  Every l0_slots entry of a listed node must name a
 * slot (the nodes' own vector pointers are not read).  The visited array is not written.
 * Returns 0, or a negative code with a message on stderr (the heaps are then unchanged). */
int64_t pion_v_quant_beam_1536(pion_quant_beam_view_1536 *view);

/* Drops the GPU copy of a graph registered by pion_v_beam_1536 or pion_v_quant_beam_1536
 * (all of them when l0_compact is NULL). */
int pion_v_b200_beam_forget(const uint32_t *l0_compact);

/* ==================================================================== group 2 */

/* Context lifecycle.  `device` < 0 picks PION_B200_DEVICE or 0.  `worker_id` is
 * recorded for messages only. */
int pion_v_b200_init(int device, int worker_id, pion_b200_ctx **out_ctx);
int pion_v_b200_shutdown(pion_b200_ctx *ctx);
/* Run this context's work on an existing CUDA stream (cudaStream_t), e.g. a
 * framework's current stream; NULL restores the context's own stream (pass
 * cudaStreamLegacy for the legacy default stream).  Work queued after a switch waits
 * for the work already queued on the previous stream (the context's scratch is
 * shared), without blocking the host. */
int pion_v_b200_set_stream(pion_b200_ctx *ctx, void *cuda_stream);
/* Waits for the context's stream and returns the first error any device-side wait
 * recorded since the last call (PION_B200_ETIMEOUT), else 0.  A call with host buffers
 * checks its own kernels' waits before it returns; a call with device buffers returns
 * once its kernels are queued, so its waits are reported here (they are never reported
 * as a later host-buffer call's failure). */
int pion_v_b200_sync(pion_b200_ctx *ctx);
/* Budget of each device-side wait in this context's FLAT INT8 tensor-core kernels, in
 * ns (<= 0 restores the default of 2 s).  A wait that runs out records
 * PION_B200_ETIMEOUT; the kernel then drains its copies and MMAs, frees its tensor
 * memory and returns, so the context stays usable.  (For tests, the environment
 * variable PION_B200_TEST_STALL=1 makes one CTA of each main pass wait on a barrier that
 * nothing arrives on.) */
int pion_v_b200_set_wait_budget(pion_b200_ctx *ctx, int64_t ns);
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
 * scoring-kernel launches (= pion_v_b200_timing_read_tag(ctx, PION_B200_TIMING_SCORING)). */
int pion_v_b200_timing_read(pion_b200_ctx *ctx, double *total_ms, int64_t *count);
/* The same for one phase.  SCORING spans every kernel that reads the index in one call;
 * inside it the FLAT INT8 tensor-core path also records its threshold pass (the sampled
 * bound and its merge) and its main pass separately. */
#define PION_B200_TIMING_SCORING 0
#define PION_B200_TIMING_THRESHOLD 1
#define PION_B200_TIMING_MAIN 2
/* pion_v_b200_flat_i8_knn_sharded: each exchange (publish, wait, merge), and within it the
 * wait-and-merge kernel alone (which holds the time spent waiting for the other ranks). */
#define PION_B200_TIMING_EXCHANGE 3
#define PION_B200_TIMING_EXCHANGE_WAIT 4
int pion_v_b200_timing_read_tag(pion_b200_ctx *ctx, int tag, double *total_ms, int64_t *count);

/* ------------------------------------------------------------ any index kind -- */
#define PION_B200_KIND_FLAT_I8 1  /* rows int8 [n x dim] + row_scale: register_flat_i8 */
#define PION_B200_KIND_FLAT_F32 2 /* rows fp32 [n x dim]: register_flat_f32 */
#define PION_B200_KIND_BQ 3       /* rows fp32 [n x dim]: register_bq */
#define PION_B200_KIND_HNSW 4     /* hnsw layout: register_hnsw */
#define PION_B200_KIND_HNSW_QUANT 5 /* hnsw + hnsw_quant layouts: register_hnsw_quant */

typedef struct pion_b200_index_desc {
    int32_t kind;            /* PION_B200_KIND_* */
    int32_t mem;             /* PION_B200_MEM_* of rows / row_scale */
    int64_t n_rows, dim, id_base;
    int32_t normalize;       /* FLAT_F32, BQ: normalise rows at ingest (COSINE) */
    int32_t reserved;
    const void *rows;
    const float *row_scale;  /* FLAT_I8 */
    const struct pion_b200_hnsw_layout *hnsw; /* HNSW, HNSW_QUANT */
    const struct pion_b200_hnsw_quant_layout *quant; /* HNSW_QUANT */
} pion_b200_index_desc;

/* One registration entry point for every index kind: dispatches on desc->kind to the
 * kind's own register call with the same arguments (and errors). */
int pion_v_b200_register_index(pion_b200_ctx *ctx, const pion_b200_index_desc *desc,
                               pion_b200_index **out_index);

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

/* merge_delta (src/commands/vector.mojo:1368-1456) for a batch: `index` is a FLAT FP32
 * index of the ingest rows [0, rows) registered at slot 0 (normalised at ingest under
 * COSINE); the graph holds slots [0, built).  ids / scores [nq x kg]: each query's graph
 * results (a -1 id ends a list), rescored in place as _exact_rescore does (slots below
 * built: 1 - dot_f32_4chain(q^, row) under COSINE, l2sq_f32_4chain(q, row) under L2;
 * then the stable insertion sort).  The rows [built, rows) are scanned exactly
 * (exact_knn, k smallest by (score, slot)) and merged: a graph entry first when its score
 * <= the delta entry's, k kept.  metric: 1 = COSINE, 0 = L2.  out_ids / out_scores
 * [nq x k] (-1 / +inf past the lists); kg <= 1024, k <= 64. */
int pion_v_b200_merge_delta(pion_b200_ctx *ctx, const pion_b200_index *index, int64_t built,
                            int metric, const float *q, int64_t nq, int64_t kg, int32_t *ids,
                            float *scores, int64_t k, int32_t *out_ids, float *out_scores,
                            int mem);

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
 * all-gather of per-shard results) instead of [nq][n_lists][k];
 * PION_B200_MERGE_PAIRS reads cand_scores as interleaved 8-byte (f32 score, i32 id)
 * pairs (one buffer, so a shard exchanges its results in one collective) and ignores
 * cand_ids, which may be NULL. */
#define PION_B200_MERGE_DESC 1
#define PION_B200_MERGE_LISTS_MAJOR 2
#define PION_B200_MERGE_PAIRS 4
int pion_v_b200_merge_topk(pion_b200_ctx *ctx, const float *cand_scores, const int32_t *cand_ids,
                           int64_t nq, int64_t n_lists, int64_t k, int flags,
                           float *out_scores, int32_t *out_ids, int mem);

/* ---------------------------------------------------- row-shard exchange -- */
/* One process per GPU, each holding a row shard (registered with id_base = its first
 * row): the shards' per-query k (score, id) pairs cross NVLink as peer stores into every
 * rank's receive buffer (shared through CUDA IPC handles), a flag per rank and step marks
 * them complete, and every rank merges the world lists itself -- the all-gather + merge
 * of src/commands/vector.mojo:4394-4436 without a collective call.  Set-up: create on
 * every rank, exchange the PION_B200_IPC_HANDLE_BYTES handles by any channel (e.g.
 * torch.distributed), connect with the world's handles (rank order).  Waits are bounded
 * by the context's wait budget (pion_v_b200_set_wait_budget): a missing peer turns into
 * PION_B200_ETIMEOUT from pion_v_b200_sync, not a hang.  `regions` independent uses per
 * step (<= 4), each double-buffered by the step's parity. */
#define PION_B200_IPC_HANDLE_BYTES 64
typedef struct pion_b200_exchange pion_b200_exchange;
int pion_v_b200_exchange_create(pion_b200_ctx *ctx, int world, int rank, int regions,
                                int64_t max_nq, int64_t k, pion_b200_exchange **out);
int pion_v_b200_exchange_handle(const pion_b200_exchange *ex, void *out_handle);
int pion_v_b200_exchange_connect(pion_b200_exchange *ex, const void *handles);
int pion_v_b200_exchange_free(pion_b200_exchange *ex);
/* The exchange's world size once connected, else -1. */
int pion_v_b200_exchange_world(const pion_b200_exchange *ex);
/* This rank's `pairs` (device, nq x k interleaved (f32 score, i32 id)) to every rank, then
 * the merged k best per query of all ranks' lists (PION_B200_MERGE_DESC for largest-first)
 * into out_scores / out_ids, or into out_scores as pairs with PION_B200_OUT_PAIRS.  `epoch`
 * (>= 1) numbers the step and must advance by one per call on every rank. */
int pion_v_b200_exchange_merge(pion_b200_ctx *ctx, pion_b200_exchange *ex, const void *pairs,
                               int64_t nq, int64_t k, uint32_t epoch, int flags,
                               float *out_scores, int32_t *out_ids);
/* Row-sharded FLAT INT8 KNN in one call (device memory, the exchange created with 2
 * regions): this rank scores its share of the threshold sample, the ranks exchange and
 * merge those k-lists into one bound per query (the k-th best of the union of every
 * rank's sample: a lower bound of the global k-th score), every rank scores its whole
 * shard from that bound, and the ranks exchange and merge their k-lists: out_scores /
 * out_ids (or pairs with PION_B200_OUT_PAIRS) hold the global top k by (score desc, id
 * asc) on every rank.  With PION_B200_SHARD_LOCAL_BOUND each rank starts its shard from
 * the k-th best of its own sample share instead (no exchange before the main pass: one
 * exchange per call; the same results). */
#define PION_B200_SHARD_LOCAL_BOUND 0x200
int pion_v_b200_flat_i8_knn_sharded(pion_b200_ctx *ctx, const pion_b200_index *ix,
                                    pion_b200_exchange *ex, const int8_t *q, const float *q_scale,
                                    int64_t nq, int64_t k, uint32_t epoch, int flags,
                                    int32_t *out_ids, float *out_scores);

/* ------------------------------------------------------------------- HNSW -- */

/* An HNSW INT8 graph in the reference's compact level-0 layout: the buffers that
 * compact_vectors and _build_l0_slots produce (src/vector/hnsw.mojo:2761-2990) and
 * that BeamView1536 hands to the beam (src/vector/beam_view.mojo:11-26), plus the
 * upper levels the greedy descent walks (src/vector/hnsw.mojo:3789-3848).  Node
 * indices are the graph's internal indices (0 <= node < num_nodes). */
typedef struct pion_b200_hnsw_layout {
    int64_t num_nodes;
    int64_t dim;             /* 1536 (the beam is the 1536-dim routine)             */
    int64_t M;               /* level-0 lists hold <= 2M <= 32, upper lists <= M     */
    int64_t entry_point;     /* node                                                 */
    int64_t max_level;       /* level of the entry point                             */
    float global_min;        /* SQ8 calibration range (_calibrate, hnsw.mojo:578)    */
    float global_max;
    int32_t metric;          /* 0 = L2, 1 = COSINE (queries are unit-normalised)     */
    int32_t reserved;
    const int8_t *compact_buffer;  /* num_nodes x compact_stride: per slot an 8-byte
                                      header (f32 |code|^2, f32 |code[0:256]|^2) then
                                      the dim int8 codes                             */
    int64_t compact_stride;        /* multiple of 16, >= compact_hdr + dim           */
    int64_t compact_hdr;           /* 8                                              */
    const uint32_t *l0_compact;    /* num_nodes x 33: count, level-0 neighbour nodes */
    const uint32_t *l0_slots;      /* num_nodes x 33: count, their compact slots     */
    const uint32_t *node_slot;     /* num_nodes: compact slot of each node           */
    const int32_t *node_ids;       /* num_nodes: external id returned for a node     */
    const uint8_t *deleted;        /* (num_nodes + 7) / 8 bytes, bit i = node i
                                      deleted; NULL = none                           */
    const int8_t *node_level;      /* num_nodes: level of each node                  */
    const int64_t *upper_offset;   /* num_nodes: first upper row of the node (-1 at
                                      level 0); level l >= 1 is row
                                      upper_offset[node] + l - 1                      */
    const uint32_t *upper_links;   /* upper_rows x (1 + M): count, neighbour nodes   */
    int64_t upper_rows;
} pion_b200_hnsw_layout;

typedef struct pion_b200_hnsw_graph pion_b200_hnsw_graph;

/* The reference's index file pion.hnsw.0 (HNSWGraph.save_to_disk / load_from_disk,
 * src/vector/hnsw.mojo:1209-1700; format v3 to v5, plain INT8 slots, global calibration):
 * pion_v_b200_hnsw_load reads one into a host graph whose layout
 * (pion_v_b200_hnsw_graph_layout) registers with pion_v_b200_register_hnsw, so a graph the
 * engine built serves on the GPU; l0_slots is derived as _build_l0_slots does.  Block-
 * quantised files (pion_v_b200_hnsw_load_quant) and per-group calibration are refused
 * (PION_B200_ESHAPE).
 * pion_v_b200_hnsw_save writes a graph as a v5 file the engine loads (max_elements: the
 * engine's capacity, which its loader checks; 0 = the largest external id + 1). */
int pion_v_b200_hnsw_load(const char *path, pion_b200_hnsw_graph **out_graph);
int pion_v_b200_hnsw_save(const pion_b200_hnsw_graph *graph, const char *path,
                          int64_t max_elements);

/* Builds an HNSW INT8 graph on the host CPU the way the reference's FT.OPTIMIZE does
 * (src/vector/hnsw.mojo:2540-2620: _calibrate, quantize, _level_of, the parallel link
 * lanes of _insert_to_graph_mt, the relink and _repair_l0 passes, compact_vectors),
 * from rows fp32[n_rows x dim] in HOST memory (normalised first when metric = 1).
 * Node i gets external id id_base + i.  n_threads link lanes (<= 0: every online
 * CPU); as in the reference, more than one lane makes the graph depend on thread
 * timing.  Needs a CPU with AVX2 and FMA (PION_B200_ESHAPE otherwise). */
int pion_v_b200_hnsw_build(const float *rows, int64_t n_rows, int64_t dim, int64_t M,
                           int64_t ef_construction, int metric, int64_t id_base, int n_threads,
                           pion_b200_hnsw_graph **out_graph);
/* The same build with batched insertion instead of racing link lanes: the nodes are
 * inserted in batches (a quarter of the nodes linked so far, at most max_batch >= 1); every
 * node of a batch does the search half of _insert_to_graph_mt (greedy descent,
 * _search_layer_mt at efConstruction, _prune_neighbors) against the graph as it stood
 * before the batch, n_threads at a time, then the batch is linked node by node in order
 * (own lists and evict-farthest backlinks), followed by the relink and repair passes and
 * compact_vectors.  The graph does not depend on the thread count; max_batch = 1 is the
 * one-lane build.  The searches of a batch are independent, which is the shape of the
 * work a GPU takes over. */
int pion_v_b200_hnsw_build_batched(const float *rows, int64_t n_rows, int64_t dim, int64_t M,
                                   int64_t ef_construction, int metric, int64_t id_base,
                                   int n_threads, int64_t max_batch,
                                   pion_b200_hnsw_graph **out_graph);
/* The batched build with the search half on a GPU: every batch of at least 64 nodes is
 * planned on ctx's device -- a warp per node does the greedy descent, _search_layer_mt at
 * efConstruction and _prune_neighbors (src/vector/hnsw.mojo:2032-2240, 3595-3628) against
 * the graph as it stood before the batch, with the host's heap and distance arithmetic --
 * and linked on the host in node order, so the graph is array for array the one
 * pion_v_b200_hnsw_build_batched builds with the same max_batch.  dim 1536,
 * ef_construction <= 1024.  Host memory in and out; n_threads prepare each batch's rows and
 * run the repair passes. */
int pion_v_b200_hnsw_build_gpu(pion_b200_ctx *ctx, const float *rows, int64_t n_rows,
                               int64_t dim, int64_t M, int64_t ef_construction, int metric,
                               int64_t id_base, int n_threads, int64_t max_batch,
                               pion_b200_hnsw_graph **out_graph);
/* The graph's buffers (host memory owned by the graph). */
int pion_v_b200_hnsw_graph_layout(const pion_b200_hnsw_graph *graph,
                                  pion_b200_hnsw_layout *out_layout);
/* Build counters: link lanes (minus the batch count after a batched build), contended
 * link drops, relinked under-linked nodes, nodes re-linked by the exit repair, links added
 * by the reachability repair. */
int pion_v_b200_hnsw_graph_stats(const pion_b200_hnsw_graph *graph, int64_t *out5);
/* The same five counters, then the nodes whose insertion a GPU planned. */
int pion_v_b200_hnsw_graph_stats6(const pion_b200_hnsw_graph *graph, int64_t *out6);
int pion_v_b200_hnsw_graph_free(pion_b200_hnsw_graph *graph);

/* Copies a graph (every pointer of `layout` in HOST memory) to the GPU.  Checks the
 * layout: dim 1536, 2M <= 32, counts within capacity, every neighbour and slot in
 * range. */
int pion_v_b200_register_hnsw(pion_b200_ctx *ctx, const pion_b200_hnsw_layout *layout,
                              pion_b200_index **out_index);

/* Batched HNSW search, one beam per query, the reference's search_fp32_scored at
 * dim 1536 (src/vector/hnsw.mojo:4136-4521): normalise (COSINE), quantise
 * (_quantize_query_to_int8, :657-680), greedy descent of the upper levels in exact
 * INT8 L2 (_upper_greedy_codes, :3789-3848), then the level-0 beam
 * beam_search_1536_ref (src/vector/reference/beam_1536.mojo:85-135) over a LinearPool
 * of ef entries (src/common/heap.mojo:133-234), with the same lane formulas, prefix
 * gate, tie order and pool discipline, so the pool equals the reference's entry for
 * entry.  q fp32[nq x 1536]; out_ids [nq x k] are node_ids of the first min(k, pool
 * size) pool entries (nearest first), out_dist their pool distances (squared L2 in
 * code space); the rest are -1 / +inf.  ef in [1, 1024], k >= 1. */
int pion_v_b200_hnsw_search(pion_b200_ctx *ctx, const pion_b200_index *index, const float *q,
                            int64_t nq, int64_t k, int64_t ef, int32_t *out_ids, float *out_dist,
                            int mem);

/* The level-0 beam of a batch of queries over a registered graph, each from a pool the
 * caller seeded: the batched form of pion_v_beam_1536 (beam_search_1536_ref,
 * src/vector/reference/beam_1536.mojo:85-135, on LinearPool, src/common/heap.mojo:133-234).
 * q_codes int8 [nq x 1536] (the codes _quantize_query_to_int8 produced), q_norm [nq] (the
 * view's query_norm_sq); pools [nq x ef] of 8-byte (f32 dist, u32 node | 0x80000000 when
 * expanded) entries; pool_size [nq] in/out; pool_cursor [nq] or NULL (0).  The nodes in a
 * pool count as visited.  Each pool is written back entry for entry as the reference leaves
 * it (its cursor is then its size).  ef in [1, 1024]. */
int pion_v_b200_hnsw_beam_batch(pion_b200_ctx *ctx, const pion_b200_index *index,
                                const int8_t *q_codes, const float *q_norm, int64_t nq,
                                int64_t ef, void *pools, int32_t *pool_size,
                                const int32_t *pool_cursor, int mem);

/* metric_scores (src/vector/hnsw.mojo:4523-4651) for INT8 codes: replaces scores[t][j] by
 * the index metric's distance between query t (normalised once under COSINE, clamped to
 * the calibration range) and the result ids[t][j] (external ids, as hnsw_search returns
 * them) dequantised at the middle of each code step: squared L2 under L2, half of it
 * (= 1 - cos) under COSINE, summed in the reference's order.  Ids that name no node keep
 * their score.  q fp32[nq x 1536]; ids, scores [nq x k].  On a block-quantised graph
 * (pion_v_b200_register_hnsw_quant) the source is its FP32 copy by node, the query
 * unclamped; without one it has no source: returns 1 and leaves every score (the
 * reference returns False). */
int pion_v_b200_hnsw_metric_scores(pion_b200_ctx *ctx, const pion_b200_index *index,
                                   const float *q, int64_t nq, int64_t k, const int32_t *ids,
                                   float *scores, int mem);

/* The GPU brute-force scan of a registered graph's slot buffer, batched.  Replaces
 * pion_metal_search_topk_w (src/ffi/metal_wrap.m:495-580) with the shader
 * int8_l2_distance_batch (src/ffi/metal_compute.metal:19-78): for each query, every slot s
 * in [0, min(num_vectors, slots)) gets d = (q_norm + slot |code|^2) - 2 * float(dot) and
 * goes through the wrapper's worst-replace loop over min(k, num_vectors) entries.
 * out_slots / out_dists [nq x k] hold the entries in the order the loop leaves them
 * (unsorted, as the engine receives them); entries past min(k, num_vectors) are -1 / +inf.
 * q_codes int8 [nq x 1536]; q_norm [nq] or NULL (then |code|^2 of the codes, as
 * norm_sq_int8_jit computes it).  k in [1, 256]. */
int pion_v_b200_slot_scan_topk(pion_b200_ctx *ctx, const pion_b200_index *index,
                               const int8_t *q_codes, const float *q_norm, int64_t nq,
                               int64_t num_vectors, int64_t k, int32_t *out_slots,
                               float *out_dists, int mem);

/* Work of the context's last slot scan or brute-force call (waits for it): out2 =
 * {queries that went through the exact CUDA-core scan, candidate slots replayed through
 * the loop}. */
int pion_v_b200_slot_last_stats(pion_b200_ctx *ctx, int64_t *out2);

/* pion_metal_register_rerank_buffer / _unregister_ (src/ffi/metal_wrap.m:674-720): FP32
 * rows [n x dim] by slot (the compact_vectors rerank buffer, hnsw.mojo:2832-2880) for
 * pion_v_b200_hnsw_brute_force; n = the graph's slots, dim = 1536; rows NULL drops them.
 * The rows are copied to the device. */
int pion_v_b200_hnsw_set_rerank_rows(pion_b200_ctx *ctx, pion_b200_index *index,
                                     const float *rows, int64_t n, int64_t dim, int mem);

/* search_gpu_brute_force (src/vector/hnsw.mojo:3916-3992) for a batch: the query
 * normalised once (COSINE) and quantised; the slot scan above with min(2 k', n, 256)
 * entries when rerank rows are set (k' = min(k, n)), else min(k', 256); with rerank rows
 * every entry's distance becomes the FP32 squared L2 of the raw query and the slot's row
 * (the engine's CPU rerank loop: 8 lanes, mul then add, halving reduce); a stable sort by
 * distance; the first k' as external ids.  out_ids / out_scores [nq x k] (-1 / +inf past
 * out_found[t]); out_found [nq]. */
int pion_v_b200_hnsw_brute_force(pion_b200_ctx *ctx, const pion_b200_index *index,
                                 const float *q, int64_t nq, int64_t k, int32_t *out_ids,
                                 float *out_scores, int32_t *out_found, int mem);

/* ------------------------------------------------ block-quantised HNSW -- */
/* The reference's three block-quantised compact formats of an HNSW graph at dim 1536
 * (compact_vectors, src/vector/hnsw.mojo:2761-2990 and 3138-3230): per slot an f32
 * reconstructed |v|^2 then 48 blocks of 32 dims, each an f16 scale and the packed codes.
 *   POLAR  PolarQuant INT4 (quantize_fp32_to_block_int4, kernels.mojo:1116-1175), stride 868
 *   NANO   NanoQuant INT2 (quantize_fp32_to_block_int2, kernels.mojo:1776-1842), stride 484
 *   TURBO  TurboQuant INT3 (quantize_fp32_to_block_int3, kernels.mojo:1589-1651), stride 676,
 *          plus per node 24 QJL sign words of the residual (qjl_compute_signs,
 *          kernels.mojo:1685-1714, random signs from an LCG seeded 42, hnsw.mojo:497-509)
 *          and the residual's squared norm. */
#define PION_B200_QUANT_POLAR 0
#define PION_B200_QUANT_NANO 1
#define PION_B200_QUANT_TURBO 2

typedef struct pion_b200_hnsw_quant_layout {
    int32_t kind;                      /* PION_B200_QUANT_*                          */
    int32_t reserved;
    int64_t num_nodes;
    const int8_t *compact;             /* num_nodes x stride, by slot (the graph's
                                          node_slot order)                           */
    int64_t stride;                    /* 868 / 484 / 676                            */
    const uint64_t *qjl;               /* TURBO: num_nodes x 24 words by node, or NULL */
    const float *qjl_res_norms;        /* TURBO: num_nodes by node, or NULL          */
    const uint64_t *qjl_random_signs;  /* TURBO: 24 words, or NULL                   */
    float qjl_lambda;                  /* 1.0                                        */
    int32_t reserved2;
    const float *rerank;               /* num_nodes x 1536 FP32 rows by node (normalised
                                          under COSINE), or NULL: no rerank         */
} pion_b200_hnsw_quant_layout;

typedef struct pion_b200_hnsw_quant pion_b200_hnsw_quant;

/* Quantises the rows a graph was built from (fp32 [n_rows x 1536] in HOST memory, node
 * order, n_rows = the graph's node count; normalised first under COSINE) into `kind`'s
 * compact buffer in the graph's slot order, with TurboQuant's QJL rows, and keeps the
 * (normalised) rows as the rerank buffer.  Float steps in the reference's order, f16
 * scales rounded to nearest even. */
int pion_v_b200_hnsw_quantize(const pion_b200_hnsw_graph *graph, const float *rows,
                              int64_t n_rows, int kind, pion_b200_hnsw_quant **out_quant);
/* The buffers (host memory owned by the quant object). */
int pion_v_b200_hnsw_quant_layout(const pion_b200_hnsw_quant *quant,
                                  pion_b200_hnsw_quant_layout *out_layout);
int pion_v_b200_hnsw_quant_free(pion_b200_hnsw_quant *quant);

/* The reference's index file of a block-quantised graph (pion.hnsw.0 with compact format
 * 1 INT4, 2 INT3, 4 INT2, HNSWGraph.save_to_disk / load_from_disk,
 * src/vector/hnsw.mojo:1209-1712): the graph, its slots and the sections the file carries
 * (FP32 rerank rows; TurboQuant's QJL rows and residual norms; the QJL random signs are
 * the LCG's, not stored).  *out_quant is NULL after a plain INT8 file (then the graph is
 * what pion_v_b200_hnsw_load returns).  Per-group calibration is refused.
 * pion_v_b200_hnsw_save_quant writes a graph with its quant buffers as a v5 file in that
 * format (zero node norms, as the engine writes them for the block formats). */
int pion_v_b200_hnsw_load_quant(const char *path, pion_b200_hnsw_graph **out_graph,
                                pion_b200_hnsw_quant **out_quant);
int pion_v_b200_hnsw_save_quant(const pion_b200_hnsw_graph *graph,
                                const pion_b200_hnsw_quant *quant, const char *path,
                                int64_t max_elements);

/* Copies a graph (its compact_buffer is not used) and its block-quantised slots (every
 * pointer in HOST memory) to the GPU.  Checks the graph as register_hnsw does and the
 * quant layout's kind, stride and sizes. */
int pion_v_b200_register_hnsw_quant(pion_b200_ctx *ctx, const pion_b200_hnsw_layout *graph,
                                    const pion_b200_hnsw_quant_layout *quant,
                                    pion_b200_index **out_index);

/* Batched block-quant HNSW search: search_fp32_scored's block-quant branches
 * (src/vector/hnsw.mojo:4136-4330) per query: normalise (COSINE), block-quantise to int8,
 * (TURBO) the query's QJL signs, the upper-level greedy with the block distance, the
 * level-0 beam quant_beam_search_1536_ref (src/vector/reference/quant_beams_1536.mojo:
 * 20-81) over MinHeap / MaxHeap (src/common/heap.mojo:48-120, 237-339), then
 * _rerank_fp32_sorted (hnsw.mojo:4052-4134): the ef results reranked by the FP32 rows
 * (when registered), stably sorted, the first k.  q fp32[nq x 1536]; out_ids /
 * out_scores [nq x k] (-1 / +inf past out_found[t]); out_found [nq].  ef in [1, 1024]. */
int pion_v_b200_hnsw_quant_search(pion_b200_ctx *ctx, const pion_b200_index *index,
                                  const float *q, int64_t nq, int64_t k, int64_t ef,
                                  int32_t *out_ids, float *out_scores, int32_t *out_found,
                                  int mem);

/* Work counters of the context's last pion_v_b200_hnsw_search (waits for it):
 * out3 = {level-0 distance evaluations, level-0 expansions, upper-level distance
 * evaluations}, summed over the batch.  After pion_v_b200_hnsw_quant_search: {distance
 * evaluations, level-0 expansions, queries re-run with a larger candidate heap}. */
int pion_v_b200_hnsw_last_stats(pion_b200_ctx *ctx, int64_t *out3);

#ifdef __cplusplus
}
#endif
#endif /* PION_VECTOR_B200_H */
