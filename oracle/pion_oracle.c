/*
 * CPU oracle for Pion's FT.SEARCH KNN hot path — TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * arm load this file's library (oracle/liboracle.so).  The product library never
 * does.  Parity status: UNPINNED (see pion_oracle.h for why and what pins it).
 *
 * Build: oracle/Makefile (gcc -O3 -march=x86-64-v2 -ffp-contract=off -pthread).
 * Every routine cites the Mojo file:line it restates, paths relative to the
 * pavelhorak/pion repository.
 */
#include "pion_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <pthread.h>
#include <stdatomic.h>


/* ------------------------------------------------------------------------- */
/* Query-level threading for the CPU baseline: a dynamic parallel-for over      */
/* [0, n) with pthreads (one item at a time from an atomic counter).            */
/* ------------------------------------------------------------------------- */
struct orc_pool_job {
    orc_item_fn fn;
    void *ctx;
    int64_t n;
    _Atomic int64_t next;
    size_t scratch_bytes;
};
static void *orc_pool_worker(void *arg) {
    struct orc_pool_job *job = (struct orc_pool_job *)arg;
    void *scratch = job->scratch_bytes ? calloc(1, job->scratch_bytes) : NULL;
    for (;;) {
        int64_t i = atomic_fetch_add(&job->next, 1);
        if (i >= job->n) break;
        job->fn(job->ctx, i, scratch);
    }
    free(scratch);
    return NULL;
}
void orc_parallel_for(int64_t n, int nthreads, size_t scratch_bytes, orc_item_fn fn,
                      void *ctx) {
    struct orc_pool_job job;
    job.fn = fn;
    job.ctx = ctx;
    job.n = n;
    atomic_init(&job.next, 0);
    job.scratch_bytes = scratch_bytes;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if (nthreads == 1 || n <= 1) {
        orc_pool_worker(&job);
        return;
    }
    pthread_t th[256];
    int started = 0;
    for (int t = 0; t < nthreads; ++t)
        if (pthread_create(&th[started], NULL, orc_pool_worker, &job) == 0) started++;
    if (started == 0) orc_pool_worker(&job);
    for (int t = 0; t < started; ++t) pthread_join(th[t], NULL);
}

/* ------------------------------------------------------------------------- */
/* SIMD reduce_add of a w-lane float vector as a halving tree: lanes [0, w/2)   */
/* are added lane-wise to lanes [w/2, w), then recursively (Mojo SIMD.reduce). */
/* ------------------------------------------------------------------------- */
static float reduce_add_tree(float *lanes, int w) {
    while (w > 1) {
        int h = w / 2;
        for (int i = 0; i < h; ++i) lanes[i] = lanes[i] + lanes[i + h];
        w = h;
    }
    return lanes[0];
}

/* ========================================================================= */
/* PKM routines                                                              */
/* ========================================================================= */

/* src/vector/pkm_kernels.mojo:152-191 (pkm_quantize_rows_i8).
 * scale = max|x| / 127 (1.0 for an all-zero row); q = trunc(x*(1/scale) +- 0.5)
 * clamped to [-127, 127]; padding columns zeroed.  Rows are read at stride d_pad. */
void orc_pkm_quantize_rows_i8(const float *src, int64_t n_rows, int64_t d, int64_t d_pad,
                              int8_t *dst, float *dst_scale) {
    for (int64_t r = 0; r < n_rows; ++r) {
        const float *sp = src + r * d_pad;
        float m = 0.0f;
        for (int64_t c = 0; c < d; ++c) {
            float a = sp[c];
            if (a < 0.0f) a = -a;
            if (a > m) m = a;
        }
        float scale = m / 127.0f;
        if (m == 0.0f) scale = 1.0f;
        float inv = 1.0f / scale;
        int8_t *dp = dst + r * d_pad;
        for (int64_t c = 0; c < d; ++c) {
            float qv = sp[c] * inv;
            int64_t qi = qv >= 0.0f ? (int64_t)(qv + 0.5f) : (int64_t)(qv - 0.5f);
            if (qi > 127) qi = 127;
            if (qi < -127) qi = -127;
            dp[c] = (int8_t)qi;
        }
        for (int64_t c = d; c < d_pad; ++c) dp[c] = 0;
        dst_scale[r] = scale;
    }
}

static inline int32_t dot_i8(const int8_t *a, const int8_t *b, int64_t n) {
    int32_t acc = 0;
    for (int64_t i = 0; i < n; ++i) acc += (int32_t)a[i] * (int32_t)b[i];
    return acc;
}

/* Epilogue of src/vector/reference/pkm_ref.mojo:58-61: (f32(dot) * row_scale) * q_scale,
 * two separately rounded products, left to right. */
static inline float i8_score(int32_t dot, float rs, float qs) {
    float s = (float)dot;
    s = s * rs;
    s = s * qs;
    return s;
}

/* src/vector/reference/pkm_ref.mojo:47-61 (ref_pkm_scores_i8). */
void orc_pkm_scores_i8(const int8_t *keys, int64_t s_rows, int64_t d_pad, const float *row_scale,
                       const int8_t *q, const float *q_scale, int64_t nq, float *dst) {
    for (int64_t t = 0; t < nq; ++t)
        for (int64_t r = 0; r < s_rows; ++r)
            dst[t * s_rows + r] =
                i8_score(dot_i8(keys + r * d_pad, q + t * d_pad, d_pad), row_scale[r], q_scale[t]);
}

/* 8-lane f32 accumulator dot over d_pad (a multiple of 8), then a tree reduce:
 * src/vector/reference/pkm_ref.mojo:22-31. */
static float dot8_f32(const float *a, const float *b, int64_t d_pad) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int64_t i = 0; i < d_pad; i += 8)
        for (int l = 0; l < 8; ++l) {
            float p = a[i + l] * b[i + l];
            acc[l] = acc[l] + p;
        }
    return reduce_add_tree(acc, 8);
}

/* src/vector/reference/pkm_ref.mojo:22-31 (ref_pkm_scores_f32). */
void orc_pkm_scores_f32(const float *keys, int64_t s_rows, int64_t d_pad, const float *q,
                        int64_t nq, float *dst) {
    for (int64_t t = 0; t < nq; ++t)
        for (int64_t r = 0; r < s_rows; ++r)
            dst[t * s_rows + r] = dot8_f32(keys + r * d_pad, q + t * d_pad, d_pad);
}

/* src/vector/reference/pkm_ref.mojo:34-44 (ref_pkm_rescore_f32). */
void orc_pkm_rescore_f32(const float *keys, int64_t d_pad, const float *q, const int32_t *idx,
                         int64_t cnt, float *dst) {
    for (int64_t t = 0; t < cnt; ++t) dst[t] = dot8_f32(keys + (int64_t)idx[t] * d_pad, q, d_pad);
}

/* src/vector/reference/pkm_ref.mojo:64-81 (_sift_down_min): min-heap on val. */
static void sift_down_min(float *val, int32_t *idx, int64_t start, int64_t n) {
    int64_t root = start;
    for (;;) {
        int64_t child = 2 * root + 1;
        if (child >= n) break;
        if (child + 1 < n && val[child + 1] < val[child]) child += 1;
        if (val[child] < val[root]) {
            float tv = val[root]; val[root] = val[child]; val[child] = tv;
            int32_t ti = idx[root]; idx[root] = idx[child]; idx[child] = ti;
            root = child;
        } else {
            break;
        }
    }
}

/* src/vector/reference/pkm_ref.mojo:84-89 (_heapify_min). */
static void heapify_min(float *val, int32_t *idx, int64_t n) {
    for (int64_t s = n / 2 - 1; s >= 0; --s) sift_down_min(val, idx, s, n);
}

/* src/vector/reference/pkm_ref.mojo:92-107 (ref_pkm_sort_desc): min-heapsort,
 * the smallest sinks to the end, leaving the array descending. */
void orc_pkm_sort_desc(float *val, int32_t *idx, int64_t n) {
    if (n <= 1) return;
    heapify_min(val, idx, n);
    for (int64_t e = n - 1; e > 0; --e) {
        float tv = val[0]; val[0] = val[e]; val[e] = tv;
        int32_t ti = idx[0]; idx[0] = idx[e]; idx[e] = ti;
        sift_down_min(val, idx, 0, e);
    }
}

/* src/vector/reference/pkm_ref.mojo:110-130 (ref_pkm_topk_max): seed with the first
 * k, heapify, admit only s > root (strict), heapsort descending.  Returns min(k, n). */
int64_t orc_pkm_topk_max(const float *scores, int64_t n, int64_t k, int32_t *out_idx,
                         float *out_val) {
    int64_t kk = k < n ? k : n;
    if (kk <= 0) return 0;
    for (int64_t i = 0; i < kk; ++i) {
        out_idx[i] = (int32_t)i;
        out_val[i] = scores[i];
    }
    heapify_min(out_val, out_idx, kk);
    for (int64_t i = kk; i < n; ++i) {
        float sv = scores[i];
        if (sv > out_val[0]) {
            out_val[0] = sv;
            out_idx[0] = (int32_t)i;
            sift_down_min(out_val, out_idx, 0, kk);
        }
    }
    orc_pkm_sort_desc(out_val, out_idx, kk);
    return kk;
}

/* src/vector/reference/pkm_ref.mojo:133-160 (ref_pkm_combine_topk). */
int64_t orc_pkm_combine_topk(const float *s0, const int32_t *i0, int64_t k0, const float *s1,
                             const int32_t *i1, int64_t k1, int64_t s_cols, int64_t k,
                             int32_t *out_id, float *out_score) {
    int64_t lim = k0 * k1;
    int64_t cap = k < lim ? k : lim;
    if (cap <= 0) return 0;
    int64_t cnt = 0;
    for (int64_t a = 0; a < k0; ++a)
        for (int64_t b = 0; b < k1; ++b) {
            float sc = s0[a] + s1[b];
            int32_t sid = (int32_t)((int64_t)i0[a] * s_cols + (int64_t)i1[b]);
            if (cnt < cap) {
                out_score[cnt] = sc;
                out_id[cnt] = sid;
                cnt += 1;
                if (cnt == cap) heapify_min(out_score, out_id, cap);
            } else if (sc > out_score[0]) {
                out_score[0] = sc;
                out_id[0] = sid;
                sift_down_min(out_score, out_id, 0, cap);
            }
        }
    orc_pkm_sort_desc(out_score, out_id, cnt);
    return cnt;
}

/* One query of the FLAT INT8 IP KNN: ref_pkm_scores_i8 for row r is computed at the
 * moment ref_pkm_topk_max reads scores[r], so the result equals the two reference
 * calls back to back (src/vector/reference/pkm_ref.mojo:47-61 then :110-130). */
static int64_t flat_i8_one(const int8_t *keys, int64_t n, int64_t d_pad, const float *row_scale,
                           const int8_t *q, float qs, int64_t k, int32_t *out_idx,
                           float *out_val) {
    int64_t kk = k < n ? k : n;
    if (kk <= 0) return 0;
    for (int64_t i = 0; i < kk; ++i) {
        out_idx[i] = (int32_t)i;
        out_val[i] = i8_score(dot_i8(keys + i * d_pad, q, d_pad), row_scale[i], qs);
    }
    heapify_min(out_val, out_idx, kk);
    for (int64_t i = kk; i < n; ++i) {
        float sv = i8_score(dot_i8(keys + i * d_pad, q, d_pad), row_scale[i], qs);
        if (sv > out_val[0]) {
            out_val[0] = sv;
            out_idx[0] = (int32_t)i;
            sift_down_min(out_val, out_idx, 0, kk);
        }
    }
    orc_pkm_sort_desc(out_val, out_idx, kk);
    return kk;
}

struct flat_i8_job {
    const int8_t *keys; int64_t n, d_pad; const float *row_scale;
    const int8_t *q; const float *q_scale; int64_t k; int32_t *out_idx; float *out_val;
};
static void flat_i8_item(void *ctx, int64_t t, void *scratch) {
    (void)scratch;
    struct flat_i8_job *j = (struct flat_i8_job *)ctx;
    int64_t k = j->k;
    int64_t got = flat_i8_one(j->keys, j->n, j->d_pad, j->row_scale, j->q + t * j->d_pad,
                              j->q_scale[t], k, j->out_idx + t * k, j->out_val + t * k);
    for (int64_t c = got; c < k; ++c) {
        j->out_idx[t * k + c] = -1;
        j->out_val[t * k + c] = -INFINITY;
    }
}

void orc_flat_i8_knn(const int8_t *keys, int64_t n, int64_t d_pad, const float *row_scale,
                     const int8_t *q, const float *q_scale, int64_t nq, int64_t k,
                     int32_t *out_idx, float *out_val, int nthreads) {
    struct flat_i8_job j = {keys, n, d_pad, row_scale, q, q_scale, k, out_idx, out_val};
    orc_parallel_for(nq, nthreads, 0, flat_i8_item, &j);
}

/* ========================================================================= */
/* Exact FP32 rows                                                           */
/* ========================================================================= */

/* src/vector/fp32_scan.mojo:17-38 (dot_f32_4chain): four 4-lane chains over
 * 16-float strides, a 4-lane tail chain on a0, ((a0+a1)+(a2+a3)).reduce_add(),
 * then a scalar tail.  fma_mad is a*b+c on x86-64-v2 (src/vector/fma_mad.mojo:21). */
float orc_dot_f32_4chain(const float *q, const float *v, int64_t dim) {
    float a[4][4] = {{0}};
    int64_t d = 0;
    for (; d + 16 <= dim; d += 16)
        for (int c = 0; c < 4; ++c)
            for (int l = 0; l < 4; ++l) {
                float p = q[d + 4 * c + l] * v[d + 4 * c + l];
                a[c][l] = p + a[c][l];
            }
    for (; d + 4 <= dim; d += 4)
        for (int l = 0; l < 4; ++l) {
            float p = q[d + l] * v[d + l];
            a[0][l] = p + a[0][l];
        }
    float t[4];
    for (int l = 0; l < 4; ++l) t[l] = (a[0][l] + a[1][l]) + (a[2][l] + a[3][l]);
    float s = reduce_add_tree(t, 4);
    for (; d < dim; ++d) s += q[d] * v[d];
    return s;
}

/* src/vector/fp32_scan.mojo:42-69 (l2sq_f32_4chain). */
float orc_l2sq_f32_4chain(const float *x, const float *y, int64_t dim) {
    float a[4][4] = {{0}};
    int64_t d = 0;
    for (; d + 16 <= dim; d += 16)
        for (int c = 0; c < 4; ++c)
            for (int l = 0; l < 4; ++l) {
                float e = x[d + 4 * c + l] - y[d + 4 * c + l];
                float p = e * e;
                a[c][l] = p + a[c][l];
            }
    for (; d + 4 <= dim; d += 4)
        for (int l = 0; l < 4; ++l) {
            float e = x[d + l] - y[d + l];
            float p = e * e;
            a[0][l] = p + a[0][l];
        }
    float t[4];
    for (int l = 0; l < 4; ++l) t[l] = (a[0][l] + a[1][l]) + (a[2][l] + a[3][l]);
    float s = reduce_add_tree(t, 4);
    for (; d < dim; ++d) {
        float e = x[d] - y[d];
        s += e * e;
    }
    return s;
}

/* src/vector/kernels.mojo:318-357 (l2_normalize_fp32): 4-lane sum of squares (SSE
 * width on x86-64-v2), tree reduce, scalar tail, inv = 1/sqrt; zero vector copied. */
void orc_l2_normalize_fp32(const float *src, float *dst, int64_t dim) {
    float acc[4] = {0, 0, 0, 0};
    int64_t i = 0;
    for (; i + 4 <= dim; i += 4)
        for (int l = 0; l < 4; ++l) {
            float p = src[i + l] * src[i + l];
            acc[l] = acc[l] + p;
        }
    float norm_sq = reduce_add_tree(acc, 4);
    for (; i < dim; ++i) norm_sq += src[i] * src[i];
    if (norm_sq <= 0.0f) {
        if (dst != src) memcpy(dst, src, (size_t)dim * sizeof(float));
        return;
    }
    float inv = 1.0f / sqrtf(norm_sq);
    for (int64_t k = 0; k < dim; ++k) dst[k] = src[k] * inv;
}

/* Query normalisation of exact_knn / _exact_rescore: a sequential scalar sum of
 * squares, inv = 1/sqrt(ss) under COSINE when ss > 0, else 1
 * (src/commands/vector.mojo:1254-1260 and :1431-1437). */
void orc_exact_query_normalize(const float *query, float *q, int64_t dim, int cosine) {
    float ss = 0.0f;
    for (int64_t d = 0; d < dim; ++d) {
        float p = query[d] * query[d];
        ss = ss + p;
    }
    float inv = (cosine && ss > 0.0f) ? 1.0f / sqrtf(ss) : 1.0f;
    for (int64_t d = 0; d < dim; ++d) q[d] = query[d] * inv;
}

/* src/commands/vector.mojo:1228-1365 (exact_knn) with every row live (no dead
 * slots, no filter, no TTL): COSINE score 1 - dot_f32_4chain(q^, row), L2 score
 * l2sq_f32_4chain; bounded max-heap of cap = min(k, n) with strict `<` admission
 * (an equal score never displaces, the earliest slot wins); popped to ascending. */
int64_t orc_exact_knn(const float *rows, int64_t n, int64_t dim, const float *query, int64_t k,
                      int cosine, int64_t *ids, float *scores) {
    if (k <= 0 || n <= 0) return 0;
    float *q = (float *)malloc((size_t)dim * sizeof(float));
    orc_exact_query_normalize(query, q, dim, cosine);
    int64_t cap = k < n ? k : n;
    float *hs = (float *)malloc((size_t)cap * sizeof(float));
    int64_t *hi = (int64_t *)malloc((size_t)cap * sizeof(int64_t));
    int64_t hn = 0;
    for (int64_t slot = 0; slot < n; ++slot) {
        const float *row = rows + slot * dim;
        float sc = cosine ? 1.0f - orc_dot_f32_4chain(q, row, dim) : orc_l2sq_f32_4chain(q, row, dim);
        if (hn == cap && !(sc < hs[0])) continue;
        if (hn < cap) {
            int64_t c = hn;
            hn += 1;
            while (c > 0) {
                int64_t par = (c - 1) / 2;
                if (hs[par] >= sc) break;
                hs[c] = hs[par];
                hi[c] = hi[par];
                c = par;
            }
            hs[c] = sc;
            hi[c] = slot;
        } else {
            int64_t c = 0;
            for (;;) {
                int64_t l = 2 * c + 1;
                if (l >= hn) break;
                int64_t m = l;
                if (l + 1 < hn && hs[l + 1] > hs[l]) m = l + 1;
                if (hs[m] <= sc) break;
                hs[c] = hs[m];
                hi[c] = hi[m];
                c = m;
            }
            hs[c] = sc;
            hi[c] = slot;
        }
    }
    int64_t cnt = hn, nn = hn;
    while (nn > 0) {
        float top_s = hs[0];
        int64_t top_i = hi[0];
        nn -= 1;
        ids[nn] = top_i;
        scores[nn] = top_s;
        float sc = hs[nn];
        int64_t si = hi[nn];
        int64_t c = 0;
        for (;;) {
            int64_t l = 2 * c + 1;
            if (l >= nn) break;
            int64_t m = l;
            if (l + 1 < nn && hs[l + 1] > hs[l]) m = l + 1;
            if (hs[m] <= sc) break;
            hs[c] = hs[m];
            hi[c] = hi[m];
            c = m;
        }
        if (nn > 0) {
            hs[c] = sc;
            hi[c] = si;
        }
    }
    free(q);
    free(hs);
    free(hi);
    return cnt;
}

struct exact_job {
    const float *rows; int64_t n, dim; const float *queries; int64_t k; int cosine;
    int64_t *ids; float *scores;
};
static void exact_item(void *ctx, int64_t t, void *scratch) {
    (void)scratch;
    struct exact_job *j = (struct exact_job *)ctx;
    int64_t k = j->k;
    int64_t got = orc_exact_knn(j->rows, j->n, j->dim, j->queries + t * j->dim, k, j->cosine,
                                j->ids + t * k, j->scores + t * k);
    for (int64_t c = got; c < k; ++c) {
        j->ids[t * k + c] = -1;
        j->scores[t * k + c] = INFINITY;
    }
}

void orc_exact_knn_batch(const float *rows, int64_t n, int64_t dim, const float *queries,
                         int64_t nq, int64_t k, int cosine, int64_t *ids, float *scores,
                         int nthreads) {
    struct exact_job j = {rows, n, dim, queries, k, cosine, ids, scores};
    orc_parallel_for(nq, nthreads, 0, exact_item, &j);
}

/* ========================================================================= */
/* Binary quantisation + FP32 rerank (composed oracle)                       */
/* ========================================================================= */

/* Sign packing of src/vector/kernels.mojo:1711-1720 (qjl_compute_signs' last step),
 * applied to the vector itself: bit b of word w is 1 iff x[64w + b] > 0. */
void orc_bq_pack_signs(const float *rows, int64_t n, int64_t dim, uint64_t *codes) {
    int64_t words = dim / 64;
    for (int64_t r = 0; r < n; ++r)
        for (int64_t w = 0; w < words; ++w) {
            uint64_t bits = 0;
            for (int b = 0; b < 64; ++b)
                if (rows[r * dim + w * 64 + b] > 0.0f) bits |= (uint64_t)1 << b;
            codes[r * words + w] = bits;
        }
}

/* src/vector/reference/quant_dots.mojo:95-100 (ref_hamming). */
int64_t orc_hamming(const uint64_t *a, const uint64_t *b, int64_t words) {
    int64_t total = 0;
    for (int64_t w = 0; w < words; ++w) total += __builtin_popcountll(a[w] ^ b[w]);
    return total;
}

/* One BQ query: Hamming shortlist of the `shortlist` smallest distances, ordered by
 * (distance, id); then exact COSINE rescoring of the shortlist with exact_knn's
 * formula (src/commands/vector.mojo:1413-1456, _exact_rescore: normalised query,
 * 1 - dot_f32_4chain) and its stable insertion sort by score; the first k are kept. */
static void bq_one(const uint64_t *codes, const float *rows, int64_t n, int64_t dim,
                   const float *query, int64_t shortlist, int64_t k, int64_t *ids, float *scores,
                   int32_t *short_ids, int32_t *short_dist, uint16_t *dist, float *q) {
    int64_t words = dim / 64;
    int64_t maxd = words * 64;
    uint64_t qc[64];
    orc_exact_query_normalize(query, q, dim, 1);
    orc_bq_pack_signs(q, 1, dim, qc);
    int64_t *hist = (int64_t *)calloc((size_t)(maxd + 1), sizeof(int64_t));
    for (int64_t r = 0; r < n; ++r) {
        dist[r] = (uint16_t)orc_hamming(qc, codes + r * words, words);
        hist[dist[r]] += 1;
    }
    int64_t sl = shortlist < n ? shortlist : n;
    /* cumulative counts by distance give each (distance, id) its rank */
    int64_t *start = (int64_t *)calloc((size_t)(maxd + 2), sizeof(int64_t));
    for (int64_t d = 0; d <= maxd; ++d) start[d + 1] = start[d] + hist[d];
    for (int64_t r = 0; r < n; ++r) {
        int64_t pos = start[dist[r]]++;
        if (pos < sl) {
            short_ids[pos] = (int32_t)r;
            short_dist[pos] = dist[r];
        }
    }
    free(hist);
    free(start);
    float *sc = (float *)malloc((size_t)sl * sizeof(float));
    int64_t *id = (int64_t *)malloc((size_t)sl * sizeof(int64_t));
    for (int64_t i = 0; i < sl; ++i) {
        id[i] = short_ids[i];
        sc[i] = 1.0f - orc_dot_f32_4chain(q, rows + id[i] * dim, dim);
    }
    for (int64_t a = 1; a < sl; ++a) {
        int64_t b = a;
        while (b > 0 && sc[b] < sc[b - 1]) {
            float ts = sc[b]; sc[b] = sc[b - 1]; sc[b - 1] = ts;
            int64_t ti = id[b]; id[b] = id[b - 1]; id[b - 1] = ti;
            b -= 1;
        }
    }
    for (int64_t j = 0; j < k; ++j) {
        ids[j] = j < sl ? id[j] : -1;
        scores[j] = j < sl ? sc[j] : INFINITY;
    }
    for (int64_t j = sl; j < shortlist; ++j) {
        short_ids[j] = -1;
        short_dist[j] = -1;
    }
    free(sc);
    free(id);
}

struct bq_job {
    const uint64_t *codes; const float *rows; int64_t n, dim; const float *queries;
    int64_t shortlist, k; int64_t *ids; float *scores; int32_t *short_ids, *short_dist;
};
static void bq_item(void *ctx, int64_t t, void *scratch) {
    struct bq_job *j = (struct bq_job *)ctx;
    uint16_t *dist = (uint16_t *)scratch;
    float *q = (float *)((char *)scratch + (((size_t)j->n * sizeof(uint16_t) + 63) & ~(size_t)63));
    bq_one(j->codes, j->rows, j->n, j->dim, j->queries + t * j->dim, j->shortlist, j->k,
           j->ids + t * j->k, j->scores + t * j->k, j->short_ids + t * j->shortlist,
           j->short_dist + t * j->shortlist, dist, q);
}

void orc_bq_knn_batch(const uint64_t *codes, const float *rows, int64_t n, int64_t dim,
                      const float *queries, int64_t nq, int64_t shortlist, int64_t k,
                      int64_t *ids, float *scores, int32_t *short_ids, int32_t *short_dist,
                      int nthreads) {
    struct bq_job j = {codes, rows, n, dim, queries, shortlist, k, ids, scores, short_ids,
                       short_dist};
    size_t bytes = (((size_t)n * sizeof(uint16_t) + 63) & ~(size_t)63) + (size_t)dim * sizeof(float);
    orc_parallel_for(nq, nthreads, bytes, bq_item, &j);
}

/* ========================================================================= */
/* Sharded merge: src/commands/vector.mojo:4394-4429.  Concatenated per-shard   */
/* lists (shard order), then a selection sort with strict `<` and swaps; the    */
/* first final_k = min(k, n_all) entries are the answer.                       */
/* ========================================================================= */
int64_t orc_shard_merge_asc(const int64_t *ids, const float *scores, int64_t n_all, int64_t k,
                            int64_t *out_ids, float *out_scores) {
    int64_t *ai = (int64_t *)malloc((size_t)(n_all > 0 ? n_all : 1) * sizeof(int64_t));
    float *as = (float *)malloc((size_t)(n_all > 0 ? n_all : 1) * sizeof(float));
    memcpy(ai, ids, (size_t)n_all * sizeof(int64_t));
    memcpy(as, scores, (size_t)n_all * sizeof(float));
    int64_t final_k = k < n_all ? k : n_all;
    for (int64_t fi = 0; fi < final_k; ++fi) {
        int64_t min_idx = fi;
        float min_score = as[fi];
        for (int64_t fj = fi + 1; fj < n_all; ++fj)
            if (as[fj] < min_score) {
                min_score = as[fj];
                min_idx = fj;
            }
        if (min_idx != fi) {
            int64_t ti = ai[fi]; ai[fi] = ai[min_idx]; ai[min_idx] = ti;
            as[min_idx] = as[fi];
            as[fi] = min_score;
        }
    }
    for (int64_t i = 0; i < final_k; ++i) {
        out_ids[i] = ai[i];
        out_scores[i] = as[i];
    }
    free(ai);
    free(as);
    return final_k;
}
