/*
 * CPU oracle for the HNSW INT8 search at dim 1536 — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's search over a compact graph, used by
 * tests/ and bench.py's CPU leg as the checker.  Parity status: UNPINNED (the
 * reference is Mojo; no golden vectors exist).  Restates, paths inside the
 * pavelhorak/pion repository:
 *   src/vector/hnsw.mojo:4136-4521     search_fp32_scored (the dim-1536 path)
 *   src/vector/hnsw.mojo:657-680       _quantize_query_to_int8
 *   src/vector/kernels.mojo:52-99      quantize_fp32_to_int8_simd (roundeven, clamp)
 *   src/vector/kernels.mojo:318-357    l2_normalize_fp32
 *   src/vector/hnsw.mojo:3789-3848     _upper_greedy_codes
 *   src/vector/reference/beam_1536.mojo:30-135   beam_search_1536_ref, _gather
 *   src/common/heap.mojo:133-234       LinearPool
 *   src/vector/hnsw.mojo:4523-4651     metric_scores (INT8 codes, global calibration)
 *   src/ffi/metal_compute.metal:19-143 INT8 L2 of every slot (the GPU brute-force scan)
 *   src/ffi/metal_wrap.m:495-580       its worst-replace top-k
 *   src/vector/hnsw.mojo:3916-3992     search_gpu_brute_force (oversample, FP32 rerank)
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "pion_oracle.h"

#define HN_DIM 1536
#define HN_CHECKED 0x80000000u

typedef struct {
    float dist;
    uint32_t id;
} pool_entry;

/* LinearPool (src/common/heap.mojo:133-234). */
typedef struct {
    pool_entry *e;
    int64_t size, cursor, ef;
} linear_pool;

static void pool_reset(linear_pool *p, int64_t ef) {
    p->ef = ef < 1 ? 1 : ef;
    p->size = 0;
    p->cursor = 0;
}

/* Accept-gated sorted insert; upper-bound position keeps equal distances in
 * insertion order; the worst entry falls off a full pool. */
static int pool_insert(linear_pool *p, float d, uint32_t id) {
    if (p->size == p->ef && d >= p->e[p->size - 1].dist) return 0;
    int64_t lo = 0, hi = p->size;
    while (lo < hi) {
        int64_t mid = (lo + hi) >> 1;
        if (p->e[mid].dist > d)
            hi = mid;
        else
            lo = mid + 1;
    }
    int64_t move_n = p->size - lo;
    if (p->size == p->ef) move_n -= 1;
    if (move_n > 0) memmove(p->e + lo + 1, p->e + lo, (size_t)move_n * sizeof(pool_entry));
    p->e[lo].dist = d;
    p->e[lo].id = id;
    if (p->size < p->ef) p->size += 1;
    if (lo < p->cursor) p->cursor = lo;
    return 1;
}

static int pool_has_next(const linear_pool *p) { return p->cursor < p->size; }

static uint32_t pool_pop(linear_pool *p) {
    pool_entry e = p->e[p->cursor];
    p->e[p->cursor].id = e.id | HN_CHECKED;
    p->cursor += 1;
    while (p->cursor < p->size && (p->e[p->cursor].id & HN_CHECKED) != 0) p->cursor += 1;
    return e.id & ~HN_CHECKED;
}

static float pool_worst(const linear_pool *p) { return p->e[p->size - 1].dist; }

/* _ref_dot / _ref_l2 (beam_1536.mojo:30-44): exact int32 sums. */
static int32_t ref_dot(const int8_t *a, const int8_t *b, int n) {
    int32_t s = 0;
    for (int i = 0; i < n; ++i) s += (int32_t)a[i] * (int32_t)b[i];
    return s;
}

static int32_t ref_l2(const int8_t *a, const int8_t *b, int n) {
    int32_t s = 0;
    for (int i = 0; i < n; ++i) {
        int32_t d = (int32_t)a[i] - (int32_t)b[i];
        s += d * d;
    }
    return s;
}

static int is_deleted(const orc_hnsw_layout *L, uint32_t i) {
    return L->deleted && ((L->deleted[i >> 3] >> (i & 7)) & 1u);
}

static const int8_t *slot_vec(const orc_hnsw_layout *L, uint32_t slot) {
    return L->compact_buffer + (int64_t)slot * L->compact_stride + L->compact_hdr;
}

/* Node norm^2 from the slot header (beam_1536.mojo:47-51). */
static float slot_norm(const int8_t *v) {
    float f;
    memcpy(&f, v - 8, 4);
    return f;
}

/* Normalise (COSINE: `passes` times; search_fp32_scored normalises, then
 * _quantize_query_to_int8 again, the brute-force scan only once) and quantise:
 * clamp(roundeven((x - gmin) * scale), 0, 254) - 127. */
static void query_codes_n(const orc_hnsw_layout *L, const float *x, float *tmp, int8_t *q,
                          int passes) {
    const float *src = x;
    if (L->metric == 1) {
        orc_l2_normalize_fp32(x, tmp, HN_DIM);
        for (int i = 1; i < passes; ++i) orc_l2_normalize_fp32(tmp, tmp, HN_DIM);
        src = tmp;
    }
    float range = L->global_max - L->global_min;
    if (range <= 0.0f) range = 1.0f;
    const float scale = 254.0f / range;
    for (int i = 0; i < HN_DIM; ++i) {
        const float norm = (src[i] - L->global_min) * scale;
        long r = lrintf(norm);
        if (r < 0) r = 0;
        if (r > 254) r = 254;
        q[i] = (int8_t)(r - 127);
    }
}

static void query_codes(const orc_hnsw_layout *L, const float *x, float *tmp, int8_t *q) {
    query_codes_n(L, x, tmp, q, 2);
}

void orc_hnsw_query_codes(const orc_hnsw_layout *L, const float *queries, int64_t nq,
                          int8_t *codes) {
    float tmp[HN_DIM];
    for (int64_t t = 0; t < nq; ++t)
        query_codes(L, queries + t * HN_DIM, tmp, codes + t * HN_DIM);
}

struct hnsw_job {
    const orc_hnsw_layout *L;
    const float *queries;
    int64_t k, ef;
    int greedy_passes;  /* normalisations before the greedy's codes (COSINE): 2, or 1 */
    int32_t *out_ids;
    float *out_dist;
    _Atomic int64_t evals, expansions, upper, bad;
};

/* Per-thread scratch: epoch, visited epochs, pool, fp32 and int8 query. */
struct hnsw_scratch {
    uint16_t epoch;
    uint16_t *visited;
    pool_entry *pool;
    float *fq;
    int8_t *q;
};

static size_t scratch_bytes(int64_t n, int64_t ef) {
    /* the sizes scratch_bind lays out, each section rounded up to 64 bytes */
    return 64 + ((size_t)n * 2 + 63) / 64 * 64 + 64 +
           ((size_t)(ef < 1 ? 1 : ef) * sizeof(pool_entry) + 63) / 64 * 64 + 64 + HN_DIM * 4 +
           64 + HN_DIM + 64;
}

static void scratch_bind(void *raw, int64_t n, int64_t ef, struct hnsw_scratch *s) {
    char *p = (char *)raw;
    uint16_t *epoch_cell = (uint16_t *)p;
    p += 64;
    s->epoch = *epoch_cell;
    s->visited = (uint16_t *)p;
    p += ((size_t)n * 2 + 63) / 64 * 64 + 64;
    s->pool = (pool_entry *)p;
    p += ((size_t)(ef < 1 ? 1 : ef) * sizeof(pool_entry) + 63) / 64 * 64 + 64;
    s->fq = (float *)p;
    p += HN_DIM * 4 + 64;
    s->q = (int8_t *)p;
}

/* _gather (beam_1536.mojo:58-81): unvisited, undeleted level-0 neighbours of c in
 * adjacency order, marked visited.  Returns -1 when a neighbour has no compact slot
 * (the reference would fall back to the engine's node pointer). */
static int gather(const orc_hnsw_layout *L, uint32_t c, uint16_t *visited, uint16_t epoch,
                  uint32_t *idxs, const int8_t **ptrs) {
    const uint32_t *row = L->l0_compact + (int64_t)c * 33;
    const uint32_t *slots = L->l0_slots + (int64_t)c * 33;
    const int count = (int)row[0];
    int n = 0;
    for (int i = 0; i < count && i < 32; ++i) {
        const uint32_t nb = row[1 + i];
        if (nb >= (uint32_t)L->num_nodes) continue;
        if (is_deleted(L, nb)) continue;
        if (visited[nb] == epoch) continue;
        visited[nb] = epoch;
        if (slots[1 + i] >= (uint32_t)L->num_nodes) return -1;
        idxs[n] = nb;
        ptrs[n] = slot_vec(L, slots[1 + i]);
        n++;
    }
    return n;
}

/* beam_search_1536_ref (src/vector/reference/beam_1536.mojo:85-135) on a seeded pool. */
static int beam_1536(const orc_hnsw_layout *L, const int8_t *q, float qn, uint16_t *visited,
                     uint16_t epoch, linear_pool *pool_p, int64_t *evals, int64_t *expansions) {
    linear_pool pool = *pool_p;
    int64_t n_evals = 0, n_expand = 0;
    struct hnsw_scratch s;
    s.visited = visited;
    s.epoch = epoch;
    uint32_t idxs[33];
    const int8_t *ptrs[33];
    /* Fill: expand the nearest unexpanded entry until the pool holds ef. */
    while (pool_has_next(&pool) && pool.size < pool.ef) {
        const uint32_t c = pool_pop(&pool);
        n_expand++;
        const int n = gather(L, c, s.visited, s.epoch, idxs, ptrs);
        if (n < 0) return -1;
        n_evals += n;
        const int batched = n - n % 4;
        for (int j = 0; j < n; ++j) {
            float d;
            if (j < batched)
                d = (qn + slot_norm(ptrs[j])) - 2.0f * (float)ref_dot(q, ptrs[j], HN_DIM);
            else
                d = (float)ref_l2(q, ptrs[j], HN_DIM);
            pool_insert(&pool, d, idxs[j]);
        }
    }
    /* Prune: expand until every pool entry is expanded. */
    while (pool_has_next(&pool)) {
        const uint32_t c = pool_pop(&pool);
        n_expand++;
        float worst = pool_worst(&pool);
        const int n = gather(L, c, s.visited, s.epoch, idxs, ptrs);
        if (n < 0) return -1;
        n_evals += n;
        const int batched = n - n % 4;
        for (int j = 0; j < n; ++j) {
            const int8_t *p = ptrs[j];
            if (j < batched) {
                const float dot =
                    (float)ref_dot(q, p, 256) + (float)ref_dot(q + 256, p + 256, 1280);
                const float d = (qn + slot_norm(p)) - 2.0f * dot;
                if (pool_insert(&pool, d, idxs[j])) worst = pool_worst(&pool);
            } else {
                const float d_prefix = (float)ref_l2(q, p, 256);
                if (d_prefix < worst * 0.175f) {
                    float running = d_prefix;
                    int exited = 0;
                    for (int b = 0; b < 5; ++b) {
                        const int off = 256 + b * 256;
                        running += (float)ref_l2(q + off, p + off, 256);
                        if (running > worst) {
                            exited = 1;
                            break;
                        }
                    }
                    if (!exited && running < worst) pool_insert(&pool, running, idxs[j]);
                }
            }
        }
    }
    *pool_p = pool;
    *evals += n_evals;
    *expansions += n_expand;
    return 0;
}

static void hnsw_item(void *ctx, int64_t t, void *raw) {
    struct hnsw_job *job = (struct hnsw_job *)ctx;
    const orc_hnsw_layout *L = job->L;
    struct hnsw_scratch s;
    scratch_bind(raw, L->num_nodes, job->ef, &s);
    int32_t *oid = job->out_ids + t * job->k;
    float *od = job->out_dist + t * job->k;
    for (int64_t i = 0; i < job->k; ++i) {
        oid[i] = -1;
        od[i] = INFINITY;
    }
    if (L->num_nodes == 0) return;
    if (++s.epoch == 0) {
        memset(s.visited, 0, (size_t)L->num_nodes * 2);
        s.epoch = 1;
    }
    *(uint16_t *)raw = s.epoch;
    query_codes(L, job->queries + t * HN_DIM, s.fq, s.q);
    const int8_t *q = s.q;
    int32_t qn_int = 0;
    for (int i = 0; i < HN_DIM; ++i) qn_int += (int32_t)q[i] * (int32_t)q[i];
    const float qn = (float)qn_int;
    int64_t n_upper = 0, n_evals = 0, n_expand = 0;
    /* FT.SEARCH's start node: _upper_level_greedy quantises the raw query (normalised
     * once, hnsw.mojo:3850-3865) before search_fp32_scored normalises it twice for the
     * beam (src/commands/vector.mojo:4514-4518, src/network/slow_path.mojo:3310-3314). */
    int8_t gq_buf[HN_DIM];
    const int8_t *gq = q;
    if (job->greedy_passes != 2) {
        float gtmp[HN_DIM];
        query_codes_n(L, job->queries + t * HN_DIM, gtmp, gq_buf, job->greedy_passes);
        gq = gq_buf;
    }

    /* _upper_greedy_codes: levels max_level..1, exact INT8 L2 on codes. */
    uint32_t curr = (uint32_t)L->entry_point;
    float curr_dist = (float)ref_l2(gq, slot_vec(L, L->node_slot[curr]), HN_DIM);
    n_upper++;
    for (int64_t l = L->max_level; l > 0; --l) {
        int changed = 1;
        while (changed) {
            changed = 0;
            const uint32_t node = curr;
            int nc = 0;
            const uint32_t *lst = NULL;
            const int64_t off = L->upper_offset[node];
            if (off >= 0 && l <= L->node_level[node]) {
                lst = L->upper_links + (off + l - 1) * (1 + L->M);
                nc = (int)lst[0];
                if (nc > L->M) nc = (int)L->M;
            }
            float best = curr_dist;
            uint32_t best_idx = curr;
            for (int i = 0; i < nc; ++i) {
                const uint32_t nidx = lst[1 + i];
                if (nidx >= (uint32_t)L->num_nodes) continue;
                if (is_deleted(L, nidx)) continue;
                const float d = (float)ref_l2(gq, slot_vec(L, L->node_slot[nidx]), HN_DIM);
                n_upper++;
                if (d < best) {
                    best = d;
                    best_idx = nidx;
                }
            }
            if (best_idx != curr) {
                curr = best_idx;
                curr_dist = best;
                changed = 1;
            }
        }
    }

    /* Base level: mark the start visited, seed the pool with its INT8 distance. */
    s.visited[curr] = s.epoch;
    linear_pool pool;
    pool.e = s.pool;
    pool_reset(&pool, job->ef);
    pool_insert(&pool, (float)ref_l2(q, slot_vec(L, L->node_slot[curr]), HN_DIM), curr);

    if (beam_1536(L, q, qn, s.visited, s.epoch, &pool, &n_evals, &n_expand) != 0) {
        job->bad++;
        return;
    }
    /* Drain: the first k entries, nearest first. */
    const int64_t n_out = job->k < pool.size ? job->k : pool.size;
    for (int64_t i = 0; i < n_out; ++i) {
        oid[i] = L->node_ids[pool.e[i].id & ~HN_CHECKED];
        od[i] = pool.e[i].dist;
    }
    job->evals += n_evals;
    job->expansions += n_expand;
    job->upper += n_upper;
}

static int hnsw_search_passes(const orc_hnsw_layout *L, const float *queries, int64_t nq,
                              int64_t k, int64_t ef, int32_t *out_ids, float *out_dist,
                              int64_t *stats3, int nthreads, int greedy_passes);

int orc_hnsw_search(const orc_hnsw_layout *L, const float *queries, int64_t nq, int64_t k,
                    int64_t ef, int32_t *out_ids, float *out_dist, int64_t *stats3, int nthreads) {
    return hnsw_search_passes(L, queries, nq, k, ef, out_ids, out_dist, stats3, nthreads, 2);
}

/* The FT.SEARCH composition: the start node as _upper_level_greedy finds it on the raw
 * query (codes of the once-normalised query), then search_fp32_scored from that node. */
int orc_hnsw_search_ft(const orc_hnsw_layout *L, const float *queries, int64_t nq, int64_t k,
                       int64_t ef, int32_t *out_ids, float *out_dist, int64_t *stats3,
                       int nthreads) {
    return hnsw_search_passes(L, queries, nq, k, ef, out_ids, out_dist, stats3, nthreads, 1);
}

static int hnsw_search_passes(const orc_hnsw_layout *L, const float *queries, int64_t nq,
                              int64_t k, int64_t ef, int32_t *out_ids, float *out_dist,
                              int64_t *stats3, int nthreads, int greedy_passes) {
    if (L->dim != HN_DIM || k < 1 || ef < 1) return -1;
    if (L->num_nodes > 0 && (L->entry_point < 0 || L->entry_point >= L->num_nodes)) return -1;
    struct hnsw_job job;
    job.L = L;
    job.queries = queries;
    job.k = k;
    job.ef = ef;
    job.greedy_passes = greedy_passes;
    job.out_ids = out_ids;
    job.out_dist = out_dist;
    job.evals = 0;
    job.expansions = 0;
    job.upper = 0;
    job.bad = 0;
    orc_parallel_for(nq, nthreads, scratch_bytes(L->num_nodes, ef), hnsw_item, &job);
    if (stats3) {
        stats3[0] += job.evals;
        stats3[1] += job.expansions;
        stats3[2] += job.upper;
    }
    return job.bad ? -1 : 0;
}

/* The level-0 beam alone from a caller-seeded pool (the contract of the reference's
 * pion_v_beam_1536): codes q[1536], qn = the query's |code|^2 as the view holds it, the
 * pool's n_init entries (dist, id with bit 31 = expanded) and cursor; the nodes of the
 * pool count as visited.  The final pool goes to out (ef entries at most); returns its
 * size, or -1. */
int64_t orc_hnsw_beam_pool(const orc_hnsw_layout *L, const int8_t *q, float qn, int64_t ef,
                           const float *init_d, const uint32_t *init_id, int64_t n_init,
                           int64_t cursor, float *out_d, uint32_t *out_id) {
    if (ef < 1) ef = 1;
    if (n_init > ef || n_init < 0) return -1;
    uint16_t *visited = (uint16_t *)calloc((size_t)L->num_nodes, sizeof(uint16_t));
    pool_entry *e = (pool_entry *)malloc((size_t)ef * sizeof(pool_entry));
    if (!visited || !e) {
        free(visited);
        free(e);
        return -1;
    }
    linear_pool pool;
    pool.e = e;
    pool.ef = ef;
    pool.size = n_init;
    pool.cursor = cursor < n_init ? cursor : n_init;
    for (int64_t i = 0; i < n_init; ++i) {
        e[i].dist = init_d[i];
        e[i].id = init_id[i];
        const uint32_t nd = init_id[i] & ~HN_CHECKED;
        if (nd < (uint32_t)L->num_nodes) visited[nd] = 1;
    }
    int64_t evals = 0, expansions = 0;
    const int rc = beam_1536(L, q, qn, visited, 1, &pool, &evals, &expansions);
    for (int64_t i = 0; rc == 0 && i < pool.size; ++i) {
        out_d[i] = e[i].dist;
        out_id[i] = e[i].id;
    }
    free(visited);
    free(e);
    return rc == 0 ? pool.size : -1;
}

/* metric_scores' FP32-copy branch (src/vector/hnsw.mojo:4586-4600, 4643-4647): the
 * rows by node (the block-quantised formats keep them so), the query normalised once under
 * COSINE and not clamped; 4 chains of 8 lanes over 32-element strides (mul then add),
 * (c0 + c1) + (c2 + c3) lane-wise, the halving reduce_add; COSINE halves it.  ids are
 * external ids (node_ids of the n nodes); scores in/out. */
void orc_metric_scores_f32(const int32_t *node_ids, int64_t n, int metric, const float *rows,
                           const float *queries, int64_t nq, int64_t k, const int32_t *ids,
                           float *scores) {
    float qc[HN_DIM];
    for (int64_t t = 0; t < nq; ++t) {
        const float *x = queries + t * HN_DIM;
        if (metric == 1)
            orc_l2_normalize_fp32(x, qc, HN_DIM);
        else
            memcpy(qc, x, HN_DIM * sizeof(float));
        for (int64_t r = 0; r < k; ++r) {
            const int32_t ext = ids[t * k + r];
            int64_t node = -1;
            for (int64_t i = 0; i < n && node < 0; ++i)
                if (node_ids[i] == ext) node = i;
            if (node < 0) continue;
            const float *v = rows + node * HN_DIM;
            float acc[4][8];
            memset(acc, 0, sizeof(acc));
            for (int d0 = 0; d0 + 32 <= HN_DIM; d0 += 32)
                for (int ch = 0; ch < 4; ++ch)
                    for (int l = 0; l < 8; ++l) {
                        const int d = d0 + 8 * ch + l;
                        const float e = qc[d] - v[d];
                        acc[ch][l] = e * e + acc[ch][l];
                    }
            float lanes[8];
            for (int l = 0; l < 8; ++l) lanes[l] = (acc[0][l] + acc[1][l]) + (acc[2][l] + acc[3][l]);
            for (int w = 8; w > 1; w /= 2)
                for (int i = 0; i < w / 2; ++i) lanes[i] = lanes[i] + lanes[i + w / 2];
            scores[t * k + r] = metric == 1 ? lanes[0] * 0.5f : lanes[0];
        }
    }
}

/* metric_scores (src/vector/hnsw.mojo:4523-4651), INT8 codes with one global calibration
 * and no FP32 copy (the Linux build): the query normalised once under COSINE, clamped to
 * [gmin, gmax]; each code dequantised at the middle of its step, c * g + (127.5 g + gmin)
 * with g = range / 254 (mul then add: the x86-64-v2 build has no FMA); 4 chains of 8 SIMD
 * lanes over 32-element strides; (c0 + c1) + (c2 + c3) lane-wise, then the SIMD reduce_add
 * (halving tree); COSINE halves the squared L2.  ids are external ids; scores in/out. */
void orc_hnsw_metric_scores(const orc_hnsw_layout *L, const float *queries, int64_t nq,
                            int64_t k, const int32_t *ids, float *scores) {
    const int64_t n = L->num_nodes;
    if (n <= 0) return;
    int64_t lo = L->node_ids[0], hi = L->node_ids[0];
    for (int64_t i = 1; i < n; ++i) {
        if (L->node_ids[i] < lo) lo = L->node_ids[i];
        if (L->node_ids[i] > hi) hi = L->node_ids[i];
    }
    int32_t *map = (int32_t *)malloc((size_t)(hi - lo + 1) * sizeof(int32_t));
    float *qc = (float *)malloc(HN_DIM * sizeof(float));
    if (!map || !qc) {
        free(map);
        free(qc);
        return;
    }
    for (int64_t i = 0; i < hi - lo + 1; ++i) map[i] = -1;
    for (int64_t i = 0; i < n; ++i) map[L->node_ids[i] - lo] = (int32_t)i;
    float range = L->global_max - L->global_min;
    if (range <= 0.0f) range = 1.0f;
    const float g = range / 254.0f;
    const float b = 127.5f * g + L->global_min;
    for (int64_t t = 0; t < nq; ++t) {
        const float *x = queries + t * HN_DIM;
        if (L->metric == 1)
            orc_l2_normalize_fp32(x, qc, HN_DIM);
        else
            memcpy(qc, x, HN_DIM * sizeof(float));
        for (int d = 0; d < HN_DIM; ++d) {
            float v = qc[d];
            if (v < L->global_min) v = L->global_min;
            if (v > L->global_max) v = L->global_max;
            qc[d] = v;
        }
        for (int64_t r = 0; r < k; ++r) {
            const int64_t ext = ids[t * k + r];
            if (ext < lo || ext > hi) continue;
            const int32_t node = map[ext - lo];
            if (node < 0) continue;
            const int8_t *c = slot_vec(L, L->node_slot[node]);
            float acc[4][8];
            memset(acc, 0, sizeof(acc));
            for (int d0 = 0; d0 + 32 <= HN_DIM; d0 += 32)
                for (int ch = 0; ch < 4; ++ch)
                    for (int l = 0; l < 8; ++l) {
                        const int d = d0 + 8 * ch + l;
                        const float xv = (float)c[d] * g + b;
                        const float e = qc[d] - xv;
                        acc[ch][l] = e * e + acc[ch][l];
                    }
            float lanes[8];
            for (int l = 0; l < 8; ++l) lanes[l] = (acc[0][l] + acc[1][l]) + (acc[2][l] + acc[3][l]);
            for (int w = 8; w > 1; w /= 2)
                for (int i = 0; i < w / 2; ++i) lanes[i] = lanes[i] + lanes[i + w / 2];
            float sc = lanes[0];
            if (L->metric == 1) sc = sc * 0.5f;
            scores[t * k + r] = sc;
        }
    }
    free(map);
    free(qc);
}

/* The GPU brute-force scan of the slot buffer for one query.
 * int8_l2_distance_batch (src/ffi/metal_compute.metal:19-78):
 *   d = query_norm + cand_norm - 2 * float(dot), cand_norm = the slot header's |code|^2.
 * pion_metal_search_topk_w (src/ffi/metal_wrap.m:495-580): num_vectors is clamped to the
 * registered slots and k to num_vectors; k entries start as (+inf, -1), worst = +inf at
 * entry 0; for every slot in order, d < worst overwrites entry worst_idx, then worst and
 * worst_idx become the first maximum of the k entries.  The entries stay in that order
 * (the caller sorts).  Returns k. */
int64_t orc_slot_scan_topk(const orc_hnsw_layout *L, const int8_t *q, float qn,
                           int64_t num_vectors, int64_t k, int32_t *out_slots, float *out_d) {
    if (num_vectors > L->num_nodes) num_vectors = L->num_nodes;
    if (num_vectors < 0) num_vectors = 0;
    if (k > num_vectors) k = num_vectors;
    if (k < 0) k = 0;
    for (int64_t i = 0; i < k; ++i) {
        out_d[i] = INFINITY;
        out_slots[i] = -1;
    }
    float worst = INFINITY;
    int64_t widx = 0;
    for (int64_t s = 0; s < num_vectors; ++s) {
        const int8_t *v = slot_vec(L, (uint32_t)s);
        int32_t dot = 0;
        for (int d = 0; d < HN_DIM; ++d) dot += (int32_t)q[d] * (int32_t)v[d];
        const float sum = qn + slot_norm(v);
        const float dist = sum - 2.0f * (float)dot;
        if (dist < worst) {
            out_d[widx] = dist;
            out_slots[widx] = (int32_t)s;
            worst = -INFINITY;
            for (int64_t j = 0; j < k; ++j)
                if (out_d[j] > worst) {
                    worst = out_d[j];
                    widx = j;
                }
        }
    }
    return k;
}

/* Exact FP32 L2^2 of the CPU rerank loop of search_gpu_brute_force (src/vector/hnsw.mojo:
 * 3954-3965): 8 SIMD lanes, lane l over elements 8i + l, acc = acc + diff * diff, then
 * the SIMD reduce_add (halving tree). */
static float rerank_l2(const float *q, const float *v) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int i = 0; i < HN_DIM / 8; ++i)
        for (int l = 0; l < 8; ++l) {
            const float diff = q[8 * i + l] - v[8 * i + l];
            acc[l] = acc[l] + diff * diff;
        }
    for (int w = 8; w > 1; w /= 2)
        for (int i = 0; i < w / 2; ++i) acc[i] = acc[i] + acc[i + w / 2];
    return acc[0];
}

/* search_gpu_brute_force (src/vector/hnsw.mojo:3916-3992) per query: codes of the query
 * normalised once (_quantize_query_to_int8), query_norm = the integer |code|^2 as f32
 * (norm_sq_int8_jit, src/vector/kernels.mojo:362-376); oversample = min(2 k', n, 256)
 * with rerank rows (k' = min(k, n)), else min(k', 256); the scan above; with rerank rows
 * every entry's distance becomes the FP32 L2^2 of the raw query and its slot's row; a
 * stable insertion sort by distance; the first k' entries as (slot's external id,
 * distance).  out_ids/out_scores [nq x k] (-1 / +inf past out_found[t]). */
void orc_hnsw_brute_force(const orc_hnsw_layout *L, const float *rerank, const float *queries,
                          int64_t nq, int64_t k, int32_t *out_ids, float *out_scores,
                          int32_t *out_found) {
    const int64_t n = L->num_nodes;
    for (int64_t i = 0; i < nq * k; ++i) {
        out_ids[i] = -1;
        out_scores[i] = INFINITY;
    }
    for (int64_t t = 0; t < nq; ++t) out_found[t] = 0;
    if (n <= 0 || k <= 0) return;
    int32_t *slot_ext = (int32_t *)malloc((size_t)n * sizeof(int32_t));
    int32_t *ids = (int32_t *)malloc(256 * sizeof(int32_t));
    float *dist = (float *)malloc(256 * sizeof(float));
    float *tmp = (float *)malloc(HN_DIM * sizeof(float));
    int8_t *codes = (int8_t *)malloc(HN_DIM);
    if (!slot_ext || !ids || !dist || !tmp || !codes) goto done;
    for (int64_t i = 0; i < n; ++i) slot_ext[i] = -1;
    for (int64_t i = 0; i < n; ++i)
        if (L->node_slot[i] < (uint32_t)n) slot_ext[L->node_slot[i]] = L->node_ids[i];
    const int64_t final_k = k < n ? k : n;
    int64_t over;
    if (rerank) {
        over = 2 * final_k;
        if (over > n) over = n;
        if (over > 256) over = 256;
    } else {
        over = final_k < 256 ? final_k : 256;
    }
    for (int64_t t = 0; t < nq; ++t) {
        const float *x = queries + t * HN_DIM;
        query_codes_n(L, x, tmp, codes, 1);
        int32_t qn_i = 0;
        for (int d = 0; d < HN_DIM; ++d) qn_i += (int32_t)codes[d] * (int32_t)codes[d];
        int64_t found = orc_slot_scan_topk(L, codes, (float)qn_i, n, over, ids, dist);
        if (rerank)
            for (int64_t i = 0; i < found; ++i)
                if (ids[i] >= 0 && ids[i] < n)
                    dist[i] = rerank_l2(x, rerank + (int64_t)ids[i] * HN_DIM);
        for (int64_t i = 1; i < found; ++i)
            for (int64_t j = i; j > 0 && dist[j] < dist[j - 1]; --j) {
                const float td = dist[j];
                dist[j] = dist[j - 1];
                dist[j - 1] = td;
                const int32_t ti = ids[j];
                ids[j] = ids[j - 1];
                ids[j - 1] = ti;
            }
        if (found > final_k) found = final_k;
        int32_t c = 0;
        for (int64_t i = 0; i < found; ++i)
            if (ids[i] >= 0 && ids[i] < n) {
                out_ids[t * k + c] = slot_ext[ids[i]];
                out_scores[t * k + c] = dist[i];
                ++c;
            }
        out_found[t] = c;
    }
done:
    free(slot_ext);
    free(ids);
    free(dist);
    free(tmp);
    free(codes);
}
