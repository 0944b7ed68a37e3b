/* CPU oracle (test infrastructure, not the product): the three block-quantised HNSW
 * searches at dim 1536, restated from the reference.
 *
 *   src/vector/kernels.mojo:1116-1175   quantize_fp32_to_block_int4 (PolarQuant)
 *   src/vector/kernels.mojo:1422-1455   quantize_fp32_to_block_int8 (the query)
 *   src/vector/kernels.mojo:1508-1520   _pack_8_int3;  :1536-1547 _unpack16_int3
 *   src/vector/kernels.mojo:1589-1651   quantize_fp32_to_block_int3 (TurboQuant)
 *   src/vector/kernels.mojo:1685-1714   qjl_compute_signs;  :981-1019 wht_fp32_1536
 *   src/vector/kernels.mojo:1729-1750   _pack_16_int2 / _unpack16_int2
 *   src/vector/kernels.mojo:1776-1842   quantize_fp32_to_block_int2 (NanoQuant)
 *   src/vector/reference/quant_dots.mojo:45-102      ref_int4/3/2_dot, ref_hamming
 *   src/vector/reference/quant_beams_1536.mojo:20-81 quant_beam_search_1536_ref
 *   src/common/heap.mojo:48-120, 237-339             MinHeap, MaxHeap
 *   src/vector/hnsw.mojo:3138-3230      TurboQuant's residual and QJL rows (by node)
 *   src/vector/hnsw.mojo:497-509        the QJL random signs (LCG seeded 42)
 *   src/vector/hnsw.mojo:4136-4330      search_fp32_scored's three block-quant branches
 *   src/vector/hnsw.mojo:4052-4134      _rerank_fp32_sorted
 *
 * Slot layout (hdr 0): f32 reconstructed |v|^2, then 48 blocks of an f16 scale and the
 * packed codes (INT4 16 bytes, INT3 12, INT2 8), stride 868 / 676 / 484.  f16 values are
 * rounded to nearest even, as the reference's Float32 -> Float16 cast is.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "pion_oracle.h"

#define QD 1536
#define QB 48
#define QW 24 /* QJL words */

uint16_t orc_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t exp = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (exp == 0xffu) return (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0u));
    const int e = (int)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        const int shift = 14 - e;
        uint32_t h = man >> shift;
        const uint32_t rem = man & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u))) ++h;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)e << 10) | (man >> 13);
    const uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
}

float orc_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu;
    uint32_t x;
    if (exp == 0) {
        if (man == 0) {
            x = sign;
        } else {  /* subnormal: normalise */
            int e = -1;
            uint32_t m = man;
            do {
                ++e;
                m <<= 1;
            } while ((m & 0x400u) == 0);
            x = sign | ((uint32_t)(127 - 15 - e) << 23) | ((m & 0x3ffu) << 13);
        }
    } else if (exp == 31) {
        x = sign | 0x7f800000u | (man << 13);
    } else {
        x = sign | ((exp - 15 + 127) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

static float load_f32(const int8_t *p) {
    float f;
    memcpy(&f, p, 4);
    return f;
}

static float load_f16(const int8_t *p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return orc_f16_to_f32(h);
}

static void store_f16(int8_t *p, float f) {
    const uint16_t h = orc_f32_to_f16(f);
    memcpy(p, &h, 2);
}

/* Int(q_f + 0.5) if q_f >= 0 else Int(q_f - 0.5): round half away from zero, then the
 * conversion truncates. */
static int round_away(float q_f) {
    return q_f >= 0.0f ? (int)(q_f + 0.5f) : (int)(q_f - 0.5f);
}

int64_t orc_quant_stride(int kind) {
    return kind == ORC_QUANT_POLAR ? 868 : kind == ORC_QUANT_NANO ? 484 : 676;
}

/* One vector's slot in the block format of `kind`. */
void orc_quant_block(int kind, const float *src, int8_t *dst) {
    float recon = 0.0f;
    int off = 4;
    const float qmax = kind == ORC_QUANT_POLAR ? 7.0f : kind == ORC_QUANT_NANO ? 1.5f : 3.0f;
    for (int b = 0; b < QB; ++b) {
        const float *x = src + b * 32;
        float absmax = 0.0f;
        for (int i = 0; i < 32; ++i) {
            const float av = x[i] >= 0 ? x[i] : -x[i];
            if (av > absmax) absmax = av;
        }
        const float scale = absmax > 0 ? absmax / qmax : 1.0f;
        const float inv = 1.0f / scale;
        int q[32];
        if (kind == ORC_QUANT_NANO) {
            const float stored = scale * 0.5f;
            store_f16(dst + off, stored);
            for (int i = 0; i < 32; ++i) {
                const float q_f = x[i] * inv + 1.5f;
                int v = round_away(q_f);
                if (v > 3) v = 3;
                if (v < 0) v = 0;
                q[i] = v;
                const float r = (float)(v * 2 - 3) * stored;
                recon = recon + r * r;
            }
        } else {
            store_f16(dst + off, scale);
            const int lo = kind == ORC_QUANT_POLAR ? -8 : -4, hi = kind == ORC_QUANT_POLAR ? 7 : 3;
            for (int i = 0; i < 32; ++i) {
                const float q_f = x[i] * inv;
                int v = round_away(q_f);
                if (v > hi) v = hi;
                if (v < lo) v = lo;
                q[i] = v;
                const float r = (float)v * scale;
                recon = recon + r * r;
            }
        }
        off += 2;
        uint8_t *d = (uint8_t *)dst + off;
        if (kind == ORC_QUANT_POLAR) {
            for (int i = 0; i < 16; ++i)
                d[i] = (uint8_t)(((q[i + 16] + 8) << 4) | (q[i] + 8));
            off += 16;
        } else if (kind == ORC_QUANT_NANO) {
            for (int g = 0; g < 8; ++g)
                d[g] = (uint8_t)(q[4 * g] | (q[4 * g + 1] << 2) | (q[4 * g + 2] << 4) |
                                 (q[4 * g + 3] << 6));
            off += 8;
        } else {
            for (int g = 0; g < 4; ++g) {
                int v[8];
                for (int i = 0; i < 8; ++i) v[i] = q[8 * g + i] + 4;
                uint8_t *o = d + 3 * g;
                o[0] = (uint8_t)(v[0] | (v[1] << 3) | ((v[2] & 3) << 6));
                o[1] = (uint8_t)((v[2] >> 2) | (v[3] << 1) | (v[4] << 4) | ((v[5] & 1) << 7));
                o[2] = (uint8_t)((v[5] >> 1) | (v[6] << 2) | (v[7] << 5));
            }
            off += 12;
        }
    }
    memcpy(dst, &recon, 4);
}

/* The 32 codes of block b of a slot (dims in order). */
static void block_codes(int kind, const int8_t *v, int b, int *c) {
    const int64_t bb = kind == ORC_QUANT_POLAR ? 18 : kind == ORC_QUANT_NANO ? 10 : 14;
    const uint8_t *d = (const uint8_t *)v + 4 + b * bb + 2;
    if (kind == ORC_QUANT_POLAR) {
        for (int i = 0; i < 16; ++i) {
            c[i] = (d[i] & 0x0f) - 8;
            c[i + 16] = (d[i] >> 4) - 8;
        }
    } else if (kind == ORC_QUANT_NANO) {
        for (int h = 0; h < 2; ++h) {
            const uint64_t p = (uint64_t)d[4 * h] | ((uint64_t)d[4 * h + 1] << 8) |
                               ((uint64_t)d[4 * h + 2] << 16) | ((uint64_t)d[4 * h + 3] << 24);
            for (int k = 0; k < 16; ++k) c[16 * h + k] = (int)((p >> (2 * k)) & 3) * 2 - 3;
        }
    } else {
        for (int g = 0; g < 4; ++g) {
            const uint64_t u = (uint64_t)d[3 * g] | ((uint64_t)d[3 * g + 1] << 8) |
                               ((uint64_t)d[3 * g + 2] << 16);
            for (int k = 0; k < 8; ++k) c[8 * g + k] = (int)((u >> (3 * k)) & 7) - 4;
        }
    }
}

/* ref_int4/int3/int2_dot: per block an exact int32 dot, times (q scale * v scale),
 * accumulated block by block. */
float orc_quant_dot(int kind, const int8_t *qc, const float *qs, const int8_t *v) {
    const int64_t bb = kind == ORC_QUANT_POLAR ? 18 : kind == ORC_QUANT_NANO ? 10 : 14;
    float total = 0.0f;
    int c[32];
    for (int b = 0; b < QB; ++b) {
        const float combined = qs[b] * load_f16(v + 4 + b * bb);
        block_codes(kind, v, b, c);
        int32_t acc = 0;
        for (int i = 0; i < 32; ++i) acc += (int32_t)qc[b * 32 + i] * c[i];
        total = total + (float)acc * combined;
    }
    return total;
}

/* quantize_fp32_to_block_int8: returns the reconstructed |q|^2. */
float orc_query_block_int8(const float *q, int8_t *codes, float *scales) {
    float recon = 0.0f;
    for (int b = 0; b < QB; ++b) {
        const float *x = q + b * 32;
        float absmax = 0.0f;
        for (int i = 0; i < 32; ++i) {
            const float av = x[i] >= 0 ? x[i] : -x[i];
            if (av > absmax) absmax = av;
        }
        const float scale = absmax > 0 ? absmax / 127.0f : 1.0f;
        const float inv = 1.0f / scale;
        scales[b] = scale;
        for (int i = 0; i < 32; ++i) {
            int v = round_away(x[i] * inv);
            if (v > 127) v = 127;
            if (v < -127) v = -127;
            codes[b * 32 + i] = (int8_t)v;
            const float r = (float)v * scale;
            recon = recon + r * r;
        }
    }
    return recon;
}

/* The fixed QJL sign flips: an LCG seeded 42, bit 33 of each state. */
void orc_qjl_random_signs(uint64_t *out) {
    uint64_t s = 42;
    for (int w = 0; w < QW; ++w) {
        uint64_t bits = 0;
        for (int b = 0; b < 64; ++b) {
            s = s * 6364136223846793005ull + 1442695040888963407ull;
            if ((s >> 33) & 1ull) bits |= 1ull << b;
        }
        out[w] = bits;
    }
}

static void wht512(float *d) {
    for (int h = 1; h < 512; h *= 2)
        for (int i = 0; i < 512; i += 2 * h)
            for (int j = 0; j < h; ++j) {
                const float x = d[i + j], y = d[i + j + h];
                d[i + j] = x + y;
                d[i + j + h] = x - y;
            }
    const float nv = 0.044194173824159216f;
    for (int i = 0; i < 512; ++i) d[i] = d[i] * nv;
}

/* qjl_compute_signs: signs of WHT(random signs * residual); returns |residual|^2. */
float orc_qjl_signs(const float *residual, const uint64_t *rs, uint64_t *dst) {
    float tmp[QD];
    float n2 = 0.0f;
    for (int i = 0; i < QD; ++i) {
        const float sv = ((rs[i >> 6] >> (i & 63)) & 1ull) ? 1.0f : -1.0f;
        const float r = residual[i];
        tmp[i] = r * sv;
        n2 = n2 + r * r;
    }
    wht512(tmp);
    wht512(tmp + 512);
    wht512(tmp + 1024);
    for (int w = 0; w < QW; ++w) {
        uint64_t bits = 0;
        for (int b = 0; b < 64; ++b)
            if (tmp[w * 64 + b] > 0) bits |= 1ull << b;
        dst[w] = bits;
    }
    return n2;
}

/* TurboQuant's QJL row of one vector (hnsw.mojo:3200-3222): residual = x - decoded. */
float orc_turbo_qjl_row(const float *src, const int8_t *slot, const uint64_t *rs,
                        uint64_t *dst) {
    float res[QD];
    int c[32];
    for (int b = 0; b < QB; ++b) {
        const float sv = load_f16(slot + 4 + b * 14);
        block_codes(ORC_QUANT_TURBO, slot, b, c);
        for (int i = 0; i < 32; ++i) res[b * 32 + i] = src[b * 32 + i] - (float)c[i] * sv;
    }
    return orc_qjl_signs(res, rs, dst);
}

/* ------------------------------------------------------------------ heaps -- */
typedef struct {
    float d;
    int64_t id;
} hnode;

typedef struct {
    hnode *a;
    int64_t n, cap;
    float worst; /* MaxHeap's cached worst */
} heap;

static int heap_grow(heap *h) {
    if (h->n < h->cap) return 0;
    const int64_t nc = h->cap ? 2 * h->cap : 64;
    hnode *p = (hnode *)realloc(h->a, (size_t)nc * sizeof(hnode));
    if (!p) return -1;
    h->a = p;
    h->cap = nc;
    return 0;
}

static void swapn(hnode *a, int64_t i, int64_t j) {
    const hnode t = a[i];
    a[i] = a[j];
    a[j] = t;
}

/* MinHeap (heap.mojo:48-120) */
static int min_push(heap *h, float d, int64_t id) {
    if (heap_grow(h)) return -1;
    h->a[h->n].d = d;
    h->a[h->n].id = id;
    int64_t c = h->n++;
    while (c > 0) {
        const int64_t p = (c - 1) / 2;
        if (h->a[c].d < h->a[p].d) {
            swapn(h->a, c, p);
            c = p;
        } else {
            break;
        }
    }
    return 0;
}

static void min_down(heap *h, int64_t c) {
    for (;;) {
        const int64_t l = 2 * c + 1, r = 2 * c + 2;
        int64_t s = c;
        if (l < h->n && h->a[l].d < h->a[s].d) s = l;
        if (r < h->n && h->a[r].d < h->a[s].d) s = r;
        if (s == c) break;
        swapn(h->a, c, s);
        c = s;
    }
}

static hnode min_pop(heap *h) {
    const hnode root = h->a[0];
    if (h->n > 1) {
        h->a[0] = h->a[--h->n];
        min_down(h, 0);
    } else {
        h->n = 0;
    }
    return root;
}

/* MaxHeap (heap.mojo:237-339) */
static void max_up(heap *h, int64_t c) {
    while (c > 0) {
        const int64_t p = (c - 1) / 2;
        if (h->a[c].d > h->a[p].d) {
            swapn(h->a, c, p);
            c = p;
        } else {
            break;
        }
    }
}

static void max_down(heap *h, int64_t c) {
    for (;;) {
        const int64_t l = 2 * c + 1, r = 2 * c + 2;
        int64_t s = c;
        if (l < h->n && h->a[l].d > h->a[s].d) s = l;
        if (r < h->n && h->a[r].d > h->a[s].d) s = r;
        if (s == c) break;
        swapn(h->a, c, s);
        c = s;
    }
}

static int max_push(heap *h, float d, int64_t id) {
    if (d > h->worst) h->worst = d;
    if (heap_grow(h)) return -1;
    h->a[h->n].d = d;
    h->a[h->n].id = id;
    max_up(h, h->n++);
    return 0;
}

static int max_push_bounded(heap *h, float d, int64_t id, int64_t ef) {
    if (h->n < ef) {
        if (heap_grow(h)) return -1;
        h->a[h->n].d = d;
        h->a[h->n].id = id;
        max_up(h, h->n++);
        if (d > h->worst) h->worst = d;
    } else if (d < h->worst) {
        h->a[0].d = d;
        h->a[0].id = id;
        max_down(h, 0);
        h->worst = h->a[0].d;
    }
    return 0;
}

static hnode max_pop(heap *h) {
    const hnode root = h->a[0];
    if (h->n > 1) {
        h->a[0] = h->a[--h->n];
        max_down(h, 0);
        h->worst = h->a[0].d;
    } else {
        h->n = 0;
        h->worst = -1e30f;
    }
    return root;
}

/* ----------------------------------------------------------------- search -- */

static const int8_t *qslot(const orc_quant_layout *L, int64_t node) {
    return L->compact + (int64_t)L->node_slot[node] * L->stride;
}

static int is_del(const orc_quant_layout *L, int64_t i) {
    return L->deleted && ((L->deleted[i >> 3] >> (i & 7)) & 1);
}

typedef struct {
    int8_t qc[QD];
    float qs[QB];
    float qn;
    uint64_t qsig[QW];
    float qres;
    int has_qjl;
} qctx;

/* The block distance; TurboQuant's QJL correction only where `qjl` is set (the beam:
 * quant_beams_1536.mojo:62-71), not in the upper-level greedy, which scores plain
 * int3_dot_single_simd distances (hnsw.mojo:4224-4246). */
static float qdist(const orc_quant_layout *L, const qctx *Q, const int8_t *v, int64_t nidx,
                   int qjl) {
    const float norm_v = load_f32(v);
    const float dot = orc_quant_dot(L->kind, Q->qc, Q->qs, v);
    if (L->kind != ORC_QUANT_TURBO || !qjl) return (Q->qn + norm_v) - 2.0f * dot;
    float qjl_c = 0.0f;
    if (Q->has_qjl) {
        int ham = 0;
        for (int w = 0; w < QW; ++w)
            ham += __builtin_popcountll(Q->qsig[w] ^ L->qjl[nidx * QW + w]);
        const float inv_m = 1.0f / 1536.0f;
        const float cos_est = (1536.0f - 2.0f * (float)ham) * inv_m;
        qjl_c = L->qjl_lambda * cos_est * (Q->qres * L->qjl_res_norms[nidx]);
    }
    return ((Q->qn + norm_v) - 2.0f * dot) - 2.0f * qjl_c;
}

/* The level-0 beam loop (quant_beams_1536.mojo:20-81) over heaps already seeded. */
static int quant_beam_run(const orc_quant_layout *L, const qctx *Q, int64_t ef,
                          uint8_t *visited, heap *cand, heap *res) {
    const int64_t n = L->num_nodes;
    while (cand->n > 0) {
        const hnode c = min_pop(cand);
        const float worst = res->worst;
        if (c.d > worst && res->n >= ef) break;
        const uint32_t *row = L->l0_compact + c.id * 33;
        const uint32_t *srow = L->l0_slots + c.id * 33;
        const int cnt = (int)row[0];
        for (int i = 0; i < cnt; ++i) {
            const int64_t nidx = row[1 + i];
            if (nidx < 0 || nidx >= n) continue;
            if (is_del(L, nidx)) continue;
            if (visited[nidx]) continue;
            visited[nidx] = 1;
            const uint32_t ns = srow[1 + i];
            const int8_t *v = ns != 0xffffffffu ? L->compact + (int64_t)ns * L->stride : qslot(L, nidx);
            const float d = qdist(L, Q, v, nidx, 1);
            if (min_push(cand, d, nidx) || max_push_bounded(res, d, nidx, ef)) return -1;
        }
    }
    return 0;
}

/* The beam from (start, start_d), as the block-quant branches seed it. */
static int quant_beam(const orc_quant_layout *L, const qctx *Q, int64_t start, float start_d,
                      int64_t ef, uint8_t *visited, heap *cand, heap *res) {
    cand->n = 0;
    res->n = 0;
    res->worst = -1e30f;
    if (min_push(cand, start_d, start) || max_push(res, start_d, start)) return -1;
    visited[start] = 1;
    return quant_beam_run(L, Q, ef, visited, cand, res);
}

/* quant_beam_search_1536_ref on a view's state: the query as codes, scales, |q|^2 and
 * QJL signs (qsig NULL: none), the heaps given as arrays (their nodes visited), both
 * written back with their sizes (candidates up to cand_cap entries; *cand_total = the
 * whole heap's size) and the results' cached worst. */
int orc_quant_beam_heaps(const orc_quant_layout *L, const int8_t *qc, const float *qs,
                         float qn, const uint64_t *qsig, float qres, int64_t ef, float *cand_d,
                         int64_t *cand_id, int64_t *cand_n, int64_t cand_cap,
                         int64_t *cand_total, float *res_d, int64_t *res_id, int64_t *res_n,
                         float *worst) {
    qctx *Q = (qctx *)calloc(1, sizeof(qctx));
    uint8_t *visited = (uint8_t *)calloc((size_t)L->num_nodes, 1);
    heap cand = {0}, res = {0};
    int rc = -1;
    if (!Q || !visited) goto out;
    memcpy(Q->qc, qc, QD);
    memcpy(Q->qs, qs, QB * sizeof(float));
    Q->qn = qn;
    if (qsig) memcpy(Q->qsig, qsig, QW * sizeof(uint64_t));
    Q->qres = qres;
    Q->has_qjl = L->kind == ORC_QUANT_TURBO && L->qjl && L->qjl_res_norms;
    for (int64_t i = 0; i < *cand_n; ++i) {
        if (heap_grow(&cand)) goto out;
        cand.a[cand.n].d = cand_d[i];
        cand.a[cand.n++].id = cand_id[i];
        visited[cand_id[i]] = 1;
    }
    for (int64_t i = 0; i < *res_n; ++i) {
        if (heap_grow(&res)) goto out;
        res.a[res.n].d = res_d[i];
        res.a[res.n++].id = res_id[i];
        visited[res_id[i]] = 1;
    }
    res.worst = *worst;
    if (quant_beam_run(L, Q, ef, visited, &cand, &res)) goto out;
    *cand_total = cand.n;
    *cand_n = cand.n < cand_cap ? cand.n : cand_cap;
    for (int64_t i = 0; i < *cand_n; ++i) {
        cand_d[i] = cand.a[i].d;
        cand_id[i] = cand.a[i].id;
    }
    *res_n = res.n;
    for (int64_t i = 0; i < res.n; ++i) {
        res_d[i] = res.a[i].d;
        res_id[i] = res.a[i].id;
    }
    *worst = res.worst;
    rc = 0;
out:
    free(cand.a);
    free(res.a);
    free(visited);
    free(Q);
    return rc;
}

/* The upper-level greedy of the block-quant branches (hnsw.mojo:4158-4188, 4220-4246,
 * 4266-4290): the loop bound is the count of the node the pass started from while
 * neighbours are read from the current best node, as the reference's loop does; NanoQuant
 * also skips deleted nodes; distances without the QJL term. */
static void quant_greedy(const orc_quant_layout *L, const qctx *Q, int64_t *node, float *dist) {
    int64_t cur = L->entry_point;
    float cd = qdist(L, Q, qslot(L, cur), cur, 0);
    const int64_t M = L->M;
    for (int64_t l = L->max_level; l >= 1; --l) {
        int changed = 1;
        while (changed) {
            changed = 0;
            if (L->node_level[cur] < l) break;
            const int64_t nc = L->upper_links[(L->upper_offset[cur] + l - 1) * (1 + M)];
            for (int64_t i = 0; i < nc; ++i) {
                if (L->node_level[cur] < l) break;
                const uint32_t *urow = L->upper_links + (L->upper_offset[cur] + l - 1) * (1 + M);
                const int64_t nidx = i < M ? (int64_t)urow[1 + i] : -1;
                if (nidx < 0 || nidx >= L->num_nodes) continue;
                if (L->kind == ORC_QUANT_NANO && is_del(L, nidx)) continue;
                const float d = qdist(L, Q, qslot(L, nidx), nidx, 0);
                if (d < cd) {
                    cd = d;
                    cur = nidx;
                    changed = 1;
                }
            }
        }
    }
    *node = cur;
    *dist = cd;
}

/* _rerank_fp32_sorted: 8-lane squared L2 in two accumulators over 16-element steps. */
static float rerank_l2(const float *q, const float *v) {
    float a[8] = {0}, b[8] = {0};
    for (int d = 0; d + 16 <= QD; d += 16)
        for (int l = 0; l < 8; ++l) {
            const float da = q[d + l] - v[d + l];
            a[l] = a[l] + da * da;
            const float db = q[d + 8 + l] - v[d + 8 + l];
            b[l] = b[l] + db * db;
        }
    float s[8];
    for (int l = 0; l < 8; ++l) s[l] = a[l] + b[l];
    for (int w = 8; w > 1; w /= 2)
        for (int i = 0; i < w / 2; ++i) s[i] = s[i] + s[i + w / 2];
    return s[0];
}

struct quant_job {
    const orc_quant_layout *L;
    const float *queries;
    int64_t k, ef;
    int32_t *out_ids;
    float *out_scores;
    int64_t *out_n;
    int failed;
};

static void quant_one(void *arg, int64_t t, void *scratch) {
    (void)scratch;
    struct quant_job *J = (struct quant_job *)arg;
    const orc_quant_layout *L = J->L;
    const int64_t n = L->num_nodes, k = J->k;
    for (int64_t j = 0; j < k; ++j) {
        J->out_ids[t * k + j] = -1;
        J->out_scores[t * k + j] = INFINITY;
    }
    J->out_n[t] = 0;
    if (n <= 0 || L->entry_point < 0) return;
    qctx *Q = (qctx *)calloc(1, sizeof(qctx));
    float *qv = (float *)malloc(QD * sizeof(float));
    uint8_t *visited = (uint8_t *)calloc((size_t)n, 1);
    heap cand = {0}, res = {0};
    if (!Q || !qv || !visited) {
        J->failed = 1;
        goto out;
    }
    const float *x = J->queries + t * QD;
    if (L->metric == 1)
        orc_l2_normalize_fp32(x, qv, QD);
    else
        memcpy(qv, x, QD * sizeof(float));
    Q->qn = orc_query_block_int8(qv, Q->qc, Q->qs);
    Q->has_qjl = L->kind == ORC_QUANT_TURBO && L->qjl && L->qjl_res_norms;
    if (L->kind == ORC_QUANT_TURBO && L->qjl_random_signs) {
        float resid[QD];
        for (int b = 0; b < QB; ++b)
            for (int i = 0; i < 32; ++i)
                resid[b * 32 + i] = qv[b * 32 + i] - (float)Q->qc[b * 32 + i] * Q->qs[b];
        Q->qres = orc_qjl_signs(resid, L->qjl_random_signs, Q->qsig);
    }
    int64_t start;
    float sd;
    quant_greedy(L, Q, &start, &sd);
    if (quant_beam(L, Q, start, sd, J->ef, visited, &cand, &res)) {
        J->failed = 1;
        goto out;
    }
    /* drain farthest first, reverse, rerank, stable insertion sort, first k */
    const int64_t m = res.n;
    int64_t *ids = (int64_t *)malloc((size_t)(m ? m : 1) * sizeof(int64_t));
    float *ds = (float *)malloc((size_t)(m ? m : 1) * sizeof(float));
    if (!ids || !ds) {
        free(ids);
        free(ds);
        J->failed = 1;
        goto out;
    }
    for (int64_t i = 0; i < m; ++i) {
        const hnode h = max_pop(&res);
        ids[m - 1 - i] = h.id;
        ds[m - 1 - i] = h.d;
    }
    if (L->rerank)
        for (int64_t i = 0; i < m; ++i)
            if (ids[i] >= 0 && ids[i] < n) ds[i] = rerank_l2(qv, L->rerank + ids[i] * QD);
    for (int64_t i = 1; i < m; ++i)
        for (int64_t j = i; j > 0 && ds[j] < ds[j - 1]; --j) {
            const float td = ds[j];
            ds[j] = ds[j - 1];
            ds[j - 1] = td;
            const int64_t ti = ids[j];
            ids[j] = ids[j - 1];
            ids[j - 1] = ti;
        }
    int64_t o = 0;
    for (int64_t i = 0; i < (m < k ? m : k); ++i)
        if (ids[i] >= 0 && ids[i] < n) {
            J->out_ids[t * k + o] = L->node_ids[ids[i]];
            J->out_scores[t * k + o] = ds[i];
            ++o;
        }
    J->out_n[t] = o;
    free(ids);
    free(ds);
out:
    free(cand.a);
    free(res.a);
    free(visited);
    free(qv);
    free(Q);
}

int orc_quant_search(const orc_quant_layout *L, const float *queries, int64_t nq, int64_t k,
                     int64_t ef, int32_t *out_ids, float *out_scores, int64_t *out_n,
                     int nthreads) {
    struct quant_job J = {L, queries, k, ef, out_ids, out_scores, out_n, 0};
    orc_parallel_for(nq, nthreads, 0, quant_one, &J);
    return J.failed ? -1 : 0;
}
