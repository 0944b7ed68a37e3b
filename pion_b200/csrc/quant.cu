// Block-quantised HNSW search on sm_100a: the three block-quant branches of the
// reference's search_fp32_scored at dim 1536 (src/vector/hnsw.mojo:4136-4330) with the
// FP32 rerank tail _rerank_fp32_sorted (hnsw.mojo:4052-4134), one warp per query.
//
//   prologue  the query normalised under COSINE (l2_normalize_fp32, kernels.mojo:318-357),
//             block-quantised to int8 (quantize_fp32_to_block_int8, kernels.mojo:1422-1455)
//             and, for TurboQuant, its QJL signs (qjl_compute_signs, kernels.mojo:1685-1714:
//             residual x random signs, three 512-point Walsh-Hadamard transforms);
//   greedy    the upper levels with the block distance (TurboQuant without its QJL term),
//             the reference's loop (hnsw.mojo:4158-4290): the bound is the count of the
//             node the pass started from while neighbours are read from the current best
//             node; NanoQuant skips deleted nodes.  The lanes score the row's remaining
//             positions at once and the first strictly closer one moves;
//   beam      quant_beam_search_1536_ref (src/vector/reference/quant_beams_1536.mojo:20-81)
//             over the reference's binary heaps (src/common/heap.mojo:48-120, 237-339):
//             candidates in a MinHeap, results in a MaxHeap bounded at ef with its cached
//             worst.  Each expansion reads the adjacency row and its slots in one round
//             trip, the lanes take one neighbour each (adjacency order) and drop deleted,
//             visited and repeated nodes; the new neighbours are then scored four lanes to a
//             neighbour (each lane 12 consecutive blocks with all its loads in flight, the
//             block terms folded lane to lane in the reference's order) and their rows sent
//             towards L2; lane 0 pushes them in adjacency order.  The heaps are kept array
//             for array as the reference keeps them (ties pop in the same order).
//   tail      the results drained farthest first and reversed, reranked by the FP32 rows
//             (two 8-lane accumulators over 16-element steps, halving reduce; two rows per
//             warp, 32 loads per lane in flight, the next pair's rows sent towards L2), a
//             stable sort by distance, the first k as external ids.
//
// Distances: (|q|^2 + |v|^2) - 2 dot, dot = sum over blocks of f32(int32 block dot) *
// (q scale * v scale); TurboQuant subtracts 2 (lambda cos_est)(|q res| |v res|) with
// cos_est = (1536 - 2 hamming) / 1536.  The int32 block dots are exact (dp4a on the codes
// with a per-block bias correction), every float step is rounded where the reference
// rounds it, so the distances, heaps and results are the reference's bit for bit.
//
// Device layout of a quantised graph: per slot f32 |v|^2, 48 f16 scales, and the packed
// codes of the reference's blocks back to back (INT4 16 bytes, INT3 12, INT2 8 per
// block: 768 / 576 / 384 bytes, 16-byte aligned rows); QJL sign words and residual norms
// by node.
//
// Memory: the candidate MinHeap's first 1024 entries sit in shared memory, the rest in a
// per-warp global region; a query whose heap outgrows it is recorded and re-run by a
// second launch with room for every node.  Visited sets are a bitmap per resident warp.
// Every loop is bounded by the node count.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "internal.h"

namespace pion {
namespace qb {

constexpr int DIM = 1536;
constexpr int NB = 48;
constexpr int QW = 24;
constexpr int WARPS = 4;
constexpr int TOP = 1024;  // candidate-heap entries in shared memory
constexpr unsigned FULL = 0xffffffffu;
constexpr float WORST0 = -1e30f;  // MaxHeap's worst when empty

struct Entry {
    float d;
    uint32_t id;
};

struct Params {
    int kind;  // kQPolar / kQNano / kQTurbo
    int metric;
    const uint8_t* codes;  // [slot][code_bytes]
    int code_bytes;
    const uint16_t* scales;  // [slot][48] f16
    const float* norms;      // [slot]
    const uint64_t* qjl;     // [node][24] or null
    const float* res_norms;  // [node] or null
    const uint64_t* rsigns;  // [24] or null
    float lambda;
    const float* rerank;  // [node][1536] or null
    const uint32_t* l0_compact;
    const uint32_t* l0_slots;
    const uint32_t* node_slot;
    const int32_t* node_ids;
    const uint8_t* deleted;
    const int8_t* node_level;
    const int64_t* upper_offset;
    const uint32_t* upper_links;
    const uint32_t* upper_slots;  // upper_links with each neighbour replaced by its slot
    int M, max_level;
    int64_t num_nodes, entry;
    const float* queries;
    int nq, k, ef;
    const int* qlist;       // queries to run, or null (all nq)
    const int* qlist_n;     // their count (device)
    uint32_t* visited;      // vis_words per resident warp
    int64_t vis_words;
    Entry* cand_tail;       // per resident warp: candidate entries [TOP, cand_cap)
    int64_t cand_cap;
    int32_t* out_ids;
    float* out_scores;
    int32_t* out_found;
    int* overflow;          // queries whose candidate heap outgrew cand_cap (null: error)
    int* overflow_n;
    unsigned* next_query;
    unsigned long long* stats;  // distance evaluations, expansions
    int* status;
    // From-heaps mode (pion_v_quant_beam_1536): one query, given as codes, scales,
    // {|q|^2, |residual|^2} and QJL signs; the level-0 beam from the caller's heaps
    // (their nodes count as visited), the heaps written back.  heap_meta: {candidates
    // in, results in, worst in (f32 bits), candidates out, results out, worst out}.
    int from_heaps;
    const int8_t* given_codes;
    const float* given_scales;
    const float* given_norms;
    const uint64_t* given_signs;
    Entry* cand_io;  // cand_io_cap entries
    int64_t cand_io_cap;
    Entry* res_io;   // ef entries
    int* heap_meta;
};

// Per-warp shared memory: this fixed part, then TOP candidate entries (also the
// prologue's transform buffer and the tail's result arrays), then ef result entries.
struct Fixed {
    int32_t qw[DIM / 4];  // query codes as dp4a words (NanoQuant: regrouped, see below)
    float qs[NB];         // query block scales
    int32_t qsum[NB];     // sums of the query block codes
    uint64_t qsig[QW];    // query QJL signs
    float nd[32];         // one batch of gathered neighbours, adjacency order: distances,
    uint32_t ni[32];      // nodes,
    uint32_t ns[32];      // slots
    float qn, qres, qinv;
    int scaled;
    int cand_n, res_n;
    float res_worst;
    int abandon;
};

__host__ __device__ constexpr size_t fixed_bytes() { return (sizeof(Fixed) + 15) / 16 * 16; }
__host__ __device__ constexpr size_t warp_bytes(int ef) {
    return fixed_bytes() + (size_t)TOP * sizeof(Entry) +
           ((size_t)ef * sizeof(Entry) + 15) / 16 * 16;
}

__device__ __forceinline__ bool is_deleted(const uint8_t* del, uint32_t i) {
    return del && ((del[i >> 3] >> (i & 7)) & 1u);
}

// ---------------------------------------------------------------- block dots --

// INT4 (PolarQuant): byte i of a block holds dim i in its low nibble and dim i + 16 in
// its high nibble, each biased by 8.
__device__ __forceinline__ int dot_i4(uint4 w, const int32_t* q, int qsum) {
    int a = 0;
    a = __dp4a((int)(w.x & 0x0f0f0f0fu), q[0], a);
    a = __dp4a((int)((w.x >> 4) & 0x0f0f0f0fu), q[4], a);
    a = __dp4a((int)(w.y & 0x0f0f0f0fu), q[1], a);
    a = __dp4a((int)((w.y >> 4) & 0x0f0f0f0fu), q[5], a);
    a = __dp4a((int)(w.z & 0x0f0f0f0fu), q[2], a);
    a = __dp4a((int)((w.z >> 4) & 0x0f0f0f0fu), q[6], a);
    a = __dp4a((int)(w.w & 0x0f0f0f0fu), q[3], a);
    a = __dp4a((int)((w.w >> 4) & 0x0f0f0f0fu), q[7], a);
    return a - 8 * qsum;
}

// INT2 (NanoQuant): 32-bit word h holds dims 16h + k at bits 2k as u in [0, 3], code
// 2u - 3.  (p >> 2s) & 0x03030303 gathers dims 16h + 4j + s (j = 0..3); the query words
// are regrouped to match: q[4h + s] = bytes of dims 16h + s, +4, +8, +12.
__device__ __forceinline__ int dot_i2(uint32_t p0, uint32_t p1, const int32_t* q, int qsum) {
    int a = 0;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        a = __dp4a((int)((p0 >> (2 * s)) & 0x03030303u), q[s], a);
        a = __dp4a((int)((p1 >> (2 * s)) & 0x03030303u), q[4 + s], a);
    }
    return 2 * a - 3 * qsum;
}

// Four 3-bit fields (bits 0-11) spread to the low bits of four bytes.
__device__ __forceinline__ uint32_t spread3(uint32_t x) {
    return (x & 7u) | ((x & 0x38u) << 5) | ((x & 0x1c0u) << 10) | ((x & 0xe00u) << 15);
}

// INT3 (TurboQuant): 24-bit group g (bytes 3g..3g+2) holds dims 8g + k at bits 3k as
// code + 4.
__device__ __forceinline__ int dot_i3(uint32_t w0, uint32_t w1, uint32_t w2, const int32_t* q,
                                      int qsum) {
    const uint32_t g0 = w0 & 0xffffffu, g1 = (w0 >> 24) | ((w1 & 0xffffu) << 8),
                   g2 = (w1 >> 16) | ((w2 & 0xffu) << 16), g3 = w2 >> 8;
    int a = 0;
    a = __dp4a((int)spread3(g0 & 0xfffu), q[0], a);
    a = __dp4a((int)spread3(g0 >> 12), q[1], a);
    a = __dp4a((int)spread3(g1 & 0xfffu), q[2], a);
    a = __dp4a((int)spread3(g1 >> 12), q[3], a);
    a = __dp4a((int)spread3(g2 & 0xfffu), q[4], a);
    a = __dp4a((int)spread3(g2 >> 12), q[5], a);
    a = __dp4a((int)spread3(g3 & 0xfffu), q[6], a);
    a = __dp4a((int)spread3(g3 >> 12), q[7], a);
    return a - 4 * qsum;
}

// The terms f32(acc_b) * (q scale * v scale) of blocks [12 sub, 12 sub + 12) of slot
// `slot` (ref_int4/3/2_dot, src/vector/reference/quant_dots.mojo:45-102): every load of
// the lane's share of the slot is issued before the first dot.
__device__ __forceinline__ void block_terms(const Params& p, const Fixed& S, uint32_t slot,
                                            int sub, float* t) {
    const int b0 = 12 * sub;
    const uint2* sc = reinterpret_cast<const uint2*>(p.scales + (size_t)slot * NB + b0);
    uint2 sv[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) sv[j] = __ldg(sc + j);
    uint16_t hs[12];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        hs[4 * j] = (uint16_t)(sv[j].x & 0xffffu);
        hs[4 * j + 1] = (uint16_t)(sv[j].x >> 16);
        hs[4 * j + 2] = (uint16_t)(sv[j].y & 0xffffu);
        hs[4 * j + 3] = (uint16_t)(sv[j].y >> 16);
    }
    const uint4* cw = reinterpret_cast<const uint4*>(p.codes + (size_t)slot * p.code_bytes);
    int acc[12];
    if (p.kind == kQPolar) {  // 16 bytes a block
        uint4 w[12];
#pragma unroll
        for (int j = 0; j < 12; ++j) w[j] = __ldg(cw + b0 + j);
#pragma unroll
        for (int j = 0; j < 12; ++j) acc[j] = dot_i4(w[j], S.qw + (b0 + j) * 8, S.qsum[b0 + j]);
    } else if (p.kind == kQNano) {  // 8 bytes a block
        uint4 w[6];
#pragma unroll
        for (int j = 0; j < 6; ++j) w[j] = __ldg(cw + b0 / 2 + j);
#pragma unroll
        for (int j = 0; j < 12; ++j) {
            const uint4 v = w[j >> 1];
            acc[j] = dot_i2((j & 1) ? v.z : v.x, (j & 1) ? v.w : v.y, S.qw + (b0 + j) * 8,
                            S.qsum[b0 + j]);
        }
    } else {  // 12 bytes a block
        uint32_t w[36];
#pragma unroll
        for (int j = 0; j < 9; ++j) {
            const uint4 v = __ldg(cw + (b0 * 12) / 16 + j);
            w[4 * j] = v.x;
            w[4 * j + 1] = v.y;
            w[4 * j + 2] = v.z;
            w[4 * j + 3] = v.w;
        }
#pragma unroll
        for (int j = 0; j < 12; ++j)
            acc[j] = dot_i3(w[3 * j], w[3 * j + 1], w[3 * j + 2], S.qw + (b0 + j) * 8,
                            S.qsum[b0 + j]);
    }
#pragma unroll
    for (int j = 0; j < 12; ++j) {
        const float combined = __fmul_rn(S.qs[b0 + j], __half2float(__ushort_as_half(hs[j])));
        t[j] = __fmul_rn((float)acc[j], combined);
    }
}

// Scores the m (<= 32) gathered neighbours (S.ni nodes at S.ns slots) into S.nd: four
// lanes per neighbour, eight neighbours at a time, each lane dotting 12 consecutive blocks
// and folding its terms onto the running sum handed over by the lane before it, so the 48
// block terms add in the reference's order.  Distance (|q|^2 + |v|^2) - 2 dot, and for
// TurboQuant with `qjl` set the QJL term (quant_beams_1536.mojo:62-71): the greedy scores
// plain block distances.  Called by the whole warp.
__device__ void score_batch(const Params& p, Fixed& S, int m, bool qjl, int lane) {
    const int sub = lane & 3, grp = lane >> 2;
    const bool with_qjl = qjl && p.kind == kQTurbo && p.qjl && p.res_norms;
    for (int base = 0; base < m; base += 8) {
        const int j = base + grp;
        const bool act = j < m;
        const uint32_t slot = act ? S.ns[j] : 0u, node = act ? S.ni[j] : 0u;
        float nv = 0.0f, rn = 0.0f;
        int ham = 0;
        if (act) {
            if (sub == 0) {
                nv = __ldg(p.norms + slot);
                if (with_qjl) rn = __ldg(p.res_norms + node);
            }
            if (with_qjl) {  // six sign words per lane
                const ulonglong2* sg =
                    reinterpret_cast<const ulonglong2*>(p.qjl + (size_t)node * QW + 6 * sub);
#pragma unroll
                for (int w = 0; w < 3; ++w) {
                    const ulonglong2 v = __ldg(sg + w);
                    ham += __popcll(S.qsig[6 * sub + 2 * w] ^ v.x) +
                           __popcll(S.qsig[6 * sub + 2 * w + 1] ^ v.y);
                }
            }
        }
        float t[12];
        if (act) {
            block_terms(p, S, slot, sub, t);
        } else {
#pragma unroll
            for (int i = 0; i < 12; ++i) t[i] = 0.0f;
        }
        float run = 0.0f;
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            if (sub == s) {
#pragma unroll
                for (int i = 0; i < 12; ++i) run = __fadd_rn(run, t[i]);
            }
            run = __shfl_sync(FULL, run, (lane & ~3) | s);
        }
        ham += __shfl_xor_sync(FULL, ham, 1);
        ham += __shfl_xor_sync(FULL, ham, 2);
        if (act && sub == 0) {
            float d = __fsub_rn(__fadd_rn(S.qn, nv), __fmul_rn(2.0f, run));
            if (with_qjl) {
                const float inv_m = __fdiv_rn(1.0f, 1536.0f);
                const float cos_est =
                    __fmul_rn(__fsub_rn(1536.0f, __fmul_rn(2.0f, (float)ham)), inv_m);
                const float qjl_c = __fmul_rn(__fmul_rn(p.lambda, cos_est), __fmul_rn(S.qres, rn));
                d = __fsub_rn(d, __fmul_rn(2.0f, qjl_c));
            }
            S.nd[j] = d;
        }
    }
    __syncwarp();
}

__device__ __forceinline__ void prefetch_l2(const void* ptr) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr));
}

// --------------------------------------------------------------------- heaps --
// Lane 0 only.  Moving a hole instead of swapping leaves the same arrays.

struct Cand {
    Entry* top;   // [0, TOP)
    Entry* tail;  // [TOP, cap)
    int64_t cap;
    __device__ __forceinline__ Entry get(int64_t i) const {
        return i < TOP ? top[i] : tail[i - TOP];
    }
    __device__ __forceinline__ void put(int64_t i, Entry e) const {
        if (i < TOP)
            top[i] = e;
        else
            tail[i - TOP] = e;
    }
};

// MinHeap.push (heap.mojo:48-120)
__device__ bool min_push(const Cand& h, int& n, Entry e) {
    if (n >= h.cap) return false;
    int64_t c = n++;
    while (c > 0) {
        const int64_t par = (c - 1) / 2;
        const Entry pe = h.get(par);
        if (e.d < pe.d) {
            h.put(c, pe);
            c = par;
        } else {
            break;
        }
    }
    h.put(c, e);
    return true;
}

// MinHeap.pop
__device__ Entry min_pop(const Cand& h, int& n) {
    const Entry root = h.get(0);
    if (n > 1) {
        --n;
        const Entry x = h.get(n);
        int64_t c = 0;
        for (;;) {
            const int64_t l = 2 * c + 1, r = 2 * c + 2;
            int64_t s = c;
            float sd = x.d;
            Entry se = x;
            if (l < n) {
                const Entry le = h.get(l);
                if (le.d < sd) {
                    s = l;
                    sd = le.d;
                    se = le;
                }
            }
            if (r < n) {
                const Entry re = h.get(r);
                if (re.d < sd) {
                    s = r;
                    se = re;
                }
            }
            if (s == c) break;
            h.put(c, se);
            c = s;
        }
        h.put(c, x);
    } else {
        n = 0;
    }
    return root;
}

// MaxHeap (heap.mojo:237-339) over a[0, n), shared memory.
__device__ void max_sift_up(Entry* a, int c, Entry e) {
    while (c > 0) {
        const int par = (c - 1) / 2;
        if (e.d > a[par].d) {
            a[c] = a[par];
            c = par;
        } else {
            break;
        }
    }
    a[c] = e;
}

__device__ void max_sift_down(Entry* a, int n, Entry x) {
    int c = 0;
    for (;;) {
        const int l = 2 * c + 1, r = 2 * c + 2;
        int s = c;
        float sd = x.d;
        if (l < n && a[l].d > sd) {
            s = l;
            sd = a[l].d;
        }
        if (r < n && a[r].d > sd) s = r;
        if (s == c) break;
        a[c] = a[s];
        c = s;
    }
    a[c] = x;
}

// push_bounded: below ef entries insert; else replace the root when closer than worst.
__device__ void max_push_bounded(Entry* a, int& n, float& worst, Entry e, int ef) {
    if (n < ef) {
        max_sift_up(a, n++, e);
        if (e.d > worst) worst = e.d;
    } else if (e.d < worst) {
        max_sift_down(a, n, e);
        worst = a[0].d;
    }
}

__device__ Entry max_pop(Entry* a, int& n, float& worst) {
    const Entry root = a[0];
    if (n > 1) {
        --n;
        max_sift_down(a, n, a[n]);
        worst = a[0].d;
    } else {
        n = 0;
        worst = WORST0;
    }
    return root;
}

// ------------------------------------------------------------------ prologue --

__device__ __forceinline__ float qv_at(const float* x, const Fixed& S, int d) {
    const float v = __ldg(x + d);
    return S.scaled ? __fmul_rn(v, S.qinv) : v;
}

__device__ __forceinline__ int round_away(float q) {
    return q >= 0.0f ? __float2int_rz(__fadd_rn(q, 0.5f)) : __float2int_rz(__fsub_rn(q, 0.5f));
}

// NanoQuant's dot regroups the query code words: word 8 b + 4 h + s = the bytes of dims
// 32 b + 16 h + s, +4, +8, +12.
__device__ void regroup_nano(Fixed& S, int lane) {
    const int8_t* qc = reinterpret_cast<const int8_t*>(S.qw);
    int32_t v[12];
#pragma unroll
    for (int r = 0; r < 12; ++r) {
        const int wi = lane + 32 * r, b = wi >> 3, m = wi & 7, h = m >> 2, s = m & 3;
        const int8_t* src = qc + b * 32 + 16 * h + s;
        v[r] = (int32_t)((uint32_t)(uint8_t)src[0] | ((uint32_t)(uint8_t)src[4] << 8) |
                         ((uint32_t)(uint8_t)src[8] << 16) | ((uint32_t)(uint8_t)src[12] << 24));
    }
    __syncwarp();
#pragma unroll
    for (int r = 0; r < 12; ++r) S.qw[lane + 32 * r] = v[r];
}

// The query's codes, scales, |q|^2 and (TurboQuant) QJL signs; `tmp` holds >= 1536 floats.
__device__ void prologue(const Params& p, Fixed& S, const float* x, float* tmp, int lane) {
    // l2_normalize_fp32: four running sums (d mod 4), (s0 + s2) + (s1 + s3)
    if (p.metric == 1) {
        float s = 0.0f;
        if (lane < 4)
            for (int d = lane; d < DIM; d += 4) {
                const float v = __ldg(x + d);
                s = __fadd_rn(s, __fmul_rn(v, v));
            }
        const float s0 = __shfl_sync(FULL, s, 0), s1 = __shfl_sync(FULL, s, 1),
                    s2 = __shfl_sync(FULL, s, 2), s3 = __shfl_sync(FULL, s, 3);
        const float ns = __fadd_rn(__fadd_rn(s0, s2), __fadd_rn(s1, s3));
        if (lane == 0) {
            S.scaled = ns > 0.0f ? 1 : 0;
            S.qinv = ns > 0.0f ? __fdiv_rn(1.0f, __fsqrt_rn(ns)) : 1.0f;
        }
    } else if (lane == 0) {
        S.scaled = 0;
        S.qinv = 1.0f;
    }
    __syncwarp();
    // quantize_fp32_to_block_int8
    int8_t* qc = reinterpret_cast<int8_t*>(S.qw);
    for (int b = 0; b < NB; ++b) {
        const float v = qv_at(x, S, b * 32 + lane);
        float am = v >= 0.0f ? v : -v;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(FULL, am, o));
        const float scale = am > 0.0f ? __fdiv_rn(am, 127.0f) : 1.0f;
        const float inv = __fdiv_rn(1.0f, scale);
        int c = round_away(__fmul_rn(v, inv));
        c = c > 127 ? 127 : (c < -127 ? -127 : c);
        qc[b * 32 + lane] = (int8_t)c;
        const int sum = __reduce_add_sync(FULL, c);
        if (lane == 0) {
            S.qs[b] = scale;
            S.qsum[b] = sum;
        }
    }
    __syncwarp();
    const bool turbo_q = p.kind == kQTurbo && p.rsigns;
    if (turbo_q) {  // residual x random signs
        for (int i = lane; i < DIM; i += 32) {
            const float r = __fsub_rn(qv_at(x, S, i), __fmul_rn((float)qc[i], S.qs[i >> 5]));
            const bool pos = (__ldg(p.rsigns + (i >> 6)) >> (i & 63)) & 1ull;
            tmp[i] = __fmul_rn(r, pos ? 1.0f : -1.0f);
        }
    }
    // the reconstructed |q|^2 and the residual's |r|^2, each summed in order
    if (lane == 0) {
        float recon = 0.0f, n2 = 0.0f;
        for (int i = 0; i < DIM; ++i) {
            const float r = __fmul_rn((float)qc[i], S.qs[i >> 5]);
            recon = __fadd_rn(recon, __fmul_rn(r, r));
            if (turbo_q) {
                const float e = __fsub_rn(qv_at(x, S, i), r);
                n2 = __fadd_rn(n2, __fmul_rn(e, e));
            }
        }
        S.qn = recon;
        S.qres = n2;
        if (!turbo_q)
            for (int w = 0; w < QW; ++w) S.qsig[w] = 0;
    }
    __syncwarp();
    if (turbo_q) {  // wht_fp32_1536: three 512-point transforms, scaled, then signs
        for (int h = 1; h < 512; h *= 2) {
            for (int t = lane; t < 3 * 256; t += 32) {
                const int seg = t >> 8, pr = t & 255;
                const int i = seg * 512 + (pr / h) * 2 * h + (pr % h), j = i + h;
                const float a = tmp[i], c = tmp[j];
                tmp[i] = __fadd_rn(a, c);
                tmp[j] = __fsub_rn(a, c);
            }
            __syncwarp();
        }
        const float nv = 0.044194173824159216f;
        for (int w = 0; w < QW; ++w) {
            const unsigned lo = __ballot_sync(FULL, __fmul_rn(tmp[w * 64 + lane], nv) > 0.0f);
            const unsigned hi = __ballot_sync(FULL, __fmul_rn(tmp[w * 64 + 32 + lane], nv) > 0.0f);
            if (lane == 0) S.qsig[w] = (uint64_t)lo | ((uint64_t)hi << 32);
        }
    }
    if (p.kind == kQNano) regroup_nano(S, lane);
    __syncwarp();
}

// The query side given by the caller (the reference's per-query beam view): codes,
// scales, |q|^2 and QJL signs as the engine computed them.
__device__ void given_query(const Params& p, Fixed& S, int lane) {
    int8_t* qc = reinterpret_cast<int8_t*>(S.qw);
    for (int b = 0; b < NB; ++b) {
        const int c = p.given_codes[b * 32 + lane];
        qc[b * 32 + lane] = (int8_t)c;
        const int sum = __reduce_add_sync(FULL, c);
        if (lane == 0) {
            S.qs[b] = p.given_scales[b];
            S.qsum[b] = sum;
        }
    }
    if (lane < QW) S.qsig[lane] = p.given_signs ? p.given_signs[lane] : 0ull;
    if (lane == 0) {
        S.qn = p.given_norms[0];
        S.qres = p.given_norms[1];
        S.scaled = 0;
        S.qinv = 1.0f;
    }
    __syncwarp();
    if (p.kind == kQNano) regroup_nano(S, lane);
    __syncwarp();
}

// -------------------------------------------------------------------- search --

__global__ void __launch_bounds__(WARPS * 32, 4) quant_search_kernel(Params p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t wb = warp_bytes(p.ef);
    unsigned char* base = smem + (size_t)warp * wb;
    Fixed& S = *reinterpret_cast<Fixed*>(base);
    Entry* top = reinterpret_cast<Entry*>(base + fixed_bytes());
    Entry* res = top + TOP;
    const int64_t gw = (int64_t)blockIdx.x * WARPS + warp;
    uint32_t* vis = p.visited + gw * p.vis_words;
    const Cand cand{top, p.cand_tail + gw * (p.cand_cap > TOP ? p.cand_cap - TOP : 0), p.cand_cap};
    const int64_t n = p.num_nodes;
    const int nlist = p.qlist ? *p.qlist_n : p.nq;
    unsigned long long evals = 0, expansions = 0;
    for (;;) {
        unsigned item = 0;
        if (lane == 0) item = atomicAdd(p.next_query, 1u);
        item = __shfl_sync(FULL, item, 0);
        if (item >= (unsigned)nlist) break;
        const int t = p.qlist ? p.qlist[item] : (int)item;
        const float* x = p.queries + (size_t)t * DIM;
        for (int64_t w = lane * 4; w < p.vis_words; w += 128)
            *reinterpret_cast<uint4*>(vis + w) = make_uint4(0, 0, 0, 0);
        if (p.from_heaps) {
            given_query(p, S, lane);
            const int cn = p.heap_meta[0], rn = p.heap_meta[1];
            if (lane == 0) {
                S.cand_n = cn;
                S.res_n = rn;
                S.res_worst = __int_as_float(p.heap_meta[2]);
                S.abandon = 0;
            }
            for (int i = lane; i < cn; i += 32) {
                const Entry e = p.cand_io[i];
                cand.put(i, e);
                atomicOr(vis + (e.id >> 5), 1u << (e.id & 31));
            }
            for (int i = lane; i < rn; i += 32) {
                const Entry e = p.res_io[i];
                res[i] = e;
                atomicOr(vis + (e.id >> 5), 1u << (e.id & 31));
            }
            __syncwarp();
        } else {
            prologue(p, S, x, reinterpret_cast<float*>(top), lane);

            // upper levels
            uint32_t cur = (uint32_t)p.entry;
            if (lane == 0) {
                S.ni[0] = cur;
                S.ns[0] = __ldg(p.node_slot + cur);
            }
            __syncwarp();
            score_batch(p, S, 1, false, lane);
            float cd = S.nd[0];
            ++evals;
            for (int l = p.max_level; l >= 1; --l) {
                for (int64_t pass = 0; pass <= n; ++pass) {  // `changed` loop
                    bool changed = false;
                    if (__ldg(p.node_level + cur) < l) break;
                    const int64_t nc =
                        __ldg(p.upper_links + (__ldg(p.upper_offset + cur) + l - 1) * (1 + p.M));
                    int64_t i = 0;
                    while (i < nc) {
                        if (__ldg(p.node_level + cur) < l) break;
                        const size_t r = (size_t)(__ldg(p.upper_offset + cur) + l - 1) * (1 + p.M);
                        const int64_t pos = i + lane;
                        uint32_t nidx = 0xffffffffu, nslot = 0;
                        if (pos < nc && pos < p.M) {
                            nidx = __ldg(p.upper_links + r + 1 + pos);
                            nslot = __ldg(p.upper_slots + r + 1 + pos);
                        }
                        bool ok = nidx < (uint64_t)n;
                        if (ok && p.kind == kQNano && is_deleted(p.deleted, nidx)) ok = false;
                        const unsigned okm = __ballot_sync(FULL, ok);
                        const int at = __popc(okm & ((1u << lane) - 1u));
                        if (ok) {
                            S.ni[at] = nidx;
                            S.ns[at] = nslot;
                        }
                        __syncwarp();
                        score_batch(p, S, __popc(okm), false, lane);
                        const float d = ok ? S.nd[at] : 0.0f;
                        evals += __popc(okm) * (lane == 0);
                        const unsigned better = __ballot_sync(FULL, ok && d < cd);
                        __syncwarp();  // every lane has read its distance before the next batch
                        if (better == 0) break;  // positions past M are never scored
                        const int f = __ffs(better) - 1;
                        cd = __shfl_sync(FULL, d, f);
                        cur = __shfl_sync(FULL, nidx, f);
                        changed = true;
                        i += f + 1;
                    }
                    if (!changed) break;
                }
            }

            // level-0 beam from (cur, cd)
            if (lane == 0) {
                S.cand_n = 0;
                S.res_n = 0;
                S.res_worst = WORST0;
                S.abandon = 0;
                min_push(cand, S.cand_n, Entry{cd, cur});
                // MaxHeap.push: the worst first, then the entry
                if (cd > S.res_worst) S.res_worst = cd;
                max_sift_up(res, S.res_n++, Entry{cd, cur});
                atomicOr(vis + (cur >> 5), 1u << (cur & 31));
            }
            __syncwarp();
        }  // from the caller's heaps or from the greedy's node
        for (int64_t step = 0; step <= n; ++step) {
            uint32_t cid = 0;
            int go = 0;
            if (lane == 0 && S.cand_n > 0) {
                const Entry c = min_pop(cand, S.cand_n);
                go = !(c.d > S.res_worst && S.res_n >= p.ef);
                cid = c.id;
            }
            go = __shfl_sync(FULL, go, 0);
            if (!go) break;
            cid = __shfl_sync(FULL, cid, 0);
            ++expansions;
            // the row, its slots and the count in one round trip (a row holds 33 words)
            const uint32_t* row = p.l0_compact + (size_t)cid * 33;
            const uint32_t cnt = __ldg(row);
            const uint32_t rn = __ldg(row + 1 + lane);
            const uint32_t rs = __ldg(p.l0_slots + (size_t)cid * 33 + 1 + lane);
            uint32_t nidx = 0xffffffffu;
            bool ok = false;
            if ((uint32_t)lane < cnt) {
                nidx = rn;
                if (nidx < (uint64_t)n) {
                    const uint32_t vw = __ldcg(vis + (nidx >> 5));
                    ok = !is_deleted(p.deleted, nidx) && !((vw >> (nidx & 31)) & 1u);
                }
            }
            // a node listed twice counts at its first position only
            const unsigned same =
                __match_any_sync(FULL, ok ? nidx : (0x80000000u | (unsigned)lane));
            ok = ok && (__ffs(same) - 1 == lane);
            const unsigned keep = __ballot_sync(FULL, ok);
            if (ok) {
                atomicOr(vis + (nidx >> 5), 1u << (nidx & 31));
                // the new neighbours are the likely next candidates: their rows towards L2
                prefetch_l2(p.l0_compact + (size_t)nidx * 33);
                prefetch_l2(p.l0_slots + (size_t)nidx * 33);
                const int at = __popc(keep & ((1u << lane) - 1u));
                S.ni[at] = nidx;
                S.ns[at] = rs != 0xffffffffu ? rs : __ldg(p.node_slot + nidx);
            }
            __syncwarp();
            score_batch(p, S, __popc(keep), true, lane);
            evals += __popc(keep) * (lane == 0);
            if (lane == 0) {
                const int m = __popc(keep);
                for (int j = 0; j < m; ++j) {
                    const Entry e{S.nd[j], S.ni[j]};
                    if (!min_push(cand, S.cand_n, e)) {
                        S.abandon = 1;
                        break;
                    }
                    max_push_bounded(res, S.res_n, S.res_worst, e, p.ef);
                }
            }
            __syncwarp();
            if (S.abandon) break;
        }
        if (p.from_heaps) {  // the heaps back to the caller
            const int cn = S.cand_n, rn = S.res_n;
            if (lane == 0) {
                p.heap_meta[3] = S.abandon ? -1 : cn;
                p.heap_meta[4] = rn;
                p.heap_meta[5] = __float_as_int(S.res_worst);
            }
            const int64_t co = cn < p.cand_io_cap ? cn : p.cand_io_cap;
            for (int64_t i = lane; i < co; i += 32) p.cand_io[i] = cand.get(i);
            for (int i = lane; i < rn; i += 32) p.res_io[i] = res[i];
            __syncwarp();
            continue;
        }
        if (S.abandon) {
            if (lane == 0) {
                if (p.stats) atomicAdd(p.stats + 2, 1ull);
                if (p.overflow) {
                    p.overflow[atomicAdd(p.overflow_n, 1)] = t;
                } else {
                    record_error(p.status, PION_B200_ESHAPE);
                }
            }
            __syncwarp();
            continue;
        }

        // drain farthest first into ascending arrays, rerank, stable sort, first k
        float* ds = reinterpret_cast<float*>(top);
        uint32_t* ids = reinterpret_cast<uint32_t*>(top) + TOP;
        const int m = S.res_n;
        __syncwarp();
        if (lane == 0) {
            int rn = S.res_n;
            float rw = S.res_worst;
            for (int i = 0; i < m; ++i) {
                const Entry e = max_pop(res, rn, rw);
                ds[m - 1 - i] = e.d;
                ids[m - 1 - i] = e.id;
            }
        }
        __syncwarp();
        if (p.rerank) {
            const int half = lane >> 4, hl = lane & 15;
            for (int b0 = 0; b0 < m; b0 += 2) {
                const int i = b0 + half;
                if (b0 + 2 + half < m) {  // the next pair's rows towards L2 (48 lines each)
                    const float* nx = p.rerank + (size_t)ids[b0 + 2 + half] * DIM;
                    for (int c = hl; c < DIM / 32; c += 16) prefetch_l2(nx + 32 * c);
                }
                float acc = 0.0f;
                if (i < m) {
                    // a lane's accumulator takes dims hl, hl + 16, ...: 32 loads in flight
                    const float* v = p.rerank + (size_t)ids[i] * DIM;
                    for (int g = 0; g < 3; ++g) {
                        float vv[32];
#pragma unroll
                        for (int u = 0; u < 32; ++u) vv[u] = __ldg(v + 16 * (32 * g + u) + hl);
#pragma unroll
                        for (int u = 0; u < 32; ++u) {
                            const int d = 16 * (32 * g + u) + hl;
                            const float df = __fsub_rn(qv_at(x, S, d), vv[u]);
                            acc = __fadd_rn(acc, __fmul_rn(df, df));
                        }
                    }
                }
                float s8 = __fadd_rn(acc, __shfl_down_sync(FULL, acc, 8, 16));
                float s4 = __fadd_rn(s8, __shfl_down_sync(FULL, s8, 4, 16));
                float s2 = __fadd_rn(s4, __shfl_down_sync(FULL, s4, 2, 16));
                float s1 = __fadd_rn(s2, __shfl_down_sync(FULL, s2, 1, 16));
                __syncwarp();
                if (hl == 0 && i < m) ds[i] = s1;
                __syncwarp();
            }
        }
        const int kk = m < p.k ? m : p.k;
        for (int j = lane; j < m; j += 32) {
            const float dj = ds[j];
            int rank = 0;
            for (int i = 0; i < m; ++i) {
                const float di = ds[i];
                rank += (di < dj || (di == dj && i < j)) ? 1 : 0;
            }
            if (rank < kk) {
                p.out_ids[(size_t)t * p.k + rank] = __ldg(p.node_ids + ids[j]);
                p.out_scores[(size_t)t * p.k + rank] = dj;
            }
        }
        for (int j = kk + lane; j < p.k; j += 32) {
            p.out_ids[(size_t)t * p.k + j] = -1;
            p.out_scores[(size_t)t * p.k + j] = __int_as_float(0x7f800000);
        }
        if (lane == 0) p.out_found[t] = kk;
        __syncwarp();
    }
    if (lane == 0 && p.stats) {
        atomicAdd(p.stats, evals);
        atomicAdd(p.stats + 1, expansions);
    }
}

}  // namespace qb

size_t quant_warp_smem(int ef) { return qb::warp_bytes(ef); }
int quant_warps_per_cta() { return qb::WARPS; }
int quant_top_entries() { return qb::TOP; }

int quant_ctas_per_sm(int ef) {
    const size_t bytes = qb::WARPS * qb::warp_bytes(ef);
    if (bytes > 227 * 1024) return 0;
    if (cudaFuncSetAttribute(qb::quant_search_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)bytes) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    int blocks = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, qb::quant_search_kernel,
                                                      qb::WARPS * 32, bytes) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return blocks;
}

int launch_quant_search(const QuantLaunch& L, cudaStream_t st) {
    qb::Params p{};
    p.kind = L.kind;
    p.metric = L.metric;
    p.codes = L.codes;
    p.code_bytes = L.code_bytes;
    p.scales = L.scales;
    p.norms = L.norms;
    p.qjl = L.qjl;
    p.res_norms = L.res_norms;
    p.rsigns = L.rsigns;
    p.lambda = L.lambda;
    p.rerank = L.rerank;
    p.l0_compact = L.l0_compact;
    p.l0_slots = L.l0_slots;
    p.node_slot = L.node_slot;
    p.node_ids = L.node_ids;
    p.deleted = L.deleted;
    p.node_level = L.node_level;
    p.upper_offset = L.upper_offset;
    p.upper_links = L.upper_links;
    p.upper_slots = L.upper_slots;
    p.M = L.M;
    p.max_level = L.max_level;
    p.num_nodes = L.num_nodes;
    p.entry = L.entry;
    p.queries = L.queries;
    p.nq = L.nq;
    p.k = L.k;
    p.ef = L.ef;
    p.qlist = L.qlist;
    p.qlist_n = L.qlist_n;
    p.visited = L.visited;
    p.vis_words = L.vis_words;
    p.cand_tail = reinterpret_cast<qb::Entry*>(L.cand_tail);
    p.cand_cap = L.cand_cap;
    p.out_ids = L.out_ids;
    p.out_scores = L.out_scores;
    p.out_found = L.out_found;
    p.overflow = L.overflow;
    p.overflow_n = L.overflow_n;
    p.next_query = L.next_query;
    p.stats = L.stats;
    p.status = L.status;
    p.from_heaps = L.from_heaps;
    p.given_codes = L.given_codes;
    p.given_scales = L.given_scales;
    p.given_norms = L.given_norms;
    p.given_signs = L.given_signs;
    p.cand_io = reinterpret_cast<qb::Entry*>(L.cand_io);
    p.cand_io_cap = L.cand_io_cap;
    p.res_io = reinterpret_cast<qb::Entry*>(L.res_io);
    p.heap_meta = L.heap_meta;
    if (L.ctas <= 0 || L.ef < 1 || L.ef > qb::TOP || L.code_bytes % 16 != 0)
        return PION_B200_ESHAPE;
    const size_t bytes = qb::WARPS * qb::warp_bytes(L.ef);
    if (cudaFuncSetAttribute(qb::quant_search_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)bytes) != cudaSuccess)
        return PION_B200_ECUDA;
    qb::quant_search_kernel<<<L.ctas, qb::WARPS * 32, bytes, st>>>(p);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

}  // namespace pion
