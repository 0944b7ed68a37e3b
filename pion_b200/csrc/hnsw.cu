// HNSW INT8 search on sm_100a: one warp per query runs the reference's
// search_fp32_scored at dim 1536 (src/vector/hnsw.mojo:4136-4521) over a graph in the
// compact level-0 layout:
//   1. greedy descent of the upper levels in exact INT8 L2, moving to the nearest
//      strictly closer neighbour of the node the step started at, first one on ties
//      (_upper_greedy_codes, hnsw.mojo:3789-3848);
//   2. the level-0 beam, beam_search_1536_ref (src/vector/reference/beam_1536.mojo:
//      85-135) over a LinearPool of ef entries (src/common/heap.mojo:133-234).
//
// The pool is a sorted (dist, node) array in shared memory.  Expanding a node loads
// its adjacency row in one round trip (the row of the likely next candidate is
// already on its way to L2), gathers its <= 32 unvisited neighbours in adjacency order
// (one per lane), asks L2 for all of their codes at once (one bulk prefetch each),
// then copies them four at a time into shared memory with cp.async and scores them
// with the whole warp: lane l dp4a's chunks l, l+32, l+64 of the neighbour against the
// same chunks of the query held in registers, so every copy is a coalesced 512-byte
// row and a lane reads back only what it copied.  The registered graph keeps its codes
// 16-byte aligned (1536 bytes per slot) with the header norm in a separate array.  The
// lane formulas are the reference's, by position j in the gathered list (batched =
// n - n % 4):
//   fill,  j <  batched: (qn + vnorm) - 2 * f32(dot)
//   fill,  j >= batched: f32(l2)
//   prune, j <  batched: (qn + vnorm) - 2 * (f32(dot[0:256]) + f32(dot[256:1536]))
//   prune, j >= batched: prefix gate f32(l2[0:256]) < worst * 0.175, then the suffix
//                        in 256-dim blocks with an exit once the sum passes `worst`
// where `worst` is the pool's last distance after the batched lanes.  All integer
// sums are exact, so every lane gets the reference's float.
//
// The batched lanes enter the pool in one warp-wide merge that equals inserting them
// one by one with LinearPool.insert (upper-bound position, so equal distances keep
// insertion order; the entry pushed past ef falls off): each candidate's position is
// its rank among the candidates by (dist, j) plus the number of pool entries with
// dist <= its dist, and each pool entry moves down, in place, by the number of
// candidates with a smaller dist.  The <= 3 tail lanes of a prune step then insert
// one at a time.
// Popping takes the first unchecked entry, which is what LinearPool's cursor with its
// CHECKED bit yields.  The pool therefore equals the reference's entry for entry.
//
// The visited set is a bitmap of num_nodes bits per resident warp in global memory,
// all zero between queries.  Each warp appends the index of every word it turns from
// zero to non-zero to its own list (up to touch_cap words) and, when the query ends,
// zeroes just those words: O(nodes visited), not O(num_nodes), per query.  A query
// that visits more words than the list holds zeroes its whole bitmap instead.  Every
// loop is bounded (the beam by the node count); a malformed graph records an error
// status instead of reading out of bounds.
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "internal.h"

namespace pion {
namespace hb {

constexpr int DIM = 1536;
constexpr int NBLK = 6;     // 256-dim blocks
constexpr int CHUNKS = 96;  // 16-byte chunks of a 1536-byte vector
constexpr int WARPS = 4;    // queries (warps) per CTA
constexpr uint32_t CHECKED = 0x80000000u;
constexpr unsigned FULL = 0xffffffffu;

struct Entry {
    float d;
    uint32_t id;
};

struct Params {
    const int8_t* codes;  // [slot][1536], 16-byte aligned
    const float* norms;   // [slot]: f32 |code|^2 (the slot header's first word)
    const uint32_t* l0_compact;
    const uint32_t* l0_slots;
    const uint32_t* node_slot;
    const int32_t* node_ids;
    const uint8_t* deleted;
    const int8_t* node_level;
    const int64_t* upper_offset;
    const uint32_t* upper_links;
    const uint32_t* upper_slots;  // upper_links with each neighbour replaced by its slot
    int M;
    int max_level;
    int64_t num_nodes;
    int64_t entry;
    const int8_t* qcodes;  // nq x DIM
    const int32_t* qblk;   // nq x 8: block norms of the query codes
    int nq, k, ef, efr;
    uint32_t* visited;  // vis_words per resident warp, all zero between queries
    int64_t vis_words;
    uint32_t* touched;  // touch_cap word indices per resident warp
    int touch_cap;
    int32_t* out_ids;
    float* out_dist;
    unsigned long long* stats;  // level-0 evaluations, expansions, upper evaluations
    unsigned* next_query;
    int* status;
    // From-pool mode (pion_v_beam_1536, pion_v_b200_hnsw_beam_batch): the level-0 beam
    // only, per query from the caller's pool (entries with their CHECKED bits, size,
    // cursor; pool_stride entries apart) and query norm, each pool written back in place
    // (cursor = size at the end).
    int from_pool;
    Entry* pool_io;
    int64_t pool_stride;
    const int* pool_size;
    const int* pool_cursor;
    const float* qn_given;
    int* pool_size_out;
};

// Per-warp shared memory: the staging rows of `stage` neighbours (copied per round
// trip), the pool, the merge's candidate positions, the gathered neighbours (slot,
// node, distance, norm), the query's block norms and the block L2s of the <= 3 prune
// tail lanes.
__host__ __device__ constexpr size_t warp_smem(int efr, int stage) {
    return (size_t)stage * DIM + (size_t)efr * sizeof(Entry) + 32 * sizeof(int) +
           4 * 32 * sizeof(uint32_t) + 8 * sizeof(int) + 4 * 8 * sizeof(int);
}

// Neighbours staged per round trip: as many as keep 28 warps (every query of a
// 4096-query batch) resident per SM.
__host__ __device__ constexpr int stage_for(int ef) { return ef <= 128 ? 4 : ef <= 512 ? 2 : 1; }

__device__ __forceinline__ bool is_deleted(const uint8_t* del, uint32_t i) {
    return del && ((del[i >> 3] >> (i & 7)) & 1u);
}

__device__ __forceinline__ int4 ldg4(const int8_t* p) {
    return __ldg(reinterpret_cast<const int4*>(p));
}

__device__ __forceinline__ int dp4a4(const int4& a, const int4& b, int acc) {
    acc = __dp4a(a.x, b.x, acc);
    acc = __dp4a(a.y, b.y, acc);
    acc = __dp4a(a.z, b.z, acc);
    return __dp4a(a.w, b.w, acc);
}

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Sums of one vector against the query, all lanes cooperating: lane l holds chunks l,
// l + 32 and l + 64 (blocks l/16, 2 + l/16, 4 + l/16).  Returns the warp totals of
// q.v and v.v and of q.v over block 0; when `tail` is set, writes the six 256-dim
// block L2s qq[b] + vv[b] - 2 dot[b] to tail[0:6].
struct VecSums {
    int dot, vv, dot0;
};

__device__ __forceinline__ VecSums reduce_sums(const int4 (&v)[3], const int4 (&q)[3], int lane,
                                              const int* qq, int* tail) {
    int d[3], s[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        d[k] = dp4a4(v[k], q[k], 0);
        s[k] = dp4a4(v[k], v[k], 0);
    }
    VecSums r;
    r.dot = d[0] + d[1] + d[2];
    r.vv = s[0] + s[1] + s[2];
    r.dot0 = lane < 16 ? d[0] : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        r.dot += __shfl_xor_sync(FULL, r.dot, o);
        r.vv += __shfl_xor_sync(FULL, r.vv, o);
        r.dot0 += __shfl_xor_sync(FULL, r.dot0, o);
    }
    if (tail) {  // warp-uniform
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) {
#pragma unroll
            for (int k = 0; k < 3; ++k) {
                d[k] += __shfl_xor_sync(FULL, d[k], o);
                s[k] += __shfl_xor_sync(FULL, s[k], o);
            }
        }
        if ((lane & 15) == 0) {
            const int h = lane >> 4;
#pragma unroll
            for (int k = 0; k < 3; ++k) {
                const int b = 2 * k + h;
                tail[b] = qq[b] + s[k] - 2 * d[k];
            }
        }
    }
    return r;
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)),
                 "l"(gsrc)
                 : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Lane's three chunks of slot `slot` into its own places of a staging row.
__device__ __forceinline__ void stage_vec(int4* row, const int8_t* codes, uint32_t slot,
                                          int lane) {
    const int4* src = reinterpret_cast<const int4*>(codes + (size_t)slot * DIM);
#pragma unroll
    for (int k = 0; k < 3; ++k) cp_async16(row + lane + 32 * k, src + lane + 32 * k);
}

__device__ __forceinline__ void read_vec(const int4* row, int lane, int4 (&v)[3]) {
#pragma unroll
    for (int k = 0; k < 3; ++k) v[k] = row[lane + 32 * k];
}

// A visited-bitmap word, read at L2 (the bitmap is only written by atomics, which act at
// L2, so an L1 copy could be stale).
__device__ __forceinline__ uint32_t ld_l2_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.global.cg.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// L2 prefetch of the (at most two) 128-byte lines holding a 132-byte adjacency row;
// both addresses lie inside the row.
__device__ __forceinline__ void prefetch_row_l2(const uint32_t* row) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(row) : "memory");
    asm volatile("prefetch.global.L2 [%0];" ::"l"(row + 32) : "memory");
}

// First index of pool[0:size) whose distance is > d.
__device__ __forceinline__ int upper_bound(const Entry* pool, int size, float d) {
    int lo = 0, hi = size;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (pool[mid].d > d)
            hi = mid;
        else
            lo = mid + 1;
    }
    return lo;
}

template <int STAGE>
__global__ void __launch_bounds__(WARPS * 32, 7) hnsw_beam_kernel(Params p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    unsigned char* base = smem + (size_t)warp * warp_smem(p.efr, STAGE);
    int4* stage = reinterpret_cast<int4*>(base);  // [STAGE][96]
    Entry* pool = reinterpret_cast<Entry*>(base + (size_t)STAGE * DIM);
    int* cub = reinterpret_cast<int*>(pool + p.efr);
    uint32_t* g_slot = reinterpret_cast<uint32_t*>(cub + 32);  // gathered, in j order
    uint32_t* g_node = g_slot + 32;
    float* g_dist = reinterpret_cast<float*>(g_node + 32);
    uint32_t* g_lane = reinterpret_cast<uint32_t*>(g_dist + 32);
    int* qq = reinterpret_cast<int*>(g_lane + 32);  // block norms of the query codes
    int* tail_l2 = qq + 8;                          // [tail lane][block]
    uint32_t* vis = p.visited + ((size_t)blockIdx.x * WARPS + warp) * (size_t)p.vis_words;
    uint32_t* touch = p.touched + ((size_t)blockIdx.x * WARPS + warp) * (size_t)p.touch_cap;
    const uint32_t nn = (uint32_t)p.num_nodes;
    const int ef = p.ef;
    unsigned n_evals = 0, n_expand = 0, n_upper = 0;  // per warp: far below 2^32

    for (;;) {
        unsigned qi = 0;
        if (lane == 0) qi = atomicAdd(p.next_query, 1u);
        qi = __shfl_sync(FULL, qi, 0);
        if (qi >= (unsigned)p.nq) break;

        int4 q[3];
        {
            const int4* qg = reinterpret_cast<const int4*>(p.qcodes + (size_t)qi * DIM);
#pragma unroll
            for (int k = 0; k < 3; ++k) q[k] = qg[lane + 32 * k];
        }
        int32_t qn_int = 0;
        if (p.from_pool) {  // block norms from the caller's codes
            int d[3];
#pragma unroll
            for (int k2 = 0; k2 < 3; ++k2) d[k2] = dp4a4(q[k2], q[k2], 0);
#pragma unroll
            for (int o = 8; o > 0; o >>= 1)
#pragma unroll
                for (int k2 = 0; k2 < 3; ++k2) d[k2] += __shfl_xor_sync(FULL, d[k2], o);
            if ((lane & 15) == 0)
#pragma unroll
                for (int k2 = 0; k2 < 3; ++k2) qq[2 * k2 + (lane >> 4)] = d[k2];
            if (lane == 0) qq[6] = qq[7] = 0;
            __syncwarp();
#pragma unroll
            for (int b = 0; b < NBLK; ++b) qn_int += qq[b];
        } else {
#pragma unroll
            for (int b = 0; b < NBLK; ++b) qn_int += p.qblk[(size_t)qi * 8 + b];
            if (lane < 8) qq[lane] = p.qblk[(size_t)qi * 8 + lane];
        }
        const float qn = p.from_pool ? p.qn_given[qi] : (float)qn_int;
        int n_touch = 0;  // words of `vis` this query turned non-zero (warp-uniform)

        // ---- upper levels: greedy in code space (skipped when starting from a pool)
        uint32_t curr = p.from_pool ? 0u : (uint32_t)p.entry;
        // (a beam started from the caller's pool has no upper levels to read)
        int64_t c_off = p.from_pool ? -1 : p.upper_offset[curr];
        int c_lvl = p.from_pool ? 0 : p.node_level[curr];
        float cd;
        if (!p.from_pool) {
            int4 v[3];
            stage_vec(stage, p.codes, p.node_slot[curr], lane);
            cp_async_wait_all();
            read_vec(stage, lane, v);
            const VecSums r = reduce_sums(v, q, lane, qq, nullptr);
            cd = (float)(qn_int + r.vv - 2 * r.dot);
        } else {
            cd = 0.0f;
        }
        n_upper += 1;
        for (int l = p.from_pool ? 0 : p.max_level; l >= 1; --l) {
            bool changed = true;
            for (int64_t guard = 0; changed && guard <= p.num_nodes; ++guard) {
                changed = false;
                int cnt = 0;
                uint32_t nb = 0xffffffffu, slot = 0;
                if (c_off >= 0 && l <= c_lvl) {
                    const size_t r0 = (size_t)(c_off + l - 1) * (1 + p.M);
                    const uint32_t craw = p.upper_links[r0];
                    if (lane < p.M) {
                        nb = p.upper_links[r0 + 1 + lane];
                        slot = p.upper_slots[r0 + 1 + lane];
                    }
                    cnt = min((int)craw, p.M);
                }
                const bool valid = lane < cnt && nb < nn && !is_deleted(p.deleted, nb);
                const unsigned vm = __ballot_sync(FULL, valid);
                int64_t nb_off = -1;
                int nb_lvl = 0;
                if (valid) {
                    prefetch_l2(p.codes + (size_t)slot * DIM, DIM);
                    nb_off = p.upper_offset[nb];
                    nb_lvl = p.node_level[nb];
                }
                n_upper += __popc(vm);
                // in list order: the first neighbour strictly closer than the best so far
                float best = cd;
                int best_lane = -1;
                for (unsigned m = vm; m;) {
                    int lanes_of[STAGE];
                    int g = 0;
#pragma unroll
                    for (int e = 0; e < STAGE; ++e) {
                        lanes_of[e] = -1;
                        if (m) {
                            const int a = __ffs(m) - 1;
                            m &= m - 1u;
                            lanes_of[e] = a;
                            stage_vec(stage + e * 96, p.codes, __shfl_sync(FULL, slot, a), lane);
                            g = e + 1;
                        }
                    }
                    cp_async_wait_all();
#pragma unroll
                    for (int e = 0; e < STAGE; ++e) {
                        if (e >= g) break;
                        int4 v[3];
                        read_vec(stage + e * 96, lane, v);
                        const VecSums r = reduce_sums(v, q, lane, qq, nullptr);
                        const float d = (float)(qn_int + r.vv - 2 * r.dot);
                        if (d < best) {
                            best = d;
                            best_lane = lanes_of[e];
                        }
                    }
                }
                if (best_lane >= 0) {
                    cd = best;
                    curr = __shfl_sync(FULL, nb, best_lane);
                    c_off = __shfl_sync(FULL, nb_off, best_lane);
                    c_lvl = __shfl_sync(FULL, nb_lvl, best_lane);
                    changed = true;
                }
            }
        }

        // ---- level 0: the beam
        int size = 1, hint = 0;
        if (p.from_pool) {
            // the caller's pool; its nodes are the ones it marked visited
            size = min(p.pool_size[qi], ef);
            hint = min(p.pool_cursor[qi], size);
            for (int i0 = 0; i0 < size; i0 += 32) {
                const int i = i0 + lane;
                bool fresh_word = false;
                uint32_t nd = 0xffffffffu;
                if (i < size) {
                    const Entry e = p.pool_io[(size_t)qi * p.pool_stride + i];
                    pool[i] = e;
                    nd = e.id & ~CHECKED;
                    if (nd < nn) fresh_word = atomicOr(&vis[nd >> 5], 1u << (nd & 31)) == 0u;
                }
                note_words(touch, p.touch_cap, n_touch, __ballot_sync(FULL, fresh_word),
                           nd >> 5, lane);
            }
        } else {
            bool fresh_word = false;
            if (lane == 0) {
                fresh_word = atomicOr(&vis[curr >> 5], 1u << (curr & 31)) == 0u;
                pool[0].d = cd;
                pool[0].id = curr;
            }
            note_words(touch, p.touch_cap, n_touch, __ballot_sync(FULL, fresh_word), curr >> 5,
                       lane);
        }
        // Look-ahead: the row of the entry predicted to be popped next (the second
        // unchecked entry at this pop) and the visited words of its neighbours, read
        // after this step's marks.  Only this warp writes its bitmap, so the words are
        // exact when the prediction holds; otherwise the step loads as usual.
        uint32_t sp_node = 0xffffffffu, sp_cnt = 0, sp_nb = 0xffffffffu, sp_sl = 0xffffffffu;
        uint32_t sp_word = 0;
        __syncwarp();
        for (int64_t step = 0;; ++step) {
            if (step > p.num_nodes) {
                if (lane == 0) record_error(p.status, PION_B200_EINVAL);
                break;
            }
            // pop: the first unchecked entry (and the one after it, prefetched)
            int pos = -1, nxt = -1;
            for (int b0 = hint & ~31; b0 < size && nxt < 0; b0 += 32) {
                const int i = b0 + lane;
                const bool un = i >= hint && i < size && !(pool[i].id & CHECKED);
                unsigned m = __ballot_sync(FULL, un);
                if (m && pos < 0) {
                    pos = b0 + __ffs(m) - 1;
                    m &= m - 1u;
                }
                if (m) nxt = b0 + __ffs(m) - 1;
            }
            if (pos < 0) break;
            const bool fill = size < ef;
            const uint32_t c = pool[pos].id;
            const uint32_t pred = nxt >= 0 ? pool[nxt].id : 0xffffffffu;
            __syncwarp();
            if (lane == 0) pool[pos].id = c | CHECKED;
            hint = pos + 1;
            n_expand += 1;

            // gather: unvisited, undeleted neighbours in adjacency order
            const bool hit = c == sp_node;  // warp-uniform
            uint32_t cnt_raw, nb_raw, sl;
            if (hit) {
                cnt_raw = sp_cnt;
                nb_raw = sp_nb;
                sl = sp_sl;
            } else {  // one round trip: every lane loads its entry and the count together
                const uint32_t* row = p.l0_compact + (size_t)c * 33;
                cnt_raw = row[0];
                nb_raw = row[1 + lane];
                sl = p.l0_slots[(size_t)c * 33 + 1 + lane];
            }
            const int cnt = min((int)cnt_raw, 32);
            const uint32_t nb = lane < cnt ? nb_raw : 0xffffffffu;
            const bool valid = lane < cnt && nb < nn && !is_deleted(p.deleted, nb);
            const unsigned key = valid ? nb : (0x80000000u | (unsigned)lane);
            const unsigned peers = __match_any_sync(FULL, key);
            bool fresh = false;
            bool fresh_word = false;
            if (valid && (__ffs(peers) - 1) == lane) {
                const uint32_t bit = 1u << (nb & 31);
                if (hit) {  // the word was read after every earlier mark of this query
                    fresh = (sp_word & bit) == 0;
                    if (fresh) fresh_word = atomicOr(&vis[nb >> 5], bit) == 0u;
                } else {
                    const uint32_t old = atomicOr(&vis[nb >> 5], bit);
                    fresh = (old & bit) == 0;
                    fresh_word = old == 0u;
                }
                if (fresh && sl >= nn) {
                    record_error(p.status, PION_B200_EINVAL);
                    fresh = false;
                }
            }
            note_words(touch, p.touch_cap, n_touch, __ballot_sync(FULL, fresh_word), nb >> 5,
                       lane);
            // look-ahead row of the predicted next pop, in flight while this step scores
            sp_node = pred;
            if (pred != 0xffffffffu) {
                const uint32_t* prow = p.l0_compact + (size_t)pred * 33;
                sp_cnt = prow[0];
                sp_nb = prow[1 + lane];
                sp_sl = p.l0_slots[(size_t)pred * 33 + 1 + lane];
            }
            const unsigned fm = __ballot_sync(FULL, fresh);
            const int n = __popc(fm);
            if (n == 0) {
                __syncwarp();  // this step's marks before the look-ahead words
                if (sp_node != 0xffffffffu) {
                    const bool sv = (int)lane < min((int)sp_cnt, 32) && sp_nb < nn;
                    sp_word = sv ? ld_l2_u32(&vis[sp_nb >> 5]) : 0xffffffffu;
                }
                continue;
            }
            const int batched = n - (n & 3);
            n_evals += n;
            float my_norm = 0.0f;  // consumed after the staging round trip
            if (fresh) {
                const int j = __popc(fm & ((1u << lane) - 1u));
                g_slot[j] = sl;
                g_node[j] = nb;
                g_lane[j] = (uint32_t)lane;
                my_norm = __ldg(p.norms + sl);
                prefetch_l2(p.codes + (size_t)sl * DIM, DIM);
            }
            __syncwarp();

            // score the gathered neighbours STAGE at a time, in j order
            for (int v0 = 0; v0 < n; v0 += STAGE) {
                const int g = min(STAGE, n - v0);
#pragma unroll
                for (int e = 0; e < STAGE; ++e)
                    if (e < g) stage_vec(stage + e * 96, p.codes, g_slot[v0 + e], lane);
                cp_async_wait_all();
                if (v0 == 0 && sp_node != 0xffffffffu) {
                    // the look-ahead row has arrived by now: its visited words (after this
                    // step's marks, ordered by the syncs above)
                    const bool sv = (int)lane < min((int)sp_cnt, 32) && sp_nb < nn;
                    sp_word = sv ? ld_l2_u32(&vis[sp_nb >> 5]) : 0xffffffffu;
                }
#pragma unroll
                for (int e = 0; e < STAGE; ++e) {
                    if (e >= g) break;
                    const int jj = v0 + e;
                    const bool tail = !fill && jj >= batched;
                    int4 v[3];
                    read_vec(stage + e * 96, lane, v);
                    const VecSums r = reduce_sums(v, q, lane, qq,
                                                  tail ? tail_l2 + (jj - batched) * 8 : nullptr);
                    float d = INFINITY;
                    if (jj < batched) {
                        const float df = fill ? (float)r.dot
                                              : __fadd_rn((float)r.dot0, (float)(r.dot - r.dot0));
                        const float vn = __shfl_sync(FULL, my_norm, (int)g_lane[jj]);
                        d = __fsub_rn(__fadd_rn(qn, vn), __fmul_rn(2.0f, df));
                    } else if (fill) {
                        d = (float)(qn_int + r.vv - 2 * r.dot);
                    }
                    if (lane == 0) g_dist[jj] = d;
                }
                __syncwarp();
            }

            // codes of the look-ahead neighbours that are still unvisited, towards L2
            if (sp_node != 0xffffffffu && (int)lane < min((int)sp_cnt, 32) && sp_nb < nn &&
                sp_sl < nn && (sp_word & (1u << (sp_nb & 31))) == 0)
                prefetch_l2(p.codes + (size_t)sp_sl * DIM, DIM);

            // batched merge (every gathered neighbour while filling): lane j holds
            // candidate j, candidates are lanes [0, ns)
            const int ns = fill ? n : batched;
            const bool in = lane < ns;
            const float d = in ? g_dist[lane] : INFINITY;
            int P = ef;
            if (in) {
                int rank = 0;
                for (int t = 0; t < ns; ++t) {
                    const float dt = g_dist[t];
                    rank += (dt < d || (dt == d && t < lane)) ? 1 : 0;
                }
                const int ub = upper_bound(pool, size, d);
                P = rank + ub;
                cub[rank] = ub;
            }
            int pmin = P;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) pmin = min(pmin, __shfl_xor_sync(FULL, pmin, o));
            if (pmin < ef) {  // something enters the pool
                __syncwarp();
                const int first = cub[0];  // entries before it stay where they are
                for (int top = ((size - 1 - first) & ~31) + first; top >= first; top -= 32) {
                    const int i = top + lane;
                    Entry e;
                    int np = ef;
                    if (i < size) {
                        e = pool[i];
                        int lo = 0, hi = ns;
                        while (lo < hi) {
                            const int mid = (lo + hi) >> 1;
                            if (cub[mid] <= i)
                                lo = mid + 1;
                            else
                                hi = mid;
                        }
                        np = i + lo;
                    }
                    __syncwarp();
                    if (np < ef) pool[np] = e;
                    __syncwarp();
                }
                if (in && P < ef) {
                    pool[P].d = d;
                    pool[P].id = g_node[lane];
                }
                hint = min(hint, pmin);
            }
            size = min(ef, size + ns);
            __syncwarp();

            // prune tail neighbours, one at a time in j order
            if (!fill) {
                const float wst = pool[size - 1].d;
                for (int jj = batched; jj < n; ++jj) {
                    const uint32_t id = g_node[jj];
                    const int* l2b = tail_l2 + (jj - batched) * 8;
                    const float dp = (float)l2b[0];
                    if (!(dp < __fmul_rn(wst, 0.175f))) continue;
                    float running = dp;
                    bool exited = false;
                    for (int b = 1; b < NBLK; ++b) {
                        running = __fadd_rn(running, (float)l2b[b]);
                        if (running > wst) {
                            exited = true;
                            break;
                        }
                    }
                    if (exited || !(running < wst)) continue;
                    // LinearPool.insert
                    if (size == ef && !(running < pool[size - 1].d)) continue;
                    const int lo = upper_bound(pool, size, running);
                    const int end = size == ef ? size - 1 : size;
                    for (int top = ((end - 1 - lo) & ~31) + lo; top >= lo; top -= 32) {
                        const int i = top + lane;
                        Entry e;
                        const bool mv = i < end;
                        if (mv) e = pool[i];
                        __syncwarp();
                        if (mv) pool[i + 1] = e;
                        __syncwarp();
                    }
                    if (lane == 0) {
                        pool[lo].d = running;
                        pool[lo].id = id;
                    }
                    size = min(size + 1, ef);
                    hint = min(hint, lo);
                    __syncwarp();
                }
            }
        }

        // back to an all-zero bitmap: the listed words, or every word if the list overflowed
        __syncwarp();
        if (n_touch <= p.touch_cap) {
            for (int i = lane; i < n_touch; i += 32) vis[touch[i]] = 0u;
        } else {
            int4* v4 = reinterpret_cast<int4*>(vis);
            const int64_t n4 = p.vis_words / 4;
            for (int64_t w = lane; w < n4; w += 32) v4[w] = make_int4(0, 0, 0, 0);
        }
        if (p.from_pool) {  // the whole pool back to the caller
            for (int i = lane; i < size; i += 32) p.pool_io[(size_t)qi * p.pool_stride + i] = pool[i];
            if (lane == 0) p.pool_size_out[qi] = size;
        }
        // drain: the first k entries, nearest first
        for (int i = lane; i < p.k; i += 32) {
            const size_t o = (size_t)qi * p.k + i;
            if (i < size) {
                const uint32_t id = pool[i].id & ~CHECKED;
                p.out_ids[o] = p.node_ids[id];
                p.out_dist[o] = pool[i].d;
            } else {
                p.out_ids[o] = -1;
                p.out_dist[o] = INFINITY;
            }
        }
        __syncwarp();
    }
    if (lane == 0) {
        atomicAdd(p.stats + 0, (unsigned long long)n_evals);
        atomicAdd(p.stats + 1, (unsigned long long)n_expand);
        atomicAdd(p.stats + 2, (unsigned long long)n_upper);
    }
}

// metric_scores (src/vector/hnsw.mojo:4523-4651) with INT8 codes: the reply score of a
// result node is the squared L2 between the query (normalised once under COSINE, then
// clamped to the calibration range) and the codes dequantised at the middle of their step,
// x = c * (range / 254) + (127.5 * range / 254 + gmin), summed as the reference does: 32
// chains (4 x 8 SIMD lanes; lane L takes elements 32 i + L in order, mul then add), lanes
// combined (c0 + c1) + (c2 + c3), then the 8-lane SIMD reduction tree; COSINE halves it.
// One warp per (query, result); ids without a node keep their score.
__global__ void hnsw_metric_kernel(const float* __restrict__ qn, int nq, int k,
                                   const int32_t* __restrict__ ids,
                                   const int32_t* __restrict__ ext_to_node, int64_t ext_base,
                                   int64_t ext_count, const uint32_t* __restrict__ node_slot,
                                   const int8_t* __restrict__ codes, float gmin, float gmax,
                                   int cosine, const float* __restrict__ rows,
                                   float* __restrict__ scores) {
    const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (w >= (int64_t)nq * k) return;  // warp-uniform
    const int64_t ext = ids[w];
    if (ext < ext_base || ext - ext_base >= ext_count) return;
    const int32_t node = ext_to_node[ext - ext_base];
    if (node < 0) return;
    float range = __fsub_rn(gmax, gmin);
    if (range <= 0.0f) range = 1.0f;
    const float a = __fdiv_rn(range, 254.0f);
    const float b = __fadd_rn(__fmul_rn(127.5f, a), gmin);
    const float* q = qn + (w / k) * DIM;
    float acc = 0.0f;
    if (rows) {  // the FP32 copy by node: the unclamped query against the row
        const float* v = rows + (size_t)node * DIM;
#pragma unroll 4
        for (int i = 0; i < DIM / 32; ++i) {
            const int d = 32 * i + lane;
            const float t = __fsub_rn(q[d], v[d]);
            acc = __fadd_rn(__fmul_rn(t, t), acc);
        }
    } else {
        const int8_t* c = codes + (size_t)node_slot[node] * DIM;
#pragma unroll 4
        for (int i = 0; i < DIM / 32; ++i) {
            const int d = 32 * i + lane;
            const float qv = fminf(fmaxf(q[d], gmin), gmax);
            const float x = __fadd_rn(__fmul_rn((float)c[d], a), b);
            const float t = __fsub_rn(qv, x);
            acc = __fadd_rn(__fmul_rn(t, t), acc);
        }
    }
    const int l = lane & 7;
    const float c0 = __shfl_sync(FULL, acc, l), c1 = __shfl_sync(FULL, acc, 8 + l);
    const float c2 = __shfl_sync(FULL, acc, 16 + l), c3 = __shfl_sync(FULL, acc, 24 + l);
    float v = __fadd_rn(__fadd_rn(c0, c1), __fadd_rn(c2, c3));  // lane l of the SIMD8 sum
#pragma unroll
    for (int h = 4; h > 0; h >>= 1) v = __fadd_rn(v, __shfl_sync(FULL, v, (l + h) & 7));
    if (lane == 0) scores[w] = cosine ? __fmul_rn(v, 0.5f) : v;
}

// Device copy of a slot buffer: codes at 16-byte aligned rows of 1536 bytes and the
// header's norm^2 in its own array.
__global__ void hnsw_relayout_kernel(const int8_t* __restrict__ src, int64_t n, int64_t stride,
                                     int64_t hdr, int8_t* __restrict__ codes,
                                     float* __restrict__ norms) {
    const int64_t total = n * (DIM / 8);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t s = i / (DIM / 8), c = i % (DIM / 8);
        const int8_t* row = src + s * stride;
        *reinterpret_cast<int2*>(codes + s * DIM + 8 * c) =
            *reinterpret_cast<const int2*>(row + hdr + 8 * c);
        if (c == 0) norms[s] = *reinterpret_cast<const float*>(row);
    }
}

// Query codes (quantize_fp32_to_int8_simd, src/vector/kernels.mojo:52-99):
// clamp(roundeven((x - gmin) * scale), 0, 254) - 127, and the six 256-dim block norms
// of the codes.  One CTA of 192 threads per query, 8 dims per thread.
__global__ void __launch_bounds__(192) hnsw_quantize_kernel(const float* __restrict__ q, int nq,
                                                            float gmin, float scale,
                                                            int8_t* __restrict__ codes,
                                                            int32_t* __restrict__ blk) {
    const int qi = blockIdx.x;
    const int t = threadIdx.x;
    const float* x = q + (size_t)qi * DIM + 8 * t;
    uint32_t w[2] = {0u, 0u};
    int s = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        int r = __float2int_rn(__fmul_rn(__fsub_rn(x[e], gmin), scale));
        r = min(max(r, 0), 254) - 127;
        s += r * r;
        w[e >> 2] |= ((uint32_t)(r & 0xff)) << (8 * (e & 3));
    }
    *reinterpret_cast<uint2*>(codes + (size_t)qi * DIM + 8 * t) = make_uint2(w[0], w[1]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(FULL, s, o);
    if ((t & 31) == 0) blk[(size_t)qi * 8 + (t >> 5)] = s;
    if (t < 2) blk[(size_t)qi * 8 + 6 + t] = 0;
}

}  // namespace hb

int hnsw_dim() { return hb::DIM; }
int hnsw_warps_per_cta() { return hb::WARPS; }
size_t hnsw_warp_smem(int ef) { return hb::warp_smem((ef + 31) / 32 * 32, hb::stage_for(ef)); }

int launch_hnsw_quantize(const float* q, int nq, float gmin, float scale, int8_t* codes,
                         int32_t* blk, cudaStream_t st) {
    if (nq <= 0) return 0;
    hb::hnsw_quantize_kernel<<<nq, 192, 0, st>>>(q, nq, gmin, scale, codes, blk);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

template <int STAGE>
static int beam_ctas_per_sm(size_t smem) {
    if (set_smem_limit((const void*)hb::hnsw_beam_kernel<STAGE>, 227 * 1024) != 0) return 0;
    int blocks = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, hb::hnsw_beam_kernel<STAGE>,
                                                      hb::WARPS * 32, smem) != cudaSuccess)
        return 0;
    return blocks;
}

// Resident CTAs of the beam kernel for this ef (0 if it does not fit).
int hnsw_ctas_per_sm(int ef) {
    const size_t smem = (size_t)hb::WARPS * hnsw_warp_smem(ef);
    if (smem > 227 * 1024) return 0;
    switch (hb::stage_for(ef)) {
        case 4: return beam_ctas_per_sm<4>(smem);
        case 2: return beam_ctas_per_sm<2>(smem);
        default: return beam_ctas_per_sm<1>(smem);
    }
}

int launch_hnsw_metric(const float* qn, int nq, int k, const int32_t* ids,
                       const int32_t* ext_to_node, int64_t ext_base, int64_t ext_count,
                       const uint32_t* node_slot, const int8_t* codes, float gmin, float gmax,
                       int cosine, const float* rows, float* scores, cudaStream_t st) {
    const int64_t warps = (int64_t)nq * k;
    if (warps <= 0) return 0;
    hb::hnsw_metric_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(
        qn, nq, k, ids, ext_to_node, ext_base, ext_count, node_slot, codes, gmin, gmax, cosine,
        rows, scores);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int launch_hnsw_relayout(const int8_t* src, int64_t n, int64_t stride, int64_t hdr,
                         int8_t* codes, float* norms, cudaStream_t st) {
    if (n <= 0) return 0;
    hb::hnsw_relayout_kernel<<<1184, 256, 0, st>>>(src, n, stride, hdr, codes, norms);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int launch_hnsw_beam(const HnswLaunch& L, cudaStream_t st) {
    hb::Params p;
    p.codes = L.codes;
    p.norms = L.norms;
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
    p.qcodes = L.qcodes;
    p.qblk = L.qblk;
    p.nq = L.nq;
    p.k = L.k;
    p.ef = L.ef;
    p.efr = (L.ef + 31) / 32 * 32;
    p.visited = L.visited;
    p.vis_words = L.vis_words;
    p.touched = L.touched;
    p.touch_cap = L.touch_cap;
    if (!p.touched || p.touch_cap < 32) return PION_B200_EINVAL;
    p.out_ids = L.out_ids;
    p.out_dist = L.out_dist;
    p.stats = L.stats;
    p.next_query = L.next_query;
    p.status = L.status;
    p.from_pool = L.pool_io != nullptr;
    p.pool_io = reinterpret_cast<hb::Entry*>(L.pool_io);
    p.pool_stride = L.pool_stride;
    p.pool_size = L.pool_size;
    p.pool_cursor = L.pool_cursor;
    p.qn_given = L.qn_given;
    p.pool_size_out = L.pool_size_out;
    const size_t smem = (size_t)hb::WARPS * hnsw_warp_smem(L.ef);
    switch (hb::stage_for(L.ef)) {
        case 4: hb::hnsw_beam_kernel<4><<<L.ctas, hb::WARPS * 32, smem, st>>>(p); break;
        case 2: hb::hnsw_beam_kernel<2><<<L.ctas, hb::WARPS * 32, smem, st>>>(p); break;
        default: hb::hnsw_beam_kernel<1><<<L.ctas, hb::WARPS * 32, smem, st>>>(p); break;
    }
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

}  // namespace pion
