// The search half of batched HNSW insertion on the GPU: for every node of a batch,
// against the graph as it stood before the batch, the greedy descent of the levels above
// the node's, _search_layer_mt at efConstruction on each level it joins, and
// _prune_neighbors -- exactly what Builder::plan (hnsw_build.cpp) computes on the host,
// so the build links the same neighbours and the graph is the same array for array
// (src/vector/hnsw.mojo:2032-2064 _search_layer_mt, :2117-2240 _insert_to_graph_mt,
// :3595-3628 _prune_neighbors).
//
// One warp per batch node (a persistent grid taking nodes from a counter):
//   greedy      dist_f32_i8 of the builder: 16 FMA chains over 16-element steps
//               (element 16 s + e in chain e), t[e] = c[e] + c[e + 8], then
//               ((t0 + t1) + (t2 + t3)) + ((t4 + t5) + (t6 + t7)); a lane per neighbour,
//               the first strict minimum of the list moves the walk, as the host's
//               running comparison does;
//   search      exact INT8 L2 = |q|^2 + |c|^2 - 2 q.c (a lane per neighbour, dp4a),
//               neighbours in list order (a repeated id counts once, at its first
//               position), the candidate min-heap and the bounded result max-heap with
//               the host's sift rules (ties resolve alike), lane 0 pushing in order;
//   prune       nearest first, a candidate kept unless some kept r is closer to it than
//               the node (a lane per kept r), then the discarded ones in order.
// The visited set is a bitmap per resident warp, all zero between searches: the words a
// search turned non-zero are listed and zeroed when it ends (all words if the list
// overflows).  The candidate heap keeps its first TOP entries in shared memory and the
// rest in a per-warp global tail; a heap that outgrows it records PION_B200_ESHAPE and the
// host plans that batch itself.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <new>
#include <thread>
#include <vector>

#include "common.cuh"
#include "hnsw_host.h"
#include "internal.h"

namespace pion {
namespace bp {

constexpr int DIM = 1536;
constexpr int WARPS = 4;
constexpr int TOP = 1024;  // candidate-heap entries in shared memory; also `all`
constexpr int MAXL = 7;    // levels 0..6
constexpr unsigned FULL = 0xffffffffu;
constexpr int TOUCH_CAP = 16384;

struct Entry {
    float d;
    uint32_t id;
};

struct Params {
    const int8_t* codes;   // [n][1536], node order
    const int32_t* cnorm;  // [n] |code|^2
    const int8_t* level;   // [n]
    const uint32_t* links;
    const uint32_t* cnt;
    const int64_t* link_base;
    const int64_t* cnt_base;
    int64_t n;
    int M, efc, max_level;
    int64_t entry;
    float scale, offset;
    const int64_t* ids;  // the batch
    const float* rows;   // [bsz][1536]: the rows the nodes are linked with
    int bsz;
    uint32_t* visited;  // [warps][vis_words], all zero between searches
    int64_t vis_words;
    uint32_t* touched;  // [warps][TOUCH_CAP]
    Entry* cand_tail;   // [warps][cand_cap - TOP]
    int64_t cand_cap;
    int32_t* out_top;  // [bsz]
    int32_t* out_n;    // [bsz][MAXL]
    uint32_t* out_id;  // [bsz][MAXL][32]
    float* out_d;      // [bsz][MAXL][32]
    unsigned* next;
    int* status;
};

struct Fixed {
    int32_t qw[DIM / 4];
    float nd[32];
    uint32_t ni[32];
    int cand_n, res_n, pruned_n, disc_n;
    uint32_t pruned[32];
    float pruned_d[32];
};

__host__ __device__ constexpr size_t fixed_bytes() { return (sizeof(Fixed) + 15) / 16 * 16; }
__host__ __device__ constexpr size_t warp_bytes(int efc) {
    return fixed_bytes() + (size_t)TOP * sizeof(Entry) +
           ((size_t)efc * sizeof(Entry) + 15) / 16 * 16;
}

__device__ __forceinline__ int dot_query(const int32_t* qw, const int8_t* c) {
    const int4* cw = reinterpret_cast<const int4*>(c);
    int a = 0;
#pragma unroll 8
    for (int j = 0; j < DIM / 16; ++j) {
        const int4 v = __ldg(cw + j);
        a = __dp4a(v.x, qw[4 * j], a);
        a = __dp4a(v.y, qw[4 * j + 1], a);
        a = __dp4a(v.z, qw[4 * j + 2], a);
        a = __dp4a(v.w, qw[4 * j + 3], a);
    }
    return a;
}

__device__ __forceinline__ int dot_pair(const int8_t* a8, const int8_t* b8) {
    const int4* aw = reinterpret_cast<const int4*>(a8);
    const int4* bw = reinterpret_cast<const int4*>(b8);
    int a = 0;
#pragma unroll 8
    for (int j = 0; j < DIM / 16; ++j) {
        const int4 u = __ldg(aw + j), v = __ldg(bw + j);
        a = __dp4a(u.x, v.x, a);
        a = __dp4a(u.y, v.y, a);
        a = __dp4a(u.z, v.z, a);
        a = __dp4a(u.w, v.w, a);
    }
    return a;
}

// The builder's dist_f32_i8 (fp32 row vs dequantised code), one lane.
__device__ float dist_f32_i8(const float* v, const int8_t* c, float scale, float offset) {
    float acc[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) acc[e] = 0.0f;
    for (int s = 0; s < DIM / 16; ++s) {
        const int4 cw = __ldg(reinterpret_cast<const int4*>(c) + s);
        const int8_t* cb = reinterpret_cast<const int8_t*>(&cw);
        const float4* vp = reinterpret_cast<const float4*>(v + 16 * s);
#pragma unroll
        for (int f = 0; f < 4; ++f) {
            const float4 x = __ldg(vp + f);
            const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                const int e = 4 * f + g;
                const float dq = __fmaf_rn((float)cb[e], scale, offset);
                const float d = __fsub_rn(xs[g], dq);
                acc[e] = __fmaf_rn(d, d, acc[e]);
            }
        }
    }
    float t[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) t[e] = __fadd_rn(acc[e], acc[e + 8]);
    return __fadd_rn(__fadd_rn(__fadd_rn(t[0], t[1]), __fadd_rn(t[2], t[3])),
                     __fadd_rn(__fadd_rn(t[4], t[5]), __fadd_rn(t[6], t[7])));
}

// ---------------------------------------------------------------- heaps --
// The host builder's MinHeap (candidates) and MaxHeap (results), operation for operation.
struct Cand {
    Entry* top;
    Entry* tail;
    int64_t cap;
    __device__ Entry get(int64_t i) const { return i < TOP ? top[i] : tail[i - TOP]; }
    __device__ void put(int64_t i, Entry e) const {
        if (i < TOP)
            top[i] = e;
        else
            tail[i - TOP] = e;
    }
};

// push: sift up while the parent is strictly farther
__device__ bool min_push(const Cand& h, int& n, Entry e) {
    if (n >= h.cap) return false;
    int64_t c = n++;
    while (c > 0) {
        const int64_t p = (c - 1) / 2;
        const Entry pe = h.get(p);
        if (pe.d <= e.d) break;
        h.put(c, pe);
        c = p;
    }
    h.put(c, e);
    return true;
}

// pop: the last entry to the root, sifted down towards the nearer child (left first)
__device__ Entry min_pop(const Cand& h, int& n) {
    const Entry root = h.get(0);
    --n;
    if (n > 0) {
        const Entry x = h.get(n);
        int64_t c = 0;
        for (;;) {
            const int64_t l = 2 * c + 1, r = l + 1;
            int64_t s = c;
            Entry se = x;
            if (l < n) {
                const Entry le = h.get(l);
                if (le.d < se.d) {
                    s = l;
                    se = le;
                }
            }
            if (r < n) {
                const Entry re = h.get(r);
                if (re.d < se.d) {
                    s = r;
                    se = re;
                }
            }
            if (s == c) break;
            h.put(c, se);
            c = s;
        }
        h.put(c, x);
    }
    return root;
}

__device__ void max_up(Entry* a, int c, Entry e) {
    while (c > 0) {
        const int p = (c - 1) / 2;
        if (a[p].d >= e.d) break;
        a[c] = a[p];
        c = p;
    }
    a[c] = e;
}

__device__ void max_down(Entry* a, int n, Entry x) {
    int c = 0;
    for (;;) {
        const int l = 2 * c + 1, r = l + 1;
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

__device__ bool push_bounded(Entry* a, int& n, Entry e, int ef) {
    if (n < ef) {
        max_up(a, n++, e);
        return true;
    }
    if (e.d < a[0].d) {
        max_down(a, n, e);
        return true;
    }
    return false;
}

__device__ Entry max_pop(Entry* a, int& n) {
    const Entry root = a[0];
    --n;
    if (n > 0) max_down(a, n, a[n]);
    return root;
}

__device__ __forceinline__ uint32_t cnt_of(const Params& p, uint32_t i, int l) {
    return __ldg(p.cnt + p.cnt_base[i] + l);
}
__device__ __forceinline__ const uint32_t* list_of(const Params& p, uint32_t i, int l) {
    return p.links + p.link_base[i] + (l == 0 ? 0 : 2 * p.M + (int64_t)(l - 1) * p.M);
}

__global__ void __launch_bounds__(WARPS * 32) plan_kernel(Params p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    unsigned char* base = smem + (size_t)warp * warp_bytes(p.efc);
    Fixed& S = *reinterpret_cast<Fixed*>(base);
    Entry* top = reinterpret_cast<Entry*>(base + fixed_bytes());
    Entry* res = top + TOP;
    const int64_t gw = (int64_t)blockIdx.x * WARPS + warp;
    uint32_t* vis = p.visited + gw * p.vis_words;
    uint32_t* touch = p.touched + gw * TOUCH_CAP;
    const Cand cand{top, p.cand_tail + gw * (p.cand_cap > TOP ? p.cand_cap - TOP : 0),
                    p.cand_cap};
    const int64_t n = p.n;
    for (;;) {
        unsigned item = 0;
        if (lane == 0) item = atomicAdd(p.next, 1u);
        item = __shfl_sync(FULL, item, 0);
        if (item >= (unsigned)p.bsz) break;
        const uint32_t id = (uint32_t)p.ids[item];
        const int lvl = p.level[id];
        const float* v = p.rows + (size_t)item * DIM;
        const int8_t* q = p.codes + (size_t)id * DIM;
        for (int w = lane; w < DIM / 4; w += 32) S.qw[w] = reinterpret_cast<const int32_t*>(q)[w];
        const int32_t qn = p.cnorm[id];
        __syncwarp();

        // ---- greedy descent of the levels above the node's
        uint32_t ep = (uint32_t)p.entry;
        for (int l = p.max_level; l > lvl; --l) {
            float best = 0.0f;
            if (lane == 0) best = dist_f32_i8(v, p.codes + (size_t)ep * DIM, p.scale, p.offset);
            best = __shfl_sync(FULL, best, 0);
            for (int64_t pass = 0; pass <= n; ++pass) {
                const uint32_t cur = ep;
                if (l > p.level[cur]) break;
                const uint32_t nc = cnt_of(p, cur, l);
                const uint32_t* lst = list_of(p, cur, l);
                uint32_t nb = 0xffffffffu;
                if ((uint32_t)lane < nc && lane < p.M) nb = lst[lane];
                const bool ok = nb < (uint64_t)n;
                float d = 0.0f;
                if (ok) d = dist_f32_i8(v, p.codes + (size_t)nb * DIM, p.scale, p.offset);
                float m = ok ? d : __int_as_float(0x7f800000);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) m = fminf(m, __shfl_xor_sync(FULL, m, o));
                const unsigned at = __ballot_sync(FULL, ok && d == m);
                if (!(m < best)) break;
                best = m;
                ep = __shfl_sync(FULL, nb, __ffs(at) - 1);
            }
        }

        // ---- search_layer + prune on every level the node joins, top down
        const int topl = lvl < p.max_level ? lvl : p.max_level;
        if (lane == 0) p.out_top[item] = topl;
        for (int l = topl, k = 0; l >= 0; --l, ++k) {
            int n_touch = 0;  // warp-uniform
            {
                bool fresh_word = false;
                if (lane == 0) {
                    const float d0 = (float)(qn + p.cnorm[ep] -
                                             2 * dot_query(S.qw, p.codes + (size_t)ep * DIM));
                    S.cand_n = 0;
                    S.res_n = 0;
                    min_push(cand, S.cand_n, Entry{d0, ep});
                    max_up(res, S.res_n++, Entry{d0, ep});
                    fresh_word = atomicOr(vis + (ep >> 5), 1u << (ep & 31)) == 0u;
                }
                note_words(touch, TOUCH_CAP, n_touch, __ballot_sync(FULL, fresh_word), ep >> 5,
                           lane);
            }
            __syncwarp();
            for (int64_t step = 0; step <= n; ++step) {
                uint32_t cid = 0;
                int go = 0;
                if (lane == 0 && S.cand_n > 0) {
                    const Entry c = min_pop(cand, S.cand_n);
                    go = !(c.d > res[0].d && S.res_n >= p.efc);
                    cid = c.id;
                }
                go = __shfl_sync(FULL, go, 0);
                if (!go) break;
                cid = __shfl_sync(FULL, cid, 0);
                if (l > p.level[cid]) continue;
                const uint32_t nc = cnt_of(p, cid, l);
                const uint32_t* lst = list_of(p, cid, l);
                uint32_t nb = 0xffffffffu;
                bool ok = false;
                if ((uint32_t)lane < nc && lane < (l == 0 ? 2 * p.M : p.M)) {
                    nb = lst[lane];
                    ok = nb < (uint64_t)n && ((__ldcg(vis + (nb >> 5)) >> (nb & 31)) & 1u) == 0u;
                }
                const unsigned same =
                    __match_any_sync(FULL, ok ? nb : (0x80000000u | (unsigned)lane));
                ok = ok && (__ffs(same) - 1 == lane);
                const unsigned keep = __ballot_sync(FULL, ok);
                bool fresh_word = false;
                if (ok) {
                    fresh_word = atomicOr(vis + (nb >> 5), 1u << (nb & 31)) == 0u;
                    const int at = __popc(keep & ((1u << lane) - 1u));
                    S.ni[at] = nb;
                    S.nd[at] = (float)(qn + p.cnorm[nb] -
                                       2 * dot_query(S.qw, p.codes + (size_t)nb * DIM));
                }
                note_words(touch, TOUCH_CAP, n_touch, __ballot_sync(FULL, fresh_word), nb >> 5,
                           lane);
                __syncwarp();
                if (lane == 0) {
                    const int m = __popc(keep);
                    for (int j = 0; j < m; ++j) {
                        const Entry e{S.nd[j], S.ni[j]};
                        if (push_bounded(res, S.res_n, e, p.efc) && !min_push(cand, S.cand_n, e))
                            record_error(p.status, PION_B200_ESHAPE);
                    }
                }
                __syncwarp();
            }
            // the bitmap back to all zero
            __syncwarp();
            if (n_touch <= TOUCH_CAP) {
                for (int i = lane; i < n_touch; i += 32) vis[touch[i]] = 0u;
            } else {
                for (int64_t w = lane; w < p.vis_words; w += 32) vis[w] = 0u;
            }
            // results farthest first into `all` (the dead candidate heap's shared memory)
            Entry* all = top;
            int na = 0;
            if (lane == 0) {
                int rn = S.res_n;
                while (rn > 0) all[na++] = max_pop(res, rn);
                S.pruned_n = 0;
                S.disc_n = 0;
            }
            na = __shfl_sync(FULL, na, 0);
            __syncwarp();
            if (na > 0) ep = all[na - 1].id;
            const int m_limit = l == 0 ? 2 * p.M : p.M;
            Entry* disc = res;  // the dead result heap's shared memory
            for (int i = na - 1; i >= 0; --i) {
                const int pn = S.pruned_n;
                if (pn >= m_limit) break;
                const Entry c = all[i];
                bool bad = false;
                if (lane < pn) {
                    const uint32_t r = S.pruned[lane];
                    const int32_t dcr = p.cnorm[c.id] + p.cnorm[r] -
                                        2 * dot_pair(p.codes + (size_t)c.id * DIM,
                                                     p.codes + (size_t)r * DIM);
                    bad = (float)dcr < c.d;
                }
                const bool good = __ballot_sync(FULL, bad) == 0;
                __syncwarp();
                if (lane == 0) {
                    if (good) {
                        S.pruned[S.pruned_n] = c.id;
                        S.pruned_d[S.pruned_n++] = c.d;
                    } else {
                        disc[S.disc_n++] = c;
                    }
                }
                __syncwarp();
            }
            if (lane == 0) {
                for (int i = 0; S.pruned_n < m_limit && i < S.disc_n; ++i) {
                    S.pruned[S.pruned_n] = disc[i].id;
                    S.pruned_d[S.pruned_n++] = disc[i].d;
                }
                p.out_n[(size_t)item * MAXL + k] = S.pruned_n;
            }
            __syncwarp();
            for (int j = lane; j < S.pruned_n; j += 32) {
                p.out_id[((size_t)item * MAXL + k) * 32 + j] = S.pruned[j];
                p.out_d[((size_t)item * MAXL + k) * 32 + j] = S.pruned_d[j];
            }
            __syncwarp();
        }
    }
}

__global__ void code_norms_kernel(const int8_t* __restrict__ codes, int64_t n,
                                  int32_t* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (i >= n) return;
    const int lane = threadIdx.x & 31;
    const int4* c = reinterpret_cast<const int4*>(codes + i * DIM);
    int a = 0;
    for (int j = lane; j < DIM / 16; j += 32) {
        const int4 v = c[j];
        a = __dp4a(v.x, v.x, a);
        a = __dp4a(v.y, v.y, a);
        a = __dp4a(v.z, v.z, a);
        a = __dp4a(v.w, v.w, a);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(FULL, a, o);
    if (lane == 0) out[i] = a;
}

// Node blocks (packed on the host, src_off[j] words into `src`) to their places.
__global__ void scatter_blocks_kernel(const uint32_t* __restrict__ src,
                                      const int64_t* __restrict__ src_off,
                                      const int64_t* __restrict__ dst_off,
                                      const int32_t* __restrict__ len, int64_t count,
                                      uint32_t* __restrict__ dst) {
    const int64_t j = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (j >= count) return;
    const int lane = threadIdx.x & 31;
    for (int w = lane; w < len[j]; w += 32) dst[dst_off[j] + w] = src[src_off[j] + w];
}

}  // namespace bp

namespace {

template <typename T>
int dev_alloc(T** p, size_t count) {
    *p = nullptr;
    if (count == 0) count = 1;
    if (cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T)) != cudaSuccess) {
        cudaGetLastError();
        return PION_B200_ENOMEM;
    }
    return 0;
}

// BatchPlanner on one context's GPU.
class GpuPlanner : public hnsw::BatchPlanner {
  public:
    explicit GpuPlanner(pion_b200_ctx* ctx) : ctx_(ctx) {}
    ~GpuPlanner() override {
        cudaSetDevice(ctx_->device);
        cudaStreamSynchronize(ctx_->stream);
        void* ps[] = {codes_, cnorm_, level_, links_, cnt_, link_base_, cnt_base_, ids_, rows_,
                      visited_, touched_, cand_tail_, out_top_, out_n_, out_id_, out_d_, next_,
                      up_src_, up_src_off_, up_dst_off_, up_len_};
        for (void* p : ps)
            if (p) cudaFree(p);
    }

    int begin(const hnsw::Graph& g, const int8_t* codes, const int64_t* link_base,
              const int64_t* cnt_base, int64_t n_links, int64_t n_counts, float scale,
              float offset, int64_t max_batch) override {
        if (g.dim != bp::DIM || g.M < 2 || 2 * g.M > 32 || g.efc < 1 || g.efc > bp::TOP ||
            g.max_level >= bp::MAXL || max_batch < 1)
            return PION_B200_ESHAPE;
        if (use_device(ctx_) != 0) return PION_B200_ENODEV;
        n_ = g.n;
        M_ = (int)g.M;
        efc_ = (int)g.efc;
        max_level_ = g.max_level;
        entry_ = g.entry;
        scale_ = scale;
        offset_ = offset;
        max_batch_ = max_batch;
        level_host_ = g.level.data();
        link_base_host_ = link_base;
        cnt_base_host_ = cnt_base;
        const int per_sm = ctas_per_sm();
        if (per_sm <= 0) return PION_B200_ESHAPE;
        int64_t ctas = (int64_t)per_sm * ctx_->num_sms;
        const int64_t need = (max_batch + bp::WARPS - 1) / bp::WARPS;
        ctas_ = ctas < need ? ctas : need;
        const int64_t warps = ctas_ * bp::WARPS;
        vis_words_ = ((n_ + 31) / 32 + 3) / 4 * 4;
        cand_cap_ = n_ + 1 < 16384 ? n_ + 1 : 16384;
        cudaStream_t st = ctx_->stream;
        if (dev_alloc(&codes_, (size_t)n_ * bp::DIM) || dev_alloc(&cnorm_, (size_t)n_) ||
            dev_alloc(&level_, (size_t)n_) || dev_alloc(&links_, (size_t)n_links) ||
            dev_alloc(&cnt_, (size_t)n_counts) || dev_alloc(&link_base_, (size_t)n_) ||
            dev_alloc(&cnt_base_, (size_t)n_) || dev_alloc(&ids_, (size_t)max_batch) ||
            dev_alloc(&rows_, (size_t)max_batch * bp::DIM) ||
            dev_alloc(&visited_, (size_t)(warps * vis_words_)) ||
            dev_alloc(&touched_, (size_t)(warps * bp::TOUCH_CAP)) ||
            dev_alloc(&cand_tail_, (size_t)(warps * (cand_cap_ > bp::TOP ? cand_cap_ - bp::TOP : 1))) ||
            dev_alloc(&out_top_, (size_t)max_batch) ||
            dev_alloc(&out_n_, (size_t)max_batch * bp::MAXL) ||
            dev_alloc(&out_id_, (size_t)max_batch * bp::MAXL * 32) ||
            dev_alloc(&out_d_, (size_t)max_batch * bp::MAXL * 32) || dev_alloc(&next_, 1))
            return PION_B200_ENOMEM;
        if (cudaMemcpyAsync(codes_, codes, (size_t)n_ * bp::DIM, cudaMemcpyHostToDevice, st) ||
            cudaMemcpyAsync(level_, g.level.data(), (size_t)n_, cudaMemcpyHostToDevice, st) ||
            cudaMemcpyAsync(link_base_, link_base, (size_t)n_ * 8, cudaMemcpyHostToDevice, st) ||
            cudaMemcpyAsync(cnt_base_, cnt_base, (size_t)n_ * 8, cudaMemcpyHostToDevice, st) ||
            cudaMemsetAsync(links_, 0xff, (size_t)n_links * 4, st) ||
            cudaMemsetAsync(cnt_, 0, (size_t)n_counts * 4, st) ||
            cudaMemsetAsync(visited_, 0, (size_t)(warps * vis_words_) * 4, st))
            return PION_B200_ECUDA;
        bp::code_norms_kernel<<<(unsigned)((n_ + 7) / 8), 256, 0, st>>>(codes_, n_, cnorm_);
        if (cudaGetLastError() != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess)
            return PION_B200_ECUDA;
        return 0;
    }

    int update(const int64_t* nodes, int64_t count, const uint32_t* links,
               const uint32_t* counts) override {
        if (count == 0) return 0;
        if (use_device(ctx_) != 0) return PION_B200_ENODEV;
        // pack the nodes' link blocks and count blocks, then scatter them on the device
        std::vector<uint32_t> src;
        std::vector<int64_t> soff, doff;
        std::vector<int32_t> len;
        soff.reserve((size_t)count * 2);
        for (int pass = 0; pass < 2; ++pass)
            for (int64_t j = 0; j < count; ++j) {
                const int64_t i = nodes[j];
                const int lv = level_host_[i];
                const int64_t at = pass == 0 ? link_base_host_[i] : cnt_base_host_[i];
                const int32_t ln = pass == 0 ? 2 * M_ + lv * M_ : 1 + lv;
                soff.push_back((int64_t)src.size());
                doff.push_back(at);
                len.push_back(ln);
                const uint32_t* from = (pass == 0 ? links : counts) + at;
                src.insert(src.end(), from, from + ln);
            }
        if (grow(&up_src_, up_src_cap_, src.size()) || grow(&up_src_off_, up_off_cap_, soff.size()) ||
            grow(&up_dst_off_, up_doff_cap_, doff.size()) || grow(&up_len_, up_len_cap_, len.size()))
            return PION_B200_ENOMEM;
        cudaStream_t st = ctx_->stream;
        if (cudaMemcpyAsync(up_src_, src.data(), src.size() * 4, cudaMemcpyHostToDevice, st) ||
            cudaMemcpyAsync(up_src_off_, soff.data(), soff.size() * 8, cudaMemcpyHostToDevice, st) ||
            cudaMemcpyAsync(up_dst_off_, doff.data(), doff.size() * 8, cudaMemcpyHostToDevice, st) ||
            cudaMemcpyAsync(up_len_, len.data(), len.size() * 4, cudaMemcpyHostToDevice, st))
            return PION_B200_ECUDA;
        const unsigned blocks = (unsigned)((count + 7) / 8);
        bp::scatter_blocks_kernel<<<blocks, 256, 0, st>>>(up_src_, up_src_off_, up_dst_off_, up_len_,
                                                          count, links_);
        bp::scatter_blocks_kernel<<<blocks, 256, 0, st>>>(up_src_, up_src_off_ + count,
                                                          up_dst_off_ + count, up_len_ + count,
                                                          count, cnt_);
        if (cudaGetLastError() != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess)
            return PION_B200_ECUDA;
        return 0;
    }

    int plan(const int64_t* ids, int64_t count, const float* rows,
             std::vector<hnsw::BuildPlan>& out) override {
        if (count <= 0 || count > max_batch_) return PION_B200_ESHAPE;
        if (use_device(ctx_) != 0) return PION_B200_ENODEV;
        cudaStream_t st = ctx_->stream;
        int* status = call_status(ctx_, PION_B200_MEM_HOST);
        if (cudaMemcpyAsync(ids_, ids, (size_t)count * 8, cudaMemcpyHostToDevice, st) ||
            cudaMemcpyAsync(rows_, rows, (size_t)count * bp::DIM * 4, cudaMemcpyHostToDevice, st) ||
            cudaMemsetAsync(next_, 0, 4, st))
            return PION_B200_ECUDA;
        bp::Params p;
        p.codes = codes_;
        p.cnorm = cnorm_;
        p.level = level_;
        p.links = links_;
        p.cnt = cnt_;
        p.link_base = link_base_;
        p.cnt_base = cnt_base_;
        p.n = n_;
        p.M = M_;
        p.efc = efc_;
        p.max_level = max_level_;
        p.entry = entry_;
        p.scale = scale_;
        p.offset = offset_;
        p.ids = ids_;
        p.rows = rows_;
        p.bsz = (int)count;
        p.visited = visited_;
        p.vis_words = vis_words_;
        p.touched = touched_;
        p.cand_tail = cand_tail_;
        p.cand_cap = cand_cap_;
        p.out_top = out_top_;
        p.out_n = out_n_;
        p.out_id = out_id_;
        p.out_d = out_d_;
        p.next = next_;
        p.status = status;
        const size_t smem = bp::WARPS * bp::warp_bytes(efc_);
        int64_t ctas = (count + bp::WARPS - 1) / bp::WARPS;
        if (ctas > ctas_) ctas = ctas_;
        bp::plan_kernel<<<(unsigned)ctas, bp::WARPS * 32, smem, st>>>(p);
        ctx_->launches++;
        if (cudaGetLastError() != cudaSuccess) return PION_B200_ECUDA;
        top_h_.resize((size_t)count);
        n_h_.resize((size_t)count * bp::MAXL);
        id_h_.resize((size_t)count * bp::MAXL * 32);
        d_h_.resize((size_t)count * bp::MAXL * 32);
        if (cudaMemcpyAsync(top_h_.data(), out_top_, (size_t)count * 4, cudaMemcpyDeviceToHost, st) ||
            cudaMemcpyAsync(n_h_.data(), out_n_, n_h_.size() * 4, cudaMemcpyDeviceToHost, st) ||
            cudaMemcpyAsync(id_h_.data(), out_id_, id_h_.size() * 4, cudaMemcpyDeviceToHost, st) ||
            cudaMemcpyAsync(d_h_.data(), out_d_, d_h_.size() * 4, cudaMemcpyDeviceToHost, st))
            return PION_B200_ECUDA;
        if (finish_sync(ctx_) != 0) return PION_B200_ECUDA;  // includes an outgrown heap
        if ((int64_t)out.size() < count) out.resize((size_t)count);
        for (int64_t j = 0; j < count; ++j) {
            hnsw::BuildPlan& pl = out[(size_t)j];
            pl.top = top_h_[(size_t)j];
            pl.ids.clear();
            pl.d.clear();
            pl.offs.assign(1, 0);
            for (int k = 0; k <= pl.top; ++k) {
                const int m = n_h_[(size_t)j * bp::MAXL + k];
                const size_t at = ((size_t)j * bp::MAXL + k) * 32;
                pl.ids.insert(pl.ids.end(), id_h_.begin() + at, id_h_.begin() + at + m);
                pl.d.insert(pl.d.end(), d_h_.begin() + at, d_h_.begin() + at + m);
                pl.offs.push_back((uint32_t)pl.ids.size());
            }
        }
        return 0;
    }

  private:
    int ctas_per_sm() const {
        const size_t smem = bp::WARPS * bp::warp_bytes(efc_);
        if (smem > 227 * 1024) return 0;
        if (set_smem_limit((const void*)bp::plan_kernel, (int)smem) != 0) return 0;
        int blocks = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, bp::plan_kernel,
                                                          bp::WARPS * 32, smem) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        return blocks;
    }

    template <typename T>
    static int grow(T** p, size_t& cap, size_t want) {
        if (want <= cap) return 0;
        if (*p) cudaFree(*p);
        *p = nullptr;
        cap = 0;
        const size_t c = want + want / 2 + 64;
        if (dev_alloc(p, c)) return PION_B200_ENOMEM;
        cap = c;
        return 0;
    }

    pion_b200_ctx* ctx_;
    int64_t n_ = 0, entry_ = 0, max_batch_ = 0, ctas_ = 0, vis_words_ = 0, cand_cap_ = 0;
    int M_ = 0, efc_ = 0, max_level_ = 0;
    float scale_ = 0.f, offset_ = 0.f;
    const int8_t* level_host_ = nullptr;
    const int64_t* link_base_host_ = nullptr;
    const int64_t* cnt_base_host_ = nullptr;
    int8_t* codes_ = nullptr;
    int32_t* cnorm_ = nullptr;
    int8_t* level_ = nullptr;
    uint32_t* links_ = nullptr;
    uint32_t* cnt_ = nullptr;
    int64_t* link_base_ = nullptr;
    int64_t* cnt_base_ = nullptr;
    int64_t* ids_ = nullptr;
    float* rows_ = nullptr;
    uint32_t* visited_ = nullptr;
    uint32_t* touched_ = nullptr;
    bp::Entry* cand_tail_ = nullptr;
    int32_t* out_top_ = nullptr;
    int32_t* out_n_ = nullptr;
    uint32_t* out_id_ = nullptr;
    float* out_d_ = nullptr;
    unsigned* next_ = nullptr;
    uint32_t* up_src_ = nullptr;
    int64_t* up_src_off_ = nullptr;
    int64_t* up_dst_off_ = nullptr;
    int32_t* up_len_ = nullptr;
    size_t up_src_cap_ = 0, up_off_cap_ = 0, up_doff_cap_ = 0, up_len_cap_ = 0;
    std::vector<int32_t> top_h_, n_h_;
    std::vector<uint32_t> id_h_;
    std::vector<float> d_h_;
};

}  // namespace
}  // namespace pion

using namespace pion;

extern "C" int pion_v_b200_hnsw_build_gpu(pion_b200_ctx* ctx, const float* rows, int64_t n_rows,
                                          int64_t dim, int64_t M, int64_t ef_construction,
                                          int metric, int64_t id_base, int n_threads,
                                          int64_t max_batch, pion_b200_hnsw_graph** out_graph) {
    if (!out_graph) return PION_B200_EINVAL;
    *out_graph = nullptr;
    if (!valid_ctx(ctx)) return PION_B200_EINVAL;
    if (max_batch < 1 || n_rows < 0 || (n_rows > 0 && !rows) || dim != bp::DIM || M < 2 ||
        M > 16 || ef_construction < 1 || ef_construction > bp::TOP ||
        (metric != 0 && metric != 1) || id_base < 0 || n_rows + id_base > INT32_MAX)
        return set_error(ctx, PION_B200_EINVAL, "hnsw_build_gpu: bad arguments");
    __builtin_cpu_init();
    if (!__builtin_cpu_supports("avx2") || !__builtin_cpu_supports("fma"))
        return set_error(ctx, PION_B200_ESHAPE, "hnsw_build_gpu needs a CPU with AVX2 and FMA");
    if (n_threads <= 0) n_threads = (int)std::thread::hardware_concurrency();
    if (n_threads <= 0) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    pion_b200_hnsw_graph* g = new (std::nothrow) pion_b200_hnsw_graph();
    if (!g) return PION_B200_ENOMEM;
    try {
        GpuPlanner planner(ctx);
        hnsw::build(rows, n_rows, dim, M, ef_construction, metric, id_base, n_threads, g->g,
                    &g->stats, max_batch, &planner);
    } catch (const std::bad_alloc&) {
        delete g;
        return set_error(ctx, PION_B200_ENOMEM, "hnsw_build_gpu: out of host memory");
    }
    *out_graph = g;
    return 0;
}
