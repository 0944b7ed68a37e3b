// HNSW INT8 graph builder on the host, in the reference's layout.
//
// Restates the reference's FT.OPTIMIZE build (src/vector/hnsw.mojo):
//   _calibrate (:578-612)           one global SQ8 range, mean +- 8 sigma (Welford)
//   quantize (:614-655)             stored code = trunc(clamp((x-gmin)/range,0,1)*254) - 127
//   _level_of (:563-576)            SplitMix64 level, ml = 1/ln(M), capped at 6
//   build_index_from_shared (:2540-2620)
//                                   serial pre-pass (levels, codes, entry = first node of
//                                   the highest level), parallel link lanes over strided
//                                   node subsets (src/main.mojo:1951-1974), relink of
//                                   under-linked nodes, _repair_l0, compact_vectors
//   _insert_to_graph_mt (:2117-2240) greedy descent in fp32-vs-code L2, _search_layer_mt
//                                   at efConstruction, _prune_neighbors, links under
//                                   per-node spinlocks with evict-farthest backlinks
//   _prune_neighbors (:3595-3628)    the heuristic keep / discarded refill
//   _relink_node_l0 (:2242-2300), _repair_l0 (:2345-2536)
//   compact_vectors (:2788-2990), _build_l0_slots (:2761-2786)
//                                   BFS slot order, 8-byte header (f32 |code|^2, f32
//                                   |code[0:256]|^2), stride rounded to 64 bytes,
//                                   l0_compact / l0_slots rows of 33 u32
//
// Like the reference's, the parallel link phase is not deterministic (lanes race on
// neighbour lists; bidirectionality is best effort).  One lane builds the same graph
// every time.  The calibration accumulates in double precision where the reference
// keeps float32 SIMD lanes, so the range can differ from the reference's in its last
// bits.
//
// This file is compiled with AVX2 + FMA; pion_v_b200_hnsw_build checks the CPU before
// calling in.

#include <immintrin.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <memory>
#include <thread>
#include <vector>

#include "hnsw_host.h"

namespace pion {
namespace hnsw {

namespace {

constexpr uint64_t kLevelSeed = 0x50494F4Eull;  // HNSW_LEVEL_SEED, hnsw.mojo:80
constexpr int kLevelCap = 6;
constexpr int64_t kCalibrationSampleMax = 65536;  // CALIBRATION_SAMPLE_MAX, hnsw.mojo:70

struct HeapNode {
    float d;
    uint32_t id;
};

// Candidate min-heap.
struct MinHeap {
    std::vector<HeapNode> a;
    void clear() { a.clear(); }
    bool empty() const { return a.empty(); }
    void push(HeapNode x) {
        a.push_back(x);
        size_t i = a.size() - 1;
        while (i > 0) {
            size_t p = (i - 1) >> 1;
            if (a[p].d <= a[i].d) break;
            std::swap(a[p], a[i]);
            i = p;
        }
    }
    HeapNode pop() {
        HeapNode top = a[0];
        a[0] = a.back();
        a.pop_back();
        size_t n = a.size(), i = 0;
        for (;;) {
            size_t l = 2 * i + 1, r = l + 1, s = i;
            if (l < n && a[l].d < a[s].d) s = l;
            if (r < n && a[r].d < a[s].d) s = r;
            if (s == i) break;
            std::swap(a[i], a[s]);
            i = s;
        }
        return top;
    }
};

// Result max-heap with the reference's push_bounded (src/common/heap.mojo:269-288).
struct MaxHeap {
    std::vector<HeapNode> a;
    void clear() { a.clear(); }
    size_t size() const { return a.size(); }
    float peek() const { return a[0].d; }
    void up(size_t i) {
        while (i > 0) {
            size_t p = (i - 1) >> 1;
            if (a[p].d >= a[i].d) break;
            std::swap(a[p], a[i]);
            i = p;
        }
    }
    void down(size_t i) {
        size_t n = a.size();
        for (;;) {
            size_t l = 2 * i + 1, r = l + 1, s = i;
            if (l < n && a[l].d > a[s].d) s = l;
            if (r < n && a[r].d > a[s].d) s = r;
            if (s == i) break;
            std::swap(a[i], a[s]);
            i = s;
        }
    }
    void push(HeapNode x) {
        a.push_back(x);
        up(a.size() - 1);
    }
    bool push_bounded(float d, uint32_t id, size_t ef) {
        if (a.size() < ef) {
            push({d, id});
            return true;
        }
        if (d < a[0].d) {
            a[0] = {d, id};
            down(0);
            return true;
        }
        return false;
    }
    HeapNode pop() {
        HeapNode top = a[0];
        a[0] = a.back();
        a.pop_back();
        if (!a.empty()) down(0);
        return top;
    }
};

// Exact squared L2 between two INT8 code vectors (the integer every reference
// kernel for it returns, e.g. l2_int8_sabd_udot, src/vector/kernels.mojo:510).
inline int32_t l2_i8(const int8_t* a, const int8_t* b, int64_t dim) {
    __m256i acc = _mm256_setzero_si256();
    int64_t i = 0;
    for (; i + 32 <= dim; i += 32) {
        const __m256i va = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(a + i));
        const __m256i vb = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(b + i));
        const __m256i d0 = _mm256_sub_epi16(_mm256_cvtepi8_epi16(_mm256_castsi256_si128(va)),
                                            _mm256_cvtepi8_epi16(_mm256_castsi256_si128(vb)));
        const __m256i d1 = _mm256_sub_epi16(_mm256_cvtepi8_epi16(_mm256_extracti128_si256(va, 1)),
                                            _mm256_cvtepi8_epi16(_mm256_extracti128_si256(vb, 1)));
        acc = _mm256_add_epi32(acc, _mm256_madd_epi16(d0, d0));
        acc = _mm256_add_epi32(acc, _mm256_madd_epi16(d1, d1));
    }
    __m128i s = _mm_add_epi32(_mm256_castsi256_si128(acc), _mm256_extracti128_si256(acc, 1));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4e));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xb1));
    int32_t r = _mm_cvtsi128_si32(s);
    for (; i < dim; ++i) {
        const int32_t d = (int32_t)a[i] - (int32_t)b[i];
        r += d * d;
    }
    return r;
}

inline float dist_i8(const int8_t* a, const int8_t* b, int64_t dim) {
    return (float)l2_i8(a, b, dim);
}

// L2 between an fp32 vector and a dequantised code, dequant = q*scale + offset with
// scale = range/254, offset = 127*scale + gmin (l2_distance_fp32_int8_fused_jit,
// src/vector/kernels.mojo:766-796).  Used only by the build's greedy descent.
inline float dist_f32_i8(const float* v, const int8_t* c, int64_t dim, float scale, float offset) {
    const __m256 vs = _mm256_set1_ps(scale), vo = _mm256_set1_ps(offset);
    __m256 acc0 = _mm256_setzero_ps(), acc1 = _mm256_setzero_ps();
    int64_t i = 0;
    for (; i + 16 <= dim; i += 16) {
        const __m128i c16 = _mm_loadu_si128(reinterpret_cast<const __m128i*>(c + i));
        const __m256 q0 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(c16));
        const __m256 q1 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_srli_si128(c16, 8)));
        const __m256 d0 = _mm256_sub_ps(_mm256_loadu_ps(v + i), _mm256_fmadd_ps(q0, vs, vo));
        const __m256 d1 = _mm256_sub_ps(_mm256_loadu_ps(v + i + 8), _mm256_fmadd_ps(q1, vs, vo));
        acc0 = _mm256_fmadd_ps(d0, d0, acc0);
        acc1 = _mm256_fmadd_ps(d1, d1, acc1);
    }
    alignas(32) float t[8];
    _mm256_store_ps(t, _mm256_add_ps(acc0, acc1));
    float r = ((t[0] + t[1]) + (t[2] + t[3])) + ((t[4] + t[5]) + (t[6] + t[7]));
    for (; i < dim; ++i) {
        const float d = v[i] - std::fma((float)c[i], scale, offset);
        r += d * d;
    }
    return r;
}

// l2_normalize_fp32 (src/vector/kernels.mojo:318-357): inv = 1/sqrt(sum x^2) with the
// sum in four lanes combined (s0+s2)+(s1+s3); a zero vector passes through.
void normalize_row(const float* x, int64_t dim, float* y) {
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    const int64_t main_end = dim & ~int64_t(3);
    for (int64_t d = 0; d < main_end; ++d) s[d & 3] += x[d] * x[d];
    float ns = (s[0] + s[2]) + (s[1] + s[3]);
    for (int64_t d = main_end; d < dim; ++d) ns += x[d] * x[d];
    if (ns <= 0.0f) {
        std::memcpy(y, x, (size_t)dim * sizeof(float));
        return;
    }
    const float inv = 1.0f / std::sqrt(ns);
    for (int64_t d = 0; d < dim; ++d) y[d] = x[d] * inv;
}

struct Builder {
    Graph& g;
    const float* rows;
    float scale = 0.f, offset = 0.f;  // dequantisation of the greedy descent
    std::unique_ptr<std::atomic<uint32_t>[]> cnt;
    std::unique_ptr<std::atomic<uint8_t>[]> locks;
    std::vector<int64_t> link_base, cnt_base;
    std::vector<uint32_t> links;
    // the distance of every list entry to the list's node (dist_i8, exact), kept beside
    // it so the evict-farthest choice reads it instead of recomputing the whole list
    std::vector<float> link_d;
    std::atomic<uint64_t> link_drops{0};

    Builder(Graph& graph, const float* r) : g(graph), rows(r) {}

    int64_t cap(int l) const { return l == 0 ? 2 * g.M : g.M; }
    int64_t list_at(int64_t i, int l) const {
        return link_base[i] + (l == 0 ? 0 : 2 * g.M + (int64_t)(l - 1) * g.M);
    }
    uint32_t* list(int64_t i, int l) { return links.data() + list_at(i, l); }
    float* dlist(int64_t i, int l) { return link_d.data() + list_at(i, l); }
    std::atomic<uint32_t>& count(int64_t i, int l) { return cnt[cnt_base[i] + l]; }
    const int8_t* code(int64_t i) const { return g.codes.data() + i * g.dim; }
    void lock(int64_t i) {
        while (locks[i].exchange(1, std::memory_order_acquire)) _mm_pause();
    }
    void unlock(int64_t i) { locks[i].store(0, std::memory_order_release); }

    // The fp32 row the build links node i with (normalised under COSINE).
    const float* row(int64_t i, std::vector<float>& buf) const {
        const float* x = rows + i * g.dim;
        if (g.metric != 1) return x;
        normalize_row(x, g.dim, buf.data());
        return buf.data();
    }

    struct Scratch {
        std::vector<uint16_t> visited;
        uint16_t epoch = 0;
        MinHeap cand;
        MaxHeap res;
        std::vector<float> fbuf;
        std::vector<HeapNode> all;
        std::vector<uint32_t> pruned, discarded;
        std::vector<float> pruned_d, discarded_d;  // their distances to the query
    };

    void init_scratch(Scratch& s) {
        s.visited.assign((size_t)g.n, 0);
        s.epoch = 0;
        s.fbuf.resize((size_t)g.dim);
    }

    // _search_layer_mt (hnsw.mojo:2032-2064): results of the ef-bounded search at
    // `level` from `ep` in s.res.
    void search_layer(const int8_t* q, int64_t ep, int64_t ef, int level, Scratch& s) {
        if (++s.epoch == 0) {
            std::fill(s.visited.begin(), s.visited.end(), 0);
            s.epoch = 1;
        }
        s.cand.clear();
        s.res.clear();
        const float d0 = dist_i8(q, code(ep), g.dim);
        s.cand.push({d0, (uint32_t)ep});
        s.res.push({d0, (uint32_t)ep});
        s.visited[ep] = s.epoch;
        while (!s.cand.empty()) {
            const HeapNode c = s.cand.pop();
            if (c.d > s.res.peek() && (int64_t)s.res.size() >= ef) break;
            if (level > g.level[c.id]) continue;
            const uint32_t nc = count(c.id, level).load(std::memory_order_acquire);
            const uint32_t* lst = list(c.id, level);
            // the codes of the unvisited neighbours towards the cache before the first
            // distance (the first lines of each; the rest follow as it streams)
            for (uint32_t i = 0; i < nc; ++i) {
                const uint32_t nb = lst[i];
                if (nb >= (uint32_t)g.n || s.visited[nb] == s.epoch) continue;
                const char* p = reinterpret_cast<const char*>(code(nb));
                _mm_prefetch(p, _MM_HINT_T0);
                _mm_prefetch(p + 64, _MM_HINT_T0);
                _mm_prefetch(p + 128, _MM_HINT_T0);
                _mm_prefetch(p + 192, _MM_HINT_T0);
            }
            for (uint32_t i = 0; i < nc; ++i) {
                const uint32_t nb = lst[i];
                if (nb >= (uint32_t)g.n) continue;
                if (s.visited[nb] == s.epoch) continue;
                s.visited[nb] = s.epoch;
                const float d = dist_i8(q, code(nb), g.dim);
                if (s.res.push_bounded(d, nb, (size_t)ef)) s.cand.push({d, nb});
            }
        }
    }

    // _prune_neighbors (hnsw.mojo:3595-3628): `all` is farthest-first.
    void prune(const std::vector<HeapNode>& all, int64_t m_limit, Scratch& s) {
        s.pruned.clear();
        s.discarded.clear();
        s.pruned_d.clear();
        s.discarded_d.clear();
        for (int64_t i = (int64_t)all.size() - 1; i >= 0; --i) {
            if ((int64_t)s.pruned.size() >= m_limit) break;
            const HeapNode c = all[i];
            bool good = true;
            for (uint32_t r : s.pruned) {
                if (dist_i8(code(c.id), code(r), g.dim) < c.d) {
                    good = false;
                    break;
                }
            }
            (good ? s.pruned : s.discarded).push_back(c.id);
            (good ? s.pruned_d : s.discarded_d).push_back(c.d);
        }
        for (size_t i = 0; (int64_t)s.pruned.size() < m_limit && i < s.discarded.size(); ++i) {
            s.pruned.push_back(s.discarded[i]);
            s.pruned_d.push_back(s.discarded_d[i]);
        }
    }

    // Position and distance of the farthest entry of node i's list at `level`
    // (first maximum; an out-of-range id counts as infinitely far).
    int64_t farthest(int64_t i, int level, uint32_t nc, float& worst) {
        const uint32_t* lst = list(i, level);
        const float* dl = dlist(i, level);
        int64_t pos = 0;
        worst = -1.0f;
        for (uint32_t k = 0; k < nc; ++k) {
            const uint32_t e = lst[k];
            if (e >= (uint32_t)g.n) {
                worst = 1e30f;
                return k;
            }
            const float d = dl[k];
            if (worst < 0.0f || d > worst) {
                worst = d;
                pos = k;
            }
        }
        return pos;
    }

    // Appends nb (at distance d from node i) to i's list when it has room.
    void add_published(int64_t i, int level, uint32_t nb, float d) {
        if (level > g.level[i]) return;
        const uint32_t c = count(i, level).load(std::memory_order_relaxed);
        if ((int64_t)c < cap(level)) {
            list(i, level)[c] = nb;
            dlist(i, level)[c] = d;
            count(i, level).store(c + 1, std::memory_order_release);
        }
    }

    void set_entry(int64_t i, int level, int64_t pos, uint32_t nb, float d) {
        list(i, level)[pos] = nb;
        dlist(i, level)[pos] = d;
    }

    // Swap-remove `target` from node i's list at `level`.
    void remove_link(int64_t i, int level, uint32_t target) {
        if (level > g.level[i]) return;
        uint32_t* lst = list(i, level);
        float* dl = dlist(i, level);
        const uint32_t c = count(i, level).load(std::memory_order_relaxed);
        for (uint32_t k = 0; k < c; ++k) {
            if (lst[k] == target) {
                lst[k] = lst[c - 1];
                dl[k] = dl[c - 1];
                count(i, level).store(c - 1, std::memory_order_release);
                return;
            }
        }
    }

    // The search half of an insertion, against the graph as it stands (read only): the
    // greedy descent, search_layer and prune of every level the node joins, the pruned
    // neighbours kept per level (level l's at [offs[l'], offs[l' + 1]) with l' counted
    // from the top).  link() applies them as insert() would; plan() then link() of one
    // node is insert() (a level's links never change a lower level's search).
    using Plan = BuildPlan;
    std::vector<int64_t>* dirty = nullptr;  // nodes whose lists link() changed

    void plan(int64_t id, Scratch& s, Plan& p) {
        const int lvl = g.level[id];
        const int8_t* q = code(id);
        const float* v = row(id, s.fbuf);
        int64_t ep = g.entry;
        p.ids.clear();
        p.d.clear();
        p.offs.assign(1, 0);
        for (int l = g.max_level; l > lvl; --l) {
            float best = dist_f32_i8(v, code(ep), g.dim, scale, offset);
            bool changed = true;
            while (changed) {
                changed = false;
                const int64_t cur = ep;
                if (l > g.level[cur]) break;
                const uint32_t nc = count(cur, l).load(std::memory_order_acquire);
                const uint32_t* lst = list(cur, l);
                for (uint32_t i = 0; i < nc; ++i) {
                    const uint32_t nb = lst[i];
                    if (nb >= (uint32_t)g.n) continue;
                    const float d = dist_f32_i8(v, code(nb), g.dim, scale, offset);
                    if (d < best) {
                        best = d;
                        ep = nb;
                        changed = true;
                    }
                }
            }
        }
        p.top = std::min(lvl, g.max_level);
        for (int l = p.top; l >= 0; --l) {
            search_layer(q, ep, g.efc, l, s);
            if (s.res.size() > 0) {
                s.all.clear();
                while (s.res.size() > 0) s.all.push_back(s.res.pop());
                ep = s.all.back().id;
                prune(s.all, cap(l), s);
                p.ids.insert(p.ids.end(), s.pruned.begin(), s.pruned.end());
                p.d.insert(p.d.end(), s.pruned_d.begin(), s.pruned_d.end());
            }
            p.offs.push_back((uint32_t)p.ids.size());
        }
    }

    // The link half: the node's own lists and the evict-farthest backlinks, level by level
    // from the top, in the order insert() makes them (one thread).
    void link(int64_t id, const Plan& p) {
        const int8_t* q = code(id);
        if (dirty) dirty->push_back(id);
        for (int l = p.top, k = 0; l >= 0; --l, ++k) {
            const int64_t m_limit = cap(l);
            for (uint32_t j = p.offs[k]; j < p.offs[k + 1]; ++j) {
                const uint32_t nb = p.ids[j];
                const float dnb = p.d[j];  // dist_i8(q, code(nb)), as the search found it
                int64_t evicted = -1;
                const uint32_t nc = count(nb, l).load(std::memory_order_relaxed);
                if ((int64_t)nc < m_limit) {
                    add_published(nb, l, (uint32_t)id, dnb);
                } else {
                    float worst;
                    const int64_t pos = farthest(nb, l, nc, worst);
                    if (dnb < worst) {
                        evicted = list(nb, l)[pos];
                        set_entry(nb, l, pos, (uint32_t)id, dnb);
                    }
                }
                if (evicted >= 0 && evicted < g.n) remove_link(evicted, l, nb);
                if (dirty) {
                    dirty->push_back(nb);
                    if (evicted >= 0 && evicted < g.n) dirty->push_back(evicted);
                }
                const uint32_t onc = count(id, l).load(std::memory_order_relaxed);
                if ((int64_t)onc < m_limit) {
                    add_published(id, l, nb, dnb);
                } else {
                    float worst;
                    const int64_t pos = farthest(id, l, onc, worst);
                    if (dnb < worst)
                        set_entry(id, l, pos, nb, dnb);
                    else
                        link_drops.fetch_add(1, std::memory_order_relaxed);
                }
            }
        }
    }

    // _insert_to_graph_mt (hnsw.mojo:2117-2240).
    void insert(int64_t id, Scratch& s) {
        const int lvl = g.level[id];
        const int8_t* q = code(id);
        const float* v = row(id, s.fbuf);
        int64_t ep = g.entry;
        for (int l = g.max_level; l > lvl; --l) {
            float best = dist_f32_i8(v, code(ep), g.dim, scale, offset);
            bool changed = true;
            while (changed) {
                changed = false;
                const int64_t cur = ep;
                if (l > g.level[cur]) break;
                const uint32_t nc = count(cur, l).load(std::memory_order_acquire);
                const uint32_t* lst = list(cur, l);
                for (uint32_t i = 0; i < nc; ++i) {
                    const uint32_t nb = lst[i];
                    if (nb >= (uint32_t)g.n) continue;
                    const float d = dist_f32_i8(v, code(nb), g.dim, scale, offset);
                    if (d < best) {
                        best = d;
                        ep = nb;
                        changed = true;
                    }
                }
            }
        }
        for (int l = std::min(lvl, g.max_level); l >= 0; --l) {
            search_layer(q, ep, g.efc, l, s);
            if (s.res.size() == 0) continue;
            s.all.clear();
            while (s.res.size() > 0) s.all.push_back(s.res.pop());
            const int64_t m_limit = cap(l);
            ep = s.all.back().id;
            prune(s.all, m_limit, s);
            for (size_t j = 0; j < s.pruned.size(); ++j) {
                const uint32_t nb = s.pruned[j];
                const float dnb = s.pruned_d[j];  // dist_i8(q, code(nb))
                int64_t evicted = -1;
                lock(nb);
                const uint32_t nc = count(nb, l).load(std::memory_order_relaxed);
                if ((int64_t)nc < m_limit) {
                    add_published(nb, l, (uint32_t)id, dnb);
                } else {
                    float worst;
                    const int64_t pos = farthest(nb, l, nc, worst);
                    if (dnb < worst) {
                        evicted = list(nb, l)[pos];
                        set_entry(nb, l, pos, (uint32_t)id, dnb);
                    }
                }
                unlock(nb);
                if (evicted >= 0 && evicted < g.n) {
                    lock(evicted);
                    remove_link(evicted, l, nb);
                    unlock(evicted);
                }
                lock(id);
                const uint32_t onc = count(id, l).load(std::memory_order_relaxed);
                if ((int64_t)onc < m_limit) {
                    add_published(id, l, nb, dnb);
                } else {
                    float worst;
                    const int64_t pos = farthest(id, l, onc, worst);
                    if (dnb < worst)
                        set_entry(id, l, pos, nb, dnb);
                    else
                        link_drops.fetch_add(1, std::memory_order_relaxed);
                }
                unlock(id);
            }
        }
    }

    bool has_link(int64_t i, uint32_t target) {
        const uint32_t c = count(i, 0).load(std::memory_order_relaxed);
        const uint32_t* lst = list(i, 0);
        for (uint32_t k = 0; k < c; ++k)
            if (lst[k] == target) return true;
        return false;
    }

    // _relink_node_l0 (hnsw.mojo:2242-2300), serial.
    void relink_l0(int64_t u, Scratch& s) {
        if (g.entry < 0 || g.n <= 1) return;
        const int8_t* q = code(u);
        search_layer(q, g.entry, g.efc, 0, s);
        if (s.res.size() == 0) return;
        s.all.clear();
        while (s.res.size() > 0) s.all.push_back(s.res.pop());
        const int64_t m_limit = 2 * g.M;
        prune(s.all, m_limit, s);
        for (size_t j = 0; j < s.pruned.size(); ++j) {
            const uint32_t nb = s.pruned[j];
            const float dnb = s.pruned_d[j];  // dist_i8(q, code(nb))
            if ((int64_t)nb == u) continue;
            if (has_link(u, nb)) continue;
            if ((int64_t)count(u, 0).load() >= m_limit) break;
            add_published(u, 0, nb, dnb);
            if (has_link(nb, (uint32_t)u)) continue;
            const uint32_t nc = count(nb, 0).load();
            if ((int64_t)nc < m_limit) {
                add_published(nb, 0, (uint32_t)u, dnb);
            } else {
                float worst;
                const int64_t pos = farthest(nb, 0, nc, worst);
                if (dnb < worst) {
                    const uint32_t ev = list(nb, 0)[pos];
                    set_entry(nb, 0, pos, (uint32_t)u, dnb);
                    if (ev < (uint32_t)g.n) remove_link(ev, 0, nb);
                }
            }
        }
    }

    void mark_reachable(int64_t start, std::vector<uint8_t>& reach, std::vector<uint32_t>& queue) {
        if (reach[start]) return;
        reach[start] = 1;
        queue.clear();
        queue.push_back((uint32_t)start);
        for (size_t h = 0; h < queue.size(); ++h) {
            const uint32_t x = queue[h];
            const uint32_t c = count(x, 0).load();
            const uint32_t* lst = list(x, 0);
            for (uint32_t k = 0; k < c; ++k) {
                const uint32_t nb = lst[k];
                if (nb >= (uint32_t)g.n || reach[nb]) continue;
                reach[nb] = 1;
                queue.push_back(nb);
            }
        }
    }

    // _repair_l0_exits (hnsw.mojo:2380-2435): re-link every node that cannot get back
    // to the entry point.
    int64_t repair_exits(Scratch& s) {
        const int64_t n = g.n;
        if (n <= 1 || g.entry < 0) return 0;
        std::vector<uint8_t> back((size_t)n, 0);
        back[g.entry] = 1;
        bool changed = true;
        while (changed) {
            changed = false;
            for (int dir = 0; dir < 2; ++dir) {
                for (int64_t j = 0; j < n; ++j) {
                    const int64_t i = dir == 0 ? j : n - 1 - j;
                    if (back[i]) continue;
                    const uint32_t c = count(i, 0).load();
                    const uint32_t* lst = list(i, 0);
                    for (uint32_t k = 0; k < c; ++k) {
                        if (lst[k] < (uint32_t)n && back[lst[k]]) {
                            back[i] = 1;
                            changed = true;
                            break;
                        }
                    }
                }
            }
        }
        int64_t relinked = 0;
        for (int64_t v = 0; v < n; ++v) {
            if (back[v]) continue;
            count(v, 0).store(0);
            relink_l0(v, s);
            if (count(v, 0).load() > 0) ++relinked;
        }
        return relinked;
    }

    // _repair_l0_reachability (hnsw.mojo:2437-2536): link every node the entry point
    // cannot reach from its closest reachable node.
    int64_t repair_reachability(Scratch& s) {
        const int64_t n = g.n;
        if (n <= 1 || g.entry < 0) return 0;
        const int64_t capl = 2 * g.M;
        std::vector<uint8_t> reach((size_t)n);
        std::vector<int32_t> indeg((size_t)n);
        std::vector<uint32_t> queue;
        int64_t total = 0;
        for (int pass = 0; pass < 3; ++pass) {
            std::fill(reach.begin(), reach.end(), 0);
            std::fill(indeg.begin(), indeg.end(), 0);
            for (int64_t i = 0; i < n; ++i) {
                const uint32_t c = count(i, 0).load();
                const uint32_t* lst = list(i, 0);
                for (uint32_t k = 0; k < c; ++k)
                    if (lst[k] < (uint32_t)n) ++indeg[lst[k]];
            }
            mark_reachable(g.entry, reach, queue);
            int64_t linked = 0;
            for (int64_t u = 0; u < n; ++u) {
                if (reach[u]) continue;
                search_layer(code(u), g.entry, g.efc, 0, s);
                s.all.clear();
                while (s.res.size() > 0) s.all.push_back(s.res.pop());  // farthest first
                int64_t pick = -1;
                float pick_d = 0.0f;  // dist_i8(code(u), code(pick)), as the search found it
                for (int64_t fi = (int64_t)s.all.size() - 1; fi >= 0; --fi) {
                    const uint32_t r = s.all[fi].id;
                    if ((int64_t)r != u && reach[r] && (int64_t)count(r, 0).load() < capl) {
                        add_published(r, 0, (uint32_t)u, s.all[fi].d);
                        pick = r;
                        pick_d = s.all[fi].d;
                        break;
                    }
                }
                for (int64_t fi = (int64_t)s.all.size() - 1; pick < 0 && fi >= 0; --fi) {
                    const uint32_t r = s.all[fi].id;
                    if ((int64_t)r == u || !reach[r]) continue;
                    const uint32_t nc = count(r, 0).load();
                    const uint32_t* lst = list(r, 0);
                    const float* dl = dlist(r, 0);
                    int64_t wpos = -1;
                    float wd = -1.0f;
                    for (uint32_t k = 0; k < nc; ++k) {
                        if (lst[k] >= (uint32_t)n) continue;
                        if (dl[k] > wd) {
                            wd = dl[k];
                            wpos = k;
                        }
                    }
                    if (wpos < 0) continue;
                    const uint32_t w = lst[wpos];
                    if (indeg[w] < 2) continue;
                    set_entry(r, 0, wpos, (uint32_t)u, s.all[fi].d);
                    --indeg[w];
                    pick = r;
                    pick_d = s.all[fi].d;
                }
                if (pick < 0) continue;
                ++indeg[u];
                if ((int64_t)count(u, 0).load() < capl && !has_link(u, (uint32_t)pick)) {
                    add_published(u, 0, (uint32_t)pick, pick_d);
                    ++indeg[pick];
                }
                ++linked;
                mark_reachable(u, reach, queue);
            }
            total += linked;
            if (linked == 0) break;
        }
        return total;
    }

    // compact_vectors + _build_l0_slots (hnsw.mojo:2761-2990) and the upper-level
    // export.
    void compact() {
        const int64_t n = g.n, dim = g.dim;
        g.hdr = 8;
        g.stride = (dim + g.hdr + 63) / 64 * 64;
        g.compact.assign((size_t)(n * g.stride), 0);
        g.node_slot.assign((size_t)n, 0xFFFFFFFFu);
        std::vector<uint32_t> order;
        order.reserve((size_t)n);
        std::vector<uint8_t> seen((size_t)n, 0);
        if (g.entry >= 0) {
            order.push_back((uint32_t)g.entry);
            seen[g.entry] = 1;
        }
        for (size_t h = 0; h < order.size(); ++h) {
            const uint32_t idx = order[h];
            for (int l = 0; l <= g.level[idx]; ++l) {
                const uint32_t c = count(idx, l).load();
                const uint32_t* lst = list(idx, l);
                for (uint32_t k = 0; k < c; ++k) {
                    const uint32_t nb = lst[k];
                    if (nb >= (uint32_t)n || seen[nb]) continue;
                    seen[nb] = 1;
                    order.push_back(nb);
                }
            }
        }
        for (int64_t i = 0; i < n; ++i)
            if (!seen[i]) order.push_back((uint32_t)i);
        for (int64_t slot = 0; slot < n; ++slot) {
            const uint32_t idx = order[slot];
            int8_t* dst = g.compact.data() + slot * g.stride;
            const int8_t* src = code(idx);
            float norm_sq = 0.0f, prefix = 0.0f;
            for (int64_t j = 0; j < dim; ++j) {
                const float v2 = (float)((int32_t)src[j] * (int32_t)src[j]);
                norm_sq += v2;
                if (j < 256) prefix += v2;
            }
            std::memcpy(dst, &norm_sq, 4);
            std::memcpy(dst + 4, &prefix, 4);
            std::memcpy(dst + g.hdr, src, (size_t)dim);
            g.node_slot[idx] = (uint32_t)slot;
        }
        g.l0_compact.assign((size_t)(n * 33), 0);
        g.l0_slots.assign((size_t)(n * 33), 0);
        for (int64_t i = 0; i < n; ++i) {
            const uint32_t c = std::min<uint32_t>(count(i, 0).load(), 32);
            const uint32_t* lst = list(i, 0);
            uint32_t actual = 0;
            for (uint32_t k = 0; k < c; ++k) {
                if (lst[k] >= (uint32_t)n) continue;
                g.l0_compact[i * 33 + 1 + actual] = lst[k];
                g.l0_slots[i * 33 + 1 + actual] = g.node_slot[lst[k]];
                ++actual;
            }
            g.l0_compact[i * 33] = actual;
            g.l0_slots[i * 33] = actual;
        }
        g.upper_offset.assign((size_t)n, -1);
        int64_t rows_total = 0;
        for (int64_t i = 0; i < n; ++i)
            if (g.level[i] > 0) {
                g.upper_offset[i] = rows_total;
                rows_total += g.level[i];
            }
        g.upper_links.assign((size_t)(rows_total * (1 + g.M)), 0);
        for (int64_t i = 0; i < n; ++i) {
            for (int l = 1; l <= g.level[i]; ++l) {
                uint32_t* row = g.upper_links.data() + (g.upper_offset[i] + l - 1) * (1 + g.M);
                const uint32_t c = std::min<uint32_t>(count(i, l).load(), (uint32_t)g.M);
                const uint32_t* lst = list(i, l);
                uint32_t actual = 0;
                for (uint32_t k = 0; k < c; ++k)
                    if (lst[k] < (uint32_t)n) row[1 + actual++] = lst[k];
                row[0] = actual;
            }
        }
        g.upper_rows = rows_total;
        g.node_ids.resize((size_t)n);
        for (int64_t i = 0; i < n; ++i) g.node_ids[i] = (int32_t)(g.id_base + i);
    }
};

// SplitMix64 level of node i (_level_of, hnsw.mojo:563-576).
int level_of(int64_t i, float ml) {
    uint64_t z = kLevelSeed + (uint64_t)(i + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z = z ^ (z >> 31);
    float r = (float)((double)(z >> 11) * (1.0 / 9007199254740992.0));
    if (r <= 0.0f) r = 1e-7f;
    int level = (int)(-std::log(r) * ml);
    return level > kLevelCap ? kLevelCap : level;
}

}  // namespace

int build(const float* rows, int64_t n, int64_t dim, int64_t M, int64_t efc, int metric,
          int64_t id_base, int n_threads, Graph& g, BuildStats* stats, int64_t max_batch,
          BatchPlanner* planner, int64_t planner_min) {
    g = Graph();
    g.n = n;
    g.dim = dim;
    g.M = M;
    g.efc = efc;
    g.metric = metric;
    g.id_base = id_base;
    Builder b(g, rows);
    std::vector<float> fbuf((size_t)dim);

    // _calibrate: Welford over the first min(n, 65536) (normalised) rows, mean +- 8 sigma.
    {
        const int64_t cn = std::min(n, kCalibrationSampleMax);
        double mean = 0.0, m2 = 0.0, cntv = 0.0;
        for (int64_t r = 0; r < cn; ++r) {
            const float* x = b.row(r, fbuf);
            for (int64_t j = 0; j < dim; ++j) {
                cntv += 1.0;
                const double d1 = x[j] - mean;
                mean += d1 / cntv;
                m2 += d1 * (x[j] - mean);
            }
        }
        const float var = cntv > 0 ? (float)(m2 / cntv) : 0.0f;
        const float sd = var > 0 ? std::sqrt(var) : 0.0f;
        float qmin = (float)mean - 8.0f * sd, qmax = (float)mean + 8.0f * sd;
        if (cntv == 0) {
            qmin = -0.20f;
            qmax = 0.20f;
        } else if (qmax - qmin < 1e-6f) {
            qmin = (float)mean - 0.20f;
            qmax = (float)mean + 0.20f;
        }
        g.gmin = qmin;
        g.gmax = qmax;
    }
    float range = g.gmax - g.gmin;
    if (range <= 0.0f) range = 1.0f;
    b.scale = range / 254.0f;
    b.offset = 127.0f * b.scale + g.gmin;

    // Serial pre-pass: levels, codes, entry = first node of the highest level.
    const float ml = 1.0f / std::log((float)M);
    g.level.resize((size_t)n);
    g.codes.resize((size_t)(n * dim));
    int best_level = -1;
    int64_t best_idx = 0;
    for (int64_t i = 0; i < n; ++i) {
        const int lv = level_of(i, ml);
        g.level[i] = (int8_t)lv;
        if (lv > best_level) {
            best_level = lv;
            best_idx = i;
        }
    }
    {
        const int nt = std::max(1, n_threads);
        std::vector<std::thread> th;
        for (int t = 0; t < nt; ++t)
            th.emplace_back([&, t]() {
                std::vector<float> buf((size_t)dim);
                for (int64_t i = t; i < n; i += nt) {
                    const float* x = b.row(i, buf);
                    int8_t* q = g.codes.data() + i * dim;
                    for (int64_t j = 0; j < dim; ++j) {
                        float nv = (x[j] - g.gmin) / range;
                        if (nv > 1.0f) nv = 1.0f;
                        if (nv < 0.0f) nv = 0.0f;
                        q[j] = (int8_t)((int)(nv * 254.0f) - 127);
                    }
                }
            });
        for (auto& x : th) x.join();
    }
    g.entry = n > 0 ? best_idx : -1;
    g.max_level = best_level;

    b.link_base.resize((size_t)n);
    b.cnt_base.resize((size_t)n);
    int64_t lt = 0, ct = 0;
    for (int64_t i = 0; i < n; ++i) {
        b.link_base[i] = lt;
        b.cnt_base[i] = ct;
        lt += 2 * M + (int64_t)g.level[i] * M;
        ct += 1 + g.level[i];
    }
    b.links.assign((size_t)lt, 0xFFFFFFFFu);
    b.link_d.assign((size_t)lt, 0.0f);
    b.cnt.reset(new std::atomic<uint32_t>[(size_t)std::max<int64_t>(ct, 1)]);
    for (int64_t i = 0; i < ct; ++i) b.cnt[i].store(0, std::memory_order_relaxed);
    b.locks.reset(new std::atomic<uint8_t>[(size_t)std::max<int64_t>(n, 1)]);
    for (int64_t i = 0; i < n; ++i) b.locks[i].store(0, std::memory_order_relaxed);

    const bool batched = max_batch > 0;
    int lanes = batched ? 1 : (n >= 4096 ? std::max(1, n_threads) : 1);
    int64_t batches = 0;
    if (n > 0 && batched) {
        // Batched insertion: the nodes of a batch are planned against the graph as it
        // stood before the batch (in parallel: the graph is read only), then linked one by
        // one in node order.  The batch grows with the graph (a quarter of the nodes
        // linked so far, at most max_batch), so the first nodes go in one at a time.
        // The result does not depend on the thread count.
        const int nt = std::max(1, n_threads);
        std::vector<Builder::Scratch> scratch((size_t)nt);
        for (auto& sc : scratch) b.init_scratch(sc);
        std::vector<int64_t> order;
        order.reserve((size_t)n);
        for (int64_t i = 0; i < n; ++i)
            if (i != g.entry) order.push_back(i);
        std::vector<Builder::Plan> plans;
        // With a planner: every node whose lists changed since its last update.
        std::vector<int64_t> dirty;
        std::vector<float> brows;
        bool use_planner =
            planner != nullptr &&
            planner->begin(g, g.codes.data(), b.link_base.data(), b.cnt_base.data(),
                           (int64_t)b.links.size(), ct, b.scale, b.offset, max_batch) == 0;
        if (use_planner) b.dirty = &dirty;
        int64_t done = 0, linked = 1;
        while (done < (int64_t)order.size()) {
            int64_t bsz = std::max<int64_t>(1, linked / 4);
            bsz = std::min(bsz, max_batch);
            bsz = std::min(bsz, (int64_t)order.size() - done);
            if ((int64_t)plans.size() < bsz) plans.resize((size_t)bsz);
            bool planned = false;
            if (use_planner && bsz >= planner_min) {
                // the graph's changes since the last batch, then this batch's rows
                std::sort(dirty.begin(), dirty.end());
                dirty.erase(std::unique(dirty.begin(), dirty.end()), dirty.end());
                const uint32_t* cnts = reinterpret_cast<const uint32_t*>(b.cnt.get());
                static_assert(sizeof(std::atomic<uint32_t>) == sizeof(uint32_t), "counts");
                if (planner->update(dirty.data(), (int64_t)dirty.size(), b.links.data(), cnts) ==
                    0) {
                    dirty.clear();
                    brows.resize((size_t)(bsz * dim));
                    const int use = (int)std::min<int64_t>(nt, bsz);
                    auto rows_of = [&](int t) {
                        std::vector<float> buf((size_t)dim);
                        for (int64_t j = t; j < bsz; j += use) {
                            const float* x = b.row(order[(size_t)(done + j)], buf);
                            std::memcpy(brows.data() + j * dim, x, (size_t)dim * sizeof(float));
                        }
                    };
                    std::vector<std::thread> th;
                    for (int t = 1; t < use; ++t) th.emplace_back(rows_of, t);
                    rows_of(0);
                    for (auto& x : th) x.join();
                    planned = planner->plan(order.data() + done, bsz, brows.data(), plans) == 0;
                    if (planned && stats) stats->planned_elsewhere += bsz;
                } else {
                    use_planner = false;  // the planner failed: the host plans the rest
                    b.dirty = nullptr;
                }
            }
            if (!planned) {
                std::atomic<int64_t> next{0};
                auto work = [&](int t) {
                    for (int64_t j = next.fetch_add(1); j < bsz; j = next.fetch_add(1))
                        b.plan(order[(size_t)(done + j)], scratch[(size_t)t], plans[(size_t)j]);
                };
                const int use = (int)std::min<int64_t>(nt, bsz);
                if (use <= 1) {
                    work(0);
                } else {
                    std::vector<std::thread> th;
                    for (int t = 1; t < use; ++t) th.emplace_back(work, t);
                    work(0);
                    for (auto& x : th) x.join();
                }
            }
            for (int64_t j = 0; j < bsz; ++j) b.link(order[(size_t)(done + j)], plans[(size_t)j]);
            done += bsz;
            linked += bsz;
            ++batches;
        }
    } else if (n > 0) {
        std::vector<std::thread> th;
        for (int t = 0; t < lanes; ++t)
            th.emplace_back([&, t]() {
                Builder::Scratch s;
                b.init_scratch(s);
                for (int64_t i = t; i < n; i += lanes)
                    if (i != g.entry) b.insert(i, s);
            });
        for (auto& x : th) x.join();
    }
    Builder::Scratch s;
    b.init_scratch(s);
    int64_t relinked = 0, exits = 0, links = 0;
    if (n > 0) {
        if (lanes > 1 || (batched && max_batch > 1))
            for (int64_t i = 0; i < n; ++i)
                if ((int64_t)b.count(i, 0).load() < M / 2) {
                    b.relink_l0(i, s);
                    ++relinked;
                }
        for (int round = 0; round < 3; ++round) {
            const int64_t e = b.repair_exits(s);
            const int64_t l = b.repair_reachability(s);
            exits += e;
            links += l;
            if (e == 0 && l == 0) break;
        }
    }
    b.compact();
    if (stats) {
        stats->lanes = batched ? -batches : lanes;
        stats->link_drops = (int64_t)b.link_drops.load();
        stats->relinked = relinked;
        stats->repaired_exits = exits;
        stats->repaired_links = links;
    }
    std::vector<int8_t>().swap(g.codes);
    return 0;
}

}  // namespace hnsw
}  // namespace pion
