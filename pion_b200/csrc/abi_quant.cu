// C-ABI of the block-quantised HNSW search: the host quantiser (hnsw_quant.cpp), device
// registration of a graph with its PolarQuant / NanoQuant / TurboQuant slots, and the
// batched search (quant.cu).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "hnsw_host.h"
#include "internal.h"

using namespace pion;

namespace {

constexpr int kDim = 1536;
constexpr int kBlocks = 48;

template <typename T>
int upload(T** dst, const T* src, size_t count) {
    *dst = nullptr;
    if (count == 0) return 0;
    if (cudaMalloc(reinterpret_cast<void**>(dst), count * sizeof(T)) != cudaSuccess) {
        cudaGetLastError();
        *dst = nullptr;
        return PION_B200_ENOMEM;
    }
    if (cudaMemcpy(*dst, src, count * sizeof(T), cudaMemcpyHostToDevice) != cudaSuccess)
        return PION_B200_ECUDA;
    return 0;
}

int64_t stride_of(int kind) { return hnsw::quant_stride(kind); }
int block_bytes(int kind) { return kind == kQPolar ? 18 : kind == kQNano ? 10 : 14; }
int code_bytes(int kind) { return kind == kQPolar ? 768 : kind == kQNano ? 384 : 576; }

// The graph checks the search relies on (the INT8 compact buffer is not used).
const char* check_graph(const pion_b200_hnsw_layout* L) {
    const int64_t n = L->num_nodes;
    if (n < 0 || n >= (int64_t)0x7fffffff) return "num_nodes out of range";
    if (L->dim != kDim) return "dim must be 1536";
    if (L->M < 1 || 2 * L->M > 32) return "M must be in [1, 16]";
    if (L->metric != 0 && L->metric != 1) return "metric must be 0 (L2) or 1 (COSINE)";
    if (n == 0) return nullptr;
    if (!L->l0_compact || !L->l0_slots || !L->node_slot || !L->node_ids || !L->node_level ||
        !L->upper_offset)
        return "null layout buffer";
    if (L->entry_point < 0 || L->entry_point >= n) return "entry_point out of range";
    if (L->max_level < 0 || L->max_level > 64) return "max_level out of range";
    if (L->upper_rows < 0 || (L->upper_rows > 0 && !L->upper_links)) return "bad upper_links";
    for (int64_t i = 0; i < n; ++i) {
        if (L->node_slot[i] >= (uint64_t)n) return "node_slot out of range";
        const int64_t off = L->upper_offset[i];
        const int lv = L->node_level[i];
        if (lv < 0) return "negative node_level";
        if (lv > 0 && (off < 0 || off + lv > L->upper_rows)) return "upper_offset out of range";
        const uint32_t* row = L->l0_compact + i * 33;
        const uint32_t* srow = L->l0_slots + i * 33;
        if (row[0] > (uint32_t)(2 * L->M)) return "level-0 count above 2M";
        for (uint32_t k = 0; k < row[0]; ++k)
            if (row[1 + k] < (uint32_t)n && srow[1 + k] != 0xffffffffu &&
                srow[1 + k] >= (uint32_t)n)
                return "l0_slots entry out of range";
    }
    return nullptr;
}

const char* check_quant(const pion_b200_hnsw_quant_layout* Q, int64_t n) {
    if (Q->kind < kQPolar || Q->kind > kQTurbo) return "unknown quant kind";
    if (Q->num_nodes != n) return "quant num_nodes differs from the graph's";
    if (Q->stride != stride_of(Q->kind)) return "stride does not match the kind";
    if (n > 0 && !Q->compact) return "null compact buffer";
    if (Q->kind == kQTurbo && (!Q->qjl) != (!Q->qjl_res_norms))
        return "qjl and qjl_res_norms go together";
    if (!std::isfinite(Q->qjl_lambda)) return "qjl_lambda not finite";
    return nullptr;
}

// Graphs registered by pion_v_quant_beam_1536, keyed by the view's host buffers.
struct QuantBeamGraph {
    const uint32_t* l0c;
    const uint32_t* l0s;
    const int8_t* comp;
    const uint64_t* qjl;
    const float* qres;
    int64_t n, stride, hdr;
    int kind, device;
    uint64_t fp;  // content fingerprint of the host tables when copied
    float* norms = nullptr;
    uint16_t* scales = nullptr;
    uint8_t* codes = nullptr;
    uint32_t* l0_compact = nullptr;
    uint32_t* l0_slots = nullptr;
    uint64_t* qjl_dev = nullptr;
    float* qres_dev = nullptr;
};
std::mutex g_qbeam_mu;
std::vector<QuantBeamGraph*> g_qbeam_graphs;

void free_qbeam_graph(QuantBeamGraph* g) {
    cudaSetDevice(g->device);
    cudaDeviceSynchronize();
    void* ps[] = {g->norms, g->scales, g->codes, g->l0_compact, g->l0_slots, g->qjl_dev,
                  g->qres_dev};
    for (void* p : ps)
        if (p) cudaFree(p);
    delete g;
}

int qbeam_fail(const char* what) {
    fprintf(stderr, "pion_vector_b200: pion_v_quant_beam_1536: %s\n", what);
    return -1;
}

uint64_t qbeam_fingerprint(const pion_quant_beam_view_1536* v) {
    uint64_t h = 0xcbf29ce484222325ull ^ (uint64_t)v->kind;
    h = sample_rows_hash(h, v->l0_compact, v->num_nodes, 33 * 4, 33 * 4);
    h = sample_rows_hash(h, v->l0_slots, v->num_nodes, 33 * 4, 33 * 4);
    h = sample_rows_hash(h, v->compact_buffer, v->num_nodes, v->compact_stride, 256);
    h = sample_rows_hash(h, v->qjl_buffer, v->num_nodes, 24 * 8, 24 * 8);
    return sample_rows_hash(h, v->qjl_res_norms, v->num_nodes, 4, 4);
}

// The registered copy of the view's graph (checked and copied on first use), keyed by
// the view's host pointers and sizes and a fingerprint of sampled rows of its tables:
// a different graph placed at the same addresses is copied again, not served stale.
QuantBeamGraph* qbeam_graph(pion_b200_ctx* ctx, const pion_quant_beam_view_1536* v,
                            const char** why) {
    std::lock_guard<std::mutex> lock(g_qbeam_mu);
    const uint64_t fp = qbeam_fingerprint(v);
    for (size_t i = 0; i < g_qbeam_graphs.size(); ++i) {
        QuantBeamGraph* g = g_qbeam_graphs[i];
        if (g->l0c == v->l0_compact && g->l0s == v->l0_slots && g->comp == v->compact_buffer &&
            g->qjl == v->qjl_buffer && g->qres == v->qjl_res_norms && g->n == v->num_nodes &&
            g->stride == v->compact_stride && g->hdr == v->compact_hdr && g->kind == v->kind &&
            g->device == ctx->device) {
            if (g->fp == fp) return g;
            free_qbeam_graph(g);  // same addresses, other content: drop the stale copy
            g_qbeam_graphs.erase(g_qbeam_graphs.begin() + (ptrdiff_t)i);
            break;
        }
    }
    const int64_t n = v->num_nodes;
    const int kind = (int)v->kind;
    const int bb = block_bytes(kind), cb = bb - 2, cbytes = code_bytes(kind);
    if (v->compact_hdr < 0 || v->compact_stride < v->compact_hdr + stride_of(kind)) {
        *why = "compact stride too small for the block format";
        return nullptr;
    }
    for (int64_t i = 0; i < n; ++i) {  // every listed neighbour names a slot
        const uint32_t* row = v->l0_compact + i * 33;
        if (row[0] > 32u) {
            *why = "a level-0 count above 32";
            return nullptr;
        }
        for (uint32_t k = 0; k < row[0]; ++k)
            if (row[1 + k] < (uint32_t)n && v->l0_slots[i * 33 + 1 + k] >= (uint32_t)n) {
                *why = "an l0_slots entry names no slot";
                return nullptr;
            }
    }
    QuantBeamGraph* g = new (std::nothrow) QuantBeamGraph{
        v->l0_compact, v->l0_slots, v->compact_buffer, v->qjl_buffer, v->qjl_res_norms, n,
        v->compact_stride, v->compact_hdr, kind, ctx->device, fp};
    if (!g) {
        *why = "out of host memory";
        return nullptr;
    }
    int rc = 0;
    try {
        std::vector<float> norms((size_t)n);
        std::vector<uint16_t> scales((size_t)n * kBlocks);
        std::vector<uint8_t> codes((size_t)n * cbytes);
        for (int64_t sl = 0; sl < n; ++sl) {
            const int8_t* src = v->compact_buffer + sl * v->compact_stride + v->compact_hdr;
            std::memcpy(&norms[sl], src, 4);
            for (int b = 0; b < kBlocks; ++b) {
                std::memcpy(&scales[sl * kBlocks + b], src + 4 + b * bb, 2);
                std::memcpy(&codes[sl * cbytes + (size_t)b * cb], src + 4 + b * bb + 2, (size_t)cb);
            }
        }
        rc = upload(&g->norms, norms.data(), norms.size());
        if (!rc) rc = upload(&g->scales, scales.data(), scales.size());
        if (!rc) rc = upload(&g->codes, codes.data(), codes.size());
    } catch (const std::bad_alloc&) {
        rc = PION_B200_ENOMEM;
    }
    if (!rc) rc = upload(&g->l0_compact, v->l0_compact, (size_t)n * 33);
    if (!rc) rc = upload(&g->l0_slots, v->l0_slots, (size_t)n * 33);
    if (!rc && kind == kQTurbo && v->qjl_buffer && v->qjl_res_norms) {
        rc = upload(&g->qjl_dev, v->qjl_buffer, (size_t)n * 24);
        if (!rc) rc = upload(&g->qres_dev, v->qjl_res_norms, (size_t)n);
    }
    if (rc) {
        free_qbeam_graph(g);
        *why = "device copy of the graph failed";
        return nullptr;
    }
    g_qbeam_graphs.push_back(g);
    return g;
}

}  // namespace

void pion::quant_beam_forget(const uint32_t* l0_compact) {
    std::lock_guard<std::mutex> lock(g_qbeam_mu);
    std::vector<QuantBeamGraph*> keep;
    for (QuantBeamGraph* g : g_qbeam_graphs) {
        if (!l0_compact || g->l0c == l0_compact)
            free_qbeam_graph(g);
        else
            keep.push_back(g);
    }
    g_qbeam_graphs.swap(keep);
}

extern "C" {

int64_t pion_v_quant_beam_1536(pion_quant_beam_view_1536* v) {
    if (!v || !v->candidates || !v->results || !v->query_block_int8 || !v->query_block_scales ||
        !v->l0_compact || !v->l0_slots || !v->compact_buffer || v->num_nodes <= 0 ||
        v->num_nodes >= 0x7fffffff)
        return qbeam_fail("bad view");
    if (v->kind < kQPolar || v->kind > kQTurbo) return qbeam_fail("unknown block format");
    const int64_t ef = v->ef < 1 ? 1 : v->ef;
    if (ef > quant_top_entries()) return qbeam_fail("ef above 1024");
    const int64_t n = v->num_nodes;
    pion_heap_list& cl = v->candidates->data;
    pion_heap_list& rl = v->results->data;
    if (cl.len < 0 || cl.capacity < cl.len || (cl.len > 0 && !cl.data) || rl.len < 0 ||
        rl.len > ef || rl.capacity < rl.len || (rl.len > 0 && !rl.data))
        return qbeam_fail("bad heaps");
    if (cl.len > n + 1) return qbeam_fail("more candidates than nodes");
    for (int64_t i = 0; i < cl.len + rl.len; ++i) {
        const int64_t id = i < cl.len ? cl.data[i].id : rl.data[i - cl.len].id;
        if (id < 0 || id >= n) return qbeam_fail("a heap entry names no node");
    }
    pion_b200_ctx* ctx = compat_default_ctx("pion_v_quant_beam_1536");
    if (!ctx) return -1;
    if (use_device(ctx) != 0) return qbeam_fail("cannot select the device");
    const char* why = "";
    QuantBeamGraph* g = qbeam_graph(ctx, v, &why);
    if (!g) return qbeam_fail(why);
    const int per_sm = quant_ctas_per_sm((int)ef);
    if (per_sm <= 0) return qbeam_fail("ef does not fit");
    cudaStream_t st = ctx->stream;
    const int64_t cand_io_cap = cl.capacity > 0 ? cl.capacity : 1;
    const size_t del_bytes = v->deleted ? (size_t)(n + 7) / 8 : 0;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off += align_up(bytes, 256);
        return o;
    };
    const size_t o_codes = take(kDim), o_scales = take(kBlocks * 4), o_norms = take(8),
                 o_signs = take(24 * 8), o_meta = take(6 * 4), o_del = take(del_bytes),
                 o_cand = take((size_t)cand_io_cap * 8), o_res = take((size_t)ef * 8),
                 o_q = take(kDim * 4);
    const int warps = quant_warps_per_cta(), top = quant_top_entries();
    const int64_t vis_words = ((n + 31) / 32 + 3) / 4 * 4;
    const int64_t cap = n + cl.len + 1;
    const size_t tail = (size_t)warps * (size_t)std::max<int64_t>(cap - top, 0) * 8;
    if (ensure(ctx->stage_in, off) != 0 || ensure(ctx->hnsw_misc, 64) != 0 ||
        ensure(ctx->hnsw_visited, (size_t)warps * vis_words * 4) != 0 ||
        ensure(ctx->scratch2, tail > 0 ? tail : 16) != 0)
        return qbeam_fail("out of device memory");
    char* base = static_cast<char*>(ctx->stage_in.ptr);
    // host side of the copies: the heaps as (f32 dist, u32 node) entries, the scalars
    std::vector<uint32_t> cand_h((size_t)cand_io_cap * 2), res_h((size_t)ef * 2);
    for (int64_t i = 0; i < cl.len; ++i) {
        std::memcpy(&cand_h[2 * i], &cl.data[i].distance, 4);
        cand_h[2 * i + 1] = (uint32_t)cl.data[i].id;
    }
    for (int64_t i = 0; i < rl.len; ++i) {
        std::memcpy(&res_h[2 * i], &rl.data[i].distance, 4);
        res_h[2 * i + 1] = (uint32_t)rl.data[i].id;
    }
    int32_t meta[6] = {(int32_t)cl.len, (int32_t)rl.len, 0, 0, 0, 0};
    std::memcpy(&meta[2], &v->results->cached_worst, 4);
    const float norms2[2] = {v->query_block_norm, v->qjl_query_res_norm};
    bool ok =
        cudaMemcpyAsync(base + o_codes, v->query_block_int8, kDim, cudaMemcpyHostToDevice, st) ==
            cudaSuccess &&
        cudaMemcpyAsync(base + o_scales, v->query_block_scales, kBlocks * 4,
                        cudaMemcpyHostToDevice, st) == cudaSuccess &&
        cudaMemcpyAsync(base + o_norms, norms2, 8, cudaMemcpyHostToDevice, st) == cudaSuccess &&
        (!v->qjl_query_signs || cudaMemcpyAsync(base + o_signs, v->qjl_query_signs, 24 * 8,
                                                cudaMemcpyHostToDevice, st) == cudaSuccess) &&
        cudaMemcpyAsync(base + o_meta, meta, sizeof(meta), cudaMemcpyHostToDevice, st) ==
            cudaSuccess &&
        (!del_bytes || cudaMemcpyAsync(base + o_del, v->deleted, del_bytes,
                                       cudaMemcpyHostToDevice, st) == cudaSuccess) &&
        (cl.len == 0 || cudaMemcpyAsync(base + o_cand, cand_h.data(), (size_t)cl.len * 8,
                                        cudaMemcpyHostToDevice, st) == cudaSuccess) &&
        (rl.len == 0 || cudaMemcpyAsync(base + o_res, res_h.data(), (size_t)rl.len * 8,
                                        cudaMemcpyHostToDevice, st) == cudaSuccess) &&
        cudaMemsetAsync(ctx->hnsw_misc.ptr, 0, 64, st) == cudaSuccess;
    if (!ok) return qbeam_fail("copy to the device failed");
    unsigned long long* stats = static_cast<unsigned long long*>(ctx->hnsw_misc.ptr);
    QuantLaunch Lc;
    Lc.kind = (int)v->kind;
    Lc.metric = 0;
    Lc.codes = g->codes;
    Lc.code_bytes = code_bytes((int)v->kind);
    Lc.scales = g->scales;
    Lc.norms = g->norms;
    Lc.qjl = g->qjl_dev;
    Lc.res_norms = g->qres_dev;
    Lc.lambda = v->qjl_lambda;
    Lc.l0_compact = g->l0_compact;
    Lc.l0_slots = g->l0_slots;
    Lc.deleted = del_bytes ? reinterpret_cast<const uint8_t*>(base + o_del) : nullptr;
    Lc.num_nodes = n;
    Lc.queries = reinterpret_cast<const float*>(base + o_q);  // not read in this mode
    Lc.nq = 1;
    Lc.k = 1;
    Lc.ef = (int)ef;
    Lc.visited = static_cast<uint32_t*>(ctx->hnsw_visited.ptr);
    ctx->vis_clean = false;  // this kernel leaves its bitmaps set
    Lc.vis_words = vis_words;
    Lc.cand_tail = ctx->scratch2.ptr;
    Lc.cand_cap = cap;
    Lc.next_query = reinterpret_cast<unsigned*>(stats + 3);
    Lc.stats = stats;
    Lc.status = call_status(ctx, PION_B200_MEM_HOST);
    Lc.ctas = 1;
    Lc.from_heaps = 1;
    Lc.given_codes = reinterpret_cast<const int8_t*>(base + o_codes);
    Lc.given_scales = reinterpret_cast<const float*>(base + o_scales);
    Lc.given_norms = reinterpret_cast<const float*>(base + o_norms);
    Lc.given_signs = v->qjl_query_signs ? reinterpret_cast<const uint64_t*>(base + o_signs)
                                        : nullptr;
    Lc.cand_io = base + o_cand;
    Lc.cand_io_cap = cand_io_cap;
    Lc.res_io = base + o_res;
    Lc.heap_meta = reinterpret_cast<int*>(base + o_meta);
    if (launch_quant_search(Lc, st) != 0) return qbeam_fail("launch failed");
    ctx->launches++;
    if (cudaMemcpyAsync(meta, base + o_meta, sizeof(meta), cudaMemcpyDeviceToHost, st) !=
            cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return qbeam_fail("copy from the device failed");
    const int32_t cn = meta[3], rn = meta[4];
    if (cn < 0 || rn < 0 || rn > ef) return qbeam_fail("bad heap sizes from the device");
    if (rn > rl.capacity) return qbeam_fail("the results heap's List is too small");
    const int64_t cw = cn < cand_io_cap ? cn : cand_io_cap;
    if ((cw > 0 && cudaMemcpy(cand_h.data(), base + o_cand, (size_t)cw * 8,
                              cudaMemcpyDeviceToHost) != cudaSuccess) ||
        (rn > 0 && cudaMemcpy(res_h.data(), base + o_res, (size_t)rn * 8,
                              cudaMemcpyDeviceToHost) != cudaSuccess))
        return qbeam_fail("copy from the device failed");
    if (finish_sync(ctx) != 0) return qbeam_fail(pion_v_b200_last_error(ctx));
    const int64_t cfit = cw < cl.capacity ? cw : cl.capacity;
    for (int64_t i = 0; i < cfit; ++i) {
        std::memcpy(&cl.data[i].distance, &cand_h[2 * i], 4);
        cl.data[i].pad = 0;
        cl.data[i].id = (int64_t)cand_h[2 * i + 1];
    }
    cl.len = cfit;
    for (int64_t i = 0; i < rn; ++i) {
        std::memcpy(&rl.data[i].distance, &res_h[2 * i], 4);
        rl.data[i].pad = 0;
        rl.data[i].id = (int64_t)res_h[2 * i + 1];
    }
    rl.len = rn;
    std::memcpy(&v->results->cached_worst, &meta[5], 4);
    return 0;
}

int pion_v_b200_hnsw_quantize(const pion_b200_hnsw_graph* graph, const float* rows,
                              int64_t n_rows, int kind, pion_b200_hnsw_quant** out_quant) {
    if (!graph || !out_quant) return PION_B200_EINVAL;
    *out_quant = nullptr;
    if (n_rows != graph->g.n || (n_rows > 0 && !rows)) {
        fprintf(stderr, "pion_vector_b200: hnsw_quantize: rows must be the graph's %lld rows\n",
                (long long)graph->g.n);
        return PION_B200_EINVAL;
    }
    pion_b200_hnsw_quant* q = new (std::nothrow) pion_b200_hnsw_quant();
    if (!q) return PION_B200_ENOMEM;
    std::string why;
    int rc = 0;
    try {
        rc = hnsw::quantize(graph->g, rows, kind, q->q, why);
    } catch (const std::bad_alloc&) {
        rc = PION_B200_ENOMEM;
        why = "out of host memory";
    }
    if (rc != 0) {
        fprintf(stderr, "pion_vector_b200: hnsw_quantize: %s\n", why.c_str());
        delete q;
        return rc;
    }
    q->n = graph->g.n;
    *out_quant = q;
    return 0;
}

int pion_v_b200_hnsw_quant_layout(const pion_b200_hnsw_quant* quant,
                                  pion_b200_hnsw_quant_layout* out) {
    if (!quant || !out) return PION_B200_EINVAL;
    const hnsw::QuantBuffers& b = quant->q;
    *out = pion_b200_hnsw_quant_layout{};
    out->kind = b.kind;
    out->num_nodes = quant->n;
    out->compact = b.compact.data();
    out->stride = b.stride;
    out->qjl = b.qjl.empty() ? nullptr : b.qjl.data();
    out->qjl_res_norms = b.qjl_res_norms.empty() ? nullptr : b.qjl_res_norms.data();
    out->qjl_random_signs = b.random_signs.empty() ? nullptr : b.random_signs.data();
    out->qjl_lambda = 1.0f;
    out->rerank = b.rerank.empty() ? nullptr : b.rerank.data();
    return 0;
}

int pion_v_b200_hnsw_quant_free(pion_b200_hnsw_quant* quant) {
    if (!quant) return PION_B200_EINVAL;
    delete quant;
    return 0;
}

int pion_v_b200_hnsw_load_quant(const char* path, pion_b200_hnsw_graph** out_graph,
                                pion_b200_hnsw_quant** out_quant) {
    if (!path || !out_graph || !out_quant) return PION_B200_EINVAL;
    *out_graph = nullptr;
    *out_quant = nullptr;
    pion_b200_hnsw_graph* gr = new (std::nothrow) pion_b200_hnsw_graph();
    pion_b200_hnsw_quant* qz = new (std::nothrow) pion_b200_hnsw_quant();
    if (!gr || !qz) {
        delete gr;
        delete qz;
        return PION_B200_ENOMEM;
    }
    std::string why;
    int rc = 0;
    try {
        rc = hnsw::load_file(path, gr->g, &qz->q, why);
    } catch (const std::bad_alloc&) {
        rc = PION_B200_ENOMEM;
        why = "out of host memory";
    }
    if (rc != 0) {
        fprintf(stderr, "pion_vector_b200: hnsw_load_quant %s: %s\n", path, why.c_str());
        delete gr;
        delete qz;
        return rc;
    }
    *out_graph = gr;
    if (qz->q.kind >= kQPolar) {
        qz->n = gr->g.n;
        *out_quant = qz;
    } else {
        delete qz;
    }
    return 0;
}

int pion_v_b200_hnsw_save_quant(const pion_b200_hnsw_graph* graph,
                                const pion_b200_hnsw_quant* quant, const char* path,
                                int64_t max_elements) {
    if (!graph || !quant || !path) return PION_B200_EINVAL;
    if (quant->n != graph->g.n) {
        fprintf(stderr, "pion_vector_b200: hnsw_save_quant: quant buffers of another graph\n");
        return PION_B200_EINVAL;
    }
    std::string why;
    int rc = 0;
    try {
        rc = hnsw::save_file(graph->g, &quant->q, path, max_elements, why);
    } catch (const std::bad_alloc&) {
        rc = PION_B200_ENOMEM;
        why = "out of host memory";
    }
    if (rc != 0) fprintf(stderr, "pion_vector_b200: hnsw_save_quant %s: %s\n", path, why.c_str());
    return rc;
}

int pion_v_b200_register_hnsw_quant(pion_b200_ctx* ctx, const pion_b200_hnsw_layout* L,
                                    const pion_b200_hnsw_quant_layout* Q,
                                    pion_b200_index** out_index) {
    if (!valid_ctx(ctx) || !out_index || !L || !Q) return PION_B200_EINVAL;
    *out_index = nullptr;
    if (const char* why = check_graph(L))
        return set_error(ctx, PION_B200_EINVAL, "register_hnsw_quant: %s", why);
    if (const char* why = check_quant(Q, L->num_nodes))
        return set_error(ctx, PION_B200_EINVAL, "register_hnsw_quant: %s", why);
    if (int rc = use_device(ctx)) return rc;
    pion_b200_index* ix = new (std::nothrow) pion_b200_index();
    if (!ix) return set_error(ctx, PION_B200_ENOMEM, "register_hnsw_quant: out of host memory");
    ix->kind = kHNSWQuant;
    ix->device = ctx->device;
    ix->n_rows = L->num_nodes;
    ix->dim = L->dim;
    auto& h = ix->hnsw;
    h.M = (int)L->M;
    h.max_level = (int)L->max_level;
    h.entry = L->entry_point;
    h.metric = L->metric;
    h.quant_kind = Q->kind;
    h.code_bytes = code_bytes(Q->kind);
    h.qjl_lambda = Q->qjl_lambda;
    const size_t n = (size_t)L->num_nodes;
    int rc = 0;
    try {
        if (n > 0) {
            // slots re-laid out as |v|^2, the 48 f16 scales and the packed codes, each
            // array 16-byte aligned per slot
            const int bb = block_bytes(Q->kind), cb = bb - 2;
            std::vector<float> norms(n);
            std::vector<uint16_t> scales(n * kBlocks);
            std::vector<uint8_t> codes(n * (size_t)h.code_bytes);
            for (size_t s = 0; s < n; ++s) {
                const int8_t* src = Q->compact + s * (size_t)Q->stride;
                std::memcpy(&norms[s], src, 4);
                for (int b = 0; b < kBlocks; ++b) {
                    std::memcpy(&scales[s * kBlocks + b], src + 4 + b * bb, 2);
                    std::memcpy(&codes[s * h.code_bytes + (size_t)b * cb], src + 4 + b * bb + 2,
                                (size_t)cb);
                }
            }
            rc = upload(&h.norms, norms.data(), n);
            if (!rc) rc = upload(&h.qscales, scales.data(), scales.size());
            if (!rc) rc = upload(&h.qcodes, codes.data(), codes.size());
            if (!rc) rc = upload(&h.l0_compact, L->l0_compact, n * 33);
            if (!rc) rc = upload(&h.l0_slots, L->l0_slots, n * 33);
            if (!rc) rc = upload(&h.node_slot, L->node_slot, n);
            if (!rc) rc = upload(&h.node_ids, L->node_ids, n);
            if (!rc) rc = upload(&h.node_level, L->node_level, n);
            if (!rc) rc = upload(&h.upper_offset, L->upper_offset, n);
            if (!rc && L->upper_rows > 0) {
                const size_t words = (size_t)L->upper_rows * (1 + L->M);
                rc = upload(&h.upper_links, L->upper_links, words);
                // the slots of the upper-level neighbours (every position of a row, as the
                // greedy may read past a row's count), so a step needs no dependent load
                std::vector<uint32_t> us(words, 0xffffffffu);
                for (size_t r = 0; r < (size_t)L->upper_rows; ++r) {
                    const uint32_t* row = L->upper_links + r * (1 + L->M);
                    us[r * (1 + L->M)] = row[0];
                    for (int64_t k = 0; k < L->M; ++k)
                        if (row[1 + k] < (uint32_t)n)
                            us[r * (1 + L->M) + 1 + k] = L->node_slot[row[1 + k]];
                }
                if (!rc) rc = upload(&h.upper_slots, us.data(), words);
            }
            if (!rc && L->deleted) rc = upload(&h.deleted, L->deleted, (n + 7) / 8);
            if (!rc && Q->kind == kQTurbo && Q->qjl) {
                rc = upload(&h.qjl, Q->qjl, n * 24);
                if (!rc) rc = upload(&h.qjl_res, Q->qjl_res_norms, n);
            }
            if (!rc && Q->kind == kQTurbo && Q->qjl_random_signs)
                rc = upload(&h.qjl_rs, Q->qjl_random_signs, 24);
            if (!rc && Q->rerank) rc = upload(&h.rerank_node, Q->rerank, n * kDim);
            if (!rc) {  // external id -> node, for metric_scores (dense id ranges only)
                int64_t lo = L->node_ids[0], hi = L->node_ids[0];
                for (size_t i = 1; i < n; ++i) {
                    lo = L->node_ids[i] < lo ? L->node_ids[i] : lo;
                    hi = L->node_ids[i] > hi ? L->node_ids[i] : hi;
                }
                const int64_t span = hi - lo + 1;
                if (span <= 4 * (int64_t)n + 1024) {
                    std::vector<int32_t> inv((size_t)span, -1);
                    for (size_t i = 0; i < n; ++i) inv[(size_t)(L->node_ids[i] - lo)] = (int32_t)i;
                    rc = upload(&h.ext_to_node, inv.data(), (size_t)span);
                    h.ext_base = lo;
                    h.ext_count = span;
                }
            }
        }
    } catch (const std::bad_alloc&) {
        rc = PION_B200_ENOMEM;
    }
    if (rc) {
        pion_v_b200_index_free(ix);
        return set_error(ctx, rc, "register_hnsw_quant: device copy failed");
    }
    *out_index = ix;
    return 0;
}

int pion_v_b200_hnsw_quant_search(pion_b200_ctx* ctx, const pion_b200_index* ix, const float* q,
                                  int64_t nq, int64_t k, int64_t ef, int32_t* out_ids,
                                  float* out_scores, int32_t* out_found, int mem) {
    if (!valid_ctx(ctx)) return PION_B200_EINVAL;
    if (!ix || ix->kind != kHNSWQuant)
        return set_error(ctx, PION_B200_EINVAL, "hnsw_quant_search: not a quantised HNSW index");
    if (ix->device != ctx->device)
        return set_error(ctx, PION_B200_EINVAL, "hnsw_quant_search: index on another device");
    if (nq < 0 || k < 1 || (nq > 0 && (!q || !out_ids || !out_scores || !out_found)))
        return set_error(ctx, PION_B200_EINVAL, "hnsw_quant_search: bad arguments");
    if (ef < 1 || ef > quant_top_entries())
        return set_error(ctx, PION_B200_ESHAPE, "hnsw_quant_search: ef %lld not in [1, %d]",
                         (long long)ef, quant_top_entries());
    if (nq > (1 << 24) || k > (1 << 16))
        return set_error(ctx, PION_B200_ESHAPE, "hnsw_quant_search: batch or k too large");
    if (mem != PION_B200_MEM_HOST && mem != PION_B200_MEM_DEVICE)
        return set_error(ctx, PION_B200_EINVAL, "hnsw_quant_search: bad mem %d", mem);
    if (nq == 0) return 0;
    if (int rc = use_device(ctx)) return rc;
    cudaStream_t st = ctx->stream;
    const auto& h = ix->hnsw;
    const size_t out_bytes = (size_t)nq * k * 4, found_bytes = (size_t)nq * 4;
    const float* dq = q;
    int32_t* di = out_ids;
    float* dv = out_scores;
    int32_t* df = out_found;
    if (mem == PION_B200_MEM_HOST) {
        if (ensure(ctx->stage_in, (size_t)nq * kDim * 4) != 0 ||
            ensure(ctx->stage_out, 2 * align_up(out_bytes, 256) + align_up(found_bytes, 256)) != 0)
            return set_error(ctx, PION_B200_ENOMEM, "hnsw_quant_search: staging");
        if (cudaMemcpyAsync(ctx->stage_in.ptr, q, (size_t)nq * kDim * 4, cudaMemcpyHostToDevice,
                            st) != cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "hnsw_quant_search: query copy failed");
        dq = static_cast<const float*>(ctx->stage_in.ptr);
        char* o = static_cast<char*>(ctx->stage_out.ptr);
        di = reinterpret_cast<int32_t*>(o);
        dv = reinterpret_cast<float*>(o + align_up(out_bytes, 256));
        df = reinterpret_cast<int32_t*>(o + 2 * align_up(out_bytes, 256));
    }
    // counters: 3 x u64 stats, then the two passes' query counters and the re-run count
    if (ensure(ctx->hnsw_misc, 64) != 0)
        return set_error(ctx, PION_B200_ENOMEM, "hnsw_quant_search: counters");
    unsigned long long* stats = static_cast<unsigned long long*>(ctx->hnsw_misc.ptr);
    unsigned* next1 = reinterpret_cast<unsigned*>(stats + 3);
    unsigned* next2 = next1 + 1;
    int* over_n = reinterpret_cast<int*>(next1 + 2);
    if (cudaMemsetAsync(ctx->hnsw_misc.ptr, 0, 64, st) != cudaSuccess)
        return set_error(ctx, PION_B200_ECUDA, "hnsw_quant_search: memset failed");
    int rc = 0;
    const int64_t n = ix->n_rows;
    if (n == 0) {
        rc = launch_fill_results(dv, di, (size_t)nq * k, INFINITY, st);
        if (!rc && cudaMemsetAsync(df, 0, found_bytes, st) != cudaSuccess) rc = PION_B200_ECUDA;
        ctx->launches++;
    } else {
        const int per_sm = quant_ctas_per_sm((int)ef);
        if (per_sm <= 0)
            return set_error(ctx, PION_B200_ESHAPE, "hnsw_quant_search: ef %lld does not fit",
                             (long long)ef);
        const int warps = quant_warps_per_cta(), top = quant_top_entries();
        int64_t ctas = (int64_t)per_sm * ctx->num_sms;
        const int64_t need = (nq + warps - 1) / warps;
        if (ctas > need) ctas = need;
        const int64_t vis_words = ((n + 31) / 32 + 3) / 4 * 4;
        // candidate heap: every node at most once, plus the start
        const int64_t cap_all = n + 1;
        int64_t cap1 = cap_all <= top ? top : (cap_all < 16384 ? cap_all : 16384);
        if (const char* e = getenv("PION_B200_QUANT_HEAP_CAP")) {  // tests: force re-runs
            const long long v = atoll(e);
            if (v >= 1 && v < cap1) cap1 = v;
        }
        const bool rerun = cap1 < cap_all;
        int64_t ctas2 = 0;
        if (rerun) {
            int64_t w2 = ((int64_t)1 << 30) / (std::max<int64_t>(cap_all - top, 1) * 8);
            if (w2 > ctas * warps) w2 = ctas * warps;
            ctas2 = w2 / warps < 1 ? 1 : w2 / warps;
        }
        const size_t tails = (size_t)std::max(ctas * warps * std::max<int64_t>(cap1 - top, 0),
                                              ctas2 * warps * std::max<int64_t>(cap_all - top, 0)) *
                             8;
        if (ensure(ctx->hnsw_visited, (size_t)ctas * warps * vis_words * 4) != 0 ||
            ensure(ctx->scratch2, tails > 0 ? tails : 16) != 0 ||
            ensure(ctx->scratch, found_bytes) != 0)
            return set_error(ctx, PION_B200_ENOMEM, "hnsw_quant_search: scratch");
        QuantLaunch Lc;
        Lc.kind = h.quant_kind;
        Lc.metric = h.metric;
        Lc.codes = h.qcodes;
        Lc.code_bytes = h.code_bytes;
        Lc.scales = h.qscales;
        Lc.norms = h.norms;
        Lc.qjl = h.qjl;
        Lc.res_norms = h.qjl_res;
        Lc.rsigns = h.qjl_rs;
        Lc.lambda = h.qjl_lambda;
        Lc.rerank = h.rerank_node;
        Lc.l0_compact = h.l0_compact;
        Lc.l0_slots = h.l0_slots;
        Lc.node_slot = h.node_slot;
        Lc.node_ids = h.node_ids;
        Lc.deleted = h.deleted;
        Lc.node_level = h.node_level;
        Lc.upper_offset = h.upper_offset;
        Lc.upper_links = h.upper_links;
        Lc.upper_slots = h.upper_slots;
        Lc.M = h.M;
        Lc.max_level = h.max_level;
        Lc.num_nodes = n;
        Lc.entry = h.entry;
        Lc.queries = dq;
        Lc.nq = (int)nq;
        Lc.k = (int)k;
        Lc.ef = (int)ef;
        Lc.visited = static_cast<uint32_t*>(ctx->hnsw_visited.ptr);
    ctx->vis_clean = false;  // this kernel leaves its bitmaps set
        Lc.vis_words = vis_words;
        Lc.cand_tail = ctx->scratch2.ptr;
        Lc.cand_cap = cap1;
        Lc.out_ids = di;
        Lc.out_scores = dv;
        Lc.out_found = df;
        Lc.overflow = rerun ? static_cast<int*>(ctx->scratch.ptr) : nullptr;
        Lc.overflow_n = over_n;
        Lc.next_query = next1;
        Lc.stats = stats;
        Lc.status = call_status(ctx, mem);
        Lc.ctas = (int)ctas;
        timing_begin(ctx);
        rc = launch_quant_search(Lc, st);
        ctx->launches++;
        if (!rc && rerun) {  // the queries whose heap outgrew cap1, with room for all
            Lc.qlist = static_cast<int*>(ctx->scratch.ptr);
            Lc.qlist_n = over_n;
            Lc.overflow = nullptr;
            Lc.cand_cap = cap_all;
            Lc.next_query = next2;
            Lc.ctas = (int)ctas2;
            rc = launch_quant_search(Lc, st);
            ctx->launches++;
        }
        timing_end(ctx);
    }
    if (rc != 0)
        return set_error(ctx, rc, "hnsw_quant_search: launch failed: %s",
                         cudaGetErrorString(cudaGetLastError()));
    if (mem == PION_B200_MEM_HOST) {
        if (cudaMemcpyAsync(out_ids, di, out_bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaMemcpyAsync(out_scores, dv, out_bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaMemcpyAsync(out_found, df, found_bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "hnsw_quant_search: result copy failed");
        return finish_sync(ctx);
    }
    return 0;
}

}  // extern "C"
