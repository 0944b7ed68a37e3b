// C-ABI for HNSW: the host builder (hnsw_build.cpp), device registration of a graph in
// the reference's compact layout, and the batched beam search (hnsw.cu).
#include <cuda_runtime.h>

#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <thread>
#include <vector>

#include "hnsw_host.h"
#include "internal.h"

using namespace pion;

namespace {

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

// Structural checks the beam kernel relies on; returns a message or nullptr.
const char* check_layout(const pion_b200_hnsw_layout* L) {
    const int64_t n = L->num_nodes;
    if (n < 0 || n >= (int64_t)0x7fffffff) return "num_nodes out of range";
    if (L->dim != hnsw_dim()) return "dim must be 1536";
    if (L->M < 1 || 2 * L->M > 32) return "M must be in [1, 16]";
    if (L->compact_hdr != 8) return "compact_hdr must be 8";
    if (L->compact_stride % 16 != 0 || L->compact_stride < L->compact_hdr + L->dim + 8)
        return "compact_stride must be a multiple of 16 and >= dim + 16";
    if (L->metric != 0 && L->metric != 1) return "metric must be 0 (L2) or 1 (COSINE)";
    if (n == 0) return nullptr;
    if (!L->compact_buffer || !L->l0_compact || !L->l0_slots || !L->node_slot || !L->node_ids ||
        !L->node_level || !L->upper_offset)
        return "null layout buffer";
    if (L->entry_point < 0 || L->entry_point >= n) return "entry_point out of range";
    if (L->max_level < 0 || L->max_level > 64) return "max_level out of range";
    if (L->upper_rows < 0 || (L->upper_rows > 0 && !L->upper_links)) return "bad upper_links";
    auto deleted = [&](uint32_t i) {
        return L->deleted && ((L->deleted[i >> 3] >> (i & 7)) & 1u);
    };
    for (int64_t i = 0; i < n; ++i) {
        if (L->node_slot[i] >= (uint64_t)n) return "node_slot out of range";
        const int64_t off = L->upper_offset[i];
        const int lv = L->node_level[i];
        if (lv < 0) return "negative node_level";
        if (off >= 0 && off + lv > L->upper_rows) return "upper_offset out of range";
        const uint32_t* row = L->l0_compact + i * 33;
        const uint32_t* srow = L->l0_slots + i * 33;
        const uint32_t c = row[0] < 32 ? row[0] : 32;
        for (uint32_t k = 0; k < c; ++k) {
            const uint32_t nb = row[1 + k];
            if (nb < (uint32_t)n && !deleted(nb) && srow[1 + k] >= (uint32_t)n)
                return "l0_slots entry out of range";
        }
    }
    return nullptr;
}

}  // namespace

extern "C" {

int pion_v_b200_hnsw_build(const float* rows, int64_t n_rows, int64_t dim, int64_t M,
                           int64_t ef_construction, int metric, int64_t id_base, int n_threads,
                           pion_b200_hnsw_graph** out_graph) {
    if (!out_graph) return PION_B200_EINVAL;
    *out_graph = nullptr;
    if (n_rows < 0 || (n_rows > 0 && !rows) || dim <= 0 || M < 2 || M > 16 ||
        ef_construction < 1 || (metric != 0 && metric != 1) || id_base < 0 ||
        n_rows + id_base > INT32_MAX || n_rows >= 0x7fffffff) {
        fprintf(stderr, "pion_vector_b200: hnsw_build: bad arguments\n");
        return PION_B200_EINVAL;
    }
    __builtin_cpu_init();
    if (!__builtin_cpu_supports("avx2") || !__builtin_cpu_supports("fma")) {
        fprintf(stderr, "pion_vector_b200: hnsw_build needs a CPU with AVX2 and FMA\n");
        return PION_B200_ESHAPE;
    }
    if (n_threads <= 0) n_threads = (int)std::thread::hardware_concurrency();
    if (n_threads <= 0) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    pion_b200_hnsw_graph* g = new (std::nothrow) pion_b200_hnsw_graph();
    if (!g) return PION_B200_ENOMEM;
    try {
        hnsw::build(rows, n_rows, dim, M, ef_construction, metric, id_base, n_threads, g->g,
                    &g->stats);
    } catch (const std::bad_alloc&) {
        delete g;
        return PION_B200_ENOMEM;
    }
    *out_graph = g;
    return 0;
}

int pion_v_b200_hnsw_build_batched(const float* rows, int64_t n_rows, int64_t dim, int64_t M,
                                   int64_t ef_construction, int metric, int64_t id_base,
                                   int n_threads, int64_t max_batch,
                                   pion_b200_hnsw_graph** out_graph) {
    if (!out_graph) return PION_B200_EINVAL;
    *out_graph = nullptr;
    if (max_batch < 1 || n_rows < 0 || (n_rows > 0 && !rows) || dim <= 0 || M < 2 || M > 16 ||
        ef_construction < 1 || (metric != 0 && metric != 1) || id_base < 0 ||
        n_rows + id_base > INT32_MAX || n_rows >= 0x7fffffff) {
        fprintf(stderr, "pion_vector_b200: hnsw_build_batched: bad arguments\n");
        return PION_B200_EINVAL;
    }
    __builtin_cpu_init();
    if (!__builtin_cpu_supports("avx2") || !__builtin_cpu_supports("fma")) {
        fprintf(stderr, "pion_vector_b200: hnsw_build_batched needs a CPU with AVX2 and FMA\n");
        return PION_B200_ESHAPE;
    }
    if (n_threads <= 0) n_threads = (int)std::thread::hardware_concurrency();
    if (n_threads <= 0) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    pion_b200_hnsw_graph* g = new (std::nothrow) pion_b200_hnsw_graph();
    if (!g) return PION_B200_ENOMEM;
    try {
        hnsw::build(rows, n_rows, dim, M, ef_construction, metric, id_base, n_threads, g->g,
                    &g->stats, max_batch);
    } catch (const std::bad_alloc&) {
        delete g;
        return PION_B200_ENOMEM;
    }
    *out_graph = g;
    return 0;
}

int pion_v_b200_hnsw_load(const char* path, pion_b200_hnsw_graph** out_graph) {
    if (!path || !out_graph) return PION_B200_EINVAL;
    *out_graph = nullptr;
    pion_b200_hnsw_graph* gr = new (std::nothrow) pion_b200_hnsw_graph();
    if (!gr) return PION_B200_ENOMEM;
    std::string why;
    int rc = 0;
    try {
        rc = hnsw::load_file(path, gr->g, nullptr, why);
    } catch (const std::bad_alloc&) {
        rc = PION_B200_ENOMEM;
        why = "out of host memory";
    }
    if (rc != 0) {
        fprintf(stderr, "pion_vector_b200: hnsw_load %s: %s\n", path, why.c_str());
        delete gr;
        return rc;
    }
    *out_graph = gr;
    return 0;
}

int pion_v_b200_hnsw_save(const pion_b200_hnsw_graph* graph, const char* path,
                          int64_t max_elements) {
    if (!graph || !path) return PION_B200_EINVAL;
    std::string why;
    int rc = 0;
    try {
        rc = hnsw::save_file(graph->g, nullptr, path, max_elements, why);
    } catch (const std::bad_alloc&) {
        rc = PION_B200_ENOMEM;
        why = "out of host memory";
    }
    if (rc != 0) fprintf(stderr, "pion_vector_b200: hnsw_save %s: %s\n", path, why.c_str());
    return rc;
}

int pion_v_b200_hnsw_graph_layout(const pion_b200_hnsw_graph* graph, pion_b200_hnsw_layout* out) {
    if (!graph || !out) return PION_B200_EINVAL;
    const hnsw::Graph& g = graph->g;
    *out = pion_b200_hnsw_layout{};
    out->num_nodes = g.n;
    out->dim = g.dim;
    out->M = g.M;
    out->entry_point = g.entry;
    out->max_level = g.max_level < 0 ? 0 : g.max_level;
    out->global_min = g.gmin;
    out->global_max = g.gmax;
    out->metric = g.metric;
    out->compact_buffer = g.compact.data();
    out->compact_stride = g.stride;
    out->compact_hdr = g.hdr;
    out->l0_compact = g.l0_compact.data();
    out->l0_slots = g.l0_slots.data();
    out->node_slot = g.node_slot.data();
    out->node_ids = g.node_ids.data();
    out->deleted = nullptr;
    out->node_level = g.level.data();
    out->upper_offset = g.upper_offset.data();
    out->upper_links = g.upper_links.data();
    out->upper_rows = g.upper_rows;
    return 0;
}

int pion_v_b200_hnsw_graph_stats(const pion_b200_hnsw_graph* graph, int64_t* out5) {
    if (!graph || !out5) return PION_B200_EINVAL;
    out5[0] = graph->stats.lanes;
    out5[1] = graph->stats.link_drops;
    out5[2] = graph->stats.relinked;
    out5[3] = graph->stats.repaired_exits;
    out5[4] = graph->stats.repaired_links;
    return 0;
}

int pion_v_b200_hnsw_graph_stats6(const pion_b200_hnsw_graph* graph, int64_t* out6) {
    if (!graph || !out6) return PION_B200_EINVAL;
    pion_v_b200_hnsw_graph_stats(graph, out6);
    out6[5] = graph->stats.planned_elsewhere;
    return 0;
}

int pion_v_b200_hnsw_graph_free(pion_b200_hnsw_graph* graph) {
    if (!graph) return PION_B200_EINVAL;
    delete graph;
    return 0;
}

int pion_v_b200_register_hnsw(pion_b200_ctx* ctx, const pion_b200_hnsw_layout* L,
                              pion_b200_index** out_index) {
    if (!valid_ctx(ctx) || !out_index || !L) return PION_B200_EINVAL;
    *out_index = nullptr;
    if (const char* why = check_layout(L))
        return set_error(ctx, PION_B200_EINVAL, "register_hnsw: %s", why);
    if (int rc = use_device(ctx)) return rc;
    pion_b200_index* ix = new (std::nothrow) pion_b200_index();
    if (!ix) return set_error(ctx, PION_B200_ENOMEM, "register_hnsw: out of host memory");
    ix->kind = kHNSW;
    ix->device = ctx->device;
    ix->n_rows = L->num_nodes;
    ix->dim = L->dim;
    auto& h = ix->hnsw;
    h.M = (int)L->M;
    h.max_level = (int)L->max_level;
    h.entry = L->entry_point;
    h.metric = L->metric;
    h.gmin = L->global_min;
    h.gmax = L->global_max;
    const size_t n = (size_t)L->num_nodes;
    int rc = 0;
    if (n > 0) {
        // the slot buffer travels once, then is re-laid out on the device as 16-byte
        // aligned code rows plus a norm array
        int8_t* slots = nullptr;
        rc = upload(&slots, L->compact_buffer, n * (size_t)L->compact_stride);
        if (!rc && (cudaMalloc(&h.codes, n * (size_t)hnsw_dim()) != cudaSuccess ||
                    cudaMalloc(&h.norms, n * sizeof(float)) != cudaSuccess)) {
            cudaGetLastError();
            rc = PION_B200_ENOMEM;
        }
        if (!rc)
            rc = launch_hnsw_relayout(slots, (int64_t)n, L->compact_stride, L->compact_hdr,
                                      h.codes, h.norms, ctx->stream);
        if (!rc && cudaStreamSynchronize(ctx->stream) != cudaSuccess) rc = PION_B200_ECUDA;
        if (slots) cudaFree(slots);
        if (!rc) rc = upload(&h.l0_compact, L->l0_compact, n * 33);
        if (!rc) rc = upload(&h.l0_slots, L->l0_slots, n * 33);
        if (!rc) rc = upload(&h.node_slot, L->node_slot, n);
        if (!rc) rc = upload(&h.node_ids, L->node_ids, n);
        if (!rc) rc = upload(&h.node_level, L->node_level, n);
        if (!rc) rc = upload(&h.upper_offset, L->upper_offset, n);
        if (!rc && L->upper_rows > 0) {
            const size_t words = (size_t)L->upper_rows * (1 + L->M);
            rc = upload(&h.upper_links, L->upper_links, words);
            // the slots of the upper-level neighbours, so the greedy descent finds a
            // neighbour's codes without a dependent load
            std::vector<uint32_t> us(words, 0xffffffffu);
            for (size_t r = 0; r < (size_t)L->upper_rows; ++r) {
                const uint32_t* row = L->upper_links + r * (1 + L->M);
                us[r * (1 + L->M)] = row[0];
                for (int64_t k = 0; k < L->M; ++k)
                    if (row[1 + k] < (uint32_t)n) us[r * (1 + L->M) + 1 + k] = L->node_slot[row[1 + k]];
            }
            if (!rc) rc = upload(&h.upper_slots, us.data(), words);
        }
        if (!rc && L->deleted) rc = upload(&h.deleted, L->deleted, (n + 7) / 8);
        if (!rc) {  // slot -> external id (gpu_slot_ext_ids, hnsw.mojo:2829-2874)
            std::vector<int32_t> se(n, -1);
            for (size_t i = 0; i < n; ++i) se[L->node_slot[i]] = L->node_ids[i];
            rc = upload(&h.slot_ext, se.data(), n);
        }
        if (!rc) {  // per 32 slots the smallest norm, for the brute-force scan's pre-test
            const size_t chunks = (n + 255) / 256 * 8;
            if (cudaMalloc(&h.chunk_vmin, chunks * sizeof(int)) != cudaSuccess) {
                cudaGetLastError();
                h.chunk_vmin = nullptr;
                rc = PION_B200_ENOMEM;
            }
            if (!rc) rc = launch_slot_chunk_vmin(h.norms, (int64_t)n, h.chunk_vmin, ctx->stream);
            if (!rc && cudaStreamSynchronize(ctx->stream) != cudaSuccess) rc = PION_B200_ECUDA;
        }
        if (!rc) {  // the slot codes as the B operand of the brute-force scan
            if (make_tmap_2d(&ix->tmap_rows, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, h.codes,
                             (uint64_t)hnsw_dim(), (uint64_t)n, (uint64_t)hnsw_dim(),
                             (uint32_t)slot_k_block(), (uint32_t)slot_tile_rows(),
                             CU_TENSOR_MAP_SWIZZLE_128B) != 0)
                rc = PION_B200_ECUDA;
            ix->has_tmap = rc == 0;
        }
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
    if (rc) {
        pion_v_b200_index_free(ix);
        return set_error(ctx, rc, "register_hnsw: device copy failed");
    }
    *out_index = ix;
    return 0;
}

int pion_v_b200_hnsw_search(pion_b200_ctx* ctx, const pion_b200_index* ix, const float* q,
                            int64_t nq, int64_t k, int64_t ef, int32_t* out_ids, float* out_dist,
                            int mem) {
    if (!valid_ctx(ctx)) return PION_B200_EINVAL;
    if (!ix || ix->kind != kHNSW) return set_error(ctx, PION_B200_EINVAL, "hnsw_search: not an HNSW index");
    if (ix->device != ctx->device)
        return set_error(ctx, PION_B200_EINVAL, "hnsw_search: index on another device");
    if (nq < 0 || k < 1 || (nq > 0 && (!q || !out_ids || !out_dist)))
        return set_error(ctx, PION_B200_EINVAL, "hnsw_search: bad arguments");
    if (ef < 1 || ef > 1024)
        return set_error(ctx, PION_B200_ESHAPE, "hnsw_search: ef %lld not in [1, 1024]",
                         (long long)ef);
    if (nq > (1 << 24) || k > (1 << 16))
        return set_error(ctx, PION_B200_ESHAPE, "hnsw_search: batch or k too large");
    if (mem != PION_B200_MEM_HOST && mem != PION_B200_MEM_DEVICE)
        return set_error(ctx, PION_B200_EINVAL, "hnsw_search: bad mem %d", mem);
    if (nq == 0) return 0;
    if (int rc = use_device(ctx)) return rc;
    cudaStream_t st = ctx->stream;
    const int dim = hnsw_dim();
    const auto& h = ix->hnsw;
    const size_t out_bytes = (size_t)nq * k * 4;
    const float* dq = q;
    int32_t* di = out_ids;
    float* dv = out_dist;
    if (mem == PION_B200_MEM_HOST) {
        if (ensure(ctx->stage_in, (size_t)nq * dim * 4) != 0 ||
            ensure(ctx->stage_out, 2 * align_up(out_bytes, 256)) != 0)
            return set_error(ctx, PION_B200_ENOMEM, "hnsw_search: staging");
        if (cudaMemcpyAsync(ctx->stage_in.ptr, q, (size_t)nq * dim * 4, cudaMemcpyHostToDevice,
                            st) != cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "hnsw_search: query copy failed");
        dq = static_cast<const float*>(ctx->stage_in.ptr);
        di = static_cast<int32_t*>(ctx->stage_out.ptr);
        dv = reinterpret_cast<float*>(static_cast<char*>(ctx->stage_out.ptr) +
                                      align_up(out_bytes, 256));
    }
    if (ensure(ctx->hnsw_misc, 64) != 0)
        return set_error(ctx, PION_B200_ENOMEM, "hnsw_search: counters");
    unsigned long long* stats = static_cast<unsigned long long*>(ctx->hnsw_misc.ptr);
    unsigned* next_query = reinterpret_cast<unsigned*>(stats + 3);
    if (cudaMemsetAsync(ctx->hnsw_misc.ptr, 0, 32, st) != cudaSuccess)
        return set_error(ctx, PION_B200_ECUDA, "hnsw_search: memset failed");
    int rc = 0;
    if (ix->n_rows == 0) {
        rc = launch_fill_results(dv, di, (size_t)nq * k, INFINITY, st);
        ctx->launches++;
    } else {
        const int per_sm = hnsw_ctas_per_sm((int)ef);
        if (per_sm <= 0)
            return set_error(ctx, PION_B200_ESHAPE, "hnsw_search: ef %lld does not fit",
                             (long long)ef);
        const int warps = hnsw_warps_per_cta();
        int64_t ctas = (int64_t)per_sm * ctx->num_sms;
        const int64_t need = (nq + warps - 1) / warps;
        if (ctas > need) ctas = need;
        HnswLaunch Lc;
        if (hnsw_visit_buffers(ctx, ctas * warps, ix->n_rows, Lc) != 0)
            return set_error(ctx, PION_B200_ENOMEM, "hnsw_search: visited bitmaps");
        size_t off = 0;
        auto take = [&](size_t bytes) {
            size_t o = off;
            off += align_up(bytes, 256);
            return o;
        };
        const size_t o_qn = take(h.metric == 1 ? (size_t)nq * dim * 4 : 0),
                     o_codes = take((size_t)nq * dim), o_blk = take((size_t)nq * 8 * 4);
        if (ensure(ctx->scratch, off) != 0)
            return set_error(ctx, PION_B200_ENOMEM, "hnsw_search: scratch");
        char* base = static_cast<char*>(ctx->scratch.ptr);
        const float* qsrc = dq;
        if (h.metric == 1) {
            // search_fp32_scored normalises the query, then _quantize_query_to_int8
            // normalises that result again in place (hnsw.mojo:4146-4149, :669-671).
            float* qn = reinterpret_cast<float*>(base + o_qn);
            rc = launch_l2_normalize_rows(dq, nq, dim, qn, nullptr, st);
            if (!rc) rc = launch_l2_normalize_rows(qn, nq, dim, qn, nullptr, st);
            ctx->launches += 2;
            qsrc = qn;
        }
        float range = h.gmax - h.gmin;
        if (range <= 0.0f) range = 1.0f;
        const float scale = 254.0f / range;
        int8_t* codes = reinterpret_cast<int8_t*>(base + o_codes);
        int32_t* blk = reinterpret_cast<int32_t*>(base + o_blk);
        if (!rc) rc = launch_hnsw_quantize(qsrc, (int)nq, h.gmin, scale, codes, blk, st);
        ctx->launches++;
        if (!rc) {
            Lc.codes = h.codes;
            Lc.norms = h.norms;
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
            Lc.num_nodes = ix->n_rows;
            Lc.entry = h.entry;
            Lc.qcodes = codes;
            Lc.qblk = blk;
            Lc.nq = (int)nq;
            Lc.k = (int)k;
            Lc.ef = (int)ef;
            Lc.out_ids = di;
            Lc.out_dist = dv;
            Lc.stats = stats;
            Lc.next_query = next_query;
            Lc.status = call_status(ctx, mem);
            Lc.ctas = (int)ctas;
            timing_begin(ctx);
            rc = launch_hnsw_beam(Lc, st);
            timing_end(ctx);
            ctx->launches++;
        }
    }
    if (rc != 0)
        return set_error(ctx, rc, "hnsw_search: launch failed: %s",
                         cudaGetErrorString(cudaGetLastError()));
    if (mem == PION_B200_MEM_HOST) {
        if (cudaMemcpyAsync(out_ids, di, out_bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaMemcpyAsync(out_dist, dv, out_bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "hnsw_search: result copy failed");
        return finish_sync(ctx);
    }
    return 0;
}

int pion_v_b200_hnsw_beam_batch(pion_b200_ctx* ctx, const pion_b200_index* ix,
                                const int8_t* q_codes, const float* q_norm, int64_t nq,
                                int64_t ef, void* pools, int32_t* pool_size,
                                const int32_t* pool_cursor, int mem) {
    if (!valid_ctx(ctx)) return PION_B200_EINVAL;
    if (!ix || ix->kind != kHNSW)
        return set_error(ctx, PION_B200_EINVAL, "hnsw_beam_batch: not an HNSW index");
    if (ix->device != ctx->device)
        return set_error(ctx, PION_B200_EINVAL, "hnsw_beam_batch: index on another device");
    if (nq < 0 || (nq > 0 && (!q_codes || !q_norm || !pools || !pool_size)))
        return set_error(ctx, PION_B200_EINVAL, "hnsw_beam_batch: bad arguments");
    if (ef < 1 || ef > 1024)
        return set_error(ctx, PION_B200_ESHAPE, "hnsw_beam_batch: ef %lld not in [1, 1024]",
                         (long long)ef);
    if (nq > (1 << 24))
        return set_error(ctx, PION_B200_ESHAPE, "hnsw_beam_batch: batch too large");
    if (mem != PION_B200_MEM_HOST && mem != PION_B200_MEM_DEVICE)
        return set_error(ctx, PION_B200_EINVAL, "hnsw_beam_batch: bad mem %d", mem);
    if (nq == 0 || ix->n_rows == 0) return 0;
    if (int rc = use_device(ctx)) return rc;
    const int per_sm = hnsw_ctas_per_sm((int)ef);
    if (per_sm <= 0)
        return set_error(ctx, PION_B200_ESHAPE, "hnsw_beam_batch: ef %lld does not fit",
                         (long long)ef);
    cudaStream_t st = ctx->stream;
    const int dim = hnsw_dim();
    const auto& h = ix->hnsw;
    const size_t cb = (size_t)nq * dim, nb = (size_t)nq * 4, pb = (size_t)nq * ef * 8;
    const int8_t* dc = q_codes;
    const float* dn = q_norm;
    void* dp = pools;
    int32_t* ds = pool_size;
    const int32_t* dcur = pool_cursor;
    int32_t* zero_cur = nullptr;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off += align_up(bytes, 256);
        return o;
    };
    const size_t o_c = take(mem == PION_B200_MEM_HOST ? cb : 0),
                 o_n = take(mem == PION_B200_MEM_HOST ? nb : 0),
                 o_p = take(mem == PION_B200_MEM_HOST ? pb : 0), o_s = take(nb),
                 o_k = take(nb);
    if (ensure(ctx->stage_in, off) != 0 || ensure(ctx->hnsw_misc, 64) != 0)
        return set_error(ctx, PION_B200_ENOMEM, "hnsw_beam_batch: staging");
    char* base = static_cast<char*>(ctx->stage_in.ptr);
    if (mem == PION_B200_MEM_HOST) {
        if (cudaMemcpyAsync(base + o_c, q_codes, cb, cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(base + o_n, q_norm, nb, cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(base + o_p, pools, pb, cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(base + o_s, pool_size, nb, cudaMemcpyHostToDevice, st) !=
                cudaSuccess ||
            (pool_cursor && cudaMemcpyAsync(base + o_k, pool_cursor, nb, cudaMemcpyHostToDevice,
                                            st) != cudaSuccess))
            return set_error(ctx, PION_B200_ECUDA, "hnsw_beam_batch: copy failed");
        dc = reinterpret_cast<const int8_t*>(base + o_c);
        dn = reinterpret_cast<const float*>(base + o_n);
        dp = base + o_p;
        ds = reinterpret_cast<int32_t*>(base + o_s);
        dcur = pool_cursor ? reinterpret_cast<const int32_t*>(base + o_k) : nullptr;
    }
    if (!dcur) {  // cursors default to 0 (the first unchecked entry is found by the scan)
        zero_cur = reinterpret_cast<int32_t*>(base + o_k);
        if (cudaMemsetAsync(zero_cur, 0, nb, st) != cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "hnsw_beam_batch: memset failed");
        dcur = zero_cur;
    }
    const int warps = hnsw_warps_per_cta();
    int64_t ctas = (int64_t)per_sm * ctx->num_sms;
    const int64_t need = (nq + warps - 1) / warps;
    if (ctas > need) ctas = need;
    HnswLaunch Lc;
    if (hnsw_visit_buffers(ctx, ctas * warps, ix->n_rows, Lc) != 0)
        return set_error(ctx, PION_B200_ENOMEM, "hnsw_beam_batch: visited bitmaps");
    unsigned long long* stats = static_cast<unsigned long long*>(ctx->hnsw_misc.ptr);
    if (cudaMemsetAsync(ctx->hnsw_misc.ptr, 0, 32, st) != cudaSuccess)
        return set_error(ctx, PION_B200_ECUDA, "hnsw_beam_batch: memset failed");
    Lc.codes = h.codes;
    Lc.norms = h.norms;
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
    Lc.num_nodes = ix->n_rows;
    Lc.entry = h.entry;
    Lc.qcodes = dc;
    Lc.qblk = nullptr;  // unused when starting from a pool
    Lc.nq = (int)nq;
    Lc.k = 0;
    Lc.ef = (int)ef;
    Lc.stats = stats;
    Lc.next_query = reinterpret_cast<unsigned*>(stats + 3);
    Lc.status = call_status(ctx, mem);
    Lc.ctas = (int)ctas;
    Lc.pool_io = dp;
    Lc.pool_stride = ef;
    Lc.pool_size = ds;
    Lc.pool_cursor = dcur;
    Lc.qn_given = dn;
    Lc.pool_size_out = ds;
    timing_begin(ctx);
    int rc = launch_hnsw_beam(Lc, st);
    timing_end(ctx);
    ctx->launches++;
    if (rc != 0)
        return set_error(ctx, rc, "hnsw_beam_batch: launch failed: %s",
                         cudaGetErrorString(cudaGetLastError()));
    if (mem == PION_B200_MEM_HOST) {
        if (cudaMemcpyAsync(pools, dp, pb, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaMemcpyAsync(pool_size, ds, nb, cudaMemcpyDeviceToHost, st) != cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "hnsw_beam_batch: result copy failed");
        return finish_sync(ctx);
    }
    return 0;
}

int pion_v_b200_hnsw_metric_scores(pion_b200_ctx* ctx, const pion_b200_index* ix, const float* q,
                                   int64_t nq, int64_t k, const int32_t* ids, float* scores,
                                   int mem) {
    if (!valid_ctx(ctx)) return PION_B200_EINVAL;
    if (!ix || (ix->kind != kHNSW && ix->kind != kHNSWQuant))
        return set_error(ctx, PION_B200_EINVAL, "hnsw_metric_scores: not an HNSW index");
    if (ix->device != ctx->device)
        return set_error(ctx, PION_B200_EINVAL, "hnsw_metric_scores: index on another device");
    if (nq < 0 || k < 1 || (nq > 0 && (!q || !ids || !scores)))
        return set_error(ctx, PION_B200_EINVAL, "hnsw_metric_scores: bad arguments");
    if (mem != PION_B200_MEM_HOST && mem != PION_B200_MEM_DEVICE)
        return set_error(ctx, PION_B200_EINVAL, "hnsw_metric_scores: bad mem %d", mem);
    if (nq == 0 || ix->n_rows == 0) return 0;
    const auto& h = ix->hnsw;
    // a block-quantised graph scores from its FP32 copy; without one it has neither source
    // and keeps its scores (the reference's `return False`)
    if (ix->kind == kHNSWQuant && !h.rerank_node) return 1;
    if (!h.ext_to_node)
        return set_error(ctx, PION_B200_ESHAPE, "hnsw_metric_scores: external ids too sparse");
    if (nq > (1 << 24) || k > (1 << 16))
        return set_error(ctx, PION_B200_ESHAPE, "hnsw_metric_scores: batch or k too large");
    if (int rc = use_device(ctx)) return rc;
    cudaStream_t st = ctx->stream;
    const int dim = hnsw_dim();
    const size_t qb = (size_t)nq * dim * 4, rb = (size_t)nq * k * 4;
    const float* dq = q;
    const int32_t* di = ids;
    float* ds = scores;
    if (mem == PION_B200_MEM_HOST) {
        if (ensure(ctx->stage_in, align_up(qb, 256) + align_up(rb, 256)) != 0 ||
            ensure(ctx->stage_out, rb) != 0)
            return set_error(ctx, PION_B200_ENOMEM, "hnsw_metric_scores: staging");
        char* in = static_cast<char*>(ctx->stage_in.ptr);
        if (cudaMemcpyAsync(in, q, qb, cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(in + align_up(qb, 256), ids, rb, cudaMemcpyHostToDevice, st) !=
                cudaSuccess ||
            cudaMemcpyAsync(ctx->stage_out.ptr, scores, rb, cudaMemcpyHostToDevice, st) !=
                cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "hnsw_metric_scores: copy failed");
        dq = reinterpret_cast<const float*>(in);
        di = reinterpret_cast<const int32_t*>(in + align_up(qb, 256));
        ds = static_cast<float*>(ctx->stage_out.ptr);
    }
    const float* qsrc = dq;
    int rc = 0;
    if (h.metric == 1) {  // metric_scores normalises the query once (hnsw.mojo:4542-4544)
        if (ensure(ctx->scratch, qb) != 0)
            return set_error(ctx, PION_B200_ENOMEM, "hnsw_metric_scores: scratch");
        float* qn = static_cast<float*>(ctx->scratch.ptr);
        rc = launch_l2_normalize_rows(dq, nq, dim, qn, nullptr, st);
        ctx->launches++;
        qsrc = qn;
    }
    if (!rc)
        rc = launch_hnsw_metric(qsrc, (int)nq, (int)k, di, h.ext_to_node, h.ext_base,
                                h.ext_count, h.node_slot, h.codes, h.gmin, h.gmax,
                                h.metric == 1, ix->kind == kHNSWQuant ? h.rerank_node : nullptr,
                                ds, st);
    ctx->launches++;
    if (rc) return set_error(ctx, rc, "hnsw_metric_scores: launch failed");
    if (mem == PION_B200_MEM_HOST) {
        if (cudaMemcpyAsync(scores, ds, rb, cudaMemcpyDeviceToHost, st) != cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "hnsw_metric_scores: result copy failed");
        return finish_sync(ctx);
    }
    return 0;
}

int pion_v_b200_hnsw_last_stats(pion_b200_ctx* ctx, int64_t* out3) {
    if (!valid_ctx(ctx) || !out3) return PION_B200_EINVAL;
    out3[0] = out3[1] = out3[2] = 0;
    if (!ctx->hnsw_misc.ptr) return 0;
    if (int rc = use_device(ctx)) return rc;
    unsigned long long v[3];
    if (cudaMemcpyAsync(v, ctx->hnsw_misc.ptr, sizeof(v), cudaMemcpyDeviceToHost, ctx->stream) !=
            cudaSuccess ||
        cudaStreamSynchronize(ctx->stream) != cudaSuccess)
        return set_error(ctx, PION_B200_ECUDA, "hnsw_last_stats: copy failed");
    for (int i = 0; i < 3; ++i) out3[i] = (int64_t)v[i];
    return 0;
}

}  // extern "C"

// ------------------------------------------------------ visited bitmaps

// Per resident warp: the touched-word list of the beam kernel (words a query turned
// non-zero, zeroed again when it ends).  16,384 entries cover ~500K visited nodes'
// words; a query past that zeroes its whole bitmap.
constexpr int kTouchCap = 16384;

int pion::hnsw_visit_buffers(pion_b200_ctx* ctx, int64_t warps, int64_t num_nodes,
                             HnswLaunch& L) {
    const int64_t vis_words = ((num_nodes + 31) / 32 + 3) / 4 * 4;
    void* before = ctx->hnsw_visited.ptr;
    if (ensure(ctx->hnsw_visited, (size_t)warps * vis_words * 4) != 0 ||
        ensure(ctx->hnsw_touched, (size_t)warps * kTouchCap * 4) != 0)
        return PION_B200_ENOMEM;
    if (ctx->hnsw_visited.ptr != before || !ctx->vis_clean) {
        // new memory, or left non-zero by another kernel: zero it once; the beam kernel
        // leaves it zero after every query
        if (cudaMemsetAsync(ctx->hnsw_visited.ptr, 0, ctx->hnsw_visited.bytes, ctx->stream) !=
            cudaSuccess)
            return PION_B200_ECUDA;
        ctx->vis_clean = true;
    }
    L.visited = static_cast<uint32_t*>(ctx->hnsw_visited.ptr);
    L.vis_words = vis_words;
    L.touched = static_cast<uint32_t*>(ctx->hnsw_touched.ptr);
    L.touch_cap = kTouchCap;
    // test hook: a smaller list, so that queries overflow it and zero their whole bitmap
    if (const char* e = getenv("PION_B200_TOUCH_CAP")) {
        const int c = atoi(e);
        if (c >= 32 && c < kTouchCap) L.touch_cap = c;
    }
    return 0;
}

extern "C" {

// ------------------------------------------------- pion_v_beam_1536 (compat)

namespace {

// Level-0 graphs registered by pion_v_beam_1536, keyed by the host buffers of the view.
struct BeamGraph {
    const uint32_t* l0c;
    const uint32_t* l0s;
    const int8_t* comp;
    int64_t n, stride, hdr;
    int device;
    uint64_t fp;  // content fingerprint of the three host tables when copied
    int8_t* codes = nullptr;
    float* norms = nullptr;
    uint32_t* l0_compact = nullptr;
    uint32_t* l0_slots = nullptr;
};
std::mutex g_beam_mu;
std::vector<BeamGraph*> g_beam_graphs;

void free_beam_graph(BeamGraph* g) {
    cudaSetDevice(g->device);
    cudaDeviceSynchronize();
    void* ps[] = {g->codes, g->norms, g->l0_compact, g->l0_slots};
    for (void* p : ps)
        if (p) cudaFree(p);
    delete g;
}

int beam_fail(const char* what) {
    fprintf(stderr, "pion_vector_b200: pion_v_beam_1536: %s\n", what);
    return -1;
}

uint64_t beam_fingerprint(const pion_beam_view_1536* v) {
    uint64_t h = 0xcbf29ce484222325ull;
    h = sample_rows_hash(h, v->l0_compact, v->num_nodes, 33 * 4, 33 * 4);
    h = sample_rows_hash(h, v->l0_slots, v->num_nodes, 33 * 4, 33 * 4);
    return sample_rows_hash(h, v->compact_buffer, v->num_nodes, v->compact_stride, 256);
}

// The registered copy of the view's graph (copied and checked on first use).  The copy
// is keyed by the view's host pointers and sizes AND a fingerprint of sampled rows of
// the three tables, so a different graph the engine placed at the same addresses is
// copied again instead of served from the stale copy.
BeamGraph* beam_graph(pion_b200_ctx* ctx, const pion_beam_view_1536* v, const char** why) {
    std::lock_guard<std::mutex> lock(g_beam_mu);
    const uint64_t fp = beam_fingerprint(v);
    for (size_t i = 0; i < g_beam_graphs.size(); ++i) {
        BeamGraph* g = g_beam_graphs[i];
        if (g->l0c == v->l0_compact && g->l0s == v->l0_slots && g->comp == v->compact_buffer &&
            g->n == v->num_nodes && g->stride == v->compact_stride && g->hdr == v->compact_hdr &&
            g->device == ctx->device) {
            if (g->fp == fp) return g;
            free_beam_graph(g);  // same addresses, other content: drop the stale copy
            g_beam_graphs.erase(g_beam_graphs.begin() + (ptrdiff_t)i);
            break;
        }
    }
    const int64_t n = v->num_nodes;
    if (v->compact_hdr != 8 || v->compact_stride % 16 != 0 ||
        v->compact_stride < v->compact_hdr + hnsw_dim() + 8) {
        *why = "compact layout must have an 8-byte header and a 16-byte multiple stride";
        return nullptr;
    }
    for (int64_t i = 0; i < n; ++i) {  // the slots the beam will read stay in bounds
        const uint32_t* row = v->l0_compact + i * 33;
        const uint32_t c = row[0] < 32 ? row[0] : 32;
        for (uint32_t k = 0; k < c; ++k)
            if (row[1 + k] < (uint32_t)n && v->l0_slots[i * 33 + 1 + k] >= (uint32_t)n) {
                *why = "an l0_slots entry is out of range";
                return nullptr;
            }
    }
    BeamGraph* g = new (std::nothrow) BeamGraph{v->l0_compact, v->l0_slots, v->compact_buffer, n,
                                                v->compact_stride, v->compact_hdr, ctx->device,
                                                fp};
    if (!g) {
        *why = "out of host memory";
        return nullptr;
    }
    int8_t* slots = nullptr;
    int rc = upload(&slots, v->compact_buffer, (size_t)n * v->compact_stride);
    if (!rc && (cudaMalloc(&g->codes, (size_t)n * hnsw_dim()) != cudaSuccess ||
                cudaMalloc(&g->norms, (size_t)n * sizeof(float)) != cudaSuccess)) {
        cudaGetLastError();
        rc = PION_B200_ENOMEM;
    }
    if (!rc)
        rc = launch_hnsw_relayout(slots, n, v->compact_stride, v->compact_hdr, g->codes, g->norms,
                                  ctx->stream);
    if (!rc && cudaStreamSynchronize(ctx->stream) != cudaSuccess) rc = PION_B200_ECUDA;
    if (slots) cudaFree(slots);
    if (!rc) rc = upload(&g->l0_compact, v->l0_compact, (size_t)n * 33);
    if (!rc) rc = upload(&g->l0_slots, v->l0_slots, (size_t)n * 33);
    if (rc) {
        free_beam_graph(g);
        *why = "device copy of the graph failed";
        return nullptr;
    }
    g_beam_graphs.push_back(g);
    return g;
}

}  // namespace

int64_t pion_v_beam_1536(pion_beam_view_1536* v) {
    if (!v || !v->pool || !v->pool->entries || !v->query_int8 || !v->l0_compact ||
        !v->l0_slots || !v->compact_buffer || v->num_nodes <= 0 || v->num_nodes >= 0x7fffffff)
        return beam_fail("bad view");
    const int64_t ef = v->ef < 1 ? 1 : v->ef;
    if (ef > 1024) return beam_fail("ef > 1024");
    pion_linear_pool* pool = v->pool;
    if (pool->size < 0 || pool->size > ef || pool->cursor < 0) return beam_fail("bad pool");
    pion_b200_ctx* ctx = compat_default_ctx("pion_v_beam_1536");
    if (!ctx) return -1;
    if (use_device(ctx) != 0) return beam_fail("cannot select the device");
    const char* why = "";
    BeamGraph* g = beam_graph(ctx, v, &why);
    if (!g) return beam_fail(why);
    cudaStream_t st = ctx->stream;
    const int dim = hnsw_dim();
    const size_t del_bytes = v->deleted ? (size_t)(v->num_nodes + 7) / 8 : 0;
    const size_t o_q = 0, o_pool = align_up(dim, 256), o_size = o_pool + align_up(ef * 8, 256),
                 o_del = o_size + 256, total = o_del + align_up(del_bytes, 256) + 256;
    if (ensure(ctx->stage_in, total) != 0 || ensure(ctx->hnsw_misc, 64) != 0)
        return beam_fail("out of device memory");
    char* base = static_cast<char*>(ctx->stage_in.ptr);
    // o_size: {size out, size in, cursor in, query norm}
    int32_t meta[4] = {0, (int32_t)pool->size,
                       (int32_t)(pool->cursor < pool->size ? pool->cursor : pool->size), 0};
    memcpy(&meta[3], &v->query_norm_sq, 4);
    if (cudaMemcpyAsync(base + o_q, v->query_int8, dim, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(base + o_size, meta, sizeof(meta), cudaMemcpyHostToDevice, st) !=
            cudaSuccess ||
        (pool->size > 0 && cudaMemcpyAsync(base + o_pool, pool->entries, (size_t)pool->size * 8,
                                           cudaMemcpyHostToDevice, st) != cudaSuccess) ||
        (del_bytes && cudaMemcpyAsync(base + o_del, v->deleted, del_bytes, cudaMemcpyHostToDevice,
                                      st) != cudaSuccess) ||
        cudaMemsetAsync(ctx->hnsw_misc.ptr, 0, 32, st) != cudaSuccess)
        return beam_fail("copy to the device failed");
    const int warps = hnsw_warps_per_cta();
    HnswLaunch Lc;
    if (hnsw_visit_buffers(ctx, warps, v->num_nodes, Lc) != 0)
        return beam_fail("out of device memory");
    if (hnsw_ctas_per_sm((int)ef) <= 0) return beam_fail("ef does not fit");
    unsigned long long* stats = static_cast<unsigned long long*>(ctx->hnsw_misc.ptr);
    Lc.codes = g->codes;
    Lc.norms = g->norms;
    Lc.l0_compact = g->l0_compact;
    Lc.l0_slots = g->l0_slots;
    Lc.deleted = del_bytes ? reinterpret_cast<const uint8_t*>(base + o_del) : nullptr;
    Lc.num_nodes = v->num_nodes;
    Lc.qcodes = reinterpret_cast<const int8_t*>(base + o_q);
    Lc.qblk = reinterpret_cast<const int32_t*>(base + o_size);  // unused when starting from a pool
    Lc.nq = 1;
    Lc.k = 0;
    Lc.ef = (int)ef;
    Lc.stats = stats;
    Lc.next_query = reinterpret_cast<unsigned*>(stats + 3);
    Lc.status = call_status(ctx, PION_B200_MEM_HOST);
    Lc.ctas = 1;
    Lc.pool_io = base + o_pool;
    Lc.pool_stride = ef;
    Lc.pool_size = reinterpret_cast<const int*>(base + o_size) + 1;
    Lc.pool_cursor = reinterpret_cast<const int*>(base + o_size) + 2;
    Lc.qn_given = reinterpret_cast<const float*>(base + o_size) + 3;
    Lc.pool_size_out = reinterpret_cast<int*>(base + o_size);
    int rc = launch_hnsw_beam(Lc, st);
    ctx->launches++;
    if (rc != 0) return beam_fail("launch failed");
    int out_size = 0;
    if (cudaMemcpyAsync(&out_size, base + o_size, sizeof(int), cudaMemcpyDeviceToHost, st) !=
            cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return beam_fail("copy from the device failed");
    if (out_size < 0 || out_size > ef) return beam_fail("bad pool size from the device");
    if (out_size > 0 && cudaMemcpy(pool->entries, base + o_pool, (size_t)out_size * 8,
                                   cudaMemcpyDeviceToHost) != cudaSuccess)
        return beam_fail("copy from the device failed");
    if (finish_sync(ctx) != 0) return beam_fail(pion_v_b200_last_error(ctx));
    pool->size = out_size;
    pool->cursor = out_size;
    return 0;
}

int pion_v_b200_beam_forget(const uint32_t* l0_compact) {
    quant_beam_forget(l0_compact);
    std::lock_guard<std::mutex> lock(g_beam_mu);
    std::vector<BeamGraph*> keep;
    for (BeamGraph* g : g_beam_graphs) {
        if (!l0_compact || g->l0c == l0_compact)
            free_beam_graph(g);
        else
            keep.push_back(g);
    }
    g_beam_graphs.swap(keep);
    return 0;
}

}  // extern "C"
