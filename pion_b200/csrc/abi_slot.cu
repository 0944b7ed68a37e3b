// C-ABI entry points of the GPU brute-force scan over a registered HNSW graph's slot
// buffer: the batched form of pion_metal_search_topk_w (src/ffi/metal_wrap.m:495-580),
// the FP32 rerank rows of pion_metal_register_rerank_buffer (:674-711), and the whole of
// search_gpu_brute_force (src/vector/hnsw.mojo:3916-3992).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>

#include "internal.h"

using namespace pion;

namespace {

constexpr int kCap = 512;      // candidates kept per (query, split) and stage
constexpr int kLocalKMax = 64;  // largest k with the per-list k-th filter in the kernel

// candidates kept per list (a list is one half of every tile of a split)
int cap_for(int k) { return k <= 16 ? kCap / 2 : (k <= 32 ? kCap : 2 * kCap); }

// PION_B200_SLOT_EXACT=1 sends every query through the exact CUDA-core scan (tests).
int force_exact() {
    const char* e = getenv("PION_B200_SLOT_EXACT");
    return e && atoi(e) != 0 ? 1 : 0;
}

struct Stage {
    int begin, end, splits;
};

// The first slots go through the exact loop from dense distance rows (no lists); their
// k-th smallest bounds everything after.  4096 slots: longer prefixes cut the candidate
// lists but cost more than they save (measured on 512K slots, 1024 queries, k 10 / 20).
// PION_B200_SLOT_PREFIX=<slots> overrides the size (tests of the list stages).
int64_t prefix_rows(int64_t nq, int64_t n_scan) {
    (void)nq;
    const int64_t tr = slot_tile_rows();
    int64_t r = 4096;
    if (const char* e = getenv("PION_B200_SLOT_PREFIX")) {
        const long long v = atoll(e);
        if (v > 0) r = (v + tr - 1) / tr * tr;
    }
    const int64_t all = (n_scan + tr - 1) / tr * tr;
    return r < all ? r : all;
}

// List stages over tiles [first, n_tiles), each bounded by the loop's worst after the
// previous ones.  k <= 64: one stage; the kernel keeps each list's own k-th smallest
// candidate (about k (1 + ln(L / k)) candidates for a list of L slots, in any slot
// order) and chains thresholds from split to split.  k > 64: stages 16x longer than
// everything before them; a stage of T tiles after B tiles passes about k * T / B slots
// per query; splits keep a list's share at a quarter of its capacity.
int plan_stages(int n_tiles, int first, int n_qt, int k, int num_sms, Stage* st) {
    int ns = 0;
    if (first >= n_tiles) return 0;
    if (k <= kLocalKMax) {
        const int s = fi8_choose_splits(n_qt, n_tiles - first, num_sms);
        st[ns++] = {first, n_tiles, s < n_tiles - first ? s : n_tiles - first};
        return ns;
    }
    int e = first;
    while (e < n_tiles) {
        const int b = e;
        e = (int64_t)b * 16 < n_tiles ? b * 16 : n_tiles;
        const int tiles = e - b;
        int s = fi8_choose_splits(n_qt, tiles, num_sms);
        const int64_t expect = (int64_t)k * tiles / b + 1;
        const int need = (int)((4 * expect + cap_for(k) - 1) / cap_for(k));
        s = s > need ? s : need;
        s = s < tiles ? s : tiles;
        st[ns++] = {b, e, s < 1 ? 1 : s};
    }
    return ns;
}

struct ScanState {
    float* qnorm;
    float* st_d;
    int32_t* st_i;
    float* st_worst;
    int* st_widx;
    int* qflag;
    int* flags;
    float* cand_d;
    int32_t* cand_i;
    int* cand_n;
    float* pub;
    int* status = nullptr;  // the call's status word (call_status)
};

// Bytes of scratch the scan needs after `off`, and the plan.
size_t scan_layout(size_t off, int64_t nq, int keff, int max_splits, ScanState* S, char* base) {
    auto take = [&](size_t bytes) {
        size_t o = off;
        off += align_up(bytes, 256);
        return o;
    };
    const size_t cand_e = (size_t)nq * max_splits * 2 * cap_for(keff);
    const size_t o_qn = take((size_t)nq * 4), o_sd = take((size_t)nq * keff * 4),
                 o_si = take((size_t)nq * keff * 4), o_sw = take((size_t)nq * 4),
                 o_sx = take((size_t)nq * 4), o_qf = take((size_t)nq * 4),
                 o_fl = take((size_t)(nq + 1) * 4), o_cd = take(cand_e * 4),
                 o_ci = take(cand_e * 4), o_cn = take((size_t)nq * max_splits * 2 * 4),
                 o_pb = take((size_t)nq * max_splits * 2 * 4);
    if (base) {
        S->qnorm = reinterpret_cast<float*>(base + o_qn);
        S->st_d = reinterpret_cast<float*>(base + o_sd);
        S->st_i = reinterpret_cast<int32_t*>(base + o_si);
        S->st_worst = reinterpret_cast<float*>(base + o_sw);
        S->st_widx = reinterpret_cast<int*>(base + o_sx);
        S->qflag = reinterpret_cast<int*>(base + o_qf);
        S->flags = reinterpret_cast<int*>(base + o_fl);
        S->cand_d = reinterpret_cast<float*>(base + o_cd);
        S->cand_i = reinterpret_cast<int32_t*>(base + o_ci);
        S->cand_n = reinterpret_cast<int*>(base + o_cn);
        S->pub = reinterpret_cast<float*>(base + o_pb);
    }
    return off;
}

int max_splits_of(const Stage* stages, int ns) {
    int m = 1;
    for (int s = 0; s < ns; ++s) m = stages[s].splits > m ? stages[s].splits : m;
    return m;
}

// The exact path for the nf queued queries, 128 at a time: their codes packed, then per
// chunk of 2^18 slots the tensor-core kernel writes all their distances and a warp per
// query runs them through the loop; the last chunk leaves the state in S.
int run_dense(pion_b200_ctx* ctx, const pion_b200_index* ix, const int8_t* codes, int nf,
              int64_t n_scan, int keff, const ScanState& S) {
    cudaStream_t st = ctx->stream;
    const auto& h = ix->hnsw;
    const int G = slot_query_tile();
    const int64_t tr = slot_tile_rows();
    int64_t clen = (int64_t)1 << 18;
    if (clen > (n_scan + tr - 1) / tr * tr) clen = (n_scan + tr - 1) / tr * tr;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off += align_up(bytes, 256);
        return o;
    };
    const size_t o_fc = take((size_t)G * hnsw_dim()), o_fq = take((size_t)G * 4),
                 o_nd = take(4), o_fd = take((size_t)G * keff * 4),
                 o_fi = take((size_t)G * keff * 4), o_fw = take((size_t)G * 4),
                 o_fx = take((size_t)G * 4), o_dn = take((size_t)G * clen * 4);
    if (ensure(ctx->scratch2, off) != 0) return PION_B200_ENOMEM;
    char* b = static_cast<char*>(ctx->scratch2.ptr);
    int8_t* fcodes = reinterpret_cast<int8_t*>(b + o_fc);
    float* fqn = reinterpret_cast<float*>(b + o_fq);
    int* n_dense = reinterpret_cast<int*>(b + o_nd);
    float* fd = reinterpret_cast<float*>(b + o_fd);
    int32_t* fi = reinterpret_cast<int32_t*>(b + o_fi);
    float* fworst = reinterpret_cast<float*>(b + o_fw);
    int* fwidx = reinterpret_cast<int*>(b + o_fx);
    float* dense = reinterpret_cast<float*>(b + o_dn);
    CUtensorMap tmap_f;
    if (make_tmap_2d(&tmap_f, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, fcodes, (uint64_t)hnsw_dim(),
                     (uint64_t)G, (uint64_t)hnsw_dim(), (uint32_t)slot_k_block(),
                     (uint32_t)G, CU_TENSOR_MAP_SWIZZLE_128B) != 0)
        return PION_B200_ECUDA;
    int rc = 0;
    for (int first = 0; first < nf && rc == 0; first += G) {
        const int count = nf - first < G ? nf - first : G;
        rc = launch_slot_gather(codes, S.qnorm, S.flags, first, count, keff, fcodes, fqn, n_dense,
                                fd, fi, fworst, fwidx, st);
        ctx->launches++;
        for (int64_t base = 0; base < n_scan && rc == 0; base += clen) {
            const int64_t len = n_scan - base < clen ? n_scan - base : clen;
            SlotTcLaunch L;
            L.tmap_q = &tmap_f;
            L.tmap_rows = &ix->tmap_rows;
            L.chunk_vmin = h.chunk_vmin;
            L.k = keff;
            L.qnorm = fqn;
            L.vnorm = h.norms;
            L.n_rows = n_scan;
            L.nq = count;
            L.tile_begin = (int)(base / tr);
            L.tile_end = (int)((base + len + tr - 1) / tr);
            const int tiles = L.tile_end - L.tile_begin;
            L.n_splits = tiles < ctx->num_sms ? tiles : ctx->num_sms;
            L.status = S.status;
            L.dense = dense;
            L.dense_base = base;
            L.dense_ld = clen;
            L.n_dense = n_dense;
            rc = launch_slot_tc(L, st);
            ctx->launches++;
            if (rc == 0)
                rc = launch_slot_dense_replay(dense, clen, base, len, n_dense, count, keff, fd, fi,
                                              fworst, fwidx, base + len >= n_scan, S.flags, first,
                                              S.st_d, S.st_i, S.st_worst, S.st_widx, nullptr, st);
            ctx->launches++;
        }
    }
    return rc;
}

// The worst-replace loop over slots [0, n_scan) for nq device query codes, leaving the
// loop's entries in S (keff of them per query).
int run_scan(pion_b200_ctx* ctx, const pion_b200_index* ix, const int8_t* codes,
             const float* qnorm_in, int nq, int64_t n_scan, int keff, const Stage* stages, int ns,
             const ScanState& S) {
    cudaStream_t st = ctx->stream;
    const auto& h = ix->hnsw;
    // bytes [32, 48) of the context's counters: slots replayed
    // (pion_v_b200_slot_last_stats)
    if (ensure(ctx->hnsw_misc, 64) != 0) return PION_B200_ENOMEM;
    unsigned long long* counters =
        reinterpret_cast<unsigned long long*>(static_cast<char*>(ctx->hnsw_misc.ptr) + 32);
    if (cudaMemsetAsync(counters, 0, 16, st) != cudaSuccess) return PION_B200_ECUDA;
    int rc = launch_slot_prep(codes, qnorm_in, nq, keff, S.qnorm, S.st_d, S.st_i, S.st_worst,
                              S.st_widx, S.qflag, S.flags, force_exact(), st);
    ctx->launches++;
    CUtensorMap tmap_q;
    if (rc == 0 && make_tmap_2d(&tmap_q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, codes,
                                (uint64_t)hnsw_dim(), (uint64_t)nq, (uint64_t)hnsw_dim(),
                                (uint32_t)slot_k_block(), (uint32_t)slot_query_tile(),
                                CU_TENSOR_MAP_SWIZZLE_128B) != 0)
        rc = PION_B200_ECUDA;
    timing_begin(ctx);
    // the prefix: dense distance rows of every query, then the exact loop over them
    const int64_t pre = prefix_rows(nq, n_scan);
    if (rc == 0) {
        const int64_t tr = slot_tile_rows();
        if (ensure(ctx->scratch2, (size_t)nq * pre * 4) != 0) rc = PION_B200_ENOMEM;
        float* dense = static_cast<float*>(ctx->scratch2.ptr);
        SlotTcLaunch L;
        L.tmap_q = &tmap_q;
        L.tmap_rows = &ix->tmap_rows;
        L.chunk_vmin = h.chunk_vmin;
        L.k = keff;
        L.qnorm = S.qnorm;
        L.vnorm = h.norms;
        L.n_rows = n_scan;
        L.nq = nq;
        L.tile_begin = 0;
        L.tile_end = (int)(pre / tr);
        const int n_qt = (nq + slot_query_tile() - 1) / slot_query_tile();
        int sp = (ctx->num_sms + n_qt - 1) / n_qt;
        L.n_splits = sp < L.tile_end ? sp : L.tile_end;
        L.status = S.status;
        L.dense = dense;
        L.dense_base = 0;
        L.dense_ld = pre;
        if (rc == 0) rc = launch_slot_tc(L, st);
        ctx->launches++;
        if (rc == 0)
            rc = launch_slot_dense_replay(dense, pre, 0, pre < n_scan ? pre : n_scan, nullptr, nq,
                                          keff, S.st_d, S.st_i, S.st_worst, S.st_widx, 0,
                                          nullptr, 0, nullptr, nullptr, nullptr, nullptr, S.qflag,
                                          st);
        ctx->launches++;
    }
    for (int s = 0; s < ns && rc == 0; ++s) {
        SlotTcLaunch L;
        L.tmap_q = &tmap_q;
        L.tmap_rows = &ix->tmap_rows;
        L.chunk_vmin = h.chunk_vmin;
        L.k = keff;
        L.bound = S.st_worst;
        L.qnorm = S.qnorm;
        L.vnorm = h.norms;
        L.n_rows = n_scan;
        L.nq = nq;
        L.tile_begin = stages[s].begin;
        L.tile_end = stages[s].end;
        L.n_splits = stages[s].splits;
        L.cap = cap_for(keff);
        L.cand_d = S.cand_d;
        L.cand_i = S.cand_i;
        L.cand_n = S.cand_n;
        L.status = S.status;
        if (keff <= kLocalKMax) {  // thresholds start "none" (0x7f7f7f7f = 3.4e38)
            L.pub = S.pub;
            if (cudaMemsetAsync(S.pub, 0x7f, (size_t)nq * stages[s].splits * 2 * 4, st) !=
                cudaSuccess)
                rc = PION_B200_ECUDA;
        }
        if (rc == 0) rc = launch_slot_tc(L, st);
        ctx->launches++;
        if (rc == 0)
            rc = launch_slot_replay(S.cand_d, S.cand_i, S.cand_n, stages[s].splits,
                                    cap_for(keff), nq, keff,
                                    S.st_d, S.st_i, S.st_worst, S.st_widx, S.qflag, S.flags,
                                    counters, st);
        ctx->launches++;
    }
    timing_end(ctx);
    // queries whose lists overflowed (or all, when forced): the exact loop over every slot
    int nf = 0;
    if (rc == 0 && (cudaMemcpyAsync(&nf, S.flags, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
                    cudaStreamSynchronize(st) != cudaSuccess))
        rc = PION_B200_ECUDA;
    ctx->slot_exact = nf;
    if (rc == 0 && nf > 0) rc = run_dense(ctx, ix, codes, nf, n_scan, keff, S);
    return rc;
}

const char* check_index(const pion_b200_ctx* ctx, const pion_b200_index* ix) {
    if (!ix || ix->kind != kHNSW) return "not an HNSW index";
    if (ix->device != ctx->device) return "index on another device";
    if (ix->n_rows > 0 && !ix->has_tmap) return "index has no slot codes";
    return nullptr;
}

}  // namespace

extern "C" {

int pion_v_b200_slot_scan_topk(pion_b200_ctx* ctx, const pion_b200_index* ix,
                               const int8_t* q_codes, const float* q_norm, int64_t nq,
                               int64_t num_vectors, int64_t k, int32_t* out_slots,
                               float* out_dists, int mem) {
    if (!valid_ctx(ctx)) return PION_B200_EINVAL;
    if (const char* why = check_index(ctx, ix))
        return set_error(ctx, PION_B200_EINVAL, "slot_scan_topk: %s", why);
    if (nq < 0 || k < 1 || (nq > 0 && (!q_codes || !out_slots || !out_dists)))
        return set_error(ctx, PION_B200_EINVAL, "slot_scan_topk: bad arguments");
    if (k > slot_kmax())
        return set_error(ctx, PION_B200_ESHAPE, "slot_scan_topk: k %lld > %d", (long long)k,
                         slot_kmax());
    if (nq > (1 << 20))
        return set_error(ctx, PION_B200_ESHAPE, "slot_scan_topk: batch too large");
    if (mem != PION_B200_MEM_HOST && mem != PION_B200_MEM_DEVICE)
        return set_error(ctx, PION_B200_EINVAL, "slot_scan_topk: bad mem %d", mem);
    if (nq == 0) return 0;
    if (int rc = use_device(ctx)) return rc;
    cudaStream_t st = ctx->stream;
    const int dim = hnsw_dim();
    // the registered slots bound the scan, and the scan bounds k (metal_wrap.m:519,560)
    int64_t n_scan = num_vectors < ix->n_rows ? num_vectors : ix->n_rows;
    if (n_scan < 0) n_scan = 0;
    const int keff = (int)(k < n_scan ? k : n_scan);
    const size_t out_bytes = (size_t)nq * k * 4;
    const int8_t* dc = q_codes;
    const float* dn = q_norm;
    int32_t* ds = out_slots;
    float* dd = out_dists;
    if (mem == PION_B200_MEM_HOST) {
        const size_t cb = align_up((size_t)nq * dim, 256);
        if (ensure(ctx->stage_in, cb + (size_t)nq * 4) != 0 ||
            ensure(ctx->stage_out, 2 * align_up(out_bytes, 256)) != 0)
            return set_error(ctx, PION_B200_ENOMEM, "slot_scan_topk: staging");
        char* in = static_cast<char*>(ctx->stage_in.ptr);
        if (cudaMemcpyAsync(in, q_codes, (size_t)nq * dim, cudaMemcpyHostToDevice, st) !=
                cudaSuccess ||
            (q_norm && cudaMemcpyAsync(in + cb, q_norm, (size_t)nq * 4, cudaMemcpyHostToDevice,
                                       st) != cudaSuccess))
            return set_error(ctx, PION_B200_ECUDA, "slot_scan_topk: query copy failed");
        dc = reinterpret_cast<const int8_t*>(in);
        dn = q_norm ? reinterpret_cast<const float*>(in + cb) : nullptr;
        ds = static_cast<int32_t*>(ctx->stage_out.ptr);
        dd = reinterpret_cast<float*>(static_cast<char*>(ctx->stage_out.ptr) +
                                      align_up(out_bytes, 256));
    }
    int rc = 0;
    if (keff == 0) {
        rc = launch_fill_results(dd, ds, (size_t)nq * k, INFINITY, st);
        ctx->launches++;
    } else {
        const int n_tiles = (int)((n_scan + slot_tile_rows() - 1) / slot_tile_rows());
        const int n_qt = (int)((nq + slot_query_tile() - 1) / slot_query_tile());
        Stage stages[16];
        const int first = (int)(prefix_rows(nq, n_scan) / slot_tile_rows());
        const int ns = plan_stages(n_tiles, first, n_qt, keff, ctx->num_sms, stages);
        const int ms = max_splits_of(stages, ns);
        ScanState S;
        const size_t need = scan_layout(0, nq, keff, ms, &S, nullptr);
        if (ensure(ctx->scratch, need) != 0)
            return set_error(ctx, PION_B200_ENOMEM, "slot_scan_topk: scratch");
        scan_layout(0, nq, keff, ms, &S, static_cast<char*>(ctx->scratch.ptr));
        S.status = call_status(ctx, mem);
        rc = run_scan(ctx, ix, dc, dn, (int)nq, n_scan, keff, stages, ns, S);
        if (rc == 0) {
            rc = launch_slot_emit(S.st_d, S.st_i, (int)nq, keff, (int)k, ds, dd, st);
            ctx->launches++;
        }
    }
    if (rc != 0)
        return set_error(ctx, rc, "slot_scan_topk: launch failed: %s",
                         cudaGetErrorString(cudaGetLastError()));
    if (mem == PION_B200_MEM_HOST) {
        if (cudaMemcpyAsync(out_slots, ds, out_bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaMemcpyAsync(out_dists, dd, out_bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "slot_scan_topk: result copy failed");
        return finish_sync(ctx);
    }
    return 0;
}

int pion_v_b200_hnsw_set_rerank_rows(pion_b200_ctx* ctx, pion_b200_index* ix, const float* rows,
                                     int64_t n, int64_t dim, int mem) {
    if (!valid_ctx(ctx)) return PION_B200_EINVAL;
    if (const char* why = check_index(ctx, ix))
        return set_error(ctx, PION_B200_EINVAL, "hnsw_set_rerank_rows: %s", why);
    if (mem != PION_B200_MEM_HOST && mem != PION_B200_MEM_DEVICE)
        return set_error(ctx, PION_B200_EINVAL, "hnsw_set_rerank_rows: bad mem %d", mem);
    if (int rc = use_device(ctx)) return rc;
    if (ix->hnsw.rerank) {  // pion_metal_unregister_rerank_buffer
        cudaStreamSynchronize(ctx->stream);
        cudaFree(ix->hnsw.rerank);
        ix->hnsw.rerank = nullptr;
    }
    if (!rows) return 0;
    if (n != ix->n_rows || dim != hnsw_dim())
        return set_error(ctx, PION_B200_ESHAPE,
                         "hnsw_set_rerank_rows: %lld x %lld rows for %lld slots of dim %d",
                         (long long)n, (long long)dim, (long long)ix->n_rows, hnsw_dim());
    const size_t bytes = (size_t)n * dim * 4;
    if (bytes == 0) return 0;
    if (cudaMalloc(&ix->hnsw.rerank, bytes) != cudaSuccess) {
        cudaGetLastError();
        ix->hnsw.rerank = nullptr;
        return set_error(ctx, PION_B200_ENOMEM, "hnsw_set_rerank_rows: %zu bytes", bytes);
    }
    if (cudaMemcpyAsync(ix->hnsw.rerank, rows, bytes,
                        mem == PION_B200_MEM_HOST ? cudaMemcpyHostToDevice
                                                  : cudaMemcpyDeviceToDevice,
                        ctx->stream) != cudaSuccess ||
        cudaStreamSynchronize(ctx->stream) != cudaSuccess) {
        cudaFree(ix->hnsw.rerank);
        ix->hnsw.rerank = nullptr;
        return set_error(ctx, PION_B200_ECUDA, "hnsw_set_rerank_rows: copy failed");
    }
    return 0;
}

int pion_v_b200_hnsw_brute_force(pion_b200_ctx* ctx, const pion_b200_index* ix, const float* q,
                                 int64_t nq, int64_t k, int32_t* out_ids, float* out_scores,
                                 int32_t* out_found, int mem) {
    if (!valid_ctx(ctx)) return PION_B200_EINVAL;
    if (const char* why = check_index(ctx, ix))
        return set_error(ctx, PION_B200_EINVAL, "hnsw_brute_force: %s", why);
    if (nq < 0 || k < 1 || (nq > 0 && (!q || !out_ids || !out_scores || !out_found)))
        return set_error(ctx, PION_B200_EINVAL, "hnsw_brute_force: bad arguments");
    if (nq > (1 << 20) || k > (1 << 16))
        return set_error(ctx, PION_B200_ESHAPE, "hnsw_brute_force: batch or k too large");
    if (mem != PION_B200_MEM_HOST && mem != PION_B200_MEM_DEVICE)
        return set_error(ctx, PION_B200_EINVAL, "hnsw_brute_force: bad mem %d", mem);
    if (nq == 0) return 0;
    if (int rc = use_device(ctx)) return rc;
    cudaStream_t st = ctx->stream;
    const int dim = hnsw_dim();
    const auto& h = ix->hnsw;
    const int64_t n = ix->n_rows;
    // hnsw.mojo:3930-3935: rerank rows oversample 2x, at most 256 entries
    const int64_t final_k = k < n ? k : n;
    int64_t over = h.rerank ? 2 * final_k : final_k;
    if (h.rerank && over > n) over = n;
    if (over > slot_kmax()) over = slot_kmax();
    const int keff = (int)over;
    const size_t qb = (size_t)nq * dim * 4, out_bytes = (size_t)nq * k * 4;
    const float* dq = q;
    int32_t* di = out_ids;
    float* dv = out_scores;
    int32_t* df = out_found;
    if (mem == PION_B200_MEM_HOST) {
        if (ensure(ctx->stage_in, qb) != 0 ||
            ensure(ctx->stage_out, 2 * align_up(out_bytes, 256) + (size_t)nq * 4) != 0)
            return set_error(ctx, PION_B200_ENOMEM, "hnsw_brute_force: staging");
        if (cudaMemcpyAsync(ctx->stage_in.ptr, q, qb, cudaMemcpyHostToDevice, st) != cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "hnsw_brute_force: query copy failed");
        dq = static_cast<const float*>(ctx->stage_in.ptr);
        char* o = static_cast<char*>(ctx->stage_out.ptr);
        di = reinterpret_cast<int32_t*>(o);
        dv = reinterpret_cast<float*>(o + align_up(out_bytes, 256));
        df = reinterpret_cast<int32_t*>(o + 2 * align_up(out_bytes, 256));
    }
    int rc = 0;
    if (keff == 0) {
        rc = launch_fill_results(dv, di, (size_t)nq * k, INFINITY, st);
        if (rc == 0 && cudaMemsetAsync(df, 0, (size_t)nq * 4, st) != cudaSuccess)
            rc = PION_B200_ECUDA;
        ctx->launches++;
    } else {
        const int n_tiles = (int)((n + slot_tile_rows() - 1) / slot_tile_rows());
        const int n_qt = (int)((nq + slot_query_tile() - 1) / slot_query_tile());
        Stage stages[16];
        const int first = (int)(prefix_rows(nq, n) / slot_tile_rows());
        const int ns = plan_stages(n_tiles, first, n_qt, keff, ctx->num_sms, stages);
        const int ms = max_splits_of(stages, ns);
        size_t off = 0;
        const size_t o_qn = off;
        off += align_up(h.metric == 1 ? qb : 0, 256);
        const size_t o_codes = off;
        off += align_up((size_t)nq * dim, 256);
        const size_t o_blk = off;
        off += align_up((size_t)nq * 8 * 4, 256);
        ScanState S;
        const size_t need = scan_layout(off, nq, keff, ms, &S, nullptr);
        if (ensure(ctx->scratch, need) != 0)
            return set_error(ctx, PION_B200_ENOMEM, "hnsw_brute_force: scratch");
        char* base = static_cast<char*>(ctx->scratch.ptr);
        scan_layout(off, nq, keff, ms, &S, base);
        S.status = call_status(ctx, mem);
        const float* qsrc = dq;
        if (h.metric == 1) {  // _quantize_query_to_int8 normalises once (hnsw.mojo:669-671)
            float* qn = reinterpret_cast<float*>(base + o_qn);
            rc = launch_l2_normalize_rows(dq, nq, dim, qn, nullptr, st);
            ctx->launches++;
            qsrc = qn;
        }
        float range = h.gmax - h.gmin;
        if (range <= 0.0f) range = 1.0f;
        int8_t* codes = reinterpret_cast<int8_t*>(base + o_codes);
        if (rc == 0)
            rc = launch_hnsw_quantize(qsrc, (int)nq, h.gmin, 254.0f / range, codes,
                                      reinterpret_cast<int32_t*>(base + o_blk), st);
        ctx->launches++;
        if (rc == 0) rc = run_scan(ctx, ix, codes, nullptr, (int)nq, n, keff, stages, ns, S);
        if (rc == 0) {
            rc = launch_slot_finish(S.st_d, S.st_i, (int)nq, keff, dq, h.rerank, h.slot_ext, n,
                                    (int)final_k, (int)k, di, dv, df, st);
            ctx->launches++;
        }
    }
    if (rc != 0)
        return set_error(ctx, rc, "hnsw_brute_force: launch failed: %s",
                         cudaGetErrorString(cudaGetLastError()));
    if (mem == PION_B200_MEM_HOST) {
        if (cudaMemcpyAsync(out_ids, di, out_bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaMemcpyAsync(out_scores, dv, out_bytes, cudaMemcpyDeviceToHost, st) !=
                cudaSuccess ||
            cudaMemcpyAsync(out_found, df, (size_t)nq * 4, cudaMemcpyDeviceToHost, st) !=
                cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "hnsw_brute_force: result copy failed");
        return finish_sync(ctx);
    }
    return 0;
}

int pion_v_b200_slot_last_stats(pion_b200_ctx* ctx, int64_t* out2) {
    if (!valid_ctx(ctx) || !out2) return PION_B200_EINVAL;
    out2[0] = out2[1] = 0;
    if (!ctx->hnsw_misc.ptr) return 0;
    if (int rc = use_device(ctx)) return rc;
    unsigned long long v[2];
    if (cudaMemcpyAsync(v, static_cast<char*>(ctx->hnsw_misc.ptr) + 32, sizeof(v),
                        cudaMemcpyDeviceToHost, ctx->stream) != cudaSuccess ||
        cudaStreamSynchronize(ctx->stream) != cudaSuccess)
        return set_error(ctx, PION_B200_ECUDA, "slot_last_stats: copy failed");
    out2[0] = ctx->slot_exact;
    out2[1] = (int64_t)v[1];
    return 0;
}

}  // extern "C"
