// C-ABI entry points of binary-quantised FLAT with FP32 rerank: sign codes
// (src/vector/kernels.mojo:1711-1720), Hamming shortlist
// (src/vector/reference/quant_dots.mojo:95-100), exact cosine rerank
// (src/commands/vector.mojo:1413-1456).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <new>

#include "internal.h"

using namespace pion;

namespace {

// PION_B200_BQ_PATH: 0 auto (one query: the popcount stream), 1 the stream for every
// query, 2 the tensor-core stages (tests).
int forced_bq_path() {
    const char* e = getenv("PION_B200_BQ_PATH");
    return e ? atoi(e) : 0;
}

// PION_B200_BQ_RERANK=1 keeps the one-query rerank on the spread-rows kernel pair
// (tests compare it with the staged kernel).
int forced_rerank_path() {
    const char* e = getenv("PION_B200_BQ_RERANK");
    return e ? atoi(e) : 0;
}

// PION_B200_BQ_STREAM=1 keeps the one-query first pass on the register kernel (tests
// compare it with the shared-memory staged one).
int forced_stream_path() {
    const char* e = getenv("PION_B200_BQ_STREAM");
    return e ? atoi(e) : 0;
}

// PION_B200_BQ_EXACT=1 sends every query through the exact popcount scan (tests).
int force_fallback() {
    const char* e = getenv("PION_B200_BQ_EXACT");
    return e && atoi(e) != 0 ? 1 : 0;
}

// Staged shortlist plan over the index tiles: [0, t1) without a bound, [t1, t2) bounded
// by the first stage's S-th distance, [t2, n_tiles) bounded by the second's.
struct Stage {
    int begin, end, splits;
};

int plan_stages(int n_tiles, int n_qt, int num_sms, Stage* st) {
    const int t1 = n_tiles < 16 ? n_tiles : 16;
    const int t2 = n_tiles < 256 ? n_tiles : 256;
    int ns = 0;
    // one tile per split: a thread sees 128 rows, within the list capacity
    st[ns++] = {0, t1, t1};
    if (t2 > t1) {
        int s = num_sms / n_qt;
        s = s < 1 ? 1 : (s > (t2 - t1) ? (t2 - t1) : s);
        st[ns++] = {t1, t2, s};
    }
    if (n_tiles > t2) st[ns++] = {t2, n_tiles, fi8_choose_splits(n_qt, n_tiles - t2, num_sms)};
    return ns;
}

}  // namespace

extern "C" {

int pion_v_b200_register_bq(pion_b200_ctx* ctx, const float* rows, int64_t n_rows, int64_t dim,
                            int64_t id_base, int normalize, int mem, pion_b200_index** out_index) {
    if (!valid_ctx(ctx) || !out_index) return PION_B200_EINVAL;
    *out_index = nullptr;
    if (n_rows < 0 || (n_rows > 0 && !rows))
        return set_error(ctx, PION_B200_EINVAL, "register_bq: null rows");
    if (dim <= 0 || dim % 64 != 0 || dim > 16384)
        return set_error(ctx, PION_B200_ESHAPE, "register_bq: dim %lld must be a multiple of 64",
                         (long long)dim);
    if (n_rows > INT32_MAX - 1 || id_base < 0 || id_base + n_rows > INT32_MAX)
        return set_error(ctx, PION_B200_ESHAPE, "register_bq: ids must fit int32");
    if (mem != PION_B200_MEM_HOST && mem != PION_B200_MEM_DEVICE)
        return set_error(ctx, PION_B200_EINVAL, "register_bq: bad mem %d", mem);
    if (int rc = use_device(ctx)) return rc;
    cudaStream_t st = ctx->stream;
    pion_b200_index* ix = new (std::nothrow) pion_b200_index();
    if (!ix) return PION_B200_ENOMEM;
    ix->kind = kBQ;
    ix->device = ctx->device;
    ix->n_rows = n_rows;
    ix->dim = dim;
    ix->id_base = id_base;
    ix->words = dim / 64;
    const size_t fbytes = (size_t)n_rows * dim * 4;
    int rc = 0;
    if (cudaMalloc(&ix->rows_f32, fbytes ? fbytes : 16) != cudaSuccess ||
        cudaMalloc(&ix->rows_i8, (size_t)(n_rows ? n_rows : 1) * dim) != cudaSuccess ||
        cudaMalloc(&ix->codes, (size_t)(n_rows ? n_rows : 1) * ix->words * 8) != cudaSuccess) {
        cudaGetLastError();
        pion_v_b200_index_free(ix);
        return set_error(ctx, PION_B200_ENOMEM, "register_bq: %zu bytes", fbytes);
    }
    if (n_rows > 0) {
        if (cudaMemcpyAsync(ix->rows_f32, rows, fbytes,
                            mem == PION_B200_MEM_HOST ? cudaMemcpyHostToDevice
                                                      : cudaMemcpyDeviceToDevice,
                            st) != cudaSuccess)
            rc = PION_B200_ECUDA;
        if (rc == 0 && normalize) {
            rc = launch_l2_normalize_rows(ix->rows_f32, n_rows, (int)dim, ix->rows_f32, nullptr,
                                          st);
            ctx->launches++;
        }
        if (rc == 0) {
            rc = launch_signs(ix->rows_f32, n_rows, (int)dim, ix->rows_i8, ix->codes, st);
            ctx->launches++;
        }
        if (rc == 0 && make_tmap_2d(&ix->tmap_rows, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ix->rows_i8,
                                    (uint64_t)dim, (uint64_t)n_rows, (uint64_t)dim,
                                    (uint32_t)bq_k_block(), (uint32_t)bq_tile_rows(),
                                    CU_TENSOR_MAP_SWIZZLE_128B) != 0)
            rc = PION_B200_ECUDA;
        ix->has_tmap = rc == 0;
    }
    if (rc == 0 && cudaStreamSynchronize(st) != cudaSuccess) rc = PION_B200_ECUDA;
    if (rc != 0) {
        pion_v_b200_index_free(ix);
        return set_error(ctx, rc, "register_bq: preparation failed");
    }
    *out_index = ix;
    return 0;
}

int pion_v_b200_bq_rerank_knn(pion_b200_ctx* ctx, const pion_b200_index* ix, const float* q,
                              int64_t nq, int64_t shortlist, int64_t k, int32_t* out_ids,
                              float* out_scores, int mem) {
    if (!valid_ctx(ctx)) return PION_B200_EINVAL;
    if (!ix || ix->kind != kBQ)
        return set_error(ctx, PION_B200_EINVAL, "bq_rerank_knn: not a BQ index");
    if (ix->device != ctx->device)
        return set_error(ctx, PION_B200_EINVAL, "bq_rerank_knn: index on another device");
    if (nq < 0 || k < 1 || shortlist < k || (nq > 0 && (!q || !out_ids || !out_scores)))
        return set_error(ctx, PION_B200_EINVAL, "bq_rerank_knn: bad arguments");
    if (shortlist > 256)
        return set_error(ctx, PION_B200_ESHAPE, "bq_rerank_knn: shortlist %lld > 256",
                         (long long)shortlist);
    if (nq > (1 << 24)) return set_error(ctx, PION_B200_ESHAPE, "bq_rerank_knn: batch too large");
    if (mem != PION_B200_MEM_HOST && mem != PION_B200_MEM_DEVICE)
        return set_error(ctx, PION_B200_EINVAL, "bq_rerank_knn: bad mem %d", mem);
    if (nq == 0) return 0;
    if (int rc = use_device(ctx)) return rc;
    cudaStream_t st = ctx->stream;
    const int dim = (int)ix->dim;
    const int kk = (int)k, S = (int)shortlist, nqi = (int)nq;
    const int words = (int)ix->words;
    const size_t out_bytes = (size_t)nq * kk * 4;
    const float* dq = q;
    int32_t* di = out_ids;
    float* dv = out_scores;
    if (mem == PION_B200_MEM_HOST) {
        if (ensure(ctx->stage_in, (size_t)nq * dim * 4) != 0 ||
            ensure(ctx->stage_out, 2 * align_up(out_bytes, 256)) != 0)
            return set_error(ctx, PION_B200_ENOMEM, "bq_rerank_knn: staging");
        if (cudaMemcpyAsync(ctx->stage_in.ptr, q, (size_t)nq * dim * 4, cudaMemcpyHostToDevice,
                            st) != cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "bq_rerank_knn: query copy failed");
        dq = static_cast<const float*>(ctx->stage_in.ptr);
        di = static_cast<int32_t*>(ctx->stage_out.ptr);
        dv = reinterpret_cast<float*>(static_cast<char*>(ctx->stage_out.ptr) +
                                      align_up(out_bytes, 256));
    }
    int rc = 0;
    const int path = forced_bq_path();
    const int rerank_path = forced_rerank_path();
    const int stream_path = forced_stream_path();
    const bool scan1 = ix->n_rows > 0 && bq_scan1_supported(words, S) &&
                       (path == 1 || (path == 0 && nq == 1));
    if (ix->n_rows == 0) {
        rc = launch_fill_results(dv, di, (size_t)nq * kk, INFINITY, st);
        ctx->launches++;
    } else if (scan1) {
        // One query: the popcount stream over the packed codes, then the same rerank.
        const int ctas = bq_scan1_ctas(ix->n_rows, words, ctx->num_sms, stream_path);
        size_t off = 0;
        auto take = [&](size_t bytes) {
            size_t o = off;
            off += align_up(bytes, 256);
            return o;
        };
        const size_t o_qn = take((size_t)nq * dim * 4), o_qnorm = take((size_t)nq * 4),
                     o_qc = take((size_t)nq * words * 8),
                     o_slid = take((size_t)nq * S * 4), o_slh = take((size_t)nq * S * 2),
                     o_sln = take((size_t)nq * 4), o_rd = take((size_t)nq * S * 4),
                     o_done = take((size_t)nq * 4),
                     o_work = take(bq_scan1_scratch(ix->n_rows, words));
        if (ensure(ctx->scratch, off) != 0)
            return set_error(ctx, PION_B200_ENOMEM, "bq_rerank_knn: scratch");
        char* base = static_cast<char*>(ctx->scratch.ptr);
        float* qn = reinterpret_cast<float*>(base + o_qn);
        uint64_t* qc = reinterpret_cast<uint64_t*>(base + o_qc);
        int32_t* sl_id = reinterpret_cast<int32_t*>(base + o_slid);
        uint16_t* sl_h = reinterpret_cast<uint16_t*>(base + o_slh);
        int* sl_n = reinterpret_cast<int*>(base + o_sln);
        const int t_all = timing_begin(ctx);
        rc = launch_query_normalize(dq, nqi, dim, qn, reinterpret_cast<float*>(base + o_qnorm),
                                    st, nullptr, qc);
        ctx->launches++;
        for (int64_t t = 0; t < nq && rc == 0; ++t) {
            rc = launch_bq_scan1(ix->codes, ix->n_rows, words, qc + (size_t)t * words, S, ctas,
                                 base + o_work, sl_id + (size_t)t * S, sl_h + (size_t)t * S,
                                 sl_n + t, call_status(ctx, mem), ctx->wait_ns, stream_path,
                                 st);
            ctx->launches += 3;
        }
        timing_end(ctx, t_all);
        if (rc == 0) {
            if (dim % 16 == 0 && rerank_path != 1)
                rc = launch_bq_rerank_staged(ix->rows_f32, dim, qn, sl_id, sl_n, S, nqi, kk,
                                             ix->id_base, reinterpret_cast<float*>(base + o_rd),
                                             reinterpret_cast<unsigned*>(base + o_done),
                                             call_status(ctx, mem), ctx->wait_ns, dv, di, st);
            else if (dim % 16 == 0)
                rc = launch_bq_rerank_wide(ix->rows_f32, dim, qn, sl_id, sl_n, S, nqi, kk,
                                           ix->id_base, reinterpret_cast<float*>(base + o_rd),
                                           dv, di, st);
            else
                rc = launch_bq_rerank(ix->rows_f32, dim, qn, sl_id, sl_n, S, nqi, kk, ix->id_base,
                                      dv, di, st);
            ctx->launches += 2;
        }
    } else {
        const int n_qt = (nqi + bq_query_tile() - 1) / bq_query_tile();
        const int n_tiles = (int)((ix->n_rows + bq_tile_rows() - 1) / bq_tile_rows());
        const int lps = bq_lists_per_split();
        const int cap = bq_cap();
        Stage stages[3];
        const int ns = plan_stages(n_tiles, n_qt, ctx->num_sms, stages);
        int max_lists = 1;
        for (int s = 0; s < ns; ++s) {
            const int nl = stages[s].splits * lps + (s > 0 ? 1 : 0);
            max_lists = nl > max_lists ? nl : max_lists;
        }
        size_t off = 0;
        auto take = [&](size_t bytes) {
            size_t o = off;
            off += align_up(bytes, 256);
            return o;
        };
        const size_t cand_e = (size_t)nq * max_lists * cap;
        const size_t o_qn = take((size_t)nq * dim * 4), o_qnorm = take((size_t)nq * 4),
                     o_qpm = take((size_t)nq * dim), o_qc = take((size_t)nq * words * 8),
                     o_id0 = take(cand_e * 4), o_h0 = take(cand_e * 2),
                     o_n0 = take((size_t)nq * max_lists * 4), o_id1 = take(cand_e * 4),
                     o_h1 = take(cand_e * 2), o_n1 = take((size_t)nq * max_lists * 4),
                     o_dm = take((size_t)nq * 4), o_slid = take((size_t)nq * S * 4),
                     o_slh = take((size_t)nq * S * 2), o_sln = take((size_t)nq * 4),
                     o_flag = take((size_t)(nq + 1) * 4 * ns + 4);
        if (ensure(ctx->scratch, off) != 0)
            return set_error(ctx, PION_B200_ENOMEM, "bq_rerank_knn: scratch");
        char* base = static_cast<char*>(ctx->scratch.ptr);
        float* qn = reinterpret_cast<float*>(base + o_qn);
        float* qnorm = reinterpret_cast<float*>(base + o_qnorm);
        int8_t* qpm = reinterpret_cast<int8_t*>(base + o_qpm);
        uint64_t* qc = reinterpret_cast<uint64_t*>(base + o_qc);
        int32_t* cid[2] = {reinterpret_cast<int32_t*>(base + o_id0),
                           reinterpret_cast<int32_t*>(base + o_id1)};
        uint16_t* ch[2] = {reinterpret_cast<uint16_t*>(base + o_h0),
                           reinterpret_cast<uint16_t*>(base + o_h1)};
        int* cn[2] = {reinterpret_cast<int*>(base + o_n0), reinterpret_cast<int*>(base + o_n1)};
        int* dot_min = reinterpret_cast<int*>(base + o_dm);
        int32_t* sl_id = reinterpret_cast<int32_t*>(base + o_slid);
        uint16_t* sl_h = reinterpret_cast<uint16_t*>(base + o_slh);
        int* sl_n = reinterpret_cast<int*>(base + o_sln);
        int* flags = reinterpret_cast<int*>(base + o_flag);  // [0] count, then query ids
        timing_begin(ctx);
        rc = launch_query_normalize(dq, nqi, dim, qn, qnorm, st, qpm, qc);
        ctx->launches++;
        CUtensorMap tmap_q;
        if (rc == 0 && make_tmap_2d(&tmap_q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, qpm, (uint64_t)dim,
                                    (uint64_t)nq, (uint64_t)dim, (uint32_t)bq_k_block(),
                                    (uint32_t)bq_query_tile(), CU_TENSOR_MAP_SWIZZLE_128B) != 0)
            rc = PION_B200_ECUDA;
        if (rc == 0 && cudaMemsetAsync(flags, 0, 4, st) != cudaSuccess) rc = PION_B200_ECUDA;
        for (int s = 0; s < ns && rc == 0; ++s) {
            const int buf = s & 1;
            const int nl = stages[s].splits * lps + (s > 0 ? 1 : 0);
            BqTcLaunch L;
            L.tmap_q = &tmap_q;
            L.tmap_rows = &ix->tmap_rows;
            L.dot_min = s > 0 ? dot_min : nullptr;
            L.n_rows = ix->n_rows;
            L.nq = nqi;
            L.dim = dim;
            L.tile_begin = stages[s].begin;
            L.tile_end = stages[s].end;
            L.n_splits = stages[s].splits;
            L.n_lists = nl;
            L.list_base = 0;
            L.cand_id = cid[buf];
            L.cand_h = ch[buf];
            L.cand_n = cn[buf];
            L.status = call_status(ctx, mem);
            rc = launch_bq_tc(L, st);
            ctx->launches++;
            if (rc != 0) break;
            if (s + 1 < ns) {
                // this stage's shortlist becomes the last list of the next stage
                const int nb = (s + 1) & 1;
                const int nl2 = stages[s + 1].splits * lps + 1;
                rc = launch_bq_select(cid[buf], ch[buf], cn[buf], nqi, nl, dim, S,
                                      cid[nb] + (size_t)(nl2 - 1) * cap,
                                      ch[nb] + (size_t)(nl2 - 1) * cap, cn[nb] + (nl2 - 1),
                                      nl2 * cap, nl2, dot_min, flags + 1, flags, 0, st);
            } else {
                rc = launch_bq_select(cid[buf], ch[buf], cn[buf], nqi, nl, dim, S, sl_id, sl_h,
                                      sl_n, S, 1, dot_min, flags + 1, flags, force_fallback(),
                                      st);
            }
            ctx->launches++;
        }
        timing_end(ctx);
        if (rc == 0) {
            rc = launch_bq_fallback(ix->codes, ix->n_rows, words, qc, flags + 1, flags, S, sl_id,
                                    sl_h, sl_n, ctx->num_sms, st);
            ctx->launches++;
        }
        if (rc == 0) {
            rc = launch_bq_rerank(ix->rows_f32, dim, qn, sl_id, sl_n, S, nqi, kk, ix->id_base, dv,
                                  di, st);
            ctx->launches++;
        }
    }
    if (rc != 0)
        return set_error(ctx, rc, "bq_rerank_knn: launch failed: %s",
                         cudaGetErrorString(cudaGetLastError()));
    if (mem == PION_B200_MEM_HOST) {
        if (cudaMemcpyAsync(out_ids, di, out_bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaMemcpyAsync(out_scores, dv, out_bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "bq_rerank_knn: result copy failed");
        return finish_sync(ctx);
    }
    return 0;
}

}  // extern "C"
