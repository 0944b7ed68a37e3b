// C-ABI entry points of the FLAT FP32 cosine path (exact_knn under COSINE,
// src/commands/vector.mojo:1228-1365) and the row normaliser of COSINE ingest
// (l2_normalize_fp32, src/vector/kernels.mojo:318-357).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <new>

#include "internal.h"

using namespace pion;

// PION_B200_F32_EXACT=1 sends every query through the exact CUDA-core scan (tests).
// Forced path selection for tests: 0 auto (one query: the exact stream), 1 the exact
// stream for every query, 2 the tensor-core shortlist.
static int forced_f32_path() {
    const char* e = getenv("PION_B200_F32_PATH");
    return e ? atoi(e) : 0;
}

static int force_exact_f32() {
    const char* e = getenv("PION_B200_F32_EXACT");
    return e && atoi(e) != 0 ? 1 : 0;
}

extern "C" {

int pion_v_b200_l2_normalize_rows(pion_b200_ctx* ctx, const float* src, int64_t n_rows,
                                  int64_t dim, float* dst, int mem) {
    if (!valid_ctx(ctx)) return PION_B200_EINVAL;
    if (n_rows < 0 || dim <= 0 || dim > (1 << 20) || (n_rows > 0 && (!src || !dst)))
        return set_error(ctx, PION_B200_EINVAL, "l2_normalize_rows: bad arguments");
    if (n_rows == 0) return 0;
    if (int rc = use_device(ctx)) return rc;
    cudaStream_t st = ctx->stream;
    const size_t bytes = (size_t)n_rows * dim * 4;
    const float* ds = src;
    float* dd = dst;
    if (mem == PION_B200_MEM_HOST) {
        if (ensure(ctx->stage_in, bytes) != 0)
            return set_error(ctx, PION_B200_ENOMEM, "l2_normalize_rows: staging");
        if (cudaMemcpyAsync(ctx->stage_in.ptr, src, bytes, cudaMemcpyHostToDevice, st) !=
            cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "l2_normalize_rows: copy failed");
        ds = dd = static_cast<float*>(ctx->stage_in.ptr);
    } else if (mem != PION_B200_MEM_DEVICE) {
        return set_error(ctx, PION_B200_EINVAL, "l2_normalize_rows: bad mem %d", mem);
    }
    int rc = launch_l2_normalize_rows(ds, n_rows, (int)dim, dd, nullptr, st);
    ctx->launches++;
    if (rc != 0) return set_error(ctx, rc, "l2_normalize_rows: launch failed");
    if (mem == PION_B200_MEM_HOST) {
        if (cudaMemcpyAsync(dst, dd, bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "l2_normalize_rows: copy back failed");
        return finish_sync(ctx);
    }
    return 0;
}

int pion_v_b200_register_flat_f32(pion_b200_ctx* ctx, const float* rows, int64_t n_rows,
                                  int64_t dim, int64_t id_base, int normalize, int mem,
                                  pion_b200_index** out_index) {
    if (!valid_ctx(ctx) || !out_index) return PION_B200_EINVAL;
    *out_index = nullptr;
    if (n_rows < 0 || (n_rows > 0 && !rows))
        return set_error(ctx, PION_B200_EINVAL, "register_flat_f32: null rows");
    if (dim <= 0 || dim % 8 != 0 || dim > 16384)
        return set_error(ctx, PION_B200_ESHAPE, "register_flat_f32: dim %lld must be a multiple "
                         "of 8 in [8, 16384]", (long long)dim);
    if (n_rows > INT32_MAX - 1 || id_base < 0 || id_base + n_rows > INT32_MAX)
        return set_error(ctx, PION_B200_ESHAPE, "register_flat_f32: ids must fit int32");
    if (mem == PION_B200_MEM_DEVICE_BORROW && normalize)
        return set_error(ctx, PION_B200_EINVAL, "register_flat_f32: a borrowed buffer cannot "
                         "be normalised in place");
    if (mem != PION_B200_MEM_HOST && mem != PION_B200_MEM_DEVICE && mem != PION_B200_MEM_DEVICE_BORROW)
        return set_error(ctx, PION_B200_EINVAL, "register_flat_f32: bad mem %d", mem);
    if (int rc = use_device(ctx)) return rc;
    cudaStream_t st = ctx->stream;
    pion_b200_index* ix = new (std::nothrow) pion_b200_index();
    if (!ix) return PION_B200_ENOMEM;
    ix->kind = kFlatF32;
    ix->device = ctx->device;
    ix->n_rows = n_rows;
    ix->dim = dim;
    ix->id_base = id_base;
    const size_t bytes = (size_t)n_rows * dim * 4;
    if (mem == PION_B200_MEM_DEVICE_BORROW) {
        ix->owns = false;
        ix->rows_f32 = const_cast<float*>(rows);
    } else {
        if (cudaMalloc(&ix->rows_f32, bytes ? bytes : 16) != cudaSuccess) {
            cudaGetLastError();
            pion_v_b200_index_free(ix);
            return set_error(ctx, PION_B200_ENOMEM, "register_flat_f32: %zu bytes", bytes);
        }
        if (n_rows > 0 && cudaMemcpyAsync(ix->rows_f32, rows, bytes,
                                          mem == PION_B200_MEM_HOST ? cudaMemcpyHostToDevice
                                                                    : cudaMemcpyDeviceToDevice,
                                          st) != cudaSuccess) {
            pion_v_b200_index_free(ix);
            return set_error(ctx, PION_B200_ECUDA, "register_flat_f32: copy failed");
        }
    }
    if ((reinterpret_cast<uintptr_t>(ix->rows_f32) & 15u) != 0) {
        pion_v_b200_index_free(ix);
        return set_error(ctx, PION_B200_EINVAL, "register_flat_f32: rows not 16-byte aligned");
    }
    if (n_rows > 0) {
        int rc = 0;
        if (normalize) {
            rc = launch_l2_normalize_rows(ix->rows_f32, n_rows, (int)dim, ix->rows_f32, nullptr,
                                          st);
            ctx->launches++;
        }
        // largest row norm, for the TF32 error bound of the certificate
        float* norms = nullptr;
        if (rc == 0 && cudaMalloc(&norms, (size_t)n_rows * 4 + 256) != cudaSuccess) {
            cudaGetLastError();
            rc = PION_B200_ENOMEM;
        }
        if (rc == 0) rc = launch_row_norms(ix->rows_f32, n_rows, (int)dim, norms, st);
        float* dmax = norms ? reinterpret_cast<float*>(reinterpret_cast<char*>(norms) +
                                                       align_up((size_t)n_rows * 4, 128))
                            : nullptr;
        if (rc == 0) rc = launch_max_reduce(norms, n_rows, dmax, st);
        if (rc == 0 && (cudaMemcpyAsync(&ix->row_norm_max, dmax, 4, cudaMemcpyDeviceToHost, st) !=
                            cudaSuccess ||
                        cudaStreamSynchronize(st) != cudaSuccess))
            rc = PION_B200_ECUDA;
        ctx->launches += 2;
        if (norms) cudaFree(norms);
        // bf16 split of the stored rows for the tensor-core shortlist
        const size_t half_bytes = (size_t)n_rows * dim * 2;
        if (rc == 0 && (cudaMalloc(&ix->rows_hi, half_bytes) != cudaSuccess ||
                        cudaMalloc(&ix->rows_lo, half_bytes) != cudaSuccess)) {
            cudaGetLastError();
            rc = PION_B200_ENOMEM;
        }
        if (rc == 0) {
            rc = launch_split_bf16(ix->rows_f32, (size_t)n_rows * dim, ix->rows_hi, ix->rows_lo,
                                   st);
            ctx->launches++;
        }
        if (rc == 0 && (make_tmap_2d(&ix->tmap_rows, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                                     ix->rows_hi, (uint64_t)dim, (uint64_t)n_rows,
                                     (uint64_t)dim * 2, (uint32_t)ff32_k_elems(),
                                     (uint32_t)ff32_tile_rows(), CU_TENSOR_MAP_SWIZZLE_128B) != 0 ||
                        make_tmap_2d(&ix->tmap_rows_lo, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                                     ix->rows_lo, (uint64_t)dim, (uint64_t)n_rows,
                                     (uint64_t)dim * 2, (uint32_t)ff32_k_elems(),
                                     (uint32_t)ff32_tile_rows(), CU_TENSOR_MAP_SWIZZLE_128B) != 0))
            rc = PION_B200_ECUDA;
        if (rc != 0) {
            pion_v_b200_index_free(ix);
            return set_error(ctx, rc, "register_flat_f32: preparation failed");
        }
        ix->has_tmap = true;
    }
    if (cudaStreamSynchronize(st) != cudaSuccess) {
        pion_v_b200_index_free(ix);
        return set_error(ctx, PION_B200_ECUDA, "register_flat_f32: stream failed");
    }
    *out_index = ix;
    return 0;
}

int pion_v_b200_flat_f32_knn(pion_b200_ctx* ctx, const pion_b200_index* ix, const float* q,
                             int64_t nq, int64_t k, int32_t* out_ids, float* out_scores, int mem) {
    if (!valid_ctx(ctx)) return PION_B200_EINVAL;
    if (!ix || ix->kind != kFlatF32)
        return set_error(ctx, PION_B200_EINVAL, "flat_f32_knn: not a FLAT FP32 index");
    if (ix->device != ctx->device)
        return set_error(ctx, PION_B200_EINVAL, "flat_f32_knn: index on another device");
    if (nq < 0 || k < 1 || (nq > 0 && (!q || !out_ids || !out_scores)))
        return set_error(ctx, PION_B200_EINVAL, "flat_f32_knn: bad arguments");
    if (k > 64) return set_error(ctx, PION_B200_ESHAPE, "flat_f32_knn: k %lld > 64", (long long)k);
    if (nq > (1 << 24)) return set_error(ctx, PION_B200_ESHAPE, "flat_f32_knn: batch too large");
    if (mem != PION_B200_MEM_HOST && mem != PION_B200_MEM_DEVICE)
        return set_error(ctx, PION_B200_EINVAL, "flat_f32_knn: bad mem %d", mem);
    if (nq == 0) return 0;
    if (int rc = use_device(ctx)) return rc;
    cudaStream_t st = ctx->stream;
    const int dim = (int)ix->dim;
    const int kk = (int)k;
    const int nqi = (int)nq;
    const size_t qbytes = align_up((size_t)nq * dim * 4, 256);
    const size_t out_bytes = (size_t)nq * kk * 4;

    const float* dq = q;
    int32_t* di = out_ids;
    float* dv = out_scores;
    if (mem == PION_B200_MEM_HOST) {
        if (ensure(ctx->stage_in, qbytes) != 0 ||
            ensure(ctx->stage_out, 2 * align_up(out_bytes, 256)) != 0)
            return set_error(ctx, PION_B200_ENOMEM, "flat_f32_knn: staging");
        if (cudaMemcpyAsync(ctx->stage_in.ptr, q, (size_t)nq * dim * 4, cudaMemcpyHostToDevice,
                            st) != cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "flat_f32_knn: query copy failed");
        dq = static_cast<const float*>(ctx->stage_in.ptr);
        di = static_cast<int32_t*>(ctx->stage_out.ptr);
        dv = reinterpret_cast<float*>(static_cast<char*>(ctx->stage_out.ptr) +
                                      align_up(out_bytes, 256));
    }
    int rc = 0;
    const int path = forced_f32_path();
    const bool scan1 = ix->n_rows > 0 && ff32_scan1_supported(dim, kk) &&
                       (path == 1 || (path == 0 && nq == 1));
    if (ix->n_rows == 0) {
        rc = launch_fill_results(dv, di, (size_t)nq * kk, INFINITY, st);
        ctx->launches++;
    } else if (scan1) {
        // One query (or forced): an exact HBM stream per query, no tensor-core shortlist.
        const int ctas = ff32_scan1_ctas(ix->n_rows, ctx->num_sms);
        const size_t n_qn = (size_t)nq * dim, n_cand = (size_t)nq * ctas * kk;
        const size_t o_qn = 0, o_qnorm = align_up(n_qn * 4, 256),
                     o_cv = o_qnorm + align_up((size_t)nq * 4, 256),
                     o_ci = o_cv + align_up(n_cand * 4, 256), total = o_ci + n_cand * 4;
        if (ensure(ctx->scratch, total) != 0)
            return set_error(ctx, PION_B200_ENOMEM, "flat_f32_knn: scratch");
        char* base = static_cast<char*>(ctx->scratch.ptr);
        float* qn = reinterpret_cast<float*>(base + o_qn);
        float* cv = reinterpret_cast<float*>(base + o_cv);
        int32_t* ci = reinterpret_cast<int32_t*>(base + o_ci);
        const int t_all = timing_begin(ctx);
        rc = launch_query_normalize(dq, nqi, dim, qn, reinterpret_cast<float*>(base + o_qnorm),
                                    st);
        ctx->launches++;
        for (int64_t t = 0; t < nq && rc == 0; ++t) {
            rc = launch_flat_f32_scan1(ix->rows_f32, ix->n_rows, dim, qn + (size_t)t * dim, kk,
                                       ctas, cv + (size_t)t * ctas * kk,
                                       ci + (size_t)t * ctas * kk, st);
            ctx->launches++;
        }
        timing_end(ctx, t_all);
        if (rc == 0) {
            rc = launch_merge_lists(cv, ci, nqi, ctas, kk, ix->id_base, false, dv, di, st);
            ctx->launches++;
        }
    } else {
        const int kc = ff32_kc(kk);
        const int n_qt = (nqi + ff32_query_tile() - 1) / ff32_query_tile();
        const int n_tiles = (int)((ix->n_rows + ff32_tile_rows() - 1) / ff32_tile_rows());
        // Threshold pass over a sample of the first tiles (one approximate dot per 32-row
        // chunk): the KC-th best is a lower bound of the final KC-th approximate dot, and
        // the main pass starts from it and scores every tile.
        const bool pre = use_prepass(n_tiles, kc, "PION_B200_F32_PREPASS");
        const int pre_tiles = pre ? bound_tiles(n_tiles, kc) : 0;
        const int splits = fi8_choose_splits(n_qt, n_tiles, ctx->num_sms);
        const int n_lists = splits;
        int bnd_splits = pre ? ctx->num_sms / n_qt : 0;
        if (pre) bnd_splits = bnd_splits < 1 ? 1 : (bnd_splits > pre_tiles ? pre_tiles : bnd_splits);
        const int chunks = ff32_exact_chunks();
        // scratch layout (floats / ints)
        const size_t n_qn = (size_t)nq * dim;
        const size_t n_cand = (size_t)nq * n_lists * kc;
        const size_t n_bnd = (size_t)nq * bnd_splits * kc;
        const size_t n_thr = (size_t)nq * kc;
        const size_t n_merged = (size_t)nq * kc;
        const size_t n_chunk = (size_t)nq * chunks * kk;
        size_t off = 0;
        auto take = [&](size_t elems) {
            size_t o = off;
            off += align_up(elems * 4, 256);
            return o;
        };
        const size_t o_qn = take(n_qn), o_qh = take(n_qn / 2 + 1), o_ql = take(n_qn / 2 + 1),
                     o_qnorm = take(nq), o_cv = take(n_cand),
                     o_ci = take(n_cand), o_sv = take(n_bnd), o_si = take(n_bnd),
                     o_pv = take(n_thr), o_pi = take(n_thr), o_mv = take(n_merged),
                     o_mi = take(n_merged), o_flag = take(nq + 1), o_chd = take(n_chunk),
                     o_chi = take(n_chunk);
        if (ensure(ctx->scratch, off) != 0)
            return set_error(ctx, PION_B200_ENOMEM, "flat_f32_knn: scratch");
        char* base = static_cast<char*>(ctx->scratch.ptr);
        float* qn = reinterpret_cast<float*>(base + o_qn);
        float* qnorm = reinterpret_cast<float*>(base + o_qnorm);
        void* qh = base + o_qh;
        void* ql = base + o_ql;
        float* cv = reinterpret_cast<float*>(base + o_cv);
        int32_t* ci = reinterpret_cast<int32_t*>(base + o_ci);
        float* sv = reinterpret_cast<float*>(base + o_sv);
        int32_t* si = reinterpret_cast<int32_t*>(base + o_si);
        float* pv = reinterpret_cast<float*>(base + o_pv);
        int32_t* pi = reinterpret_cast<int32_t*>(base + o_pi);
        float* mv = reinterpret_cast<float*>(base + o_mv);
        int32_t* mi = reinterpret_cast<int32_t*>(base + o_mi);
        int* flags = reinterpret_cast<int*>(base + o_flag);  // [0] = count, then query ids
        float* chd = reinterpret_cast<float*>(base + o_chd);
        int32_t* chi = reinterpret_cast<int32_t*>(base + o_chi);

        timing_begin(ctx);
        rc = launch_query_normalize(dq, nqi, dim, qn, qnorm, st);
        ctx->launches++;
        if (rc == 0) {
            rc = launch_split_bf16(qn, (size_t)nq * dim, qh, ql, st);
            ctx->launches++;
        }
        CUtensorMap tmap_qh, tmap_ql;
        if (rc == 0 && (make_tmap_2d(&tmap_qh, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, qh,
                                     (uint64_t)dim, (uint64_t)nq, (uint64_t)dim * 2,
                                     (uint32_t)ff32_k_elems(), (uint32_t)ff32_query_tile(),
                                     CU_TENSOR_MAP_SWIZZLE_128B) != 0 ||
                        make_tmap_2d(&tmap_ql, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ql,
                                     (uint64_t)dim, (uint64_t)nq, (uint64_t)dim * 2,
                                     (uint32_t)ff32_k_elems(), (uint32_t)ff32_query_tile(),
                                     CU_TENSOR_MAP_SWIZZLE_128B) != 0))
            rc = PION_B200_ECUDA;
        Ff32TcLaunch L;
        L.tmap_qh = &tmap_qh;
        L.tmap_ql = &tmap_ql;
        L.tmap_rh = &ix->tmap_rows;
        L.tmap_rl = &ix->tmap_rows_lo;
        L.n_rows = ix->n_rows;
        L.nq = nqi;
        L.dim = dim;
        L.kc = kc;
        L.status = call_status(ctx, mem);
        if (rc == 0 && pre) {
            L.tile_begin = 0;
            L.tile_end = pre_tiles;
            L.n_splits = bnd_splits;
            L.n_lists = bnd_splits;
            L.cand_val = sv;
            L.cand_idx = si;
            L.thr0 = nullptr;
            L.bound_mode = 1;
            rc = launch_flat_bf16x3_tc(L, st);
            ctx->launches++;
            if (rc == 0) {
                rc = launch_merge_lists(sv, si, nqi, bnd_splits, kc, 0, true, pv, pi, st);
                ctx->launches++;
            }
        }
        if (rc == 0) {
            L.tile_begin = 0;
            L.tile_end = n_tiles;
            L.n_splits = splits;
            L.n_lists = n_lists;
            L.cand_val = cv;
            L.cand_idx = ci;
            L.thr0 = pre ? pv + (kc - 1) : nullptr;
            L.thr0_stride = kc;
            L.bound_mode = 0;
            rc = launch_flat_bf16x3_tc(L, st);
            ctx->launches++;
        }
        timing_end(ctx);
        if (rc == 0) {
            rc = launch_merge_lists(cv, ci, nqi, n_lists, kc, 0, true, mv, mi, st);
            ctx->launches++;
        }
        if (rc == 0 && cudaMemsetAsync(flags, 0, sizeof(int), st) != cudaSuccess)
            rc = PION_B200_ECUDA;
        if (rc == 0) {
            rc = launch_rescore_certify(ix->rows_f32, dim, qn, qnorm, ix->row_norm_max, mv, mi,
                                        nqi, kc, kk, ix->id_base, dv, di, flags + 1, flags,
                                        force_exact_f32(), st);
            ctx->launches++;
        }
        if (rc == 0) {
            rc = launch_exact_fallback(ix->rows_f32, ix->n_rows, dim, qn, flags + 1, flags, nqi,
                                       kk, ix->id_base, chd, chi, dv, di, ctx->num_sms, st);
            ctx->launches += 2;
        }
    }
    if (rc != 0)
        return set_error(ctx, rc, "flat_f32_knn: launch failed: %s",
                         cudaGetErrorString(cudaGetLastError()));
    if (mem == PION_B200_MEM_HOST) {
        if (cudaMemcpyAsync(out_ids, di, out_bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaMemcpyAsync(out_scores, dv, out_bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "flat_f32_knn: result copy failed");
        return finish_sync(ctx);
    }
    return 0;
}

int pion_v_b200_merge_delta(pion_b200_ctx* ctx, const pion_b200_index* ix, int64_t built,
                            int metric, const float* q, int64_t nq, int64_t kg, int32_t* ids,
                            float* scores, int64_t k, int32_t* out_ids, float* out_scores,
                            int mem) {
    if (!valid_ctx(ctx)) return PION_B200_EINVAL;
    if (!ix || ix->kind != kFlatF32)
        return set_error(ctx, PION_B200_EINVAL, "merge_delta: not a FLAT FP32 index of the rows");
    if (ix->device != ctx->device)
        return set_error(ctx, PION_B200_EINVAL, "merge_delta: index on another device");
    if (ix->id_base != 0)
        return set_error(ctx, PION_B200_EINVAL, "merge_delta: the rows index must start at slot 0");
    if (nq < 0 || kg < 1 || k < 1 || built < 0 || (metric != 0 && metric != 1) ||
        (nq > 0 && (!q || !ids || !scores || !out_ids || !out_scores)))
        return set_error(ctx, PION_B200_EINVAL, "merge_delta: bad arguments");
    if (kg > delta_kg_max() || k > 64 || nq > (1 << 22))
        return set_error(ctx, PION_B200_ESHAPE, "merge_delta: kg %lld or k %lld too large",
                         (long long)kg, (long long)k);
    if (mem != PION_B200_MEM_HOST && mem != PION_B200_MEM_DEVICE)
        return set_error(ctx, PION_B200_EINVAL, "merge_delta: bad mem %d", mem);
    if (nq == 0) return 0;
    if (int rc = use_device(ctx)) return rc;
    cudaStream_t st = ctx->stream;
    const int dim = (int)ix->dim;
    const int64_t n_rows = ix->n_rows;
    const int64_t b = built < n_rows ? built : n_rows;
    const size_t qb = (size_t)nq * dim * 4, gb = (size_t)nq * kg * 4, ob = (size_t)nq * k * 4;
    const float* dq = q;
    int32_t* dgi = ids;
    float* dgs = scores;
    int32_t* doi = out_ids;
    float* dos = out_scores;
    if (mem == PION_B200_MEM_HOST) {
        if (ensure(ctx->stage_in, align_up(qb, 256)) != 0 ||
            ensure(ctx->stage_out, 2 * align_up(gb, 256) + 2 * align_up(ob, 256)) != 0)
            return set_error(ctx, PION_B200_ENOMEM, "merge_delta: staging");
        char* o = static_cast<char*>(ctx->stage_out.ptr);
        dq = static_cast<const float*>(ctx->stage_in.ptr);
        dgi = reinterpret_cast<int32_t*>(o);
        dgs = reinterpret_cast<float*>(o + align_up(gb, 256));
        doi = reinterpret_cast<int32_t*>(o + 2 * align_up(gb, 256));
        dos = reinterpret_cast<float*>(o + 2 * align_up(gb, 256) + align_up(ob, 256));
        if (cudaMemcpyAsync(const_cast<float*>(dq), q, qb, cudaMemcpyHostToDevice, st) !=
                cudaSuccess ||
            cudaMemcpyAsync(dgi, ids, gb, cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(dgs, scores, gb, cudaMemcpyHostToDevice, st) != cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "merge_delta: copy failed");
    }
    const int chunks = ff32_exact_chunks();
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off += align_up(bytes, 256);
        return o;
    };
    const size_t o_q = take(qb), o_qn = take((size_t)nq * 4), o_ng = take((size_t)nq * 4),
                 o_fl = take((size_t)(nq + 1) * 4),
                 o_cd = take((size_t)nq * chunks * k * 4), o_ci = take((size_t)nq * chunks * k * 4),
                 o_dd = take(ob), o_di = take(ob);
    if (ensure(ctx->scratch, off) != 0)
        return set_error(ctx, PION_B200_ENOMEM, "merge_delta: scratch");
    char* base = static_cast<char*>(ctx->scratch.ptr);
    const float* qx = dq;
    int rc = 0;
    if (metric == 1) {  // exact_knn / _exact_rescore normalise the query (vector.mojo:1254)
        rc = launch_query_normalize(dq, (int)nq, dim, reinterpret_cast<float*>(base + o_q),
                                    reinterpret_cast<float*>(base + o_qn), st);
        ctx->launches++;
        qx = reinterpret_cast<const float*>(base + o_q);
    }
    int* n_graph = reinterpret_cast<int*>(base + o_ng);
    int32_t* ddi = reinterpret_cast<int32_t*>(base + o_di);
    float* dds = reinterpret_cast<float*>(base + o_dd);
    timing_begin(ctx);
    if (rc == 0) {
        rc = launch_delta_rescore(ix->rows_f32, dim, b, metric == 0, qx, (int)nq, (int)kg, dgi,
                                  dgs, n_graph, st);
        ctx->launches++;
    }
    if (rc == 0) {
        if (n_rows > b) {  // exact_knn over the rows ingested since the build
            rc = launch_exact_scan_all(ix->rows_f32 + (size_t)b * dim, n_rows - b, dim, qx,
                                       (int)nq, (int)k, b, metric == 0,
                                       reinterpret_cast<int*>(base + o_fl),
                                       reinterpret_cast<float*>(base + o_cd),
                                       reinterpret_cast<int32_t*>(base + o_ci), dds, ddi,
                                       ctx->num_sms, st);
            ctx->launches += 3;
        } else {
            rc = launch_fill_results(dds, ddi, (size_t)nq * k, INFINITY, st);
            ctx->launches++;
        }
    }
    if (rc == 0) {
        rc = launch_delta_merge(dgi, dgs, n_graph, (int)kg, ddi, dds, (int)k, (int)nq, (int)k,
                                doi, dos, st);
        ctx->launches++;
    }
    timing_end(ctx);
    if (rc != 0)
        return set_error(ctx, rc, "merge_delta: launch failed: %s",
                         cudaGetErrorString(cudaGetLastError()));
    if (mem == PION_B200_MEM_HOST) {
        if (cudaMemcpyAsync(ids, dgi, gb, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaMemcpyAsync(scores, dgs, gb, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaMemcpyAsync(out_ids, doi, ob, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaMemcpyAsync(out_scores, dos, ob, cudaMemcpyDeviceToHost, st) != cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "merge_delta: result copy failed");
        return finish_sync(ctx);
    }
    return 0;
}

}  // extern "C"
