// C-ABI layer of libpion_vector_b200: contexts, device-resident index registration
// and the batched query entry points declared in include/pion_vector_b200.h.
//
// Conventions follow the reference's CUDA shim (src/ffi/cuda_wrap.c:153-437,
// src/ffi/cuda_kernels.cu:1330-1346): int status, 0 ok, negative error, message kept
// per context (and printed to stderr for the pion_v_* group, which has no status).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <new>
#include <utility>

#include "internal.h"

namespace pion {

int set_error(pion_b200_ctx* ctx, int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    if (ctx) ctx->last_error = buf;
    return code;
}

int ensure(DevBuf& b, size_t bytes) {
    if (bytes <= b.bytes) return 0;
    size_t want = bytes + bytes / 4 + 4096;
    void* p = nullptr;
    if (cudaMalloc(&p, want) != cudaSuccess) {
        cudaGetLastError();
        return PION_B200_ENOMEM;
    }
    if (b.ptr) cudaFree(b.ptr);
    b.ptr = p;
    b.bytes = want;
    return 0;
}

int set_smem_limit(const void* kernel, int bytes) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return PION_B200_ECUDA;
    }
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, int> done;  // (kernel, device) -> bytes set
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_pair(kernel, dev);
    const auto it = done.find(key);
    if (it != done.end() && it->second >= bytes) return 0;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
        cudaSuccess) {
        cudaGetLastError();
        return PION_B200_ECUDA;
    }
    done[key] = bytes;
    return 0;
}

uint64_t sample_rows_hash(uint64_t h, const void* base, int64_t n_rows, int64_t row_bytes,
                          int64_t take_bytes) {
    if (!base || n_rows <= 0 || row_bytes <= 0) return h;
    if (take_bytes > row_bytes) take_bytes = row_bytes;
    const unsigned char* p = static_cast<const unsigned char*>(base);
    const int64_t samples = n_rows < 64 ? n_rows : 64;
    for (int64_t j = 0; j <= samples; ++j) {
        const int64_t row = j == samples ? n_rows - 1 : j * n_rows / samples;
        const unsigned char* r = p + row * row_bytes;
        int64_t b = 0;
        for (; b + 8 <= take_bytes; b += 8) {
            uint64_t w;
            memcpy(&w, r + b, 8);
            h = (h ^ w) * 0x100000001b3ull;
            h ^= h >> 29;
        }
        for (; b < take_bytes; ++b) h = (h ^ r[b]) * 0x100000001b3ull;
        h = (h ^ (uint64_t)row) * 0x9e3779b97f4a7c15ull;
    }
    return h;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// 2-D tensor map, row-major: `inner` elements per row (contiguous), `outer` rows.
// Out-of-range boxes read as zero.
int make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base,
                 uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                 uint32_t box_outer, CUtensorMapSwizzle swizzle) {
    (void)elem_bytes;
    EncodeTiledFn fn = encode_fn();
    if (!fn) return PION_B200_ECUDA;
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (row_stride_bytes & 15u) != 0)
        return PION_B200_EINVAL;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_stride_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : PION_B200_ECUDA;
}

int* call_status(pion_b200_ctx* ctx, int mem) {
    return ctx->d_status + (mem == PION_B200_MEM_HOST ? 0 : 1);
}

// Queues a copy of both status words into pinned host memory.
int queue_status_readback(pion_b200_ctx* ctx) {
    return cudaMemcpyAsync(ctx->h_status, ctx->d_status, 2 * sizeof(int), cudaMemcpyDeviceToHost,
                           ctx->stream) == cudaSuccess
               ? 0
               : PION_B200_ECUDA;
}

// Synchronises the stream, then turns a status recorded in words [first, last] into a
// code (and clears them).  Host-memory calls check word 0 only: a device-memory call's
// failure stays in word 1 for pion_v_b200_sync and is never reported as a later
// host-memory call's own.
static int sync_words(pion_b200_ctx* ctx, int first, int last) {
    if (queue_status_readback(ctx) != 0)
        return set_error(ctx, PION_B200_ECUDA, "status copy failed: %s",
                         cudaGetErrorString(cudaGetLastError()));
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess)
        return set_error(ctx, PION_B200_ECUDA, "stream failed: %s", cudaGetErrorString(e));
    for (int w = first; w <= last; ++w) {
        const int st = ctx->h_status[w];
        if (st != 0) {
            ctx->h_status[w] = 0;
            cudaMemsetAsync(ctx->d_status + w, 0, sizeof(int), ctx->stream);
            cudaStreamSynchronize(ctx->stream);
            return set_error(ctx, st, "device-side wait gave up (status %d, %s-memory call)",
                             st, w == 0 ? "host" : "device");
        }
    }
    return 0;
}

int finish_sync(pion_b200_ctx* ctx) { return sync_words(ctx, 0, 0); }

bool valid_ctx(const pion_b200_ctx* ctx) { return ctx != nullptr && ctx->d_status; }

int use_device(pion_b200_ctx* ctx) {
    if (cudaSetDevice(ctx->device) != cudaSuccess)
        return set_error(ctx, PION_B200_ENODEV, "cudaSetDevice(%d) failed", ctx->device);
    return 0;
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

int timing_begin(pion_b200_ctx* ctx, int tag) {
    if (!ctx->timing) return -1;
    if (ctx->ev_used == ctx->ev_start.size()) {
        if (ctx->ev_used >= 65536) return -1;
        cudaEvent_t a, b;
        if (cudaEventCreate(&a) != cudaSuccess) return -1;
        if (cudaEventCreate(&b) != cudaSuccess) {
            cudaEventDestroy(a);
            return -1;
        }
        ctx->ev_start.push_back(a);
        ctx->ev_end.push_back(b);
        ctx->ev_tag.push_back(0);
        ctx->ev_closed.push_back(false);
    }
    const int slot = (int)ctx->ev_used++;
    ctx->ev_tag[slot] = tag;
    ctx->ev_closed[slot] = false;
    ctx->ev_open = slot;
    cudaEventRecord(ctx->ev_start[slot], ctx->stream);
    return slot;
}

void timing_end(pion_b200_ctx* ctx, int slot) {
    if (!ctx->timing) return;
    if (slot < 0) slot = ctx->ev_open;
    if (slot < 0 || (size_t)slot >= ctx->ev_used || ctx->ev_closed[slot]) return;
    cudaEventRecord(ctx->ev_end[slot], ctx->stream);
    ctx->ev_closed[slot] = true;
}

}  // namespace pion

using namespace pion;

extern "C" {

int pion_v_b200_init(int device, int worker_id, pion_b200_ctx** out_ctx) {
    if (!out_ctx) return PION_B200_EINVAL;
    *out_ctx = nullptr;
    if (device < 0) {
        const char* env = getenv("PION_B200_DEVICE");
        device = env ? atoi(env) : 0;
    }
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device >= n) {
        cudaGetLastError();
        fprintf(stderr, "pion_vector_b200: no CUDA device %d\n", device);
        return PION_B200_ENODEV;
    }
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return PION_B200_ENODEV;
    if (prop.major != 10) {
        fprintf(stderr, "pion_vector_b200: device %d is sm_%d%d, need sm_100\n", device,
                prop.major, prop.minor);
        return PION_B200_ENODEV;
    }
    if (cudaSetDevice(device) != cudaSuccess) return PION_B200_ENODEV;
    pion_b200_ctx* ctx = new (std::nothrow) pion_b200_ctx();
    if (!ctx) return PION_B200_ENOMEM;
    ctx->device = device;
    ctx->worker_id = worker_id;
    ctx->num_sms = prop.multiProcessorCount;
    if (cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&ctx->d_status, 2 * sizeof(int)) != cudaSuccess ||
        cudaMallocHost(&ctx->h_status, 2 * sizeof(int)) != cudaSuccess) {
        pion_v_b200_shutdown(ctx);
        return PION_B200_ENOMEM;
    }
    ctx->stream = ctx->own_stream;
    ctx->h_status[0] = ctx->h_status[1] = 0;
    cudaMemset(ctx->d_status, 0, 2 * sizeof(int));
    cudaDeviceSynchronize();
    *out_ctx = ctx;
    return 0;
}

int pion_v_b200_shutdown(pion_b200_ctx* ctx) {
    if (!ctx) return PION_B200_EINVAL;
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    DevBuf* bufs[] = {&ctx->scratch,      &ctx->scratch2,     &ctx->stage_in,
                      &ctx->stage_out,    &ctx->hnsw_visited, &ctx->hnsw_misc,
                      &ctx->hnsw_touched};
    for (DevBuf* b : bufs)
        if (b->ptr) cudaFree(b->ptr);
    if (ctx->d_status) cudaFree(ctx->d_status);
    if (ctx->h_status) cudaFreeHost(ctx->h_status);
    if (ctx->switch_ev) cudaEventDestroy(ctx->switch_ev);
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    for (cudaEvent_t e : ctx->ev_start) cudaEventDestroy(e);
    for (cudaEvent_t e : ctx->ev_end) cudaEventDestroy(e);
    delete ctx;
    return 0;
}

int pion_v_b200_set_stream(pion_b200_ctx* ctx, void* cuda_stream) {
    if (!valid_ctx(ctx)) return PION_B200_EINVAL;
    cudaStream_t next = cuda_stream ? static_cast<cudaStream_t>(cuda_stream) : ctx->own_stream;
    if (next != ctx->stream) {
        // The context's scratch is shared by both streams: work queued from now on waits
        // for everything already queued on the previous stream.
        if (int rc = use_device(ctx)) return rc;
        if (!ctx->switch_ev &&
            cudaEventCreateWithFlags(&ctx->switch_ev, cudaEventDisableTiming) != cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "set_stream: event create failed");
        if (cudaEventRecord(ctx->switch_ev, ctx->stream) != cudaSuccess ||
            cudaStreamWaitEvent(next, ctx->switch_ev, 0) != cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "set_stream: stream ordering failed");
    }
    ctx->stream = next;
    return 0;
}

int pion_v_b200_set_wait_budget(pion_b200_ctx* ctx, int64_t ns) {
    if (!valid_ctx(ctx)) return PION_B200_EINVAL;
    ctx->wait_ns = ns > 0 ? (uint64_t)ns : kDefaultWaitNs;
    return 0;
}

int pion_v_b200_sync(pion_b200_ctx* ctx) {
    if (!valid_ctx(ctx)) return PION_B200_EINVAL;
    if (int rc = use_device(ctx)) return rc;
    return sync_words(ctx, 0, 1);
}

const char* pion_v_b200_last_error(const pion_b200_ctx* ctx) {
    return ctx ? ctx->last_error.c_str() : "null context";
}

int64_t pion_v_b200_launch_count(const pion_b200_ctx* ctx) { return ctx ? ctx->launches : 0; }

int pion_v_b200_timing_enable(pion_b200_ctx* ctx, int enable) {
    if (!valid_ctx(ctx)) return PION_B200_EINVAL;
    if (int rc = use_device(ctx)) return rc;
    cudaStreamSynchronize(ctx->stream);
    ctx->timing = enable != 0;
    ctx->ev_used = 0;
    ctx->ev_open = -1;
    return 0;
}

int pion_v_b200_timing_read_tag(pion_b200_ctx* ctx, int tag, double* total_ms, int64_t* count) {
    if (!valid_ctx(ctx) || !total_ms || !count) return PION_B200_EINVAL;
    if (int rc = use_device(ctx)) return rc;
    if (cudaStreamSynchronize(ctx->stream) != cudaSuccess)
        return set_error(ctx, PION_B200_ECUDA, "timing_read: stream failed");
    double sum = 0.0;
    int64_t n = 0;
    for (size_t i = 0; i < ctx->ev_used; ++i) {
        if (ctx->ev_tag[i] != tag || !ctx->ev_closed[i]) continue;
        // the events may sit on a stream other than the current one
        if (cudaEventSynchronize(ctx->ev_end[i]) != cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "timing_read: event %zu", i);
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, ctx->ev_start[i], ctx->ev_end[i]) != cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "timing_read: event %zu", i);
        sum += ms;
        ++n;
    }
    *total_ms = sum;
    *count = n;
    return 0;
}

int pion_v_b200_timing_read(pion_b200_ctx* ctx, double* total_ms, int64_t* count) {
    return pion_v_b200_timing_read_tag(ctx, PION_B200_TIMING_SCORING, total_ms, count);
}

int pion_v_b200_reserve(pion_b200_ctx* ctx, int64_t max_nq, int64_t max_k) {
    if (!valid_ctx(ctx) || max_nq < 0 || max_k < 0) return PION_B200_EINVAL;
    if (int rc = use_device(ctx)) return rc;
    const size_t lists = 64;  // upper bound on splits per query tile
    size_t cand = (size_t)max_nq * lists * (size_t)max_k * 8 + (size_t)ctx->num_sms * 8 * max_k * 8;
    if (ensure(ctx->scratch, cand) != 0)
        return set_error(ctx, PION_B200_ENOMEM, "reserve: %zu bytes", cand);
    return 0;
}

int pion_v_b200_register_index(pion_b200_ctx* ctx, const pion_b200_index_desc* d,
                               pion_b200_index** out_index) {
    if (!valid_ctx(ctx) || !out_index) return PION_B200_EINVAL;
    if (!d) return set_error(ctx, PION_B200_EINVAL, "register_index: null descriptor");
    switch (d->kind) {
        case PION_B200_KIND_FLAT_I8:
            return pion_v_b200_register_flat_i8(ctx, static_cast<const int8_t*>(d->rows),
                                                d->row_scale, d->n_rows, d->dim, d->id_base,
                                                d->mem, out_index);
        case PION_B200_KIND_FLAT_F32:
            return pion_v_b200_register_flat_f32(ctx, static_cast<const float*>(d->rows),
                                                 d->n_rows, d->dim, d->id_base, d->normalize,
                                                 d->mem, out_index);
        case PION_B200_KIND_BQ:
            return pion_v_b200_register_bq(ctx, static_cast<const float*>(d->rows), d->n_rows,
                                           d->dim, d->id_base, d->normalize, d->mem, out_index);
        case PION_B200_KIND_HNSW:
            return pion_v_b200_register_hnsw(ctx, d->hnsw, out_index);
        case PION_B200_KIND_HNSW_QUANT:
            return pion_v_b200_register_hnsw_quant(ctx, d->hnsw, d->quant, out_index);
        default:
            *out_index = nullptr;
            return set_error(ctx, PION_B200_EINVAL, "register_index: unknown kind %d", d->kind);
    }
}

int64_t pion_v_b200_index_rows(const pion_b200_index* index) { return index ? index->n_rows : -1; }

int pion_v_b200_index_free(pion_b200_index* index) {
    if (!index) return PION_B200_EINVAL;
    cudaSetDevice(index->device);
    cudaDeviceSynchronize();
    if (index->owns) {
        if (index->rows_i8) cudaFree(index->rows_i8);
        if (index->row_scale) cudaFree(index->row_scale);
        if (index->rows_f32) cudaFree(index->rows_f32);
    }
    if (index->tile_rs_max) cudaFree(index->tile_rs_max);
    if (index->rows_hi) cudaFree(index->rows_hi);
    if (index->rows_lo) cudaFree(index->rows_lo);
    if (index->codes) cudaFree(index->codes);
    void* hn[] = {index->hnsw.codes,      index->hnsw.norms,        index->hnsw.l0_compact,
                  index->hnsw.l0_slots,
                  index->hnsw.node_slot,  index->hnsw.node_ids,     index->hnsw.deleted,
                  index->hnsw.node_level, index->hnsw.upper_offset, index->hnsw.upper_links,
                  index->hnsw.upper_slots, index->hnsw.ext_to_node,
                  index->hnsw.slot_ext,   index->hnsw.rerank,       index->hnsw.chunk_vmin,
                  index->hnsw.qcodes,     index->hnsw.qscales,      index->hnsw.qjl,
                  index->hnsw.qjl_res,    index->hnsw.qjl_rs,       index->hnsw.rerank_node};
    for (void* p : hn)
        if (p) cudaFree(p);
    delete index;
    return 0;
}

// ------------------------------------------------------------------ FLAT INT8

int pion_v_b200_register_flat_i8(pion_b200_ctx* ctx, const int8_t* rows, const float* row_scale,
                                 int64_t n_rows, int64_t dim, int64_t id_base, int mem,
                                 pion_b200_index** out_index) {
    if (!valid_ctx(ctx) || !out_index) return PION_B200_EINVAL;
    *out_index = nullptr;
    if (n_rows < 0 || (n_rows > 0 && (!rows || !row_scale)))
        return set_error(ctx, PION_B200_EINVAL, "register_flat_i8: null rows");
    if (dim <= 0 || dim % 16 != 0 || dim > 16384)
        return set_error(ctx, PION_B200_ESHAPE, "register_flat_i8: dim %lld must be a multiple "
                         "of 16 in [16, 16384]", (long long)dim);
    if (n_rows > INT32_MAX - 1 || id_base < 0 || id_base + n_rows > INT32_MAX)
        return set_error(ctx, PION_B200_ESHAPE, "register_flat_i8: ids must fit int32");
    if (mem != PION_B200_MEM_HOST && mem != PION_B200_MEM_DEVICE && mem != PION_B200_MEM_DEVICE_BORROW)
        return set_error(ctx, PION_B200_EINVAL, "register_flat_i8: bad mem %d", mem);
    if (int rc = use_device(ctx)) return rc;
    pion_b200_index* ix = new (std::nothrow) pion_b200_index();
    if (!ix) return PION_B200_ENOMEM;
    ix->kind = kFlatI8;
    ix->device = ctx->device;
    ix->n_rows = n_rows;
    ix->dim = dim;
    ix->id_base = id_base;
    const size_t rbytes = (size_t)n_rows * (size_t)dim;
    const int n_tiles = (int)((n_rows + fi8_tile_rows() - 1) / fi8_tile_rows());
    if (mem == PION_B200_MEM_DEVICE_BORROW) {
        ix->owns = false;
        ix->rows_i8 = const_cast<int8_t*>(rows);
        ix->row_scale = const_cast<float*>(row_scale);
    } else {
        if (cudaMalloc(&ix->rows_i8, rbytes ? rbytes : 16) != cudaSuccess ||
            cudaMalloc(&ix->row_scale, (size_t)(n_rows ? n_rows : 1) * sizeof(float)) != cudaSuccess) {
            cudaGetLastError();
            pion_v_b200_index_free(ix);
            return set_error(ctx, PION_B200_ENOMEM, "register_flat_i8: %zu bytes", rbytes);
        }
        const cudaMemcpyKind kind =
            mem == PION_B200_MEM_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
        if (n_rows > 0 &&
            (cudaMemcpyAsync(ix->rows_i8, rows, rbytes, kind, ctx->stream) != cudaSuccess ||
             cudaMemcpyAsync(ix->row_scale, row_scale, (size_t)n_rows * 4, kind, ctx->stream) !=
                 cudaSuccess)) {
            pion_v_b200_index_free(ix);
            return set_error(ctx, PION_B200_ECUDA, "register_flat_i8: copy failed");
        }
    }
    if ((reinterpret_cast<uintptr_t>(ix->rows_i8) & 15u) != 0) {
        pion_v_b200_index_free(ix);
        return set_error(ctx, PION_B200_EINVAL, "register_flat_i8: rows not 16-byte aligned");
    }
    if (cudaMalloc(&ix->tile_rs_max, (size_t)(n_tiles > 0 ? n_tiles : 1) * sizeof(float)) !=
        cudaSuccess) {
        cudaGetLastError();
        pion_v_b200_index_free(ix);
        return set_error(ctx, PION_B200_ENOMEM, "register_flat_i8: tile maxima");
    }
    if (n_rows > 0) {
        if (launch_tile_max(ix->row_scale, n_rows, ix->tile_rs_max, ctx->stream) != 0) {
            pion_v_b200_index_free(ix);
            return set_error(ctx, PION_B200_ECUDA, "register_flat_i8: tile max launch");
        }
        ctx->launches++;
        if (make_tmap_2d(&ix->tmap_rows, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ix->rows_i8,
                         (uint64_t)dim, (uint64_t)n_rows, (uint64_t)dim, (uint32_t)fi8_k_block(),
                         (uint32_t)fi8_tile_rows(), CU_TENSOR_MAP_SWIZZLE_128B) != 0) {
            pion_v_b200_index_free(ix);
            return set_error(ctx, PION_B200_ECUDA, "register_flat_i8: tensor map");
        }
        ix->has_tmap = true;
    }
    if (cudaStreamSynchronize(ctx->stream) != cudaSuccess) {
        pion_v_b200_index_free(ix);
        return set_error(ctx, PION_B200_ECUDA, "register_flat_i8: %s",
                         cudaGetErrorString(cudaGetLastError()));
    }
    *out_index = ix;
    return 0;
}

// Test hook (PION_B200_TEST_STALL=1): one CTA of the next main passes waits on a
// barrier nothing arrives on, so the wait runs out after the context's budget and the
// call reports PION_B200_ETIMEOUT (no fault, the GPU stays usable).
static int test_stall() {
    const char* e = getenv("PION_B200_TEST_STALL");
    return e && atoi(e) == 1 ? 1 : 0;
}

// Forced path selection for tests: 0 auto, 1 one-query scan, 2 tensor-core kernel.
static int forced_i8_path() {
    const char* e = getenv("PION_B200_I8_PATH");
    return e ? atoi(e) : 0;
}

}  // extern "C"

// Index tiles scored by the threshold pre-pass: 8 tiles (2048 rows) per result
// slot, at least 64 tiles (16384 rows) -- enough that the sample's k-th score is
// close to the final one on clustered data, where a query's neighbours are a small
// fraction of the rows.
int pion::prepass_tiles(int k) { return k * 8 > 64 ? k * 8 : 64; }

// Tiles sampled by the threshold pass: about 1/6 of the index (the main pass scores
// every tile again), at least 8 and enough 32-row chunks for k candidates, at most
// prepass_tiles(k).
int pion::bound_tiles(int n_tiles, int k) {
    int t = n_tiles / 6;
    const int lo = 8 > (k + 3) / 4 ? 8 : (k + 3) / 4;
    if (t < lo) t = lo;
    const int hi = prepass_tiles(k);
    return t > hi ? hi : t;
}

// The threshold pass runs whenever the index is more than twice its sample: without a
// starting threshold every CTA's first tiles pay the full insertion cost, which measured
// twice the whole step at 125K and 250K rows as well as at 1M.  The environment variable
// `env` (PION_B200_I8_PREPASS / PION_B200_F32_PREPASS) = 0 turns it off.
bool pion::use_prepass(int n_tiles, int k, const char* env) {
    const char* e = getenv(env);
    if (e && atoi(e) == 0) return false;
    return n_tiles > 2 * bound_tiles(n_tiles, k);
}

extern "C" {

int pion_v_b200_flat_i8_knn(pion_b200_ctx* ctx, const pion_b200_index* ix, const int8_t* q,
                            const float* q_scale, int64_t nq, int64_t k, int32_t* out_ids,
                            float* out_scores, int mem) {
    if (!valid_ctx(ctx)) return PION_B200_EINVAL;
    // interleaved (score, id) pairs in out_scores (device memory only)
    const bool pairs_out = (mem & PION_B200_OUT_PAIRS) != 0;
    mem &= ~PION_B200_OUT_PAIRS;
    if (pairs_out) {
        if (mem != PION_B200_MEM_DEVICE || (reinterpret_cast<uintptr_t>(out_scores) & 7u) != 0)
            return set_error(ctx, PION_B200_EINVAL,
                             "flat_i8_knn: pairs out need 8-byte aligned device memory");
        out_ids = reinterpret_cast<int32_t*>(out_scores) + 1;
    }
    const int oes = pairs_out ? 2 : 1;
    if (!ix || ix->kind != kFlatI8)
        return set_error(ctx, PION_B200_EINVAL, "flat_i8_knn: not a FLAT INT8 index");
    if (ix->device != ctx->device)
        return set_error(ctx, PION_B200_EINVAL, "flat_i8_knn: index on device %d, context on %d",
                         ix->device, ctx->device);
    if (nq < 0 || k < 1 || (nq > 0 && (!q || !q_scale || !out_ids || !out_scores)))
        return set_error(ctx, PION_B200_EINVAL, "flat_i8_knn: bad arguments");
    if (k > 64) return set_error(ctx, PION_B200_ESHAPE, "flat_i8_knn: k %lld > 64", (long long)k);
    if (nq > (1 << 24)) return set_error(ctx, PION_B200_ESHAPE, "flat_i8_knn: batch too large");
    if (mem != PION_B200_MEM_HOST && mem != PION_B200_MEM_DEVICE)
        return set_error(ctx, PION_B200_EINVAL, "flat_i8_knn: bad mem %d", mem);
    if (nq == 0) return 0;
    if (int rc = use_device(ctx)) return rc;
    cudaStream_t st = ctx->stream;
    const int dim = (int)ix->dim;
    const int kk = (int)k;
    const int nqi = (int)nq;

    const int8_t* dq = q;
    const float* dqs = q_scale;
    int32_t* di = out_ids;
    float* dv = out_scores;
    const size_t q_bytes = align_up((size_t)nq * dim, 256);
    const size_t out_bytes = (size_t)nq * kk * 4;
    if (mem == PION_B200_MEM_HOST) {
        if (ensure(ctx->stage_in, q_bytes + (size_t)nq * 4) != 0 ||
            ensure(ctx->stage_out, 2 * align_up(out_bytes, 256)) != 0)
            return set_error(ctx, PION_B200_ENOMEM, "flat_i8_knn: staging");
        int8_t* sq = static_cast<int8_t*>(ctx->stage_in.ptr);
        float* sqs = reinterpret_cast<float*>(sq + q_bytes);
        if (cudaMemcpyAsync(sq, q, (size_t)nq * dim, cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(sqs, q_scale, (size_t)nq * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "flat_i8_knn: query copy failed");
        dq = sq;
        dqs = sqs;
        di = static_cast<int32_t*>(ctx->stage_out.ptr);
        dv = reinterpret_cast<float*>(static_cast<char*>(ctx->stage_out.ptr) + align_up(out_bytes, 256));
    } else if ((reinterpret_cast<uintptr_t>(q) & 15u) != 0) {
        return set_error(ctx, PION_B200_EINVAL, "flat_i8_knn: queries not 16-byte aligned");
    }

    int rc = 0;
    if (ix->n_rows == 0) {
        // Empty index: every result slot is padding (id -1, score -inf).
        rc = launch_fill_results(dv, di, (size_t)nq * kk, -INFINITY, st, oes);
        ctx->launches++;
    }
    const int path = forced_i8_path();
    const bool use_scan = ix->n_rows > 0 && (path == 1 || (path == 0 && nq == 1));
    if (ix->n_rows > 0 && use_scan) {
        const int ctas = fi8_scan1_ctas(ix->n_rows, ctx->num_sms);
        const size_t cbytes = (size_t)ctas * kk * 8;
        if (ensure(ctx->scratch, cbytes * (size_t)nq) != 0)
            return set_error(ctx, PION_B200_ENOMEM, "flat_i8_knn: scratch");
        float* cv = static_cast<float*>(ctx->scratch.ptr);
        int32_t* ci = reinterpret_cast<int32_t*>(cv + (size_t)nq * ctas * kk);
        for (int64_t t = 0; t < nq && rc == 0; ++t) {
            timing_begin(ctx);
            rc = launch_flat_i8_scan1(ix->rows_i8, ix->row_scale, ix->n_rows, dim,
                                      dq + (size_t)t * dim, dqs + t, kk, ctas,
                                      cv + (size_t)t * ctas * kk, ci + (size_t)t * ctas * kk, st);
            timing_end(ctx);
            ctx->launches++;
        }
        if (rc == 0) {
            rc = launch_merge_lists(cv, ci, nqi, ctas, kk, ix->id_base, true, dv, di, st, false, 0,
                                    false, oes);
            ctx->launches++;
        }
    } else if (ix->n_rows > 0) {
        const int n_qt = (nqi + fi8_query_tile() - 1) / fi8_query_tile();
        const int n_tiles = (int)((ix->n_rows + fi8_tile_rows() - 1) / fi8_tile_rows());
        const int lps = fi8_lists_per_split(kk);
        // Threshold pass over a sample of the first tiles: one exact score per 32-row chunk
        // (bound_mode), whose k-th best per query is an exact lower bound of the final
        // k-th score; the main pass starts from it, so its integer pre-filter rejects
        // almost every row at once.  The main pass then scores every tile.
        const bool pre = use_prepass(n_tiles, kk, "PION_B200_I8_PREPASS");
        int pre_tiles = pre ? bound_tiles(n_tiles, kk) : 0;
        if (pre) {  // tuning hook: the sample's size in tiles (the result is exact for any)
            const char* e = getenv("PION_B200_I8_SAMPLE");
            const int want = e ? atoi(e) : 0;
            if (want > 0) pre_tiles = want < n_tiles ? want : n_tiles;
        }
        const int splits = fi8_choose_splits(n_qt, n_tiles, ctx->num_sms);
        const int n_lists = splits * lps;
        int bnd_splits = pre ? ctx->num_sms / n_qt : 0;
        if (pre) bnd_splits = bnd_splits < 1 ? 1 : (bnd_splits > pre_tiles ? pre_tiles : bnd_splits);
        const int bnd_lists = bnd_splits * lps;
        const size_t ncand = (size_t)nq * n_lists * kk;
        const size_t nbnd = (size_t)nq * bnd_lists * kk;
        const size_t nthr = pre ? (size_t)nq * kk : 0;
        if (ensure(ctx->scratch, (ncand + nbnd + nthr) * 8) != 0)
            return set_error(ctx, PION_B200_ENOMEM, "flat_i8_knn: scratch");
        float* cv = static_cast<float*>(ctx->scratch.ptr);
        int32_t* ci = reinterpret_cast<int32_t*>(cv + ncand);
        float* bv = reinterpret_cast<float*>(ci + ncand);
        int32_t* bi = reinterpret_cast<int32_t*>(bv + nbnd);
        float* tv = reinterpret_cast<float*>(bi + nbnd);
        int32_t* ti = reinterpret_cast<int32_t*>(tv + nthr);
        CUtensorMap tmap_q;
        if (make_tmap_2d(&tmap_q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, dq, (uint64_t)dim,
                         (uint64_t)nq, (uint64_t)dim, (uint32_t)fi8_k_block(),
                         (uint32_t)fi8_query_tile(), CU_TENSOR_MAP_SWIZZLE_128B) != 0)
            return set_error(ctx, PION_B200_ECUDA, "flat_i8_knn: query tensor map");
        Fi8TcLaunch L;
        L.tmap_q = &tmap_q;
        L.tmap_rows = &ix->tmap_rows;
        L.row_scale = ix->row_scale;
        L.tile_rs_max = ix->tile_rs_max;
        L.q_scale = dqs;
        L.n_rows = ix->n_rows;
        L.nq = nqi;
        L.dim = dim;
        L.k = kk;
        L.status = call_status(ctx, mem);
        L.wait_ns = ctx->wait_ns;
        const int t_all = timing_begin(ctx);
        if (pre) {
            const int t_pre = timing_begin(ctx, PION_B200_TIMING_THRESHOLD);
            L.tile_begin = 0;
            L.tile_end = pre_tiles;
            L.n_splits = bnd_splits;
            L.n_lists = bnd_lists;
            L.cand_val = bv;
            L.cand_idx = bi;
            L.thr0 = nullptr;
            L.bound_mode = 1;
            rc = launch_flat_i8_tc(L, st);
            ctx->launches++;
            if (rc == 0) {  // per query: the k best chunk scores; the k-th is the bound
                rc = launch_merge_lists(bv, bi, nqi, bnd_lists, kk, 0, true, tv, ti, st);
                ctx->launches++;
            }
            timing_end(ctx, t_pre);
        }
        if (rc == 0) {
            const int t_main = timing_begin(ctx, PION_B200_TIMING_MAIN);
            L.tile_begin = 0;
            L.tile_end = n_tiles;
            L.n_splits = splits;
            L.n_lists = n_lists;
            L.cand_val = cv;
            L.cand_idx = ci;
            L.thr0 = pre ? tv + (kk - 1) : nullptr;
            L.thr0_stride = kk;
            L.bound_mode = 0;
            L.test_stall = test_stall();
            rc = launch_flat_i8_tc(L, st);
            ctx->launches++;
            timing_end(ctx, t_main);
        }
        timing_end(ctx, t_all);
        if (rc == 0) {
            rc = launch_merge_lists(cv, ci, nqi, n_lists, kk, ix->id_base, true, dv, di, st, false,
                                    0, false, oes);
            ctx->launches++;
        }
    }
    if (rc != 0)
        return set_error(ctx, rc, "flat_i8_knn: launch failed: %s",
                         cudaGetErrorString(cudaGetLastError()));
    if (mem == PION_B200_MEM_HOST) {
        if (cudaMemcpyAsync(out_ids, di, out_bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaMemcpyAsync(out_scores, dv, out_bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "flat_i8_knn: result copy failed");
        return finish_sync(ctx);
    }
    return 0;
}

// ------------------------------------------------------- row-sharded search

int pion_v_b200_flat_i8_knn_sharded(pion_b200_ctx* ctx, const pion_b200_index* ix,
                                    pion_b200_exchange* ex, const int8_t* q,
                                    const float* q_scale, int64_t nq, int64_t k, uint32_t epoch,
                                    int flags, int32_t* out_ids, float* out_scores) {
    if (!valid_ctx(ctx)) return PION_B200_EINVAL;
    if (!ix || ix->kind != kFlatI8 || ix->device != ctx->device)
        return set_error(ctx, PION_B200_EINVAL, "flat_i8_knn_sharded: not a FLAT INT8 index here");
    const bool pairs_out = (flags & PION_B200_OUT_PAIRS) != 0;
    if (pairs_out && out_scores) out_ids = reinterpret_cast<int32_t*>(out_scores) + 1;
    if (!ex || nq < 1 || k < 1 || k > 64 || !q || !q_scale || !out_ids || !out_scores ||
        epoch == 0 || (reinterpret_cast<uintptr_t>(q) & 15u) != 0)
        return set_error(ctx, PION_B200_EINVAL, "flat_i8_knn_sharded: bad arguments");
    if (int rc = use_device(ctx)) return rc;
    cudaStream_t st = ctx->stream;
    const int dim = (int)ix->dim;
    const int kk = (int)k, nqi = (int)nq;
    const int world = pion_v_b200_exchange_world(ex);
    if (world < 1) return set_error(ctx, PION_B200_EINVAL, "flat_i8_knn_sharded: no exchange");
    const int n_qt = (nqi + fi8_query_tile() - 1) / fi8_query_tile();
    const int n_tiles = (int)((ix->n_rows + fi8_tile_rows() - 1) / fi8_tile_rows());
    const int lps = fi8_lists_per_split(kk);
    // this rank's share of the sample one index of the whole would take
    int sample = 0;
    if (n_tiles > 0) {
        int total = bound_tiles(n_tiles * world, kk);
        const char* e = getenv("PION_B200_I8_SAMPLE");  // tuning hook, as in flat_i8_knn
        if (e && atoi(e) > 0) total = atoi(e);
        sample = (total + world - 1) / world;
        sample = sample < 2 ? 2 : sample;
        sample = sample > n_tiles ? n_tiles : sample;
    }
    const int splits = n_tiles > 0 ? fi8_choose_splits(n_qt, n_tiles, ctx->num_sms) : 1;
    const int n_lists = splits * lps;
    int bnd_splits = ctx->num_sms / n_qt;
    bnd_splits = bnd_splits < 1 ? 1 : (bnd_splits > sample ? (sample > 0 ? sample : 1) : bnd_splits);
    const int bnd_lists = bnd_splits * lps;
    const size_t ncand = (size_t)nq * n_lists * kk, nbnd = (size_t)nq * bnd_lists * kk;
    const size_t npair = (size_t)nq * kk * 2;  // floats / ints of one pair list
    if (ensure(ctx->scratch, (ncand + nbnd) * 8 + 3 * npair * 4 + 1024) != 0)
        return set_error(ctx, PION_B200_ENOMEM, "flat_i8_knn_sharded: scratch");
    float* cv = static_cast<float*>(ctx->scratch.ptr);
    int32_t* ci = reinterpret_cast<int32_t*>(cv + ncand);
    float* bv = reinterpret_cast<float*>(ci + ncand);
    int32_t* bi = reinterpret_cast<int32_t*>(bv + nbnd);
    float* lbp = reinterpret_cast<float*>(align_up(reinterpret_cast<uintptr_t>(bi + nbnd), 256));
    float* gbp = lbp + npair;  // the merged bound lists (pairs)
    float* lfp = gbp + npair;  // this shard's final k per query (pairs)
    int rc = 0;
    const int t_all = timing_begin(ctx);
    CUtensorMap tmap_q;
    Fi8TcLaunch L;
    if (n_tiles > 0) {
        if (make_tmap_2d(&tmap_q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, q, (uint64_t)dim, (uint64_t)nq,
                         (uint64_t)dim, (uint32_t)fi8_k_block(), (uint32_t)fi8_query_tile(),
                         CU_TENSOR_MAP_SWIZZLE_128B) != 0)
            return set_error(ctx, PION_B200_ECUDA, "flat_i8_knn_sharded: query tensor map");
        L.tmap_q = &tmap_q;
        L.tmap_rows = &ix->tmap_rows;
        L.row_scale = ix->row_scale;
        L.tile_rs_max = ix->tile_rs_max;
        L.q_scale = q_scale;
        L.n_rows = ix->n_rows;
        L.nq = nqi;
        L.dim = dim;
        L.k = kk;
        L.status = call_status(ctx, PION_B200_MEM_DEVICE);
        L.wait_ns = ctx->wait_ns;
        // 1. this rank's sample in bound mode, its k best chunk scores per query
        const int t_pre = timing_begin(ctx, PION_B200_TIMING_THRESHOLD);
        L.tile_begin = 0;
        L.tile_end = sample;
        L.n_splits = bnd_splits;
        L.n_lists = bnd_lists;
        L.cand_val = bv;
        L.cand_idx = bi;
        L.bound_mode = 1;
        rc = launch_flat_i8_tc(L, st);
        ctx->launches++;
        timing_end(ctx, t_pre);
    } else {
        rc = launch_fill_results(lbp, reinterpret_cast<int32_t*>(lbp) + 1, (size_t)nq * kk,
                                 -INFINITY, st, 2);
        ctx->launches++;
    }
    // 2. every rank's sample lists -> one bound per query (the union's k-th best); the
    // local merge publishes its result straight into every rank's receive buffer
    const bool local_bound = (flags & PION_B200_SHARD_LOCAL_BOUND) != 0;
    const bool fused_bnd = n_tiles > 0 && bnd_lists <= exchange_max_lists() && !local_bound;
    if (rc == 0 && n_tiles > 0 && !fused_bnd) {
        rc = launch_merge_lists(bv, bi, nqi, bnd_lists, kk, ix->id_base, true, lbp,
                                reinterpret_cast<int32_t*>(lbp) + 1, st, false, 0, false, 2);
        ctx->launches++;
    }
    if (rc == 0 && local_bound)
        gbp = lbp;  // this rank's own sample bound
    else if (rc == 0 && fused_bnd)
        rc = exchange_lists_merge(ctx, ex, 0, bv, bi, bnd_lists, ix->id_base, nq, k, epoch, true,
                                  gbp, reinterpret_cast<int32_t*>(gbp) + 1, 2);
    else if (rc == 0)
        rc = exchange_merge(ctx, ex, 0, lbp, nq, k, epoch, true, gbp,
                            reinterpret_cast<int32_t*>(gbp) + 1, 2);
    // 3. the whole shard from that bound, merged to this shard's k per query
    if (rc == 0 && n_tiles > 0) {
        const int t_main = timing_begin(ctx, PION_B200_TIMING_MAIN);
        L.tile_begin = 0;
        L.tile_end = n_tiles;
        L.n_splits = splits;
        L.n_lists = n_lists;
        L.cand_val = cv;
        L.cand_idx = ci;
        L.thr0 = gbp + 2 * (kk - 1);
        L.thr0_stride = 2 * kk;
        L.bound_mode = 0;
        rc = launch_flat_i8_tc(L, st);
        ctx->launches++;
        timing_end(ctx, t_main);
    }
    // 4. every shard's k -> the global k
    const bool fused_fin = n_tiles > 0 && n_lists <= exchange_max_lists();
    if (rc == 0 && n_tiles > 0 && !fused_fin) {
        rc = launch_merge_lists(cv, ci, nqi, n_lists, kk, ix->id_base, true, lfp,
                                reinterpret_cast<int32_t*>(lfp) + 1, st, false, 0, false, 2);
        ctx->launches++;
    } else if (rc == 0 && n_tiles == 0) {
        rc = launch_fill_results(lfp, reinterpret_cast<int32_t*>(lfp) + 1, (size_t)nq * kk,
                                 -INFINITY, st, 2);
        ctx->launches++;
    }
    if (rc == 0 && fused_fin)
        rc = exchange_lists_merge(ctx, ex, 1, cv, ci, n_lists, ix->id_base, nq, k, epoch, true,
                                  out_scores, out_ids, pairs_out ? 2 : 1);
    else if (rc == 0)
        rc = exchange_merge(ctx, ex, 1, lfp, nq, k, epoch, true, out_scores, out_ids,
                            pairs_out ? 2 : 1);
    timing_end(ctx, t_all);
    if (rc != 0)
        return set_error(ctx, rc, "flat_i8_knn_sharded: failed: %s",
                         cudaGetErrorString(cudaGetLastError()));
    return 0;
}

// --------------------------------------------------------------- utilities

int pion_v_b200_quantize_rows_i8(pion_b200_ctx* ctx, const float* src, int64_t n_rows, int64_t d,
                                 int64_t d_pad, int8_t* dst, float* dst_scale, int mem) {
    if (!valid_ctx(ctx)) return PION_B200_EINVAL;
    if (n_rows < 0 || d < 0 || d_pad < d || d_pad > (1 << 20) ||
        (n_rows > 0 && (!src || !dst || !dst_scale)))
        return set_error(ctx, PION_B200_EINVAL, "quantize_rows_i8: bad arguments");
    if (n_rows == 0) return 0;
    if (int rc = use_device(ctx)) return rc;
    cudaStream_t st = ctx->stream;
    const float* ds = src;
    int8_t* dd = dst;
    float* dsc = dst_scale;
    const size_t in_bytes = (size_t)n_rows * d_pad * 4;
    const size_t out_bytes = align_up((size_t)n_rows * d_pad, 256);
    if (mem == PION_B200_MEM_HOST) {
        if (ensure(ctx->stage_in, in_bytes) != 0 ||
            ensure(ctx->stage_out, out_bytes + (size_t)n_rows * 4) != 0)
            return set_error(ctx, PION_B200_ENOMEM, "quantize_rows_i8: staging");
        if (cudaMemcpyAsync(ctx->stage_in.ptr, src, in_bytes, cudaMemcpyHostToDevice, st) !=
            cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "quantize_rows_i8: copy failed");
        ds = static_cast<const float*>(ctx->stage_in.ptr);
        dd = static_cast<int8_t*>(ctx->stage_out.ptr);
        dsc = reinterpret_cast<float*>(static_cast<char*>(ctx->stage_out.ptr) + out_bytes);
    } else if (mem != PION_B200_MEM_DEVICE) {
        return set_error(ctx, PION_B200_EINVAL, "quantize_rows_i8: bad mem %d", mem);
    }
    int rc = launch_quantize_rows_i8(ds, n_rows, (int)d, (int)d_pad, dd, dsc, st);
    ctx->launches++;
    if (rc != 0) return set_error(ctx, rc, "quantize_rows_i8: launch failed");
    if (mem == PION_B200_MEM_HOST) {
        if (cudaMemcpyAsync(dst, dd, (size_t)n_rows * d_pad, cudaMemcpyDeviceToHost, st) !=
                cudaSuccess ||
            cudaMemcpyAsync(dst_scale, dsc, (size_t)n_rows * 4, cudaMemcpyDeviceToHost, st) !=
                cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "quantize_rows_i8: copy back failed");
        return finish_sync(ctx);
    }
    return 0;
}

int pion_v_b200_merge_topk(pion_b200_ctx* ctx, const float* cand_scores, const int32_t* cand_ids,
                           int64_t nq, int64_t n_lists, int64_t k, int flags,
                           float* out_scores, int32_t* out_ids, int mem) {
    if (!valid_ctx(ctx)) return PION_B200_EINVAL;
    const bool pairs = (flags & PION_B200_MERGE_PAIRS) != 0;
    if (nq < 0 || n_lists < 1 || k < 1 ||
        (nq > 0 && (!cand_scores || (!pairs && !cand_ids) || !out_scores || !out_ids)))
        return set_error(ctx, PION_B200_EINVAL, "merge_topk: bad arguments");
    if (n_lists > 2048 || k > 4096)
        return set_error(ctx, PION_B200_ESHAPE, "merge_topk: n_lists <= 2048, k <= 4096");
    if (pairs && (reinterpret_cast<uintptr_t>(cand_scores) & 7u) != 0)
        return set_error(ctx, PION_B200_EINVAL, "merge_topk: pairs not 8-byte aligned");
    if (nq == 0) return 0;
    if (int rc = use_device(ctx)) return rc;
    cudaStream_t st = ctx->stream;
    const size_t cand = (size_t)nq * n_lists * k;
    const size_t outn = (size_t)nq * k;
    const float* cv = cand_scores;
    const int32_t* ci = cand_ids;
    float* ov = out_scores;
    int32_t* oi = out_ids;
    if (mem == PION_B200_MEM_HOST) {
        if (ensure(ctx->stage_in, cand * 8) != 0 || ensure(ctx->stage_out, outn * 8) != 0)
            return set_error(ctx, PION_B200_ENOMEM, "merge_topk: staging");
        float* sv = static_cast<float*>(ctx->stage_in.ptr);
        int32_t* si = reinterpret_cast<int32_t*>(sv + cand);
        bool ok;
        if (pairs)
            ok = cudaMemcpyAsync(sv, cand_scores, cand * 8, cudaMemcpyHostToDevice, st) ==
                 cudaSuccess;
        else
            ok = cudaMemcpyAsync(sv, cand_scores, cand * 4, cudaMemcpyHostToDevice, st) ==
                     cudaSuccess &&
                 cudaMemcpyAsync(si, cand_ids, cand * 4, cudaMemcpyHostToDevice, st) ==
                     cudaSuccess;
        if (!ok) return set_error(ctx, PION_B200_ECUDA, "merge_topk: copy failed");
        cv = sv;
        ci = si;
        ov = static_cast<float*>(ctx->stage_out.ptr);
        oi = reinterpret_cast<int32_t*>(ov + outn);
    } else if (mem != PION_B200_MEM_DEVICE) {
        return set_error(ctx, PION_B200_EINVAL, "merge_topk: bad mem %d", mem);
    }
    int rc = launch_merge_lists(cv, ci, (int)nq, (int)n_lists, (int)k, 0,
                                (flags & PION_B200_MERGE_DESC) != 0, ov, oi, st,
                                (flags & PION_B200_MERGE_LISTS_MAJOR) != 0, 0, pairs);
    ctx->launches++;
    if (rc != 0) return set_error(ctx, rc, "merge_topk: launch failed");
    if (mem == PION_B200_MEM_HOST) {
        if (cudaMemcpyAsync(out_scores, ov, outn * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaMemcpyAsync(out_ids, oi, outn * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess)
            return set_error(ctx, PION_B200_ECUDA, "merge_topk: copy back failed");
        return finish_sync(ctx);
    }
    return 0;
}

}  // extern "C"
