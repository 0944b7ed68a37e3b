// FLAT INT8 KNN entry point that allocates no device memory.
//
// For callers that cannot call cudaMalloc on the query path: an engine whose
// device memory is entirely owned by another allocator (a fixed pool reserved at
// start-up, so any extra cudaMalloc fails or breaks its accounting), or a query
// thread that must not take cudaMalloc's implicit device-wide synchronisation.
// The regular pion_v_b200_flat_i8_knn keeps its candidate lists in context
// scratch that grows with cudaMalloc; this variant puts the same scratch in one
// file-scope __device__ array of fixed size instead.
//
// The array removes the allocation but adds sharing: every call on a device uses
// the same array and it keeps the last call's contents, so two calls whose kernels
// overlap on the GPU (different streams, or different host threads) race on it and
// corrupt each other's results.  Serialise the calls per device.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "internal.h"

namespace pion {

// Scratch size limit of the no-allocation entry point (bytes).  Every GPU that
// loads the library holds this array until the process exits.
constexpr size_t kStaticScratchBytes = 8u << 20;
constexpr int kMaxDevices = 64;

// Static device scratch: [status word (256 B)] [tile maxima] [candidate lists].
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// Device address of g_static_scratch, looked up once per device.  In host code the
// symbol is only a host-side stand-in, never a device address.
static void* g_scratch_addr[kMaxDevices];
static std::mutex g_scratch_mu;

static int static_scratch(int device, unsigned char** out) {
    if (device < 0 || device >= kMaxDevices) return PION_B200_ENODEV;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[device]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess || !p) {
            fprintf(stderr, "pion_vector_b200: cudaGetSymbolAddress failed on device %d: %s\n",
                    device, cudaGetErrorString(e));
            cudaGetLastError();
            return PION_B200_ECUDA;
        }
        g_scratch_addr[device] = p;
    }
    *out = static_cast<unsigned char*>(g_scratch_addr[device]);
    return 0;
}

static size_t round256(size_t x) { return (x + 255) / 256 * 256; }

}  // namespace pion

using namespace pion;

extern "C" int pion_v_b200_flat_i8_knn_static(const int8_t* rows, const float* row_scale,
                                              int64_t n_rows, int64_t dim, const int8_t* q,
                                              const float* q_scale, int64_t nq, int64_t k,
                                              int32_t* out_ids, float* out_scores,
                                              void* cuda_stream) {
    if (nq < 0 || n_rows < 0 || k < 1 ||
        (nq > 0 && (!q || !q_scale || !out_ids || !out_scores)) ||
        (n_rows > 0 && (!rows || !row_scale)))
        return PION_B200_EINVAL;
    if (dim <= 0 || dim % 16 != 0 || dim > 16384 || k > 64 || n_rows > INT32_MAX - 1) {
        fprintf(stderr, "pion_vector_b200: flat_i8_knn_static: unsupported shape (dim %lld, "
                        "k %lld)\n", (long long)dim, (long long)k);
        return PION_B200_ESHAPE;
    }
    if ((reinterpret_cast<uintptr_t>(rows) & 15u) || (reinterpret_cast<uintptr_t>(q) & 15u))
        return PION_B200_EINVAL;
    if (nq == 0) return 0;
    cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return PION_B200_ENODEV;
    int num_sms = 0;
    if (cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
        return PION_B200_ENODEV;
    unsigned char* base = nullptr;
    if (int rc = static_scratch(device, &base)) return rc;

    // Lay out the scratch for this call and refuse what does not fit.
    const int kk = (int)k;
    const int nqi = (int)nq;
    const int n_tiles = (int)((n_rows + fi8_tile_rows() - 1) / fi8_tile_rows());
    const bool scan = (nq == 1);
    int lists = 1, splits = 1;
    if (n_rows > 0) {
        if (scan) {
            lists = fi8_scan1_ctas(n_rows, num_sms);
        } else {
            splits = fi8_choose_splits((nqi + fi8_query_tile() - 1) / fi8_query_tile(), n_tiles,
                                       num_sms);
            lists = splits * fi8_lists_per_split(kk);
        }
    }
    const size_t status_bytes = 256;
    const size_t tiles_bytes = round256((size_t)(n_tiles > 0 ? n_tiles : 1) * sizeof(float));
    const size_t ncand = (size_t)nq * lists * kk;
    const size_t need = status_bytes + tiles_bytes + 2 * round256(ncand * 4);
    if (need > kStaticScratchBytes) {
        fprintf(stderr, "pion_vector_b200: flat_i8_knn_static needs %zu bytes of scratch for "
                        "nq=%lld, k=%lld, %lld rows; the static limit is %zu\n",
                need, (long long)nq, (long long)k, (long long)n_rows, kStaticScratchBytes);
        return PION_B200_ESHAPE;
    }
    int* status = reinterpret_cast<int*>(base);
    float* tile_max = reinterpret_cast<float*>(base + status_bytes);
    float* cv = reinterpret_cast<float*>(base + status_bytes + tiles_bytes);
    int32_t* ci = reinterpret_cast<int32_t*>(base + status_bytes + tiles_bytes +
                                             round256(ncand * 4));
    // The array keeps the previous call's contents: the status word must start at 0.
    if (cudaMemsetAsync(status, 0, sizeof(int), st) != cudaSuccess) return PION_B200_ECUDA;

    int rc = 0;
    if (n_rows == 0) {
        rc = launch_fill_results(out_scores, out_ids, (size_t)nq * kk, -INFINITY, st);
    } else if (scan) {
        rc = launch_flat_i8_scan1(rows, row_scale, n_rows, (int)dim, q, q_scale, kk, lists, cv,
                                  ci, st);
        if (rc == 0)
            rc = launch_merge_lists(cv, ci, 1, lists, kk, 0, true, out_scores, out_ids, st);
    } else {
        CUtensorMap tmap_q, tmap_rows;
        if (make_tmap_2d(&tmap_q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, q, (uint64_t)dim,
                         (uint64_t)nq, (uint64_t)dim, (uint32_t)fi8_k_block(),
                         (uint32_t)fi8_query_tile(), CU_TENSOR_MAP_SWIZZLE_128B) != 0 ||
            make_tmap_2d(&tmap_rows, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rows, (uint64_t)dim,
                         (uint64_t)n_rows, (uint64_t)dim, (uint32_t)fi8_k_block(),
                         (uint32_t)fi8_tile_rows(), CU_TENSOR_MAP_SWIZZLE_128B) != 0)
            return PION_B200_ECUDA;
        rc = launch_tile_max(row_scale, n_rows, tile_max, st);
        if (rc == 0) {
            Fi8TcLaunch L;
            L.tmap_q = &tmap_q;
            L.tmap_rows = &tmap_rows;
            L.row_scale = row_scale;
            L.tile_rs_max = tile_max;
            L.q_scale = q_scale;
            L.n_rows = n_rows;
            L.nq = nqi;
            L.dim = (int)dim;
            L.k = kk;
            L.tile_begin = 0;
            L.tile_end = n_tiles;
            L.n_splits = splits;
            L.n_lists = lists;
            L.cand_val = cv;
            L.cand_idx = ci;
            L.status = status;
            rc = launch_flat_i8_tc(L, st);
        }
        if (rc == 0)
            rc = launch_merge_lists(cv, ci, nqi, lists, kk, 0, true, out_scores, out_ids, st);
    }
    if (rc != 0) return rc;
    int h_status = 0;
    if (cudaMemcpyAsync(&h_status, status, sizeof(int), cudaMemcpyDeviceToHost, st) !=
            cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return PION_B200_ECUDA;
    return h_status;
}
