// merge_delta on the GPU (src/commands/vector.mojo:1368-1456): the graph's results
// rescored exactly from the FP32 ingest rows (_exact_rescore), the rows ingested since
// the build scanned exactly (exact_knn over [built, rows)), and the two ascending lists
// merged.
//   delta_rescore_kernel  a CTA per query: for every graph result whose slot is below
//                         `built`, COSINE 1 - dot_f32_4chain(q^, row) or L2
//                         l2sq_f32_4chain(q, row) (16 half-warps, one result each);
//                         others keep their score; then _exact_rescore's insertion sort
//                         (stable: rank = #smaller + #equal before it).
//   delta_merge_kernel    a warp per query: the merge loop of merge_delta, a graph entry
//                         first when its score <= the delta entry's, k kept.
#include <cstdint>

#include "exact_fp32.cuh"
#include "internal.h"

namespace pion {
namespace delta {

constexpr int THREADS = 256;
constexpr int KG_MAX = 1024;

__global__ void __launch_bounds__(THREADS)
    delta_rescore_kernel(const float* __restrict__ rows, int dim, int64_t built, int l2,
                         const float* __restrict__ q, int kg, int32_t* __restrict__ ids,
                         float* __restrict__ scores, int* __restrict__ n_graph) {
    __shared__ float sd[KG_MAX];
    __shared__ int32_t si[KG_MAX];
    __shared__ int n_s;
    const int t = blockIdx.x;
    const int lane = threadIdx.x & 31, half = lane >> 4, hl = lane & 15;
    const int slot = (threadIdx.x >> 5) * 2 + half;  // 16 half-warps
    const unsigned hmask = half ? 0xffff0000u : 0x0000ffffu;
    int32_t* gi = ids + (size_t)t * kg;
    float* gs = scores + (size_t)t * kg;
    const float* qv = q + (size_t)t * dim;
    if (threadIdx.x == 0) {  // the list ends at its first empty entry
        int n = 0;
        while (n < kg && gi[n] >= 0) ++n;
        n_s = n;
    }
    __syncthreads();
    const int n = n_s;
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        sd[j] = gs[j];
        si[j] = gi[j];
    }
    __syncthreads();
    for (int base = 0; base < n; base += 16) {  // every half-warp iterates alike
        const int j = base + slot;
        const int32_t id = j < n ? si[j] : -1;
        const bool ok = id >= 0 && id < built;
        if (ok) {
            const float* row = rows + (size_t)id * dim;
            const float d = l2 ? l2sq4chain_half(qv, row, dim, hl, hmask)
                               : __fsub_rn(1.0f, dot4chain_half(qv, row, dim, hl, hmask));
            if (hl == 0) sd[j] = d;
        }
    }
    __syncthreads();
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        const float d = sd[j];
        int rank = 0;
        for (int i = 0; i < n; ++i) rank += (sd[i] < d || (sd[i] == d && i < j)) ? 1 : 0;
        gs[rank] = d;
        gi[rank] = si[j];
    }
    if (threadIdx.x == 0) n_graph[t] = n;
}

__global__ void delta_merge_kernel(const int32_t* __restrict__ gi, const float* __restrict__ gs,
                                   const int* __restrict__ n_graph, int kg,
                                   const int32_t* __restrict__ di, const float* __restrict__ ds,
                                   int kd, int nq, int k, int32_t* __restrict__ out_i,
                                   float* __restrict__ out_s) {
    const int t = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (t >= nq || (threadIdx.x & 31) != 0) return;
    const int na = n_graph[t];
    int nb = 0;
    while (nb < kd && di[(size_t)t * kd + nb] >= 0) ++nb;
    int a = 0, b = 0, o = 0;
    while (o < k && (a < na || b < nb)) {
        const bool take_a = b >= nb || (a < na && gs[(size_t)t * kg + a] <= ds[(size_t)t * kd + b]);
        if (take_a) {
            out_i[(size_t)t * k + o] = gi[(size_t)t * kg + a];
            out_s[(size_t)t * k + o] = gs[(size_t)t * kg + a];
            ++a;
        } else {
            out_i[(size_t)t * k + o] = di[(size_t)t * kd + b];
            out_s[(size_t)t * k + o] = ds[(size_t)t * kd + b];
            ++b;
        }
        ++o;
    }
    for (; o < k; ++o) {
        out_i[(size_t)t * k + o] = -1;
        out_s[(size_t)t * k + o] = INFINITY;
    }
}

}  // namespace delta

int delta_kg_max() { return delta::KG_MAX; }

int launch_delta_rescore(const float* rows, int dim, int64_t built, int l2, const float* q, int nq,
                         int kg, int32_t* ids, float* scores, int* n_graph, cudaStream_t st) {
    if (nq <= 0) return 0;
    if (kg < 1 || kg > delta::KG_MAX) return PION_B200_ESHAPE;
    delta::delta_rescore_kernel<<<nq, delta::THREADS, 0, st>>>(rows, dim, built, l2, q, kg, ids,
                                                                scores, n_graph);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int launch_delta_merge(const int32_t* gi, const float* gs, const int* n_graph, int kg,
                       const int32_t* di, const float* ds, int kd, int nq, int k, int32_t* out_i,
                       float* out_s, cudaStream_t st) {
    if (nq <= 0) return 0;
    delta::delta_merge_kernel<<<(nq + 7) / 8, 256, 0, st>>>(gi, gs, n_graph, kg, di, ds, kd, nq, k,
                                                             out_i, out_s);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

}  // namespace pion
