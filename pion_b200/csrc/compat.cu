// The reference-compatible symbols Pion's engine binds from libpion_vector
// (vendor/pion-vector/linux-x86_64/MANIFEST; call sites src/vector/vector_abi.mojo:33-99,
// src/vector/pkm_kernels.mojo:88-266): same names, arguments and results, computed
// on the GPU.  Every pointer is a host pointer into engine-owned buffers; each call
// copies its inputs to the device, computes, and copies the outputs back.  There is
// no error channel in the reference: failures print to stderr and leave the outputs
// untouched.
//
// Exactness: pkm_scores_i8 is bit-identical (exact int32 dot, the reference's
// epilogue order); pkm_scores_f32 / pkm_rescore_f32 reproduce the reference's
// 8-lane accumulation order; pkm_topk_max, pkm_sort_desc and pkm_combine_topk return
// the reference's ids, values and order, ties included (their heap algorithms are
// replayed exactly on the device; pkm_topk_max first discards, in parallel, every
// element the reference's heap provably never admits).
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>

#include "common.cuh"
#include "internal.h"

namespace pion {
namespace compat {

// ------------------------------------------------------------- scores --------

// One warp per (row, query): 16-byte chunks, dp4a, warp sum; the reference epilogue
// (f32(dot) * row_scale) * q_scale (src/vector/reference/pkm_ref.mojo:58-61).
__global__ void scores_i8_kernel(const int8_t* __restrict__ keys, int64_t s_rows, int d_pad,
                                 const float* __restrict__ rs, const int8_t* __restrict__ q,
                                 const float* __restrict__ qs, float* __restrict__ dst) {
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    const int t = blockIdx.y;
    if (r >= s_rows) return;
    const int lane = threadIdx.x & 31;
    const int4* kr = reinterpret_cast<const int4*>(keys + r * d_pad);
    const int4* qr = reinterpret_cast<const int4*>(q + (size_t)t * d_pad);
    int acc = 0;
    for (int c = lane; c < d_pad / 16; c += 32) {
        const int4 a = kr[c];
        const int4 b = qr[c];
        acc = __dp4a(a.x, b.x, acc);
        acc = __dp4a(a.y, b.y, acc);
        acc = __dp4a(a.z, b.z, acc);
        acc = __dp4a(a.w, b.w, acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0)
        dst[(size_t)t * s_rows + r] = __fmul_rn(__fmul_rn(__int2float_rn(acc), rs[r]), qs[t]);
}

// 8 lanes per dot: lane l sums products l, l+8, l+16, ... in order (the reference's
// 8-wide accumulator, src/vector/reference/pkm_ref.mojo:22-31), then the halving-tree
// lane sum.  Returns the dot to every lane of the 8-lane group.
__device__ __forceinline__ float dot8(const float* __restrict__ a, const float* __restrict__ b,
                                      int d_pad, int l) {
    float acc = 0.0f;
    for (int i = l; i < d_pad; i += 8) acc = __fadd_rn(acc, __fmul_rn(a[i], b[i]));
    const unsigned m = 0xffffffffu;
    acc = __fadd_rn(acc, __shfl_down_sync(m, acc, 4, 8));  // lanes 0-3: a_l + a_{l+4}
    acc = __fadd_rn(acc, __shfl_down_sync(m, acc, 2, 8));  // lanes 0-1
    acc = __fadd_rn(acc, __shfl_down_sync(m, acc, 1, 8));  // lane 0
    return __shfl_sync(m, acc, 0, 8);
}

// dst[t * s_rows + r] = <q[t], keys[r]>, 4 (row, query) pairs per warp.
__global__ void scores_f32_kernel(const float* __restrict__ keys, int64_t s_rows, int d_pad,
                                  const float* __restrict__ q, int nq, float* __restrict__ dst) {
    const int64_t pair = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 3;
    const int l = threadIdx.x & 7;
    const bool ok = pair < s_rows * (int64_t)nq;
    const int64_t pp = ok ? pair : 0;
    const int64_t t = pp / s_rows, r = pp % s_rows;
    const float v = dot8(keys + r * d_pad, q + t * d_pad, d_pad, l);
    if (ok && l == 0) dst[t * s_rows + r] = v;
}

__global__ void rescore_f32_kernel(const float* __restrict__ keys, int d_pad,
                                   const float* __restrict__ q, const int32_t* __restrict__ idx,
                                   int64_t cnt, float* __restrict__ dst) {
    const int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 3;
    const int l = threadIdx.x & 7;
    const bool ok = t < cnt;
    const int64_t row = ok ? idx[t] : 0;
    const float v = dot8(keys + row * d_pad, q, d_pad, l);
    if (ok && l == 0) dst[t] = v;
}

// --------------------------------------------------- heap routines (replayed) --
// src/vector/reference/pkm_ref.mojo:64-107: min-heap sift-down, heapify, heapsort.
__device__ void sift_down_min(float* val, int32_t* idx, int64_t start, int64_t n) {
    int64_t root = start;
    for (;;) {
        int64_t child = 2 * root + 1;
        if (child >= n) break;
        if (child + 1 < n && val[child + 1] < val[child]) child += 1;
        if (val[child] < val[root]) {
            float tv = val[root]; val[root] = val[child]; val[child] = tv;
            int32_t ti = idx[root]; idx[root] = idx[child]; idx[child] = ti;
            root = child;
        } else {
            break;
        }
    }
}

__device__ void heapify_min(float* val, int32_t* idx, int64_t n) {
    for (int64_t s = n / 2 - 1; s >= 0; --s) sift_down_min(val, idx, s, n);
}

__device__ void sort_desc(float* val, int32_t* idx, int64_t n) {
    if (n <= 1) return;
    heapify_min(val, idx, n);
    for (int64_t e = n - 1; e > 0; --e) {
        float tv = val[0]; val[0] = val[e]; val[e] = tv;
        int32_t ti = idx[0]; idx[0] = idx[e]; idx[e] = ti;
        sift_down_min(val, idx, 0, e);
    }
}

__global__ void sort_desc_kernel(float* val, int32_t* idx, int64_t n) {
    if (threadIdx.x == 0 && blockIdx.x == 0) sort_desc(val, idx, n);
}

// src/vector/reference/pkm_ref.mojo:133-160 (ref_pkm_combine_topk), one thread.
__global__ void combine_topk_kernel(const float* s0, const int32_t* i0, int64_t k0,
                                    const float* s1, const int32_t* i1, int64_t k1,
                                    int64_t s_cols, int64_t k, int32_t* out_id, float* out_score,
                                    int64_t* out_cnt) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const int64_t lim = k0 * k1;
    const int64_t cap = k < lim ? k : lim;
    if (cap <= 0) {
        *out_cnt = 0;
        return;
    }
    int64_t cnt = 0;
    for (int64_t a = 0; a < k0; ++a)
        for (int64_t b = 0; b < k1; ++b) {
            const float sc = __fadd_rn(s0[a], s1[b]);
            const int32_t sid = (int32_t)((int64_t)i0[a] * s_cols + (int64_t)i1[b]);
            if (cnt < cap) {
                out_score[cnt] = sc;
                out_id[cnt] = sid;
                cnt += 1;
                if (cnt == cap) heapify_min(out_score, out_id, cap);
            } else if (sc > out_score[0]) {
                out_score[0] = sc;
                out_id[0] = sid;
                sift_down_min(out_score, out_id, 0, cap);
            }
        }
    sort_desc(out_score, out_id, cnt);
    *out_cnt = cnt;
}

// ------------------------------------------------------------------ top-k max --
// ref_pkm_topk_max (src/vector/reference/pkm_ref.mojo:110-130) admits element i >= k
// iff s_i > (k-th largest of s_0..s_{i-1}).  For a block b of the input, L_b = k-th
// largest over blocks 0..b-1 is <= that threshold for every i in b, so an element with
// s_i <= L_b is never admitted.  The survivors (i < k, or s_i > L_b) in index order,
// replayed through the reference heap, give the reference's exact result.
constexpr int TK_BLOCK = 2048;
constexpr int TK_THREADS = 256;
constexpr int TK_KMAX = 256;

// Block-local top-k values (descending) by a bitonic sort of the block in shared memory.
__global__ void __launch_bounds__(TK_THREADS) block_topk_kernel(const float* __restrict__ s,
                                                                int64_t n, int k,
                                                                float* __restrict__ blk) {
    __shared__ float v[TK_BLOCK];
    const int64_t base = (int64_t)blockIdx.x * TK_BLOCK;
    for (int i = threadIdx.x; i < TK_BLOCK; i += TK_THREADS)
        v[i] = base + i < n ? s[base + i] : -INFINITY;
    __syncthreads();
    for (int size = 2; size <= TK_BLOCK; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < TK_BLOCK / 2; i += TK_THREADS) {
                const int lo = 2 * i - (i & (stride - 1));
                const int hi = lo + stride;
                const bool desc = ((lo & size) == 0);
                const float a = v[lo], b = v[hi];
                // NaN-free inputs: order descending within ascending-bit blocks
                if (desc ? (a < b) : (a > b)) {
                    v[lo] = b;
                    v[hi] = a;
                }
            }
            __syncthreads();
        }
    for (int j = threadIdx.x; j < k; j += TK_THREADS) blk[(size_t)blockIdx.x * k + j] = v[j];
}

// One warp: L[b] = k-th largest of the values of blocks < b (running top-k merge).
__global__ void prefix_bounds_kernel(const float* __restrict__ blk, int nb, int k,
                                     float* __restrict__ bound) {
    __shared__ float run[TK_KMAX], nxt[TK_KMAX];
    const int lane = threadIdx.x;
    for (int j = lane; j < k; j += 32) run[j] = -INFINITY;
    int have = 0;
    __syncwarp();
    for (int b = 0; b < nb; ++b) {
        if (lane == 0) bound[b] = have >= k ? run[k - 1] : -INFINITY;
        // merge run (desc) with blk[b] (desc): lane 0 walks both lists (k <= 256)
        if (lane == 0) {
            const float* x = blk + (size_t)b * k;
            int i = 0, j = 0;
            for (int o = 0; o < k; ++o) {
                if (j >= k || (i < k && run[i] >= x[j])) nxt[o] = run[i++];
                else nxt[o] = x[j++];
            }
        }
        __syncwarp();
        for (int j = lane; j < k; j += 32) run[j] = nxt[j];
        have += TK_BLOCK;
        __syncwarp();
    }
}

// Survivors of block b in index order: sv/si[b * TK_BLOCK + j], count cnt[b].
__global__ void __launch_bounds__(TK_THREADS) survivors_kernel(const float* __restrict__ s,
                                                               int64_t n, int k,
                                                               const float* __restrict__ bound,
                                                               float* __restrict__ sv,
                                                               int32_t* __restrict__ si,
                                                               int* __restrict__ cnt) {
    __shared__ int warp_tot[TK_THREADS / 32];
    __shared__ int base_s;
    const int64_t base = (int64_t)blockIdx.x * TK_BLOCK;
    const float L = bound[blockIdx.x];
    if (threadIdx.x == 0) base_s = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    for (int off = 0; off < TK_BLOCK; off += TK_THREADS) {
        const int64_t i = base + off + threadIdx.x;
        const bool keep = i < n && (i < k || s[i] > L);
        const unsigned bal = __ballot_sync(0xffffffffu, keep);
        if (lane == 0) warp_tot[w] = __popc(bal);
        __syncthreads();
        int before = base_s;
        for (int x = 0; x < w; ++x) before += warp_tot[x];
        if (keep) {
            const int pos = before + __popc(bal & ((1u << lane) - 1u));
            sv[base + pos] = s[i];
            si[base + pos] = (int32_t)i;
        }
        __syncthreads();
        if (threadIdx.x == 0)
            for (int x = 0; x < TK_THREADS / 32; ++x) base_s += warp_tot[x];
        __syncthreads();
    }
    if (threadIdx.x == 0) cnt[blockIdx.x] = base_s;
}

// One thread: the reference heap over the survivors, then the heapsort.
__global__ void replay_topk_kernel(const float* __restrict__ sv, const int32_t* __restrict__ si,
                                   const int* __restrict__ cnt, int nb, int64_t kk,
                                   int32_t* __restrict__ out_idx, float* __restrict__ out_val) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    int64_t seeded = 0;
    for (int b = 0; b < nb; ++b)
        for (int j = 0; j < cnt[b]; ++j) {
            const size_t p = (size_t)b * TK_BLOCK + j;
            const int32_t i = si[p];
            const float v = sv[p];
            if (i < kk) {  // the first k elements seed the heap (all survive)
                out_idx[i] = i;
                out_val[i] = v;
                if (++seeded == kk) heapify_min(out_val, out_idx, kk);
            } else if (v > out_val[0]) {
                out_val[0] = v;
                out_idx[0] = i;
                sift_down_min(out_val, out_idx, 0, kk);
            }
        }
    sort_desc(out_val, out_idx, kk);
}

}  // namespace compat

// -------------------------------------------------------------- host side ---

namespace {

// One default context per calling thread (the engine calls from each worker's own
// pthread), released when the thread exits.
struct ThreadCtx {
    pion_b200_ctx* ctx = nullptr;
    ~ThreadCtx() {
        if (ctx) pion_v_b200_shutdown(ctx);
    }
};
thread_local ThreadCtx tl_ctx;

pion_b200_ctx* default_ctx(const char* who) {
    if (!tl_ctx.ctx && pion_v_b200_init(-1, 0, &tl_ctx.ctx) != 0) {
        fprintf(stderr, "pion_vector_b200: %s: no usable B200 device\n", who);
        tl_ctx.ctx = nullptr;
    }
    return tl_ctx.ctx;
}

}  // namespace

pion_b200_ctx* compat_default_ctx(const char* who) { return default_ctx(who); }

namespace {

int fail(const char* who, const char* what) {
    fprintf(stderr, "pion_vector_b200: %s: %s\n", who, what);
    return -1;
}

// Device scratch carved from the default context's buffer.
struct Carve {
    char* base;
    size_t off = 0;
    explicit Carve(void* p) : base(static_cast<char*>(p)) {}
    template <typename T>
    T* take(size_t n) {
        T* p = reinterpret_cast<T*>(base + off);
        off += (n * sizeof(T) + 255) / 256 * 256;
        return p;
    }
};

size_t carve_size(std::initializer_list<size_t> bytes) {
    size_t s = 0;
    for (size_t b : bytes) s += (b + 255) / 256 * 256;
    return s;
}

bool h2d(void* d, const void* h, size_t n, cudaStream_t st) {
    return n == 0 || cudaMemcpyAsync(d, h, n, cudaMemcpyHostToDevice, st) == cudaSuccess;
}
bool d2h(void* h, const void* d, size_t n, cudaStream_t st) {
    return n == 0 || cudaMemcpyAsync(h, d, n, cudaMemcpyDeviceToHost, st) == cudaSuccess;
}

}  // namespace
}  // namespace pion

using namespace pion;

extern "C" {

int64_t pion_v_abi_version(void) { return PION_B200_ABI_VERSION; }

int64_t pion_v_isa(void) { return 100; }

void pion_v_pkm_scores_i8(const int8_t* keys, int64_t s_rows, int64_t d_pad,
                          const float* row_scale, const int8_t* q, const float* q_scale,
                          int64_t nq, float* dst) {
    const char* who = "pion_v_pkm_scores_i8";
    if (s_rows <= 0 || nq <= 0) return;
    if (!keys || !row_scale || !q || !q_scale || !dst || d_pad <= 0 || d_pad % 16 != 0 ||
        nq > 65535) {
        fail(who, "bad arguments (d_pad must be a multiple of 16)");
        return;
    }
    pion_b200_ctx* c = default_ctx(who);
    if (!c || use_device(c) != 0) return;
    const size_t kb = (size_t)s_rows * d_pad, qb = (size_t)nq * d_pad, ob = (size_t)nq * s_rows * 4;
    if (ensure(c->scratch, carve_size({kb, (size_t)s_rows * 4, qb, (size_t)nq * 4, ob})) != 0) {
        fail(who, "device memory");
        return;
    }
    Carve cv(c->scratch.ptr);
    int8_t* dk = cv.take<int8_t>(kb);
    float* drs = cv.take<float>(s_rows);
    int8_t* dq = cv.take<int8_t>(qb);
    float* dqs = cv.take<float>(nq);
    float* dd = cv.take<float>((size_t)nq * s_rows);
    cudaStream_t st = c->stream;
    if (!h2d(dk, keys, kb, st) || !h2d(drs, row_scale, s_rows * 4, st) || !h2d(dq, q, qb, st) ||
        !h2d(dqs, q_scale, nq * 4, st)) {
        fail(who, "copy failed");
        return;
    }
    dim3 grid((unsigned)((s_rows + 7) / 8), (unsigned)nq);
    compat::scores_i8_kernel<<<grid, 256, 0, st>>>(dk, s_rows, (int)d_pad, drs, dq, dqs, dd);
    c->launches++;
    if (cudaGetLastError() != cudaSuccess || !d2h(dst, dd, ob, st) || finish_sync(c) != 0)
        fail(who, "launch failed");
}

void pion_v_pkm_scores_f32(const float* keys, int64_t s_rows, int64_t d_pad, const float* q,
                           int64_t nq, float* dst) {
    const char* who = "pion_v_pkm_scores_f32";
    if (s_rows <= 0 || nq <= 0) return;
    if (!keys || !q || !dst || d_pad <= 0 || d_pad % 8 != 0) {
        fail(who, "bad arguments (d_pad must be a multiple of 8)");
        return;
    }
    pion_b200_ctx* c = default_ctx(who);
    if (!c || use_device(c) != 0) return;
    const size_t kb = (size_t)s_rows * d_pad * 4, qb = (size_t)nq * d_pad * 4,
                 ob = (size_t)nq * s_rows * 4;
    if (ensure(c->scratch, carve_size({kb, qb, ob})) != 0) {
        fail(who, "device memory");
        return;
    }
    Carve cv(c->scratch.ptr);
    float* dk = cv.take<float>(kb / 4);
    float* dq = cv.take<float>(qb / 4);
    float* dd = cv.take<float>(ob / 4);
    cudaStream_t st = c->stream;
    if (!h2d(dk, keys, kb, st) || !h2d(dq, q, qb, st)) {
        fail(who, "copy failed");
        return;
    }
    const int64_t threads = s_rows * nq * 8;
    compat::scores_f32_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(
        dk, s_rows, (int)d_pad, dq, (int)nq, dd);
    c->launches++;
    if (cudaGetLastError() != cudaSuccess || !d2h(dst, dd, ob, st) || finish_sync(c) != 0)
        fail(who, "launch failed");
}

void pion_v_pkm_rescore_f32(const float* keys, int64_t d_pad, const float* q, const int32_t* idx,
                            int64_t cnt, float* dst) {
    const char* who = "pion_v_pkm_rescore_f32";
    if (cnt <= 0) return;
    if (!keys || !q || !idx || !dst || d_pad <= 0 || d_pad % 8 != 0) {
        fail(who, "bad arguments (d_pad must be a multiple of 8)");
        return;
    }
    // the key table's extent is implied by the largest index
    int64_t rows = 0;
    for (int64_t t = 0; t < cnt; ++t) {
        if (idx[t] < 0) {
            fail(who, "negative index");
            return;
        }
        rows = idx[t] + 1 > rows ? idx[t] + 1 : rows;
    }
    pion_b200_ctx* c = default_ctx(who);
    if (!c || use_device(c) != 0) return;
    const size_t kb = (size_t)rows * d_pad * 4;
    if (ensure(c->scratch, carve_size({kb, (size_t)d_pad * 4, (size_t)cnt * 4, (size_t)cnt * 4})) !=
        0) {
        fail(who, "device memory");
        return;
    }
    Carve cv(c->scratch.ptr);
    float* dk = cv.take<float>(kb / 4);
    float* dq = cv.take<float>(d_pad);
    int32_t* di = cv.take<int32_t>(cnt);
    float* dd = cv.take<float>(cnt);
    cudaStream_t st = c->stream;
    if (!h2d(dk, keys, kb, st) || !h2d(dq, q, d_pad * 4, st) || !h2d(di, idx, cnt * 4, st)) {
        fail(who, "copy failed");
        return;
    }
    compat::rescore_f32_kernel<<<(unsigned)((cnt * 8 + 255) / 256), 256, 0, st>>>(
        dk, (int)d_pad, dq, di, cnt, dd);
    c->launches++;
    if (cudaGetLastError() != cudaSuccess || !d2h(dst, dd, cnt * 4, st) || finish_sync(c) != 0)
        fail(who, "launch failed");
}

int64_t pion_v_pkm_topk_max(const float* scores, int64_t n, int64_t k, int32_t* out_idx,
                            float* out_val) {
    const char* who = "pion_v_pkm_topk_max";
    const int64_t kk = k < n ? k : n;
    if (kk <= 0) return 0;
    if (!scores || !out_idx || !out_val) return fail(who, "null pointer"), 0;
    if (kk > compat::TK_KMAX || n > INT32_MAX)
        return fail(who, "k must be <= 256 and n < 2^31"), 0;
    pion_b200_ctx* c = default_ctx(who);
    if (!c || use_device(c) != 0) return 0;
    const int nb = (int)((n + compat::TK_BLOCK - 1) / compat::TK_BLOCK);
    const size_t padded = (size_t)nb * compat::TK_BLOCK;
    if (ensure(c->scratch, carve_size({(size_t)n * 4, (size_t)nb * kk * 4, (size_t)nb * 4,
                                       padded * 4, padded * 4, (size_t)nb * 4, (size_t)kk * 4,
                                       (size_t)kk * 4})) != 0)
        return fail(who, "device memory"), 0;
    Carve cv(c->scratch.ptr);
    float* ds = cv.take<float>(n);
    float* blk = cv.take<float>((size_t)nb * kk);
    float* bound = cv.take<float>(nb);
    float* sv = cv.take<float>(padded);
    int32_t* si = cv.take<int32_t>(padded);
    int* cnt = cv.take<int>(nb);
    int32_t* oi = cv.take<int32_t>(kk);
    float* ov = cv.take<float>(kk);
    cudaStream_t st = c->stream;
    if (!h2d(ds, scores, (size_t)n * 4, st)) return fail(who, "copy failed"), 0;
    compat::block_topk_kernel<<<nb, compat::TK_THREADS, 0, st>>>(ds, n, (int)kk, blk);
    compat::prefix_bounds_kernel<<<1, 32, 0, st>>>(blk, nb, (int)kk, bound);
    compat::survivors_kernel<<<nb, compat::TK_THREADS, 0, st>>>(ds, n, (int)kk, bound, sv, si,
                                                                cnt);
    compat::replay_topk_kernel<<<1, 32, 0, st>>>(sv, si, cnt, nb, kk, oi, ov);
    c->launches += 4;
    if (cudaGetLastError() != cudaSuccess || !d2h(out_idx, oi, kk * 4, st) ||
        !d2h(out_val, ov, kk * 4, st) || finish_sync(c) != 0)
        return fail(who, "launch failed"), 0;
    return kk;
}

void pion_v_pkm_sort_desc(float* val, int32_t* idx, int64_t n) {
    const char* who = "pion_v_pkm_sort_desc";
    if (n <= 1) return;
    if (!val || !idx) {
        fail(who, "null pointer");
        return;
    }
    pion_b200_ctx* c = default_ctx(who);
    if (!c || use_device(c) != 0) return;
    if (ensure(c->scratch, carve_size({(size_t)n * 4, (size_t)n * 4})) != 0) {
        fail(who, "device memory");
        return;
    }
    Carve cv(c->scratch.ptr);
    float* dv = cv.take<float>(n);
    int32_t* di = cv.take<int32_t>(n);
    cudaStream_t st = c->stream;
    if (!h2d(dv, val, n * 4, st) || !h2d(di, idx, n * 4, st)) {
        fail(who, "copy failed");
        return;
    }
    compat::sort_desc_kernel<<<1, 32, 0, st>>>(dv, di, n);
    c->launches++;
    if (cudaGetLastError() != cudaSuccess || !d2h(val, dv, n * 4, st) || !d2h(idx, di, n * 4, st) ||
        finish_sync(c) != 0)
        fail(who, "launch failed");
}

int64_t pion_v_pkm_combine_topk(const float* s0, const int32_t* i0, int64_t k0, const float* s1,
                                const int32_t* i1, int64_t k1, int64_t s_cols, int64_t k,
                                int32_t* out_id, float* out_score) {
    const char* who = "pion_v_pkm_combine_topk";
    const int64_t lim = k0 * k1;
    const int64_t cap = k < lim ? k : lim;
    if (cap <= 0) return 0;
    if (!s0 || !i0 || !s1 || !i1 || !out_id || !out_score) return fail(who, "null pointer"), 0;
    pion_b200_ctx* c = default_ctx(who);
    if (!c || use_device(c) != 0) return 0;
    if (ensure(c->scratch, carve_size({(size_t)k0 * 4, (size_t)k0 * 4, (size_t)k1 * 4,
                                       (size_t)k1 * 4, (size_t)cap * 4, (size_t)cap * 4, 8})) != 0)
        return fail(who, "device memory"), 0;
    Carve cv(c->scratch.ptr);
    float* d0 = cv.take<float>(k0);
    int32_t* e0 = cv.take<int32_t>(k0);
    float* d1 = cv.take<float>(k1);
    int32_t* e1 = cv.take<int32_t>(k1);
    int32_t* oi = cv.take<int32_t>(cap);
    float* os = cv.take<float>(cap);
    int64_t* ocnt = cv.take<int64_t>(1);
    cudaStream_t st = c->stream;
    if (!h2d(d0, s0, k0 * 4, st) || !h2d(e0, i0, k0 * 4, st) || !h2d(d1, s1, k1 * 4, st) ||
        !h2d(e1, i1, k1 * 4, st))
        return fail(who, "copy failed"), 0;
    compat::combine_topk_kernel<<<1, 32, 0, st>>>(d0, e0, k0, d1, e1, k1, s_cols, k, oi, os, ocnt);
    c->launches++;
    int64_t got = 0;
    if (cudaGetLastError() != cudaSuccess || !d2h(&got, ocnt, 8, st) || finish_sync(c) != 0)
        return fail(who, "launch failed"), 0;
    if (!d2h(out_id, oi, got * 4, st) || !d2h(out_score, os, got * 4, st) || finish_sync(c) != 0)
        return fail(who, "copy back failed"), 0;
    return got;
}

}  // extern "C"
