// FLAT FP32 cosine KNN on B200 (sm_100a): exact_knn under COSINE.
//
// Reference semantics (pavelhorak/pion):
//   exact_knn  src/commands/vector.mojo:1228-1365: query normalised with a
//     sequential sum of squares, inv = 1/sqrt(ss); score = 1 - dot_f32_4chain(q^, row);
//     k smallest, an equal score never displaces an earlier slot.
//   dot_f32_4chain  src/vector/fp32_scan.mojo:17-38: four 4-lane chains over 16-float
//     strides, ((a0+a1)+(a2+a3)) then a halving-tree lane sum, then a scalar tail;
//     a*b+c as two roundings (fma_mad on x86-64-v2, src/vector/fma_mad.mojo:21).
//   l2_normalize_fp32  src/vector/kernels.mojo:318-357 (rows at COSINE ingest).
//
// Pipeline per batch:
//   1. query_normalize_kernel    exact_knn's normalisation, one thread per query.
//   2. flat_bf16x3_tc_kernel     approximate dots on tcgen05 (kind::f16 with bf16
//                                operands, TMEM accumulators, TMA 128B-swizzled tiles):
//                                every fp32 value is split x = hi + lo into two bf16s
//                                and q.v ~ qh.vh + qh.vl + ql.vh, accumulated in fp32;
//                                each query keeps its top-KC by approximate dot (fused,
//                                no score matrix), with the same sampled lower-bound
//                                pre-pass as the INT8 path.
//   3. merge_lists_kernel        top-KC candidates per query.
//   4. rescore_certify_kernel    exact reference dot (4-chain order) of the KC
//                                candidates, top-k by (distance, id), and a proof that
//                                no other row can rank: every row outside the candidates
//                                has approx <= A_KC, so exact <= A_KC + eps; if
//                                fl(1 - (A_KC + eps)) > the k-th distance, the answer is
//                                exact.  Otherwise the query is flagged.
//   5. exact_scan_kernel         flagged queries only: exact distances of every row on
//                                CUDA cores, then a merge.  Results are exact either way.
#include <cuda_bf16.h>

#include <cstdint>
#include <cstdio>

#include "common.cuh"
#include "exact_fp32.cuh"
#include "internal.h"

namespace pion {
namespace ff32 {

constexpr int BM = 128;             // queries per CTA tile
constexpr int BN = 256;             // index rows per tile
constexpr int BK = 128;             // bytes of K per stage: 64 bf16 elements
constexpr int KEL = BK / 2;         // bf16 elements per stage row
constexpr int STAGES = 4;
constexpr int UMMA_KB = 32;         // bytes of K per tcgen05.mma (16 bf16)
constexpr int A_BYTES = BM * BK;
constexpr int B_BYTES = BN * BK;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_WARPS = 4;
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr uint32_t TMEM_COLS = 2 * BN;
constexpr uint32_t IDESC = make_idesc_bf16(BM, BN);
constexpr size_t SMEM_PIPE_BYTES = 1024 + (size_t)STAGES * STAGE_BYTES + 256;
constexpr size_t STASH_BYTES = 32 * 32 * 4;
constexpr size_t SMEM_BYTES = SMEM_PIPE_BYTES + EPI_WARPS * STASH_BYTES;

struct TcParams {
    const float* thr0;  // optional per-query lower bound on the final KC-th approx dot
    int thr0_stride;
    int64_t n_rows;
    int nq;
    int kc;             // list length kept per (query, split)
    int tile_begin;
    int tile_end;
    int n_splits;
    int kseg;           // 128-byte K blocks per split term (ceil(dim / 64))
    int n_lists;
    int list_base;
    int bound_mode;     // 1: keep one approximate dot per 32-row chunk (threshold pass)
    float* cand_val;
    int32_t* cand_idx;
    int* status;
};

template <int KCAP>
struct ApproxTop {
    TopKDesc<KCAP> top;
    float thr;
    float floor_thr;
};

// One 32-column chunk of approximate dots (fp32 bit patterns in TMEM).
template <int KCAP>
__device__ __forceinline__ void scan_chunk_f(const uint32_t (&r)[32], int64_t col0,
                                             int64_t valid, int kc, uint32_t* stash, int lane,
                                             ApproxTop<KCAP>& st) {
    float mx = __uint_as_float(r[0]);
#pragma unroll
    for (int j = 1; j < 32; ++j) mx = fmaxf(mx, __uint_as_float(r[j]));
    uint32_t mask = 0;
    if (mx > st.thr) {
#pragma unroll
        for (int j = 0; j < 32; ++j) mask |= (__uint_as_float(r[j]) > st.thr ? 1u : 0u) << j;
        if (valid < 32) mask &= valid <= 0 ? 0u : ((1u << valid) - 1u);
    }
    if (!__any_sync(0xffffffffu, mask != 0u)) return;
#pragma unroll
    for (int j = 0; j < 32; ++j) stash[j * 32 + lane] = r[j];
    __syncwarp();
#pragma unroll 1
    while (mask) {
        const int j = __ffs(mask) - 1;
        mask &= mask - 1u;
        const float s = __uint_as_float(stash[j * 32 + lane]);
        if (s > st.thr) {
            st.top.insert(s, (int32_t)(col0 + j));
            st.thr = fmaxf(st.top.kth(kc), st.floor_thr);
        }
    }
    __syncwarp();
}

// Threshold pass: the largest approximate dot of each 32-column chunk (first column on
// ties) is offered to the top list.  The rows offered are distinct, so the KC-th best of
// them is a lower bound of the final KC-th approximate dot.
template <int KCAP>
__device__ __forceinline__ void bound_chunk_f(const uint32_t (&r)[32], int64_t col0,
                                              int64_t valid, int kc, ApproxTop<KCAP>& st) {
    float mx = -INFINITY;
    int jm = -1;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const float v = __uint_as_float(r[j]);
        const bool take = j < valid && (jm < 0 || v > mx);
        mx = take ? v : mx;
        jm = take ? j : jm;
    }
    if (jm >= 0 && mx > st.thr) {
        st.top.insert(mx, (int32_t)(col0 + jm));
        st.thr = fmaxf(st.top.kth(kc), st.floor_thr);
    }
}

// K runs over three segments of the dimension: (qh, vh), (qh, vl), (ql, vh).
template <int KCAP>
__global__ void __launch_bounds__(THREADS, 1)
    flat_bf16x3_tc_kernel(const __grid_constant__ CUtensorMap tmap_qh,
                          const __grid_constant__ CUtensorMap tmap_ql,
                          const __grid_constant__ CUtensorMap tmap_rh,
                          const __grid_constant__ CUtensorMap tmap_rl, TcParams p) {
    const int kblocks = 3 * p.kseg;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * A_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    uint32_t* stash_all = reinterpret_cast<uint32_t*>(smem + (SMEM_PIPE_BYTES - 1024));

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int qt = blockIdx.x;
    const int split = blockIdx.y;
    const int span = p.tile_end - p.tile_begin;
    const int t_begin = p.tile_begin + (int)((int64_t)span * split / p.n_splits);
    const int t_end = p.tile_begin + (int)((int64_t)span * (split + 1) / p.n_splits);
    const int my_tiles = t_end - t_begin;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 32 * EPI_WARPS);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {  // TMA producer
            tma_prefetch_desc(&tmap_qh);
            tma_prefetch_desc(&tmap_ql);
            tma_prefetch_desc(&tmap_rh);
            tma_prefetch_desc(&tmap_rl);
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_parity[STAGES];
            bool issued[STAGES];
            for (int s = 0; s < STAGES; ++s) issued[s] = false, issued_parity[s] = 0;
            bool ok = true;
            for (int t = 0; t < my_tiles && ok; ++t) {
                const int row0 = (t_begin + t) * BN;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, abort_flag)) {
                        ok = false;
                        break;
                    }
                    const int seg = kb / p.kseg;
                    const int kx = (kb - seg * p.kseg) * KEL;
                    mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
                    tma_load_2d(sA + stage * A_BYTES, seg < 2 ? &tmap_qh : &tmap_ql, &full[stage],
                                kx, qt * BM);
                    tma_load_2d(sB + stage * B_BYTES, seg == 1 ? &tmap_rl : &tmap_rh,
                                &full[stage], kx, row0);
                    issued[stage] = true;
                    issued_parity[stage] = phase;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            for (int s = 0; s < STAGES; ++s)
                if (issued[s]) mbar_wait(&full[s], issued_parity[s], p.status, nullptr);
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            int stage = 0;
            uint32_t phase = 0;
            for (int t = 0; t < my_tiles; ++t) {
                const int buf = t & 1;
                const uint32_t use = (uint32_t)(t >> 1);
                if (!mbar_wait(&tempty[buf], (use & 1u) ^ 1u, p.status, abort_flag)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(buf * BN);
                bool ok = true;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&full[stage], phase, p.status, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + stage * A_BYTES);
                    const uint32_t b0 = smem_u32(sB + stage * B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < BK / UMMA_KB; ++kk)
                        mma_bf16(d_tmem, make_sw128_kmajor_desc(a0 + kk * UMMA_KB),
                                 make_sw128_kmajor_desc(b0 + kk * UMMA_KB), IDESC,
                                 (kb | kk) != 0 ? 1u : 0u);
                    tc_commit(&empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                tc_commit(&tfull[buf]);
            }
            tc_commit(drain);
            mbar_wait(drain, 0, p.status, nullptr);
        }
    } else {
        // epilogue: one thread per query (TMEM lane), all 256 columns of each tile
        const int ew = warp - 2;
        uint32_t* stash = stash_all + ew * (STASH_BYTES / 4);
        const int lg = warp & 3;
        const int row = lg * 32 + lane;
        const int q = qt * BM + row;
        const bool q_ok = q < p.nq;
        ApproxTop<KCAP> st;
        st.top.init();
        st.floor_thr = -INFINITY;
        if (q_ok && p.thr0) {
            const float t0 = p.thr0[(size_t)q * p.thr0_stride];
            if (t0 > -INFINITY) st.floor_thr = nextafterf(t0, -INFINITY);
        }
        st.thr = q_ok ? st.floor_thr : INFINITY;
        for (int t = 0; t < my_tiles; ++t) {
            const int buf = t & 1;
            const uint32_t use = (uint32_t)(t >> 1);
            const int tile = t_begin + t;
            const int64_t col0 = (int64_t)tile * BN;
            const int64_t valid = p.n_rows - col0;
            const bool got = mbar_wait(&tfull[buf], use & 1u, p.status, abort_flag);
            if (!__all_sync(0xffffffffu, got)) break;
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(lg * 32) << 16) + (uint32_t)(buf * BN);
            uint32_t ra[32];
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                __syncwarp();
                tmem_ld32(taddr + (uint32_t)(c * 32), ra);
                tmem_ld_wait_regs(ra);
                if (p.bound_mode)
                    bound_chunk_f<KCAP>(ra, col0 + c * 32, valid - c * 32, p.kc, st);
                else
                    scan_chunk_f<KCAP>(ra, col0 + c * 32, valid - c * 32, p.kc, stash, lane, st);
            }
            tc_fence_before();
            mbar_arrive(&tempty[buf]);
        }
        if (q_ok) {
            const size_t base = ((size_t)q * p.n_lists + p.list_base + split) * p.kc;
#pragma unroll
            for (int j = 0; j < KCAP; ++j)
                if (j < p.kc) {
                    p.cand_val[base + j] = st.top.v[j];
                    p.cand_idx[base + j] = st.top.i[j];
                }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// Staged row pitch in floats: 16-byte aligned rows for dim % 4 == 0 (and rows 4 banks
// apart), else one float of padding.
__host__ __device__ inline int normalize_pitch(int dim) {
    return (dim & 3) == 0 ? dim + 4 : dim + 1;
}

// exact_knn's query normalisation (src/commands/vector.mojo:1254-1260): a sequential
// sum of squares, inv = 1/sqrt(ss) (1 if ss == 0), y = x * inv.  A CTA stages ROWS
// queries in shared memory with coalesced loads (rows 16-byte aligned when dim % 4 == 0);
// one thread per query runs the sequential sum, reading four elements per shared load so
// that only the addition chain is serial; all threads write the result.  qnorm (|y|,
// which only feeds the certification bound, whose 1 % slack covers its rounding) is a
// warp reduction.  With `codes` (dim % 64 == 0) it also writes the normalised query's
// sign code (bit b of word w = y[64w + b] > 0) and, with `pm`, its +-1 bytes: the BQ
// query encoding.
__global__ void query_normalize_kernel(const float* __restrict__ q, int nq, int dim, int rows,
                                       float* __restrict__ out, float* __restrict__ qnorm,
                                       int8_t* __restrict__ pm, uint64_t* __restrict__ codes) {
    extern __shared__ __align__(16) float qsm[];  // [rows][pitch]
    __shared__ float inv_s[32];
    const int q0 = blockIdx.x * rows;
    const int nr = min(rows, nq - q0);
    const int pitch = normalize_pitch(dim);
    if ((dim & 3) == 0) {  // 128-bit loads, all of a thread's in flight together
        const int d4 = dim >> 2;
#pragma unroll 4
        for (int i = threadIdx.x; i < nr * d4; i += blockDim.x) {
            const int r = i / d4, c = i - r * d4;
            reinterpret_cast<float4*>(qsm + r * pitch)[c] =
                reinterpret_cast<const float4*>(q + (size_t)(q0 + r) * dim)[c];
        }
    } else {
        for (int r = 0; r < nr; ++r)
            for (int d = threadIdx.x; d < dim; d += blockDim.x)
                qsm[r * pitch + d] = q[(size_t)(q0 + r) * dim + d];
    }
    __syncthreads();
    if (threadIdx.x < nr) {
        const float* x = qsm + threadIdx.x * pitch;
        float ss = 0.0f;
        if ((dim & 3) == 0) {
            const float4* x4 = reinterpret_cast<const float4*>(x);
#pragma unroll 8
            for (int d4 = 0; d4 < (dim >> 2); ++d4) {
                const float4 v = x4[d4];
                ss = __fadd_rn(ss, __fmul_rn(v.x, v.x));
                ss = __fadd_rn(ss, __fmul_rn(v.y, v.y));
                ss = __fadd_rn(ss, __fmul_rn(v.z, v.z));
                ss = __fadd_rn(ss, __fmul_rn(v.w, v.w));
            }
        } else {
#pragma unroll 16
            for (int d = 0; d < dim; ++d) ss = __fadd_rn(ss, __fmul_rn(x[d], x[d]));
        }
        inv_s[threadIdx.x] = ss > 0.0f ? __fdiv_rn(1.0f, __fsqrt_rn(ss)) : 1.0f;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < nr * dim; i += blockDim.x) {
        const int r = i / dim, d = i - r * dim;
        out[(size_t)(q0 + r) * dim + d] = __fmul_rn(qsm[r * pitch + d], inv_s[r]);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int r = warp; r < nr; r += nw) {
        const float inv = inv_s[r];
        float n2 = 0.0f;
        for (int d = lane; d < dim; d += 32) {
            const float y = __fmul_rn(qsm[r * pitch + d], inv);
            n2 = fmaf(y, y, n2);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) n2 += __shfl_xor_sync(0xffffffffu, n2, o);
        if (lane == 0) qnorm[q0 + r] = sqrtf(n2);
    }
    if (codes) {  // a warp per (row, 64-element word)
        const int words = dim / 64;
        for (int t = warp; t < nr * words; t += nw) {
            const int r = t / words, wd = t - r * words;
            const float inv = inv_s[r];
            const float a = __fmul_rn(qsm[r * pitch + wd * 64 + lane], inv);
            const float b = __fmul_rn(qsm[r * pitch + wd * 64 + 32 + lane], inv);
            const unsigned lo = __ballot_sync(0xffffffffu, a > 0.0f);
            const unsigned hi = __ballot_sync(0xffffffffu, b > 0.0f);
            if (pm) {
                pm[(size_t)(q0 + r) * dim + wd * 64 + lane] = a > 0.0f ? 1 : -1;
                pm[(size_t)(q0 + r) * dim + wd * 64 + 32 + lane] = b > 0.0f ? 1 : -1;
            }
            if (lane == 0) codes[(size_t)(q0 + r) * words + wd] = ((uint64_t)hi << 32) | lo;
        }
    }
}

// l2_normalize_fp32 (src/vector/kernels.mojo:318-357) of whole rows: four lanes of
// sequential sums (lane l takes the elements l, l+4, ...), combined (s0 + s2) + (s1 + s3),
// the scalar tail added in order, inv = 1/sqrt; a zero row passes through.  A CTA stages
// ROWS rows in shared memory with coalesced loads (in place is allowed: every element is
// read before any is written), four threads per row run the lane sums, all threads write.
__global__ void l2_normalize_rows_kernel(const float* src, int64_t n_rows, int dim, int rows,
                                         float* dst, float* __restrict__ norms) {
    extern __shared__ float xs[];  // [rows][dim + 1]
    __shared__ float lane_s[32 * 4];
    __shared__ float inv_s[32];
    const int64_t r0 = (int64_t)blockIdx.x * rows;
    const int nr = (int)min((int64_t)rows, n_rows - r0);
    const int pitch = dim + 1;
    for (int r = 0; r < nr; ++r)
        for (int d = threadIdx.x; d < dim; d += blockDim.x)
            xs[r * pitch + d] = src[(size_t)(r0 + r) * dim + d];
    __syncthreads();
    const int main_end = dim & ~3;
    if (threadIdx.x < 4 * nr) {
        const int r = threadIdx.x >> 2, l = threadIdx.x & 3;
        const float* x = xs + r * pitch;
        float acc = 0.0f;
        for (int d = l; d < main_end; d += 4) acc = __fadd_rn(acc, __fmul_rn(x[d], x[d]));
        lane_s[threadIdx.x] = acc;
    }
    __syncthreads();
    if (threadIdx.x < nr) {
        const int r = threadIdx.x;
        const float* x = xs + r * pitch;
        const float* a = lane_s + 4 * r;
        float ns = __fadd_rn(__fadd_rn(a[0], a[2]), __fadd_rn(a[1], a[3]));
        for (int d = main_end; d < dim; ++d) ns = __fadd_rn(ns, __fmul_rn(x[d], x[d]));
        const float inv = ns <= 0.0f ? 0.0f : __fdiv_rn(1.0f, __fsqrt_rn(ns));
        inv_s[r] = ns <= 0.0f ? -1.0f : inv;  // -1: zero row, copied unchanged
        if (norms) norms[r0 + r] = ns <= 0.0f ? 0.0f : __fmul_rn(__fsqrt_rn(ns), inv);
    }
    __syncthreads();
    for (int r = 0; r < nr; ++r) {
        const float inv = inv_s[r];
        for (int d = threadIdx.x; d < dim; d += blockDim.x) {
            const float x = xs[r * pitch + d];
            dst[(size_t)(r0 + r) * dim + d] = inv < 0.0f ? x : __fmul_rn(x, inv);
        }
    }
}

// Row L2 norms (for the certification bound) without normalising.
__global__ void row_norms_kernel(const float* __restrict__ rows, int64_t n_rows, int dim,
                                 float* __restrict__ norms) {
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (r >= n_rows) return;
    const int lane = threadIdx.x & 31;
    float s = 0.0f;
    for (int d = lane; d < dim; d += 32) s = fmaf(rows[r * dim + d], rows[r * dim + d], s);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) norms[r] = sqrtf(s);
}

__global__ void max_reduce_kernel(const float* __restrict__ x, int64_t n, float* out) {
    float m = 0.0f;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        m = fmaxf(m, x[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) atomicMax(reinterpret_cast<int*>(out), __float_as_int(m));
}

// One CTA per query: exact 4-chain dots of the kc candidates (rows prefetched into L2
// first), then warp 0 selects the k best by (distance, id) and certifies.  dim % 16 == 0:
// 128 threads, four lanes per candidate (dot4chain_quad: 128-bit loads, twelve in
// flight, the query in shared memory); otherwise 256 threads, a half-warp per candidate
// (dot4chain_half).
__global__ void __launch_bounds__(256) rescore_certify_kernel(
    const float* __restrict__ rows, int dim, const float* __restrict__ qn,
    const float* __restrict__ qnorm, float row_norm_max, const float* __restrict__ cand_v,
    const int32_t* __restrict__ cand_i, int nq, int kc, int k, int64_t id_base,
    float* __restrict__ out_d, int32_t* __restrict__ out_i, int* __restrict__ flagged,
    int* __restrict__ n_flagged, int force_exact) {
    extern __shared__ __align__(16) float sm[];
    const int q = blockIdx.x;
    if (q >= nq) return;
    const int lane = threadIdx.x & 31;
    const bool quad = (dim & 15) == 0;
    float* dist = quad ? sm + dim : sm;
    int32_t* ids = reinterpret_cast<int32_t*>(dist + kc);
    const float* qv = qn + (size_t)q * dim;
    const int hw = threadIdx.x >> 4;  // half-warp of the CTA
    const int hl = lane & 15;
    const unsigned hmask = (lane >> 4) ? 0xffff0000u : 0x0000ffffu;
    if ((dim & 3) == 0)
        for (int j = threadIdx.x; j < kc; j += blockDim.x) {
            const int32_t id = cand_i[(size_t)q * kc + j];
            if (id >= 0) prefetch_row_f32_l2(rows + (size_t)id * dim, dim);
        }
    if (quad) {
        float4* qs4 = reinterpret_cast<float4*>(sm);
        for (int c = threadIdx.x; c < (dim >> 2); c += blockDim.x)
            qs4[c] = reinterpret_cast<const float4*>(qv)[c];
        __syncthreads();
        const int quads = blockDim.x >> 2;
        for (int j0 = 0; j0 < kc; j0 += quads) {  // every lane of the warp takes part
            const int j = j0 + (threadIdx.x >> 2);
            const int32_t id = j < kc ? cand_i[(size_t)q * kc + j] : -1;
            const float s = dot4chain_quad<12>(qs4, id >= 0 ? rows + (size_t)id * dim : nullptr,
                                               dim);
            if ((threadIdx.x & 3) == 0 && j < kc) {
                dist[j] = id >= 0 ? __fsub_rn(1.0f, s) : INFINITY;
                ids[j] = id;
            }
        }
    } else {
        const int halves = blockDim.x >> 4;
        for (int j0 = 0; j0 < kc; j0 += halves) {
            const int j = j0 + hw;
            const int32_t id = j < kc ? cand_i[(size_t)q * kc + j] : -1;
            float d = INFINITY;
            if (id >= 0) {
                const float s = dot4chain_half(qv, rows + (size_t)id * dim, dim, hl, hmask);
                d = __fsub_rn(1.0f, s);
            }
            if (hl == 0 && j < kc) {
                dist[j] = d;
                ids[j] = id;
            }
        }
    }
    __syncthreads();
    if (threadIdx.x >= 32) return;
    int n_valid = 0;
    for (int j = 0; j < kc; ++j) n_valid += ids[j] >= 0 ? 1 : 0;
    __syncwarp();
    // k rounds of warp arg-min over the kc candidates
    float kth_d = INFINITY;
    for (int r = 0; r < k; ++r) {
        float bd = INFINITY;
        int32_t bi = -1;
        int bs = -1;
        for (int j = lane; j < kc; j += 32)
            if (ids[j] >= 0 && (bs < 0 || better_asc(dist[j], ids[j], bd, bi))) {
                bd = dist[j];
                bi = ids[j];
                bs = j;
            }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float od = __shfl_xor_sync(0xffffffffu, bd, o);
            const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            const int os = __shfl_xor_sync(0xffffffffu, bs, o);
            if (os >= 0 && (bs < 0 || better_asc(od, oi, bd, bi))) {
                bd = od;
                bi = oi;
                bs = os;
            }
        }
        if (lane == 0) {
            out_d[(size_t)q * k + r] = bs >= 0 ? bd : INFINITY;
            out_i[(size_t)q * k + r] = bs >= 0 ? (int32_t)(bi + id_base) : -1;
        }
        if (bs >= 0) {
            kth_d = bd;
            if (lane == (bs & 31)) ids[bs] = -2;  // taken
        } else {
            kth_d = INFINITY;
        }
        __syncwarp();
    }
    // Certificate: rows outside the candidates have approx dot <= A_KC (the kc-th
    // approximate score), so their exact dot <= A_KC + eps.
    if (lane == 0) {
        bool ok = true;
        if (n_valid >= kc) {
            const float a_kc = cand_v[(size_t)q * kc + kc - 1];
            // Split error: x = hi + lo + e with |e| <= 2^-18 |x|, so each product misses
            // at most ~3 * 2^-18 |q_i v_i| (lo*lo and the e terms) < 2^-15 |q_i v_i|.
            // fp32 accumulation in the MMA over 3 * dim terms (<= 2^-14) and in the
            // reference's 4 chains (<= 2^-15), all relative to sum |q_i v_i| <=
            // |q| * max|v| (Cauchy-Schwarz).
            const float eps = (0x1p-15f + 0x1p-14f + 0x1p-15f) * qnorm[q] * row_norm_max * 1.01f;
            const float best_outside = __fsub_rd(1.0f, __fadd_ru(a_kc, eps));
            ok = (kth_d < INFINITY) && best_outside > kth_d;
        }
        if (!ok || force_exact) flagged[atomicAdd(n_flagged, 1)] = q;
    }
}

// Flagged queries: exact distances of every row.  Work item = (flagged slot, chunk
// of rows); each warp scores two rows at a time (one per half) and keeps a top-k in
// registers of lane 0 of each half; the CTA merges its 16 half-lists into one list
// per item.  Persistent: exits at once when nothing is flagged.
constexpr int EX_THREADS = 256;
constexpr int EX_KMAX = 64;

template <bool L2>
__global__ void __launch_bounds__(EX_THREADS)
    exact_scan_kernel(const float* __restrict__ rows, int64_t n_rows, int dim,
                      const float* __restrict__ qn, const int* __restrict__ flagged,
                      const int* __restrict__ n_flagged, int n_chunks, int k,
                      float* __restrict__ chunk_d, int32_t* __restrict__ chunk_i) {
    __shared__ float ld[16 * EX_KMAX];
    __shared__ int32_t li[16 * EX_KMAX];
    __shared__ int item_s;
    const int nf = *n_flagged;
    const int total = nf * n_chunks;
    const int w = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int half = lane >> 4;
    const int hl = lane & 15;
    const unsigned hmask = half ? 0xffff0000u : 0x0000ffffu;
    const int slot = w * 2 + half;  // 16 half-warps
    const int64_t chunk_rows = (n_rows + n_chunks - 1) / n_chunks;
    for (int item = blockIdx.x; item < total; item += gridDim.x) {
        const int f = item / n_chunks;
        const int c = item % n_chunks;
        const int q = flagged[f];
        const float* qv = qn + (size_t)q * dim;
        const int64_t r0 = (int64_t)c * chunk_rows;
        const int64_t r1 = r0 + chunk_rows < n_rows ? r0 + chunk_rows : n_rows;
        // list in shared memory, maintained by lane 0 of the half (sorted asc)
        float* my_d = ld + slot * EX_KMAX;
        int32_t* my_i = li + slot * EX_KMAX;
        if (hl == 0)
            for (int j = 0; j < k; ++j) {
                my_d[j] = INFINITY;
                my_i[j] = -1;
            }
        __syncwarp();
        for (int64_t r = r0 + slot; r < r1 + 16; r += 16) {
            // every half-warp of the warp iterates the same number of times
            const bool valid = r < r1;
            float dd = INFINITY;
            if (valid)
                dd = L2 ? l2sq4chain_half(qv, rows + r * dim, dim, hl, hmask)
                        : __fsub_rn(1.0f, dot4chain_half(qv, rows + r * dim, dim, hl, hmask));
            else __syncwarp(hmask);
            if (valid && hl == 0 && better_asc(dd, (int32_t)r, my_d[k - 1], my_i[k - 1])) {
                int j = k - 1;
                while (j > 0 && better_asc(dd, (int32_t)r, my_d[j - 1], my_i[j - 1])) {
                    my_d[j] = my_d[j - 1];
                    my_i[j] = my_i[j - 1];
                    --j;
                }
                my_d[j] = dd;
                my_i[j] = (int32_t)r;
            }
            if (r >= r1) break;
        }
        __syncthreads();
        if (w == 0) {  // merge the 16 sorted half-lists into this item's list
            int cur = 0;
            for (int j = 0; j < k; ++j) {
                float bd = lane < 16 && cur < k ? ld[lane * EX_KMAX + cur] : INFINITY;
                int32_t bi = lane < 16 && cur < k ? li[lane * EX_KMAX + cur] : -1;
                int bl = lane < 16 ? lane : -1;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float od = __shfl_xor_sync(0xffffffffu, bd, o);
                    const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    const int ol = __shfl_xor_sync(0xffffffffu, bl, o);
                    if (ol >= 0 && (bl < 0 || better_asc(od, oi, bd, bi) ||
                                    (od == bd && oi == bi && ol < bl))) {
                        bd = od;
                        bi = oi;
                        bl = ol;
                    }
                }
                if (lane == bl) ++cur;
                if (lane == 0) {
                    chunk_d[((size_t)f * n_chunks + c) * k + j] = bd;
                    chunk_i[((size_t)f * n_chunks + c) * k + j] = bi;
                }
            }
        }
        __syncthreads();
    }
    (void)item_s;
}

// Flagged queries: merge the chunk lists and overwrite the query's result row.
__global__ void exact_merge_kernel(const float* __restrict__ chunk_d,
                                   const int32_t* __restrict__ chunk_i,
                                   const int* __restrict__ flagged, const int* __restrict__ n_flagged,
                                   int n_chunks, int k, int64_t id_base, float* __restrict__ out_d,
                                   int32_t* __restrict__ out_i) {
    const int f = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (f >= *n_flagged) return;
    const int lane = threadIdx.x & 31;
    const int q = flagged[f];
    // lists are short (n_chunks <= 32): lane l owns list l
    int cur = 0;
    for (int j = 0; j < k; ++j) {
        const bool has = lane < n_chunks && cur < k;
        float bd = has ? chunk_d[((size_t)f * n_chunks + lane) * k + cur] : INFINITY;
        int32_t bi = has ? chunk_i[((size_t)f * n_chunks + lane) * k + cur] : -1;
        int bl = lane < n_chunks ? lane : -1;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float od = __shfl_xor_sync(0xffffffffu, bd, o);
            const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            const int ol = __shfl_xor_sync(0xffffffffu, bl, o);
            if (ol >= 0 && (bl < 0 || better_asc(od, oi, bd, bi) ||
                            (od == bd && oi == bi && ol < bl))) {
                bd = od;
                bi = oi;
                bl = ol;
            }
        }
        if (lane == bl) ++cur;
        if (lane == 0) {
            out_d[(size_t)q * k + j] = bd;
            out_i[(size_t)q * k + j] = bi >= 0 ? (int32_t)(bi + id_base) : -1;
        }
    }
}

// ------------------------------------------------------------- one query scan
// exact_knn for ONE query as an HBM stream (COSINE: 1 - dot_f32_4chain(q^, row)).  Four
// lanes per row; lane j owns chain j of the reference's 4 x 4 accumulators (elements
// 16 i + 4 j .. 16 i + 4 j + 3), so every step is one 128-bit non-allocating load of the
// row and one shared-memory load of the query.  A 4 x 4 transpose across the group
// then gives lane l the l-th lane of every chain, t[l] = (c0 + c1) + (c2 + c3), and the
// lane sum (t0 + t2) + (t1 + t3): src/vector/fp32_scan.mojo:17-38 in order.
constexpr int S1_THREADS = 128;
constexpr int S1_GROUPS = S1_THREADS / 4;  // rows in flight per CTA (one list each)
constexpr int S1_UNROLL = 12;              // 16-element steps in flight per lane
constexpr int S1_MAX_DIM = 16384;

template <int KCAP>
__global__ void __launch_bounds__(S1_THREADS)
    flat_f32_scan1_kernel(const float* __restrict__ rows, int64_t n_rows, int dim,
                          const float* __restrict__ qn, int k, int64_t rows_per_cta,
                          float* cand_d, int32_t* cand_i) {
    extern __shared__ __align__(16) float s1_smem[];
    float4* qv = reinterpret_cast<float4*>(s1_smem);  // dim / 4
    float* lv = s1_smem + dim;                        // [S1_GROUPS][KCAP] of -distance
    int32_t* li = reinterpret_cast<int32_t*>(lv + S1_GROUPS * KCAP);
    for (int c = threadIdx.x; c < (dim >> 2); c += S1_THREADS)
        qv[c] = reinterpret_cast<const float4*>(qn)[c];
    __syncthreads();
    const int g = threadIdx.x >> 2;
    const int j = threadIdx.x & 3;
    const int64_t r0 = (int64_t)blockIdx.x * rows_per_cta;
    int64_t r1 = r0 + rows_per_cta;
    if (r1 > n_rows) r1 = n_rows;
    TopKDesc<KCAP> top;  // (-distance desc, id asc) == (distance asc, id asc)
    top.init();
    float thr = -INFINITY;
    // Warp-uniform trip count (rows past r1 are masked), so the full-warp shuffles of
    // dot4chain_quad always see all 32 lanes.
    for (int64_t base = r0; base < r1; base += S1_GROUPS) {
        const int64_t r = base + g;
        const bool valid = r < r1;
        const float dot = dot4chain_quad<S1_UNROLL>(qv, valid ? rows + r * dim : nullptr, dim);
        if (valid && j == 0) {
            const float neg = -__fsub_rn(1.0f, dot);
            if (neg > thr) {
                top.insert(neg, (int32_t)r);
                thr = top.kth(k);
            }
        }
    }
    if (j == 0) {
#pragma unroll
        for (int e = 0; e < KCAP; ++e) {
            lv[g * KCAP + e] = top.v[e];
            li[g * KCAP + e] = top.i[e];
        }
    }
    __syncthreads();
    // Warp 0 merges the CTA's S1_GROUPS sorted lists (lane = list) into k.
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        int cur = 0;
        for (int e = 0; e < k; ++e) {
            float bv = cur < KCAP ? lv[lane * KCAP + cur] : -INFINITY;
            int32_t bi = cur < KCAP ? li[lane * KCAP + cur] : -1;
            int bl = lane;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
                const int ol = __shfl_xor_sync(0xffffffffu, bl, o);
                if (better_desc(ov, oi, bv, bi) || (ov == bv && oi == bi && ol < bl)) {
                    bv = ov;
                    bi = oi;
                    bl = ol;
                }
            }
            if (lane == bl) ++cur;
            if (lane == 0) {
                cand_d[(size_t)blockIdx.x * k + e] = -bv;  // padding: +inf
                cand_i[(size_t)blockIdx.x * k + e] = bi;
            }
        }
    }
}

}  // namespace ff32

// =========================================================== host launchers ==

bool ff32_scan1_supported(int dim, int k) {
    return dim % 16 == 0 && dim <= ff32::S1_MAX_DIM && k >= 1 && k <= 64;
}

// One wave: 115 registers a thread leave room for four 128-thread CTAs per SM (a second
// wave doubled the lists the merge reads: 145 -> 139 us per search at 100K rows).
int ff32_scan1_ctas(int64_t n_rows, int num_sms) {
    int64_t ctas = (int64_t)num_sms * 4;
    const int64_t min_rows = 2 * ff32::S1_GROUPS;
    if (ctas * min_rows > n_rows) ctas = (n_rows + min_rows - 1) / min_rows;
    return (int)(ctas < 1 ? 1 : ctas);
}

template <int KCAP>
static int launch_scan1_k(const float* rows, int64_t n_rows, int dim, const float* qn, int k,
                          int ctas, float* cand_d, int32_t* cand_i, cudaStream_t st) {
    const size_t smem = (size_t)dim * 4 + (size_t)ff32::S1_GROUPS * KCAP * 8;
    if (smem > 48 * 1024 &&
        set_smem_limit((const void*)ff32::flat_f32_scan1_kernel<KCAP>, (int)smem) != 0)
        return PION_B200_ECUDA;
    const int64_t per = (n_rows + ctas - 1) / ctas;
    ff32::flat_f32_scan1_kernel<KCAP><<<ctas, ff32::S1_THREADS, smem, st>>>(rows, n_rows, dim, qn,
                                                                           k, per, cand_d, cand_i);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int launch_flat_f32_scan1(const float* rows, int64_t n_rows, int dim, const float* qn, int k,
                          int ctas, float* cand_d, int32_t* cand_i, cudaStream_t st) {
    if (!ff32_scan1_supported(dim, k) || n_rows <= 0) return PION_B200_ESHAPE;
    if (k <= 16) return launch_scan1_k<16>(rows, n_rows, dim, qn, k, ctas, cand_d, cand_i, st);
    if (k <= 32) return launch_scan1_k<32>(rows, n_rows, dim, qn, k, ctas, cand_d, cand_i, st);
    return launch_scan1_k<64>(rows, n_rows, dim, qn, k, ctas, cand_d, cand_i, st);
}

int ff32_tile_rows() { return ff32::BN; }
int ff32_query_tile() { return ff32::BM; }
int ff32_k_elems() { return ff32::KEL; }
int ff32_kc(int k) { return k <= 16 ? 32 : 64; }

// Rows staged per CTA by the normalisation kernels: up to 8, within 96 KB of shared
// memory (one row of the largest supported dim, 16384, takes 64 KB).
static int staged_rows(int dim) {
    const int per = (int)((96 * 1024) / ((size_t)ff32::normalize_pitch(dim) * 4));
    return per < 1 ? 1 : per > 8 ? 8 : per;
}

template <typename K>
static bool allow_big_smem(K kernel) {
    return set_smem_limit((const void*)kernel, 200 * 1024) == 0;
}

int launch_query_normalize(const float* q, int nq, int dim, float* out, float* qnorm,
                           cudaStream_t st, int8_t* pm, uint64_t* codes) {
    if (nq <= 0) return 0;
    if (codes && dim % 64 != 0) return PION_B200_ESHAPE;
    if (!allow_big_smem(ff32::query_normalize_kernel)) return PION_B200_ECUDA;
    const int rows = staged_rows(dim);
    const size_t smem = (size_t)rows * ff32::normalize_pitch(dim) * 4;
    ff32::query_normalize_kernel<<<(nq + rows - 1) / rows, 256, smem, st>>>(
        q, nq, dim, rows, out, qnorm, pm, codes);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int launch_l2_normalize_rows(const float* src, int64_t n_rows, int dim, float* dst, float* norms,
                             cudaStream_t st) {
    if (n_rows <= 0) return 0;
    if (!allow_big_smem(ff32::l2_normalize_rows_kernel)) return PION_B200_ECUDA;
    const int rows = staged_rows(dim);
    const size_t smem = (size_t)rows * (dim + 1) * 4;
    ff32::l2_normalize_rows_kernel<<<(unsigned)((n_rows + rows - 1) / rows), 256, smem, st>>>(
        src, n_rows, dim, rows, dst, norms);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int launch_row_norms(const float* rows, int64_t n_rows, int dim, float* norms, cudaStream_t st) {
    if (n_rows <= 0) return 0;
    ff32::row_norms_kernel<<<(unsigned)((n_rows + 7) / 8), 256, 0, st>>>(rows, n_rows, dim, norms);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int launch_max_reduce(const float* x, int64_t n, float* out, cudaStream_t st) {
    if (cudaMemsetAsync(out, 0, sizeof(float), st) != cudaSuccess) return PION_B200_ECUDA;
    if (n <= 0) return 0;
    ff32::max_reduce_kernel<<<256, 256, 0, st>>>(x, n, out);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

template <int KCAP>
static int launch_bf16x3_k(const Ff32TcLaunch& L, const ff32::TcParams& p, int n_qt,
                           cudaStream_t st) {
    if (set_smem_limit((const void*)ff32::flat_bf16x3_tc_kernel<KCAP>, (int)ff32::SMEM_BYTES) != 0)
        return PION_B200_ECUDA;
    dim3 grid(n_qt, p.n_splits);
    ff32::flat_bf16x3_tc_kernel<KCAP><<<grid, ff32::THREADS, ff32::SMEM_BYTES, st>>>(
        *L.tmap_qh, *L.tmap_ql, *L.tmap_rh, *L.tmap_rl, p);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

// Split fp32 values into bf16 pairs: hi = bf16(x), lo = bf16(x - hi) (x - hi is exact).
__global__ void split_bf16_kernel(const float* __restrict__ x, size_t n,
                                  __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        const float v = x[i];
        const __nv_bfloat16 h = __float2bfloat16_rn(v);
        hi[i] = h;
        lo[i] = __float2bfloat16_rn(v - __bfloat162float(h));
    }
}

int launch_split_bf16(const float* x, size_t n, void* hi, void* lo, cudaStream_t st) {
    if (n == 0) return 0;
    size_t blocks = (n + 255) / 256;
    if (blocks > 65536) blocks = 65536;
    split_bf16_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, n, static_cast<__nv_bfloat16*>(hi),
                                                        static_cast<__nv_bfloat16*>(lo));
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int launch_flat_bf16x3_tc(const Ff32TcLaunch& L, cudaStream_t st) {
    ff32::TcParams p;
    p.thr0 = L.thr0;
    p.thr0_stride = L.thr0_stride;
    p.n_rows = L.n_rows;
    p.nq = L.nq;
    p.kc = L.kc;
    p.tile_begin = L.tile_begin;
    p.tile_end = L.tile_end;
    p.n_splits = L.n_splits;
    p.kseg = (L.dim + ff32::KEL - 1) / ff32::KEL;
    p.n_lists = L.n_lists;
    p.list_base = L.list_base;
    p.bound_mode = L.bound_mode;
    p.cand_val = L.cand_val;
    p.cand_idx = L.cand_idx;
    p.status = L.status;
    if (p.tile_end <= p.tile_begin || p.n_splits < 1 || p.list_base + p.n_splits > p.n_lists)
        return PION_B200_ESHAPE;
    const int n_qt = (L.nq + ff32::BM - 1) / ff32::BM;
    switch (L.kc) {
        case 32: return launch_bf16x3_k<32>(L, p, n_qt, st);
        case 64: return launch_bf16x3_k<64>(L, p, n_qt, st);
        default: return PION_B200_ESHAPE;
    }
}

int launch_rescore_certify(const float* rows, int dim, const float* qn, const float* qnorm,
                           float row_norm_max, const float* cand_v, const int32_t* cand_i, int nq,
                           int kc, int k, int64_t id_base, float* out_d, int32_t* out_i,
                           int* flagged, int* n_flagged, int force_exact, cudaStream_t st) {
    if (nq <= 0) return 0;
    const bool quad = dim % 16 == 0;
    const size_t smem = (size_t)kc * 8 + (quad ? (size_t)dim * 4 : 0);
    if (smem > 48 * 1024 &&
        set_smem_limit((const void*)ff32::rescore_certify_kernel, (int)smem) != 0)
        return PION_B200_ECUDA;
    ff32::rescore_certify_kernel<<<nq, quad ? 128 : 256, smem, st>>>(rows, dim, qn, qnorm, row_norm_max,
                                                        cand_v, cand_i, nq, kc, k, id_base, out_d,
                                                        out_i, flagged, n_flagged, force_exact);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int ff32_exact_chunks() { return 32; }

namespace ff32 {
__global__ void iota_kernel(int* flagged, int* n_flagged, int nq) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nq; i += gridDim.x * blockDim.x)
        flagged[i] = i;
    if (blockIdx.x == 0 && threadIdx.x == 0) *n_flagged = nq;
}
}  // namespace ff32

// exact_knn over every row for every query (the exact scan with all queries queued):
// COSINE 1 - dot_f32_4chain(q^, row) with q^ given, or L2 l2sq_f32_4chain(q, row);
// [nq x k] ascending by (distance, row + id_base).  `queue` holds nq + 1 ints.
int launch_exact_scan_all(const float* rows, int64_t n_rows, int dim, const float* q, int nq,
                          int k, int64_t id_base, int l2, int* queue, float* chunk_d,
                          int32_t* chunk_i, float* out_d, int32_t* out_i, int num_sms,
                          cudaStream_t st) {
    if (nq <= 0) return 0;
    if (k < 1 || k > ff32::EX_KMAX) return PION_B200_ESHAPE;
    const int chunks = ff32_exact_chunks();
    int* flagged = queue + 1;
    ff32::iota_kernel<<<(nq + 255) / 256 < 1024 ? (nq + 255) / 256 : 1024, 256, 0, st>>>(
        flagged, queue, nq);
    if (l2)
        ff32::exact_scan_kernel<true><<<num_sms * 2, ff32::EX_THREADS, 0, st>>>(
            rows, n_rows, dim, q, flagged, queue, chunks, k, chunk_d, chunk_i);
    else
        ff32::exact_scan_kernel<false><<<num_sms * 2, ff32::EX_THREADS, 0, st>>>(
            rows, n_rows, dim, q, flagged, queue, chunks, k, chunk_d, chunk_i);
    if (cudaGetLastError() != cudaSuccess) return PION_B200_ECUDA;
    ff32::exact_merge_kernel<<<(nq + 3) / 4, 128, 0, st>>>(chunk_d, chunk_i, flagged, queue,
                                                           chunks, k, id_base, out_d, out_i);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int launch_exact_fallback(const float* rows, int64_t n_rows, int dim, const float* qn,
                          const int* flagged, const int* n_flagged, int nq, int k,
                          int64_t id_base, float* chunk_d, int32_t* chunk_i, float* out_d,
                          int32_t* out_i, int num_sms, cudaStream_t st) {
    if (k > ff32::EX_KMAX) return PION_B200_ESHAPE;
    const int chunks = ff32_exact_chunks();
    ff32::exact_scan_kernel<false><<<num_sms * 2, ff32::EX_THREADS, 0, st>>>(
        rows, n_rows, dim, qn, flagged, n_flagged, chunks, k, chunk_d, chunk_i);
    if (cudaGetLastError() != cudaSuccess) return PION_B200_ECUDA;
    ff32::exact_merge_kernel<<<(nq + 3) / 4, 128, 0, st>>>(chunk_d, chunk_i, flagged, n_flagged,
                                                           chunks, k, id_base, out_d, out_i);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

}  // namespace pion
