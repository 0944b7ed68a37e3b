// Binary-quantised FLAT with FP32 rerank on B200 (sm_100a).
//
// Codes: bit b of word w is 1 iff x[64w + b] > 0 (the sign packing of
// src/vector/kernels.mojo:1711-1720, applied to the normalised vector).  Hamming
// distance = popcount(a XOR b) over the words (src/vector/reference/quant_dots.mojo:
// 95-100).  Shortlist: the S smallest Hamming distances by (distance, id).  Rerank:
// exact_knn's COSINE formula 1 - dot_f32_4chain(q^, row) on the shortlist and the
// stable insertion sort of _exact_rescore (src/commands/vector.mojo:1413-1456): equal
// scores keep shortlist order.
//
// On ±1 vectors, dot = (bits equal) - (bits differ) = dim - 2 * hamming, so the
// Hamming distances of a whole query batch come from the INT8 tensor-core pipeline
// (tcgen05 kind::i8) over a ±1-expanded copy of the codes:
//   bq_tc_kernel        collects, per (query, split), every row under the query's
//                       current Hamming bound (no score matrix);
//   bq_select_kernel    exact S-th smallest distance per query from a histogram of the
//                       small-integer distances, then the S best by (distance, id);
//   bq_fallback_kernel  queries whose candidate lists overflowed: exact popcount scan
//                       of the packed codes;
//   bq_rerank_kernel    exact fp32 rerank of the shortlist.
// The bound comes from staged samples: the S-th distance of the first rows bounds the
// final S-th distance, and later rows (larger ids) must beat it strictly.
#include <cstdint>
#include <cstdio>

#include "common.cuh"
#include "exact_fp32.cuh"
#include "internal.h"

namespace pion {
namespace bq {

constexpr int BM = 128, BN = 256, BK = 128, STAGES = 4, UMMA_K = 32;
constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_WARPS = 8;
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr uint32_t TMEM_COLS = 2 * BN;
constexpr uint32_t IDESC = make_idesc_i8(BM, BN);
constexpr size_t SMEM_PIPE_BYTES = 1024 + (size_t)STAGES * STAGE_BYTES + 256;
constexpr size_t STASH_BYTES = 32 * 32 * 4;
constexpr size_t SMEM_BYTES = SMEM_PIPE_BYTES + EPI_WARPS * STASH_BYTES;
constexpr int CAP = 256;  // candidates kept per (query, list)

struct TcParams {
    const int* dot_min;   // per query: collect rows with dot >= dot_min (nullptr: all)
    int64_t n_rows;
    int nq;
    int dim;
    int tile_begin, tile_end, n_splits, kblocks;
    int n_lists, list_base;
    int32_t* cand_id;     // [nq][n_lists][CAP]
    uint16_t* cand_h;     // [nq][n_lists][CAP]
    int* cand_n;          // [nq][n_lists]
    int* status;
};

template <int HALVES>
__global__ void __launch_bounds__(THREADS, 1)
    bq_tc_kernel(const __grid_constant__ CUtensorMap tmap_q,
                 const __grid_constant__ CUtensorMap tmap_rows, TcParams p) {
    constexpr int COLS = BN / HALVES;
    constexpr int CHUNKS = COLS / 32;
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
            tma_prefetch_desc(&tmap_q);
            tma_prefetch_desc(&tmap_rows);
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_parity[STAGES];
            bool issued[STAGES];
            for (int s = 0; s < STAGES; ++s) issued[s] = false, issued_parity[s] = 0;
            bool ok = true;
            for (int t = 0; t < my_tiles && ok; ++t) {
                const int row0 = (t_begin + t) * BN;
                for (int kb = 0; kb < p.kblocks; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, abort_flag)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
                    tma_load_2d(sA + stage * A_BYTES, &tmap_q, &full[stage], kb * BK, qt * BM);
                    tma_load_2d(sB + stage * B_BYTES, &tmap_rows, &full[stage], kb * BK, row0);
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
                for (int kb = 0; kb < p.kblocks; ++kb) {
                    if (!mbar_wait(&full[stage], phase, p.status, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + stage * A_BYTES);
                    const uint32_t b0 = smem_u32(sB + stage * B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < BK / UMMA_K; ++kk)
                        mma_i8(d_tmem, make_sw128_kmajor_desc(a0 + kk * UMMA_K),
                               make_sw128_kmajor_desc(b0 + kk * UMMA_K), IDESC,
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
        // epilogue: collect every column with dot >= dot_min into this thread's list
        const int ew = warp - 2;
        uint32_t* stash = stash_all + ew * (STASH_BYTES / 4);
        const int lg = warp & 3;
        const int half = ew >> 2;
        const int q = qt * BM + lg * 32 + lane;
        const bool q_ok = q < p.nq;
        const int dmin = !q_ok ? INT32_MAX : (p.dot_min ? p.dot_min[q] : INT32_MIN);
        const size_t list = (size_t)(q_ok ? q : 0) * p.n_lists + p.list_base +
                            (size_t)split * HALVES + half;
        int32_t* out_id = p.cand_id + list * CAP;
        uint16_t* out_h = p.cand_h + list * CAP;
        int count = 0;
        for (int t = 0; t < my_tiles; ++t) {
            const int buf = t & 1;
            const uint32_t use = (uint32_t)(t >> 1);
            const int tile = t_begin + t;
            const int64_t col0 = (int64_t)tile * BN + half * COLS;
            const int64_t valid = p.n_rows - col0;
            const bool got = mbar_wait(&tfull[buf], use & 1u, p.status, abort_flag);
            if (!__all_sync(0xffffffffu, got)) break;
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(lg * 32) << 16) +
                                   (uint32_t)(buf * BN + half * COLS);
#pragma unroll 1
            for (int c = 0; c < CHUNKS; ++c) {
                uint32_t r[32];
                __syncwarp();
                tmem_ld32(taddr + (uint32_t)(c * 32), r);
                tmem_ld_wait_regs(r);
                int32_t mx = (int32_t)r[0];
#pragma unroll
                for (int j = 1; j < 32; ++j) mx = max(mx, (int32_t)r[j]);
                uint32_t mask = 0;
                if (mx >= dmin) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) mask |= ((int32_t)r[j] >= dmin ? 1u : 0u) << j;
                    const int64_t vc = valid - c * 32;
                    if (vc < 32) mask &= vc <= 0 ? 0u : ((1u << vc) - 1u);
                }
                if (!__any_sync(0xffffffffu, mask != 0u)) continue;
#pragma unroll
                for (int j = 0; j < 32; ++j) stash[j * 32 + lane] = r[j];
                __syncwarp();
#pragma unroll 1
                while (mask) {
                    const int j = __ffs(mask) - 1;
                    mask &= mask - 1u;
                    if (count < CAP) {
                        const int32_t dv = (int32_t)stash[j * 32 + lane];
                        out_id[count] = (int32_t)(col0 + c * 32 + j);
                        out_h[count] = (uint16_t)((p.dim - dv) >> 1);
                    }
                    ++count;
                }
                __syncwarp();
            }
            tc_fence_before();
            mbar_arrive(&tempty[buf]);
        }
        if (q_ok) p.cand_n[list] = count;  // > CAP means the list overflowed
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ------------------------------------------------------------ preparation --

// Signs of one row: ±1 int8 (x > 0 -> +1) and the packed code (bit b of word w).
// One warp per row, 64 elements (one word) per lane step.
__global__ void signs_kernel(const float* __restrict__ x, int64_t n_rows, int dim,
                             int8_t* __restrict__ pm, uint64_t* __restrict__ codes) {
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (r >= n_rows) return;
    const int lane = threadIdx.x & 31;
    const float* xr = x + r * dim;
    const int words = dim / 64;
    for (int w = 0; w < words; ++w) {
        const float a = xr[w * 64 + lane], b = xr[w * 64 + 32 + lane];
        const unsigned lo = __ballot_sync(0xffffffffu, a > 0.0f);
        const unsigned hi = __ballot_sync(0xffffffffu, b > 0.0f);
        if (pm) {
            pm[r * dim + w * 64 + lane] = a > 0.0f ? 1 : -1;
            pm[r * dim + w * 64 + 32 + lane] = b > 0.0f ? 1 : -1;
        }
        if (lane == 0) codes[r * words + w] = ((uint64_t)hi << 32) | lo;
    }
}

// ------------------------------------------------------------- selection --
constexpr int SEL_THREADS = 256;
constexpr int SEL_TIES = 2048;

__device__ __forceinline__ void bitonic_sort_u64(uint64_t* v, int n_pow2) {
    for (int size = 2; size <= n_pow2; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < n_pow2 / 2; i += blockDim.x) {
                const int lo = 2 * i - (i & (stride - 1));
                const int hi = lo + stride;
                const bool asc = ((lo & size) == 0);
                const uint64_t a = v[lo], b = v[hi];
                if (asc ? (a > b) : (a < b)) {
                    v[lo] = b;
                    v[hi] = a;
                }
            }
            __syncthreads();
        }
}

// One CTA per query: the S best candidates by (distance, id) from its lists, sorted.
// Writes the shortlist, its length, the next stage's bound (dot_min: rows must have a
// distance strictly below the S-th one) and flags queries whose lists overflowed.
__global__ void __launch_bounds__(SEL_THREADS)
    bq_select_kernel(const int32_t* __restrict__ cid, const uint16_t* __restrict__ ch,
                     const int* __restrict__ cn, int n_lists, int dim, int S,
                     int32_t* __restrict__ out_id, uint16_t* __restrict__ out_h,
                     int* __restrict__ out_n, int out_qstride, int n_qstride,
                     int* __restrict__ next_dot_min, int* __restrict__ flagged,
                     int* __restrict__ n_flagged, int force_flag) {
    extern __shared__ int sm_hist[];  // dim + 1 bins, then the lists' counts
    int* scnt = sm_hist + ((dim + 1 + 3) & ~3);
    __shared__ uint64_t keys[512];
    __shared__ int32_t ties[SEL_TIES];
    __shared__ int warp_tot[SEL_THREADS / 32];
    __shared__ int n_keys, n_ties, overflow, dstar, below, total_s;
    const int q = blockIdx.x;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    for (int i = threadIdx.x; i <= dim; i += SEL_THREADS) sm_hist[i] = 0;
    if (threadIdx.x == 0) {
        n_keys = n_ties = overflow = 0;
        total_s = 0;
    }
    __syncthreads();
    // the lists' counts in one pass (every load in flight at once), then the candidates
    // of all lists as one flat range: a query's lists are contiguous, [n_lists][CAP]
    const size_t qbase = (size_t)q * n_lists;
    int my_total = 0;
    for (int l = threadIdx.x; l < n_lists; l += SEL_THREADS) {
        const int c = cn[qbase + l];
        if (c > CAP) overflow = 1;
        const int m = c < CAP ? c : CAP;
        scnt[l] = m;
        my_total += m;
    }
    if (my_total) atomicAdd(&total_s, my_total);
    __syncthreads();
    const int flat = n_lists * CAP;
    const uint16_t* chq = ch + qbase * CAP;
    const int32_t* cidq = cid + qbase * CAP;
#pragma unroll 4
    for (int e = threadIdx.x; e < flat; e += SEL_THREADS)
        if ((e % CAP) < scnt[e / CAP]) atomicAdd(&sm_hist[chq[e]], 1);
    __syncthreads();
    // smallest d with count(h <= d) >= want (all candidates when fewer than S): per-thread
    // runs of bins, a block scan of their sums, the run that crosses scanned by its thread
    const int want = total_s < S ? total_s : S;
    {
        const int per = (dim + 1 + SEL_THREADS - 1) / SEL_THREADS;
        const int lo = threadIdx.x * per;
        int sum = 0;
        for (int i = lo; i < lo + per && i <= dim; ++i) sum += sm_hist[i];
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        if (lane == 31) warp_tot[w] = incl;
        if (threadIdx.x == 0) {
            dstar = -1;
            below = 0;
        }
        __syncthreads();
        for (int v = 0; v < w; ++v) incl += warp_tot[v];
        const int excl = incl - sum;
        if (want > 0 && excl < want && incl >= want) {
            int acc = excl, d = lo;
            for (; d < lo + per && d <= dim; ++d) {
                if (acc + sm_hist[d] >= want) break;
                acc += sm_hist[d];
            }
            dstar = d;
            below = acc;
        }
        __syncthreads();
    }
    const int D = dstar;
    if (D >= 0) {
#pragma unroll 4
        for (int e = threadIdx.x; e < flat; e += SEL_THREADS) {
            if ((e % CAP) >= scnt[e / CAP]) continue;
            const int h = chq[e];
            if (h < D) {
                const int pos = atomicAdd(&n_keys, 1);
                if (pos < 512) keys[pos] = ((uint64_t)h << 32) | (uint32_t)cidq[e];
            } else if (h == D) {
                const int pos = atomicAdd(&n_ties, 1);
                if (pos < SEL_TIES) ties[pos] = cidq[e];
            }
        }
    }
    __syncthreads();
    if (D >= 0 && n_ties > SEL_TIES && threadIdx.x == 0) overflow = 1;
    // the (want - below) smallest ids among the ties at D
    const int nt = n_ties < SEL_TIES ? n_ties : SEL_TIES;
    int p2 = 1;
    while (p2 < nt) p2 <<= 1;
    for (int i = nt + threadIdx.x; i < p2; i += SEL_THREADS) ties[i] = INT32_MAX;
    __syncthreads();
    if (D >= 0 && nt > 1) {
        for (int size = 2; size <= p2; size <<= 1)
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                for (int i = threadIdx.x; i < p2 / 2; i += SEL_THREADS) {
                    const int lo = 2 * i - (i & (stride - 1));
                    const int hi = lo + stride;
                    const bool asc = ((lo & size) == 0);
                    const int32_t a = ties[lo], b = ties[hi];
                    if (asc ? (a > b) : (a < b)) {
                        ties[lo] = b;
                        ties[hi] = a;
                    }
                }
                __syncthreads();
            }
    }
    const int take = want - below;
    for (int i = threadIdx.x; i < take && D >= 0; i += SEL_THREADS)
        keys[below + i] = ((uint64_t)D << 32) | (uint32_t)ties[i];
    __syncthreads();
    // sort the shortlist by (distance, id)
    int sp2 = 1;
    while (sp2 < want) sp2 <<= 1;
    for (int i = want + threadIdx.x; i < sp2; i += SEL_THREADS) keys[i] = ~0ull;
    __syncthreads();
    if (want > 1) bitonic_sort_u64(keys, sp2);
    for (int i = threadIdx.x; i < S; i += SEL_THREADS) {
        out_id[(size_t)q * out_qstride + i] = i < want ? (int32_t)(uint32_t)keys[i] : -1;
        out_h[(size_t)q * out_qstride + i] = i < want ? (uint16_t)(keys[i] >> 32) : (uint16_t)0xffff;
    }
    if (threadIdx.x == 0) {
        out_n[(size_t)q * n_qstride] = want;
        // later rows (larger ids) enter only with a distance below the S-th one
        next_dot_min[q] = (total_s >= S && D >= 0) ? dim - 2 * (D - 1) : INT32_MIN;
        if (overflow || force_flag) flagged[atomicAdd(n_flagged, 1)] = q;
    }
}

// Flagged queries: the exact shortlist from every packed code (popcount of XOR),
// one CTA per flagged query: a histogram pass, then an in-order collection.
__global__ void __launch_bounds__(SEL_THREADS)
    bq_fallback_kernel(const uint64_t* __restrict__ codes, int64_t n_rows, int words,
                       const uint64_t* __restrict__ qcodes, const int* __restrict__ flagged,
                       const int* __restrict__ n_flagged, int S, int32_t* __restrict__ out_id,
                       uint16_t* __restrict__ out_h, int* __restrict__ out_n) {
    extern __shared__ int fb_hist[];
    __shared__ uint64_t keys[512];
    __shared__ int dstar, below, n_keys, n_tie_taken;
    const int dim = words * 64;
    for (int f = blockIdx.x; f < *n_flagged; f += gridDim.x) {
        const int q = flagged[f];
        const uint64_t* qc = qcodes + (size_t)q * words;
        for (int i = threadIdx.x; i <= dim; i += SEL_THREADS) fb_hist[i] = 0;
        if (threadIdx.x == 0) n_keys = n_tie_taken = 0;
        __syncthreads();
        for (int64_t r = threadIdx.x; r < n_rows; r += SEL_THREADS) {
            int h = 0;
            for (int w = 0; w < words; ++w) h += __popcll(codes[r * words + w] ^ qc[w]);
            atomicAdd(&fb_hist[h], 1);
        }
        __syncthreads();
        const int want = n_rows < S ? (int)n_rows : S;
        if (threadIdx.x == 0) {
            int acc = 0, d = 0;
            for (d = 0; d <= dim; ++d) {
                if (acc + fb_hist[d] >= want) break;
                acc += fb_hist[d];
            }
            dstar = d;
            below = acc;
        }
        __syncthreads();
        const int D = dstar, need = want - below;
        // rows in order, block by block: h < D always, h == D while ties are needed
        for (int64_t base = 0; base < n_rows; base += SEL_THREADS) {
            const int64_t r = base + threadIdx.x;
            int h = dim + 1;
            if (r < n_rows) {
                h = 0;
                for (int w = 0; w < words; ++w) h += __popcll(codes[r * words + w] ^ qc[w]);
            }
            if (h < D) keys[atomicAdd(&n_keys, 1)] = ((uint64_t)h << 32) | (uint32_t)r;
            // ties in row order: a block-wide ordered rank
            const bool tie = (h == D);
            __shared__ int warp_cnt[SEL_THREADS / 32];
            const unsigned bal = __ballot_sync(0xffffffffu, tie);
            const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
            if (lane == 0) warp_cnt[w] = __popc(bal);
            __syncthreads();
            int before = n_tie_taken;
            for (int x = 0; x < w; ++x) before += warp_cnt[x];
            const int rank = before + __popc(bal & ((1u << lane) - 1u));
            if (tie && rank < need) keys[below + rank] = ((uint64_t)h << 32) | (uint32_t)r;
            __syncthreads();
            if (threadIdx.x == 0)
                for (int x = 0; x < SEL_THREADS / 32; ++x) n_tie_taken += warp_cnt[x];
            __syncthreads();
        }
        int sp2 = 1;
        while (sp2 < want) sp2 <<= 1;
        for (int i = want + threadIdx.x; i < sp2; i += SEL_THREADS) keys[i] = ~0ull;
        __syncthreads();
        if (want > 1) bitonic_sort_u64(keys, sp2);
        for (int i = threadIdx.x; i < S; i += SEL_THREADS) {
            out_id[(size_t)q * S + i] = i < want ? (int32_t)(uint32_t)keys[i] : -1;
            out_h[(size_t)q * S + i] = i < want ? (uint16_t)(keys[i] >> 32) : (uint16_t)0xffff;
        }
        if (threadIdx.x == 0) out_n[q] = want;
        __syncthreads();
    }
}

// ---------------------------------------------------------------- rerank --
// One CTA per query: its 16 half-warps take the shortlist (in (distance, id) order) 16
// rows at a time, exact 4-chain cosine distances with the rows prefetched into L2; then
// warp 0 keeps the k best by (score, shortlist position): the stable insertion sort of
// _exact_rescore keeps equal scores in shortlist order.
__global__ void __launch_bounds__(256) bq_rerank_kernel(
    const float* __restrict__ rows, int dim, const float* __restrict__ qn,
    const int32_t* __restrict__ sl_id, const int* __restrict__ sl_n, int S, int nq, int k,
    int64_t id_base, float* __restrict__ out_d, int32_t* __restrict__ out_i) {
    extern __shared__ __align__(16) float rr[];
    const int q = blockIdx.x;
    if (q >= nq) return;
    const int lane = threadIdx.x & 31;
    const bool quad = (dim & 15) == 0;  // four lanes per row, the query in shared memory
    float* dist = quad ? rr + dim : rr;
    const float* qv = qn + (size_t)q * dim;
    const int n = sl_n[q];
    for (int j = threadIdx.x; j < n; j += blockDim.x)
        prefetch_row_f32_l2(rows + (size_t)sl_id[(size_t)q * S + j] * dim, dim);
    if (quad) {
        float4* qs4 = reinterpret_cast<float4*>(rr);
        for (int c = threadIdx.x; c < (dim >> 2); c += blockDim.x)
            qs4[c] = reinterpret_cast<const float4*>(qv)[c];
        __syncthreads();
        const int quads = blockDim.x >> 2;
        for (int j0 = 0; j0 < n; j0 += quads) {  // every lane of the warp takes part
            const int j = j0 + (threadIdx.x >> 2);
            const float* row = j < n ? rows + (size_t)sl_id[(size_t)q * S + j] * dim : nullptr;
            const float s = dot4chain_quad<12>(qs4, row, dim);
            if ((threadIdx.x & 3) == 0 && j < n) dist[j] = __fsub_rn(1.0f, s);
        }
    } else {
        const int hw = threadIdx.x >> 4;  // 16 half-warps, one shortlisted row each
        const int hl = lane & 15;
        const unsigned hmask = (lane >> 4) ? 0xffff0000u : 0x0000ffffu;
        const int halves = blockDim.x >> 4;
        for (int j0 = 0; j0 < n; j0 += halves) {
            const int j = j0 + hw;
            if (j < n) {
                const int32_t id = sl_id[(size_t)q * S + j];
                const float s = dot4chain_half(qv, rows + (size_t)id * dim, dim, hl, hmask);
                if (hl == 0) dist[j] = __fsub_rn(1.0f, s);
            }
        }
    }
    __syncthreads();
    if (threadIdx.x >= 32) return;
    for (int r = 0; r < k; ++r) {
        float bd = INFINITY;
        int bp = -1;
        for (int j = lane; j < n; j += 32)
            if (dist[j] == dist[j] && (bp < 0 || dist[j] < bd)) {  // first (lowest j) wins ties
                bd = dist[j];
                bp = j;
            }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float od = __shfl_xor_sync(0xffffffffu, bd, o);
            const int op = __shfl_xor_sync(0xffffffffu, bp, o);
            if (op >= 0 && (bp < 0 || od < bd || (od == bd && op < bp))) {
                bd = od;
                bp = op;
            }
        }
        if (lane == 0) {
            out_d[(size_t)q * k + r] = bp >= 0 ? bd : INFINITY;
            out_i[(size_t)q * k + r] =
                bp >= 0 ? (int32_t)(sl_id[(size_t)q * S + bp] + id_base) : -1;
        }
        if (bp >= 0 && lane == (bp & 31)) dist[bp] = __int_as_float(0x7fffffff);  // taken (NaN)
        __syncwarp();
    }
}

// ------------------------------------------------------- one query: popcount stream
// The Hamming shortlist of ONE query as an HBM stream over the packed codes (no ±1
// expansion): 4 lanes per row, each 128-bit load two code words, XOR with the query's
// words and popcount; every distance is kept (u16, 2 bytes per row) and counted in a
// histogram.  Then the S-th smallest distance D* comes from the histogram; rows below
// D* are collected in any order, rows at D* are taken by ascending row id (the
// (distance, id) order of the batched path), and the shortlist is sorted.
constexpr int B1_THREADS = 256;
constexpr int B1_GROUPS = B1_THREADS / 4;
constexpr int B1_MAX_WORDS = 256;   // dim <= 16384
constexpr int B1_TIECAP = 8192;     // ties at D* sorted in shared memory; more: ordered scan
constexpr int B1_RPI = 4;           // rows per group per iteration
constexpr int B1_CPL = 3;           // 16-byte chunks per lane held in registers (<= 1536 dims)

__device__ __forceinline__ uint4 ld_stream_u4(const uint4* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Adds this CTA's shared histogram into the global one, bins 0..this CTA's own want-th
// smallest distance only: the global want-th smallest D* is at most every CTA's, so every
// bin <= D* still gets every CTA's count, and the bins above D* are never read.  (Adding
// every nonzero bin made the CTAs queue on the same few L2 lines at the end.)  Called by
// all B1_THREADS threads after a barrier.
__device__ void flush_hist_truncated(const int* b1_hist, int dim, int want, int* hist) {
    __shared__ int warp_tot[B1_THREADS / 32];
    __shared__ int cut;
    const int per = (dim + 1 + B1_THREADS - 1) / B1_THREADS;
    const int lo = threadIdx.x * per;
    int sum = 0;
    for (int i = lo; i < lo + per && i <= dim; ++i) sum += b1_hist[i];
    int incl = sum;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) warp_tot[w] = incl;
    if (threadIdx.x == 0) cut = dim;
    __syncthreads();
    for (int v = 0; v < w; ++v) incl += warp_tot[v];
    const int excl = incl - sum;
    if (excl < want && incl >= want) {  // the crossing is in this thread's bins
        int acc = excl, d = lo;
        for (; d < lo + per && d <= dim; ++d) {
            acc += b1_hist[d];
            if (acc >= want) break;
        }
        cut = d;
    }
    __syncthreads();
    for (int i = threadIdx.x; i <= cut; i += B1_THREADS)
        if (b1_hist[i]) atomicAdd(&hist[i], b1_hist[i]);
}

// Pass 1: dist[r] and the global histogram (hist[0..dim], zeroed by the caller).
__global__ void __launch_bounds__(B1_THREADS)
    bq_scan1_hist_kernel(const uint64_t* __restrict__ codes, int64_t n_rows, int words,
                         const uint64_t* __restrict__ qcode, int64_t rows_per_cta, int want,
                         uint16_t* __restrict__ dist, int* __restrict__ hist) {
    extern __shared__ int b1_hist[];  // dim + 1 bins
    __shared__ uint4 qv[B1_MAX_WORDS / 2];
    const int dim = words * 64;
    const int chunks = words >> 1;  // 16-byte chunks per row
    for (int i = threadIdx.x; i <= dim; i += B1_THREADS) b1_hist[i] = 0;
    for (int c = threadIdx.x; c < chunks; c += B1_THREADS)
        qv[c] = reinterpret_cast<const uint4*>(qcode)[c];
    __syncthreads();
    const int g = threadIdx.x >> 2;
    const int j = threadIdx.x & 3;
    const int64_t r0 = (int64_t)blockIdx.x * rows_per_cta;
    int64_t r1 = r0 + rows_per_cta;
    if (r1 > n_rows) r1 = n_rows;
    // B1_RPI rows per group per iteration, every chunk load of all of them issued before
    // the first popcount (up to 12 loads in flight per lane at 1536 dims)
    for (int64_t base = r0; base < r1; base += (int64_t)B1_GROUPS * B1_RPI) {
        int h[B1_RPI];
#pragma unroll
        for (int u = 0; u < B1_RPI; ++u) h[u] = 0;
        if (chunks <= 4 * B1_CPL) {
            uint4 a[B1_RPI][B1_CPL];
#pragma unroll
            for (int u = 0; u < B1_RPI; ++u) {
                const int64_t r = base + (int64_t)u * B1_GROUPS + g;
                const uint4* rp = reinterpret_cast<const uint4*>(codes + r * words);
#pragma unroll
                for (int i = 0; i < B1_CPL; ++i)
                    if (r < r1 && j + 4 * i < chunks) a[u][i] = ld_stream_u4(rp + j + 4 * i);
            }
#pragma unroll
            for (int u = 0; u < B1_RPI; ++u) {
                const int64_t r = base + (int64_t)u * B1_GROUPS + g;
#pragma unroll
                for (int i = 0; i < B1_CPL; ++i)
                    if (r < r1 && j + 4 * i < chunks) {
                        const uint4 b = qv[j + 4 * i];
                        h[u] += __popc(a[u][i].x ^ b.x) + __popc(a[u][i].y ^ b.y) +
                                __popc(a[u][i].z ^ b.z) + __popc(a[u][i].w ^ b.w);
                    }
            }
        } else {  // long codes: one row at a time
#pragma unroll 1
            for (int u = 0; u < B1_RPI; ++u) {
                const int64_t r = base + (int64_t)u * B1_GROUPS + g;
                if (r >= r1) continue;
                const uint4* rp = reinterpret_cast<const uint4*>(codes + r * words);
                for (int c = j; c < chunks; c += 4) {
                    const uint4 a = ld_stream_u4(rp + c);
                    const uint4 b = qv[c];
                    h[u] += __popc(a.x ^ b.x) + __popc(a.y ^ b.y) + __popc(a.z ^ b.z) +
                            __popc(a.w ^ b.w);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < B1_RPI; ++u) {
            const int64_t r = base + (int64_t)u * B1_GROUPS + g;
            int hu = h[u];
            hu += __shfl_xor_sync(0xffffffffu, hu, 1);
            hu += __shfl_xor_sync(0xffffffffu, hu, 2);
            if (r < r1 && j == 0) {
                dist[r] = (uint16_t)hu;
                atomicAdd(&b1_hist[hu], 1);
            }
        }
    }
    __syncthreads();
    flush_hist_truncated(b1_hist, dim, want, hist);
}

// Pass 1 through shared memory, for rows of at most B1S_MAX_ROW_BYTES: each CTA streams
// its contiguous row range in stages of B1S_ROWS rows, one bulk copy per stage
// (cp.async.bulk, completing on the stage's mbarrier) and B1S_STAGES stages in flight, so
// the bytes in flight do not depend on registers; 4 lanes per row then popcount from
// shared memory.  Same outputs as bq_scan1_hist_kernel.
constexpr int B1S_ROWS = 64;    // 12 KB stages at 1536 dims, two per CTA: seven CTAs per SM
constexpr int B1S_STAGES = 2;   // (measured: deeper rings at fewer CTAs per SM were slower)
constexpr int B1S_MAX_ROW_BYTES = 384;  // dim <= 3072

__global__ void __launch_bounds__(B1_THREADS)
    bq_scan1_stream_kernel(const uint64_t* __restrict__ codes, int64_t n_rows, int words,
                           const uint64_t* __restrict__ qcode, int64_t rows_per_cta, int want,
                           uint16_t* __restrict__ dist, int* __restrict__ hist, int* status,
                           uint64_t wait_ns) {
    extern __shared__ __align__(128) uint8_t b1s_smem[];
    const int dim = words * 64;
    const int row_bytes = words * 8;
    const int chunks = words >> 1;
    uint8_t* ring = b1s_smem;
    int* b1_hist = reinterpret_cast<int*>(ring + (size_t)B1S_STAGES * B1S_ROWS * row_bytes);
    uint4* qv = reinterpret_cast<uint4*>(b1_hist + ((dim + 1 + 3) & ~3));
    uint64_t* full = reinterpret_cast<uint64_t*>(qv + chunks);
    __shared__ int abort_flag;
    const int64_t r0 = (int64_t)blockIdx.x * rows_per_cta;
    int64_t r1 = r0 + rows_per_cta;
    if (r1 > n_rows) r1 = n_rows;
    const int n_stages = r1 > r0 ? (int)((r1 - r0 + B1S_ROWS - 1) / B1S_ROWS) : 0;
    auto issue = [&](int it) {  // thread 0: stage `it` of this CTA's range into its slot
        const int64_t a = r0 + (int64_t)it * B1S_ROWS;
        const int64_t b = a + B1S_ROWS < r1 ? a + B1S_ROWS : r1;
        const uint32_t bytes = (uint32_t)((b - a) * row_bytes);
        uint64_t* bar = &full[it % B1S_STAGES];
        mbar_arrive_expect_tx(bar, bytes);
        bulk_load(ring + (size_t)(it % B1S_STAGES) * B1S_ROWS * row_bytes,
                  reinterpret_cast<const uint8_t*>(codes) + a * row_bytes, bytes, bar);
    };
    if (threadIdx.x == 0) {  // the first stages are in flight while the CTA sets up
        abort_flag = 0;
        for (int s = 0; s < B1S_STAGES; ++s) mbar_init(&full[s], 1);
        fence_barrier_init();
        for (int it = 0; it < B1S_STAGES && it < n_stages; ++it) issue(it);
    }
    for (int i = threadIdx.x; i <= dim; i += B1_THREADS) b1_hist[i] = 0;
    for (int c = threadIdx.x; c < chunks; c += B1_THREADS)
        qv[c] = reinterpret_cast<const uint4*>(qcode)[c];
    __syncthreads();
    const int g = threadIdx.x >> 2, j = threadIdx.x & 3;
    int it = 0;
    for (; it < n_stages; ++it) {
        const int slot = it % B1S_STAGES;
        if (!mbar_wait(&full[slot], (uint32_t)((it / B1S_STAGES) & 1), status, &abort_flag,
                       wait_ns))
            break;
        const uint8_t* st = ring + (size_t)slot * B1S_ROWS * row_bytes;
        const int64_t base = r0 + (int64_t)it * B1S_ROWS;
#pragma unroll
        for (int u = 0; u < B1S_ROWS / B1_GROUPS; ++u) {
            const int rr = u * B1_GROUPS + g;
            const int64_t r = base + rr;
            const uint4* rp = reinterpret_cast<const uint4*>(st + (size_t)rr * row_bytes);
            int h = 0;
            if (r < r1)
                for (int c = j; c < chunks; c += 4) {
                    const uint4 a = rp[c];
                    const uint4 b = qv[c];
                    h += __popc(a.x ^ b.x) + __popc(a.y ^ b.y) + __popc(a.z ^ b.z) +
                         __popc(a.w ^ b.w);
                }
            h += __shfl_xor_sync(0xffffffffu, h, 1);
            h += __shfl_xor_sync(0xffffffffu, h, 2);
            if (r < r1 && j == 0) {
                dist[r] = (uint16_t)h;
                atomicAdd(&b1_hist[h], 1);
            }
        }
        __syncthreads();  // every thread is done with the slot: refill it
        if (threadIdx.x == 0 && it + B1S_STAGES < n_stages) issue(it + B1S_STAGES);
    }
    if (it < n_stages) {
        // a wait ran out: let the copies already issued land before the CTA exits
        if (threadIdx.x == 0) {
            const int last = n_stages < it + B1S_STAGES ? n_stages : it + B1S_STAGES;
            for (int t = it; t < last; ++t)
                mbar_wait(&full[t % B1S_STAGES], (uint32_t)((t / B1S_STAGES) & 1), nullptr,
                          nullptr, wait_ns);
        }
        __syncthreads();
        return;
    }
    __syncthreads();
    flush_hist_truncated(b1_hist, dim, want, hist);
}

size_t b1s_smem_bytes(int words) {
    const int dim = words * 64;
    return (size_t)B1S_STAGES * B1S_ROWS * words * 8 + (size_t)((dim + 1 + 3) & ~3) * 4 +
           (size_t)(words >> 1) * 16 + B1S_STAGES * 8;
}

// D* = the smallest d with #(dist <= d) >= want, and #(dist < D*), by one CTA's scan
// of the histogram (every CTA of pass 2 recomputes it: 6 KB of reads).
__device__ void b1_threshold(const int* __restrict__ hist, int dim, int want, int* d_out,
                             int* below_out) {
    __shared__ int seg[B1_THREADS];
    const int per = (dim + 1 + B1_THREADS - 1) / B1_THREADS;
    const int lo = threadIdx.x * per;
    int sum = 0;
    for (int i = lo; i < lo + per && i <= dim; ++i) sum += hist[i];
    seg[threadIdx.x] = sum;
    __syncthreads();
    if (threadIdx.x == 0) {
        int acc = 0, t = 0;
        for (; t < B1_THREADS; ++t) {
            if (acc + seg[t] >= want) break;
            acc += seg[t];
        }
        int d = t * per;
        for (; d <= dim; ++d) {
            if (acc + hist[d] >= want) break;
            acc += hist[d];
        }
        *d_out = d;
        *below_out = acc;
    }
    __syncthreads();
}

// Pass 2: rows below D* as (dist << 32 | row) keys, rows at D* as row ids (unordered,
// counted; at most B1_TIECAP kept).  meta: [0] keys, [1] ties, [2] D*, [3] below.
__global__ void __launch_bounds__(B1_THREADS)
    bq_scan1_collect_kernel(const uint16_t* __restrict__ dist, int64_t n_rows, int dim,
                            const int* __restrict__ hist, int want, int64_t rows_per_cta,
                            uint64_t* __restrict__ keys, int32_t* __restrict__ ties,
                            int* __restrict__ meta) {
    __shared__ int D, below;
    b1_threshold(hist, dim, want, &D, &below);
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        meta[2] = D;
        meta[3] = below;
    }
    const int64_t r0 = (int64_t)blockIdx.x * rows_per_cta;
    int64_t r1 = r0 + rows_per_cta;
    if (r1 > n_rows) r1 = n_rows;
    for (int64_t r = r0 + threadIdx.x; r < r1; r += B1_THREADS) {
        const int h = dist[r];
        if (h < D) {
            keys[atomicAdd(&meta[0], 1)] = ((uint64_t)h << 32) | (uint32_t)r;
        } else if (h == D) {
            const int t = atomicAdd(&meta[1], 1);
            if (t < B1_TIECAP) ties[t] = (int32_t)r;
        }
    }
}

// Pass 3 (one CTA): the first (want - below) rows at D* by id -- sorted in shared memory,
// or, when there are more than B1_TIECAP of them, by an ordered scan of dist -- then the
// shortlist sorted by (distance, id).
__global__ void __launch_bounds__(1024)
    bq_scan1_finish_kernel(const uint16_t* __restrict__ dist, int64_t n_rows,
                           const uint64_t* __restrict__ keys_in, const int32_t* __restrict__ ties,
                           const int* __restrict__ meta, int want, int S,
                           int32_t* __restrict__ out_id, uint16_t* __restrict__ out_h,
                           int* __restrict__ out_n) {
    extern __shared__ uint64_t b1_keys[];  // B1_TIECAP (ties) then 512 (shortlist)
    uint64_t* tk = b1_keys;
    uint64_t* sk = b1_keys + B1_TIECAP;
    __shared__ int warp_cnt[32];
    __shared__ int taken;
    const int D = meta[2], below = meta[3], n_tie = meta[1];
    const int need = want - below;
    for (int i = threadIdx.x; i < below; i += blockDim.x) sk[i] = keys_in[i];
    if (n_tie <= B1_TIECAP) {
        int p2 = 1;
        while (p2 < n_tie) p2 <<= 1;
        for (int i = threadIdx.x; i < p2; i += blockDim.x)
            tk[i] = i < n_tie ? (uint64_t)(uint32_t)ties[i] : ~0ull;
        __syncthreads();
        if (n_tie > 1) bitonic_sort_u64(tk, p2);
        for (int i = threadIdx.x; i < need; i += blockDim.x)
            sk[below + i] = ((uint64_t)D << 32) | tk[i];
    } else {
        if (threadIdx.x == 0) taken = 0;
        __syncthreads();
        const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
        for (int64_t base = 0; base < n_rows && taken < need; base += blockDim.x) {
            const int64_t r = base + threadIdx.x;
            const bool tie = r < n_rows && dist[r] == D;
            const unsigned bal = __ballot_sync(0xffffffffu, tie);
            if (lane == 0) warp_cnt[w] = __popc(bal);
            __syncthreads();
            int before = taken;
            for (int x = 0; x < w; ++x) before += warp_cnt[x];
            const int rank = before + __popc(bal & ((1u << lane) - 1u));
            if (tie && rank < need) sk[below + rank] = ((uint64_t)D << 32) | (uint32_t)r;
            __syncthreads();
            if (threadIdx.x == 0)
                for (int x = 0; x < nw; ++x) taken += warp_cnt[x];
            __syncthreads();
        }
    }
    __syncthreads();
    int p2 = 1;
    while (p2 < want) p2 <<= 1;
    for (int i = want + threadIdx.x; i < p2; i += blockDim.x) sk[i] = ~0ull;
    __syncthreads();
    if (want > 1) bitonic_sort_u64(sk, p2);
    for (int i = threadIdx.x; i < S; i += blockDim.x) {
        out_id[i] = i < want ? (int32_t)(uint32_t)sk[i] : -1;
        out_h[i] = i < want ? (uint16_t)(sk[i] >> 32) : (uint16_t)0xffff;
    }
    if (threadIdx.x == 0) *out_n = want;
}

// Rerank for few queries: the shortlist rows spread over many CTAs, 4 lanes per row
// (dot4chain_quad: the 4-chain order with 128-bit loads), distances to `dist`; then a
// warp per query picks the k best by (distance, shortlist position) exactly as the
// tail of bq_rerank_kernel does.
constexpr int RW_THREADS = 128;
constexpr int RW_ROWS = RW_THREADS / 4;

__global__ void __launch_bounds__(RW_THREADS)
    bq_rerank_rows_kernel(const float* __restrict__ rows, int dim, const float* __restrict__ qn,
                          const int32_t* __restrict__ sl_id, const int* __restrict__ sl_n, int S,
                          float* __restrict__ dist) {
    extern __shared__ float4 rw_q[];  // dim / 4
    const int q = blockIdx.y;
    for (int c = threadIdx.x; c < (dim >> 2); c += RW_THREADS)
        rw_q[c] = reinterpret_cast<const float4*>(qn + (size_t)q * dim)[c];
    __syncthreads();
    const int jj = blockIdx.x * RW_ROWS + (threadIdx.x >> 2);
    const bool valid = jj < sl_n[q];
    const float* row = valid ? rows + (size_t)sl_id[(size_t)q * S + jj] * dim : nullptr;
    const float dot = dot4chain_quad<12>(rw_q, row, dim);
    if (valid && (threadIdx.x & 3) == 0) dist[(size_t)q * S + jj] = __fsub_rn(1.0f, dot);
}

__global__ void __launch_bounds__(128)
    bq_rerank_pick_kernel(const float* __restrict__ dist_in, const int32_t* __restrict__ sl_id,
                          const int* __restrict__ sl_n, int S, int nq, int k, int64_t id_base,
                          float* __restrict__ out_d, int32_t* __restrict__ out_i) {
    __shared__ float dist_all[4][256];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * 4 + w;
    if (q >= nq) return;
    float* dist = dist_all[w];
    const int n = sl_n[q];
    for (int j = lane; j < n; j += 32) dist[j] = dist_in[(size_t)q * S + j];
    __syncwarp();
    for (int r = 0; r < k; ++r) {
        float bd = INFINITY;
        int bp = -1;
        for (int j = lane; j < n; j += 32)
            if (dist[j] == dist[j] && (bp < 0 || dist[j] < bd)) {  // first (lowest j) wins ties
                bd = dist[j];
                bp = j;
            }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float od = __shfl_xor_sync(0xffffffffu, bd, o);
            const int op = __shfl_xor_sync(0xffffffffu, bp, o);
            if (op >= 0 && (bp < 0 || od < bd || (od == bd && op < bp))) {
                bd = od;
                bp = op;
            }
        }
        if (lane == 0) {
            out_d[(size_t)q * k + r] = bp >= 0 ? bd : INFINITY;
            out_i[(size_t)q * k + r] =
                bp >= 0 ? (int32_t)(sl_id[(size_t)q * S + bp] + id_base) : -1;
        }
        if (bp >= 0 && lane == (bp & 31)) dist[bp] = __int_as_float(0x7fffffff);  // taken (NaN)
        __syncwarp();
    }
}

// Rerank for few queries with the shortlist rows staged in shared memory: a one-warp CTA
// per 8 shortlist rows pulls them in with one bulk copy each (all in flight at once, one
// DRAM round trip), then 4 lanes per row run the reference's 4-chain dot from shared
// memory (lane j = chain j, the same transpose and sums as dot4chain_quad); the last CTA
// of a query to finish picks the k best by (distance, shortlist position).
constexpr int RS_ROWS = 8;
constexpr int RS_PAD = 16;  // floats between staged rows (rows 64 B apart in the banks)

__global__ void __launch_bounds__(32)
    bq_rerank_staged_kernel(const float* __restrict__ rows, int dim, const float* __restrict__ qn,
                            const int32_t* __restrict__ sl_id, const int* __restrict__ sl_n,
                            int S, int k, int64_t id_base, float* dist, unsigned* done,
                            int* status, uint64_t wait_ns, float* __restrict__ out_d,
                            int32_t* __restrict__ out_i) {
    extern __shared__ __align__(16) uint8_t rs_smem[];
    const int pitch = dim + RS_PAD;
    float4* qs = reinterpret_cast<float4*>(rs_smem);
    float* rsm = reinterpret_cast<float*>(rs_smem + (size_t)dim * 4);
    uint64_t* bar = reinterpret_cast<uint64_t*>(rs_smem + (size_t)dim * 4 +
                                                (size_t)RS_ROWS * pitch * 4);
    const int q = blockIdx.y, lane = threadIdx.x;
    const int n = sl_n[q];
    const int j0 = blockIdx.x * RS_ROWS;
    const int nr = n - j0 < 0 ? 0 : (n - j0 > RS_ROWS ? RS_ROWS : n - j0);
    if (nr > 0) {
        if (lane == 0) {
            mbar_init(bar, 1);
            fence_barrier_init();
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)(nr * dim * 4));
        __syncwarp();
        if (lane < nr)
            bulk_load(rsm + (size_t)lane * pitch,
                      rows + (size_t)sl_id[(size_t)q * S + j0 + lane] * dim, (uint32_t)dim * 4,
                      bar);
        for (int c = lane; c < (dim >> 2); c += 32)
            qs[c] = reinterpret_cast<const float4*>(qn + (size_t)q * dim)[c];
        __syncwarp();
        bool ok = mbar_wait(bar, 0, status, nullptr, wait_ns);
        if (!ok) mbar_wait(bar, 0, nullptr, nullptr, wait_ns);  // let the copies land
        ok = __all_sync(0xffffffffu, ok);
        const int r = lane >> 2, j = lane & 3;
        float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
        if (ok && r < nr) {
            const float4* rp = reinterpret_cast<const float4*>(rsm + (size_t)r * pitch) + j;
            const int steps = dim >> 4;
#pragma unroll 8
            for (int i = 0; i < steps; ++i) {
                const float4 v = rp[i * 4];
                const float4 qv = qs[i * 4 + j];
                a0 = __fadd_rn(__fmul_rn(qv.x, v.x), a0);
                a1 = __fadd_rn(__fmul_rn(qv.y, v.y), a1);
                a2 = __fadd_rn(__fmul_rn(qv.z, v.z), a2);
                a3 = __fadd_rn(__fmul_rn(qv.w, v.w), a3);
            }
        }
        const int gbase = lane & ~3;
        const float own = sel4(a0, a1, a2, a3, j);
        const float r1 = __shfl_xor_sync(0xffffffffu, sel4(a0, a1, a2, a3, j ^ 1), 1);
        const float r2 = __shfl_xor_sync(0xffffffffu, sel4(a0, a1, a2, a3, j ^ 2), 2);
        const float r3 = __shfl_xor_sync(0xffffffffu, sel4(a0, a1, a2, a3, j ^ 3), 3);
        const float c0 = sel4(own, r1, r2, r3, j ^ 0);
        const float c1 = sel4(own, r1, r2, r3, j ^ 1);
        const float c2 = sel4(own, r1, r2, r3, j ^ 2);
        const float c3 = sel4(own, r1, r2, r3, j ^ 3);
        const float t = __fadd_rn(__fadd_rn(c0, c1), __fadd_rn(c2, c3));
        const float t0 = __shfl_sync(0xffffffffu, t, gbase + 0);
        const float t1 = __shfl_sync(0xffffffffu, t, gbase + 1);
        const float t2 = __shfl_sync(0xffffffffu, t, gbase + 2);
        const float t3 = __shfl_sync(0xffffffffu, t, gbase + 3);
        const float dot = __fadd_rn(__fadd_rn(t0, t2), __fadd_rn(t1, t3));
        if (r < nr && j == 0) dist[(size_t)q * S + j0 + r] = __fsub_rn(1.0f, dot);
        __threadfence();
    }
    unsigned last = 0;
    if (lane == 0) last = atomicAdd(&done[q], 1u) == gridDim.x - 1 ? 1u : 0u;
    if (!__shfl_sync(0xffffffffu, last, 0)) return;
    __threadfence();
    if (lane == 0) done[q] = 0;  // ready for the next call (stream-ordered)
    float* dl = rsm;             // n <= 256 distances fit in the staged rows' room
    for (int j = lane; j < n; j += 32) dl[j] = __ldcg(dist + (size_t)q * S + j);
    __syncwarp();
    for (int rr = 0; rr < k; ++rr) {
        float bd = INFINITY;
        int bp = -1;
        for (int j = lane; j < n; j += 32)
            if (dl[j] == dl[j] && (bp < 0 || dl[j] < bd)) {  // first (lowest j) wins ties
                bd = dl[j];
                bp = j;
            }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float od = __shfl_xor_sync(0xffffffffu, bd, o);
            const int op = __shfl_xor_sync(0xffffffffu, bp, o);
            if (op >= 0 && (bp < 0 || od < bd || (od == bd && op < bp))) {
                bd = od;
                bp = op;
            }
        }
        if (lane == 0) {
            out_d[(size_t)q * k + rr] = bp >= 0 ? bd : INFINITY;
            out_i[(size_t)q * k + rr] =
                bp >= 0 ? (int32_t)(sl_id[(size_t)q * S + bp] + id_base) : -1;
        }
        if (bp >= 0 && lane == (bp & 31)) dl[bp] = __int_as_float(0x7fffffff);  // taken (NaN)
        __syncwarp();
    }
}

}  // namespace bq

// =========================================================== host launchers ==

bool bq_scan1_supported(int words, int S) {
    return words % 2 == 0 && words <= bq::B1_MAX_WORDS && S >= 1 && S <= 512;
}

// One full wave of the first pass: as many CTAs as fit on the SMs at once (the register
// pass's 84 registers a thread allow 2 CTAs of 256 threads per SM; the staged pass's
// ~31 KB of shared memory 7).
int bq_scan1_ctas(int64_t n_rows, int words, int num_sms, int stream_path) {
    int per_sm = 0;
    cudaError_t e;
    if (words * 8 <= bq::B1S_MAX_ROW_BYTES && stream_path != 1) {
        const size_t ssm = bq::b1s_smem_bytes(words);
        e = set_smem_limit((const void*)bq::bq_scan1_stream_kernel, (int)ssm) == 0
                ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                      &per_sm, bq::bq_scan1_stream_kernel, bq::B1_THREADS, ssm)
                : cudaErrorInvalidValue;
    } else {
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, bq::bq_scan1_hist_kernel,
                                                          bq::B1_THREADS,
                                                          (size_t)(words * 64 + 1) * 4);
    }
    if (e != cudaSuccess || per_sm < 1) {
        cudaGetLastError();
        per_sm = 2;
    }
    int64_t ctas = (int64_t)num_sms * per_sm;
    const int64_t min_rows = 4 * bq::B1_GROUPS;
    if (ctas * min_rows > n_rows) ctas = (n_rows + min_rows - 1) / min_rows;
    return (int)(ctas < 1 ? 1 : ctas);
}

size_t bq_scan1_scratch(int64_t n_rows, int words) {
    return (size_t)(n_rows * 2 + 255) / 256 * 256 + (size_t)(words * 64 + 1 + 63) / 64 * 256 +
           512 * 8 + bq::B1_TIECAP * 4 + 256;
}

int launch_bq_scan1(const uint64_t* codes, int64_t n_rows, int words, const uint64_t* qcode,
                    int S, int ctas, void* scratch, int32_t* sl_id, uint16_t* sl_h, int* sl_n,
                    int* status, uint64_t wait_ns, int stream_path, cudaStream_t st) {
    if (!bq_scan1_supported(words, S) || n_rows <= 0) return PION_B200_ESHAPE;
    const int dim = words * 64;
    char* base = static_cast<char*>(scratch);
    uint16_t* dist = reinterpret_cast<uint16_t*>(base);
    size_t off = (size_t)(n_rows * 2 + 255) / 256 * 256;
    int* hist = reinterpret_cast<int*>(base + off);
    off += (size_t)(dim + 1 + 63) / 64 * 256;
    uint64_t* keys = reinterpret_cast<uint64_t*>(base + off);
    off += 512 * 8;
    int32_t* ties = reinterpret_cast<int32_t*>(base + off);
    off += bq::B1_TIECAP * 4;
    int* meta = reinterpret_cast<int*>(base + off);
    const int want = n_rows < S ? (int)n_rows : S;
    if (cudaMemsetAsync(hist, 0, (size_t)(dim + 1) * 4, st) != cudaSuccess ||
        cudaMemsetAsync(meta, 0, 16, st) != cudaSuccess)
        return PION_B200_ECUDA;
    const int64_t per = (n_rows + ctas - 1) / ctas;
    if (words * 8 <= bq::B1S_MAX_ROW_BYTES && stream_path != 1) {
        const size_t ssm = bq::b1s_smem_bytes(words);
        if (set_smem_limit((const void*)bq::bq_scan1_stream_kernel, (int)ssm) != 0)
            return PION_B200_ECUDA;
        bq::bq_scan1_stream_kernel<<<ctas, bq::B1_THREADS, ssm, st>>>(
            codes, n_rows, words, qcode, per, want, dist, hist, status, wait_ns);
    } else {
        const size_t hsm = (size_t)(dim + 1) * 4;
        if (hsm > 48 * 1024 &&
            set_smem_limit((const void*)bq::bq_scan1_hist_kernel, (int)hsm) != 0)
            return PION_B200_ECUDA;
        bq::bq_scan1_hist_kernel<<<ctas, bq::B1_THREADS, hsm, st>>>(codes, n_rows, words, qcode,
                                                                     per, want, dist, hist);
    }
    bq::bq_scan1_collect_kernel<<<ctas, bq::B1_THREADS, 0, st>>>(dist, n_rows, dim, hist, want,
                                                                  per, keys, ties, meta);
    const size_t fsm = (size_t)(bq::B1_TIECAP + 512) * 8;
    if (set_smem_limit((const void*)bq::bq_scan1_finish_kernel, (int)fsm) != 0)
        return PION_B200_ECUDA;
    bq::bq_scan1_finish_kernel<<<1, 1024, fsm, st>>>(dist, n_rows, keys, ties, meta, want, S,
                                                     sl_id, sl_h, sl_n);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int bq_tile_rows() { return bq::BN; }
int bq_query_tile() { return bq::BM; }
int bq_k_block() { return bq::BK; }
int bq_cap() { return bq::CAP; }
int bq_lists_per_split() { return bq::EPI_WARPS / 4; }

int launch_signs(const float* x, int64_t n_rows, int dim, int8_t* pm, uint64_t* codes,
                 cudaStream_t st) {
    if (n_rows <= 0) return 0;
    bq::signs_kernel<<<(unsigned)((n_rows + 7) / 8), 256, 0, st>>>(x, n_rows, dim, pm, codes);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int launch_bq_tc(const BqTcLaunch& L, cudaStream_t st) {
    bq::TcParams p;
    p.dot_min = L.dot_min;
    p.n_rows = L.n_rows;
    p.nq = L.nq;
    p.dim = L.dim;
    p.tile_begin = L.tile_begin;
    p.tile_end = L.tile_end;
    p.n_splits = L.n_splits;
    p.kblocks = (L.dim + bq::BK - 1) / bq::BK;
    p.n_lists = L.n_lists;
    p.list_base = L.list_base;
    p.cand_id = L.cand_id;
    p.cand_h = L.cand_h;
    p.cand_n = L.cand_n;
    p.status = L.status;
    if (p.tile_end <= p.tile_begin || p.n_splits < 1 ||
        p.list_base + p.n_splits * bq_lists_per_split() > p.n_lists)
        return PION_B200_ESHAPE;
    if (set_smem_limit((const void*)bq::bq_tc_kernel<bq::EPI_WARPS / 4>, (int)bq::SMEM_BYTES) != 0)
        return PION_B200_ECUDA;
    dim3 grid((L.nq + bq::BM - 1) / bq::BM, L.n_splits);
    bq::bq_tc_kernel<bq::EPI_WARPS / 4><<<grid, bq::THREADS, bq::SMEM_BYTES, st>>>(
        *L.tmap_q, *L.tmap_rows, p);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int launch_bq_select(const int32_t* cid, const uint16_t* ch, const int* cn, int nq, int n_lists,
                     int dim, int S, int32_t* out_id, uint16_t* out_h, int* out_n,
                     int out_qstride, int n_qstride, int* next_dot_min, int* flagged,
                     int* n_flagged, int force_flag, cudaStream_t st) {
    if (nq <= 0) return 0;
    if (S > 256) return PION_B200_ESHAPE;
    const size_t smem = (size_t)((dim + 1 + 3) & ~3) * 4 + (size_t)n_lists * 4;
    if (smem > 48 * 1024 && set_smem_limit((const void*)bq::bq_select_kernel, (int)smem) != 0)
        return PION_B200_ECUDA;
    bq::bq_select_kernel<<<nq, bq::SEL_THREADS, smem, st>>>(
        cid, ch, cn, n_lists, dim, S, out_id, out_h, out_n, out_qstride, n_qstride, next_dot_min,
        flagged, n_flagged, force_flag);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int launch_bq_fallback(const uint64_t* codes, int64_t n_rows, int words, const uint64_t* qcodes,
                       const int* flagged, const int* n_flagged, int S, int32_t* out_id,
                       uint16_t* out_h, int* out_n, int num_sms, cudaStream_t st) {
    bq::bq_fallback_kernel<<<num_sms, bq::SEL_THREADS, (size_t)(words * 64 + 1) * 4, st>>>(
        codes, n_rows, words, qcodes, flagged, n_flagged, S, out_id, out_h, out_n);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int launch_bq_rerank_wide(const float* rows, int dim, const float* qn, const int32_t* sl_id,
                          const int* sl_n, int S, int nq, int k, int64_t id_base, float* dist,
                          float* out_d, int32_t* out_i, cudaStream_t st) {
    if (nq <= 0) return 0;
    if (dim % 16 != 0 || S > 256 || (size_t)dim * 4 > 48 * 1024) return PION_B200_ESHAPE;
    dim3 grid((S + bq::RW_ROWS - 1) / bq::RW_ROWS, nq);
    bq::bq_rerank_rows_kernel<<<grid, bq::RW_THREADS, (size_t)dim * 4, st>>>(rows, dim, qn, sl_id,
                                                                            sl_n, S, dist);
    bq::bq_rerank_pick_kernel<<<(nq + 3) / 4, 128, 0, st>>>(dist, sl_id, sl_n, S, nq, k, id_base,
                                                            out_d, out_i);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int launch_bq_rerank_staged(const float* rows, int dim, const float* qn, const int32_t* sl_id,
                            const int* sl_n, int S, int nq, int k, int64_t id_base, float* dist,
                            unsigned* done, int* status, uint64_t wait_ns, float* out_d,
                            int32_t* out_i, cudaStream_t st) {
    if (nq <= 0) return 0;
    const size_t smem = (size_t)dim * 4 + (size_t)bq::RS_ROWS * (dim + bq::RS_PAD) * 4 + 16;
    if (dim % 16 != 0 || S > 256 || smem > 200 * 1024) return PION_B200_ESHAPE;
    if (smem > 48 * 1024 &&
        set_smem_limit((const void*)bq::bq_rerank_staged_kernel, (int)smem) != 0)
        return PION_B200_ECUDA;
    if (cudaMemsetAsync(done, 0, (size_t)nq * 4, st) != cudaSuccess) return PION_B200_ECUDA;
    dim3 grid((S + bq::RS_ROWS - 1) / bq::RS_ROWS, nq);
    bq::bq_rerank_staged_kernel<<<grid, 32, smem, st>>>(rows, dim, qn, sl_id, sl_n, S, k, id_base,
                                                        dist, done, status, wait_ns, out_d, out_i);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int launch_bq_rerank(const float* rows, int dim, const float* qn, const int32_t* sl_id,
                     const int* sl_n, int S, int nq, int k, int64_t id_base, float* out_d,
                     int32_t* out_i, cudaStream_t st) {
    if (nq <= 0) return 0;
    const size_t smem = (size_t)S * 4 + (dim % 16 == 0 ? (size_t)dim * 4 : 0);
    if (smem > 48 * 1024 && set_smem_limit((const void*)bq::bq_rerank_kernel, (int)smem) != 0)
        return PION_B200_ECUDA;
    bq::bq_rerank_kernel<<<nq, 256, smem, st>>>(rows, dim, qn, sl_id, sl_n, S, nq, k, id_base,
                                                out_d, out_i);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

}  // namespace pion
