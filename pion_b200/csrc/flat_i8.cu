// FLAT INT8 inner-product KNN on B200 (sm_100a).
//
// Reference semantics (pavelhorak/pion):
//   score(t, r) = (f32(dot_i32(q[t], keys[r])) * row_scale[r]) * q_scale[t]
//     src/vector/reference/pkm_ref.mojo:47-61 (ref_pkm_scores_i8)
//   top-k largest per query, seeded in index order, strict `>` admission
//     src/vector/reference/pkm_ref.mojo:110-130 (ref_pkm_topk_max)
//   rows quantised per row, scale = max|x|/127
//     src/vector/pkm_kernels.mojo:152-191 (pkm_quantize_rows_i8)
//
// Kernels:
//   flat_i8_tc_kernel     batched scoring on tcgen05 (kind::i8, TMEM accumulators,
//                         TMA-staged 128B-swizzled tiles) with the top-k fused into
//                         the TMEM epilogue: no score matrix reaches HBM.
//   flat_i8_scan1_kernel  one query: an HBM stream of 128-bit loads with dp4a and a
//                         fused top-k.
//   merge_lists_kernel    per-query merge of sorted candidate lists.
//   quantize_rows_i8_kernel, tile_max_kernel  index preparation.
#include <cstdint>
#include <cstdio>
#include <cstdlib>

#include "common.cuh"
#include "internal.h"

namespace pion {
namespace fi8 {

constexpr int BM = 128;             // queries per CTA tile (UMMA M, TMEM lanes)
constexpr int BN = 256;             // index rows per tile (UMMA N, TMEM columns)
constexpr int BK = 128;             // bytes of K per pipeline stage (one swizzle row)
constexpr int STAGES = 4;
constexpr int UMMA_K = 32;          // int8 K consumed by one tcgen05.mma
constexpr int A_BYTES = BM * BK;    // 16 KB
constexpr int B_BYTES = BN * BK;    // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
// Threads: warp 0 TMA producer, warp 1 MMA issuer, then 4 or 8 epilogue warps.
constexpr uint32_t TMEM_COLS = 2 * BN;  // double-buffered accumulator
constexpr uint32_t IDESC = make_idesc_i8(BM, BN);
constexpr size_t SMEM_PIPE_BYTES = 1024 + (size_t)STAGES * STAGE_BYTES + 256;
// per epilogue warp: a 32-value row per lane for the candidate path
constexpr size_t STASH_BYTES = 32 * 32 * 4;
__host__ __device__ constexpr size_t smem_bytes(int epi_warps) {
    return SMEM_PIPE_BYTES + (size_t)epi_warps * STASH_BYTES;
}

static_assert(BN <= 256 && BN % 16 == 0, "UMMA N");
static_assert(BK % UMMA_K == 0, "K step");

struct TcParams {
    const float* row_scale;    // [n_rows]
    const float* tile_rs_max;  // [n_tiles] max row_scale over each BN-row tile
    const float* q_scale;      // [nq]
    const float* thr0;         // optional per-query lower bound on the final k-th score
    int thr0_stride;           // elements between consecutive queries' bounds
    int64_t n_rows;
    int nq;
    int k;
    int tile_begin;            // index tiles [tile_begin, tile_end) are scored
    int tile_end;
    int n_splits;
    int kblocks;
    int n_lists;               // candidate lists per query in cand_* (layout [nq][n_lists][k])
    int list_base;             // first list this launch writes
    int bound_mode;            // 1: keep one exact score per 32-row chunk (threshold pass)
    float* cand_val;
    int32_t* cand_idx;
    int* status;
    uint64_t wait_ns;          // budget of every mbarrier wait
    int test_stall;            // 1: CTA (0, 0)'s MMA warp first waits on a barrier that
                               // nothing arrives on (exercises the timeout path)
};

// score(d) = fl(fl(fl(d) * rs) * qs), the reference epilogue for one dot product.
__device__ __forceinline__ float i8_score(int32_t d, float rs, float qs) {
    return __fmul_rn(__fmul_rn(__int2float_rn(d), rs), qs);
}

// Integer pre-filter: an integer d such that every dot <= d scores <= thr in a tile
// whose row scales are all <= rs_max, given inv = fl(1 / fl(rs_max * qs)).
// fl(x*y) is monotone in each non-negative factor, so score(d) <= fl(fl(fl(d) *
// rs_max) * qs) <= d * rs_max * qs * (1 + 2^-24)^3.  est = fl(thr * inv) exceeds
// thr / (rs_max * qs) by at most (1 + 2^-24)^3; shrinking it by 2^-20 and taking two
// off its floor leaves d < thr / (rs_max * qs) * (1 - 5.9e-7), so score(d) < thr.
// Returns INT32_MIN (score everything exactly) when thr < 0 or nothing is finite.
__device__ __forceinline__ int32_t dot_bound(float thr, float inv) {
    if (!(thr >= 0.0f)) return INT32_MIN;
    float est = __fmul_rz(thr, inv);
    est = __fmul_rz(est, 1.0f - 0x1p-20f);
    if (!(est < 2.0e9f)) return INT32_MIN;
    return __float2int_rz(est) - 2;
}

// rsv[c] for a loop-variant c without indexing the register array dynamically.
template <int N>
__device__ __forceinline__ float sel_rs(const float (&rsv)[N], int c) {
    float v = rsv[0];
#pragma unroll
    for (int i = 1; i < N; ++i) v = (c == i) ? rsv[i] : v;
    return v;
}

// Epilogue state of one query (one thread).
template <int KCAP>
struct QueryTop {
    TopKDesc<KCAP> top;
    float thr;        // admission threshold: max(current k-th score, lower bound - 1 ulp)
    float floor_thr;  // the lower bound - 1 ulp (or -inf)
    int32_t dmin;     // integer pre-filter for the current tile
};

// One 32-column chunk of TMEM accumulators: integer pre-filter into a candidate
// mask, then the exact reference score for the candidates, ascending columns.
// Candidates are common on clustered data (a lane has one in a few percent of the
// chunks, so most chunks have some lane with one), so this path is lane-local: a lane
// with candidates parks its own 32 values in its own row of `stash` (eight 16-byte
// stores, slots XOR-swizzled by lane so a quarter-warp's stores hit distinct banks)
// and reads them back by index; the row scale comes from L1 (the tile's scales were
// just loaded).  No warp synchronisation: lanes without candidates go on at once.
template <int KCAP>
__device__ __forceinline__ void scan_chunk(const uint32_t (&r)[32], int64_t col0, int64_t valid,
                                           const float* __restrict__ row_scale, float qs,
                                           float inv, int k, uint32_t* stash, int lane,
                                           QueryTop<KCAP>& st) {
    // Common case first: one max-reduction says whether any column can qualify.
    int32_t mx = (int32_t)r[0];
#pragma unroll
    for (int j = 1; j < 32; ++j) mx = max(mx, (int32_t)r[j]);
    if (!(mx > st.dmin)) return;
    uint32_t mask;
    if (st.dmin == INT32_MIN) {
        mask = 0xffffffffu;
    } else {
        // bit j = (r[j] > dmin) = sign of dmin - r[j] (|r| < 2^25 and dmin < 2^31 - 2^25:
        // no overflow), shifted in by two independent funnel-shift chains
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int j = 15; j >= 0; --j) {
            lo = __funnelshift_l((uint32_t)(st.dmin - (int32_t)r[j]), lo, 1);
            hi = __funnelshift_l((uint32_t)(st.dmin - (int32_t)r[j + 16]), hi, 1);
        }
        mask = lo | (hi << 16);
    }
    if (valid < 32) mask &= valid <= 0 ? 0u : ((1u << valid) - 1u);
    if (!mask) return;
    uint4* row4 = reinterpret_cast<uint4*>(stash + lane * 32);
    const int sw = lane & 7;
#pragma unroll
    for (int i = 0; i < 8; ++i)
        row4[i ^ sw] = make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
    const uint32_t* row = stash + lane * 32;
#pragma unroll 1
    while (mask) {
        const int j = __ffs(mask) - 1;
        mask &= mask - 1u;
        const int32_t dv = (int32_t)row[(((j >> 2) ^ sw) << 2) | (j & 3)];
        if (dv <= st.dmin) continue;
        const int64_t col = col0 + j;
        const float s = i8_score(dv, __ldg(&row_scale[col]), qs);
        if (s > st.thr) {
            st.top.insert(s, (int32_t)col);
            st.thr = fmaxf(st.top.kth(k), st.floor_thr);
            st.dmin = dot_bound(st.thr, inv);
        }
    }
}

// Threshold pass: one exact score per 32-column chunk, that of the chunk's largest dot
// (first column on ties), offered to the top-k.  The rows offered are distinct, so the
// k-th best of them is at most the k-th best score of the chunks' rows: a lower bound
// of the final k-th score that costs one candidate per chunk instead of every column
// above the running threshold.
template <int KCAP>
__device__ __forceinline__ void bound_chunk(const uint32_t (&r)[32], int64_t col0, int64_t valid,
                                            float rs_lane, float qs, float inv, int k,
                                            QueryTop<KCAP>& st) {
    int32_t mx = INT32_MIN;
    int jm = 0;
    bool any = false;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const int32_t v = (int32_t)r[j];
        const bool take = j < valid && (!any || v > mx);
        mx = take ? v : mx;
        jm = take ? j : jm;
        any = any || j < valid;
    }
    const float rs = __shfl_sync(0xffffffffu, rs_lane, jm);  // lane j holds column j's scale
    if (any && mx > st.dmin) {
        const float s = i8_score(mx, rs, qs);
        if (s > st.thr) {
            st.top.insert(s, (int32_t)(col0 + jm));
            st.thr = fmaxf(st.top.kth(k), st.floor_thr);
            st.dmin = dot_bound(st.thr, inv);
        }
    }
}

template <int KCAP>
__device__ __forceinline__ void process_chunk(bool bound, const uint32_t (&r)[32], int64_t col0,
                                              int64_t valid, float rs_lane,
                                              const float* __restrict__ row_scale, float qs,
                                              float inv, int k, uint32_t* stash, int lane,
                                              QueryTop<KCAP>& st) {
    if (bound)
        bound_chunk<KCAP>(r, col0, valid, rs_lane, qs, inv, k, st);
    else
        scan_chunk<KCAP>(r, col0, valid, row_scale, qs, inv, k, stash, lane, st);
}

template <int KCAP, int EPI_WARPS>
__global__ void __launch_bounds__(64 + 32 * EPI_WARPS, 1)
    flat_i8_tc_kernel(const __grid_constant__ CUtensorMap tmap_q,
                      const __grid_constant__ CUtensorMap tmap_rows, TcParams p) {
    constexpr int HALVES = EPI_WARPS / 4;        // column slices of one TMEM lane quarter
    constexpr int COLS = BN / HALVES;            // columns per epilogue warp per tile
    constexpr int CHUNKS = COLS / 32;
    static_assert(CHUNKS % 2 == 0, "chunks are processed in pairs");
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
    uint64_t* stall = drain + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(stall + 1);
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
        mbar_init(stall, 1);
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
        // ------------------------------------------------------ TMA producer
        if (lane == 0) {
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
                    if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, abort_flag, p.wait_ns)) {
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
            // Every copy this thread issued lands before the CTA may exit.
            for (int s = 0; s < STAGES; ++s)
                if (issued[s]) mbar_wait(&full[s], issued_parity[s], p.status, nullptr, p.wait_ns);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------- MMA issuer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            // Test hook: a wait that runs out (nothing arrives on `stall`), after which the
            // pipeline drains and the CTA frees its TMEM and returns with ETIMEOUT recorded.
            const bool stalled = p.test_stall && blockIdx.x == 0 && blockIdx.y == 0 &&
                                 !mbar_wait(stall, 0, p.status, abort_flag, p.wait_ns);
            for (int t = 0; t < my_tiles && !stalled; ++t) {
                const int buf = t & 1;
                const uint32_t use = (uint32_t)(t >> 1);
                if (!mbar_wait(&tempty[buf], (use & 1u) ^ 1u, p.status, abort_flag, p.wait_ns))
                    break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(buf * BN);
                bool ok = true;
                for (int kb = 0; kb < p.kblocks; ++kb) {
                    if (!mbar_wait(&full[stage], phase, p.status, abort_flag, p.wait_ns)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + stage * A_BYTES);
                    const uint32_t b0 = smem_u32(sB + stage * B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < BK / UMMA_K; ++kk) {
                        mma_i8(d_tmem, make_sw128_kmajor_desc(a0 + kk * UMMA_K),
                               make_sw128_kmajor_desc(b0 + kk * UMMA_K), IDESC,
                               (kb | kk) != 0 ? 1u : 0u);
                    }
                    tc_commit(&empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                tc_commit(&tfull[buf]);
            }
            // All MMAs issued above complete before TMEM is released.
            tc_commit(drain);
            mbar_wait(drain, 0, p.status, nullptr, p.wait_ns);
        }
    } else {
        // --------------------------------------------- epilogue: score + top-k
        const int ew = warp - 2;
        uint32_t* stash = stash_all + ew * (STASH_BYTES / 4);
        const int lg = warp & 3;  // TMEM lane quarter this warp may read
        const int half = ew >> 2; // column slice of each tile
        const int row = lg * 32 + lane;
        const int q = qt * BM + row;
        const bool q_ok = q < p.nq;
        const float qs = q_ok ? p.q_scale[q] : 0.0f;
        QueryTop<KCAP> st;
        st.top.init();
        st.floor_thr = -INFINITY;
        if (q_ok && p.thr0) {
            const float t0 = p.thr0[(size_t)q * p.thr0_stride];
            // rows scoring exactly the bound may still rank in the top k (ties break by id)
            if (t0 > -INFINITY) st.floor_thr = nextafterf(t0, -INFINITY);
        }
        st.thr = st.floor_thr;
        const bool bound = p.bound_mode != 0;
        for (int t = 0; t < my_tiles; ++t) {
            const int buf = t & 1;
            const uint32_t use = (uint32_t)(t >> 1);
            const int tile = t_begin + t;
            const int64_t col0 = (int64_t)tile * BN + half * COLS;
            const int64_t valid = p.n_rows - col0;  // columns of this slice inside the index
            // Row scales of this slice (lane j of chunk c: column c*32 + j) and the tile
            // maximum, loaded before the wait so that their latency hides behind it.
            float rsv[CHUNKS];
#pragma unroll
            for (int c = 0; c < CHUNKS; ++c)
                rsv[c] = (c * 32 + lane < valid) ? __ldg(&p.row_scale[col0 + c * 32 + lane]) : 0.f;
            const float rs_max = __ldg(&p.tile_rs_max[tile]);
            // Every lane waits; the warp proceeds only if all of them saw the phase,
            // so the warp-collective TMEM loads below stay convergent.
            const bool got = mbar_wait(&tfull[buf], use & 1u, p.status, abort_flag, p.wait_ns);
            if (!__all_sync(0xffffffffu, got)) break;
            tc_fence_after();
            const float inv = __frcp_rn(__fmul_rn(rs_max, qs));
            st.dmin = q_ok ? dot_bound(st.thr, inv) : INT32_MAX;
            const uint32_t taddr = tmem_base + ((uint32_t)(lg * 32) << 16) +
                                   (uint32_t)(buf * BN + half * COLS);
            if constexpr (KCAP <= 32) {
                uint32_t ra[32], rb[32];
                tmem_ld32(taddr, ra);
                tmem_ld_wait_regs(ra);
                // Chunks in pairs: the load of the next chunk is in flight while the
                // current one is scanned.
#pragma unroll 1
                for (int c = 0; c < CHUNKS; c += 2) {
                    __syncwarp();
                    tmem_ld32(taddr + (uint32_t)((c + 1) * 32), rb);
                    process_chunk<KCAP>(bound, ra, col0 + c * 32, valid - c * 32,
                                        sel_rs<CHUNKS>(rsv, c), p.row_scale, qs, inv, p.k,
                                        stash, lane, st);
                    __syncwarp();
                    tmem_ld_wait_regs(rb);
                    if (c + 2 < CHUNKS) tmem_ld32(taddr + (uint32_t)((c + 2) * 32), ra);
                    process_chunk<KCAP>(bound, rb, col0 + (c + 1) * 32, valid - (c + 1) * 32,
                                        sel_rs<CHUNKS>(rsv, c + 1), p.row_scale, qs, inv,
                                        p.k, stash, lane, st);
                    __syncwarp();
                    if (c + 2 < CHUNKS) tmem_ld_wait_regs(ra);
                }
            } else {
                // a 64-entry list leaves no registers for a second chunk buffer
#pragma unroll 1
                for (int c = 0; c < CHUNKS; ++c) {
                    uint32_t ra[32];
                    __syncwarp();
                    tmem_ld32(taddr + (uint32_t)(c * 32), ra);
                    tmem_ld_wait_regs(ra);
                    process_chunk<KCAP>(bound, ra, col0 + c * 32, valid - c * 32,
                                        sel_rs<CHUNKS>(rsv, c), p.row_scale, qs, inv, p.k,
                                        stash, lane, st);
                }
            }
            tc_fence_before();
            mbar_arrive(&tempty[buf]);
        }
        if (q_ok) {
            const size_t base =
                ((size_t)q * p.n_lists + p.list_base + (size_t)split * HALVES + half) * p.k;
#pragma unroll
            for (int j = 0; j < KCAP; ++j)
                if (j < p.k) {
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

// Max row scale per BN-row tile, for the integer admission bound above.
__global__ void tile_max_kernel(const float* rs, int64_t n_rows, int tile, float* out,
                                int n_tiles) {
    const int t = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (t >= n_tiles) return;
    const int lane = threadIdx.x & 31;
    float m = 0.0f;
    for (int64_t r = (int64_t)t * tile + lane; r < (int64_t)(t + 1) * tile && r < n_rows; r += 32)
        m = fmaxf(m, rs[r]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) out[t] = m;
}

// ------------------------------------------------------------- one query scan
constexpr int SCAN_THREADS = 256;
constexpr int SCAN_GROUP = 8;                      // lanes per row: 8 x 16 B = 128 B
constexpr int SCAN_GROUPS = SCAN_THREADS / SCAN_GROUP;
constexpr int SCAN_MAX_CHUNKS = 1024;              // dim <= 16384
constexpr int SCAN_PER_LANE = 12;                  // fully unrolled up to dim 1536

__device__ __forceinline__ int4 ld_stream(const int4* p) {
    int4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

template <int KCAP>
__global__ void __launch_bounds__(SCAN_THREADS)
    flat_i8_scan1_kernel(const int8_t* __restrict__ rows, const float* __restrict__ row_scale,
                         int64_t n_rows, int dim, const int8_t* __restrict__ q,
                         const float* __restrict__ q_scale, int k, int64_t rows_per_cta,
                         float* cand_val, int32_t* cand_idx) {
    __shared__ int4 qv[SCAN_MAX_CHUNKS];
    __shared__ float lv[SCAN_GROUPS * KCAP];
    __shared__ int32_t li[SCAN_GROUPS * KCAP];
    const int chunks = dim >> 4;
    for (int c = threadIdx.x; c < chunks; c += SCAN_THREADS)
        qv[c] = reinterpret_cast<const int4*>(q)[c];
    __syncthreads();
    const float qsc = q_scale[0];
    const int g = threadIdx.x / SCAN_GROUP;
    const int gl = threadIdx.x % SCAN_GROUP;
    const int64_t r0 = (int64_t)blockIdx.x * rows_per_cta;
    int64_t r1 = r0 + rows_per_cta;
    if (r1 > n_rows) r1 = n_rows;
    TopKDesc<KCAP> top;
    top.init();
    float thr = -INFINITY;
    // The trip count is the same for every lane of the CTA (rows past r1 are masked),
    // so the full-warp shuffles below always see all 32 lanes.
    for (int64_t base = r0; base < r1; base += SCAN_GROUPS) {
        const int64_t r = base + g;
        const bool valid = r < r1;
        int acc = 0;
        if (valid) {
            const int4* rp = reinterpret_cast<const int4*>(rows + r * dim);
            if (KCAP <= 16 && chunks <= SCAN_GROUP * SCAN_PER_LANE) {
                // every load of the row in flight at once (12 per lane at dim 1536)
                int4 a[SCAN_PER_LANE];
#pragma unroll
                for (int i = 0; i < SCAN_PER_LANE; ++i) {
                    const int c = gl + i * SCAN_GROUP;
                    if (c < chunks) a[i] = ld_stream(rp + c);
                }
#pragma unroll
                for (int i = 0; i < SCAN_PER_LANE; ++i) {
                    const int c = gl + i * SCAN_GROUP;
                    if (c < chunks) {
                        const int4 b = qv[c];
                        acc = __dp4a(a[i].x, b.x, acc);
                        acc = __dp4a(a[i].y, b.y, acc);
                        acc = __dp4a(a[i].z, b.z, acc);
                        acc = __dp4a(a[i].w, b.w, acc);
                    }
                }
            } else {
#pragma unroll 4
                for (int c = gl; c < chunks; c += SCAN_GROUP) {
                    const int4 a = ld_stream(rp + c);
                    const int4 b = qv[c];
                    acc = __dp4a(a.x, b.x, acc);
                    acc = __dp4a(a.y, b.y, acc);
                    acc = __dp4a(a.z, b.z, acc);
                    acc = __dp4a(a.w, b.w, acc);
                }
            }
        }
        acc += __shfl_xor_sync(0xffffffffu, acc, 1);
        acc += __shfl_xor_sync(0xffffffffu, acc, 2);
        acc += __shfl_xor_sync(0xffffffffu, acc, 4);
        if (valid) {
            const float s = __fmul_rn(__fmul_rn(__int2float_rn(acc), __ldg(&row_scale[r])), qsc);
            if (s > thr) {
                top.insert(s, (int32_t)r);
                thr = top.kth(k);
            }
        }
    }
    if (gl == 0) {
#pragma unroll
        for (int j = 0; j < KCAP; ++j) {
            lv[g * KCAP + j] = top.v[j];
            li[g * KCAP + j] = top.i[j];
        }
    }
    __syncthreads();
    // Warp 0 merges the CTA's SCAN_GROUPS sorted lists (one per lane) into k.
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        int cur = 0;
        for (int j = 0; j < k; ++j) {
            float hv = cur < KCAP ? lv[lane * KCAP + cur] : -INFINITY;
            int32_t hi = cur < KCAP ? li[lane * KCAP + cur] : -1;
            float bv = hv;
            int32_t bi = hi;
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
                cand_val[(size_t)blockIdx.x * k + j] = bv;
                cand_idx[(size_t)blockIdx.x * k + j] = bi;
            }
        }
    }
}

}  // namespace fi8

// ------------------------------------------------------------------ merging --
// One warp per query merges n_lists sorted lists of k (score, id) pairs into the k
// best by (score, id), adding id_offset to valid ids.  Input layouts: [nq][n_lists][k]
// (list stride k) or lists-major [n_lists][nq][k] (an all-gather of per-shard lists);
// scores and ids either in two arrays (es = 1) or interleaved as 8-byte (f32 score,
// i32 id) pairs (es = 2, ci = the ids' view of the same buffer).
//
// When a query's lists fit the warp's shared-memory slice they are staged there with
// coalesced loads first, so the k selection rounds read shared memory only.  Each lane
// keeps the best head of its own lists (l = lane, lane + 32, ...) across rounds and
// rescans them only when one of its lists supplied the winner.
constexpr int MERGE_WARPS = 4;
constexpr int MERGE_MAX_LISTS = 2048;
constexpr int MERGE_STAGE_ENTRIES = 1024;  // per warp: 8 KB of staged pairs

template <bool DESC, bool STAGED>
__global__ void __launch_bounds__(MERGE_WARPS * 32)
    merge_lists_kernel(const float* __restrict__ cv, const int32_t* __restrict__ ci, int es,
                       int nq, int n_lists, int k, int64_t id_offset, float* out_v,
                       int32_t* out_i, int lists_major, int out_stride, int out_es, int lm_nq) {
    __shared__ uint16_t cursor[MERGE_WARPS][STAGED ? MERGE_STAGE_ENTRIES : MERGE_MAX_LISTS];
    __shared__ float stage_v[STAGED ? MERGE_WARPS : 1][STAGED ? MERGE_STAGE_ENTRIES : 1];
    __shared__ int32_t stage_i[STAGED ? MERGE_WARPS : 1][STAGED ? MERGE_STAGE_ENTRIES : 1];
    const int w = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int q = blockIdx.x * MERGE_WARPS + w;
    if (q >= nq) return;
    for (int l = lane; l < n_lists; l += 32) cursor[w][l] = 0;
    const float pad = DESC ? -INFINITY : INFINITY;
    // entry c of list l of query q sits at element (base + l * lstride + c) * es
    const size_t base = lists_major ? (size_t)q * k : (size_t)q * n_lists * k;
    const size_t lstride = lists_major ? (size_t)lm_nq * k : (size_t)k;
    if (STAGED) {
        // eight loads in flight per lane before the first store (a query's lists are
        // one contiguous run unless lists-major)
        const int total = n_lists * k;
        constexpr int U = 8;
        for (int e0 = lane; e0 < total; e0 += 32 * U) {
            float v[U];
            int32_t id[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int e = e0 + 32 * u;
                if (e < total) {
                    size_t at;
                    if (lists_major) {
                        const int l = e / k, c = e - l * k;
                        at = (base + (size_t)l * lstride + c) * es;
                    } else {
                        at = (base + (size_t)e) * es;
                    }
                    v[u] = cv[at];
                    id[u] = ci[at];
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int e = e0 + 32 * u;
                if (e < total) {
                    stage_v[w][e] = v[u];
                    stage_i[w][e] = id[u];
                }
            }
        }
    }
    __syncwarp();
    auto head = [&](int l, int c, float& v, int32_t& id) {
        if (STAGED) {
            v = stage_v[w][l * k + c];
            id = stage_i[w][l * k + c];
        } else {
            const size_t at = (base + (size_t)l * lstride + c) * es;
            v = cv[at];
            id = ci[at];
        }
    };
    // best head among this lane's own lists
    auto lane_best = [&](float& bv, int32_t& bi, int& bl) {
        bv = pad;
        bi = -1;
        bl = -1;
        for (int l = lane; l < n_lists; l += 32) {
            const int c = cursor[w][l];
            if (c >= k) continue;
            float v;
            int32_t id;
            head(l, c, v, id);
            if (bl < 0 || merge_better<DESC>(v, id, bv, bi)) {
                bv = v;
                bi = id;
                bl = l;
            }
        }
    };
    float mv;
    int32_t mi;
    int ml;
    lane_best(mv, mi, ml);
    for (int j = 0; j < k; ++j) {
        float bv = mv;
        int32_t bi = mi;
        int bl = ml;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            const int ol = __shfl_xor_sync(0xffffffffu, bl, o);
            const bool take = (ol >= 0) && (bl < 0 || merge_better<DESC>(ov, oi, bv, bi) ||
                                            (ov == bv && oi == bi && ol < bl));
            if (take) {
                bv = ov;
                bi = oi;
                bl = ol;
            }
        }
        if (lane == 0) {
            const size_t o = ((size_t)q * out_stride + j) * out_es;
            out_v[o] = bl >= 0 ? bv : pad;
            out_i[o] = (bl >= 0 && bi >= 0) ? (int32_t)(bi + id_offset) : -1;
        }
        if (bl >= 0 && (bl & 31) == lane) {
            cursor[w][bl] += 1;
            lane_best(mv, mi, ml);
        }
    }
}

// Many lists per query (a one-query scan's per-CTA lists): one CTA per query.  Each of
// its MB_WARPS warps merges a contiguous range of the lists (heads read from global
// memory, each lane keeping the best head of its own lists), the warps' k-lists meet in
// shared memory, and warp 0 merges those.  Order and padding as merge_lists_kernel.
constexpr int MB_WARPS = 8;
constexpr int MB_KMAX = 64;

template <bool DESC>
__global__ void __launch_bounds__(MB_WARPS * 32)
    merge_lists_block_kernel(const float* __restrict__ cv, const int32_t* __restrict__ ci,
                             int es, int nq, int n_lists, int k, int64_t id_offset, float* out_v,
                             int32_t* out_i, int lists_major, int out_stride, int out_es,
                             int lm_nq) {
    __shared__ float wv[MB_WARPS][MB_KMAX];
    __shared__ int32_t wi[MB_WARPS][MB_KMAX];
    __shared__ uint16_t cursor[MERGE_MAX_LISTS];
    const int q = blockIdx.x;
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float pad = DESC ? -INFINITY : INFINITY;
    const size_t base = lists_major ? (size_t)q * k : (size_t)q * n_lists * k;
    const size_t lstride = lists_major ? (size_t)lm_nq * k : (size_t)k;
    for (int l = threadIdx.x; l < n_lists; l += blockDim.x) cursor[l] = 0;
    __syncthreads();
    const int l0 = (int)((int64_t)n_lists * w / MB_WARPS);
    const int l1 = (int)((int64_t)n_lists * (w + 1) / MB_WARPS);
    auto lane_best = [&](float& bv, int32_t& bi, int& bl) {
        bv = pad;
        bi = -1;
        bl = -1;
        for (int l = l0 + lane; l < l1; l += 32) {
            const int c = cursor[l];
            if (c >= k) continue;
            const size_t at = (base + (size_t)l * lstride + c) * es;
            const float v = cv[at];
            const int32_t id = ci[at];
            if (bl < 0 || merge_better<DESC>(v, id, bv, bi)) {
                bv = v;
                bi = id;
                bl = l;
            }
        }
    };
    // phase 1: warp w's lists -> its k best in shared memory
    float mv;
    int32_t mi;
    int ml;
    lane_best(mv, mi, ml);
    for (int j = 0; j < k; ++j) {
        float bv = mv;
        int32_t bi = mi;
        int bl = ml;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            const int ol = __shfl_xor_sync(0xffffffffu, bl, o);
            if ((ol >= 0) && (bl < 0 || merge_better<DESC>(ov, oi, bv, bi) ||
                              (ov == bv && oi == bi && ol < bl))) {
                bv = ov;
                bi = oi;
                bl = ol;
            }
        }
        if (lane == 0) {
            wv[w][j] = bl >= 0 ? bv : pad;
            wi[w][j] = bl >= 0 ? bi : -1;
        }
        if (bl >= 0 && ((bl - l0) & 31) == lane) {
            cursor[bl] += 1;
            lane_best(mv, mi, ml);
        }
    }
    __syncthreads();
    // phase 2: warp 0 merges the MB_WARPS lists (list = lane < MB_WARPS)
    if (w != 0) return;
    int cur = 0;
    for (int j = 0; j < k; ++j) {
        const bool has = lane < MB_WARPS && cur < k;
        float bv = has ? wv[lane][cur] : pad;
        int32_t bi = has ? wi[lane][cur] : -1;
        int bl = has ? lane : -1;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            const int ol = __shfl_xor_sync(0xffffffffu, bl, o);
            if ((ol >= 0) && (bl < 0 || merge_better<DESC>(ov, oi, bv, bi) ||
                              (ov == bv && oi == bi && ol < bl))) {
                bv = ov;
                bi = oi;
                bl = ol;
            }
        }
        if (lane == bl) ++cur;
        if (lane == 0) {
            const size_t o = ((size_t)q * out_stride + j) * out_es;
            out_v[o] = bl >= 0 ? bv : pad;
            out_i[o] = (bl >= 0 && bi >= 0) ? (int32_t)(bi + id_offset) : -1;
        }
    }
}

__global__ void fill_results_kernel(float* v, int32_t* i, size_t n, float value, int es) {
    for (size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x; t < n;
         t += (size_t)gridDim.x * blockDim.x) {
        v[t * es] = value;
        i[t * es] = -1;
    }
}

// ------------------------------------------------------------- quantisation --
// pkm_quantize_rows_i8 (src/vector/pkm_kernels.mojo:152-191), one warp per row.
// max|x| is order-independent; the divides and the +-0.5 rounding use the same
// IEEE round-to-nearest operations as the reference, then truncate toward zero.
__global__ void quantize_rows_i8_kernel(const float* __restrict__ src, int64_t n_rows, int d,
                                        int d_pad, int8_t* __restrict__ dst,
                                        float* __restrict__ dst_scale) {
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (r >= n_rows) return;
    const int lane = threadIdx.x & 31;
    const float* sp = src + r * d_pad;
    float m = 0.0f;
    for (int c = lane; c < d; c += 32) m = fmaxf(m, fabsf(sp[c]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float scale = __fdiv_rn(m, 127.0f);
    if (m == 0.0f) scale = 1.0f;
    const float inv = __fdiv_rn(1.0f, scale);
    int8_t* dp = dst + r * d_pad;
    for (int c = lane; c < d_pad; c += 32) {
        int qi = 0;
        if (c < d) {
            const float qv = __fmul_rn(sp[c], inv);
            qi = qv >= 0.0f ? __float2int_rz(__fadd_rn(qv, 0.5f))
                            : __float2int_rz(__fsub_rn(qv, 0.5f));
            qi = qi > 127 ? 127 : (qi < -127 ? -127 : qi);
        }
        dp[c] = (int8_t)qi;
    }
    if (lane == 0) dst_scale[r] = scale;
}

// =========================================================== host launchers ==

int fi8_tile_rows() { return fi8::BN; }

int launch_tile_max(const float* rs, int64_t n_rows, float* out, cudaStream_t st) {
    const int n_tiles = (int)((n_rows + fi8::BN - 1) / fi8::BN);
    if (n_tiles <= 0) return 0;
    const int warps = 8;
    fi8::tile_max_kernel<<<(n_tiles + warps - 1) / warps, warps * 32, 0, st>>>(rs, n_rows, fi8::BN, out,
                                                                          n_tiles);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int launch_quantize_rows_i8(const float* src, int64_t n_rows, int d, int d_pad, int8_t* dst,
                            float* dst_scale, cudaStream_t st) {
    if (n_rows <= 0) return 0;
    const int warps = 8;
    const int64_t blocks = (n_rows + warps - 1) / warps;
    quantize_rows_i8_kernel<<<(unsigned)blocks, warps * 32, 0, st>>>(src, n_rows, d, d_pad, dst,
                                                                     dst_scale);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int launch_fill_results(float* v, int32_t* i, size_t n, float value, cudaStream_t st, int es) {
    if (n == 0) return 0;
    const unsigned blocks = (unsigned)((n + 255) / 256 < 1024 ? (n + 255) / 256 : 1024);
    fill_results_kernel<<<blocks, 256, 0, st>>>(v, i, n, value, es);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int launch_merge_lists(const float* cv, const int32_t* ci, int nq, int n_lists, int k,
                       int64_t id_offset, bool descending, float* out_v, int32_t* out_i,
                       cudaStream_t st, bool lists_major, int out_stride, bool pairs,
                       int out_es, int lm_nq) {
    if (nq <= 0) return 0;
    if (n_lists < 1 || n_lists > MERGE_MAX_LISTS || k < 1 || k > 65535) return PION_B200_ESHAPE;
    if (out_stride <= 0) out_stride = k;
    const int es = pairs ? 2 : 1;
    if (pairs) ci = reinterpret_cast<const int32_t*>(cv) + 1;
    const int lm = lists_major ? 1 : 0;
    if (lm_nq <= 0) lm_nq = nq;  // lists-major: query slots per list
    if (lm_nq < nq) return PION_B200_ESHAPE;
    if (n_lists > 128 && k <= MB_KMAX) {  // few queries, many lists: a CTA per query
        if (descending)
            merge_lists_block_kernel<true><<<nq, MB_WARPS * 32, 0, st>>>(
                cv, ci, es, nq, n_lists, k, id_offset, out_v, out_i, lm, out_stride, out_es, lm_nq);
        else
            merge_lists_block_kernel<false><<<nq, MB_WARPS * 32, 0, st>>>(
                cv, ci, es, nq, n_lists, k, id_offset, out_v, out_i, lm, out_stride, out_es, lm_nq);
        return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
    }
    const int blocks = (nq + MERGE_WARPS - 1) / MERGE_WARPS;
    const bool staged = (int64_t)n_lists * k <= MERGE_STAGE_ENTRIES;
#define PION_MERGE_GO(D, S)                                                              \
    merge_lists_kernel<D, S><<<blocks, MERGE_WARPS * 32, 0, st>>>(cv, ci, es, nq, n_lists, k, \
                                                                  id_offset, out_v, out_i, lm, \
                                                                  out_stride, out_es, lm_nq)
    if (descending) {
        if (staged) PION_MERGE_GO(true, true); else PION_MERGE_GO(true, false);
    } else {
        if (staged) PION_MERGE_GO(false, true); else PION_MERGE_GO(false, false);
    }
#undef PION_MERGE_GO
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

// Splits of the index across CTAs for a batch of n_qt query tiles.  One CTA fills an
// SM (its shared memory), so the launch runs in waves of num_sms CTAs and an SM pays a
// CTA's fixed cost (set-up, pipeline fill and drain, about two tiles' worth) once per
// wave: the modelled time is waves x (2 + the largest CTA's tiles); the smallest wins,
// fewer splits on ties.
int fi8_choose_splits(int n_qt, int n_tiles, int num_sms) {
    int best = 1;
    long best_cost = -1;
    for (int s = 1; s <= 256; ++s) {
        if (s > 1 && n_tiles / s < 4) break;
        const long total = (long)n_qt * s;
        const long waves = (total + num_sms - 1) / num_sms;
        const long cost = waves * (2 + (n_tiles + s - 1) / s);
        if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            best = s;
        }
    }
    return best;
}

int fi8_kcap(int k) { return k <= 16 ? 16 : (k <= 32 ? 32 : (k <= 64 ? 64 : 0)); }

template <int KCAP, int EPI_WARPS>
static int launch_tc_k(const CUtensorMap& tq, const CUtensorMap& tr, const fi8::TcParams& p,
                       int n_qt, cudaStream_t st) {
    if (set_smem_limit((const void*)fi8::flat_i8_tc_kernel<KCAP, EPI_WARPS>,
                       (int)fi8::smem_bytes(EPI_WARPS)) != 0)
        return PION_B200_ECUDA;
    dim3 grid(n_qt, p.n_splits);
    fi8::flat_i8_tc_kernel<KCAP, EPI_WARPS>
        <<<grid, 64 + 32 * EPI_WARPS, fi8::smem_bytes(EPI_WARPS), st>>>(tq, tr, p);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

// Epilogue warps per CTA: 8 (two per TMEM lane quarter, each taking half of the
// columns) for a 16-entry register top-k, else 4 (the 320-thread block caps a
// thread at 168 registers).
static int fi8_epi_warps(int k) { return k <= 16 ? 8 : 4; }

int fi8_lists_per_split(int k) { return fi8_epi_warps(k) / 4; }

int launch_flat_i8_tc(const Fi8TcLaunch& L, cudaStream_t st) {
    fi8::TcParams p;
    p.row_scale = L.row_scale;
    p.tile_rs_max = L.tile_rs_max;
    p.q_scale = L.q_scale;
    p.thr0 = L.thr0;
    p.thr0_stride = L.thr0_stride;
    p.n_rows = L.n_rows;
    p.nq = L.nq;
    p.k = L.k;
    p.tile_begin = L.tile_begin;
    p.tile_end = L.tile_end;
    p.n_splits = L.n_splits;
    p.kblocks = (L.dim + fi8::BK - 1) / fi8::BK;
    p.n_lists = L.n_lists;
    p.list_base = L.list_base;
    p.bound_mode = L.bound_mode;
    p.cand_val = L.cand_val;
    p.cand_idx = L.cand_idx;
    p.status = L.status;
    p.wait_ns = L.wait_ns;
    p.test_stall = L.test_stall;
    if (p.tile_end <= p.tile_begin || p.n_splits < 1) return PION_B200_ESHAPE;
    if (p.list_base + p.n_splits * fi8_lists_per_split(p.k) > p.n_lists) return PION_B200_ESHAPE;
    const int n_qt = (L.nq + fi8::BM - 1) / fi8::BM;
    const int ew = fi8_epi_warps(L.k);
    // k = 10 (the FT.SEARCH default): a list of exactly ten entries, whose k-th is its last
    // one, instead of 16 with a select tree (PION_B200_I8_KCAP16=1 keeps 16, for tests)
    if (L.k == 10 && !getenv("PION_B200_I8_KCAP16"))
        return launch_tc_k<10, 8>(*L.tmap_q, *L.tmap_rows, p, n_qt, st);
    switch (fi8_kcap(L.k)) {
        case 16: return ew == 8 ? launch_tc_k<16, 8>(*L.tmap_q, *L.tmap_rows, p, n_qt, st)
                                : PION_B200_ESHAPE;
        case 32: return launch_tc_k<32, 4>(*L.tmap_q, *L.tmap_rows, p, n_qt, st);
        case 64: return launch_tc_k<64, 4>(*L.tmap_q, *L.tmap_rows, p, n_qt, st);
        default: return PION_B200_ESHAPE;
    }
}

int fi8_query_tile() { return fi8::BM; }
int fi8_k_block() { return fi8::BK; }

// One wave at k <= 32: two 256-thread CTAs per SM (two waves measured 278 us per search at
// 1M rows against 261 us for one).
int fi8_scan1_ctas(int64_t n_rows, int num_sms) {
    int64_t ctas = (int64_t)num_sms * 2;
    const int64_t min_rows = 256;
    if (ctas * min_rows > n_rows) ctas = (n_rows + min_rows - 1) / min_rows;
    return (int)(ctas < 1 ? 1 : ctas);
}

int launch_flat_i8_scan1(const int8_t* rows, const float* row_scale, int64_t n_rows, int dim,
                         const int8_t* q, const float* q_scale, int k, int ctas, float* cand_val,
                         int32_t* cand_idx, cudaStream_t st) {
    if (dim % 16 != 0 || dim / 16 > fi8::SCAN_MAX_CHUNKS) return PION_B200_ESHAPE;
    const int64_t rows_per_cta = (n_rows + ctas - 1) / ctas;
    switch (fi8_kcap(k)) {
        case 16:
            fi8::flat_i8_scan1_kernel<16><<<ctas, fi8::SCAN_THREADS, 0, st>>>(
                rows, row_scale, n_rows, dim, q, q_scale, k, rows_per_cta, cand_val, cand_idx);
            break;
        case 32:
            fi8::flat_i8_scan1_kernel<32><<<ctas, fi8::SCAN_THREADS, 0, st>>>(
                rows, row_scale, n_rows, dim, q, q_scale, k, rows_per_cta, cand_val, cand_idx);
            break;
        case 64:
            fi8::flat_i8_scan1_kernel<64><<<ctas, fi8::SCAN_THREADS, 0, st>>>(
                rows, row_scale, n_rows, dim, q, q_scale, k, rows_per_cta, cand_val, cand_idx);
            break;
        default:
            return PION_B200_ESHAPE;
    }
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

}  // namespace pion
