// GPU brute-force scan of the HNSW slot buffer on B200 (sm_100a): the engine's INT8
// "GPU vector engine" path (search_gpu_brute_force, src/vector/hnsw.mojo:3916-3992).
//
//   int8_l2_distance_batch / int8_l2_batch_multiquery (src/ffi/metal_compute.metal:19-143):
//       d = query_norm + cand_norm - 2 * float(dot_i32), cand_norm = the slot header's
//       f32 |code|^2;
//   pion_metal_search_topk_w (src/ffi/metal_wrap.m:495-580): k entries of (+inf, -1),
//       worst = +inf at entry 0; every slot in order: d < worst overwrites entry
//       worst_idx, then worst / worst_idx = the first maximum of the entries.
//
// Which entries survive, and where, depends on the order of the scan, so the loop is
// replayed exactly.  A slot can only be admitted if its distance is below the k-th
// smallest distance of the slots before it, which is at most the loop's worst after any
// earlier prefix; the loop needs only a superset of the admitted slots, in slot order:
//   slot_tc_kernel      tcgen05 INT8 dot products of 128 queries x 256 slots per tile;
//                       per (query, split, tile half) the slots with d below the query's
//                       current worst (and, for k <= 64, below the list's own k-th
//                       candidate), in slot order (no distance matrix);
//   slot_replay_kernel  warp per query: the worst-replace loop over those lists, split
//                       by split (the two halves merged), continuing from the previous
//                       stage's state;
//   queries whose lists overflowed: the same tensor-core kernel writes all their
//                       distances, chunk by chunk, and slot_dense_replay_kernel runs the
//                       loop over every slot.
// The host splits the slots into stages; the worst carried into a stage bounds it.
#include <climits>
#include <cstdint>
#include <cstdio>

#include "common.cuh"
#include "internal.h"

namespace pion {
namespace slot {

constexpr int DIM = 1536;
constexpr int BM = 128, BN = 256, BK = 128, STAGES = 4, UMMA_K = 32;
constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_WARPS = 8;  // two per TMEM lane quadrant, each on half of a tile
constexpr int HALF = BN / 2;
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr uint32_t TMEM_COLS = 2 * BN;
constexpr uint32_t IDESC = make_idesc_i8(BM, BN);
constexpr size_t SMEM_PIPE_BYTES = 1024 + (size_t)STAGES * STAGE_BYTES + 256;
// per epilogue warp: a chunk's 32 x 32 dots and its 32 norms
constexpr size_t STASH_BYTES = 32 * 33 * 4;
constexpr size_t SMEM_BYTES = SMEM_PIPE_BYTES + EPI_WARPS * STASH_BYTES;
constexpr int KPL = 8;          // loop entries per lane
constexpr int KMAX = 32 * KPL;  // largest k

// The shader's distance: (query_norm + cand_norm) - 2 * float(dot), rounded per step.
__device__ __forceinline__ float l2_dist(float qn, float vn, int32_t dot) {
    return __fsub_rn(__fadd_rn(qn, vn), __fmul_rn(2.0f, __int2float_rn(dot)));
}

struct TcParams {
    int k;               // loop entries
    const float* bound;  // per query: collect slots with d < bound (the loop's worst)
    const float* qnorm;  // per query |q|^2
    const float* vnorm;  // per slot |v|^2
    int64_t n_rows;      // slots scanned
    int nq;
    int tile_begin, tile_end, n_splits, kblocks, cap;
    float* cand_d;       // [nq][n_splits][2][cap]: per split, the two tile halves
    int32_t* cand_i;
    int* cand_n;         // [nq][n_splits][2]; above cap: the list overflowed
    int* status;
    // dense mode: every distance of slots [dense_base, dense_base + dense_ld) for the
    // first *n_dense queries, row-major [query][slot - dense_base]
    float* dense;
    int64_t dense_base, dense_ld;
    const int* n_dense;
    // per 32-slot chunk (padded to whole tiles): min over the chunk of floor(vn), or
    // -2^30 where a norm is beyond 2^26
    const int* chunk_vmin;
    // [nq][n_splits][2]: each list's current threshold, published after every tile
    // (k <= 64).  Every slot of split s comes before every slot of split s + 1, so a
    // list of split s + 1 may use split s's values, which already fold in those of
    // split s - 1: the chain carries the tightest earlier threshold forward.
    float* pub;
};

// Max of bv[0, N) into bv[0] / bp[0] by halving (any N): entry i meets entry i + ceil(N/2),
// the later one winning only when strictly larger.  Unrolled at compile time, so the
// arrays stay in registers.
template <int N>
struct MaxTree {
    __device__ __forceinline__ static void run(float* bv, int* bp) {
        constexpr int H = (N + 1) / 2;
#pragma unroll
        for (int i = 0; i < N - H; ++i) {
            const bool up = bv[i + H] > bv[i];
            bv[i] = up ? bv[i + H] : bv[i];
            bp[i] = up ? bp[i + H] : bp[i];
        }
        MaxTree<H>::run(bv, bp);
    }
};
template <>
struct MaxTree<1> {
    __device__ __forceinline__ static void run(float*, int*) {}
};

// The k smallest candidates of a list so far, unsorted in registers (entries past k hold
// -inf and never count), and where the largest sits.  insert() overwrites the largest
// with d and returns the new largest, i.e. the k-th smallest candidate: independent
// selects and a depth-ceil(log2 KCAP) max tree (KCAP need not be a power of two: the
// 20-entry lists of the brute-force search's top-20 cost 19 comparisons, not 31).  selp
// keeps the runtime position from being folded back into an indexed access (which would
// move the array to local memory).
template <int KCAP>
struct LocalTopK {
    float v[KCAP];
    int mpos;
    __device__ __forceinline__ void init(int k) {
#pragma unroll
        for (int m = 0; m < KCAP; ++m) v[m] = m < k ? INFINITY : -INFINITY;
        mpos = 0;
    }
    __device__ __forceinline__ float insert(float d) {
#pragma unroll
        for (int m = 0; m < KCAP; ++m)
            v[m] = __uint_as_float(selp_u32(__float_as_uint(d), __float_as_uint(v[m]), m == mpos));
        float bv[KCAP];
        int bp[KCAP];
#pragma unroll
        for (int m = 0; m < KCAP; ++m) {
            bv[m] = v[m];
            bp[m] = m;
        }
        MaxTree<KCAP>::run(bv, bp);
        mpos = bp[0];
        return bv[0];
    }
};

// KCAP > 0 (k <= KCAP): a lane also drops slots that are not below the k-th smallest
// candidate of its own list so far.  Those slots come earlier in the scan, so the loop's
// worst at a slot is at most that k-th distance and such a slot cannot enter the loop;
// near neighbours that sit together in slot order (the BFS slot layout keeps graph
// neighbourhoods together) then cost about k (1 + ln(run / k)) candidates instead of the
// whole run.
//
// DENSE: the exact path for queries whose lists overflowed; the epilogue writes every
// distance (transposed through shared memory so that each store is one 128-byte row
// segment) and collects nothing.
template <int KCAP, bool DENSE>
__global__ void __launch_bounds__(THREADS, 1)
    slot_tc_kernel(const __grid_constant__ CUtensorMap tmap_q,
                   const __grid_constant__ CUtensorMap tmap_rows, TcParams p) {
    // whole CTA, before any barrier
    if (DENSE && (int)blockIdx.x * BM >= (p.n_dense ? *p.n_dense : p.nq)) return;
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
        // epilogue: lane = query (TMEM lane); warp half h takes slots [128 h, 128 h + 128)
        // of every tile, in order, into its own list
        const int ew = warp - 2;
        const int lg = warp & 3;
        const int half = ew >> 2;
        uint32_t* stash = stash_all + ew * (STASH_BYTES / 4);
        float* stash_v = reinterpret_cast<float*>(stash + 32 * 32);
        const int q = qt * BM + lg * 32 + lane;
        const bool q_ok = q < p.nq;
        const float bound = q_ok && !DENSE ? p.bound[q] : -INFINITY;
        const float qn = q_ok ? p.qnorm[q] : 0.0f;
        const size_t list = ((size_t)(q_ok ? q : 0) * p.n_splits + split) * 2 + half;
        float* out_d = p.cand_d + list * p.cap;
        int32_t* out_i = p.cand_i + list * p.cap;
        int count = 0;
        constexpr int KT = KCAP > 0 ? KCAP : 1;
        LocalTopK<KT> top;
        top.init(KCAP > 0 ? p.k : 0);
        float thr = bound;  // min(bound, this list's k-th candidate)
        // Integer pre-test of d < thr: 2 dot - floor(vn) > floor(qn - thr) - 64.  The
        // float rounding of d stays below 64 at these magnitudes (|qn|, |vn| < 2^26), so
        // the test passes every slot that can pass the exact one.
        auto int_floor = [&](float t) {
            if (!(t > -INFINITY)) return INT_MAX;  // nothing can pass
            const float x = qn - t;
            return t < INFINITY && fabsf(x) < 67108864.0f && fabsf(qn) < 67108864.0f
                       ? (int)floorf(x) - 64
                       : INT_MIN;
        };
        int ithr = int_floor(thr);
        // this half's slot norms for the next tile load while the current one is scored
        constexpr int HC = HALF / 32;
        float vnext[HC];
        int mnext[HC];  // per 32-slot chunk: the smallest floor(vn) (coarse pre-test)
        auto load_norms = [&](int tile) {
#pragma unroll
            for (int c = 0; c < HC; ++c) {
                const int64_t col = (int64_t)tile * BN + half * HALF + c * 32 + lane;
                vnext[c] = col < p.n_rows ? p.vnorm[col] : 0.0f;
                mnext[c] = p.chunk_vmin[((int64_t)tile * BN + half * HALF) / 32 + c];
            }
        };
        if (my_tiles > 0) load_norms(t_begin);
        // the previous split's published thresholds (read one tile ahead of their use)
        const bool chain = KCAP > 0 && !DENSE && p.pub != nullptr && q_ok;
        float* my_pub = chain ? p.pub + ((size_t)q * p.n_splits + split) * 2 + half : nullptr;
        const float* prev_pub =
            chain && split > 0 ? p.pub + ((size_t)q * p.n_splits + split - 1) * 2 : nullptr;
        float ext = INFINITY;
        if (prev_pub) ext = fminf(__ldcg(prev_pub), __ldcg(prev_pub + 1));
        for (int t = 0; t < my_tiles; ++t) {
            const int buf = t & 1;
            const uint32_t use = (uint32_t)(t >> 1);
            const int64_t col0 = (int64_t)(t_begin + t) * BN + half * HALF;
            if (ext < thr) {
                thr = ext;
                ithr = int_floor(thr);
            }
            if (prev_pub) ext = fminf(__ldcg(prev_pub), __ldcg(prev_pub + 1));
            float vcur[HC];
            int vicur[HC], mcur[HC];
#pragma unroll
            for (int c = 0; c < HC; ++c) {
                vcur[c] = vnext[c];
                mcur[c] = mnext[c];
                // floor(vn) as an int; a norm beyond 2^26 passes every pre-test
                vicur[c] = fabsf(vcur[c]) < 67108864.0f ? (int)floorf(vcur[c]) : -(1 << 30);
            }
            if (t + 1 < my_tiles) load_norms(t_begin + t + 1);
            const bool got = mbar_wait(&tfull[buf], use & 1u, p.status, abort_flag);
            if (!__all_sync(0xffffffffu, got)) break;
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(lg * 32) << 16) +
                                   (uint32_t)(buf * BN + half * HALF);
            // one 32-slot chunk: dense rows, or the candidates below the threshold
            auto chunk = [&](const uint32_t(&r)[32], int c) {
                const int64_t c0 = col0 + c * 32;
                const float vl = vcur[c];
                if constexpr (DENSE) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const float v = __shfl_sync(0xffffffffu, vl, j);
                        stash[j * 32 + lane] = __float_as_uint(l2_dist(qn, v, (int32_t)r[j]));
                    }
                    __syncwarp();
                    const int64_t col = c0 + lane;  // this lane's slot, for 32 queries
                    const int nd = p.n_dense ? *p.n_dense : p.nq;
                    if (col < p.n_rows) {
                        for (int qq = 0; qq < 32; ++qq) {
                            const int f = qt * BM + lg * 32 + qq;
                            if (f < nd)
                                p.dense[(size_t)f * p.dense_ld + (col - p.dense_base)] =
                                    __uint_as_float(stash[lane * 32 + qq]);
                        }
                    }
                    __syncwarp();
                    return;
                }
                // coarse pre-test with the chunk's smallest norm: 2 max(dot) - min(floor vn)
                // > ithr is necessary for any column to pass; usually no lane passes
                int32_t mx = (int32_t)r[0];
#pragma unroll
                for (int j = 1; j < 32; ++j) mx = max(mx, (int32_t)r[j]);
                const bool coarse = 2 * (int64_t)mx - mcur[c] > (int64_t)ithr;
                if (!__any_sync(0xffffffffu, coarse)) return;
                // the chunk's 32 floor norms (lane j holds column j's) for every lane
                int* vrow = reinterpret_cast<int*>(stash_v);
                vrow[lane] = vicur[c];
                __syncwarp();
                if (!coarse) return;
                // From here on each lane works alone: no warp synchronisation.
                uint32_t mask;
                if (ithr == INT_MIN) {
                    mask = 0xffffffffu;
                } else {
                    // bit j = (2 dot_j - v_j > ithr) = sign of ithr - (2 dot_j - v_j), two
                    // funnel-shift chains (|2 dot - v| < 2^31 - 2^27, |ithr| < 2^27)
                    uint32_t lo = 0, hi = 0;
                    const int4* v4 = reinterpret_cast<const int4*>(vrow);
#pragma unroll
                    for (int i = 3; i >= 0; --i) {
                        const int4 a = v4[i], b = v4[i + 4];
                        const int va[4] = {a.x, a.y, a.z, a.w}, vb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
                        for (int e = 3; e >= 0; --e) {
                            const int j = 4 * i + e;
                            lo = __funnelshift_l(
                                (uint32_t)(ithr - (2 * (int32_t)r[j] - va[e])), lo, 1);
                            hi = __funnelshift_l(
                                (uint32_t)(ithr - (2 * (int32_t)r[j + 16] - vb[e])), hi, 1);
                        }
                    }
                    mask = lo | (hi << 16);
                }
                const int64_t vc = p.n_rows - c0;
                if (vc < 32) mask &= vc <= 0 ? 0u : ((1u << vc) - 1u);
                if (!mask) return;
                // this lane's 32 dots into its own stash row (16-byte slots XOR-swizzled by
                // lane), read back by index
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
                    const float d = l2_dist(qn, __ldg(&p.vnorm[c0 + j]),
                                            (int32_t)row[(((j >> 2) ^ sw) << 2) | (j & 3)]);
                    if (!(d < thr)) continue;  // the threshold moved within this chunk
                    if (count < p.cap) {
                        out_d[count] = d;
                        out_i[count] = (int32_t)(c0 + j);
                    }
                    ++count;
                    if constexpr (KCAP > 0) {
                        thr = fminf(thr, top.insert(d));
                        ithr = int_floor(thr);
                    }
                }
            };
            if constexpr (KCAP <= 32) {
                // chunks in pairs: the next chunk's TMEM load is in flight while the
                // current one is scanned
                uint32_t ra[32], rb[32];
                tmem_ld32(taddr, ra);
                tmem_ld_wait_regs(ra);
#pragma unroll
                for (int c = 0; c < HC; c += 2) {
                    __syncwarp();
                    tmem_ld32(taddr + (uint32_t)((c + 1) * 32), rb);
                    chunk(ra, c);
                    __syncwarp();
                    tmem_ld_wait_regs(rb);
                    if (c + 2 < HC) tmem_ld32(taddr + (uint32_t)((c + 2) * 32), ra);
                    chunk(rb, c + 1);
                    __syncwarp();
                    if (c + 2 < HC) tmem_ld_wait_regs(ra);
                }
            } else {
                // a 64-entry list leaves no registers for a second chunk buffer
#pragma unroll
                for (int c = 0; c < HC; ++c) {
                    uint32_t ra[32];
                    __syncwarp();
                    tmem_ld32(taddr + (uint32_t)(c * 32), ra);
                    tmem_ld_wait_regs(ra);
                    chunk(ra, c);
                }
            }
            tc_fence_before();
            mbar_arrive(&tempty[buf]);
            if (my_pub) __stcg(my_pub, thr);
        }
        if (!DENSE && q_ok) p.cand_n[list] = count;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ------------------------------------------------------- the worst-replace loop --
// The k entries live in a warp: entry p at lane p % 32, register p / 32.

// worst / worst_idx after an update: the first entry holding the maximum, over entries
// above -inf (the loop starts from worst = -inf and takes strictly larger values); if
// there is none the loop leaves worst = -inf and worst_idx unchanged.
__device__ __forceinline__ void first_max(const float (&sd)[KPL], int k, int lane, float& worst,
                                          int& widx) {
    float v = -INFINITY;
    int pos = -1;
#pragma unroll
    for (int m = 0; m < KPL; ++m) {
        const int pp = m * 32 + lane;
        if (pp < k && sd[m] > v) {
            v = sd[m];
            pos = pp;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int op = __shfl_xor_sync(0xffffffffu, pos, o);
        if (op >= 0 && (pos < 0 || ov > v || (ov == v && op < pos))) {
            v = ov;
            pos = op;
        }
    }
    worst = v;
    if (pos >= 0) widx = pos;
}

// One candidate through the loop (warp-uniform d, id).
__device__ __forceinline__ void admit(float d, int32_t id, float (&sd)[KPL], int32_t (&si)[KPL],
                                      int k, int lane, float& worst, int& widx) {
    if (!(d < worst)) return;
    const int hit = lane == (widx & 31) ? (widx >> 5) : -1;
#pragma unroll
    for (int m = 0; m < KPL; ++m) {
        sd[m] = m == hit ? d : sd[m];
        si[m] = m == hit ? id : si[m];
    }
    first_max(sd, k, lane, worst, widx);
}

// 32 candidates (one per lane, in order) through the loop.
__device__ __forceinline__ void admit32(bool valid, float dj, int32_t ij, float (&sd)[KPL],
                                        int32_t (&si)[KPL], int k, int lane, float& worst,
                                        int& widx) {
    uint32_t mask = __ballot_sync(0xffffffffu, valid && dj < worst);
    while (mask) {
        const int s = __ffs(mask) - 1;
        mask &= mask - 1u;
        const float d = __shfl_sync(0xffffffffu, dj, s);
        const int32_t id = __shfl_sync(0xffffffffu, ij, s);
        admit(d, id, sd, si, k, lane, worst, widx);
    }
}

__device__ __forceinline__ void load_state(const float* st_d, const int32_t* st_i, int q, int k,
                                           int lane, float (&sd)[KPL], int32_t (&si)[KPL]) {
#pragma unroll
    for (int m = 0; m < KPL; ++m) {
        const int pp = m * 32 + lane;
        sd[m] = pp < k ? st_d[(size_t)q * k + pp] : -INFINITY;
        si[m] = pp < k ? st_i[(size_t)q * k + pp] : -1;
    }
}

__device__ __forceinline__ void store_state(float* st_d, int32_t* st_i, int q, int k, int lane,
                                            const float (&sd)[KPL], const int32_t (&si)[KPL]) {
#pragma unroll
    for (int m = 0; m < KPL; ++m) {
        const int pp = m * 32 + lane;
        if (pp < k) {
            st_d[(size_t)q * k + pp] = sd[m];
            st_i[(size_t)q * k + pp] = si[m];
        }
    }
}

// Warp per query: the loop's initial state, the query norm (given, or the integer
// |code|^2 as f32: norm_sq_int8_jit, src/vector/kernels.mojo:362-376) and, with
// force_exact, every query queued for the exact scan.
__global__ void __launch_bounds__(256)
    slot_prep_kernel(const int8_t* __restrict__ codes, const float* __restrict__ qnorm_in, int nq,
                     int k, float* __restrict__ qnorm, float* __restrict__ st_d,
                     int32_t* __restrict__ st_i, float* __restrict__ st_worst,
                     int* __restrict__ st_widx, int* __restrict__ qflag, int* __restrict__ flags,
                     int force_exact) {
    const int q = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (q >= nq) return;
    float qn;
    if (qnorm_in) {
        qn = qnorm_in[q];
    } else {
        const int4* c = reinterpret_cast<const int4*>(codes + (size_t)q * DIM);
        int s = 0;
#pragma unroll
        for (int u = 0; u < DIM / 16 / 32; ++u) {
            const int4 v = c[lane + 32 * u];
            s = __dp4a(v.x, v.x, s);
            s = __dp4a(v.y, v.y, s);
            s = __dp4a(v.z, v.z, s);
            s = __dp4a(v.w, v.w, s);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        qn = __int2float_rn(s);
    }
    for (int p = lane; p < k; p += 32) {
        st_d[(size_t)q * k + p] = INFINITY;
        st_i[(size_t)q * k + p] = -1;
    }
    if (lane == 0) {
        qnorm[q] = qn;
        st_widx[q] = 0;
        qflag[q] = force_exact;
        st_worst[q] = force_exact ? -INFINITY : INFINITY;
        if (force_exact) flags[1 + q] = q;
        if (force_exact && q == 0) flags[0] = nq;
    }
}

// Warp per query: the stage's lists through the loop in slot order.  A split has two
// lists (the two halves of every tile), each in slot order; they are merged 32 at a
// time: the 32 smallest slots of the next 32 of each list are the next 32 of the merge.
// A list that overflowed sends the query to the exact path; later stages then collect
// nothing for it (its bound becomes -inf).
__global__ void __launch_bounds__(256, 2)
    slot_replay_kernel(const float* __restrict__ cand_d, const int32_t* __restrict__ cand_i,
                       const int* __restrict__ cand_n, int n_splits, int cap, int nq, int k,
                       float* __restrict__ st_d, int32_t* __restrict__ st_i,
                       float* __restrict__ st_worst, int* __restrict__ st_widx,
                       int* __restrict__ qflag, int* __restrict__ flags,
                       unsigned long long* __restrict__ counters) {
    __shared__ float mrg_d[8][32];
    __shared__ int32_t mrg_i[8][32];
    const int wib = threadIdx.x >> 5;
    const int q = blockIdx.x * 8 + wib;
    const int lane = threadIdx.x & 31;
    if (q >= nq || qflag[q]) return;  // warp-uniform
    // overflow anywhere: the exact path takes the query
    bool over = false;
    for (int l = lane; l < 2 * n_splits; l += 32) over |= cand_n[(size_t)q * 2 * n_splits + l] > cap;
    if (__any_sync(0xffffffffu, over)) {
        if (lane == 0) {
            qflag[q] = 1;
            st_worst[q] = -INFINITY;
            flags[1 + atomicAdd(flags, 1)] = q;
        }
        return;
    }
    int replayed = 0;
    float sd[KPL];
    int32_t si[KPL];
    load_state(st_d, st_i, q, k, lane, sd, si);
    float worst = st_worst[q];
    int widx = st_widx[q];
    for (int sp = 0; sp < n_splits; ++sp) {
        const size_t l0 = ((size_t)q * n_splits + sp) * 2;
        const int n0 = cand_n[l0], n1 = cand_n[l0 + 1];
        const float* d0 = cand_d + l0 * cap;
        const float* d1 = d0 + cap;
        const int32_t* i0 = cand_i + l0 * cap;
        const int32_t* i1 = i0 + cap;
        replayed += n0 + n1;
        int p0 = 0, p1 = 0;
        while (p0 < n0 || p1 < n1) {
            const bool v0 = p0 + lane < n0, v1 = p1 + lane < n1;
            const int32_t a0 = v0 ? i0[p0 + lane] : INT_MAX;
            const int32_t a1 = v1 ? i1[p1 + lane] : INT_MAX;
            const float e0 = v0 ? d0[p0 + lane] : INFINITY;
            const float e1 = v1 ? d1[p1 + lane] : INFINITY;
            int r0 = lane, r1 = lane;  // ranks in the merge of the two windows
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                r0 += __shfl_sync(0xffffffffu, a1, j) < a0 ? 1 : 0;
                r1 += __shfl_sync(0xffffffffu, a0, j) < a1 ? 1 : 0;
            }
            const bool t0 = v0 && r0 < 32, t1 = v1 && r1 < 32;
            if (t0) {
                mrg_d[wib][r0] = e0;
                mrg_i[wib][r0] = a0;
            }
            if (t1) {
                mrg_d[wib][r1] = e1;
                mrg_i[wib][r1] = a1;
            }
            const int c0 = __popc(__ballot_sync(0xffffffffu, t0));
            const int c1 = __popc(__ballot_sync(0xffffffffu, t1));
            __syncwarp();
            const int m = c0 + c1;
            admit32(lane < m, lane < m ? mrg_d[wib][lane] : INFINITY,
                    lane < m ? mrg_i[wib][lane] : -1, sd, si, k, lane, worst, widx);
            __syncwarp();
            p0 += c0;
            p1 += c1;
        }
    }
    store_state(st_d, st_i, q, k, lane, sd, si);
    if (lane == 0) {
        st_worst[q] = worst;
        st_widx[q] = widx;
        if (replayed) atomicAdd(&counters[1], (unsigned long long)replayed);
    }
}

// The exact path, step 1: the queued queries' codes and norms, packed (dense index f
// = the f-th queued query), and their loop state reset.
__global__ void slot_gather_kernel(const int8_t* __restrict__ qcodes,
                                   const float* __restrict__ qnorm, const int* __restrict__ flags,
                                   int first, int count, int k, int8_t* __restrict__ fcodes,
                                   float* __restrict__ fqn, int* __restrict__ n_dense,
                                   float* __restrict__ fd, int32_t* __restrict__ fi,
                                   float* __restrict__ fworst, int* __restrict__ fwidx) {
    const int nf = min(max(flags[0] - first, 0), count);
    if (blockIdx.x == 0 && threadIdx.x == 0) *n_dense = nf;
    for (int f = blockIdx.x; f < nf; f += gridDim.x) {
        const int q = flags[1 + first + f];
        const int4* src = reinterpret_cast<const int4*>(qcodes + (size_t)q * DIM);
        int4* dst = reinterpret_cast<int4*>(fcodes + (size_t)f * DIM);
        for (int i = threadIdx.x; i < DIM / 16; i += blockDim.x) dst[i] = src[i];
        for (int i = threadIdx.x; i < k; i += blockDim.x) {
            fd[(size_t)f * k + i] = INFINITY;
            fi[(size_t)f * k + i] = -1;
        }
        if (threadIdx.x == 0) {
            fqn[f] = qnorm[q];
            fworst[f] = INFINITY;
            fwidx[f] = 0;
        }
    }
}

// Dense distances through the loop, warp per query, in slot order, one chunk per launch.
// Queued mode (flags): query f of the queue; its state lives in fd.. until the last
// chunk, then goes back to the query's entries.  Prefix mode (flags null): query f
// itself, state in fd.. = the queries' entries; queries already queued are skipped.
__global__ void __launch_bounds__(256, 2)
    slot_dense_replay_kernel(const float* __restrict__ dense, int64_t ld, int64_t base,
                             int64_t len, const int* __restrict__ n_dense, int count, int k,
                             float* __restrict__ fd, int32_t* __restrict__ fi,
                             float* __restrict__ fworst, int* __restrict__ fwidx, int last,
                             const int* __restrict__ flags, int first, float* __restrict__ st_d,
                             int32_t* __restrict__ st_i, float* __restrict__ st_worst,
                             int* __restrict__ st_widx, const int* __restrict__ qflag) {
    const int f = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (f >= (n_dense ? *n_dense : count)) return;  // warp-uniform
    if (!flags && qflag && qflag[f]) return;
    float sd[KPL];
    int32_t si[KPL];
    load_state(fd, fi, f, k, lane, sd, si);
    float worst = fworst[f];
    int widx = fwidx[f];
    const float* row = dense + (size_t)f * ld;
    // 512 distances per round, loaded a round ahead (16 loads in flight per lane): the
    // loop itself is short, so the row's load latency would otherwise bound it
    constexpr int U = 16;
    float nx[U];
#pragma unroll
    for (int u = 0; u < U; ++u) nx[u] = u * 32 + lane < len ? row[u * 32 + lane] : INFINITY;
    for (int64_t b = 0; b < len; b += U * 32) {
        float cur[U];
#pragma unroll
        for (int u = 0; u < U; ++u) cur[u] = nx[u];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t j = b + U * 32 + u * 32 + lane;
            nx[u] = j < len ? __ldcs(row + j) : INFINITY;
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t j = b + u * 32 + lane;
            admit32(j < len, cur[u], (int32_t)(base + j), sd, si, k, lane, worst, widx);
        }
    }
    if (last && flags) {
        const int q = flags[1 + first + f];
        store_state(st_d, st_i, q, k, lane, sd, si);
        if (lane == 0) {
            st_worst[q] = worst;
            st_widx[q] = widx;
        }
    } else {
        store_state(fd, fi, f, k, lane, sd, si);
        if (lane == 0) {
            fworst[f] = worst;
            fwidx[f] = widx;
        }
    }
}

// Per 32-slot chunk, padded to whole tiles: the smallest floor(vn) of its slots (slots
// past n count as 0; a norm beyond 2^26 counts as -2^30), for the coarse pre-test.
__global__ void slot_chunk_vmin_kernel(const float* __restrict__ vnorm, int64_t n,
                                       int64_t n_chunks, int* __restrict__ out) {
    const int64_t c = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (c >= n_chunks) return;
    const int64_t s = c * 32 + lane;
    const float v = s < n ? vnorm[s] : 0.0f;
    int m = fabsf(v) < 67108864.0f ? (int)floorf(v) : -(1 << 30);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = min(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) out[c] = m;
}

// The loop's entries as pion_metal_search_topk_w leaves them: [nq x k_out], entries past
// k as (-1, +inf).
__global__ void slot_emit_kernel(const float* __restrict__ st_d, const int32_t* __restrict__ st_i,
                                 int nq, int k, int k_out, int32_t* __restrict__ out_slots,
                                 float* __restrict__ out_d) {
    const int64_t total = (int64_t)nq * k_out;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t q = i / k_out, p = i % k_out;
        out_slots[i] = p < k ? st_i[q * k + p] : -1;
        out_d[i] = p < k ? st_d[q * k + p] : INFINITY;
    }
}

// search_gpu_brute_force's tail (src/vector/hnsw.mojo:3951-3992), a CTA per query: with
// rerank rows every entry's distance becomes the FP32 L2^2 of the raw query and the
// slot's row in the CPU loop's order (8 SIMD lanes, lane l over elements 8i + l,
// acc = acc + diff * diff, then the halving reduce_add); the stable insertion sort by
// distance (rank = #smaller + #equal before it); the first final_k as (external id,
// distance).
__global__ void __launch_bounds__(256)
    slot_finish_kernel(const float* __restrict__ st_d, const int32_t* __restrict__ st_i, int k,
                       const float* __restrict__ q_raw, const float* __restrict__ rerank,
                       const int32_t* __restrict__ slot_ext, int64_t n, int final_k, int k_out,
                       int32_t* __restrict__ out_ids, float* __restrict__ out_scores,
                       int32_t* __restrict__ out_found) {
    __shared__ float sdist[KMAX];
    __shared__ int32_t sslot[KMAX];
    __shared__ float qs[DIM];
    const int q = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int p = threadIdx.x; p < k; p += blockDim.x) {
        sdist[p] = st_d[(size_t)q * k + p];
        sslot[p] = st_i[(size_t)q * k + p];
    }
    if (rerank)
        for (int i = threadIdx.x; i < DIM; i += blockDim.x) qs[i] = q_raw[(size_t)q * DIM + i];
    __syncthreads();
    if (rerank) {
        const int l = lane & 7;
        for (int base = warp * 4; base < k; base += 32) {
            const int cand = base + (lane >> 3);
            const int32_t s = cand < k ? sslot[cand] : -1;
            const bool ok = s >= 0 && s < n;
            float acc = 0.0f;
            if (ok) {
                const float* v = rerank + (size_t)s * DIM;
#pragma unroll 8
                for (int i = 0; i < DIM / 8; ++i) {
                    const float diff = __fsub_rn(qs[8 * i + l], v[8 * i + l]);
                    acc = __fadd_rn(acc, __fmul_rn(diff, diff));
                }
            }
#pragma unroll
            for (int h = 4; h > 0; h >>= 1)
                acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, acc, (lane & ~7) | ((l + h) & 7)));
            if (ok && l == 0) sdist[cand] = acc;
        }
        __syncthreads();
    }
    const int found = k < final_k ? k : final_k;
    for (int p = threadIdx.x; p < k; p += blockDim.x) {
        const float d = sdist[p];
        int rank = 0;
        for (int j = 0; j < k; ++j) {
            const float dj = sdist[j];
            rank += (dj < d || (dj == d && j < p)) ? 1 : 0;
        }
        if (rank < found) {
            const int32_t s = sslot[p];
            out_ids[(size_t)q * k_out + rank] = s >= 0 && s < n ? slot_ext[s] : -1;
            out_scores[(size_t)q * k_out + rank] = d;
        }
    }
    for (int p = found + threadIdx.x; p < k_out; p += blockDim.x) {
        out_ids[(size_t)q * k_out + p] = -1;
        out_scores[(size_t)q * k_out + p] = INFINITY;
    }
    if (threadIdx.x == 0) out_found[q] = found;
}

}  // namespace slot

int slot_tile_rows() { return slot::BN; }
int slot_query_tile() { return slot::BM; }
int slot_k_block() { return slot::BK; }
int slot_kmax() { return slot::KMAX; }

int launch_slot_prep(const int8_t* codes, const float* qnorm_in, int nq, int k, float* qnorm,
                     float* st_d, int32_t* st_i, float* st_worst, int* st_widx, int* qflag,
                     int* flags, int force_exact, cudaStream_t st) {
    if (nq <= 0) return 0;
    if (cudaMemsetAsync(flags, 0, 4, st) != cudaSuccess) return PION_B200_ECUDA;
    slot::slot_prep_kernel<<<(nq + 7) / 8, 256, 0, st>>>(codes, qnorm_in, nq, k, qnorm, st_d,
                                                          st_i, st_worst, st_widx, qflag, flags,
                                                          force_exact);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

template <int KCAP, bool DENSE>
static int slot_tc_go(dim3 grid, const SlotTcLaunch& L, const slot::TcParams& p,
                      cudaStream_t st) {
    if (set_smem_limit((const void*)slot::slot_tc_kernel<KCAP, DENSE>, (int)slot::SMEM_BYTES) != 0)
        return PION_B200_ECUDA;
    slot::slot_tc_kernel<KCAP, DENSE><<<grid, slot::THREADS, slot::SMEM_BYTES, st>>>(
        *L.tmap_q, *L.tmap_rows, p);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int launch_slot_tc(const SlotTcLaunch& L, cudaStream_t st) {
    slot::TcParams p;
    p.bound = L.bound;
    p.qnorm = L.qnorm;
    p.vnorm = L.vnorm;
    p.n_rows = L.n_rows;
    p.nq = L.nq;
    p.k = L.k;
    p.tile_begin = L.tile_begin;
    p.tile_end = L.tile_end;
    p.n_splits = L.n_splits;
    p.kblocks = slot::DIM / slot::BK;
    p.cap = L.cap;
    p.cand_d = L.cand_d;
    p.cand_i = L.cand_i;
    p.cand_n = L.cand_n;
    p.status = L.status;
    p.dense = L.dense;
    p.dense_base = L.dense_base;
    p.dense_ld = L.dense_ld;
    p.n_dense = L.n_dense;
    p.pub = L.pub;
    p.chunk_vmin = L.chunk_vmin;
    if (p.tile_end <= p.tile_begin || p.n_splits < 1 || p.n_splits > p.tile_end - p.tile_begin)
        return PION_B200_ESHAPE;
    if (p.k < 1 || p.k > slot::KMAX) return PION_B200_ESHAPE;
    dim3 grid((L.nq + slot::BM - 1) / slot::BM, L.n_splits);
    if (L.dense) {  // the chunk must hold every slot of the tile range
        if ((int64_t)L.tile_begin * slot::BN < L.dense_base ||
            (int64_t)L.tile_end * slot::BN > L.dense_base + L.dense_ld)
            return PION_B200_ESHAPE;
        return slot_tc_go<0, true>(grid, L, p, st);
    }
    if (p.cap < slot::HALF) return PION_B200_ESHAPE;
    if (p.k <= 16) return slot_tc_go<16, false>(grid, L, p, st);
    if (p.k <= 20) return slot_tc_go<20, false>(grid, L, p, st);
    if (p.k <= 32) return slot_tc_go<32, false>(grid, L, p, st);
    if (p.k <= 64) return slot_tc_go<64, false>(grid, L, p, st);
    return slot_tc_go<0, false>(grid, L, p, st);
}

int launch_slot_replay(const float* cand_d, const int32_t* cand_i, const int* cand_n, int n_lists,
                       int cap, int nq, int k, float* st_d, int32_t* st_i, float* st_worst,
                       int* st_widx, int* qflag, int* flags, unsigned long long* counters,
                       cudaStream_t st) {
    if (nq <= 0) return 0;
    if (k < 1 || k > slot::KMAX) return PION_B200_ESHAPE;
    slot::slot_replay_kernel<<<(nq + 7) / 8, 256, 0, st>>>(cand_d, cand_i, cand_n, n_lists, cap,
                                                            nq, k, st_d, st_i, st_worst, st_widx,
                                                            qflag, flags, counters);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int launch_slot_gather(const int8_t* qcodes, const float* qnorm, const int* flags, int first,
                       int count, int k, int8_t* fcodes, float* fqn, int* n_dense, float* fd,
                       int32_t* fi, float* fworst, int* fwidx, cudaStream_t st) {
    if (k < 1 || k > slot::KMAX) return PION_B200_ESHAPE;
    slot::slot_gather_kernel<<<count < 1024 ? count : 1024, 128, 0, st>>>(
        qcodes, qnorm, flags, first, count, k, fcodes, fqn, n_dense, fd, fi, fworst, fwidx);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int launch_slot_dense_replay(const float* dense, int64_t ld, int64_t base, int64_t len,
                             const int* n_dense, int count, int k, float* fd, int32_t* fi,
                             float* fworst, int* fwidx, int last, const int* flags, int first,
                             float* st_d, int32_t* st_i, float* st_worst, int* st_widx,
                             const int* qflag, cudaStream_t st) {
    if (k < 1 || k > slot::KMAX) return PION_B200_ESHAPE;
    if (count <= 0) return 0;
    slot::slot_dense_replay_kernel<<<(count + 7) / 8, 256, 0, st>>>(
        dense, ld, base, len, n_dense, count, k, fd, fi, fworst, fwidx, last, flags, first, st_d,
        st_i, st_worst, st_widx, qflag);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int launch_slot_chunk_vmin(const float* vnorm, int64_t n, int* out, cudaStream_t st) {
    const int64_t n_chunks = (n + slot::BN - 1) / slot::BN * (slot::BN / 32);
    if (n_chunks <= 0) return 0;
    slot::slot_chunk_vmin_kernel<<<(unsigned)((n_chunks + 7) / 8), 256, 0, st>>>(vnorm, n,
                                                                               n_chunks, out);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int launch_slot_emit(const float* st_d, const int32_t* st_i, int nq, int k, int k_out,
                     int32_t* out_slots, float* out_d, cudaStream_t st) {
    if (nq <= 0 || k_out <= 0) return 0;
    const int64_t total = (int64_t)nq * k_out;
    const int blocks = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
    slot::slot_emit_kernel<<<blocks, 256, 0, st>>>(st_d, st_i, nq, k, k_out, out_slots, out_d);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

int launch_slot_finish(const float* st_d, const int32_t* st_i, int nq, int k, const float* q_raw,
                       const float* rerank, const int32_t* slot_ext, int64_t n, int final_k,
                       int k_out, int32_t* out_ids, float* out_scores, int32_t* out_found,
                       cudaStream_t st) {
    if (nq <= 0) return 0;
    if (k < 1 || k > slot::KMAX) return PION_B200_ESHAPE;
    slot::slot_finish_kernel<<<nq, 256, 0, st>>>(st_d, st_i, k, q_raw, rerank, slot_ext, n,
                                                  final_k, k_out, out_ids, out_scores, out_found);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

}  // namespace pion
