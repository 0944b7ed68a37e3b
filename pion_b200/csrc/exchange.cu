// The shard exchange of a row-sharded FLAT search over NVLink peer memory: every rank's
// k (score, id) pairs per query go straight into every other rank's receive buffer with
// peer stores, a flag per (rank, step) says they are there, and each rank merges the
// world lists itself -- the all-gather and merge of src/commands/vector.mojo:4394-4436
// (concatenate each shard's results, keep the best k) without a collective library call.
//
// Buffers: one device allocation per rank, shared with the other processes through CUDA
// IPC handles: regions (one per exchange use within a step, e.g. the threshold bound and
// the final lists), each double-buffered by the step's parity, each [world][max_nq][k]
// 8-byte pairs, and a flag word per (region, parity, source rank).
//
// Ordering.  A rank may run at most one step ahead of any other: to publish step s + 2
// into parity (s & 1) it must have merged step s + 1, which needed every rank's step
// s + 1 flag, raised only after that rank had merged step s (read parity s & 1).  So a
// double buffer per region is enough.
//
// Publishing: every CTA stores its share of the pairs to every rank (itself included),
// fences at system scope and counts itself done; the last CTA raises this rank's flag on
// every rank with a system-scope release store.  In the sharded search the kernel that
// merges the shard's candidate lists publishes its result directly (merge_publish_kernel).
// Waiting: in each CTA of the merging kernel, lane r of warp 0 reads flag r with
// system-scope acquire loads until it holds the step's epoch, and the CTA's barrier
// releases the other warps; the wait is bounded (a %globaltimer budget), after which it
// records PION_B200_ETIMEOUT and returns, so a rank whose peer died gets an error instead
// of a hang.  An exchange is two kernels: publish (or merge + publish), wait + merge.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <new>

#include "common.cuh"
#include "internal.h"

struct pion_b200_exchange {
    int device = 0;
    int world = 0;
    int rank = 0;
    int regions = 0;
    int64_t max_nq = 0;
    int64_t k = 0;
    size_t region_bytes = 0;  // one parity of one region: world * max_nq * k * 8
    size_t flags_off = 0;     // flags after the pair regions
    char* base = nullptr;     // this rank's allocation
    char* peer[64] = {};      // every rank's allocation as mapped here (peer[rank] = base)
    unsigned* counter = nullptr;  // publish kernels' done-CTA counter (own memory)
    bool connected = false;
};

namespace pion {
namespace ex {

constexpr int PUB_THREADS = 256;

struct PeerPtrs {
    char* p[64];
};

// Stores `pairs` (nq x k, 8 bytes each) into slot `rank` of every rank's region, then the
// last CTA raises this rank's flag (value `epoch`) on every rank.
__global__ void __launch_bounds__(PUB_THREADS)
    publish_kernel(const uint2* __restrict__ pairs, int64_t count, PeerPtrs peers, int world,
                   int rank, size_t region_off, size_t slot_bytes, size_t flag_off,
                   unsigned epoch, unsigned* counter) {
    for (int r = 0; r < world; ++r) {
        uint2* dst = reinterpret_cast<uint2*>(peers.p[r] + region_off + (size_t)rank * slot_bytes);
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count;
             i += (int64_t)gridDim.x * blockDim.x)
            dst[i] = pairs[i];
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned done = atomicAdd(counter, 1u);
        if (done == gridDim.x - 1) {  // every CTA's stores are fenced: raise the flags
            *counter = 0;             // ready for the next publish (stream-ordered)
            __threadfence_system();
            for (int r = 0; r < world; ++r) {
                unsigned* f = reinterpret_cast<unsigned*>(peers.p[r] + flag_off) + rank;
                asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(epoch)
                             : "memory");
            }
        }
    }
}

// Warp-level k-way merge of n sorted lists of k entries each, by (score, id) (descending
// scores when DESC), padding ids (< 0) last.  The lists' heads sit in shared memory
// (hv/hi/cur, one slot per list); fetch(l, c, v, id) reads entry c of list l.  Each lane
// owns lists lane, lane + 32, ...; per output the warp reduces the lanes' best heads and
// the winning list's lane fetches its next entry.  emit(j, score, id) runs on lane 0.
template <bool DESC, typename Fetch, typename Emit>
__device__ __forceinline__ void warp_merge(int n_lists, int k, float* hv, int32_t* hi,
                                           uint16_t* cur, Fetch fetch, Emit emit) {
    const int lane = threadIdx.x & 31;
    const float pad = DESC ? -INFINITY : INFINITY;
    for (int l = lane; l < n_lists; l += 32) {
        fetch(l, 0, hv[l], hi[l]);
        cur[l] = 1;
    }
    __syncwarp();
    auto lane_best = [&](float& bv, int32_t& bi, int& bl) {
        bv = pad;
        bi = -1;
        bl = -1;
        for (int l = lane; l < n_lists; l += 32) {
            if (cur[l] > k) continue;  // exhausted
            const float v = hv[l];
            const int32_t id = hi[l];
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
            if ((ol >= 0) && (bl < 0 || merge_better<DESC>(ov, oi, bv, bi) ||
                              (ov == bv && oi == bi && ol < bl))) {
                bv = ov;
                bi = oi;
                bl = ol;
            }
        }
        if (lane == 0) emit(j, bl >= 0 ? bv : pad, (bl >= 0 && bi >= 0) ? bi : -1);
        if (j + 1 < k && bl >= 0 && (bl & 31) == lane) {
            const int c = cur[bl];
            if (c < k) fetch(bl, c, hv[bl], hi[bl]);
            cur[bl] = (uint16_t)(c + 1);
            lane_best(mv, mi, ml);
        }
    }
}

constexpr int MP_WARPS = 4;
constexpr int MP_MAX_LISTS = 512;
constexpr int MP_KMAX = 64;
constexpr int MP_STAGE = 768;  // entries per warp staged in shared memory by merge_publish
constexpr int WM_STAGE = 512;  // pairs per warp staged in shared memory by wait_merge

// This shard's lists [nq][n_lists][k] merged to its k per query, ids + id_offset, stored
// as pairs into slot `rank` of every rank's region (peer stores); then the last CTA raises
// this rank's flag on every rank.
template <bool DESC>
__global__ void __launch_bounds__(MP_WARPS * 32)
    merge_publish_kernel(const float* __restrict__ cv, const int32_t* __restrict__ ci, int nq,
                         int n_lists, int k, int64_t id_offset, PeerPtrs peers, int world,
                         int rank, size_t region_off, size_t slot_bytes, size_t flag_off,
                         unsigned epoch, unsigned* counter) {
    __shared__ float hv[MP_WARPS][MP_MAX_LISTS];
    __shared__ int32_t hi[MP_WARPS][MP_MAX_LISTS];
    __shared__ uint16_t cur[MP_WARPS][MP_MAX_LISTS];
    __shared__ uint2 outp[MP_WARPS][MP_KMAX];
    __shared__ uint2 stage[MP_WARPS][MP_STAGE];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * MP_WARPS + w;
    if (q < nq) {
        const size_t base = (size_t)q * n_lists * k;
        // the query's lists are contiguous: one coalesced pass brings them all in
        const bool staged = n_lists * k <= MP_STAGE;
        if (staged) {
            for (int e = lane; e < n_lists * k; e += 32)
                stage[w][e] = make_uint2(__float_as_uint(cv[base + e]), (uint32_t)ci[base + e]);
            __syncwarp();
        }
        warp_merge<DESC>(
            n_lists, k, hv[w], hi[w], cur[w],
            [&](int l, int c, float& v, int32_t& id) {
                if (staged) {
                    const uint2 p = stage[w][l * k + c];
                    v = __uint_as_float(p.x);
                    id = (int32_t)p.y;
                } else {
                    v = cv[base + (size_t)l * k + c];
                    id = ci[base + (size_t)l * k + c];
                }
            },
            [&](int j, float v, int32_t id) {
                outp[w][j] = make_uint2(__float_as_uint(v),
                                        (uint32_t)(id >= 0 ? (int32_t)(id + id_offset) : -1));
            });
        __syncwarp();
        for (int e = lane; e < world * k; e += 32) {
            const int r = e / k, j = e - r * k;
            uint2* dst = reinterpret_cast<uint2*>(peers.p[r] + region_off +
                                                  (size_t)rank * slot_bytes) + (size_t)q * k + j;
            *dst = outp[w][j];
        }
    }
    __syncthreads();  // the CTA's stores happen before thread 0's system-scope fence
    if (threadIdx.x == 0) {
        __threadfence_system();
        const unsigned done = atomicAdd(counter, 1u);
        if (done == gridDim.x - 1) {  // every CTA's stores are fenced: raise the flags
            *counter = 0;
            __threadfence_system();
            for (int r = 0; r < world; ++r) {
                unsigned* f = reinterpret_cast<unsigned*>(peers.p[r] + flag_off) + rank;
                asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(epoch)
                             : "memory");
            }
        }
    }
}

// Every rank's flag of this epoch (warp 0 of each CTA polls, lane r for rank r, bounded),
// then the world lists of query q (region: [world][max_nq][k] pairs) merged into out
// (out_es 2: pairs).
template <bool DESC>
__global__ void __launch_bounds__(MP_WARPS * 32)
    wait_merge_kernel(const char* __restrict__ region, const unsigned* flags, int world,
                      unsigned epoch, uint64_t budget_ns, int* status, int nq, int max_nq, int k,
                      float* out_v, int32_t* out_i, int out_es) {
    __shared__ float hv[MP_WARPS][64];
    __shared__ int32_t hi[MP_WARPS][64];
    __shared__ uint16_t cur[MP_WARPS][64];
    __shared__ uint2 stage[MP_WARPS][WM_STAGE];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * MP_WARPS + w;
    if (w == 0) {
        bool ok = true;
        if (lane < world) {
            const uint64_t t0 = globaltimer_ns();
            unsigned spins = 0;
            for (;;) {
                unsigned v;
                asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + lane)
                             : "memory");
                if (v == epoch) break;
                __nanosleep(64);
                if ((++spins & 63u) == 0 && globaltimer_ns() - t0 > budget_ns) {
                    ok = false;
                    break;
                }
            }
        }
        if (!__all_sync(0xffffffffu, ok) && lane == 0) record_error(status, PION_B200_ETIMEOUT);
    }
    __syncthreads();  // the acquiring lanes' view is the CTA's before any pair is read
    if (q >= nq) return;
    const uint2* pr = reinterpret_cast<const uint2*>(region);
    const size_t lstride = (size_t)max_nq * k;
    const bool staged = world * k <= WM_STAGE;
    if (staged) {
        for (int e = lane; e < world * k; e += 32) {
            const int r = e / k, j = e - r * k;
            stage[w][e] = __ldcg(pr + (size_t)r * lstride + (size_t)q * k + j);
        }
        __syncwarp();
    }
    warp_merge<DESC>(
        world, k, hv[w], hi[w], cur[w],
        [&](int l, int c, float& v, int32_t& id) {
            const uint2 p = staged ? stage[w][l * k + c]
                                   : __ldcg(pr + (size_t)l * lstride + (size_t)q * k + c);
            v = __uint_as_float(p.x);
            id = (int32_t)p.y;
        },
        [&](int j, float v, int32_t id) {
            const size_t o = ((size_t)q * k + j) * out_es;
            out_v[o] = v;
            out_i[o] = id;
        });
}

}  // namespace ex
}  // namespace pion

using namespace pion;

extern "C" {

int pion_v_b200_exchange_create(pion_b200_ctx* ctx, int world, int rank, int regions,
                                int64_t max_nq, int64_t k, pion_b200_exchange** out) {
    if (!valid_ctx(ctx) || !out) return PION_B200_EINVAL;
    *out = nullptr;
    if (world < 1 || world > 64 || rank < 0 || rank >= world || regions < 1 || regions > 4 ||
        max_nq < 1 || k < 1 || k > 64)
        return set_error(ctx, PION_B200_EINVAL, "exchange_create: bad arguments");
    if (int rc = use_device(ctx)) return rc;
    pion_b200_exchange* e = new (std::nothrow) pion_b200_exchange();
    if (!e) return PION_B200_ENOMEM;
    e->device = ctx->device;
    e->world = world;
    e->rank = rank;
    e->regions = regions;
    e->max_nq = max_nq;
    e->k = k;
    e->region_bytes = align_up((size_t)world * max_nq * k * 8, 256);
    e->flags_off = (size_t)regions * 2 * e->region_bytes;
    const size_t total = e->flags_off + (size_t)regions * 2 * 64 * 4;
    if (cudaMalloc(&e->base, total) != cudaSuccess ||
        cudaMalloc(&e->counter, sizeof(unsigned)) != cudaSuccess ||
        cudaMemset(e->base + e->flags_off, 0, (size_t)regions * 2 * 64 * 4) != cudaSuccess ||
        cudaMemset(e->counter, 0, sizeof(unsigned)) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess) {
        cudaGetLastError();
        if (e->base) cudaFree(e->base);
        if (e->counter) cudaFree(e->counter);
        delete e;
        return set_error(ctx, PION_B200_ENOMEM, "exchange_create: device memory");
    }
    e->peer[rank] = e->base;
    *out = e;
    return 0;
}

int pion_v_b200_exchange_handle(const pion_b200_exchange* e, void* out_handle) {
    if (!e || !out_handle) return PION_B200_EINVAL;
    if (cudaSetDevice(e->device) != cudaSuccess) return PION_B200_ENODEV;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, e->base) != cudaSuccess) {
        cudaGetLastError();
        return PION_B200_ECUDA;
    }
    static_assert(sizeof(h) <= PION_B200_IPC_HANDLE_BYTES, "handle size");
    memset(out_handle, 0, PION_B200_IPC_HANDLE_BYTES);
    memcpy(out_handle, &h, sizeof(h));
    return 0;
}

int pion_v_b200_exchange_connect(pion_b200_exchange* e, const void* handles) {
    if (!e || !handles || e->connected) return PION_B200_EINVAL;
    if (cudaSetDevice(e->device) != cudaSuccess) return PION_B200_ENODEV;
    for (int r = 0; r < e->world; ++r) {
        if (r == e->rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const char*>(handles) + (size_t)r * PION_B200_IPC_HANDLE_BYTES,
               sizeof(h));
        void* p = nullptr;
        if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            fprintf(stderr, "pion_vector_b200: exchange_connect: rank %d cannot map rank %d\n",
                    e->rank, r);
            return PION_B200_ECUDA;
        }
        e->peer[r] = static_cast<char*>(p);
    }
    e->connected = true;
    return 0;
}

int pion_v_b200_exchange_world(const pion_b200_exchange* e) {
    return e && e->connected ? e->world : -1;
}

int pion_v_b200_exchange_free(pion_b200_exchange* e) {
    if (!e) return PION_B200_EINVAL;
    cudaSetDevice(e->device);
    cudaDeviceSynchronize();
    for (int r = 0; r < e->world; ++r)
        if (r != e->rank && e->peer[r]) cudaIpcCloseMemHandle(e->peer[r]);
    if (e->base) cudaFree(e->base);
    if (e->counter) cudaFree(e->counter);
    delete e;
    return 0;
}

}  // extern "C"

namespace pion {

static ex::PeerPtrs peer_ptrs(const pion_b200_exchange* e) {
    ex::PeerPtrs pp;
    for (int r = 0; r < 64; ++r) pp.p[r] = r < e->world ? e->peer[r] : nullptr;
    return pp;
}

static bool exchange_ok(const pion_b200_ctx* ctx, const pion_b200_exchange* e, int region,
                        int64_t nq, int64_t k, uint32_t epoch) {
    return e && e->connected && region >= 0 && region < e->regions && nq >= 1 &&
           nq <= e->max_nq && k == e->k && epoch != 0 && e->device == ctx->device;
}

// Every rank's flag of this epoch, then the merged world lists into out.
static int exchange_wait_merge(pion_b200_ctx* ctx, pion_b200_exchange* e, int region,
                               int64_t nq, uint32_t epoch, bool descending, float* out_v,
                               int32_t* out_i, int out_es) {
    if (e->world > 64 || e->k > ex::MP_KMAX) return PION_B200_ESHAPE;
    const int parity = (int)(epoch & 1u);
    const char* reg = e->base + (size_t)(region * 2 + parity) * e->region_bytes;
    const unsigned* flags = reinterpret_cast<const unsigned*>(
        e->base + e->flags_off + (size_t)(region * 2 + parity) * 64 * 4);
    const int blocks = (int)((nq + ex::MP_WARPS - 1) / ex::MP_WARPS);
    int* status = call_status(ctx, PION_B200_MEM_DEVICE);
    const int t_wait = timing_begin(ctx, PION_B200_TIMING_EXCHANGE_WAIT);
    if (descending)
        ex::wait_merge_kernel<true><<<blocks, ex::MP_WARPS * 32, 0, ctx->stream>>>(
            reg, flags, e->world, epoch, ctx->wait_ns, status, (int)nq, (int)e->max_nq,
            (int)e->k, out_v, out_i, out_es);
    else
        ex::wait_merge_kernel<false><<<blocks, ex::MP_WARPS * 32, 0, ctx->stream>>>(
            reg, flags, e->world, epoch, ctx->wait_ns, status, (int)nq, (int)e->max_nq,
            (int)e->k, out_v, out_i, out_es);
    ctx->launches++;
    timing_end(ctx, t_wait);
    return cudaGetLastError() == cudaSuccess ? 0 : PION_B200_ECUDA;
}

// Publish ready-made pairs (nq x k), wait, merge.
int exchange_merge(pion_b200_ctx* ctx, pion_b200_exchange* e, int region, const void* pairs,
                   int64_t nq, int64_t k, uint32_t epoch, bool descending, float* out_v,
                   int32_t* out_i, int out_es) {
    if (!exchange_ok(ctx, e, region, nq, k, epoch)) return PION_B200_EINVAL;
    cudaStream_t st = ctx->stream;
    const int parity = (int)(epoch & 1u);
    const size_t region_off = (size_t)(region * 2 + parity) * e->region_bytes;
    const size_t slot_bytes = (size_t)e->max_nq * e->k * 8;
    const size_t flag_off = e->flags_off + (size_t)(region * 2 + parity) * 64 * 4;
    const int64_t count = nq * k;
    const int t_ex = timing_begin(ctx, PION_B200_TIMING_EXCHANGE);
    int blocks = (int)((count + ex::PUB_THREADS - 1) / ex::PUB_THREADS);
    if (blocks > ctx->num_sms) blocks = ctx->num_sms;
    if (blocks < 1) blocks = 1;
    ex::publish_kernel<<<blocks, ex::PUB_THREADS, 0, st>>>(
        static_cast<const uint2*>(pairs), count, peer_ptrs(e), e->world, e->rank, region_off,
        slot_bytes, flag_off, epoch, e->counter);
    ctx->launches++;
    if (cudaGetLastError() != cudaSuccess) return PION_B200_ECUDA;
    const int rc = exchange_wait_merge(ctx, e, region, nq, epoch, descending, out_v, out_i, out_es);
    timing_end(ctx, t_ex);
    return rc;
}

int exchange_max_lists() { return ex::MP_MAX_LISTS; }

// This shard's candidate lists [nq][n_lists][k] merged and published in one kernel, then
// waited for and merged by another: two kernels for the whole exchange step.
int exchange_lists_merge(pion_b200_ctx* ctx, pion_b200_exchange* e, int region,
                         const float* cv, const int32_t* ci, int n_lists, int64_t id_offset,
                         int64_t nq, int64_t k, uint32_t epoch, bool descending, float* out_v,
                         int32_t* out_i, int out_es) {
    if (!exchange_ok(ctx, e, region, nq, k, epoch)) return PION_B200_EINVAL;
    if (n_lists < 1 || n_lists > ex::MP_MAX_LISTS || k > ex::MP_KMAX) return PION_B200_ESHAPE;
    cudaStream_t st = ctx->stream;
    const int parity = (int)(epoch & 1u);
    const size_t region_off = (size_t)(region * 2 + parity) * e->region_bytes;
    const size_t slot_bytes = (size_t)e->max_nq * e->k * 8;
    const size_t flag_off = e->flags_off + (size_t)(region * 2 + parity) * 64 * 4;
    const int blocks = (int)((nq + ex::MP_WARPS - 1) / ex::MP_WARPS);
    const int t_ex = timing_begin(ctx, PION_B200_TIMING_EXCHANGE);
    if (descending)
        ex::merge_publish_kernel<true><<<blocks, ex::MP_WARPS * 32, 0, st>>>(
            cv, ci, (int)nq, n_lists, (int)k, id_offset, peer_ptrs(e), e->world, e->rank,
            region_off, slot_bytes, flag_off, epoch, e->counter);
    else
        ex::merge_publish_kernel<false><<<blocks, ex::MP_WARPS * 32, 0, st>>>(
            cv, ci, (int)nq, n_lists, (int)k, id_offset, peer_ptrs(e), e->world, e->rank,
            region_off, slot_bytes, flag_off, epoch, e->counter);
    ctx->launches++;
    if (cudaGetLastError() != cudaSuccess) return PION_B200_ECUDA;
    const int rc = exchange_wait_merge(ctx, e, region, nq, epoch, descending, out_v, out_i, out_es);
    timing_end(ctx, t_ex);
    return rc;
}

}  // namespace pion

extern "C" int pion_v_b200_exchange_merge(pion_b200_ctx* ctx, pion_b200_exchange* e,
                                          const void* pairs, int64_t nq, int64_t k,
                                          uint32_t epoch, int flags, float* out_scores,
                                          int32_t* out_ids) {
    if (!valid_ctx(ctx)) return PION_B200_EINVAL;
    if (int rc = use_device(ctx)) return rc;
    const bool pairs_out = (flags & PION_B200_OUT_PAIRS) != 0;
    if (!pairs || !out_scores || (!pairs_out && !out_ids))
        return set_error(ctx, PION_B200_EINVAL, "exchange_merge: bad arguments");
    if (pairs_out) out_ids = reinterpret_cast<int32_t*>(out_scores) + 1;
    const int rc = exchange_merge(ctx, e, 0, pairs, nq, k, epoch,
                                  (flags & PION_B200_MERGE_DESC) != 0, out_scores, out_ids,
                                  pairs_out ? 2 : 1);
    if (rc != 0) return set_error(ctx, rc, "exchange_merge: failed");
    return 0;
}
