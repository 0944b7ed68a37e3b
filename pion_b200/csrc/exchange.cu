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
// every rank with a system-scope release store.  Waiting: lane r of one warp reads flag r
// with system-scope acquire loads until it holds the step's epoch; the wait is bounded (a
// %globaltimer budget), after which it records PION_B200_ETIMEOUT and returns, so a rank
// whose peer died gets an error instead of a hang.
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

// Waits until every rank's flag holds `epoch` (bounded), recording a timeout otherwise.
__global__ void wait_flags_kernel(const unsigned* flags, int world, unsigned epoch,
                                  uint64_t budget_ns, int* status) {
    const int lane = threadIdx.x;
    bool ok = true;
    if (lane < world) {
        const uint64_t t0 = globaltimer_ns();
        unsigned spins = 0;
        for (;;) {
            unsigned v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + lane)
                         : "memory");
            if (v == epoch) break;
            if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > budget_ns) {
                ok = false;
                break;
            }
        }
    }
    if (!ok) record_error(status, PION_B200_ETIMEOUT);
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

// Publish + wait + merge on the context's stream (device memory): region `region`,
// parity of `epoch`.  The merged k per query go to out_v / out_i (out_es = 2: pairs).
int exchange_merge(pion_b200_ctx* ctx, pion_b200_exchange* e, int region, const void* pairs,
                   int64_t nq, int64_t k, uint32_t epoch, bool descending, float* out_v,
                   int32_t* out_i, int out_es) {
    if (!e || !e->connected || region < 0 || region >= e->regions || nq < 1 ||
        nq > e->max_nq || k != e->k || epoch == 0 || e->device != ctx->device)
        return PION_B200_EINVAL;
    cudaStream_t st = ctx->stream;
    const int parity = (int)(epoch & 1u);
    const size_t region_off = (size_t)(region * 2 + parity) * e->region_bytes;
    const size_t slot_bytes = (size_t)e->max_nq * e->k * 8;
    const size_t flag_off = e->flags_off + (size_t)(region * 2 + parity) * 64 * 4;
    ex::PeerPtrs pp;
    for (int r = 0; r < 64; ++r) pp.p[r] = r < e->world ? e->peer[r] : nullptr;
    const int64_t count = nq * k;
    int blocks = (int)((count + ex::PUB_THREADS - 1) / ex::PUB_THREADS);
    if (blocks > ctx->num_sms) blocks = ctx->num_sms;
    if (blocks < 1) blocks = 1;
    ex::publish_kernel<<<blocks, ex::PUB_THREADS, 0, st>>>(
        static_cast<const uint2*>(pairs), count, pp, e->world, e->rank, region_off, slot_bytes,
        flag_off, epoch, e->counter);
    ex::wait_flags_kernel<<<1, 64, 0, st>>>(
        reinterpret_cast<const unsigned*>(e->base + flag_off), e->world, epoch, ctx->wait_ns,
        call_status(ctx, PION_B200_MEM_DEVICE));
    ctx->launches += 2;
    if (cudaGetLastError() != cudaSuccess) return PION_B200_ECUDA;
    // the world lists, lists-major with a slot stride of max_nq entries: merge the
    // [world][max_nq][k] pairs as [world][nq][k] by viewing each slot from its start
    return launch_merge_lists(reinterpret_cast<const float*>(e->base + region_off), nullptr,
                              (int)nq, e->world, (int)k, 0, descending, out_v, out_i, st,
                              true, 0, true, out_es, (int)e->max_nq);
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
