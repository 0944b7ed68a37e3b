// Shared device-side helpers for the B200 (sm_100a) KNN kernels: status codes,
// mbarrier / TMA / tcgen05 wrappers written as inline PTX, and bounded waits.
//
// Every wait in these kernels is bounded by a wall-clock budget read from
// %globaltimer.  A wait that runs out records PION_B200_ETIMEOUT in the launch's
// status word and returns false; the caller then drains what it has in flight and
// leaves, so a stuck pipeline ends the kernel with an error instead of hanging the GPU.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/pion_vector_b200.h"

namespace pion {

// Wall-clock budget of one bounded wait (nanoseconds).  Kernels finish in
// milliseconds; two seconds without progress means the pipeline is broken.
constexpr uint64_t kWaitBudgetNs = 2000000000ull;

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void record_error(int* status, int code) {
    if (status) atomicCAS(status, 0, code);
}

// ---------------------------------------------------------------- mbarrier --
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete.  Returns false (and
// records a timeout) if the budget runs out or another thread already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status,
                                          volatile int* abort_flag,
                                          uint64_t budget_ns = kWaitBudgetNs) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((++spins & 63u) == 0) {
            if (abort_flag && *abort_flag) return false;
            if (globaltimer_ns() - t0 > budget_ns) {
                record_error(status, PION_B200_ETIMEOUT);
                if (abort_flag) *abort_flag = 1;
                return false;
            }
        }
    }
}

// ---------------------------------------------------------------------- TMA --
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled bulk tensor load global -> shared, completing on an mbarrier.
// x is the innermost (contiguous) coordinate in elements; callers keep x*elem
// a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// 1-D bulk copy global -> shared (both addresses 16-B aligned, bytes % 16 == 0).
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes,
                                          uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// ------------------------------------------------------------------ tcgen05 --
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(smem_slot)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Arrives once on `bar` when every tcgen05.mma issued so far by this thread is done.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, int8 x int8 -> int32.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, tf32 x tf32 -> f32.
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, bf16 x bf16 -> f32 (kind::f16).
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives TMEM lane
// (lane_base + i), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Waits for this thread's TMEM loads; the registers of `r` are operands of the
// wait, so no use of them can be scheduled before it.
__device__ __forceinline__ void tmem_ld_wait_regs(uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.wait::ld.sync.aligned;"
        : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
          "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]),
          "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]),
          "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]),
          "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]),
          "+r"(r[31])
        :
        : "memory");
}

// Shared-memory matrix descriptor for a K-major operand staged by TMA with the
// 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart (SBO), the
// leading-dimension offset unused for this layout, descriptor version 1 (sm_100),
// layout type 2 (SWIZZLE_128B) in bits 61-63.  `smem_addr` must lie inside a
// 1024-byte aligned tile; advancing along K inside the 128-byte row is done by
// adding the byte offset to the start address.
__device__ __forceinline__ uint64_t make_sw128_kmajor_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);  // start address
    d |= static_cast<uint64_t>(1u) << 16;                      // LBO (unused, 16 B)
    d |= static_cast<uint64_t>(1024u >> 4) << 32;              // SBO = 1024 B
    d |= static_cast<uint64_t>(1u) << 46;                      // version
    d |= static_cast<uint64_t>(2u) << 61;                      // SWIZZLE_128B
    return d;
}

// Instruction descriptor, kind::i8: s8 x s8 -> s32, both operands K-major.
__host__ __device__ constexpr uint32_t make_idesc_i8(int m, int n) {
    return (2u << 4)                                   // D format: S32
           | (1u << 7)                                 // A: signed 8-bit
           | (1u << 10)                                // B: signed 8-bit
           | (static_cast<uint32_t>(n >> 3) << 17)     // N / 8
           | (static_cast<uint32_t>(m >> 4) << 24);    // M / 16
}

// Instruction descriptor, kind::tf32: tf32 x tf32 -> f32, both operands K-major.
__host__ __device__ constexpr uint32_t make_idesc_tf32(int m, int n) {
    return (1u << 4)                                   // D format: F32
           | (2u << 7)                                 // A: TF32
           | (2u << 10)                                // B: TF32
           | (static_cast<uint32_t>(n >> 3) << 17)
           | (static_cast<uint32_t>(m >> 4) << 24);
}

// Instruction descriptor, kind::f16 with bf16 operands -> f32, both K-major.
__host__ __device__ constexpr uint32_t make_idesc_bf16(int m, int n) {
    return (1u << 4)                                   // D format: F32
           | (1u << 7)                                 // A: BF16
           | (1u << 10)                                // B: BF16
           | (static_cast<uint32_t>(n >> 3) << 17)
           | (static_cast<uint32_t>(m >> 4) << 24);
}

// ------------------------------------------------------ visited-word lists --
// A warp's visited bitmap is kept all zero between searches by listing the words it turns
// non-zero.  Appends the words that lanes in `mask` turned non-zero (lane L's word `w`) to
// the warp's list; n is the warp-uniform count (it may pass cap: then the list is
// incomplete and the search zeroes the whole bitmap).  Call with the whole warp.
__device__ __forceinline__ void note_words(uint32_t* list, int cap, int& n, unsigned mask,
                                           uint32_t w, int lane) {
    if (!mask) return;
    if (mask & (1u << lane)) {
        const int at = n + __popc(mask & ((1u << lane) - 1u));
        if (at < cap) list[at] = w;
    }
    n += __popc(mask);
}

// ------------------------------------------------------- top-k in registers --
// PTX select: the compiler cannot fold a chain of these back into an indexed
// access, which would move the whole register array to local memory.
__device__ __forceinline__ uint32_t selp_u32(uint32_t a, uint32_t b, bool take_a) {
    uint32_t r;
    asm("{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %3, 0;\n\tselp.b32 %0, %1, %2, p;\n\t}"
        : "=r"(r)
        : "r"(a), "r"(b), "r"((uint32_t)take_a));
    return r;
}

// A sorted (descending) list of KCAP (score, id) pairs kept in registers.  Scans
// present ids in ascending order, so the list is ordered by (score desc, id asc).
// Insertion is low-latency: every entry is compared with the new pair at once
// (the entries ahead of it form a prefix), then every slot picks its new value
// independently, instead of a KCAP-long chain of dependent compare-swaps.
template <int KCAP>
struct TopKDesc {
    float v[KCAP];
    int32_t i[KCAP];
    __device__ __forceinline__ void init() {
#pragma unroll
        for (int j = 0; j < KCAP; ++j) {
            v[j] = -INFINITY;
            i[j] = -1;
        }
    }
    __device__ __forceinline__ void insert(float s, int32_t id) {
        bool ahead[KCAP];
#pragma unroll
        for (int j = 0; j < KCAP; ++j)
            ahead[j] = v[j] > s || (v[j] == s && i[j] >= 0 && (id < 0 || i[j] < id));
        float nv[KCAP];
        int32_t ni[KCAP];
#pragma unroll
        for (int j = 0; j < KCAP; ++j) {
            const bool at = !ahead[j] && (j == 0 || ahead[j - 1]);
            const float prev_v = j == 0 ? s : v[j - 1];
            const int32_t prev_i = j == 0 ? id : i[j - 1];
            nv[j] = ahead[j] ? v[j] : (at ? s : prev_v);
            ni[j] = ahead[j] ? i[j] : (at ? id : prev_i);
        }
#pragma unroll
        for (int j = 0; j < KCAP; ++j) {
            v[j] = nv[j];
            i[j] = ni[j];
        }
    }
    // The k-th best score (1 <= k <= KCAP) by a log-depth select tree over the bits
    // of k - 1.  A capacity that is not a power of two is only used with k == KCAP: the
    // last entry.
    __device__ __forceinline__ float kth(int k) const {
        if constexpr ((KCAP & (KCAP - 1)) != 0) return v[KCAP - 1];
        uint32_t t[KCAP];
#pragma unroll
        for (int j = 0; j < KCAP; ++j) t[j] = __float_as_uint(v[j]);
        const uint32_t want = (uint32_t)(k - 1);
#pragma unroll
        for (int w = KCAP / 2, b = 0; w >= 1; w /= 2, ++b) {
            const bool hi = (want >> b) & 1u;
#pragma unroll
            for (int j = 0; j < w; ++j) t[j] = selp_u32(t[2 * j + 1], t[2 * j], hi);
        }
        return __uint_as_float(t[0]);
    }
};

// (score desc, id asc) strict ordering used by every merge.
__device__ __forceinline__ bool better_desc(float sa, int32_t ia, float sb, int32_t ib) {
    if (sa != sb) return sa > sb;
    if (ia < 0) return false;
    if (ib < 0) return true;
    return ia < ib;
}

// (score desc, id asc) when DESC, else (score asc, id asc); a padding id (< 0) last.
template <bool DESC>
__device__ __forceinline__ bool merge_better(float sa, int32_t ia, float sb, int32_t ib) {
    if (DESC) return better_desc(sa, ia, sb, ib);
    if (sa != sb) return sa < sb;
    if (ia < 0) return false;
    if (ib < 0) return true;
    return ia < ib;
}

}  // namespace pion
