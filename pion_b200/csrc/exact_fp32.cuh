// Exact reference arithmetic shared by the FP32 and BQ rerank kernels.
#pragma once

#include <cstdint>

namespace pion {

// dot_f32_4chain over `dim` floats by 16 lanes of a warp: lane L (< 16) owns chain
// L/4, lane L%4, and sums elements L, L+16, ... in order; the tail chain, the
// ((a0+a1)+(a2+a3)) combine, the halving-tree lane sum and the scalar tail follow
// src/vector/fp32_scan.mojo:17-38 exactly.  `half` selects lanes 0-15 or 16-31; the
// result is returned to every lane of that half.
__device__ __forceinline__ float dot4chain_half(const float* __restrict__ q,
                                                const float* __restrict__ v, int dim,
                                                int hl /* lane within half */, unsigned mask) {
    const int main_end = dim & ~15;
    float acc = 0.0f;
    // unrolled so that the loads run ahead of the (unchanged) addition chain
#pragma unroll 8
    for (int d = hl; d < main_end; d += 16) acc = __fadd_rn(__fmul_rn(q[d], v[d]), acc);
    // 4-element tail blocks continue chain 0 (lanes 0..3)
    int d4 = main_end;
    for (; d4 + 4 <= dim; d4 += 4)
        if (hl < 4) acc = __fadd_rn(__fmul_rn(q[d4 + hl], v[d4 + hl]), acc);
    // t[l] = (a0[l] + a1[l]) + (a2[l] + a3[l]): chains c at lanes 4c + l
    const int base = (threadIdx.x & 31) & 16;  // 0 or 16
    const int l = hl & 3;
    const float a0 = __shfl_sync(mask, acc, base + l);
    const float a1 = __shfl_sync(mask, acc, base + 4 + l);
    const float a2 = __shfl_sync(mask, acc, base + 8 + l);
    const float a3 = __shfl_sync(mask, acc, base + 12 + l);
    const float t = __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
    // reduce_add of the 4 lanes t[0..3]: (t0 + t2) + (t1 + t3)
    const float t0 = __shfl_sync(mask, t, base + 0);
    const float t1 = __shfl_sync(mask, t, base + 1);
    const float t2 = __shfl_sync(mask, t, base + 2);
    const float t3 = __shfl_sync(mask, t, base + 3);
    float s = __fadd_rn(__fadd_rn(t0, t2), __fadd_rn(t1, t3));
    for (int d = d4; d < dim; ++d) s = __fadd_rn(s, __fmul_rn(q[d], v[d]));
    return s;
}

// l2sq_f32_4chain (src/vector/fp32_scan.mojo:42-66) by 16 lanes, the chains of
// dot4chain_half over e = q - v with acc = acc + e * e (two roundings).
__device__ __forceinline__ float l2sq4chain_half(const float* __restrict__ q,
                                                 const float* __restrict__ v, int dim, int hl,
                                                 unsigned mask) {
    const int main_end = dim & ~15;
    float acc = 0.0f;
#pragma unroll 8
    for (int d = hl; d < main_end; d += 16) {
        const float e = __fsub_rn(q[d], v[d]);
        acc = __fadd_rn(__fmul_rn(e, e), acc);
    }
    int d4 = main_end;
    for (; d4 + 4 <= dim; d4 += 4)
        if (hl < 4) {
            const float e = __fsub_rn(q[d4 + hl], v[d4 + hl]);
            acc = __fadd_rn(__fmul_rn(e, e), acc);
        }
    const int base = (threadIdx.x & 31) & 16;
    const int l = hl & 3;
    const float a0 = __shfl_sync(mask, acc, base + l);
    const float a1 = __shfl_sync(mask, acc, base + 4 + l);
    const float a2 = __shfl_sync(mask, acc, base + 8 + l);
    const float a3 = __shfl_sync(mask, acc, base + 12 + l);
    const float t = __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
    const float t0 = __shfl_sync(mask, t, base + 0);
    const float t1 = __shfl_sync(mask, t, base + 1);
    const float t2 = __shfl_sync(mask, t, base + 2);
    const float t3 = __shfl_sync(mask, t, base + 3);
    float s = __fadd_rn(__fadd_rn(t0, t2), __fadd_rn(t1, t3));
    for (int d = d4; d < dim; ++d) {
        const float e = __fsub_rn(q[d], v[d]);
        s = __fadd_rn(s, __fmul_rn(e, e));
    }
    return s;
}

// Asks L2 for whole rows of `dim` floats ahead of the dot products (one bulk prefetch per
// row; rows start 16-byte aligned and dim * 4 is a multiple of 16).
__device__ __forceinline__ void prefetch_row_f32_l2(const float* row, int dim) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(row), "r"((uint32_t)dim * 4u)
                 : "memory");
}

__device__ __forceinline__ float4 ld_stream_f4(const float4* p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ float sel4(float a0, float a1, float a2, float a3, int i) {
    return i == 0 ? a0 : (i == 1 ? a1 : (i == 2 ? a2 : a3));
}

// dot_f32_4chain over `dim` (a multiple of 16) floats by a group of 4 consecutive lanes:
// lane j (= lane & 3) owns chain j of the reference's 4 x 4 accumulators, i.e. elements
// 16 i + 4 j .. 16 i + 4 j + 3, read with 128-bit non-allocating loads (`row` may be
// null for a masked group: zero accumulators); q4 holds the query as float4 (shared
// memory).  A 4 x 4 transpose then gives lane l the l-th lane of every chain,
// t[l] = (c0 + c1) + (c2 + c3), and the lane sum (t0 + t2) + (t1 + t3) returned to all
// four lanes: src/vector/fp32_scan.mojo:17-38 in order.  Every lane of the warp must
// call it (full-warp shuffles).
template <int UNROLL>
__device__ __forceinline__ float dot4chain_quad(const float4* __restrict__ q4,
                                                const float* __restrict__ row, int dim) {
    const int j = threadIdx.x & 3;
    const int gbase = (threadIdx.x & 31) & ~3;
    const int steps = dim >> 4;
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
    if (row) {
        const float4* rp = reinterpret_cast<const float4*>(row) + j;
        for (int i0 = 0; i0 < steps; i0 += UNROLL) {
            float4 v[UNROLL];
#pragma unroll
            for (int u = 0; u < UNROLL; ++u)
                if (i0 + u < steps) v[u] = ld_stream_f4(rp + (size_t)(i0 + u) * 4);
#pragma unroll
            for (int u = 0; u < UNROLL; ++u)
                if (i0 + u < steps) {
                    const float4 q = q4[(i0 + u) * 4 + j];
                    a0 = __fadd_rn(__fmul_rn(q.x, v[u].x), a0);
                    a1 = __fadd_rn(__fmul_rn(q.y, v[u].y), a1);
                    a2 = __fadd_rn(__fmul_rn(q.z, v[u].z), a2);
                    a3 = __fadd_rn(__fmul_rn(q.w, v[u].w), a3);
                }
        }
    }
    // round x: lane j receives lane (j ^ x)'s accumulator j = lane j of chain j ^ x
    const float own = sel4(a0, a1, a2, a3, j);
    const float r1 = __shfl_xor_sync(0xffffffffu, sel4(a0, a1, a2, a3, j ^ 1), 1);
    const float r2 = __shfl_xor_sync(0xffffffffu, sel4(a0, a1, a2, a3, j ^ 2), 2);
    const float r3 = __shfl_xor_sync(0xffffffffu, sel4(a0, a1, a2, a3, j ^ 3), 3);
    // chain m's lane j arrived in round j ^ m
    const float c0 = sel4(own, r1, r2, r3, j ^ 0);
    const float c1 = sel4(own, r1, r2, r3, j ^ 1);
    const float c2 = sel4(own, r1, r2, r3, j ^ 2);
    const float c3 = sel4(own, r1, r2, r3, j ^ 3);
    const float t = __fadd_rn(__fadd_rn(c0, c1), __fadd_rn(c2, c3));
    const float t0 = __shfl_sync(0xffffffffu, t, gbase + 0);
    const float t1 = __shfl_sync(0xffffffffu, t, gbase + 1);
    const float t2 = __shfl_sync(0xffffffffu, t, gbase + 2);
    const float t3 = __shfl_sync(0xffffffffu, t, gbase + 3);
    return __fadd_rn(__fadd_rn(t0, t2), __fadd_rn(t1, t3));
}

// (distance asc, id asc)
__device__ __forceinline__ bool better_asc(float da, int32_t ia, float db, int32_t ib) {
    if (da != db) return da < db;
    if (ia < 0) return false;
    if (ib < 0) return true;
    return ia < ib;
}

}  // namespace pion
