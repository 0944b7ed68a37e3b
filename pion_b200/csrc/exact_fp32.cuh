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

// (distance asc, id asc)
__device__ __forceinline__ bool better_asc(float da, int32_t ia, float db, int32_t ib) {
    if (da != db) return da < db;
    if (ia < 0) return false;
    if (ib < 0) return true;
    return ia < ib;
}

}  // namespace pion
