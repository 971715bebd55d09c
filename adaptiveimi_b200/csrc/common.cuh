// common.cuh -- shared device helpers for the IMI B200 kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#define IMI_DEV __device__ __forceinline__

namespace imi {

// bf16 bits -> fp32 (exact widening, the same as the reference's bf16_to_fp32,
// kmeans_core.cpp:808-812).
IMI_DEV float bf16_bits_to_f32(uint16_t h) { return __uint_as_float(static_cast<uint32_t>(h) << 16); }
IMI_DEV float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
IMI_DEV float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Monotone float -> uint32 map (larger float -> larger key; -0 and +0 map apart
// but compare as adjacent, NaN is not produced by the callers).
IMI_DEV uint32_t ord_f32(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

IMI_DEV float warp_sum(float v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
IMI_DEV int warp_sum_i(int v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Squared L2 distance in the reference's lane order (kmeans_core.cpp:22-44):
// lane l accumulates fma(d, d, acc) over dims l, l+8, ...; lanes are summed
// left to right.  `x` is in registers (DIM floats), `c` is in shared memory.
// DIM is a multiple of 8 for every geometry this library supports.
template <int DIM>
IMI_DEV float dist_lanes8(const float (&x)[DIM], const float* __restrict__ c) {
    float lane[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) lane[l] = 0.0f;
#pragma unroll
    for (int i = 0; i < DIM; i += 8) {
        const float4 c0 = *reinterpret_cast<const float4*>(c + i);
        const float4 c1 = *reinterpret_cast<const float4*>(c + i + 4);
        float d;
        d = __fsub_rn(x[i + 0], c0.x); lane[0] = __fmaf_rn(d, d, lane[0]);
        d = __fsub_rn(x[i + 1], c0.y); lane[1] = __fmaf_rn(d, d, lane[1]);
        d = __fsub_rn(x[i + 2], c0.z); lane[2] = __fmaf_rn(d, d, lane[2]);
        d = __fsub_rn(x[i + 3], c0.w); lane[3] = __fmaf_rn(d, d, lane[3]);
        d = __fsub_rn(x[i + 4], c1.x); lane[4] = __fmaf_rn(d, d, lane[4]);
        d = __fsub_rn(x[i + 5], c1.y); lane[5] = __fmaf_rn(d, d, lane[5]);
        d = __fsub_rn(x[i + 6], c1.z); lane[6] = __fmaf_rn(d, d, lane[6]);
        d = __fsub_rn(x[i + 7], c1.w); lane[7] = __fmaf_rn(d, d, lane[7]);
    }
    float t = __fadd_rn(lane[0], lane[1]);
    t = __fadd_rn(t, lane[2]);
    t = __fadd_rn(t, lane[3]);
    t = __fadd_rn(t, lane[4]);
    t = __fadd_rn(t, lane[5]);
    t = __fadd_rn(t, lane[6]);
    return __fadd_rn(t, lane[7]);
}

// Same distance with both operands in memory (generic dim, multiple of 8).
IMI_DEV float dist_lanes8_mem(const float* __restrict__ a, const float* __restrict__ c, int dim) {
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int i = 0; i < dim; i += 8) {
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            float d = __fsub_rn(a[i + l], c[i + l]);
            lane[l] = __fmaf_rn(d, d, lane[l]);
        }
    }
    float t = __fadd_rn(lane[0], lane[1]);
#pragma unroll
    for (int l = 2; l < 8; ++l) t = __fadd_rn(t, lane[l]);
    return t;
}

// 128-bit unsigned helpers (exact fixed-point sums).
struct u128 {
    unsigned long long lo, hi;
};
IMI_DEV u128 u128_add(u128 a, u128 b) {
    u128 r;
    r.lo = a.lo + b.lo;
    r.hi = a.hi + b.hi + (r.lo < a.lo ? 1ull : 0ull);
    return r;
}
IMI_DEV bool u128_ge(u128 a, u128 b) { return a.hi > b.hi || (a.hi == b.hi && a.lo >= b.lo); }
IMI_DEV u128 u128_shfl_up(u128 v, int d) {
    u128 r;
    r.lo = __shfl_up_sync(0xffffffffu, v.lo, d);
    r.hi = __shfl_up_sync(0xffffffffu, v.hi, d);
    return r;
}

}  // namespace imi
