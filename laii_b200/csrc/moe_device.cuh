/*
 * Device helpers shared by the MoE-FFN kernels.
 *
 * Floating point: the library is built with -fmad=false -ftz=true, so every
 * a*b+c below is two roundings unless written as __fmaf_rn; that lets the
 * kernels follow the reference's evaluation order exactly (the reference runs
 * with FTZ/DAZ set, include/lfm2_simd_avx2.h:49-80).
 */
#ifndef LFM_MOE_DEVICE_CUH
#define LFM_MOE_DEVICE_CUH

#include <cuda_fp16.h>
#include <stdint.h>

#include "lfm_formats.h"

#define LFM_FULL_MASK 0xFFFFFFFFu

/* exp(x) rounded to fp32 from a double-precision evaluation.  The reference
 * calls glibc expf (an error bound of about half an ulp); going through double
 * keeps our sigmoid/SiLU within rounding of it far more often than a
 * single-precision expf would.  Calls CUDA's double exp. */
__device__ __forceinline__ float lfm_expf(float x) { return (float)exp((double)x); }

__device__ __forceinline__ float lfm_h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

/* Sum of 16 per-lane partials (lanes base..base+15 of a 16-wide segment) in
 * the reference's tree: v_l = a_l + a_{l+8}; s_l = v_l + v_{l+4};
 * (s_0 + s_2) + (s_1 + s_3)   (two 8-wide accumulators added, then
 * include/lfm2_simd_avx2.h:286-293).  Result valid in the segment's lane 0. */
__device__ __forceinline__ float lfm_hsum16_ref(float a) {
    const float v = __fadd_rn(a, __shfl_down_sync(LFM_FULL_MASK, a, 8, 16));
    const float s = __fadd_rn(v, __shfl_down_sync(LFM_FULL_MASK, v, 4, 16));
    const float p = __fadd_rn(s, __shfl_down_sync(LFM_FULL_MASK, s, 2, 16));
    return __fadd_rn(p, __shfl_down_sync(LFM_FULL_MASK, p, 1, 16));
}

__device__ __forceinline__ float lfm_warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(LFM_FULL_MASK, v, o));
    return v;
}

__device__ __forceinline__ int lfm_warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(LFM_FULL_MASK, v, o);
    return v;
}

/* 6-bit scale and min of sub-blocks 2g and 2g+1 from the 12 scale bytes
 * (given as three 32-bit words).  Same unpacking as lfm_q4k_scale_min. */
__device__ __forceinline__ void lfm_q4k_pair_scales(uint32_t s0, uint32_t s1, uint32_t s2, int g, int &sc_lo,
                                                    int &m_lo, int &sc_hi, int &m_hi) {
    uint8_t s[12];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        s[i] = (uint8_t)(s0 >> (8 * i));
        s[4 + i] = (uint8_t)(s1 >> (8 * i));
        s[8 + i] = (uint8_t)(s2 >> (8 * i));
    }
    int j = 2 * g;
    if (j < 4) {
        sc_lo = s[j] & 63; m_lo = s[j + 4] & 63;
        sc_hi = s[j + 1] & 63; m_hi = s[j + 5] & 63;
    } else {
        sc_lo = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        m_lo = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
        sc_hi = (s[j + 5] & 0x0F) | ((s[j - 3] >> 6) << 4);
        m_hi = (s[j + 5] >> 4) | ((s[j + 1] >> 6) << 4);
    }
}

/* 128-bit read-only streaming load (weights are read once per forward). */
__device__ __forceinline__ uint4 lfm_ldg_stream(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

#endif /* LFM_MOE_DEVICE_CUH */
