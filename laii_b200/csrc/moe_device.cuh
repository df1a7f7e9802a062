/*
 * Device helpers shared by the MoE-FFN kernels.
 *
 * Floating point: the library is built with -fmad=false -ftz=true, so every
 * a*b+c below is two roundings unless written as __fmaf_rn; that lets the
 * kernels follow the reference's evaluation order exactly (the reference runs
 * with FTZ/DAZ set, include/lfm2_simd_avx2.h:49-80).
 *
 * Waits: every mbarrier wait is bounded by wall time (%globaltimer); on
 * timeout the kernel records LFM_DEVERR_TIMEOUT in the device error word and
 * abandons its work instead of hanging.
 */
#ifndef LFM_MOE_DEVICE_CUH
#define LFM_MOE_DEVICE_CUH

#include <cuda_fp16.h>
#include <stdint.h>

#include "lfm_formats.h"
#include "moe_internal.h"

#define LFM_FULL_MASK 0xFFFFFFFFu

/* Bound on any single wait inside a kernel (ns). */
#define LFM_WAIT_LIMIT_NS 200000000ull

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

/* 6-bit scale and min of sub-blocks 2g and 2g+1 from the 12 scale bytes
 * (three little-endian words s0 = bytes 0-3, s1 = 4-7, s2 = 8-11), without
 * branching on g.  Sub-block j < 4 keeps scale/min in the low 6 bits of byte j
 * and byte j+4; j >= 4 keeps the low nibbles in byte j+4 and the top 2 bits in
 * bits 6-7 of bytes j-4 (scale) and j (min) -- the layout lfm_q4k_scale_min
 * reads.  sh = 16*(g&1) selects the byte pair for both halves. */
__device__ __forceinline__ void lfm_q4k_pair_scales(uint32_t s0, uint32_t s1, uint32_t s2, int g, int &sc_lo,
                                                    int &m_lo, int &sc_hi, int &m_hi) {
    const uint32_t sh = 16u * (uint32_t)(g & 1);
    const uint32_t a0 = s0 >> sh, a1 = s1 >> sh, a2 = s2 >> sh;
    if (g < 2) {  /* uniform per quarter-warp group of 4 lanes; both sides are a handful of ops */
        sc_lo = (int)(a0 & 63u);
        sc_hi = (int)((a0 >> 8) & 63u);
        m_lo = (int)(a1 & 63u);
        m_hi = (int)((a1 >> 8) & 63u);
    } else {
        sc_lo = (int)((a2 & 15u) | (((a0 >> 6) & 3u) << 4));
        sc_hi = (int)(((a2 >> 8) & 15u) | (((a0 >> 14) & 3u) << 4));
        m_lo = (int)(((a2 >> 4) & 15u) | (((a1 >> 6) & 3u) << 4));
        m_hi = (int)(((a2 >> 12) & 15u) | (((a1 >> 14) & 3u) << 4));
    }
}

/* ------------------------------------------------------------------------
 * mbarrier + bulk-copy (TMA, non-tensor) + programmatic dependent launch
 * ------------------------------------------------------------------------ */
__device__ __forceinline__ uint32_t lfm_smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void lfm_mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(lfm_smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void lfm_fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void lfm_mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(lfm_smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void lfm_mbar_arrive_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(lfm_smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool lfm_mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(lfm_smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t lfm_globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

/* Wait for phase `parity` of `bar`, for at most LFM_WAIT_LIMIT_NS.  On
 * timeout: set the error bit and return false. */
__device__ __forceinline__ bool lfm_mbar_wait(uint64_t *bar, uint32_t parity, uint32_t *err) {
    if (lfm_mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = lfm_globaltimer();
    while (!lfm_mbar_try_wait(bar, parity)) {
        if (lfm_globaltimer() - t0 > LFM_WAIT_LIMIT_NS) {
            atomicOr(err, LFM_DEVERR_TIMEOUT);
            return false;
        }
    }
    return true;
}

/* L2 policy for data read exactly once (expert weights). */
__device__ __forceinline__ uint64_t lfm_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

/* Global -> shared bulk copy completing on `bar` (16-byte aligned, bytes % 16 == 0). */
__device__ __forceinline__ void lfm_bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                             uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            lfm_smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(lfm_smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ void lfm_bulk_g2s_plain(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     lfm_smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(lfm_smem_u32(bar))
                 : "memory");
}

/* Bulk prefetch of global memory into L2 (bytes % 16 == 0, 16-byte aligned). */
__device__ __forceinline__ void lfm_prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

/* Programmatic dependent launch: wait for the preceding kernel's results /
 * let the next kernel start its prologue. */
__device__ __forceinline__ void lfm_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void lfm_pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

/* Named barrier over the first `threads` threads of the block (id 1..15). */
__device__ __forceinline__ void lfm_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

/* ------------------------------------------------------------------------
 * Q4_K x Q8_K: 8 weight rows per warp
 * ------------------------------------------------------------------------ */

struct RowDebug {
    int32_t *sub_dots;  /* [8 rows][nb][8] or NULL */
    int32_t *acc;       /* [8 rows][nb] */
    int32_t *mins;      /* [8 rows][nb] */
};

/* Q8_K activation rows staged in shared memory for one (expert, chunk) pair:
 *   qs  [nt][cols]   within each 256-byte super-block, the 16-byte chunk
 *                    (group g, part k) -- bytes 64g+16k.. -- is stored at
 *                    chunk 4k+g, so the 4 lane groups of a warp reading part k
 *                    hit 4 distinct bank groups (and the 8 rows broadcast);
 *   bs  [nt][nb][16] bsums;   d [nt][nb] scales. */
struct ActSmem {
    const uint8_t *qs;
    const int16_t *bs;
    const float *d;
    uint32_t cols, nb;
};

__host__ __device__ constexpr size_t lfm_act_slot_bytes(uint32_t cols) {
    return (size_t)LFM_GEMV_CHUNK * cols + (size_t)LFM_GEMV_CHUNK * (cols / 256) * 36;
}

__device__ __forceinline__ ActSmem lfm_act_slot(const uint8_t *base, uint32_t cols) {
    const uint32_t nb = cols / 256;
    return ActSmem{base, reinterpret_cast<const int16_t *>(base + (size_t)LFM_GEMV_CHUNK * cols),
                   reinterpret_cast<const float *>(base + (size_t)LFM_GEMV_CHUNK * cols + (size_t)LFM_GEMV_CHUNK * nb * 32),
                   cols, nb};
}

/* Copy nt Q8 rows (global row ids rows[t]) into a slot; threads tid of nthr. */
__device__ __forceinline__ void lfm_stage_act(const Q8Rows &src, const int *rows, int nt, uint8_t *slot, int tid,
                                              int nthr) {
    const uint32_t cols = src.cols, nb = cols / 256, qv = cols / 16;
    uint8_t *qs = slot;
    int16_t *bs = reinterpret_cast<int16_t *>(slot + (size_t)LFM_GEMV_CHUNK * cols);
    float *dd = reinterpret_cast<float *>(slot + (size_t)LFM_GEMV_CHUNK * cols + (size_t)LFM_GEMV_CHUNK * nb * 32);
    for (uint32_t q = tid; q < (uint32_t)nt * qv; q += nthr) {
        const uint32_t t = q / qv, c = q % qv;
        const uint32_t sb = c >> 4, gk = c & 15;             /* logical chunk 4g+k of super-block sb */
        const uint32_t phys = sb * 16 + (gk & 3) * 4 + (gk >> 2);
        const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(src.qs + (size_t)rows[t] * cols) + c);
        reinterpret_cast<uint4 *>(qs + (size_t)t * cols)[phys] = v;
    }
    for (uint32_t q = tid; q < (uint32_t)nt * nb * 2; q += nthr) {
        const uint32_t t = q / (nb * 2), c = q % (nb * 2);
        reinterpret_cast<uint4 *>(bs + (size_t)t * nb * 16)[c] =
            __ldcg(reinterpret_cast<const uint4 *>(src.bs + (size_t)rows[t] * nb * 16) + c);
    }
    for (uint32_t q = tid; q < (uint32_t)nt * nb; q += nthr) {
        const uint32_t t = q / nb, c = q % nb;
        dd[(size_t)t * nb + c] = __ldcg(src.d + (size_t)rows[t] * nb + c);
    }
}

/* 16-byte load from shared memory (kShared) or through a generic pointer. */
template <bool kShared>
__device__ __forceinline__ uint4 lfm_ld16(const uint8_t *p) {
    if (kShared) {
        uint4 v;
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                     : "r"(lfm_smem_u32(p)));
        return v;
    }
    return *reinterpret_cast<const uint4 *>(p);
}

/*
 * Dots of 8 consecutive Q4_K weight rows (row r at w + r*rstride, shared memory
 * when kSharedW) -- and, for kMats == 2, of the 8 rows at w1 -- with nt (<= 8)
 * staged Q8_K activation rows.
 *
 * Lane 4*r + g owns weight row r and the 32 nibble bytes of group g (sub-blocks
 * 2g and 2g+1) of every super-block.  For each super-block b in order and each
 * token: sub-block dots with __dp4a, the exact integer super-block sums
 *   acc = sum_j sc_j * dot_j,   mins = sum_j m_j * (bsum_{2j} + bsum_{2j+1})
 * (reduced over the row's 4 lanes; integer, so any order), then the fp32 update
 * of the reference's 4-row AVX-VNNI kernel (tools/lfm2_cpuid_quants.c:1189-1257):
 *   sum = fma(d8*d, acc, fma(-(d8*dmin), mins, sum)),  skipped when d8 == 0.
 * The running sums stay in registers; every lane of a row ends with the row's
 * results s0[t] (and s1[t]).
 */
template <int kMats, bool kDebug, bool kSharedW = true>
__device__ __forceinline__ void lfm_q4k_rows8(const uint8_t *w0, const uint8_t *w1, uint32_t rstride,
                                              const ActSmem &act, int nt, float (&s0)[LFM_GEMV_CHUNK],
                                              float (&s1)[LFM_GEMV_CHUNK], RowDebug dbg) {
    const int lane = threadIdx.x & 31;
    const int r = lane >> 2, g = lane & 3;
    const uint32_t nb = act.nb;
    const uint8_t *row0 = w0 + (size_t)r * rstride;
    const uint8_t *row1 = kMats == 2 ? w1 + (size_t)r * rstride : nullptr;
#pragma unroll
    for (int t = 0; t < LFM_GEMV_CHUNK; ++t) { s0[t] = 0.0f; s1[t] = 0.0f; }
    for (uint32_t b = 0; b < nb; ++b) {
        int sc0l, m0l, sc0h, m0h, sc1l = 0, m1l = 0, sc1h = 0, m1h = 0;
        uint32_t wl0[8], wh0[8], wl1[8], wh1[8];
        float d0, dm0, d1 = 0.0f, dm1 = 0.0f;
        {
            const uint8_t *blk = row0 + (size_t)b * LFM_Q4K_BYTES;
            const uint4 hdr = lfm_ld16<kSharedW>(blk);
            const uint4 qa = lfm_ld16<kSharedW>(blk + 16 + 32 * g);
            const uint4 qb = lfm_ld16<kSharedW>(blk + 32 + 32 * g);
            lfm_q4k_pair_scales(hdr.y, hdr.z, hdr.w, g, sc0l, m0l, sc0h, m0h);
            d0 = lfm_h2f((uint16_t)(hdr.x & 0xFFFFu));
            dm0 = lfm_h2f((uint16_t)(hdr.x >> 16));
            const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) { wl0[i] = w[i] & 0x0F0F0F0Fu; wh0[i] = (w[i] >> 4) & 0x0F0F0F0Fu; }
        }
        if (kMats == 2) {
            const uint8_t *blk = row1 + (size_t)b * LFM_Q4K_BYTES;
            const uint4 hdr = lfm_ld16<kSharedW>(blk);
            const uint4 qa = lfm_ld16<kSharedW>(blk + 16 + 32 * g);
            const uint4 qb = lfm_ld16<kSharedW>(blk + 32 + 32 * g);
            lfm_q4k_pair_scales(hdr.y, hdr.z, hdr.w, g, sc1l, m1l, sc1h, m1h);
            d1 = lfm_h2f((uint16_t)(hdr.x & 0xFFFFu));
            dm1 = lfm_h2f((uint16_t)(hdr.x >> 16));
            const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) { wl1[i] = w[i] & 0x0F0F0F0Fu; wh1[i] = (w[i] >> 4) & 0x0F0F0F0Fu; }
        }
#pragma unroll
        for (int t = 0; t < LFM_GEMV_CHUNK; ++t) {
            if (t < nt) {
                /* this lane's 64 activation bytes: parts k = 0..3 of group g, at chunks 4k+g */
                const uint8_t *xb = act.qs + (size_t)t * act.cols + 256 * b + 16 * g;
                const uint4 x0 = lfm_ld16<true>(xb), x1 = lfm_ld16<true>(xb + 64);
                const uint4 x2 = lfm_ld16<true>(xb + 128), x3 = lfm_ld16<true>(xb + 192);
                uint2 bw;
                float d8;
                asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];"
                             : "=r"(bw.x), "=r"(bw.y)
                             : "r"(lfm_smem_u32(act.bs + ((size_t)t * nb + b) * 16 + 4 * g)));
                asm volatile("ld.shared.f32 %0, [%1];" : "=f"(d8) : "r"(lfm_smem_u32(act.d + (size_t)t * nb + b)));
                const int xl[8] = {(int)x0.x, (int)x0.y, (int)x0.z, (int)x0.w, (int)x1.x, (int)x1.y, (int)x1.z, (int)x1.w};
                const int xh[8] = {(int)x2.x, (int)x2.y, (int)x2.z, (int)x2.w, (int)x3.x, (int)x3.y, (int)x3.z, (int)x3.w};
                const int bp0 = (int)(int16_t)(bw.x & 0xFFFFu) + (int)(int16_t)(bw.x >> 16);
                const int bp1 = (int)(int16_t)(bw.y & 0xFFFFu) + (int)(int16_t)(bw.y >> 16);
                /* four independent 2-deep chains per sum (exact integers: any order) */
                int pl0[4], ph0[4], pl1[4], ph1[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    pl0[i] = __dp4a((int)wl0[i + 4], xl[i + 4], __dp4a((int)wl0[i], xl[i], 0));
                    ph0[i] = __dp4a((int)wh0[i + 4], xh[i + 4], __dp4a((int)wh0[i], xh[i], 0));
                    if (kMats == 2) {
                        pl1[i] = __dp4a((int)wl1[i + 4], xl[i + 4], __dp4a((int)wl1[i], xl[i], 0));
                        ph1[i] = __dp4a((int)wh1[i + 4], xh[i + 4], __dp4a((int)wh1[i], xh[i], 0));
                    }
                }
                const int dl0 = (pl0[0] + pl0[1]) + (pl0[2] + pl0[3]);
                const int dh0 = (ph0[0] + ph0[1]) + (ph0[2] + ph0[3]);
                const int dl1 = kMats == 2 ? (pl1[0] + pl1[1]) + (pl1[2] + pl1[3]) : 0;
                const int dh1 = kMats == 2 ? (ph1[0] + ph1[1]) + (ph1[2] + ph1[3]) : 0;
                if (kDebug && dbg.sub_dots) {
                    dbg.sub_dots[((size_t)r * nb + b) * 8 + 2 * g] = dl0;
                    dbg.sub_dots[((size_t)r * nb + b) * 8 + 2 * g + 1] = dh0;
                }
                int a0 = sc0l * dl0 + sc0h * dh0, n0 = m0l * bp0 + m0h * bp1;
                int a1 = sc1l * dl1 + sc1h * dh1, n1 = m1l * bp0 + m1h * bp1;
                a0 += __shfl_xor_sync(LFM_FULL_MASK, a0, 1);
                n0 += __shfl_xor_sync(LFM_FULL_MASK, n0, 1);
                if (kMats == 2) {
                    a1 += __shfl_xor_sync(LFM_FULL_MASK, a1, 1);
                    n1 += __shfl_xor_sync(LFM_FULL_MASK, n1, 1);
                }
                a0 += __shfl_xor_sync(LFM_FULL_MASK, a0, 2);
                n0 += __shfl_xor_sync(LFM_FULL_MASK, n0, 2);
                if (kMats == 2) {
                    a1 += __shfl_xor_sync(LFM_FULL_MASK, a1, 2);
                    n1 += __shfl_xor_sync(LFM_FULL_MASK, n1, 2);
                }
                if (kDebug && dbg.acc && g == 0) {
                    dbg.acc[(size_t)r * nb + b] = a0;
                    dbg.mins[(size_t)r * nb + b] = n0;
                }
                if (d8 != 0.0f) {
                    s0[t] = __fmaf_rn(__fmul_rn(d8, d0), (float)a0, __fmaf_rn(-__fmul_rn(d8, dm0), (float)n0, s0[t]));
                    if (kMats == 2)
                        s1[t] = __fmaf_rn(__fmul_rn(d8, d1), (float)a1, __fmaf_rn(-__fmul_rn(d8, dm1), (float)n1, s1[t]));
                }
            }
        }
    }
}

/* Shared-memory row stride of staged weight rows: rows stay contiguous so an
 * item is one bulk copy per matrix (the two rows a quarter-warp reads may share
 * a bank group: a 2-way conflict on 3 loads per super-block, cheaper than 8
 * copies per matrix). */
__host__ __device__ inline uint32_t lfm_stage_stride(uint32_t row_bytes) { return row_bytes; }

/* Q8_K of one 256-value block held 8 per lane (values v[], elements 8*lane..):
 * d = max/127, q = RNE(x*(127/max)), bsums of the unsaturated codes
 * (tools/lfm2_cpuid_quants.c:584-631).  Writes into Q8 row `r`, block `b`. */
__device__ __forceinline__ void lfm_quant_block_warp(const float v[8], Q8Rows dst, size_t r, uint32_t b) {
    const int lane = threadIdx.x & 31;
    const uint32_t nb = dst.cols / 256;
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = lfm_warp_max(amax);
    int q[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int part = 0;
    if (amax != 0.0f) {
        const float s = __fdiv_rn(127.0f, amax);
#pragma unroll
        for (int i = 0; i < 8; ++i) { q[i] = __float2int_rn(__fmul_rn(v[i], s)); part += q[i]; }
    }
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        lo |= (uint32_t)(uint8_t)(int8_t)max(-128, min(127, q[i])) << (8 * i);
        hi |= (uint32_t)(uint8_t)(int8_t)max(-128, min(127, q[4 + i])) << (8 * i);
    }
    *reinterpret_cast<uint2 *>(dst.qs + r * dst.cols + 256 * b + 8 * lane) = make_uint2(lo, hi);
    const int pair = part + __shfl_xor_sync(LFM_FULL_MASK, part, 1);
    if ((lane & 1) == 0) dst.bs[(r * nb + b) * 16 + (lane >> 1)] = (int16_t)pair;
    if (lane == 0) dst.d[r * nb + b] = amax == 0.0f ? 0.0f : __fdiv_rn(amax, 127.0f);
}

#endif /* LFM_MOE_DEVICE_CUH */
