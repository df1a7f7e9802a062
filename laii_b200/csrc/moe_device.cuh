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
/* exp for SwiGLU's SiLU: CUDA's single-precision expf (within 2 ulp).  The
 * layer's fp32 outputs are compared under a tolerance, so the double-precision
 * round trip above (one double exp per element of h: the cost of the SwiGLU
 * kernel at prefill sizes) is kept for the router, where an ulp can decide a
 * top-K near-tie. */
__device__ __forceinline__ float lfm_silu_expf(float x) { return expf(x); }

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

/* The same test, but the thread may be suspended (for at most hint_ns) until
 * the phase completes: a waiting warp then takes no issue slots from the
 * warps doing the work. */
__device__ __forceinline__ bool lfm_mbar_try_wait_sleep(uint64_t *bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(lfm_smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}
#define LFM_WAIT_SLEEP_NS 20000u /* longest single suspension inside a bounded wait */

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
    while (!lfm_mbar_try_wait_sleep(bar, parity, LFM_WAIT_SLEEP_NS)) {
        if (lfm_globaltimer() - t0 > LFM_WAIT_LIMIT_NS) {
            atomicOr(err, LFM_DEVERR_TIMEOUT);
            return false;
        }
    }
    return true;
}

/* Flags another GPU writes (expert parallelism over peer memory). */
__device__ __forceinline__ uint32_t lfm_ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void lfm_st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int32_t lfm_ld_relaxed_sys(const int32_t *p) {
    int32_t v;
    asm volatile("ld.relaxed.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

/* One thread: wait until flags[0..n) all reach `epoch` (wrap-safe), for at
 * most wait_ns in total.  On timeout: set the error bit and return false. */
__device__ __forceinline__ bool lfm_wait_flags(const uint32_t *flags, uint32_t n, uint32_t epoch, uint64_t wait_ns,
                                               uint32_t *err) {
    const uint64_t t0 = lfm_globaltimer();
    for (uint32_t p = 0; p < n; ++p) {
        while ((int32_t)(lfm_ld_acquire_sys(flags + p) - epoch) < 0) {
            if (lfm_globaltimer() - t0 > wait_ns) {
                atomicOr(err, LFM_DEVERR_TIMEOUT);
                return false;
            }
            __nanosleep(64);
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

/* 2-D tiled tensor copy (no multicast) of the box at element coordinates
 * (x, y) into shared memory, completing on `bar`; x * element size must be a
 * multiple of 16 bytes. */
__device__ __forceinline__ void lfm_tma_load_2d(void *dst, const CUtensorMap *tm, uint32_t x, uint32_t y,
                                                uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            lfm_smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(lfm_smem_u32(bar))
        : "memory");
}

/* The same copy with an L2 cache policy (lfm_policy_evict_first for data read
 * once, so it leaves the rest of the working set in L2). */
__device__ __forceinline__ void lfm_tma_load_2d_hint(void *dst, const CUtensorMap *tm, uint32_t x, uint32_t y,
                                                     uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(
            lfm_smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(lfm_smem_u32(bar)), "l"(policy)
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
 * Q4_K x Q8_K: one super-block per lane
 * ------------------------------------------------------------------------ */

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

/* Q8_K activation rows staged in shared memory, one 304-byte record per
 * (row, super-block):  [0,256) codes, [256,288) the 16 bsums, [288,292) d.
 * Records of a row are consecutive (row stride nb*304), so lane h of a row
 * group reading super-block 8p+h hits bank group (3h + j) mod 8 for 16-byte
 * chunk j: the 8 super-block lanes of a warp never conflict, every offset
 * inside a record is an immediate, and the 4 row groups read the same
 * addresses (broadcast). */
#define LFM_ACT_REC 304u

struct ActSlot {
    const uint8_t *rec;  /* row 0, super-block 0 */
    uint32_t nb;
};

__host__ __device__ constexpr size_t lfm_act_slot_bytes(uint32_t cols, uint32_t rows_cap = LFM_GEMV_CHUNK) {
    return (size_t)rows_cap * (cols / 256) * LFM_ACT_REC;
}

__device__ __forceinline__ ActSlot lfm_act_slot(const uint8_t *base, uint32_t cols) { return ActSlot{base, cols / 256}; }

/* Copy nt Q8 rows (global row ids rows[t]) into a slot; threads tid of nthr. */
__device__ __forceinline__ void lfm_stage_act(const Q8Rows &src, const int *rows, int nt, uint8_t *slot, int tid,
                                              int nthr) {
    const uint32_t cols = src.cols, nb = cols / 256;
    /* 19 16-byte pieces per record: 16 of codes, 2 of bsums, then d (4 bytes) */
    const uint32_t per_row = nb * 19;
    for (uint32_t q = tid; q < (uint32_t)nt * per_row; q += nthr) {
        const uint32_t t = q / per_row, r = q % per_row, b = r / 19, j = r % 19;
        const size_t row = (size_t)rows[t];
        uint8_t *dst = slot + ((size_t)t * nb + b) * LFM_ACT_REC + 16 * j;
        if (j < 16) {
            *reinterpret_cast<uint4 *>(dst) = __ldcg(reinterpret_cast<const uint4 *>(src.qs + row * cols + 256 * b) + j);
        } else if (j < 18) {
            *reinterpret_cast<uint4 *>(dst) =
                __ldcg(reinterpret_cast<const uint4 *>(src.bs + (row * nb + b) * 16) + (j - 16));
        } else {
            *reinterpret_cast<float *>(dst) = __ldcg(src.d + row * nb + b);
        }
    }
}

/* 32-bit load from shared memory. */
__device__ __forceinline__ uint32_t lfm_lds32(const uint8_t *p) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(lfm_smem_u32(p)));
    return v;
}

/* sum of 4 products of unsigned bytes of a with signed bytes of b, plus c */
__device__ __forceinline__ int lfm_dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

/*
 * One Q4_K super-block (the 144 bytes at w) against super-block b of kNt staged
 * Q8_K rows (records rec + toff[t]), as the reference's Q4_K x Q8_K
 * row kernels form it (tools/lfm2_cpuid_quants.c:421-457, :1189-1257):
 *   dot_j   = sum_{l<32} q4[32j+l] * q8[32j+l]          (sub-block j = 0..7)
 *   acc     = sum_j sc_j * dot_j
 *   mins    = sum_j m_j * (bsum[2j] + bsum[2j+1])
 * and the operands of its fp32 update  sum = fma(d8*d, acc, fma(-(d8*dmin), mins, sum)):
 *   out[t] = (d8*d, (float)acc, d8*dmin, (float)mins),
 * or (-0, 0, 0, 0) -- an exact identity of that update -- when d8 == 0 (the
 * reference skips such blocks).  Nibble layout: byte l of 32-byte group c
 * holds element l of sub-block 2c (low nibble) and of 2c+1 (high nibble); the
 * high nibbles are used in place (w & 0xF0F0F0F0 = 16 * nibble, unsigned) and
 * the exact dot divided by 16 afterwards.  Integers: the order is free.
 * kDebug: dbg[0..7] = token 0's sub-block dots, dbg[8] = acc, dbg[9] = mins.
 */
template <int kNt, bool kSharedW, bool kDebug>
__device__ __forceinline__ void lfm_q4k_sb(const uint8_t *w, const uint8_t *rec, const uint32_t (&toff)[kNt],
                                           float4 (&out)[kNt], int32_t *dbg) {
    const uint4 hdr = lfm_ld16<kSharedW>(w);
    const uint32_t s0 = hdr.y, s1 = hdr.z, s2 = hdr.w;
    /* 6-bit scales and mins of sub-blocks 0-3 (low 6 bits of bytes 0-3 / 4-7)
     * and 4-7 (low / high nibble of bytes 8-11, top 2 bits from bytes 0-3 / 4-7) */
    const uint32_t scA = s0 & 0x3F3F3F3Fu;
    const uint32_t scB = (s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u);
    const uint32_t mA = s1 & 0x3F3F3F3Fu;
    const uint32_t mB = ((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u);
    /* m_j duplicated into the byte pair __dp2a multiplies bsum 2j and 2j+1 by */
    const int mm0 = (int)__byte_perm(mA, 0, 0x1100), mm1 = (int)__byte_perm(mA, 0, 0x3322);
    const int mm2 = (int)__byte_perm(mB, 0, 0x1100), mm3 = (int)__byte_perm(mB, 0, 0x3322);
    int acc[kNt];
#pragma unroll
    for (int t = 0; t < kNt; ++t) acc[t] = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint4 qa = lfm_ld16<kSharedW>(w + 16 + 32 * c), qb = lfm_ld16<kSharedW>(w + 32 + 32 * c);
        const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        int lo[8];
        uint32_t hi[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            lo[i] = (int)(q[i] & 0x0F0F0F0Fu);
            hi[i] = q[i] & 0xF0F0F0F0u;
        }
        const int sc_lo = (int)(((c < 2 ? scA : scB) >> (16 * (c & 1))) & 0xFFu);
        const int sc_hi = (int)(((c < 2 ? scA : scB) >> (16 * (c & 1) + 8)) & 0xFFu);
#pragma unroll
        for (int t = 0; t < kNt; ++t) {
            const uint8_t *xr = rec + toff[t] + 64 * c;
            const uint4 x0 = lfm_ld16<true>(xr), x1 = lfm_ld16<true>(xr + 16);
            const uint4 x2 = lfm_ld16<true>(xr + 32), x3 = lfm_ld16<true>(xr + 48);
            int dl = __dp4a(lo[0], (int)x0.x, 0);
            dl = __dp4a(lo[1], (int)x0.y, dl);
            dl = __dp4a(lo[2], (int)x0.z, dl);
            dl = __dp4a(lo[3], (int)x0.w, dl);
            dl = __dp4a(lo[4], (int)x1.x, dl);
            dl = __dp4a(lo[5], (int)x1.y, dl);
            dl = __dp4a(lo[6], (int)x1.z, dl);
            dl = __dp4a(lo[7], (int)x1.w, dl);
            int dh = lfm_dp4a_us(hi[0], (int)x2.x, 0);
            dh = lfm_dp4a_us(hi[1], (int)x2.y, dh);
            dh = lfm_dp4a_us(hi[2], (int)x2.z, dh);
            dh = lfm_dp4a_us(hi[3], (int)x2.w, dh);
            dh = lfm_dp4a_us(hi[4], (int)x3.x, dh);
            dh = lfm_dp4a_us(hi[5], (int)x3.y, dh);
            dh = lfm_dp4a_us(hi[6], (int)x3.z, dh);
            dh = lfm_dp4a_us(hi[7], (int)x3.w, dh);
            dh >>= 4; /* exact: a multiple of 16 */
            acc[t] += sc_lo * dl + sc_hi * dh;
            if (kDebug && t == 0) {
                dbg[2 * c] = dl;
                dbg[2 * c + 1] = dh;
            }
        }
    }
    const float d = lfm_h2f((uint16_t)(hdr.x & 0xFFFFu)), dmin = lfm_h2f((uint16_t)(hdr.x >> 16));
#pragma unroll
    for (int t = 0; t < kNt; ++t) {
        const uint8_t *xr = rec + toff[t];
        const uint4 p0 = lfm_ld16<true>(xr + 256), p1 = lfm_ld16<true>(xr + 272);
        const float d8 = __uint_as_float(lfm_lds32(xr + 288));
        int mins = __dp2a_lo((int)p0.x, mm0, 0);
        mins = __dp2a_hi((int)p0.y, mm0, mins);
        mins = __dp2a_lo((int)p0.z, mm1, mins);
        mins = __dp2a_hi((int)p0.w, mm1, mins);
        mins = __dp2a_lo((int)p1.x, mm2, mins);
        mins = __dp2a_hi((int)p1.y, mm2, mins);
        mins = __dp2a_lo((int)p1.z, mm3, mins);
        mins = __dp2a_hi((int)p1.w, mm3, mins);
        if (kDebug && t == 0) {
            dbg[8] = acc[0];
            dbg[9] = mins;
        }
        out[t] = d8 != 0.0f ? make_float4(__fmul_rn(d8, d), (float)acc[t], __fmul_rn(d8, dmin), (float)mins)
                            : make_float4(-0.0f, 0.0f, 0.0f, 0.0f);
    }
}

/* The reference's fp32 update over n super-blocks in order, from the operands
 * lfm_q4k_sb produced: e = (d8*d, acc, d8*dmin, mins) at e0, e0 + estride, ... */
__device__ __forceinline__ float lfm_q4k_chain(float sum, const uint8_t *e0, uint32_t estride, uint32_t n) {
#pragma unroll
    for (uint32_t h = 0; h < 8; ++h) {
        if (h < n) {
            const uint4 v = lfm_ld16<true>(e0 + (size_t)h * estride);
            sum = __fmaf_rn(__uint_as_float(v.x), __uint_as_float(v.y),
                            __fmaf_rn(-__uint_as_float(v.z), __uint_as_float(v.w), sum));
        }
    }
    return sum;
}

/* Q8_K of one 256-value block held 8 per lane (elements 8*lane..8*lane+7),
 * written as a 304-byte activation record in shared memory: d = max/127,
 * q = RNE(x*(127/max)) saturated to int8, bsums of the unsaturated codes
 * (tools/lfm2_cpuid_quants.c:584-631). */
__device__ __forceinline__ void lfm_quant_block_rec(const float v[8], uint8_t *rec) {
    const int lane = threadIdx.x & 31;
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = lfm_warp_max(amax);
    int q[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int part = 0;
    if (amax != 0.0f) {
        const float sc = __fdiv_rn(127.0f, amax);
#pragma unroll
        for (int i = 0; i < 8; ++i) { q[i] = __float2int_rn(__fmul_rn(v[i], sc)); part += q[i]; }
    }
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        lo |= (uint32_t)(uint8_t)(int8_t)max(-128, min(127, q[i])) << (8 * i);
        hi |= (uint32_t)(uint8_t)(int8_t)max(-128, min(127, q[4 + i])) << (8 * i);
    }
    *reinterpret_cast<uint2 *>(rec + 8 * lane) = make_uint2(lo, hi);
    const int pair = part + __shfl_xor_sync(LFM_FULL_MASK, part, 1);
    if ((lane & 1) == 0) *reinterpret_cast<int16_t *>(rec + 256 + lane) = (int16_t)pair;
    if (lane == 0) *reinterpret_cast<float *>(rec + 288) = amax == 0.0f ? 0.0f : __fdiv_rn(amax, 127.0f);
}

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
