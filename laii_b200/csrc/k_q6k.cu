/*
 * Q6_K expert down projection (GGUF Q4_K_M checkpoints store some
 * ffn_down_exps as Q6_K; the reference selects its Q6_K x Q8_K kernels by the
 * tensor's type, tools/lfm2_decode_1x4.c:618-630).
 *
 * Work list: the dispatch tables' (active expert u, 8-token chunk c) pairs, as
 * for the Q4_K GEMVs.  A warp computes down rows r of expert e for the chunk's
 * nt <= 8 slots: y[slot][r] = Down_e[r,:] . hq[slot].
 *
 * Super-block layout (block_q6_K, 210 bytes, tools/lfm2_cpuid_quants.c:101-106):
 * ql[128], qh[64], int8 scales[16], fp16 d.  Value v = 128h + 32m + k (half h,
 * quarter m, k < 32) keeps its low four bits in ql[64h + 32(m%2) + k] (the
 * high nibble when m >= 2) and its top two bits at bits 2m..2m+1 of
 * qh[32h + k]; its scale is scales[v/16] (the reference's unpacking,
 * tools/lfm2_cpuid_quants.c:1509-1512).
 *
 * Lane l owns, in each half h, the values 128h + {2l, 2l+1, 2l+64, 2l+65}: they
 * come from the 16-bit word ql[64h + 2l .. +1] (low nibbles: 2l, 2l+1; high
 * nibbles: 2l+64, 2l+65) and the word qh[32h + (2l & 31) .. +1] (bits 2m0 and
 * 2m0+4 per byte, m0 = l >= 16), with scales (l/8) + {0, 4} + 8h.  Each lane
 * packs sc*q of a value pair as two int16 and dots it with the pair's Q8_K
 * codes by dp2a.
 *
 * Work unit of a CTA (8 warps): one dispatch pair and 32 consecutive down rows.
 *  - Each warp starts 16-byte cp.async copies of its 4 weight rows into its own
 *    shared-memory slab: a row of nb 210-byte blocks starts only 2-byte
 *    aligned, so the copy covers the 16-byte aligned span around it and the
 *    row is read at its offset inside the span (the upload pads the tensor by
 *    16 bytes so the span of the last row stays inside the allocation).
 *  - Meanwhile the CTA stages the pair's Q8_K activations (codes, bsums, d of
 *    its nt tokens) in shared memory once for all 32 rows (64 KB a CTA at I = 1792: three CTAs an SM).
 *  - Then each warp computes its rows from shared memory only.
 *
 * Exact integer part per (token, super-block): the lanes' dp2a sums, lanes
 * 0..15 subtract 32*sc_j*bsums_j, and one warp reduction (redux.sync) gives
 * total = sum sc*q*q8 - 32*sum sc_j*bsums_j, the reference's integer (:1485,
 * :1531).  fp32 update in the reference's AVX-VNNI order, per super-block in
 * order and skipped where d8 == 0:
 *   sum = fma(d8 * d, (float)total, sum)                          (:1534)
 * Integer bounds: |sc*q| <= 128*63 fits int16; |sc*q*q8| <= 128*63*128 per
 * value, 256 values: < 2^29.
 */
#include "moe_device.cuh"
#include "moe_internal.h"

namespace {

constexpr int kCh = LFM_GEMV_CHUNK; /* tokens per pair (8) */
constexpr int kWarps = 8;
constexpr int kRowsPerWarp = 4;
constexpr int kUnitRows = kWarps * kRowsPerWarp; /* 32 */
constexpr uint32_t kMaxNb = 12;                  /* I <= 3072: 109 KB of shared memory a CTA */

/* bytes of one staged weight row: the 16-byte aligned span around nb blocks */
__host__ __device__ inline uint32_t q6k_row_span(uint32_t nb) { return (nb * LFM_Q6K_BYTES + 14u + 15u) & ~15u; }
__host__ __device__ inline size_t q6k_smem(uint32_t nb) {
    return (size_t)kWarps * kRowsPerWarp * q6k_row_span(nb) /* weights */
           + (size_t)kCh * nb * 256 + (size_t)kCh * nb * 32 + (size_t)kCh * nb * 4; /* qs, bsums, d */
}

__device__ __forceinline__ uint32_t ld_s16(const uint8_t *p) { return *reinterpret_cast<const unsigned short *>(p); }

/* Two int16 lanes (a low, b high) of one 32-bit word, for dp2a. */
__device__ __forceinline__ int pack16(int a, int b) { return (int)(((uint32_t)a & 0xFFFFu) | ((uint32_t)b << 16)); }

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(lfm_smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__global__ void __launch_bounds__(kWarps * 32) k_q6k_down(MoeLayerDev L, Q8Rows hq, RouteTables rt, float *y) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t D = L.D, I = L.I, nb = I / 256;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = lane >= 16 ? 1 : 0;        /* quarter of the low-nibble values */
    const uint32_t qh_off = (2u * lane) & 31u;
    const uint32_t span = q6k_row_span(nb);
    uint8_t *wsl = smem + (size_t)warp * kRowsPerWarp * span;            /* this warp's rows */
    uint8_t *qs_s = smem + (size_t)kWarps * kRowsPerWarp * span;         /* [kCh][I] */
    int16_t *bs_s = reinterpret_cast<int16_t *>(qs_s + (size_t)kCh * I); /* [kCh][nb][16] */
    float *d_s = reinterpret_cast<float *>(bs_s + (size_t)kCh * nb * 16); /* [kCh][nb] */
    const uint32_t groups = D / kUnitRows;
    const uint64_t n_units = (uint64_t)__ldcg(rt.summary + 3) * groups;
    for (uint64_t u = blockIdx.x; u < n_units; u += gridDim.x) {
        const uint32_t j = (uint32_t)(u / groups), r0 = (uint32_t)(u % groups) * kUnitRows + warp * kRowsPerWarp;
        const int2 pr = __ldcg(rt.pairs + j);
        const int e = __ldcg(rt.act + pr.x);
        const int n_e = __ldcg(rt.counts + e), off_e = __ldcg(rt.offsets + e);
        const int slot0 = off_e + pr.y * kCh;
        const int nt = min(kCh, n_e - pr.y * kCh);
        __syncthreads(); /* the previous unit's activations and rows are no longer read */
        /* weights: this warp's rows, 16-byte copies of each row's aligned span */
        uint32_t rem[kRowsPerWarp]; /* offset of row i inside its staged span */
#pragma unroll
        for (int i = 0; i < kRowsPerWarp; ++i) {
            const uint8_t *rs = L.down + ((size_t)e * D + r0 + i) * nb * LFM_Q6K_BYTES;
            rem[i] = (uint32_t)(reinterpret_cast<uintptr_t>(rs) & 15u);
            const uint8_t *a = rs - rem[i];
            const uint32_t n16 = (rem[i] + nb * LFM_Q6K_BYTES + 15u) >> 4;
            for (uint32_t c = lane; c < n16; c += 32) cp_async16(wsl + (size_t)i * span + 16u * c, a + 16u * c);
        }
        /* activations of the pair's nt tokens, once for the CTA */
        for (uint32_t c = threadIdx.x; c < (uint32_t)nt * (I / 16); c += blockDim.x) {
            const uint32_t t = c / (I / 16), o = c % (I / 16);
            reinterpret_cast<int4 *>(qs_s + (size_t)t * I)[o] =
                __ldg(reinterpret_cast<const int4 *>(hq.qs + (size_t)(slot0 + t) * I) + o);
        }
        for (uint32_t c = threadIdx.x; c < (uint32_t)nt * nb * 2; c += blockDim.x) {
            const uint32_t t = c / (nb * 2), o = c % (nb * 2);
            reinterpret_cast<int4 *>(bs_s + (size_t)t * nb * 16)[o] =
                __ldg(reinterpret_cast<const int4 *>(hq.bs + (size_t)(slot0 + t) * nb * 16) + o);
        }
        for (uint32_t c = threadIdx.x; c < (uint32_t)nt * nb; c += blockDim.x)
            d_s[c] = __ldg(hq.d + (size_t)slot0 * nb + c);
        cp_async_wait_all();
        __syncthreads(); /* activations staged; every lane's weight copies landed */

        for (int i = 0; i < kRowsPerWarp; ++i) {
            const uint8_t *row = wsl + (size_t)i * span + rem[i];
            float sum[kCh];
#pragma unroll
            for (int t = 0; t < kCh; ++t) sum[t] = 0.0f;
            for (uint32_t b = 0; b < nb; ++b) {
                const uint8_t *blk = row + (size_t)b * LFM_Q6K_BYTES;
                const int8_t *sc = reinterpret_cast<const int8_t *>(blk + 192);
                int P[2][2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t ql = ld_s16(blk + 64 * h + 2 * lane), qh = ld_s16(blk + 128 + 32 * h + qh_off);
                    const int s_lo = sc[8 * h + (lane >> 3)], s_hi = sc[8 * h + 4 + (lane >> 3)];
                    const int sh = 2 * m0;
                    const int q0 = (int)((ql & 15u) | ((qh >> sh) & 3u) << 4);
                    const int q1 = (int)((ql >> 8 & 15u) | ((qh >> (8 + sh)) & 3u) << 4);
                    const int q2 = (int)((ql >> 4 & 15u) | ((qh >> (sh + 4)) & 3u) << 4);
                    const int q3 = (int)((ql >> 12 & 15u) | ((qh >> (12 + sh)) & 3u) << 4);
                    P[h][0] = pack16(q0 * s_lo, q1 * s_lo);
                    P[h][1] = pack16(q2 * s_hi, q3 * s_hi);
                }
                const int scl = lane < 16 ? (int)sc[lane] : 0;
                const float dw = lfm_h2f((uint16_t)ld_s16(blk + 208));
#pragma unroll
                for (int t = 0; t < kCh; ++t) {
                    if (t < nt) { /* warp-uniform */
                        const uint8_t *q8 = reinterpret_cast<const uint8_t *>(qs_s + (size_t)t * I + (size_t)b * 256);
                        int part = __dp2a_lo(P[0][0], (int)ld_s16(q8 + 2 * lane), 0);
                        part = __dp2a_lo(P[0][1], (int)ld_s16(q8 + 64 + 2 * lane), part);
                        part = __dp2a_lo(P[1][0], (int)ld_s16(q8 + 128 + 2 * lane), part);
                        part = __dp2a_lo(P[1][1], (int)ld_s16(q8 + 192 + 2 * lane), part);
                        if (lane < 16) part -= 32 * scl * (int)bs_s[((size_t)t * nb + b) * 16 + lane];
                        const int total = __reduce_add_sync(LFM_FULL_MASK, part);
                        const float d8 = d_s[t * nb + b];
                        if (d8 != 0.0f) sum[t] = __fmaf_rn(__fmul_rn(d8, dw), __int2float_rn(total), sum[t]);
                    }
                }
            }
#pragma unroll
            for (int t = 0; t < kCh; ++t)
                if (t < nt && lane == t) y[(size_t)(slot0 + t) * D + r0 + i] = sum[t];
        }
    }
}

}  // namespace

cudaError_t lfm_launch_down_q6k(const MoeLayerDev &L, Q8Rows hq, const RouteTables &rt, float *y, int grid,
                                cudaStream_t s) {
    if (!L.down_q6k || L.I % 256 || L.I / 256 > kMaxNb || L.D % kUnitRows) return cudaErrorInvalidValue;
    static size_t cache[16];
    const size_t smem = q6k_smem(L.I / 256);
    cudaError_t e = lfm_smem_attr((const void *)k_q6k_down, smem, cache);
    if (e != cudaSuccess) return e;
    k_q6k_down<<<grid * 3, kWarps * 32, smem, s>>>(L, hq, rt, y);
    return cudaGetLastError();
}
