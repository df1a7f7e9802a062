/*
 * Q6_K expert down projection (GGUF Q4_K_M checkpoints store some
 * ffn_down_exps as Q6_K; the reference selects its Q6_K x Q8_K kernels by the
 * tensor's type, tools/lfm2_decode_1x4.c:618-630).
 *
 * Work list: the dispatch tables' (active expert u, 8-token chunk c) pairs, as
 * for the Q4_K GEMVs.  One warp computes one down row r of expert e for the
 * chunk's nt <= 8 slots: y[slot][r] = Down_e[r,:] . hq[slot].
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
 * 2m0+4 per byte, m0 = l >= 16), with scales (l/8) + {0, 4} + 8h.  So a warp
 * reads each weight byte once, in 16-bit words (a 210-byte block is only
 * 2-byte aligned), and the scales are loaded by lanes 0..15 and shared by
 * shuffles.  Each lane packs sc*q of a value pair as two int16 and dots it
 * with the pair's Q8_K codes by dp2a.
 *
 * A warp first loads the weight words of up to 4 super-blocks of its row (all
 * in flight at once), then computes them: two DRAM round trips for a row of
 * 6 or 7 super-blocks (I = 1536, 1792) instead of one per super-block.  (8 at
 * once needs 157 registers a thread, 4 needs 96.)
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
constexpr int kSb = 4;              /* super-blocks whose weights are loaded together */

__device__ __forceinline__ uint32_t ld_u16(const uint8_t *p) {
    return __ldg(reinterpret_cast<const unsigned short *>(p));
}

/* Two int16 lanes (a low, b high) of one 32-bit word, for dp2a. */
__device__ __forceinline__ int pack16(int a, int b) { return (int)(((uint32_t)a & 0xFFFFu) | ((uint32_t)b << 16)); }

__global__ void __launch_bounds__(kWarps * 32) k_q6k_down(MoeLayerDev L, Q8Rows hq, RouteTables rt, float *y) {
    const uint32_t D = L.D, I = L.I, nb = I / 256;
    const int lane = threadIdx.x & 31;
    const int m0 = lane >= 16 ? 1 : 0;        /* quarter of the low-nibble values */
    const uint32_t qh_off = (2u * lane) & 31u;
    const uint64_t n_items = (uint64_t)__ldcg(rt.summary + 3) * D;
    const uint64_t step = (uint64_t)gridDim.x * kWarps;
    for (uint64_t it = (uint64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); it < n_items; it += step) {
        const uint32_t j = (uint32_t)(it / D), r = (uint32_t)(it % D);
        const int2 pr = __ldcg(rt.pairs + j);
        const int e = __ldcg(rt.act + pr.x);
        const int n_e = __ldcg(rt.counts + e), off_e = __ldcg(rt.offsets + e);
        const int slot0 = off_e + pr.y * kCh;
        const int nt = min(kCh, n_e - pr.y * kCh);
        const uint8_t *row = L.down + ((size_t)e * D + r) * nb * LFM_Q6K_BYTES;
        float sum[kCh];
#pragma unroll
        for (int t = 0; t < kCh; ++t) sum[t] = 0.0f;
        for (uint32_t b0 = 0; b0 < nb; b0 += kSb) {
            const uint32_t ns = min((uint32_t)kSb, nb - b0);
            uint32_t wl[kSb][2], wh[kSb][2], dv[kSb];
            int scv[kSb];
#pragma unroll
            for (int i = 0; i < kSb; ++i) {
                if ((uint32_t)i < ns) {
                    const uint8_t *blk = row + (size_t)(b0 + i) * LFM_Q6K_BYTES;
                    wl[i][0] = ld_u16(blk + 2 * lane);
                    wl[i][1] = ld_u16(blk + 64 + 2 * lane);
                    wh[i][0] = ld_u16(blk + 128 + qh_off);
                    wh[i][1] = ld_u16(blk + 160 + qh_off);
                    scv[i] = lane < 16 ? (int)__ldg(reinterpret_cast<const int8_t *>(blk + 192 + lane)) : 0;
                    dv[i] = ld_u16(blk + 208);
                }
            }
#pragma unroll
            for (int i = 0; i < kSb; ++i) {
                if ((uint32_t)i >= ns) break;
                const uint32_t b = b0 + i;
                /* packed sc*q pairs: P[h][0] = values 2l, 2l+1; P[h][1] = 2l+64, 2l+65 (+128h) */
                int P[2][2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t ql = wl[i][h], qh = wh[i][h];
                    const int s_lo = __shfl_sync(LFM_FULL_MASK, scv[i], 8 * h + (lane >> 3));
                    const int s_hi = __shfl_sync(LFM_FULL_MASK, scv[i], 8 * h + 4 + (lane >> 3));
                    const int sh = 2 * m0;
                    const int q0 = (int)((ql & 15u) | ((qh >> sh) & 3u) << 4);
                    const int q1 = (int)((ql >> 8 & 15u) | ((qh >> (8 + sh)) & 3u) << 4);
                    const int q2 = (int)((ql >> 4 & 15u) | ((qh >> (sh + 4)) & 3u) << 4);
                    const int q3 = (int)((ql >> 12 & 15u) | ((qh >> (12 + sh)) & 3u) << 4);
                    P[h][0] = pack16(q0 * s_lo, q1 * s_lo);
                    P[h][1] = pack16(q2 * s_hi, q3 * s_hi);
                }
                const float dw = lfm_h2f((uint16_t)dv[i]);
#pragma unroll
                for (int t = 0; t < kCh; ++t) {
                    if (t < nt) { /* warp-uniform */
                        const size_t slot = (size_t)(slot0 + t);
                        const uint8_t *q8 = reinterpret_cast<const uint8_t *>(hq.qs + slot * I + (size_t)b * 256);
                        int part = __dp2a_lo(P[0][0], (int)ld_u16(q8 + 2 * lane), 0);
                        part = __dp2a_lo(P[0][1], (int)ld_u16(q8 + 64 + 2 * lane), part);
                        part = __dp2a_lo(P[1][0], (int)ld_u16(q8 + 128 + 2 * lane), part);
                        part = __dp2a_lo(P[1][1], (int)ld_u16(q8 + 192 + 2 * lane), part);
                        if (lane < 16) part -= 32 * scv[i] * (int)__ldg(hq.bs + (slot * nb + b) * 16 + lane);
                        const int total = __reduce_add_sync(LFM_FULL_MASK, part);
                        const float d8 = __ldg(hq.d + slot * nb + b);
                        if (d8 != 0.0f) sum[t] = __fmaf_rn(__fmul_rn(d8, dw), __int2float_rn(total), sum[t]);
                    }
                }
            }
        }
#pragma unroll
        for (int t = 0; t < kCh; ++t)
            if (t < nt && lane == t) y[(size_t)(slot0 + t) * D + r] = sum[t];
    }
}

}  // namespace

cudaError_t lfm_launch_down_q6k(const MoeLayerDev &L, Q8Rows hq, const RouteTables &rt, float *y, int grid,
                                cudaStream_t s) {
    if (!L.down_q6k || L.I % 256) return cudaErrorInvalidValue;
    k_q6k_down<<<grid * 8, kWarps * 32, 0, s>>>(L, hq, rt, y);
    return cudaGetLastError();
}
