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
 * ql[128], qh[64], int8 scales[16], fp16 d.  Lane l of the warp owns, in each
 * half (128 values) of the super-block, the four values l, l+32, l+64, l+96:
 *   q(l)    = ql[l]      & 15 | (qh[l]      & 3) << 4
 *   q(l+32) = ql[l+32]   & 15 | (qh[l] >> 2 & 3) << 4
 *   q(l+64) = ql[l]     >> 4  | (qh[l] >> 4 & 3) << 4
 *   q(l+96) = ql[l+32]  >> 4  | (qh[l] >> 6 & 3) << 4
 * (the reference's unpacking, tools/lfm2_cpuid_quants.c:1509-1512), with the
 * signed scale of sub-block value/16.  So the weight loads of a warp are 32
 * consecutive bytes each, and so are the activation loads of every token.
 *
 * Exact integer part per (token, super-block): each lane's sum of sc*q*q8 over
 * its eight values, lanes 0..15 subtract 32*sc_j*bsums_j, and one warp
 * reduction (redux.sync) gives  total = sum sc*q*q8 - 32*sum sc_j*bsums_j,
 * the reference's integer (:1485, :1531).  fp32 update in the reference's AVX-VNNI
 * order, per super-block in order and skipped where d8 == 0:
 *   sum = fma(d8 * d, (float)total, sum)                          (:1534)
 * Integer bounds: |sc*q*q8| <= 127*63*127 per value, 256 values: < 2^29.
 */
#include "moe_device.cuh"
#include "moe_internal.h"

namespace {

constexpr int kCh = LFM_GEMV_CHUNK; /* tokens per pair (8) */
constexpr int kWarps = 8;

__global__ void __launch_bounds__(kWarps * 32) k_q6k_down(MoeLayerDev L, Q8Rows hq, RouteTables rt, float *y) {
    const uint32_t D = L.D, I = L.I, nb = I / 256;
    const int lane = threadIdx.x & 31;
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
        for (uint32_t b = 0; b < nb; ++b) {
            const uint8_t *blk = row + (size_t)b * LFM_Q6K_BYTES;
            const int8_t *sc = reinterpret_cast<const int8_t *>(blk + 192);
            /* w[h][m]: sc * q of value 128h + 32m + lane */
            int w[2][4];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t a = __ldg(blk + 64 * h + lane), c = __ldg(blk + 64 * h + 32 + lane);
                const uint32_t qh = __ldg(blk + 128 + 32 * h + lane);
                const int s = lane >> 4;
                w[h][0] = (int)((a & 15u) | (qh & 3u) << 4) * (int)__ldg(sc + 8 * h + 0 + s);
                w[h][1] = (int)((c & 15u) | (qh >> 2 & 3u) << 4) * (int)__ldg(sc + 8 * h + 2 + s);
                w[h][2] = (int)((a >> 4) | (qh >> 4 & 3u) << 4) * (int)__ldg(sc + 8 * h + 4 + s);
                w[h][3] = (int)((c >> 4) | (qh >> 6 & 3u) << 4) * (int)__ldg(sc + 8 * h + 6 + s);
            }
            const int scl = lane < 16 ? (int)__ldg(sc + lane) : 0;
            const float dw = lfm_h2f(__ldg(reinterpret_cast<const unsigned short *>(blk + 208)));
#pragma unroll
            for (int t = 0; t < kCh; ++t) {
                if (t < nt) { /* warp-uniform */
                    const size_t slot = (size_t)(slot0 + t);
                    const int8_t *q8 = hq.qs + slot * I + (size_t)b * 256;
                    int part = 0;
#pragma unroll
                    for (int h = 0; h < 2; ++h)
#pragma unroll
                        for (int m = 0; m < 4; ++m) part += w[h][m] * (int)__ldg(q8 + 128 * h + 32 * m + lane);
                    if (lane < 16) part -= 32 * scl * (int)__ldg(hq.bs + (slot * nb + b) * 16 + lane);
                    const int total = __reduce_add_sync(LFM_FULL_MASK, part);
                    const float d8 = __ldg(hq.d + slot * nb + b);
                    if (d8 != 0.0f) sum[t] = __fmaf_rn(__fmul_rn(d8, dw), __int2float_rn(total), sum[t]);
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
