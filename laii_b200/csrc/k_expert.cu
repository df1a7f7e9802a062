/*
 * K3 grouped Q4_K expert GEMVs (decode / verify path) and K4 combine.
 *
 * Work is grouped by expert: block (e, row tile) streams its rows of expert e
 * once and applies them to every token routed to e (in chunks of 8 tokens
 * whose Q8_K activations are staged in shared memory).  One warp computes one
 * weight row: lane 4*bl + g owns 32 bytes of nibbles (group g = sub-blocks 2g
 * and 2g+1) of super-block 8p + bl, loaded as 128-bit streaming loads, and
 * forms the sub-block dots with __dp4a.  The integer super-block sums
 *   acc = sum_j sc_j * dot_j,  mins = sum_j m_j * (bsum_{2j} + bsum_{2j+1})
 * are exact (any summation order), and the fp32 update per super-block is the
 * reference 4-row AVX-VNNI kernel's, in super-block order:
 *   sum = fma(d8*d, acc, fma(-(d8*dmin), mins, sum))
 * (tools/lfm2_cpuid_quants.c:1189-1257; Q4_K x Q8_K math :421-457).
 *
 * gate|up: h = (g / (1 + exp(-g))) * u per (token, expert, row)
 *   (tools/lfm2_decode_1x4.c:976-985), then k_quant_rows makes Q8_K(h) per 256
 *   (tools/lfm2_cpuid_quants.c:584-631).
 * down: y[slot][r] = Down_e[r] . Q8_K(h_slot).
 * combine: x[t][r] = fma(w_k, y[slot(t,k)][r], x[t][r]) for k = 0..K-1 in
 *   order (tools/lfm2_moe_checkpoint.c:266-269, :338-364).
 */
#include "moe_device.cuh"
#include "moe_internal.h"

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kRowsPerBlock = 64;
constexpr int kChunk = 8;  /* tokens per staged activation chunk */

struct ActView {
    const int8_t *qs;    /* [kChunk][cols] */
    const float *d;      /* [kChunk][nb]   */
    const int16_t *bs;   /* [kChunk][nb][16] */
    uint32_t cols, nb;
};

/* Per-warp scratch used to hand the 8 per-super-block integer sums of each
 * token to the lane that runs that token's fp32 chain. */
struct WarpXfer {
    int2 ints[kChunk][8];
    float2 scales[8];
};

struct RowDebug {
    int32_t *sub_dots;  /* [nb][8] for the current (vec,row) or NULL */
    int32_t *acc;       /* [nb] */
    int32_t *mins;      /* [nb] */
};

/* Dot of one Q4_K row with nt (<= kChunk) staged Q8_K activation rows.
 * Returns, in lane t < nt, the fp32 result for token t. */
template <bool kDebug>
__device__ __forceinline__ float q4k_row_dot(const uint8_t *__restrict__ row, const ActView &a, int nt,
                                             WarpXfer &xf, RowDebug dbg) {
    const int lane = threadIdx.x & 31;
    const int bl = lane >> 2, g = lane & 3;
    float sum = 0.0f;
    for (uint32_t p = 0; p * 8 < a.nb; ++p) {
        const uint32_t b = p * 8 + bl;
        const bool valid = b < a.nb;
        uint4 hdr = make_uint4(0, 0, 0, 0), q0 = hdr, q1 = hdr;
        if (valid) {
            const uint8_t *blk = row + (size_t)b * LFM_Q4K_BYTES;
            hdr = lfm_ldg_stream(blk);
            q0 = lfm_ldg_stream(blk + 16 + 32 * g);
            q1 = lfm_ldg_stream(blk + 32 + 32 * g);
        }
        int sc_lo, m_lo, sc_hi, m_hi;
        lfm_q4k_pair_scales(hdr.y, hdr.z, hdr.w, g, sc_lo, m_lo, sc_hi, m_hi);
        const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        if (g == 0 && valid)
            xf.scales[bl] = make_float2(lfm_h2f((uint16_t)(hdr.x & 0xFFFFu)), lfm_h2f((uint16_t)(hdr.x >> 16)));
        for (int t = 0; t < nt; ++t) {
            int acc = 0, mins = 0;
            if (valid) {
                const uint4 *q8 = reinterpret_cast<const uint4 *>(a.qs + (size_t)t * a.cols + 256 * b + 64 * g);
                const uint4 x0 = q8[0], x1 = q8[1], x2 = q8[2], x3 = q8[3];
                const int xl[8] = {(int)x0.x, (int)x0.y, (int)x0.z, (int)x0.w, (int)x1.x, (int)x1.y, (int)x1.z, (int)x1.w};
                const int xh[8] = {(int)x2.x, (int)x2.y, (int)x2.z, (int)x2.w, (int)x3.x, (int)x3.y, (int)x3.z, (int)x3.w};
                int dlo = 0, dhi = 0;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    dlo = __dp4a((int)(w[i] & 0x0F0F0F0Fu), xl[i], dlo);
                    dhi = __dp4a((int)((w[i] >> 4) & 0x0F0F0F0Fu), xh[i], dhi);
                }
                const int16_t *bsp = a.bs + ((size_t)t * a.nb + b) * 16 + 4 * g;
                const uint2 bw = *reinterpret_cast<const uint2 *>(bsp);
                const int b0 = (int)(int16_t)(bw.x & 0xFFFFu), b1 = (int)(int16_t)(bw.x >> 16);
                const int b2 = (int)(int16_t)(bw.y & 0xFFFFu), b3 = (int)(int16_t)(bw.y >> 16);
                acc = sc_lo * dlo + sc_hi * dhi;
                mins = m_lo * (b0 + b1) + m_hi * (b2 + b3);
                if (kDebug && dbg.sub_dots) {
                    dbg.sub_dots[b * 8 + 2 * g] = dlo;
                    dbg.sub_dots[b * 8 + 2 * g + 1] = dhi;
                }
            }
            acc += __shfl_xor_sync(LFM_FULL_MASK, acc, 1);
            acc += __shfl_xor_sync(LFM_FULL_MASK, acc, 2);
            mins += __shfl_xor_sync(LFM_FULL_MASK, mins, 1);
            mins += __shfl_xor_sync(LFM_FULL_MASK, mins, 2);
            if (g == 0 && valid) {
                xf.ints[t][bl] = make_int2(acc, mins);
                if (kDebug && dbg.acc) { dbg.acc[b] = acc; dbg.mins[b] = mins; }
            }
        }
        __syncwarp();
        if (lane < nt) {
            const uint32_t nbl = min(8u, a.nb - p * 8);
            for (uint32_t j = 0; j < nbl; ++j) {
                const uint32_t bb = p * 8 + j;
                const float d8 = a.d[(size_t)lane * a.nb + bb];
                if (d8 == 0.0f) continue;
                const int2 v = xf.ints[lane][j];
                const float2 sc = xf.scales[j];
                const float dd = __fmul_rn(d8, sc.x);
                const float dm = __fmul_rn(d8, sc.y);
                sum = __fmaf_rn(dd, (float)v.x, __fmaf_rn(-dm, (float)v.y, sum));
            }
        }
        __syncwarp();
    }
    return sum;
}

/* Stage the Q8_K rows of nt tokens into shared memory (16-byte copies). */
__device__ void stage_rows(Q8Rows src, const int *rows, int nt, uint32_t nb, int8_t *sqs, float *sd,
                           int16_t *sbs) {
    const uint32_t cols = src.cols;
    const uint32_t qv = cols / 16, bv = nb * 2;  /* uint4 per row: qs, bsums */
    for (uint32_t i = threadIdx.x; i < (uint32_t)nt * qv; i += blockDim.x) {
        const uint32_t t = i / qv, c = i % qv;
        reinterpret_cast<uint4 *>(sqs + (size_t)t * cols)[c] =
            reinterpret_cast<const uint4 *>(src.qs + (size_t)rows[t] * cols)[c];
    }
    for (uint32_t i = threadIdx.x; i < (uint32_t)nt * bv; i += blockDim.x) {
        const uint32_t t = i / bv, c = i % bv;
        reinterpret_cast<uint4 *>(sbs + (size_t)t * nb * 16)[c] =
            reinterpret_cast<const uint4 *>(src.bs + (size_t)rows[t] * nb * 16)[c];
    }
    for (uint32_t i = threadIdx.x; i < (uint32_t)nt * nb; i += blockDim.x) {
        const uint32_t t = i / nb, c = i % nb;
        sd[(size_t)t * nb + c] = src.d[(size_t)rows[t] * nb + c];
    }
}

__host__ __device__ constexpr size_t act_smem_bytes(uint32_t cols) {
    return (size_t)kChunk * cols + (size_t)kChunk * (cols / 256) * 32 + (size_t)kChunk * (cols / 256) * 4;
}

__global__ void __launch_bounds__(kThreads) k_gateup(MoeLayerDev L, Q8Rows xq, RouteTables rt,
                                                     float *__restrict__ h) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ WarpXfer xfer[kWarps];
    __shared__ int tok[kChunk];
    const uint32_t e = blockIdx.x;
    const int n = rt.counts[e];
    if (n == 0) return;
    const int base = rt.offsets[e];
    const uint32_t D = L.D, I = L.I, nb = D / 256;
    const uint32_t r0 = blockIdx.y * kRowsPerBlock;
    const uint32_t r1 = min(I, r0 + kRowsPerBlock);
    int8_t *sqs = reinterpret_cast<int8_t *>(smem);
    int16_t *sbs = reinterpret_cast<int16_t *>(smem + (size_t)kChunk * D);
    float *sd = reinterpret_cast<float *>(smem + (size_t)kChunk * D + (size_t)kChunk * nb * 32);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t row_bytes = (size_t)nb * LFM_Q4K_BYTES;
    const uint8_t *G = L.gate + (size_t)e * I * row_bytes;
    const uint8_t *U = L.up + (size_t)e * I * row_bytes;
    const ActView av{sqs, sd, sbs, D, nb};
    for (int c0 = 0; c0 < n; c0 += kChunk) {
        const int nt = min(kChunk, n - c0);
        __syncthreads();
        if (threadIdx.x < nt) tok[threadIdx.x] = rt.perm[base + c0 + threadIdx.x] / (int)L.K;
        __syncthreads();
        stage_rows(xq, tok, nt, nb, sqs, sd, sbs);
        __syncthreads();
        for (uint32_t r = r0 + warp; r < r1; r += kWarps) {
            const float gv = q4k_row_dot<false>(G + (size_t)r * row_bytes, av, nt, xfer[warp], RowDebug{});
            const float uv = q4k_row_dot<false>(U + (size_t)r * row_bytes, av, nt, xfer[warp], RowDebug{});
            if (lane < nt) {
                const float silu = __fdiv_rn(gv, __fadd_rn(1.0f, lfm_expf(-gv)));
                h[(size_t)(base + c0 + lane) * I + r] = __fmul_rn(silu, uv);
            }
        }
    }
}

__global__ void __launch_bounds__(kThreads) k_down(MoeLayerDev L, Q8Rows hq, RouteTables rt,
                                                   float *__restrict__ y) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ WarpXfer xfer[kWarps];
    __shared__ int slot[kChunk];
    const uint32_t e = blockIdx.x;
    const int n = rt.counts[e];
    if (n == 0) return;
    const int base = rt.offsets[e];
    const uint32_t D = L.D, I = L.I, nb = I / 256;
    const uint32_t r0 = blockIdx.y * kRowsPerBlock;
    const uint32_t r1 = min(D, r0 + kRowsPerBlock);
    int8_t *sqs = reinterpret_cast<int8_t *>(smem);
    int16_t *sbs = reinterpret_cast<int16_t *>(smem + (size_t)kChunk * I);
    float *sd = reinterpret_cast<float *>(smem + (size_t)kChunk * I + (size_t)kChunk * nb * 32);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t row_bytes = (size_t)nb * LFM_Q4K_BYTES;
    const uint8_t *W = L.down + (size_t)e * D * row_bytes;
    const ActView av{sqs, sd, sbs, I, nb};
    for (int c0 = 0; c0 < n; c0 += kChunk) {
        const int nt = min(kChunk, n - c0);
        __syncthreads();
        if (threadIdx.x < nt) slot[threadIdx.x] = base + c0 + threadIdx.x;
        __syncthreads();
        stage_rows(hq, slot, nt, nb, sqs, sd, sbs);
        __syncthreads();
        for (uint32_t r = r0 + warp; r < r1; r += kWarps) {
            const float v = q4k_row_dot<false>(W + (size_t)r * row_bytes, av, nt, xfer[warp], RowDebug{});
            if (lane < nt) y[(size_t)(base + c0 + lane) * D + r] = v;
        }
    }
}

/* Q8_K of fp32 rows: one warp per 256-element block, 8 elements per lane
 * (d = max/127, q = RNE(x*(127/max)), bsums of unsaturated codes). */
__global__ void __launch_bounds__(kThreads) k_quant_rows(const float *__restrict__ src, uint32_t rows,
                                                         uint32_t cols, Q8Rows dst) {
    const uint32_t nb = cols / 256;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t gw = blockIdx.x * kWarps + warp;
    if (gw >= rows * nb) return;
    const uint32_t r = gw / nb, b = gw % nb;
    const float4 *p = reinterpret_cast<const float4 *>(src + (size_t)r * cols + 256 * b + 8 * lane);
    const float4 a0 = p[0], a1 = p[1];
    const float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
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
    *reinterpret_cast<uint2 *>(dst.qs + (size_t)r * cols + 256 * b + 8 * lane) = make_uint2(lo, hi);
    const int pair = part + __shfl_xor_sync(LFM_FULL_MASK, part, 1);
    if ((lane & 1) == 0) dst.bs[((size_t)r * nb + b) * 16 + (lane >> 1)] = (int16_t)pair;
    if (lane == 0) dst.d[(size_t)r * nb + b] = amax == 0.0f ? 0.0f : __fdiv_rn(amax, 127.0f);
}

__global__ void __launch_bounds__(256) k_combine(float *__restrict__ x, uint32_t D, uint32_t K, RouteTables rt,
                                                 const float *__restrict__ y) {
    const uint32_t t = blockIdx.x;
    __shared__ int s_slot[LFM_GPU_MAX_TOPK_DEV];
    __shared__ float s_w[LFM_GPU_MAX_TOPK_DEV];
    if (threadIdx.x < K) {
        s_slot[threadIdx.x] = rt.inv[(size_t)t * K + threadIdx.x];
        s_w[threadIdx.x] = rt.w[(size_t)t * K + threadIdx.x];
    }
    __syncthreads();
    float *xt = x + (size_t)t * D;
    for (uint32_t r = threadIdx.x; r < D; r += blockDim.x) {
        float v = xt[r];
        for (uint32_t k = 0; k < K; ++k) {
            const int s = s_slot[k];
            if (s >= 0) v = __fmaf_rn(s_w[k], y[(size_t)s * D + r], v);
        }
        xt[r] = v;
    }
}

/* Debug: every (vector, row) pair through q4k_row_dot with its integer parts. */
__global__ void __launch_bounds__(kThreads) k_debug_rows(const uint8_t *__restrict__ w, uint32_t n_rows,
                                                         uint32_t n_cols, Q8Rows xq, uint32_t n_vec,
                                                         int32_t *sub_dots, int32_t *acc, int32_t *mins,
                                                         float *rows_out) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ WarpXfer xfer[kWarps];
    __shared__ int vrow[1];
    const uint32_t nb = n_cols / 256;
    const uint32_t v = blockIdx.x;
    int8_t *sqs = reinterpret_cast<int8_t *>(smem);
    int16_t *sbs = reinterpret_cast<int16_t *>(smem + (size_t)kChunk * n_cols);
    float *sd = reinterpret_cast<float *>(smem + (size_t)kChunk * n_cols + (size_t)kChunk * nb * 32);
    if (threadIdx.x == 0) vrow[0] = (int)v;
    __syncthreads();
    stage_rows(xq, vrow, 1, nb, sqs, sd, sbs);
    __syncthreads();
    const ActView av{sqs, sd, sbs, n_cols, nb};
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t row_bytes = (size_t)nb * LFM_Q4K_BYTES;
    for (uint32_t r = blockIdx.y * kWarps + warp; r < n_rows; r += gridDim.y * kWarps) {
        const size_t o = (size_t)v * n_rows + r;
        RowDebug dbg{sub_dots + o * nb * 8, acc + o * nb, mins + o * nb};
        const float s = q4k_row_dot<true>(w + r * row_bytes, av, 1, xfer[warp], dbg);
        if (lane == 0) rows_out[o] = s;
    }
}

/* Internal Q8 rows <-> 292-byte GGUF block_q8_K. */
__global__ void k_q8_to_gguf(Q8Rows q, uint32_t rows, uint8_t *out) {
    const uint32_t nb = q.cols / 256;
    const uint32_t blk = blockIdx.x;
    if (blk >= rows * nb) return;
    const uint32_t r = blk / nb, b = blk % nb;
    uint8_t *o = out + (size_t)blk * LFM_Q8K_BYTES;
    for (uint32_t i = threadIdx.x; i < 256; i += blockDim.x) o[4 + i] = (uint8_t)q.qs[(size_t)r * q.cols + 256 * b + i];
    if (threadIdx.x < 16) {
        const int16_t v = q.bs[((size_t)r * nb + b) * 16 + threadIdx.x];
        memcpy(o + 260 + 2 * threadIdx.x, &v, 2);
    }
    if (threadIdx.x == 0) {
        const float d = q.d[(size_t)r * nb + b];
        memcpy(o, &d, 4);
    }
}

__global__ void k_gguf_to_q8(const uint8_t *in, uint32_t rows, Q8Rows q) {
    const uint32_t nb = q.cols / 256;
    const uint32_t blk = blockIdx.x;
    if (blk >= rows * nb) return;
    const uint32_t r = blk / nb, b = blk % nb;
    const uint8_t *s = in + (size_t)blk * LFM_Q8K_BYTES;
    for (uint32_t i = threadIdx.x; i < 256; i += blockDim.x) q.qs[(size_t)r * q.cols + 256 * b + i] = (int8_t)s[4 + i];
    if (threadIdx.x < 16) {
        int16_t v;
        memcpy(&v, s + 260 + 2 * threadIdx.x, 2);
        q.bs[((size_t)r * nb + b) * 16 + threadIdx.x] = v;
    }
    if (threadIdx.x == 0) {
        float d;
        memcpy(&d, s, 4);
        q.d[(size_t)r * nb + b] = d;
    }
}

cudaError_t set_smem(const void *fn, size_t bytes) {
    if (bytes <= 48 * 1024) return cudaSuccess;
    return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

}  // namespace

cudaError_t lfm_launch_gateup(const MoeLayerDev &L, uint32_t T, Q8Rows xq, const RouteTables &rt, float *h,
                              cudaStream_t s) {
    (void)T;
    const size_t smem = act_smem_bytes(L.D);
    cudaError_t e = set_smem((const void *)k_gateup, smem);
    if (e != cudaSuccess) return e;
    const dim3 grid(L.E, (L.I + kRowsPerBlock - 1) / kRowsPerBlock);
    k_gateup<<<grid, kThreads, smem, s>>>(L, xq, rt, h);
    return cudaGetLastError();
}

cudaError_t lfm_launch_quant_rows(const float *h, uint32_t rows, uint32_t cols, Q8Rows hq, cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    const uint32_t warps = rows * (cols / 256);
    k_quant_rows<<<(warps + kWarps - 1) / kWarps, kThreads, 0, s>>>(h, rows, cols, hq);
    return cudaGetLastError();
}

cudaError_t lfm_launch_down(const MoeLayerDev &L, uint32_t T, Q8Rows hq, const RouteTables &rt, float *y,
                            cudaStream_t s) {
    (void)T;
    const size_t smem = act_smem_bytes(L.I);
    cudaError_t e = set_smem((const void *)k_down, smem);
    if (e != cudaSuccess) return e;
    const dim3 grid(L.E, (L.D + kRowsPerBlock - 1) / kRowsPerBlock);
    k_down<<<grid, kThreads, smem, s>>>(L, hq, rt, y);
    return cudaGetLastError();
}

cudaError_t lfm_launch_combine(const MoeLayerDev &L, float *x, uint32_t T, const RouteTables &rt, const float *y,
                               cudaStream_t s) {
    if (T == 0) return cudaSuccess;
    k_combine<<<T, 256, 0, s>>>(x, L.D, L.K, rt, y);
    return cudaGetLastError();
}

cudaError_t lfm_launch_debug_q4k_rows(const uint8_t *w, uint32_t n_rows, uint32_t n_cols, Q8Rows xq,
                                      uint32_t n_vec, int32_t *sub_dots, int32_t *acc, int32_t *mins,
                                      float *rows_out, cudaStream_t s) {
    const size_t smem = act_smem_bytes(n_cols);
    cudaError_t e = set_smem((const void *)k_debug_rows, smem);
    if (e != cudaSuccess) return e;
    const uint32_t gy = min(64u, (n_rows + kWarps - 1) / kWarps);
    k_debug_rows<<<dim3(n_vec, gy), kThreads, smem, s>>>(w, n_rows, n_cols, xq, n_vec, sub_dots, acc, mins, rows_out);
    return cudaGetLastError();
}

cudaError_t lfm_launch_q8_to_gguf(Q8Rows q, uint32_t rows, uint8_t *out, cudaStream_t s) {
    const uint32_t n = rows * (q.cols / 256);
    if (n == 0) return cudaSuccess;
    k_q8_to_gguf<<<n, 128, 0, s>>>(q, rows, out);
    return cudaGetLastError();
}

cudaError_t lfm_launch_gguf_to_q8(const uint8_t *in, uint32_t rows, Q8Rows q, cudaStream_t s) {
    const uint32_t n = rows * (q.cols / 256);
    if (n == 0) return cudaSuccess;
    k_gguf_to_q8<<<n, 128, 0, s>>>(in, rows, q);
    return cudaGetLastError();
}
