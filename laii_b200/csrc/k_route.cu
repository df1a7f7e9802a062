/*
 * K1 router and K2 dispatch of the lfm2moe MoE-FFN.
 *
 * K1 (k_route): fused RMSNorm -> fp32 router GEMV -> sigmoid -> exp_probs_b
 * biased top-K -> normalised unbiased weights, plus Q8_K of the normalised row.
 * Grid (ceil(E/4), T): each 64-thread block recomputes its token's RMSNorm
 * (8 KB, L2-resident) and scores 4 experts, one per half-warp, so the
 * 256-512 KB router matrix is read by E/4 SMs in parallel instead of one.  The
 * last block to finish a token (arrival counter, no waiting) runs the top-K
 * and the Q8_K quantisation.
 *
 * Evaluation order matches the reference bit for bit:
 *  - sum of squares / router dot: 16 running lanes, each a sequential FMA chain
 *    over elements l, l+16, l+32, ... then the 8/4/2/1 tree
 *    (tools/lfm2_decode_1x4.c:98-113, include/lfm2_simd_avx2.h:676-687);
 *  - inv_rms = 1/sqrtf(ss/D + eps), xb = (x*inv)*w (tools/lfm2_decode_1x4.c:114-133);
 *  - Q8_K: d = max/127, q = RNE(x*(127/max)), bsums of unsaturated codes
 *    (tools/lfm2_decode_1x4.c:150-186);
 *  - top-K: K rounds of argmax with ties to the lowest index, weights are the
 *    unbiased sigmoids normalised by routed_scale/(sum + 1e-20)
 *    (tools/lfm2_moe_checkpoint.c:183-239).
 *  Only exp() can differ (see lfm_expf), which is why parity allows near-ties.
 *
 * K2 (k_dispatch): one block; histogram of the T*K expert ids, exclusive scan,
 * scatter into per-expert contiguous slots (perm) and the inverse map (inv).
 */
#include "moe_device.cuh"
#include "moe_internal.h"

namespace {

constexpr int kRouteThreads = 64;
constexpr int kExpertsPerBlock = 4;

__device__ __forceinline__ void route_topk_and_quant(const MoeLayerDev &L, uint32_t t, const float *xb,
                                                     Q8Rows xq, const RouteTables &rt, const float *logits_t) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t E = L.E, K = L.K;
    if (E > 0 && warp == 0) {
        float sig[8], sel[8];  /* experts lane + 32*i, E <= 256 */
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t e = lane + 32u * i;
            sig[i] = 0.0f;
            sel[i] = -INFINITY;
            if (e < E) {
                const float z = __ldcg(logits_t + e);
                sig[i] = __fdiv_rn(1.0f, __fadd_rn(1.0f, lfm_expf(-z)));
                sel[i] = L.bias ? __fadd_rn(sig[i], L.bias[e]) : sig[i];
            }
        }
        float wk[LFM_GPU_MAX_TOPK_DEV];
        int ik[LFM_GPU_MAX_TOPK_DEV];
        for (uint32_t k = 0; k < K; ++k) {
            float bv = -1e30f;
            int bi = (int)E;  /* sentinel: nothing beat -1e30 */
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t e = lane + 32u * i;
                if (e < E && sel[i] > bv) { bv = sel[i]; bi = (int)e; }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(LFM_FULL_MASK, bv, o);
                const int oi = __shfl_xor_sync(LFM_FULL_MASK, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
            }
            if (bi == (int)E) bi = 0;  /* the reference keeps best_e = 0 */
            ik[k] = bi;
            float s_b = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                if (lane + 32u * i == (uint32_t)bi) { s_b = sig[i]; sel[i] = -1e30f; }
            }
            wk[k] = __shfl_sync(LFM_FULL_MASK, s_b, bi & 31);
        }
        if (L.norm_topk) {
            float s = 0.0f;
            for (uint32_t k = 0; k < K; ++k) s = __fadd_rn(s, wk[k]);
            const float inv = __fdiv_rn(L.routed_scale, __fadd_rn(s, 1e-20f));
            for (uint32_t k = 0; k < K; ++k) wk[k] = __fmul_rn(wk[k], inv);
        } else if (L.routed_scale != 1.0f) {
            for (uint32_t k = 0; k < K; ++k) wk[k] = __fmul_rn(wk[k], L.routed_scale);
        }
        if (lane == 0) {
            for (uint32_t k = 0; k < K; ++k) {
                rt.idx[(size_t)t * K + k] = ik[k];
                rt.w[(size_t)t * K + k] = wk[k];
            }
        }
    }
    /* Q8_K of xb: one warp per 256-element block, 8 elements per lane. */
    const uint32_t nb = L.D / 256;
    for (uint32_t b = warp; b < nb; b += kRouteThreads / 32) {
        const float *src = xb + 256 * b + 8 * lane;
        float v[8];
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) { v[i] = src[i]; amax = fmaxf(amax, fabsf(v[i])); }
        amax = lfm_warp_max(amax);
        int8_t *qdst = xq.qs + (size_t)t * xq.cols + 256 * b + 8 * lane;
        int q[8];
        int part = 0;
        if (amax == 0.0f) {
#pragma unroll
            for (int i = 0; i < 8; ++i) q[i] = 0;
        } else {
            const float s = __fdiv_rn(127.0f, amax);
#pragma unroll
            for (int i = 0; i < 8; ++i) { q[i] = __float2int_rn(__fmul_rn(v[i], s)); part += q[i]; }
        }
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int a = max(-128, min(127, q[i])), c = max(-128, min(127, q[4 + i]));
            lo |= (uint32_t)(uint8_t)(int8_t)a << (8 * i);
            hi |= (uint32_t)(uint8_t)(int8_t)c << (8 * i);
        }
        *reinterpret_cast<uint2 *>(qdst) = make_uint2(lo, hi);
        const int pair = part + __shfl_xor_sync(LFM_FULL_MASK, part, 1);
        if ((lane & 1) == 0) xq.bs[((size_t)t * nb + b) * 16 + (lane >> 1)] = (int16_t)pair;
        if (lane == 0) xq.d[(size_t)t * nb + b] = amax == 0.0f ? 0.0f : __fdiv_rn(amax, 127.0f);
    }
}

__global__ void __launch_bounds__(kRouteThreads) k_route(MoeLayerDev L, const float *__restrict__ x,
                                                         Q8Rows xq, RouteTables rt) {
    extern __shared__ float xb[];  /* [D] */
    __shared__ float s_inv;
    __shared__ int s_last;
    const uint32_t t = blockIdx.y;
    const uint32_t D = L.D;
    const float *xt = x + (size_t)t * D;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

    /* RMSNorm: 16 sequential FMA chains in warp 0, reference tree, then inv. */
    if (warp == 0) {
        float acc = 0.0f;
        if (lane < 16) {
#pragma unroll 8
            for (uint32_t i = 0; i < D; i += 16) {
                const float v = xt[i + lane];
                acc = __fmaf_rn(v, v, acc);
            }
        }
        const float ss = lfm_hsum16_ref(acc);
        if (lane == 0) s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), L.eps)));
    }
    __syncthreads();
    const float inv = s_inv;
    for (uint32_t i = threadIdx.x; i < D; i += kRouteThreads) {
        const float n = __fmul_rn(xt[i], inv);
        xb[i] = L.ffn_norm ? __fmul_rn(n, L.ffn_norm[i]) : n;
    }
    __syncthreads();

    /* Router logits: one expert per half-warp, 16-lane chain + reference tree. */
    if (L.E > 0) {
        const uint32_t e = blockIdx.x * kExpertsPerBlock + warp * 2 + (lane >> 4);
        const uint32_t l16 = lane & 15;
        float acc = 0.0f;
        if (e < L.E) {
            const float *wr = L.router_w + (size_t)e * D;
#pragma unroll 8
            for (uint32_t i = 0; i < D; i += 16) acc = __fmaf_rn(__ldg(wr + i + l16), xb[i + l16], acc);
        }
        const float z = lfm_hsum16_ref(acc);
        if (l16 == 0 && e < L.E) rt.logits[(size_t)t * L.E + e] = z;
        __threadfence();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(&rt.tok_count[t], 1u);
        s_last = prev == gridDim.x - 1;
        if (s_last) rt.tok_count[t] = 0;  /* every other block of this token has arrived */
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    route_topk_and_quant(L, t, xb, xq, rt, rt.logits + (size_t)t * L.E);
}

__global__ void __launch_bounds__(1024) k_dispatch(uint32_t T, uint32_t E, uint32_t K, RouteTables rt) {
    __shared__ int cnt[LFM_GPU_MAX_EXPERTS_DEV];
    __shared__ int off[LFM_GPU_MAX_EXPERTS_DEV + 1];
    __shared__ int cur[LFM_GPU_MAX_EXPERTS_DEV];
    const uint32_t n = T * K;
    for (uint32_t e = threadIdx.x; e < E; e += blockDim.x) { cnt[e] = 0; cur[e] = 0; }
    __syncthreads();
    for (uint32_t a = threadIdx.x; a < n; a += blockDim.x) {
        const int e = rt.idx[a];
        if ((unsigned)e < E) atomicAdd(&cnt[e], 1);
        else atomicOr(rt.err, LFM_DEVERR_EXPERT_ID);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int s = 0, uniq = 0, mx = 0;
        for (uint32_t e = 0; e < E; ++e) {
            off[e] = s;
            s += cnt[e];
            uniq += cnt[e] > 0;
            mx = max(mx, cnt[e]);
        }
        off[E] = s;
        rt.summary[0] = uniq;
        rt.summary[1] = mx;
        rt.summary[2] = s;
        if (rt.loads) { rt.loads[0] += (unsigned long long)uniq; rt.loads[1] += 1ull; }
    }
    __syncthreads();
    for (uint32_t e = threadIdx.x; e <= E; e += blockDim.x) {
        rt.offsets[e] = off[e];
        if (e < E) rt.counts[e] = cnt[e];
    }
    for (uint32_t a = threadIdx.x; a < n; a += blockDim.x) {
        const int e = rt.idx[a];
        if ((unsigned)e < E) {
            const int pos = off[e] + atomicAdd(&cur[e], 1);
            rt.perm[pos] = (int)a;
            rt.inv[a] = pos;
        } else {
            rt.inv[a] = -1;
        }
    }
}

__global__ void k_dense_tables(uint32_t T, RouteTables rt) {
    for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < T; t += gridDim.x * blockDim.x) {
        rt.idx[t] = 0;
        rt.w[t] = 1.0f;
    }
}

}  // namespace

cudaError_t lfm_launch_dense_tables(uint32_t T, const RouteTables &rt, cudaStream_t s) {
    k_dense_tables<<<(T + 255) / 256, 256, 0, s>>>(T, rt);
    return cudaGetLastError();
}

cudaError_t lfm_launch_route(const MoeLayerDev &L, const float *x, uint32_t T, Q8Rows xq, const RouteTables &rt,
                             cudaStream_t s) {
    if (T == 0) return cudaSuccess;
    const uint32_t gx = L.E > 0 ? (L.E + kExpertsPerBlock - 1) / kExpertsPerBlock : 1;
    const size_t smem = sizeof(float) * L.D;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(k_route, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    k_route<<<dim3(gx, T), kRouteThreads, smem, s>>>(L, x, xq, rt);
    return cudaGetLastError();
}

cudaError_t lfm_launch_dispatch(const MoeLayerDev &L, uint32_t T, const RouteTables &rt, cudaStream_t s) {
    k_dispatch<<<1, 1024, 0, s>>>(T, L.E, L.K, rt);
    return cudaGetLastError();
}
