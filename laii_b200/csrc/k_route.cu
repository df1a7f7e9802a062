/*
 * K1 router (+ K2 dispatch) of the lfm2moe MoE-FFN.
 *
 * k_route, grid (ceil(E/4), T), 64 threads: block (bx, t) scores experts
 * 4*bx .. 4*bx+3 for token t.
 *  1. Bulk (TMA) copies bring the block's 4 router rows (32 KB at D=2048) and
 *     ffn_norm into shared memory; they are issued before griddepcontrol.wait,
 *     so they overlap the tail of the kernel that produces x.  Another bulk
 *     copy brings x[t] once that kernel has finished.
 *  2. RMSNorm with the reference's evaluation order: 16 sequential FMA chains
 *     over elements l, l+16, ... then the 8/4/2/1 tree, inv = 1/sqrtf(ss/D+eps),
 *     xb = (x*inv)*w   (tools/lfm2_decode_1x4.c:98-133).
 *  3. Router logits, one expert per half-warp with the same 16-chain order
 *     as lfm2_vec_dot_f32_avx2 (include/lfm2_simd_avx2.h:676-687).
 *  4. The last block of token t (arrival counter; nobody waits) computes
 *     sigmoid, exp_probs_b-biased top-K (ties to the lowest index) and the
 *     normalised unbiased weights (tools/lfm2_moe_checkpoint.c:183-239), and
 *     Q8_K of xb (tools/lfm2_decode_1x4.c:150-186).
 *  5. The last token to finish (second counter) builds the dispatch tables:
 *     per-expert histogram, exclusive scan, slot permutation and its inverse,
 *     the list of active experts and of (expert, 8-token chunk) work pairs.
 * Dense layers skip 3-4 and route every token to expert 0 with weight 1
 * (x + down(x) exactly, tools/lfm2_decode_1x4.c:1086-1103).
 * Only exp() can differ from the reference (see lfm_expf): routing parity
 * allows near-ties.
 */
#include <cooperative_groups.h>

#include "moe_device.cuh"
#include "moe_internal.h"

namespace cg = cooperative_groups;

namespace {

constexpr int kRouteThreads = 64;
constexpr int kExpertsPerBlock = 4;

struct RouteSmem {
    uint64_t bar_w, bar_x;
    float inv;
    int last;
    int cnt[LFM_GPU_MAX_EXPERTS_DEV];
    int off[LFM_GPU_MAX_EXPERTS_DEV + 1];
    int cur[LFM_GPU_MAX_EXPERTS_DEV];
};

__device__ void route_dispatch(const MoeLayerDev &L, uint32_t T, const RouteTables &rt, RouteSmem &s) {
    const uint32_t E = L.dense ? 1u : L.E, K = L.dense ? 1u : L.K;
    const uint32_t n = T * K;
    for (uint32_t e = threadIdx.x; e < E; e += blockDim.x) { s.cnt[e] = 0; s.cur[e] = 0; }
    __syncthreads();
    for (uint32_t a = threadIdx.x; a < n; a += blockDim.x) {
        const int e = __ldcg(rt.idx + a);
        if ((unsigned)e < E) atomicAdd(&s.cnt[e], 1);
        else atomicOr(rt.err, LFM_DEVERR_EXPERT_ID);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int acc = 0, uniq = 0, mx = 0, pairs = 0;
        for (uint32_t e = 0; e < E; ++e) {
            s.off[e] = acc;
            acc += s.cnt[e];
            mx = max(mx, s.cnt[e]);
            if (s.cnt[e] > 0) {
                rt.act[uniq] = (int)e;
                const int nch = (s.cnt[e] + LFM_GEMV_CHUNK - 1) / LFM_GEMV_CHUNK;
                for (int c = 0; c < nch; ++c) rt.pairs[pairs + c] = make_int2(uniq, c);
                pairs += nch;
                ++uniq;
            }
        }
        s.off[E] = acc;
        rt.summary[0] = uniq;
        rt.summary[1] = mx;
        rt.summary[2] = acc;
        rt.summary[3] = pairs;
        if (rt.loads && !L.dense) { rt.loads[0] += (unsigned long long)uniq; rt.loads[1] += 1ull; }
    }
    __syncthreads();
    for (uint32_t e = threadIdx.x; e <= E; e += blockDim.x) {
        rt.offsets[e] = s.off[e];
        if (e < E) rt.counts[e] = s.cnt[e];
    }
    for (uint32_t a = threadIdx.x; a < n; a += blockDim.x) {
        const int e = __ldcg(rt.idx + a);
        if ((unsigned)e < E) {
            const int pos = s.off[e] + atomicAdd(&s.cur[e], 1);
            rt.perm[pos] = (int)a;
            rt.inv[a] = pos;
        } else {
            rt.inv[a] = -1;
        }
    }
}

/* Top-K of token t from its E logits (global memory written by other blocks,
 * read through L2; or this block's shared memory). */
__device__ void route_topk(const MoeLayerDev &L, uint32_t t, const RouteTables &rt, const float *logits_t,
                           bool global_logits) {
    const int lane = threadIdx.x & 31;
    const uint32_t E = L.E, K = L.K;
    float sig[8], sel[8]; /* experts lane + 32*i, E <= 256 */
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t e = lane + 32u * i;
        sig[i] = 0.0f;
        sel[i] = -INFINITY;
        if (e < E) {
            const float z = global_logits ? __ldcg(logits_t + e) : logits_t[e];
            sig[i] = __fdiv_rn(1.0f, __fadd_rn(1.0f, lfm_expf(-z)));
            sel[i] = L.bias ? __fadd_rn(sig[i], L.bias[e]) : sig[i];
        }
    }
    float wk[LFM_GPU_MAX_TOPK_DEV];
    int ik[LFM_GPU_MAX_TOPK_DEV];
    for (uint32_t k = 0; k < K; ++k) {
        float bv = -1e30f;
        int bi = (int)E; /* sentinel: nothing beat -1e30 */
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
        if (bi == (int)E) bi = 0; /* the reference keeps best_e = 0 */
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

__global__ void __launch_bounds__(kRouteThreads) k_route(MoeLayerDev L, const float *__restrict__ x, uint32_t T,
                                                         Q8Rows xq, RouteTables rt) {
    extern __shared__ __align__(128) uint8_t dsm[];
    __shared__ RouteSmem s;
    const uint32_t t = blockIdx.y, D = L.D;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float *xs = reinterpret_cast<float *>(dsm); /* [D] raw x, then xb */
    float *nw = xs + D;                         /* [D] ffn_norm        */
    float *ws = nw + D;                         /* [4][D] router rows  */
    const uint32_t e0 = blockIdx.x * kExpertsPerBlock;
    const uint32_t ne = L.dense ? 0u : min((uint32_t)kExpertsPerBlock, L.E - e0);
    const uint32_t w_bytes = (ne + (L.ffn_norm ? 1u : 0u)) * D * 4;

    if (threadIdx.x == 0) {
        lfm_mbar_init(&s.bar_w, 1);
        lfm_mbar_init(&s.bar_x, 1);
        lfm_fence_mbar_init();
    }
    __syncthreads();
    lfm_pdl_launch_dependents();
    /* constant weights: fetch before waiting on the producer of x */
    if (threadIdx.x == 0 && w_bytes > 0) {
        lfm_mbar_arrive_tx(&s.bar_w, w_bytes);
        if (ne > 0) lfm_bulk_g2s_plain(ws, L.router_w + (size_t)e0 * D, ne * D * 4, &s.bar_w);
        if (L.ffn_norm) lfm_bulk_g2s_plain(nw, L.ffn_norm, D * 4, &s.bar_w);
    }
    lfm_pdl_wait(); /* x is produced by the previous kernel on the stream */
    if (threadIdx.x == 0) {
        lfm_mbar_arrive_tx(&s.bar_x, D * 4);
        lfm_bulk_g2s_plain(xs, x + (size_t)t * D, D * 4, &s.bar_x);
    }
    const bool ok_x = lfm_mbar_wait(&s.bar_x, 0, rt.err);

    if (warp == 0) {
        float acc = 0.0f;
        if (lane < 16 && ok_x) {
#pragma unroll 16
            for (uint32_t i = 0; i < D; i += 16) {
                const float v = xs[i + lane];
                acc = __fmaf_rn(v, v, acc);
            }
        }
        const float ss = lfm_hsum16_ref(acc);
        if (lane == 0) s.inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), L.eps)));
    }
    const bool ok_w = w_bytes == 0 || lfm_mbar_wait(&s.bar_w, 0, rt.err);
    __syncthreads();
    const float inv = s.inv;
    for (uint32_t i = threadIdx.x; i < D; i += kRouteThreads) {
        const float n = __fmul_rn(xs[i], inv);
        xs[i] = L.ffn_norm ? __fmul_rn(n, nw[i]) : n;
    }
    __syncthreads();

    if (ne > 0) {
        const uint32_t el = warp * 2 + (lane >> 4), l16 = lane & 15;
        float acc = 0.0f;
        if (el < ne && ok_w) {
            const float *wr = ws + (size_t)el * D;
#pragma unroll 16
            for (uint32_t i = 0; i < D; i += 16) acc = __fmaf_rn(wr[i + l16], xs[i + l16], acc);
        }
        const float z = lfm_hsum16_ref(acc);
        if (l16 == 0 && el < ne) rt.logits[(size_t)t * L.E + e0 + el] = z;
        __threadfence();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(&rt.tok_count[t], 1u);
        s.last = prev == gridDim.x - 1;
        if (s.last) rt.tok_count[t] = 0; /* every other block of this token has arrived */
    }
    __syncthreads();
    if (!s.last) return;
    __threadfence();

    if (L.dense) {
        if (threadIdx.x == 0) { rt.idx[t] = 0; rt.w[t] = 1.0f; }
    } else if (warp == 0) {
        route_topk(L, t, rt, rt.logits + (size_t)t * L.E, true);
    }
    const uint32_t nb = D / 256;
    for (uint32_t b = warp; b < nb; b += kRouteThreads / 32) {
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = xs[256 * b + 8 * lane + i];
        lfm_quant_block_warp(v, xq, t, b);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(rt.done, 1u);
        s.last = prev == T - 1;
        if (s.last) *rt.done = 0;
    }
    __syncthreads();
    if (!s.last) return;
    __threadfence();
    route_dispatch(L, T, rt, s);
}

/*
 * Decode-size router (T <= 16): one thread-block cluster of C <= 8 CTAs.
 * CTA c scores experts [c*epc, c*epc + epc) for every token (router rows and
 * ffn_norm bulk-copied before griddepcontrol.wait, x after it), computes each
 * token's RMSNorm itself, and writes its logits straight into CTA 0's shared
 * memory (distributed shared memory).  One cluster barrier later CTA 0 runs
 * top-K, Q8_K and the dispatch for all tokens: no global atomics or fences on
 * the critical path.  Same evaluation order as k_route.
 */
constexpr int kClusterThreads = 512;
constexpr int kClusterMaxT = 16;

__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_sync_release_acquire() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__global__ void __launch_bounds__(kClusterThreads) k_route_cluster(MoeLayerDev L, const float *__restrict__ x,
                                                                   uint32_t T, uint32_t epc, Q8Rows xq,
                                                                   RouteTables rt) {
    extern __shared__ __align__(128) uint8_t dsm[];
    __shared__ RouteSmem s;
    __shared__ float s_inv[kClusterMaxT];
    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t c = cluster.block_rank();
    const uint32_t D = L.D, E = L.E;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int hw = threadIdx.x >> 4, l16 = threadIdx.x & 15; /* half-warp */
    float *xs = reinterpret_cast<float *>(dsm);   /* [T][D] x, then xb */
    float *nw = xs + (size_t)T * D;               /* [D] ffn_norm      */
    float *ws = nw + D;                           /* [epc][D] router rows */
    float *lg = ws + (size_t)epc * D;             /* [T][E] logits (used in CTA 0) */
    const uint32_t e0 = c * epc;
    const uint32_t ne = e0 < E ? min(epc, E - e0) : 0u;
    const uint32_t w_bytes = (ne + (L.ffn_norm ? 1u : 0u)) * D * 4;

    if (threadIdx.x == 0) {
        lfm_mbar_init(&s.bar_w, 1);
        lfm_mbar_init(&s.bar_x, 1);
        lfm_fence_mbar_init();
    }
    cluster_arrive_relaxed(); /* every CTA of the cluster has started (for the DSMEM writes below) */
    __syncthreads();
    lfm_pdl_launch_dependents();
    if (threadIdx.x == 0 && w_bytes > 0) {
        lfm_mbar_arrive_tx(&s.bar_w, w_bytes);
        if (ne > 0) lfm_bulk_g2s_plain(ws, L.router_w + (size_t)e0 * D, ne * D * 4, &s.bar_w);
        if (L.ffn_norm) lfm_bulk_g2s_plain(nw, L.ffn_norm, D * 4, &s.bar_w);
    }
    lfm_pdl_wait();
    if (threadIdx.x == 0) {
        lfm_mbar_arrive_tx(&s.bar_x, T * D * 4);
        lfm_bulk_g2s_plain(xs, x, T * D * 4, &s.bar_x);
    }
    const bool ok_x = lfm_mbar_wait(&s.bar_x, 0, rt.err);
    /* RMSNorm sum of squares: one half-warp per token */
    {
        float acc = 0.0f;
        if (hw < (int)T && ok_x) {
            const float *xt = xs + (size_t)hw * D;
#pragma unroll 16
            for (uint32_t i = 0; i < D; i += 16) acc = __fmaf_rn(xt[i + l16], xt[i + l16], acc);
        }
        const float ss = lfm_hsum16_ref(acc);
        if (l16 == 0 && hw < (int)T)
            s_inv[hw] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), L.eps)));
    }
    const bool ok_w = w_bytes == 0 || lfm_mbar_wait(&s.bar_w, 0, rt.err);
    __syncthreads();
    for (uint32_t q = threadIdx.x; q < T * D; q += kClusterThreads) {
        const uint32_t t = q / D, i = q % D;
        const float n = __fmul_rn(xs[q], s_inv[t]);
        xs[q] = L.ffn_norm ? __fmul_rn(n, nw[i]) : n;
    }
    __syncthreads();
    cluster_wait();
    /* logits for (expert, token) pairs, one half-warp each, written into CTA 0 */
    float *lg0 = cluster.map_shared_rank(lg, 0);
    /* warp-uniform trip count: both half-warps of a warp reach the shuffles together */
    for (uint32_t base = 2u * warp; base < ne * T; base += kClusterThreads / 16) {
        const uint32_t p = base + (uint32_t)(hw & 1);
        const bool valid = p < ne * T;
        const uint32_t el = valid ? p / T : 0u, t = valid ? p % T : 0u;
        float acc = 0.0f;
        if (ok_w && valid) {
            const float *wr = ws + (size_t)el * D, *xt = xs + (size_t)t * D;
#pragma unroll 16
            for (uint32_t i = 0; i < D; i += 16) acc = __fmaf_rn(wr[i + l16], xt[i + l16], acc);
        }
        const float z = lfm_hsum16_ref(acc);
        if (l16 == 0 && valid) lg0[(size_t)t * E + e0 + el] = z;
    }
    cluster_sync_release_acquire();
    if (c != 0) return;

    for (uint32_t t = warp; t < T; t += kClusterThreads / 32) route_topk(L, t, rt, lg + (size_t)t * E, false);
    const uint32_t nb = D / 256;
    for (uint32_t q = warp; q < T * nb; q += kClusterThreads / 32) {
        const uint32_t t = q / nb, b = q % nb;
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = xs[(size_t)t * D + 256 * b + 8 * lane + i];
        lfm_quant_block_warp(v, xq, t, b);
    }
    if (rt.logits) /* keep the logits observable like the multi-block path does */
        for (uint32_t q = threadIdx.x; q < T * E; q += kClusterThreads) rt.logits[q] = lg[q];
    __syncthreads();
    route_dispatch(L, T, rt, s);
}

/* Dispatch tables alone, for rows whose experts are given (expert parallelism). */
__global__ void __launch_bounds__(256) k_dispatch_only(MoeLayerDev L, uint32_t T, RouteTables rt) {
    __shared__ RouteSmem s;
    route_dispatch(L, T, rt, s);
}

}  // namespace

cudaError_t lfm_launch_dispatch(const MoeLayerDev &L, uint32_t T, const RouteTables &rt, cudaStream_t s) {
    if (T == 0) return cudaSuccess;
    k_dispatch_only<<<1, 256, 0, s>>>(L, T, rt);
    return cudaGetLastError();
}

size_t lfm_route_smem(uint32_t D) { return sizeof(float) * D * (2 + kExpertsPerBlock); }

/* Shared memory of the cluster router, or 0 when (T, D, E) does not fit it. */
static size_t route_cluster_smem(const MoeLayerDev &L, uint32_t T, uint32_t *epc_out) {
    if (L.dense || T == 0 || T > kClusterMaxT || L.E == 0) return 0;
    const uint32_t epc = (L.E + 7) / 8;
    const size_t bytes = sizeof(float) * ((size_t)T * L.D + L.D + (size_t)epc * L.D + (size_t)T * L.E);
    if (bytes > 200 * 1024) return 0;
    *epc_out = epc;
    return bytes;
}

cudaError_t lfm_launch_route(const MoeLayerDev &L, const float *x, uint32_t T, Q8Rows xq, const RouteTables &rt,
                             cudaStream_t s, bool pdl) {
    if (T == 0) return cudaSuccess;
    uint32_t epc = 0;
    const size_t csmem = route_cluster_smem(L, T, &epc);
    if (csmem > 0) {
        static size_t cache[16];
        cudaError_t e = lfm_smem_attr((const void *)k_route_cluster, csmem, cache);
        if (e != cudaSuccess) return e;
        const uint32_t C = (L.E + epc - 1) / epc;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(C);
        cfg.blockDim = dim3(kClusterThreads);
        cfg.dynamicSmemBytes = csmem;
        cfg.stream = s;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = C;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 2;
        return cudaLaunchKernelEx(&cfg, k_route_cluster, L, x, T, epc, xq, rt);
    }
    const uint32_t gx = L.dense ? 1u : (L.E + kExpertsPerBlock - 1) / kExpertsPerBlock;
    static size_t cache[16];
    const size_t smem = lfm_route_smem(L.D);
    cudaError_t e = lfm_smem_attr((const void *)k_route, smem, cache);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(gx, T);
    cfg.blockDim = dim3(kRouteThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_route, L, x, T, xq, rt);
}
