/*
 * K1 router (+ K2 dispatch) of the lfm2moe MoE-FFN.
 *
 * Evaluation order (the reference's, so Q8_K of x is bit-exact and only exp()
 * can move a logit by an ulp):
 *   RMSNorm: 16 sequential FMA chains over elements l, l+16, ... then the
 *     8/4/2/1 tree, inv = 1/sqrtf(ss/D+eps), xb = (x*inv)*w
 *     (tools/lfm2_decode_1x4.c:98-133);
 *   logits: the same 16-chain order as lfm2_vec_dot_f32_avx2
 *     (include/lfm2_simd_avx2.h:676-687);
 *   sigmoid, exp_probs_b-biased top-K (ties to the lowest index), normalised
 *     unbiased weights (tools/lfm2_moe_checkpoint.c:183-239);
 *   Q8_K of xb (tools/lfm2_decode_1x4.c:150-186).
 * Three implementations by size:
 *   T <= 16        k_route_cluster, one thread-block cluster (below);
 *   16 < T <= 256  k_route_dec, one launch (4 tokens x 8 experts a CTA);
 *   above          k_norm_q8 + k_router_tiles + the dispatch launches.
 * Dispatch tables (route_dispatch): per-expert histogram, exclusive scan,
 * slot permutation and its inverse, the active experts and their (expert,
 * 8-token chunk) work pairs.  Dense layers route every token to expert 0 with
 * weight 1 (x + down(x) exactly, tools/lfm2_decode_1x4.c:1086-1103).
 */
#include <cooperative_groups.h>

#include "moe_device.cuh"
#include "moe_internal.h"

namespace cg = cooperative_groups;

namespace {

struct RouteSmem {
    uint64_t bar_w, bar_x;
    float inv;
    int last;
    int cnt[LFM_GPU_MAX_EXPERTS_DEV];
    int off[LFM_GPU_MAX_EXPERTS_DEV + 1];
    int cur[LFM_GPU_MAX_EXPERTS_DEV];
    int act[LFM_GPU_MAX_EXPERTS_DEV]; /* active experts, in id order */
    int pb[LFM_GPU_MAX_EXPERTS_DEV];  /* first work pair of each active expert */
    int tbb[LFM_GPU_MAX_EXPERTS_DEV + 1]; /* first token block of each active expert (tcgen05 plan) */
    int uniq, bad;
    int wsum[32][4]; /* block scans: per-warp sums, then their exclusive prefixes */
    int tot[4];      /* block scans: totals */
};

/* Inclusive sum over the warp (every lane gets its own prefix). */
__device__ __forceinline__ int warp_incl_scan(int v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(LFM_FULL_MASK, v, o);
        if (lane >= o) v += u;
    }
    return v;
}

/* Exclusive scans over the block of three per-thread counts (thread order),
 * and the block's largest v[3]; every thread of the block calls it.  Totals in
 * s.tot[0..2], the maximum in s.tot[3]. */
__device__ __forceinline__ void block_scan3(const int (&v)[4], int (&ex)[3], RouteSmem &s) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (int)(blockDim.x >> 5);
    int in[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) in[j] = warp_incl_scan(v[j]);
    const int mx = __reduce_max_sync(LFM_FULL_MASK, v[3]);
    if (lane == 31) {
#pragma unroll
        for (int j = 0; j < 3; ++j) s.wsum[warp][j] = in[j];
        s.wsum[warp][3] = mx;
    }
    __syncthreads();
    if (warp == 0) {
        int w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = lane < nw ? s.wsum[lane][j] : 0;
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            const int iw = warp_incl_scan(w[j]);
            if (lane < nw) s.wsum[lane][j] = iw - w[j];
            if (lane == 31) s.tot[j] = iw;
        }
        const int m = __reduce_max_sync(LFM_FULL_MASK, w[3]);
        if (lane == 0) s.tot[3] = m;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < 3; ++j) ex[j] = s.wsum[warp][j] + in[j] - v[j];
}

/* The tcgen05 GEMMs' tile plans from the counts just formed (token blocks of
 * <= nt slots per active expert; tiles with the token blocks fastest, so the
 * CTAs that share a weight block run together and share it through L2).
 * Thread u scans the token blocks of active expert u (blockDim.x >= E); warp w
 * then writes the tiles of experts w, w + 8, ..., lane l those of row block l,
 * with no division while an expert has at most kPlanDirect token blocks. */
constexpr int kPlanDirect = 8;
__device__ void route_plan(const RouteTables &rt, RouteSmem &s) {
    const UmmaPlanOut &P = rt.plan;
    const int nt = (int)P.nt, nrg = (int)P.rows_gu / 128, nrd = (int)P.rows_dn / 128;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    __syncthreads();
    const int U = s.uniq;
    {
        const int u = (int)threadIdx.x;
        const int v[4] = {u < U ? (s.cnt[s.act[u]] + nt - 1) / nt : 0, 0, 0, 0};
        int ex[3];
        block_scan3(v, ex, s);
        if (u < U) s.tbb[u] = ex[0];
        if (threadIdx.x == 0) {
            const int tot = s.tot[0];
            s.tbb[U] = tot;
            s.bad = (uint32_t)tot > P.max_tb || (uint32_t)(2 * tot * nrg) > P.max_gu || (uint32_t)(tot * nrd) > P.max_dn;
            if (s.bad) atomicOr(rt.err, LFM_DEVERR_SEGMENT);
            P.counts[0] = s.bad ? 0 : 2 * tot * nrg;
            P.counts[1] = s.bad ? 0 : tot;
            P.counts[2] = s.bad ? 0 : tot * nrd;
            P.counts[3] = s.bad ? 0 : tot;
        }
    }
    __syncthreads();
    if (s.bad) return;
    for (int u = warp; u < U; u += nwarps) {
        const int e = s.act[u], cnt = s.cnt[e], off = s.off[e], t0 = s.tbb[u], n = s.tbb[u + 1] - t0;
        for (int i = lane; i < n; i += 32) P.tbs[t0 + i] = LfmUTokBlock{off + i * nt, min(nt, cnt - i * nt)};
        LfmUTile *gu = P.tiles_gu + 2 * t0 * nrg, *dn = P.tiles_dn + t0 * nrd;
        if (n <= kPlanDirect) {
            /* gate and up tiles of a block side by side: index 2 (rb n + i) + m */
            for (int rb = lane; rb < nrg; rb += 32)
                for (int i = 0; i < n; ++i) {
                    gu[2 * (rb * n + i)] = LfmUTile{e, t0 + i, rb * 128, 0};
                    gu[2 * (rb * n + i) + 1] = LfmUTile{e, t0 + i, rb * 128, 1};
                }
            for (int rb = lane; rb < nrd; rb += 32)
                for (int i = 0; i < n; ++i) dn[rb * n + i] = LfmUTile{e, t0 + i, rb * 128, 0};
        } else {
            for (int q = lane; q < 2 * n * nrg; q += 32) {
                const int m = q & 1, rb = (q >> 1) / n, i = (q >> 1) - rb * n;
                gu[q] = LfmUTile{e, t0 + i, rb * 128, m};
            }
            for (int q = lane; q < n * nrd; q += 32) {
                const int rb = q / n, i = q - rb * n;
                dn[q] = LfmUTile{e, t0 + i, rb * 128, 0};
            }
        }
    }
}

/* Expert parallelism: this block's counts (s.cnt) into every rank's count
 * table, then its cnt_flag there.  Every thread fences its own writes (the
 * Q8_K rows and slots the expert ranks read next) before the flag. */
__device__ void route_publish_counts(const EpPublish &pub, const int *cnt) {
    const uint32_t epoch = __ldcg(pub.step) + 1u;
    const size_t row = ((size_t)(epoch & 1u) * LFM_EP_MAX_RANKS + pub.rank) * pub.E;
    for (uint32_t q = threadIdx.x; q < pub.world * pub.E; q += blockDim.x) {
        const uint32_t p = q / pub.E, e = q - p * pub.E;
        pub.table[p][row + e] = cnt[e];
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < pub.world) lfm_st_release_sys(pub.cnt_flag[threadIdx.x] + pub.rank, epoch);
}
__device__ void route_publish(const EpPublish &pub, const RouteSmem &s) { route_publish_counts(pub, s.cnt); }

/* The dispatch tables from the per-expert counts in s.cnt: offsets, active
 * experts, GEMV work pairs, summary and load statistics (s.off, s.act,
 * s.uniq set for the slot pass and the tile plans).  Thread e takes expert e
 * (blockDim.x >= E) in one block-wide scan, so active experts stay in id order. */
__device__ void route_tables(const MoeLayerDev &L, const RouteTables &rt, RouteSmem &s) {
    const uint32_t E = L.dense ? 1u : L.E;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    {
        const uint32_t e = threadIdx.x;
        const int c = e < E ? s.cnt[e] : 0;
        const int v[4] = {c, c > 0 ? 1 : 0, (c + LFM_GEMV_CHUNK - 1) / LFM_GEMV_CHUNK, c};
        int ex[3];
        block_scan3(v, ex, s);
        if (e < E) {
            s.off[e] = ex[0];
            rt.offsets[e] = ex[0];
            rt.counts[e] = c;
            if (c > 0) {
                s.act[ex[1]] = (int)e;
                s.pb[ex[1]] = ex[2];
                rt.act[ex[1]] = (int)e;
            }
        }
        if (threadIdx.x == 0) {
            const int tot = s.tot[0], uniq = s.tot[1];
            s.off[E] = tot;
            rt.offsets[E] = tot;
            s.uniq = uniq;
            rt.summary[0] = uniq;
            rt.summary[1] = s.tot[3];
            rt.summary[2] = tot;
            rt.summary[3] = s.tot[2];
            if (rt.loads && !L.dense) { /* reductions: nothing waits for them */
                atomicAdd(rt.loads, (unsigned long long)uniq);
                atomicAdd(rt.loads + 1, 1ull);
            }
        }
    }
    __syncthreads();
    /* active experts and their (expert, 8-token chunk) work pairs */
    for (int u = warp; u < s.uniq; u += nwarps) {
        const int e = s.act[u];
        const int nch = (s.cnt[e] + LFM_GEMV_CHUNK - 1) / LFM_GEMV_CHUNK;
        for (int c = lane; c < nch; c += 32) rt.pairs[s.pb[u] + c] = make_int2(u, c);
    }
    __syncthreads();
}

/* Expert id of assignment a for the dispatch passes (-1: none or out of range). */
__device__ __forceinline__ int dispatch_id(const RouteTables &rt, uint32_t a, uint32_t n, uint32_t E, bool flag) {
    int e = -1;
    if (a < n) {
        e = __ldcg(rt.idx + a);
        if ((unsigned)e >= E) {
            if (flag) atomicOr(rt.err, LFM_DEVERR_EXPERT_ID);
            e = -1;
        }
    }
    return e;
}

__device__ void route_dispatch(const MoeLayerDev &L, uint32_t T, const RouteTables &rt, RouteSmem &s) {
    const uint32_t E = L.dense ? 1u : L.E, K = L.dense ? 1u : L.K;
    const uint32_t n = T * K;
    const int lane = threadIdx.x & 31;
    /* up to kPre ids per thread are loaded once, all in flight together, and
     * serve both passes; larger n falls back to loads in each pass */
    constexpr int kPre = 4;
    const uint32_t npass = (n + blockDim.x - 1) / blockDim.x;
    const bool pre = npass <= (uint32_t)kPre;
    int ev[kPre];
#pragma unroll
    for (int i = 0; i < kPre; ++i) {
        const uint32_t a = threadIdx.x + i * blockDim.x;
        ev[i] = pre && a < n ? __ldcg(rt.idx + a) : -1;
    }
    bool bad_id = false;
#pragma unroll
    for (int i = 0; i < kPre; ++i) {
        const uint32_t a = threadIdx.x + i * blockDim.x;
        if (pre && a < n && (unsigned)ev[i] >= E) { bad_id = true; ev[i] = -1; }
    }
    if (bad_id) atomicOr(rt.err, LFM_DEVERR_EXPERT_ID);
    for (uint32_t e = threadIdx.x; e < E; e += blockDim.x) { s.cnt[e] = 0; s.cur[e] = 0; }
    __syncthreads();
    /* histogram: one shared-memory atomic per run of equal expert ids in a warp */
    for (uint32_t i = 0; i < npass; ++i) {
        const uint32_t a = i * blockDim.x + threadIdx.x;
        int e = -1;
        if (pre) {
#pragma unroll
            for (int j = 0; j < kPre; ++j)
                if ((uint32_t)j == i) e = ev[j];
        } else {
            e = dispatch_id(rt, a, n, E, true);
        }
        const unsigned m = __match_any_sync(LFM_FULL_MASK, e);
        if (e >= 0 && lane == __ffs(m) - 1) atomicAdd(&s.cnt[e], __popc(m));
    }
    __syncthreads();
    route_tables(L, rt, s);
    /* slots: a run of equal ids in a warp takes consecutive slots with one atomic */
    for (uint32_t i = 0; i < npass; ++i) {
        const uint32_t a = i * blockDim.x + threadIdx.x;
        int e = -1;
        if (pre) {
#pragma unroll
            for (int j = 0; j < kPre; ++j)
                if ((uint32_t)j == i) e = ev[j];
        } else {
            e = dispatch_id(rt, a, n, E, false);
        }
        const unsigned m = __match_any_sync(LFM_FULL_MASK, e);
        const int leader = __ffs(m) - 1;
        int base = 0;
        if (e >= 0 && lane == leader) base = atomicAdd(&s.cur[e], __popc(m));
        base = __shfl_sync(LFM_FULL_MASK, base, leader);
        if (e >= 0) {
            const int pos = s.off[e] + base + __popc(m & ((1u << lane) - 1u));
            rt.perm[pos] = (int)a;
            rt.inv[a] = pos;
        } else if (a < n) {
            rt.inv[a] = -1;
        }
    }
    if (rt.plan.nt) route_plan(rt, s);
}

/* Order key of a biased score: a larger score gives a larger key and equal
 * scores give equal keys (+0 and -0, and, as the flush-to-zero compare sees
 * them, a denormal and 0); what the reference's strict > against -1e30 never
 * selects (-1e30 and below, NaN) gives 0. */
__device__ __forceinline__ uint32_t route_key(float v) {
    if (!(v > -1e30f)) return 0u;
    uint32_t b = __float_as_uint(v);
    if ((b & 0x7f800000u) == 0u) b = 0u;
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

/* Top-K of token t from its E logits (global memory written by other blocks,
 * read through L2; or this block's shared memory), kPer experts a lane
 * (E <= 32 * kPer).  The loops are unrolled kPer times only: this tail runs
 * once per token group on a cold instruction cache, so the code it executes
 * is kept short. */
template <int kPer>
__device__ void route_topk_n(const MoeLayerDev &L, uint32_t t, const RouteTables &rt,
                                          const float *logits_t, bool global_logits) {
    const int lane = threadIdx.x & 31;
    const uint32_t E = L.E, K = L.K;
    float z[kPer], b[kPer], sig[kPer], sel[kPer]; /* experts lane + 32*i */
#pragma unroll
    for (int i = 0; i < kPer; ++i) { /* every load first */
        const uint32_t e = lane + 32u * i;
        z[i] = 0.0f;
        b[i] = 0.0f;
        if (e < E) {
            z[i] = global_logits ? __ldcg(logits_t + e) : logits_t[e];
            if (L.bias) b[i] = __ldg(L.bias + e);
        }
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const uint32_t e = lane + 32u * i;
        sig[i] = 0.0f;
        sel[i] = -INFINITY;
        if (e < E) {
            sig[i] = __fdiv_rn(1.0f, __fadd_rn(1.0f, lfm_expf(-z[i])));
            sel[i] = L.bias ? __fadd_rn(sig[i], b[i]) : sig[i];
        }
    }
    /* K rounds of argmax under the reference's rule (strict >, the lowest id
     * among equals, nothing at or below -1e30): each lane's best of its own
     * experts (ascending ids, strict >), then the warp's largest order key and
     * the lowest id holding it, by two reductions.  Lane k keeps round k. */
    int my_i = 0;
    float my_w = 0.0f, s = 0.0f;
    for (uint32_t k = 0; k < K; ++k) {
        uint32_t bkey = 0u;
        int bi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const uint32_t e = lane + 32u * i, key = e < E ? route_key(sel[i]) : 0u;
            if (key > bkey) { bkey = key; bi = (int)e; }
        }
        const uint32_t mkey = __reduce_max_sync(LFM_FULL_MASK, bkey);
        /* mkey == 0: nothing beat -1e30 and the reference keeps best_e = 0 */
        const int win = mkey == 0u ? 0 : __reduce_min_sync(LFM_FULL_MASK, bkey == mkey ? bi : 0x7fffffff);
        float s_b = 0.0f;
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            if (lane + 32u * i == (uint32_t)win) { s_b = sig[i]; sel[i] = -1e30f; }
        }
        const float wk = __shfl_sync(LFM_FULL_MASK, s_b, win & 31);
        s = __fadd_rn(s, wk); /* sum of the K weights in round order */
        if ((uint32_t)lane == k) { my_i = win; my_w = wk; }
    }
    if (L.norm_topk)
        my_w = __fmul_rn(my_w, __fdiv_rn(L.routed_scale, __fadd_rn(s, 1e-20f)));
    else if (L.routed_scale != 1.0f)
        my_w = __fmul_rn(my_w, L.routed_scale);
    if ((uint32_t)lane < K) {
        rt.idx[(size_t)t * K + lane] = my_i;
        rt.w[(size_t)t * K + lane] = my_w;
    }
}

__device__ __forceinline__ void route_topk(const MoeLayerDev &L, uint32_t t, const RouteTables &rt,
                                           const float *logits_t, bool global_logits) {
    if (L.E <= 32)
        route_topk_n<1>(L, t, rt, logits_t, global_logits);
    else if (L.E <= 64)
        route_topk_n<2>(L, t, rt, logits_t, global_logits);
    else
        route_topk_n<8>(L, t, rt, logits_t, global_logits);
}

/*
 * Decode-size router (T <= 16): one thread-block cluster of C <= 8 CTAs.
 * CTA c scores experts [c*epc, c*epc + epc) for every token (router rows and
 * ffn_norm bulk-copied before griddepcontrol.wait, x after it), computes each
 * token's RMSNorm itself, and writes its logits straight into CTA 0's shared
 * memory (distributed shared memory).  One cluster barrier later CTA 0 runs
 * top-K, Q8_K and the dispatch for all tokens: no global atomics or fences on
 * the critical path.  Same evaluation order as the prefill router.
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
                                                                   RouteTables rt, EpPublish pub) {
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
    if (pub.world) {
        __syncthreads();
        route_publish(pub, s);
    }
}

/*
 * Prefill-size router (T > 16): three launches instead of one block per
 * (token, 4 experts).
 *  k_norm_q8      one warp per token: the RMSNorm sum of squares (the
 *                 reference's 16 chains + tree), then Q8_K of xb; 1/rms is kept
 *                 for the next pass.  Dense layers route every token to expert
 *                 0 with weight 1 here.
 *  k_router_tiles a CTA scores TT tokens against 32 experts from 256-column
 *                 slices of the router rows and of x (tensor copies, two or
 *                 four slices in flight), then the top-K of each token.
 *  k_dispatch_wide the dispatch tables from one 1024-thread block.
 */
constexpr int kNormWarps = 4;

/* One warp per token: the row lands in shared memory with 16-byte loads issued
 * together, lanes 0-15 run the sum-of-squares chains over it, then the warp
 * quantises xb = (x * inv) * ffn_norm one 256-block at a time.  Dynamic shared
 * memory: kNormWarps * D floats. */
__global__ void __launch_bounds__(kNormWarps * 32) k_norm_q8(MoeLayerDev L, const float *__restrict__ x, uint32_t T,
                                                             Q8Rows xq, RouteTables rt) {
    extern __shared__ __align__(16) float nsm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t t = blockIdx.x * kNormWarps + warp;
    if (t >= T) return;
    const uint32_t D = L.D;
    float *xs = nsm + (size_t)warp * D;
    const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)t * D);
    for (uint32_t i = lane; i < D / 4; i += 32) reinterpret_cast<float4 *>(xs)[i] = __ldg(xr + i);
    __syncwarp();
    float acc = 0.0f;
    if (lane < 16) {
#pragma unroll 16
        for (uint32_t i = 0; i < D; i += 16) {
            const float v = xs[i + lane];
            acc = __fmaf_rn(v, v, acc);
        }
    }
    const float ss = lfm_hsum16_ref(acc);
    const float inv = __shfl_sync(LFM_FULL_MASK, __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), L.eps))), 0);
    if (lane == 0) {
        rt.rms[t] = inv;
        if (L.dense) { rt.idx[t] = 0; rt.w[t] = 1.0f; }
    }
    for (uint32_t b = 0; b < D / 256; ++b) {
        const float4 p0 = reinterpret_cast<const float4 *>(xs + 256 * b + 8 * lane)[0];
        const float4 p1 = reinterpret_cast<const float4 *>(xs + 256 * b + 8 * lane)[1];
        const float xv[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
        float nw[8] = {1, 1, 1, 1, 1, 1, 1, 1};
        if (L.ffn_norm) {
            const float4 w0 = __ldg(reinterpret_cast<const float4 *>(L.ffn_norm + 256 * b + 8 * lane));
            const float4 w1 = __ldg(reinterpret_cast<const float4 *>(L.ffn_norm + 256 * b + 8 * lane) + 1);
            nw[0] = w0.x; nw[1] = w0.y; nw[2] = w0.z; nw[3] = w0.w; nw[4] = w1.x; nw[5] = w1.y; nw[6] = w1.z; nw[7] = w1.w;
        }
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float n = __fmul_rn(xv[i], inv);
            v[i] = L.ffn_norm ? __fmul_rn(n, nw[i]) : n;
        }
        lfm_quant_block_warp(v, xq, t, b);
    }
}

constexpr int kRtSlice = 256;   /* columns per slice */
constexpr int kRtExperts = 32;  /* experts per pass  */

template <int TT, int TPT>
struct RouterTile {
    static constexpr int kW = kRtExperts * kRtSlice * 4;  /* router rows of a slice (tensor copy, zero-filled) */
    static constexpr int kX = TT * kRtSlice * 4;          /* the tokens' x of a slice (tensor copy)            */
    static constexpr int kStage = kW + kX + kRtSlice * 4; /* + ffn_norm of the slice                            */
    static constexpr int kGroups = 16;
    static constexpr int kTokGroups = TT / TPT;
    static constexpr int kEpt = kRtExperts / (kGroups / kTokGroups); /* experts per thread per pass */
};

/* CTA (tile, p) scores TT tokens against experts [32p, 32p + 32).  Per
 * 256-column slice: the router rows (box 256 x 32 of router_w, rows past E
 * read as zero) and the tokens' x (box 256 x TT) arrive by one tensor copy
 * each, ffn_norm by a bulk copy, NS slices in flight; xb is rebuilt in place
 * from x, 1/rms and ffn_norm exactly as k_norm_q8 forms it; thread (chain l,
 * group g) advances chain l of TPT tokens x EPT experts through the slice --
 * each chain in the reference's column order -- and after the last slice the
 * 16-lane tree gives the logits.  One warp per token then takes the top-K:
 * at once when E <= 32, else in the last of the tile's CTAs to arrive (a
 * counter per tile), from the logits every CTA wrote to global memory. */
template <int TT, int TPT, int NS>
__global__ void __launch_bounds__(256) k_router_tiles(const __grid_constant__ CUtensorMap tmw,
                                                      const __grid_constant__ CUtensorMap tmx, MoeLayerDev L,
                                                      uint32_t T, RouteTables rt) {
    using RT = RouterTile<TT, TPT>;
    constexpr int EPT = RT::kEpt;
    extern __shared__ __align__(128) uint8_t dsm[];
    __shared__ uint64_t bars[NS];
    __shared__ float s_inv[TT];
    __shared__ int s_last;
    const uint32_t D = L.D, E = L.E;
    const uint32_t tok0 = blockIdx.x * TT, pass = blockIdx.y;
    const uint32_t nt = min((uint32_t)TT, T - tok0);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int l = threadIdx.x & 15, g = threadIdx.x >> 4;
    const int tg = g % RT::kTokGroups, eg = g / RT::kTokGroups;
    float *lg = reinterpret_cast<float *>(dsm + NS * RT::kStage); /* [TT][E] logits */
    const uint32_t nq = D / kRtSlice; /* slices of this CTA's pass */
    if (threadIdx.x == 0) {
        for (int i = 0; i < NS; ++i) lfm_mbar_init(&bars[i], 1);
        lfm_fence_mbar_init();
    }
    if (threadIdx.x < TT) s_inv[threadIdx.x] = threadIdx.x < nt ? __ldcg(rt.rms + tok0 + threadIdx.x) : 0.0f;
    __syncthreads();
    auto issue = [&](uint32_t sl) {
        uint8_t *st = dsm + (sl % NS) * RT::kStage;
        uint64_t *bar = &bars[sl % NS];
        lfm_mbar_arrive_tx(bar, RT::kW + RT::kX + (L.ffn_norm ? kRtSlice * 4 : 0));
        lfm_tma_load_2d(st, &tmw, sl * kRtSlice, pass * kRtExperts, bar);
        lfm_tma_load_2d(st + RT::kW, &tmx, sl * kRtSlice, tok0, bar);
        if (L.ffn_norm) lfm_bulk_g2s_plain(st + RT::kW + RT::kX, L.ffn_norm + sl * kRtSlice, kRtSlice * 4, bar);
    };
    if (threadIdx.x == 0)
        for (uint32_t q = 0; q < nq && q < NS - 1; ++q) issue(q);
    float acc[TPT][EPT];
#pragma unroll
    for (int j = 0; j < TPT; ++j)
#pragma unroll
        for (int k = 0; k < EPT; ++k) acc[j][k] = 0.0f;
    bool ok = true;
    for (uint32_t q = 0; q < nq; ++q) {
        const uint32_t sl = q;
        /* stage (q + NS - 1) % NS was last read in iteration q - 1, which every thread has left */
        if (threadIdx.x == 0 && q + NS - 1 < nq) issue(q + NS - 1);
        ok = ok && lfm_mbar_wait(&bars[q % NS], (q / NS) & 1u, rt.err);
        float *st = reinterpret_cast<float *>(dsm + (q % NS) * RT::kStage);
        const float *ws = st;
        float *xs = st + kRtExperts * kRtSlice;
        const float *nw = xs + TT * kRtSlice;
        for (uint32_t i = threadIdx.x; i < nt * kRtSlice; i += blockDim.x) {
            const uint32_t t = i / kRtSlice, c = i % kRtSlice;
            const float n = __fmul_rn(xs[i], s_inv[t]);
            xs[i] = L.ffn_norm ? __fmul_rn(n, nw[c]) : n;
        }
        __syncthreads();
        if (ok) {
#pragma unroll 4
            for (int c = 0; c < kRtSlice / 16; ++c) {
                const int i = 16 * c + l;
                float xv[TPT];
#pragma unroll
                for (int j = 0; j < TPT; ++j) xv[j] = xs[(tg * TPT + j) * kRtSlice + i];
#pragma unroll
                for (int k = 0; k < EPT; ++k) {
                    const float wv = ws[(eg * EPT + k) * kRtSlice + i];
#pragma unroll
                    for (int j = 0; j < TPT; ++j) acc[j][k] = __fmaf_rn(wv, xv[j], acc[j][k]);
                }
            }
        }
        if (sl == nq - 1) {
#pragma unroll
            for (int j = 0; j < TPT; ++j)
#pragma unroll
                for (int k = 0; k < EPT; ++k) {
                    const float z = lfm_hsum16_ref(acc[j][k]);
                    const uint32_t t = tg * TPT + j, e = eg * EPT + k;
                    if (l == 0 && pass * kRtExperts + e < E) lg[t * kRtExperts + e] = z;
                }
        }
        __syncthreads();
    }
    if (!ok) return;
    const uint32_t ne = min((uint32_t)kRtExperts, E - pass * kRtExperts);
    for (uint32_t t = warp; t < nt; t += blockDim.x / 32)
        for (uint32_t e = lane; e < ne; e += 32)
            rt.logits[(size_t)(tok0 + t) * E + pass * kRtExperts + e] = lg[t * kRtExperts + e];
    if (gridDim.y == 1) {
        for (uint32_t t = warp; t < nt; t += blockDim.x / 32) route_topk(L, tok0 + t, rt, lg + t * kRtExperts, false);
        return;
    }
    /* several passes: the tile's last CTA takes the top-K from every pass's logits */
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(rt.tok_count + blockIdx.x, 1u) == gridDim.y - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (threadIdx.x == 0) rt.tok_count[blockIdx.x] = 0;
    for (uint32_t t = warp; t < nt; t += blockDim.x / 32)
        route_topk(L, tok0 + t, rt, rt.logits + (size_t)(tok0 + t) * E, true);
}

/*
 * Decode-size route in one launch (16 < T <= kDecMaxT = 256): CTA (g, p) takes tokens
 * [4g, 4g + 4) and experts [8p, 8p + 8).  Its router rows and ffn_norm arrive
 * by bulk copy before griddepcontrol.wait (they do not depend on the preceding
 * kernel), the tokens' x after it.  Warp w takes token w: its RMSNorm in the
 * reference's order (16 chains + tree), xb = (x * inv) * ffn_norm in place,
 * then the Q8_K blocks b = p, p + P, ... of xb (the P CTAs of a token group
 * share the token's blocks).  A half-warp then takes an expert and two tokens:
 * lane l runs chain l of both logits, then the 16-lane tree, and the logits go
 * to global memory.  The last CTA of a token group (arrival counter per group)
 * takes those tokens' top-K; the last group to finish (counter rt.done) builds
 * the dispatch tables and the tcgen05 tile plans.  Replaces k_norm_q8 +
 * k_router_tiles + k_dispatch_wide at these sizes.
 */
constexpr uint32_t kDecMaxT = 256; /* measured against the three launches below: 25 vs 35 us at T=256, E=32;
                                     34 vs 37 at E=64; at T=512 (E=64) 52 vs 46, so they take over there */
constexpr uint32_t kDecTok = 4, kDecExp = 8;
constexpr uint32_t kDecThreads = 256;
static_assert(kDecTok <= kDecThreads / 32, "a warp per token");

__global__ void __launch_bounds__(kDecThreads) k_route_dec(MoeLayerDev L, const float *__restrict__ x, uint32_t T,
                                                           Q8Rows xq, RouteTables rt, EpPublish pub) {
    extern __shared__ __align__(16) float dsm_dec[];
    __shared__ uint64_t bar_w, bar_x;
    __shared__ int s_last;
    __shared__ RouteSmem s;
    const uint32_t D = L.D, E = L.E;
    const uint32_t tg = blockIdx.x, pg = blockIdx.y;
    const uint32_t tok0 = tg * kDecTok, e0 = pg * kDecExp;
    const uint32_t nt = min(kDecTok, T - tok0), ne = min(kDecExp, E - e0);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t ld = D + 16;                /* padded rows: the two half-warps of a warp read other banks */
    float *ws = dsm_dec;                       /* [8][ld] router rows     */
    float *xs = ws + (size_t)kDecExp * ld;     /* [4][ld] x, then xb      */
    float *nw = xs + (size_t)kDecTok * ld;     /* [D]     ffn_norm        */
    if (threadIdx.x == 0) {
        lfm_mbar_init(&bar_w, 1);
        lfm_mbar_init(&bar_x, 1);
        lfm_fence_mbar_init();
        const uint32_t wb = ne * D * 4 + (L.ffn_norm ? D * 4 : 0);
        lfm_mbar_arrive_tx(&bar_w, wb);
        for (uint32_t e = 0; e < ne; ++e) lfm_bulk_g2s_plain(ws + (size_t)e * ld, L.router_w + (size_t)(e0 + e) * D, D * 4, &bar_w);
        if (L.ffn_norm) lfm_bulk_g2s_plain(nw, L.ffn_norm, D * 4, &bar_w);
    }
    lfm_pdl_launch_dependents();
    lfm_pdl_wait(); /* x, and every table this kernel writes, belong to the preceding kernels */
    if (threadIdx.x == 0) {
        lfm_mbar_arrive_tx(&bar_x, nt * D * 4);
        for (uint32_t t = 0; t < nt; ++t) lfm_bulk_g2s_plain(xs + (size_t)t * ld, x + (size_t)(tok0 + t) * D, D * 4, &bar_x);
    }
    __syncthreads();
    bool ok = true;
    if (threadIdx.x == 0) ok = lfm_mbar_wait(&bar_x, 0, rt.err) && lfm_mbar_wait(&bar_w, 0, rt.err);
    if (threadIdx.x == 0) s_last = ok ? 1 : 0;
    __syncthreads();
    if (!s_last) return;
    if ((uint32_t)warp < nt) {
        /* token w: RMSNorm (lanes 0-15 run the 16 chains, then the tree) */
        float *xr = xs + (size_t)warp * ld;
        float acc = 0.0f;
        if (lane < 16) {
#pragma unroll 16
            for (uint32_t i = 0; i < D; i += 16) {
                const float v = xr[i + lane];
                acc = __fmaf_rn(v, v, acc);
            }
        }
        const float ss = __shfl_sync(LFM_FULL_MASK, lfm_hsum16_ref(acc), 0);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), L.eps)));
        if (pg == 0 && lane == 0) rt.rms[tok0 + warp] = inv;
        /* xb = (x * inv) * ffn_norm in place, four columns a lane */
        for (uint32_t c = 4 * lane; c < D; c += 128) {
            float4 v = *reinterpret_cast<const float4 *>(xr + c);
            v.x = __fmul_rn(v.x, inv);
            v.y = __fmul_rn(v.y, inv);
            v.z = __fmul_rn(v.z, inv);
            v.w = __fmul_rn(v.w, inv);
            if (L.ffn_norm) {
                const float4 n = *reinterpret_cast<const float4 *>(nw + c);
                v.x = __fmul_rn(v.x, n.x);
                v.y = __fmul_rn(v.y, n.y);
                v.z = __fmul_rn(v.z, n.z);
                v.w = __fmul_rn(v.w, n.w);
            }
            *reinterpret_cast<float4 *>(xr + c) = v;
        }
        __syncwarp();
        /* this CTA's share of the token's Q8_K blocks */
        for (uint32_t b = pg; b < D / 256; b += gridDim.y) {
            const float4 p0 = reinterpret_cast<const float4 *>(xr + 256 * b + 8 * lane)[0];
            const float4 p1 = reinterpret_cast<const float4 *>(xr + 256 * b + 8 * lane)[1];
            const float v[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
            lfm_quant_block_warp(v, xq, tok0 + warp, b);
        }
    }
    __syncthreads();
    /* logits: half-warp h takes expert h % 8 and tokens h / 8, h / 8 + 2; lane l runs chain l of both */
    {
        const int hw = threadIdx.x >> 4, l = threadIdx.x & 15;
        constexpr int kPairs = kDecTok * kDecExp / (kDecThreads / 16);
        static_assert(kPairs == 2, "two tokens a half-warp");
        const uint32_t e = (uint32_t)hw % kDecExp, t0 = (uint32_t)hw / kDecExp, t1 = t0 + 2;
        const float *wr = ws + (size_t)min(e, ne - 1) * ld + l;
        const float *x0 = xs + (size_t)min(t0, nt - 1) * ld + l, *x1 = xs + (size_t)min(t1, nt - 1) * ld + l;
        float a0 = 0.0f, a1 = 0.0f;
#pragma unroll 8
        for (uint32_t i = 0; i < D; i += 16) {
            const float w = wr[i];
            a0 = __fmaf_rn(w, x0[i], a0);
            a1 = __fmaf_rn(w, x1[i], a1);
        }
        const float z0 = lfm_hsum16_ref(a0), z1 = lfm_hsum16_ref(a1);
        if (l == 0 && e < ne) {
            if (t0 < nt) rt.logits[(size_t)(tok0 + t0) * E + e0 + e] = z0;
            if (t1 < nt) rt.logits[(size_t)(tok0 + t1) * E + e0 + e] = z1;
        }
    }
    /* the last expert-group CTA of this token group takes its tokens' top-K */
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(rt.tok_count + tg, 1u) == gridDim.y - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (threadIdx.x == 0) rt.tok_count[tg] = 0;
    if ((uint32_t)warp < nt) route_topk(L, tok0 + warp, rt, rt.logits + (size_t)(tok0 + warp) * E, true);
    /* the last token group to finish builds the dispatch tables and tile plans */
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(rt.done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (threadIdx.x == 0) *rt.done = 0;
    route_dispatch(L, T, rt, s);
    if (pub.world) {
        __syncthreads();
        route_publish(pub, s);
    }
}

__global__ void __launch_bounds__(1024) k_dispatch_wide(MoeLayerDev L, uint32_t T, RouteTables rt, EpPublish pub) {
    __shared__ RouteSmem s;
    route_dispatch(L, T, rt, s);
    if (pub.world) {
        __syncthreads();
        route_publish(pub, s);
    }
}

/*
 * Dispatch of many assignments (T*K >= kSplitMin) over one CTA per 1024-assignment
 * chunk, in two launches instead of one block walking them all:
 *  k_dispatch_hist   each CTA counts its chunk per expert (chunk[c][e]); the
 *                    last CTA to arrive (counter rt.done) turns the chunk counts
 *                    into totals, the tables, the tile plans, and each chunk's
 *                    first rank inside every expert segment (chunk[c][e]);
 *  k_dispatch_slots  each CTA places its chunk at offset + chunk rank + its own
 *                    running rank; for expert parallelism the last CTA to
 *                    finish publishes the counts once every slot is written.
 * The order inside an expert segment changes no result.
 */
constexpr uint32_t kDispChunk = 1024;
constexpr uint32_t kSplitMin = 4096;

__global__ void __launch_bounds__(kDispChunk) k_dispatch_hist(MoeLayerDev L, uint32_t T, RouteTables rt) {
    __shared__ RouteSmem s;
    __shared__ int s_last;
    const uint32_t E = L.E, n = T * L.K, c = blockIdx.x;
    const int lane = threadIdx.x & 31;
    for (uint32_t e = threadIdx.x; e < E; e += blockDim.x) s.cnt[e] = 0;
    __syncthreads();
    const int e = dispatch_id(rt, c * kDispChunk + threadIdx.x, n, E, true);
    const unsigned m = __match_any_sync(LFM_FULL_MASK, e);
    if (e >= 0 && lane == __ffs(m) - 1) atomicAdd(&s.cnt[e], __popc(m));
    __syncthreads();
    for (uint32_t q = threadIdx.x; q < E; q += blockDim.x) rt.chunk[(size_t)c * E + q] = s.cnt[q];
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(rt.done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (threadIdx.x == 0) *rt.done = 0;
    /* chunk counts -> rank of each chunk's first slot in the expert's segment:
     * one warp per expert, 32 chunks per step through a warp scan */
    const int warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    for (uint32_t q = warp; q < E; q += nwarps) {
        int acc = 0;
        for (uint32_t c0 = 0; c0 < gridDim.x; c0 += 32) {
            const uint32_t cc = c0 + lane;
            int *p = rt.chunk + (size_t)cc * E + q;
            const int v = cc < gridDim.x ? __ldcg(p) : 0;
            int incl = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int u = __shfl_up_sync(LFM_FULL_MASK, incl, o);
                if (lane >= o) incl += u;
            }
            if (cc < gridDim.x) *p = acc + incl - v;
            acc += __shfl_sync(LFM_FULL_MASK, incl, 31);
        }
        if (lane == 0) s.cnt[q] = acc;
    }
    __syncthreads();
    route_tables(L, rt, s);
    if (rt.plan.nt) route_plan(rt, s);
}

__global__ void __launch_bounds__(kDispChunk) k_dispatch_slots(MoeLayerDev L, uint32_t T, RouteTables rt,
                                                               EpPublish pub) {
    __shared__ int cur[LFM_GPU_MAX_EXPERTS_DEV];
    __shared__ int s_last;
    const uint32_t E = L.E, n = T * L.K, c = blockIdx.x;
    const int lane = threadIdx.x & 31;
    for (uint32_t q = threadIdx.x; q < E; q += blockDim.x)
        cur[q] = __ldcg(rt.offsets + q) + __ldcg(rt.chunk + (size_t)c * E + q);
    __syncthreads();
    const uint32_t a = c * kDispChunk + threadIdx.x;
    const int e = dispatch_id(rt, a, n, E, false);
    const unsigned m = __match_any_sync(LFM_FULL_MASK, e);
    const int leader = __ffs(m) - 1;
    int base = 0;
    if (e >= 0 && lane == leader) base = atomicAdd(&cur[e], __popc(m));
    base = __shfl_sync(LFM_FULL_MASK, base, leader);
    if (e >= 0) {
        const int pos = base + __popc(m & ((1u << lane) - 1u));
        rt.perm[pos] = (int)a;
        rt.inv[a] = pos;
    } else if (a < n) {
        rt.inv[a] = -1;
    }
    if (!pub.world) return;
    /* expert parallelism: every CTA's slots (and the Q8_K rows before them) before the counts go out */
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(rt.done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (threadIdx.x == 0) *rt.done = 0;
    for (uint32_t q = threadIdx.x; q < E; q += blockDim.x) cur[q] = __ldcg(rt.counts + q);
    __syncthreads();
    route_publish_counts(pub, cur);
}

/* Dispatch tables alone, for rows whose experts are given (expert parallelism). */
__global__ void __launch_bounds__(256) k_dispatch_only(MoeLayerDev L, uint32_t T, RouteTables rt) {
    __shared__ RouteSmem s;
    route_dispatch(L, T, rt, s);
}

/* Expert parallelism, expert rank: wait for every home rank's per-expert
 * counts, then lay out the received slots -- local expert el, then home rank
 * r, then r's own slot order -- as the dispatch tables of the shard (counts,
 * offsets, active experts, tcgen05 tile plans) plus rowmap[slot] = (r << 24)
 * | r's slot, which the gather reads r's perm and Q8_K rows through.  The
 * home rank's slot of its i-th assignment to expert e is its exclusive
 * prefix of counts before e, plus i (route_dispatch's slot order). */
__global__ void __launch_bounds__(1024) k_ep_plan(EpStep st, uint32_t first, uint32_t count, RouteTables rt) {
    __shared__ RouteSmem s;
    __shared__ int tab[LFM_EP_MAX_RANKS][LFM_GPU_MAX_EXPERTS_DEV];
    __shared__ int pre[LFM_EP_MAX_RANKS][LFM_GPU_MAX_EXPERTS_DEV];  /* home ranks before r, per local expert */
    __shared__ int hoff[LFM_EP_MAX_RANKS][LFM_GPU_MAX_EXPERTS_DEV]; /* r's first slot of expert first + el */
    __shared__ int ok;
    const UmmaPlanOut &P = rt.plan;
    const uint32_t W = st.world, E = st.E;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    lfm_pdl_launch_dependents();
    lfm_pdl_wait(); /* the step counter, tables and plans belong to the preceding kernels */
    const uint32_t epoch = __ldcg(st.self.step) + st.ahead;
    if (threadIdx.x == 0) ok = lfm_wait_flags(st.self.cnt_flag, W, epoch, st.wait_ns, st.err) ? 1 : 0;
    __syncthreads();
    if (!ok) {
        if (threadIdx.x < 4) P.counts[threadIdx.x] = 0;
        if (threadIdx.x == 0) *st.self.n_recv = 0;
        return;
    }
    const int32_t *t0 = st.self.table + (size_t)(epoch & 1u) * LFM_EP_MAX_RANKS * E;
    for (uint32_t q = threadIdx.x; q < W * E; q += blockDim.x) tab[q / E][q % E] = lfm_ld_relaxed_sys(t0 + q);
    __syncthreads();
    if (threadIdx.x < W) { /* home rank r's slot prefix up to each of this shard's experts */
        const uint32_t r = threadIdx.x;
        int acc = 0;
        for (uint32_t e = 0; e < first; ++e) acc += tab[r][e];
        for (uint32_t el = 0; el < count; ++el) {
            hoff[r][el] = acc;
            acc += tab[r][first + el];
        }
    }
    if (threadIdx.x >= 32 && threadIdx.x - 32 < count) {
        const uint32_t el = threadIdx.x - 32;
        int acc = 0;
        for (uint32_t r = 0; r < W; ++r) {
            pre[r][el] = acc;
            acc += tab[r][first + el];
        }
        s.cnt[el] = acc;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int acc = 0, uniq = 0;
        for (uint32_t el = 0; el < count; ++el) {
            s.off[el] = acc;
            acc += s.cnt[el];
            if (s.cnt[el] > 0) s.act[uniq++] = (int)el;
        }
        s.off[count] = acc;
        s.uniq = uniq;
        s.bad = acc < 0 || (uint32_t)acc > st.max_recv;
        if (s.bad) atomicOr(st.err, LFM_DEVERR_SEGMENT);
        *st.self.n_recv = s.bad ? 0 : acc;
        if (rt.loads) {
            atomicAdd(rt.loads, (unsigned long long)uniq);
            atomicAdd(rt.loads + 1, 1ull);
        }
    }
    __syncthreads();
    if (s.bad) {
        if (threadIdx.x < 4) P.counts[threadIdx.x] = 0;
        return;
    }
    for (uint32_t q = warp; q < count * W; q += nwarps) { /* (local expert, home rank) runs of slots */
        const uint32_t el = q / W, r = q % W;
        const int n = tab[r][first + el], dst = s.off[el] + pre[r][el], src = hoff[r][el];
        for (int i = lane; i < n; i += 32) st.self.rowmap[dst + i] = (r << 24) | (uint32_t)(src + i);
    }
    route_plan(rt, s);
}

}  // namespace

cudaError_t lfm_launch_ep_plan(const EpStep &st, uint32_t first, uint32_t count, const RouteTables &rt,
                               cudaStream_t s, bool pdl) {
    if (st.world == 0 || st.world > LFM_EP_MAX_RANKS || st.E > LFM_GPU_MAX_EXPERTS_DEV || count > st.E ||
        first + count > st.E || !rt.plan.nt)
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(1024);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_ep_plan, st, first, count, rt);
}

cudaError_t lfm_launch_dispatch(const MoeLayerDev &L, uint32_t T, const RouteTables &rt, cudaStream_t s) {
    if (T == 0) return cudaSuccess;
    k_dispatch_only<<<1, 256, 0, s>>>(L, T, rt);
    return cudaGetLastError();
}

template <int TT, int TPT, int NS>
static cudaError_t launch_router_tiles(const MoeLayerDev &L, const float *x, uint32_t T, const RouteTables &rt,
                                       cudaStream_t s) {
    using RT = RouterTile<TT, TPT>;
    CUtensorMap tmw, tmx;
    if (!lfm_tmap_2d(&tmw, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, L.router_w, L.D, L.E, (uint64_t)L.D * 4, kRtSlice,
                     kRtExperts) ||
        !lfm_tmap_2d(&tmx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, x, L.D, T, (uint64_t)L.D * 4, kRtSlice, TT))
        return cudaErrorInvalidValue;
    const size_t smem = NS * RT::kStage + sizeof(float) * TT * kRtExperts;
    static size_t cache[16];
    cudaError_t e = lfm_smem_attr((const void *)k_router_tiles<TT, TPT, NS>, smem, cache);
    if (e != cudaSuccess) return e;
    const dim3 grid((T + TT - 1) / TT, (L.E + kRtExperts - 1) / kRtExperts);
    k_router_tiles<TT, TPT, NS><<<grid, 256, smem, s>>>(tmw, tmx, L, T, rt);
    return cudaGetLastError();
}

static size_t route_dec_smem(const MoeLayerDev &L, uint32_t T) {
    if (L.dense || T <= kClusterMaxT || T > kDecMaxT || L.E > LFM_GPU_MAX_EXPERTS_DEV) return 0;
    const size_t bytes = sizeof(float) * ((size_t)(kDecTok + kDecExp) * (L.D + 16) + L.D);
    return bytes <= 200 * 1024 ? bytes : 0;
}

static cudaError_t launch_route_dec(const MoeLayerDev &L, const float *x, uint32_t T, Q8Rows xq, const RouteTables &rt,
                                   cudaStream_t s, bool pdl, const EpPublish &pub, size_t smem) {
    static size_t cache[16];
    cudaError_t e = lfm_smem_attr((const void *)k_route_dec, smem, cache);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((T + kDecTok - 1) / kDecTok, (L.E + kDecExp - 1) / kDecExp);
    cfg.blockDim = dim3(kDecThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_route_dec, L, x, T, xq, rt, pub);
}

/* T > 16: normalise + quantise, score (all experts per CTA), dispatch. */
static cudaError_t launch_route_prefill(const MoeLayerDev &L, const float *x, uint32_t T, Q8Rows xq,
                                        const RouteTables &rt, cudaStream_t s, const EpPublish &pub) {
    const size_t nsmem = sizeof(float) * kNormWarps * L.D;
    static size_t cache[16];
    cudaError_t e = lfm_smem_attr((const void *)k_norm_q8, nsmem, cache);
    if (e != cudaSuccess) return e;
    k_norm_q8<<<(T + kNormWarps - 1) / kNormWarps, kNormWarps * 32, nsmem, s>>>(L, x, T, xq, rt);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if (!L.dense) {
        /* enough CTAs for the grid, two or more resident per SM below 4096 tokens */
        /* several tokens per thread: each shared-memory load of a router value feeds TPT FMAs */
        if (T >= 4096) e = launch_router_tiles<16, 4, 2>(L, x, T, rt, s);
        else if (T >= 1024) e = launch_router_tiles<8, 2, 2>(L, x, T, rt, s);
        else if (T >= 256) e = launch_router_tiles<4, 2, 2>(L, x, T, rt, s);
        else e = launch_router_tiles<2, 2, 2>(L, x, T, rt, s);
        if (e != cudaSuccess) return e;
    }
    const uint32_t n = T * lfm_layer_K(L);
    if (!L.dense && rt.chunk && n >= kSplitMin) {
        const uint32_t nc = (n + kDispChunk - 1) / kDispChunk;
        k_dispatch_hist<<<nc, kDispChunk, 0, s>>>(L, T, rt);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        k_dispatch_slots<<<nc, kDispChunk, 0, s>>>(L, T, rt, pub);
        return cudaGetLastError();
    }
    k_dispatch_wide<<<1, 1024, 0, s>>>(L, T, rt, pub);
    return cudaGetLastError();
}

/* Shared memory of the cluster router, or 0 when (T, D, E) does not fit it. */
static size_t route_cluster_smem(const MoeLayerDev &L, uint32_t T, uint32_t *epc_out) {
    if (L.dense || T == 0 || T > kClusterMaxT || L.E == 0) return 0;
    const uint32_t epc = (L.E + 7) / 8;
    const size_t bytes = sizeof(float) * ((size_t)T * L.D + L.D + (size_t)epc * L.D + (size_t)T * L.E);
    if (bytes > 200 * 1024) return 0;
    *epc_out = epc;
    return bytes;
}

uint32_t lfm_route_kernels(const MoeLayerDev &L, uint32_t T) {
    uint32_t epc = 0;
    if (T == 0) return 0;
    if (route_cluster_smem(L, T, &epc) > 0) return 1;
    if (route_dec_smem(L, T) > 0) return 1;
    if (L.dense) return 2u;
    return T * L.K >= kSplitMin ? 4u : 3u; /* the wide dispatch splits in two at many assignments */
}

cudaError_t lfm_launch_route(const MoeLayerDev &L, const float *x, uint32_t T, Q8Rows xq, const RouteTables &rt,
                             cudaStream_t s, bool pdl, const EpPublish *pub_in) {
    if (T == 0) return cudaSuccess;
    const EpPublish pub = pub_in ? *pub_in : EpPublish{};
    if (pub.world > LFM_EP_MAX_RANKS || (pub.world && L.E > LFM_GPU_MAX_EXPERTS_DEV)) return cudaErrorInvalidValue;
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
        return cudaLaunchKernelEx(&cfg, k_route_cluster, L, x, T, epc, xq, rt, pub);
    }
    const size_t dsmem = route_dec_smem(L, T);
    if (dsmem > 0) return launch_route_dec(L, x, T, xq, rt, s, pdl, pub, dsmem);
    return launch_route_prefill(L, x, T, xq, rt, s, pub);
}
