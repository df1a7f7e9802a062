/*
 * Fused decode layer: the whole lfm2moe FFN layer (or a dense SwiGLU layer)
 * for T <= 16 tokens in ONE cooperative launch of one CTA per SM.
 *
 * The separate-kernel path (k_route -> k_gemv<2> -> k_quant_rows -> k_gemv<1>
 * -> k_combine) pays a launch, a prologue (tables read back from L2, first
 * copies issued) and a tail per kernel; at decode sizes those fixed costs, not
 * HBM, set the layer time.  Here the phases are separated by grid-wide
 * barriers (arrival counter + generation word in global memory, bounded
 * waits) and every CTA keeps the routing tables in its own shared memory:
 *
 *  1. x, ffn_norm and the CTA's router rows are bulk-copied into shared
 *     memory; RMSNorm in the reference's 16-lane order, xb = (x*inv)*w
 *     (tools/lfm2_decode_1x4.c:98-133); router logits distributed: CTA c
 *     scores dots [c*T*E/G, (c+1)*T*E/G) (expert-major, one half-warp each,
 *     include/lfm2_simd_avx2.h:676-687) and quantises its share of the T*D/256
 *     Q8_K records (tools/lfm2_decode_1x4.c:150-186); both go to global
 *     memory; grid barrier; every CTA bulk-copies all records back.
 *  2. every CTA reads the T*E logits and computes, identically, the biased
 *     top-K and weights (tools/lfm2_moe_checkpoint.c:183-239) and the dispatch
 *     tables: per-expert counts, offsets, a slot order that is a pure function
 *     of the routing (assignment a gets rank #{a' < a : e(a') = e(a)} in its
 *     expert's segment), and the (expert, 8-token chunk) pairs.
 *  3. gate|up: the CTA's range of (pair, 2-row) items through per-warp rings of
 *     bulk-copy stages (as k_gemv); h = silu(g)*u to global.  Each warp's ring
 *     continues straight into its down units, so down weights are already in
 *     flight across the grid barrier that follows.
 *  4. down: the h rows of the CTA's pairs are quantised to Q8_K records in
 *     shared memory (tools/lfm2_cpuid_quants.c:584-631), then the (pair,
 *     4-row) items; y to global; grid barrier.
 *  5. combine: x[t][r] = fma(w_k, y[slot(t,k)][r], x[t][r]) for k in order
 *     (tools/lfm2_moe_checkpoint.c:266-269), the CTA's slice of T*D.
 * Dense layers skip the router: every token goes to expert 0 with weight 1,
 * so the combine is x + down exactly (tools/lfm2_decode_1x4.c:1086-1103).
 *
 * Co-residency of all CTAs is guaranteed by the cooperative launch.  Every
 * wait (mbarrier or grid barrier) is bounded; after a timeout the CTA stops
 * working, lets its copies in flight land and leaves with the error word set.
 */
#include "moe_device.cuh"
#include "moe_internal.h"

namespace {

constexpr int kW = 12;
constexpr int kMaxS = 4;
constexpr int kMaxT = LFM_FUSED_MAX_T;
constexpr int kMaxTK = kMaxT * LFM_GPU_MAX_TOPK_DEV;
constexpr int kMaxPairs = LFM_GPU_MAX_EXPERTS_DEV + kMaxTK / LFM_GEMV_CHUNK + 1;
constexpr int kCh = LFM_GEMV_CHUNK;
constexpr uint32_t kUnitSb = 8;
constexpr size_t kSmemBudget = 212 * 1024; /* dynamic; the static LayerShared is ~9 KB */

struct LayerShared {
    uint64_t full[kW][kMaxS];
    uint64_t bar_in; /* bulk copy of x, ffn_norm and this CTA's router rows */
    float inv_rms[kMaxT];
    int idx[kMaxTK];
    float wk[kMaxTK];
    int cnt[LFM_GPU_MAX_EXPERTS_DEV];
    int off[LFM_GPU_MAX_EXPERTS_DEV + 1];
    int perm[kMaxTK];
    int inv[kMaxTK];
    int tok[kMaxTK]; /* token of each dispatch slot */
    int pe[kMaxPairs], ps0[kMaxPairs], pnt[kMaxPairs];
    int npairs;
    uint32_t gu_lo, gu_hi, dn_lo, dn_hi; /* this CTA's item ranges */
    unsigned gen0;
    int ok;
    int abort;
};

struct LayerArgs {
    MoeLayerDev L;
    float *x;
    uint32_t T;
    RouteTables rt;  /* logits (exchange), err, loads, summary, idx/w (CTA 0 mirrors them) */
    float *h;        /* [T*K][I] */
    float *y;        /* [T*K][D] */
    unsigned *gbar;  /* [2]: arrival count, generation */
    uint8_t *xrec;   /* [T][D/256] Q8_K records of the normalised rows (exchange) */
    float *scores;   /* [T*E][2]: sigmoid and biased selection score (exchange) */
    uint32_t S;      /* stages per warp */
    uint32_t dslots; /* down pairs staged per phase */
};

__device__ __forceinline__ int ld_volatile_int(const int *p) { return *reinterpret_cast<const volatile int *>(p); }

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu(unsigned *p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned atom_add_release_gpu(unsigned *p, unsigned v) {
    unsigned old;
    asm volatile("atom.add.release.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

/* Grid barriers of one launch, numbered k = 1..nbar.  gb[0] counts arrivals
 * (k*G after barrier k; reset to 0 by the last arrival of the last barrier),
 * gb[1] is a generation word read once at kernel start (sh.gen0): barrier k
 * is complete when it has advanced by k.  Arrival is one release atomic by
 * thread 0 after bar.sync, so the CTA's global writes are published; the last
 * arrival publishes the new generation. */
__device__ void grid_arrive(unsigned *gb, LayerShared &sh, uint32_t k, uint32_t nbar) {
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned target = k * gridDim.x;
        if (atom_add_release_gpu(gb, 1u) == target - 1) {
            if (k == nbar) gb[0] = 0u; /* nobody reads the count again in this launch */
            st_release_gpu(gb + 1, sh.gen0 + k);
        }
    }
}

/* Wait until barrier k is complete (bounded). */
__device__ bool grid_wait(unsigned *gb, LayerShared &sh, uint32_t k, uint32_t *err) {
    if (threadIdx.x == 0) {
        bool ok = true;
        const unsigned g0 = sh.gen0;
        if ((int)(ld_acquire_gpu(gb + 1) - g0) < (int)k) {
            const uint64_t t0 = lfm_globaltimer();
            while ((int)(ld_acquire_gpu(gb + 1) - g0) < (int)k) {
                if (lfm_globaltimer() - t0 > LFM_WAIT_LIMIT_NS) {
                    atomicOr(err, LFM_DEVERR_TIMEOUT);
                    ok = false;
                    break;
                }
            }
        }
        sh.ok = ok ? 1 : 0;
    }
    __syncthreads();
    return sh.ok != 0;
}

/* Operand entry (super-block lane h, token t, row group g) of a unit, written
 * over the consumed stage: 16 bytes at ((h*8 + (t^h))*4 + g)*16.  The XOR
 * skew makes both the integer lanes' stores (fixed t) and the chain lanes'
 * loads (fixed h) touch 8 distinct 16-byte bank groups per 8 lanes. */
__device__ __forceinline__ uint32_t opnd_off(int h, int t, int g) { return (uint32_t)(((h * 8 + (t ^ h)) * 4 + g) * 16); }

__device__ __forceinline__ void st_opnd(uint8_t *st, int h, int t, int g, const float4 &o) {
    const uint32_t a = lfm_smem_u32(st + opnd_off(h, t, g));
    asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(a), "f"(o.x), "f"(o.y), "f"(o.z), "f"(o.w) : "memory");
}

/* Integer phase of one unit (see k_gemv): operands written over the stage. */
template <int kNt>
__device__ __forceinline__ void unit_ints(const uint8_t *wsb, const uint8_t *rec, const uint32_t (&toff8)[kCh],
                                          bool act, uint8_t *st, int g, int h) {
    float4 o[kNt];
    uint32_t toff[kNt];
#pragma unroll
    for (int t = 0; t < kNt; ++t) toff[t] = toff8[t];
    if (act) lfm_q4k_sb<kNt, true, false>(wsb, rec, toff, o, nullptr);
    __syncwarp();
    if (act) {
#pragma unroll
        for (int t = 0; t < kNt; ++t) st_opnd(st, h, t, g, o[t]);
    }
    __syncwarp();
}

/* fp32 update chain of row group g, token t over the unit's n super-blocks
 * in order, from the operand entries (see lfm_q4k_chain). */
__device__ __forceinline__ float chain_swz(float sum, const uint8_t *st, int t, int g, uint32_t n) {
#pragma unroll
    for (int h = 0; h < 8; ++h) {
        if ((uint32_t)h < n) {
            const uint4 v = lfm_ld16<true>(st + opnd_off(h, t, g));
            sum = __fmaf_rn(__uint_as_float(v.x), __uint_as_float(v.y),
                            __fmaf_rn(-__uint_as_float(v.z), __uint_as_float(v.w), sum));
        }
    }
    return sum;
}

__device__ __forceinline__ void unit_dispatch(int nt, const uint8_t *wsb, const uint8_t *rec,
                                              const uint32_t (&toff)[kCh], bool act, uint8_t *st, int g, int h) {
    if (nt <= 1) unit_ints<1>(wsb, rec, toff, act, st, g, h);
    else if (nt <= 2) unit_ints<2>(wsb, rec, toff, act, st, g, h);
    else if (nt <= 3) unit_ints<3>(wsb, rec, toff, act, st, g, h);
    else if (nt <= 4) unit_ints<4>(wsb, rec, toff, act, st, g, h);
    else unit_ints<8>(wsb, rec, toff, act, st, g, h);
}

/* Biased top-K of token t, one warp, from sigmoid scores sg and selection
 * scores sl (= sg + exp_probs_b) of its E experts in shared memory
 * (tools/lfm2_moe_checkpoint.c:183-239; ties to the lowest index). */
__device__ void layer_topk(const MoeLayerDev &L, uint32_t t, const float *sg, const float *sl, LayerShared &sh) {
    const int lane = threadIdx.x & 31;
    const uint32_t E = L.E, K = L.K;
    float sig[8], sel[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t e = lane + 32u * i;
        sig[i] = e < E ? sg[e] : 0.0f;
        sel[i] = e < E ? sl[e] : -INFINITY;
    }
    float wk[LFM_GPU_MAX_TOPK_DEV];
    int ik[LFM_GPU_MAX_TOPK_DEV];
    for (uint32_t k = 0; k < K; ++k) {
        float bv = -1e30f;
        int bi = (int)E;
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
            sh.idx[t * K + k] = ik[k];
            sh.wk[t * K + k] = wk[k];
        }
    }
}

/* Items of pair j cost about kUnitCost + nt units of work (nt = its tokens);
 * CTAs take equal shares of the total.  split_count(target) = number of items
 * whose cost interval starts below target (monotone, so consecutive CTAs'
 * ranges tile the item list). */
constexpr uint32_t kUnitCost = 3;
__device__ uint32_t split_count(const LayerShared &sh, uint32_t P, uint32_t gpp, uint32_t target) {
    uint32_t cum = 0, n = 0;
    for (uint32_t j = 0; j < P; ++j) {
        const uint32_t w = kUnitCost + (uint32_t)sh.pnt[j];
        const uint32_t span = w * gpp;
        if (target >= cum + span) {
            n += gpp;
        } else {
            if (target > cum) n += (target - cum + w - 1) / w;
            break;
        }
        cum += span;
    }
    return n;
}

/* A warp's walk over items lo + w, lo + w + W, ... of [lo, hi): pair j and
 * item r within it, advanced without divisions. */
struct ItemCursor {
    uint32_t j, r, left;
    __device__ void init(uint32_t lo, uint32_t hi, uint32_t w, uint32_t W, uint32_t gpp) {
        const uint32_t n = hi > lo ? hi - lo : 0;
        left = n > w ? (n - w + W - 1) / W : 0;
        const uint32_t i = lo + w;
        j = i / gpp;
        r = i - j * gpp;
    }
    __device__ void next(uint32_t W, uint32_t gpp) {
        --left;
        r += W;
        while (r >= gpp) { r -= gpp; ++j; }
    }
};

__global__ void __launch_bounds__(kW * 32, 1) k_moe_layer(LayerArgs A) {
    extern __shared__ __align__(128) uint8_t dsm[];
    __shared__ LayerShared sh;
    const MoeLayerDev &L = A.L;
    const uint32_t T = A.T, D = L.D, I = L.I;
    const uint32_t E = L.dense ? 1u : L.E, K = lfm_layer_K(L);
    const uint32_t nbD = D / 256, nbI = I / 256;
    const uint32_t W = blockDim.x >> 5, S = A.S;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 3, h = lane & 7, l16 = lane & 15;
    const uint32_t rs_gu = min(nbD, kUnitSb) * LFM_Q4K_BYTES, rs_dn = min(nbI, kUnitSb) * LFM_Q4K_BYTES;
    const uint32_t stage_bytes = 4 * max(rs_gu, rs_dn);
    uint8_t *my_stages = dsm + (size_t)warp * S * stage_bytes;
    uint8_t *act = dsm + (size_t)W * S * stage_bytes; /* x records (gate|up), then h records (down) */
    const size_t dslot_bytes = lfm_act_slot_bytes(I);
    unsigned *gb = A.gbar;
    uint32_t *err = A.rt.err;

    /* ---- 0. bulk-copy x, ffn_norm and this CTA's router rows into the (idle) ring memory ---- */
    const uint32_t ndots = L.dense ? 0u : T * E; /* dot p = e*T + t: a CTA's dots share few experts */
    const uint32_t d0 = ndots * blockIdx.x / gridDim.x, d1 = ndots * (blockIdx.x + 1) / gridDim.x;
    const uint32_t e_lo = d0 < d1 ? d0 / T : 0u, nrows = d0 < d1 ? (d1 - 1) / T - e_lo + 1 : 0u;
    float *xs = reinterpret_cast<float *>(dsm);
    float *nw = xs + (size_t)T * D;
    float *bs = nw + D;                                  /* exp_probs_b, padded to 4 */
    const uint32_t nbias = L.dense || !L.bias ? 0u : (L.E + 3u) & ~3u;
    float *wsr = bs + nbias;
    if (lane == 0) {
        for (uint32_t s = 0; s < S; ++s) lfm_mbar_init(&sh.full[warp][s], 1);
        if (warp == 0) lfm_mbar_init(&sh.bar_in, 1);
        lfm_fence_mbar_init();
    }
    if (threadIdx.x == 0) {
        sh.abort = 0;
        sh.gen0 = ld_acquire_gpu(gb + 1); /* no barrier of this launch can complete before every CTA has started */
    }
    const uint32_t nbar = 3; /* records/scores exchange; all h written; all y written */
    uint32_t bar_k = 0;
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint32_t bytes = (T * D + (L.ffn_norm ? D : 0u) + nbias + nrows * D) * 4u;
        lfm_mbar_arrive_tx(&sh.bar_in, bytes);
        lfm_bulk_g2s_plain(xs, A.x, T * D * 4u, &sh.bar_in);
        if (L.ffn_norm) lfm_bulk_g2s_plain(nw, L.ffn_norm, D * 4u, &sh.bar_in);
        if (nbias) lfm_bulk_g2s_plain(bs, L.bias, nbias * 4u, &sh.bar_in);
        if (nrows) lfm_bulk_g2s_plain(wsr, L.router_w + (size_t)e_lo * D, nrows * D * 4u, &sh.bar_in);
    }
    bool alive = lfm_mbar_wait(&sh.bar_in, 0, err);

    /* ---- 1. RMSNorm; xb = (x*inv)*w in place; router logits and this CTA's
     *         share of the Q8_K records, both exchanged through global memory ---- */
    for (uint32_t t0 = 2u * warp; t0 < T; t0 += 2u * W) { /* warp-uniform: half-warp per token */
        const uint32_t t = t0 + (uint32_t)(lane >> 4);
        const bool valid = t < T && alive;
        float acc = 0.0f;
        if (valid) {
            const float *xt = xs + (size_t)t * D;
#pragma unroll 16
            for (uint32_t i = 0; i < D; i += 16) acc = __fmaf_rn(xt[i + l16], xt[i + l16], acc);
        }
        const float ss = lfm_hsum16_ref(acc);
        if (l16 == 0 && t < T) sh.inv_rms[t] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), L.eps)));
    }
    __syncthreads();
    for (uint32_t t = 0; t < T; ++t) {
        const float inv = sh.inv_rms[t];
        float *xt = xs + (size_t)t * D;
        for (uint32_t i = threadIdx.x; i < D; i += blockDim.x) {
            const float n = __fmul_rn(xt[i], inv);
            xt[i] = L.ffn_norm ? __fmul_rn(n, nw[i]) : n;
        }
    }
    __syncthreads();
    if (!L.dense) {
        for (uint32_t base = d0 + 2u * warp; base < d1; base += 2u * W) { /* warp-uniform trip count */
            const uint32_t p = base + (uint32_t)(lane >> 4);
            const bool valid = p < d1 && alive;
            const uint32_t e = valid ? p / T : e_lo, t = valid ? p - e * T : 0u;
            float acc = 0.0f;
            if (valid) {
                const float *xt = xs + (size_t)t * D, *wr = wsr + (size_t)(e - e_lo) * D;
#pragma unroll 16
                for (uint32_t i = 0; i < D; i += 16) acc = __fmaf_rn(wr[i + l16], xt[i + l16], acc);
            }
            const float z = lfm_hsum16_ref(acc);
            if (l16 == 0 && valid) {
                const float sgm = __fdiv_rn(1.0f, __fadd_rn(1.0f, lfm_expf(-z)));
                A.rt.logits[(size_t)t * E + e] = z;
                reinterpret_cast<float2 *>(A.scores)[(size_t)t * E + e] =
                    make_float2(sgm, nbias ? __fadd_rn(sgm, bs[e]) : sgm);
            }
        }
    }
    {
        const uint32_t nq = T * nbD;
        const uint32_t q0 = nq * blockIdx.x / gridDim.x, q1 = nq * (blockIdx.x + 1) / gridDim.x;
        for (uint32_t q = q0 + warp; q < q1; q += W) {
            const uint32_t t = q / nbD, b = q - t * nbD;
            const float *xp = xs + (size_t)t * D + 256 * b + 8 * lane;
            const float v[8] = {xp[0], xp[1], xp[2], xp[3], xp[4], xp[5], xp[6], xp[7]};
            lfm_quant_block_rec(v, act + (size_t)q * LFM_ACT_REC); /* build in shared, then publish */
            __syncwarp();
            const uint4 *src = reinterpret_cast<const uint4 *>(act + (size_t)q * LFM_ACT_REC);
            uint4 *dst = reinterpret_cast<uint4 *>(A.xrec + (size_t)q * LFM_ACT_REC);
            for (uint32_t c = lane; c < LFM_ACT_REC / 16; c += 32) dst[c] = src[c];
        }
    }
    grid_arrive(gb, sh, ++bar_k, nbar);
    alive = grid_wait(gb, sh, bar_k, err) && alive; /* also: every warp is done with xs */
    if (threadIdx.x == 0 && alive) { /* every row's records, from global into shared */
        asm volatile("fence.proxy.async.global;" ::: "memory"); /* generic-proxy writes, read by the bulk copy */
        const uint32_t bytes = T * nbD * LFM_ACT_REC;
        lfm_mbar_arrive_tx(&sh.bar_in, bytes);
        lfm_bulk_g2s_plain(act, A.xrec, bytes, &sh.bar_in);
    }

    /* ---- 2. routing and dispatch tables (identical in every CTA) ---- */
    if (!L.dense) {
        float *sg = wsr, *sl = sg + (size_t)T * E; /* x / norm / router rows are no longer needed */
        for (uint32_t q = threadIdx.x; q < T * E; q += blockDim.x) {
            const float2 v = __ldcg(reinterpret_cast<const float2 *>(A.scores) + q);
            sg[q] = v.x;
            sl[q] = v.y;
        }
        __syncthreads();
        for (uint32_t t = warp; t < T; t += W) layer_topk(L, t, sg + (size_t)t * E, sl + (size_t)t * E, sh);
    } else {
        for (uint32_t t = threadIdx.x; t < T; t += blockDim.x) { sh.idx[t] = 0; sh.wk[t] = 1.0f; }
    }
    __syncthreads();
    const uint32_t n_as = T * K;
    const uint32_t gpp_gu = I / 2, gpp_dn = D / 4;
    if (warp == 0) {
        /* counts and, in assignment order, each assignment's rank within its expert */
        for (uint32_t e = lane; e < E; e += 32) sh.cnt[e] = 0;
        __syncwarp();
        for (uint32_t base = 0; base < n_as; base += 32) {
            const uint32_t a = base + lane;
            int e = a < n_as ? sh.idx[a] : -1;
            if (a < n_as && (unsigned)e >= E) { atomicOr(err, LFM_DEVERR_EXPERT_ID); e = -1; }
            const int key = e >= 0 ? e : -2 - lane; /* unmatched for invalid slots */
            const unsigned m = __match_any_sync(LFM_FULL_MASK, key);
            const int r = __popc(m & ((1u << lane) - 1u));
            if (e >= 0) sh.inv[a] = sh.cnt[e] + r; /* rank, turned into the slot below */
            __syncwarp();
            if (e >= 0 && 31 - __clz(m) == lane) sh.cnt[e] += __popc(m);
            __syncwarp();
        }
        /* lane l owns experts 8l .. 8l+7: offsets and pair list by warp scans */
        int c[8], csum = 0, psum = 0, mx = 0, uq = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t e = 8u * lane + j;
            c[j] = e < E ? sh.cnt[e] : 0;
            csum += c[j];
            psum += (c[j] + kCh - 1) / kCh;
            mx = max(mx, c[j]);
            uq += c[j] > 0;
        }
        int cex = csum, pex = psum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int x1 = __shfl_up_sync(LFM_FULL_MASK, cex, o), x2 = __shfl_up_sync(LFM_FULL_MASK, pex, o);
            if (lane >= o) { cex += x1; pex += x2; }
        }
        cex -= csum; /* exclusive */
        pex -= psum;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t e = 8u * lane + j;
            if (e < E) sh.off[e] = cex;
            for (int s0 = 0; s0 < c[j]; s0 += kCh) {
                sh.pe[pex] = (int)e;
                sh.ps0[pex] = cex + s0;
                sh.pnt[pex] = min(kCh, c[j] - s0);
                ++pex;
            }
            cex += c[j];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            mx = max(mx, __shfl_xor_sync(LFM_FULL_MASK, mx, o));
            uq += __shfl_xor_sync(LFM_FULL_MASK, uq, o);
        }
        const int np_all = __shfl_sync(LFM_FULL_MASK, pex, 31), total = __shfl_sync(LFM_FULL_MASK, cex, 31);
        if (lane == 31) {
            sh.off[E] = cex;
            sh.npairs = pex;
            if (blockIdx.x == 0) {
                A.rt.summary[0] = uq;
                A.rt.summary[1] = mx;
                A.rt.summary[2] = cex;
                A.rt.summary[3] = pex;
                if (A.rt.loads && !L.dense) { atomicAdd(A.rt.loads, (unsigned long long)uq); atomicAdd(A.rt.loads + 1, 1ull); }
            }
        }
        __syncwarp();
        for (uint32_t a = lane; a < n_as; a += 32) {
            const int e = sh.idx[a];
            int pos = -1;
            if ((unsigned)e < E) {
                pos = sh.off[e] + sh.inv[a];
                sh.perm[pos] = (int)a;
                sh.tok[pos] = (int)(a / K);
            }
            sh.inv[a] = pos;
            if (blockIdx.x == 0) {
                A.rt.idx[a] = e;
                A.rt.w[a] = sh.wk[a];
            }
        }
        (void)total;
        if (lane < 4) { /* this CTA's cost-weighted item ranges (totals < 2^32: P*gpp*11) */
            const uint32_t P = (uint32_t)np_all;
            const uint32_t gpp = lane < 2 ? gpp_gu : gpp_dn;
            uint32_t tot = 0;
            for (uint32_t j = 0; j < P; ++j) tot += (kUnitCost + (uint32_t)sh.pnt[j]) * gpp;
            const uint32_t bb = blockIdx.x + (lane & 1);
            const uint32_t n = split_count(sh, P, gpp, (uint32_t)((uint64_t)tot * bb / gridDim.x));
            if (lane == 0) sh.gu_lo = n;
            else if (lane == 1) sh.gu_hi = n;
            else if (lane == 2) sh.dn_lo = n;
            else sh.dn_hi = n;
        }
    }
    __syncthreads();

    if (alive) alive = lfm_mbar_wait(&sh.bar_in, 1, err); /* the records copied after barrier 1 */

    /* ---- 3. per-warp unit streams: gate|up units, then down units ---- */
    const uint32_t np_gu = (nbD + kUnitSb - 1) / kUnitSb, np_dn = (nbI + kUnitSb - 1) / kUnitSb;
    const uint32_t gu_lo = sh.gu_lo, gu_hi = sh.gu_hi, dn_lo = sh.dn_lo, dn_hi = sh.dn_hi;
    const uint64_t policy = lfm_policy_evict_first();
    /* producer (lane 0): its own cursors, pass and stage */
    ItemCursor pc;
    pc.init(gu_lo, gu_hi, warp, W, gpp_gu);
    bool p_gu = true;
    if (pc.left == 0) { p_gu = false; pc.init(dn_lo, dn_hi, warp, W, gpp_dn); }
    uint32_t p_pass = 0, p_stage = 0, in_flight = 0;
    auto issue = [&]() {
        if (pc.left == 0) return;
        const uint32_t npass = p_gu ? np_gu : np_dn, R = p_gu ? 2u : 4u, nb = p_gu ? nbD : nbI;
        const uint32_t rows_total = p_gu ? I : D, rs = p_gu ? rs_gu : rs_dn;
        const size_t row_bytes = (size_t)nb * LFM_Q4K_BYTES;
        const size_t row0 = (size_t)sh.pe[pc.j] * rows_total + (size_t)pc.r * R;
        const uint32_t nsb = min(kUnitSb, nb - kUnitSb * p_pass);
        const uint32_t seg = nsb * LFM_Q4K_BYTES;
        uint64_t *bar = &sh.full[warp][p_stage];
        uint8_t *dst = my_stages + (size_t)p_stage * stage_bytes;
        lfm_mbar_arrive_tx(bar, 4u * seg);
        for (uint32_t m = 0; m < (p_gu ? 2u : 1u); ++m) {
            const uint8_t *base = p_gu ? (m == 0 ? L.gate : L.up) : L.down;
            const uint8_t *src = base + row0 * row_bytes + (size_t)p_pass * kUnitSb * LFM_Q4K_BYTES;
            uint8_t *d = dst + (size_t)m * R * rs;
            if (npass == 1) {
                lfm_bulk_g2s(d, src, R * (uint32_t)row_bytes, bar, policy);
            } else {
                for (uint32_t r = 0; r < R; ++r) lfm_bulk_g2s(d + (size_t)r * rs, src + (size_t)r * row_bytes, seg, bar, policy);
            }
        }
        ++in_flight;
        p_stage = p_stage + 1 == S ? 0 : p_stage + 1;
        if (++p_pass == npass) {
            p_pass = 0;
            pc.next(W, p_gu ? gpp_gu : gpp_dn);
            if (pc.left == 0 && p_gu) { p_gu = false; pc.init(dn_lo, dn_hi, warp, W, gpp_dn); }
        }
    };
    if (lane == 0 && alive)
        for (uint32_t s = 0; s < S; ++s) issue();

    /* consumer: stage and parity of the next unit */
    uint32_t c_stage = 0, c_par = 0;
    bool stop = !alive;
    auto run_unit = [&](int nt, uint32_t rs, uint32_t nb, uint32_t p, const uint8_t *rec_base,
                        const uint32_t (&toff)[kCh], float &run) -> bool {
        bool ok = !ld_volatile_int(&sh.abort) && lfm_mbar_wait(&sh.full[warp][c_stage], c_par, err);
        ok = __all_sync(LFM_FULL_MASK, ok);
        if (!ok) {
            if (lane == 0) atomicExch(&sh.abort, 1);
            return false;
        }
        uint8_t *st = my_stages + (size_t)c_stage * stage_bytes;
        const uint32_t nsb = min(kUnitSb, nb - kUnitSb * p);
        unit_dispatch(nt, st + (size_t)g * rs + (size_t)h * LFM_Q4K_BYTES,
                      rec_base + (size_t)(kUnitSb * p + h) * LFM_ACT_REC, toff, (uint32_t)h < nsb, st, g, h);
        if (h < nt) run = chain_swz(run, st, h, g, nsb);
        __syncwarp(); /* stage free again */
        if (++c_stage == S) { c_stage = 0; c_par ^= 1u; }
        if (lane == 0) {
            --in_flight;
            issue();
        }
        return true;
    };

    /* gate|up: activations are the records of all T tokens */
    {
        ItemCursor cc;
        cc.init(gu_lo, gu_hi, warp, W, gpp_gu);
        while (cc.left > 0 && !stop) {
            const int nt = sh.pnt[cc.j], slot0 = sh.ps0[cc.j];
            const uint32_t row0 = cc.r * 2;
            uint32_t toff[kCh];
#pragma unroll
            for (int t = 0; t < kCh; ++t) toff[t] = (uint32_t)sh.tok[slot0 + (t < nt ? t : 0)] * nbD * LFM_ACT_REC;
            float run = 0.0f;
            for (uint32_t p = 0; p < np_gu && !stop; ++p)
                if (!run_unit(nt, rs_gu, nbD, p, act, toff, run)) stop = true;
            if (stop) break;
            const float u = __shfl_down_sync(LFM_FULL_MASK, run, 16);
            if (lane < 16 && h < nt) {
                const float silu = __fdiv_rn(run, __fadd_rn(1.0f, lfm_silu_expf(-run)));
                A.h[(size_t)(slot0 + h) * I + row0 + g] = __fmul_rn(silu, u);
            }
            cc.next(W, gpp_gu);
        }
    }
    grid_arrive(gb, sh, ++bar_k, nbar);
    alive = grid_wait(gb, sh, bar_k, err) && alive;
    if (!alive) stop = true;

    /* ---- 4. down: h rows of the CTA's pairs as Q8_K records, then the items ---- */
    if (alive && dn_lo < dn_hi) {
        const uint32_t j_first = dn_lo / gpp_dn, j_last = (dn_hi - 1) / gpp_dn;
        ItemCursor cc;
        cc.init(dn_lo, dn_hi, warp, W, gpp_dn);
        for (uint32_t jp = j_first; jp <= j_last; jp += A.dslots) {
            const uint32_t np = min(A.dslots, j_last - jp + 1);
            __syncthreads(); /* the previous phase's records are no longer read */
            for (uint32_t task = warp; task < np * kCh * nbI; task += W) {
                const uint32_t q = task / (kCh * nbI), r = task - q * (kCh * nbI), t = r / nbI, b = r - t * nbI;
                if ((int)t < sh.pnt[jp + q]) {
                    const float4 *hp = reinterpret_cast<const float4 *>(A.h + (size_t)(sh.ps0[jp + q] + t) * I + 256 * b + 8 * lane);
                    const float4 a0 = __ldcg(hp), a1 = __ldcg(hp + 1);
                    const float vv[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                    lfm_quant_block_rec(vv, act + q * dslot_bytes + ((size_t)t * nbI + b) * LFM_ACT_REC);
                }
            }
            __syncthreads();
            while (cc.left > 0 && cc.j < jp + np) {
                if (!stop) {
                    const int nt = sh.pnt[cc.j], slot0 = sh.ps0[cc.j];
                    const uint32_t row0 = cc.r * 4;
                    uint32_t toff[kCh];
#pragma unroll
                    for (int t = 0; t < kCh; ++t) toff[t] = (uint32_t)(t < nt ? t : 0) * nbI * LFM_ACT_REC;
                    float run = 0.0f;
                    for (uint32_t p = 0; p < np_dn && !stop; ++p)
                        if (!run_unit(nt, rs_dn, nbI, p, act + (cc.j - jp) * dslot_bytes, toff, run)) stop = true;
                    if (!stop && h < nt) A.y[(size_t)(slot0 + h) * D + row0 + g] = run;
                }
                cc.next(W, gpp_dn);
            }
        }
    }
    grid_arrive(gb, sh, ++bar_k, nbar);
    alive = grid_wait(gb, sh, bar_k, err) && alive;

    /* ---- 5. combine: this CTA's slice of x ---- */
    if (alive) {
        const uint32_t n = T * D;
        const uint32_t c0 = n * blockIdx.x / gridDim.x, c1 = n * (blockIdx.x + 1) / gridDim.x;
        for (uint32_t q = c0 + threadIdx.x; q < c1; q += blockDim.x) {
            const uint32_t t = q / D, r = q - t * D;
            float acc = A.x[q];
            for (uint32_t kk = 0; kk < K; ++kk) {
                const int slot = sh.inv[t * K + kk];
                if (slot >= 0) acc = __fmaf_rn(sh.wk[t * K + kk], __ldcg(A.y + (size_t)slot * D + r), acc);
            }
            A.x[q] = acc;
        }
    }
    /* leave no copy in flight into this CTA's shared memory */
    if (lane == 0)
        for (; in_flight > 0; --in_flight) {
            lfm_mbar_wait(&sh.full[warp][c_stage], c_par, err);
            if (++c_stage == S) { c_stage = 0; c_par ^= 1u; }
        }
}

struct FusedPlan {
    uint32_t warps, stages, dslots;
    size_t smem;
};

FusedPlan fused_plan(const MoeLayerDev &L, uint32_t T, uint32_t grid) {
    FusedPlan none{0, 0, 0, 0};
    const uint32_t K = lfm_layer_K(L);
    if (T == 0 || T > (uint32_t)kMaxT || T * K > (uint32_t)kMaxTK) return none;
    if (!L.dense && (L.E > LFM_GPU_MAX_EXPERTS_DEV || L.E < 1)) return none;
    const uint32_t nbD = L.D / 256, nbI = L.I / 256;
    const size_t stage = 4 * (size_t)(nbD > nbI ? min(nbD, kUnitSb) : min(nbI, kUnitSb)) * LFM_Q4K_BYTES;
    const size_t x_rec = (size_t)T * nbD * LFM_ACT_REC;
    for (uint32_t want = 3; want >= 2; --want) {
        for (uint32_t dslots = 2; dslots >= 1; --dslots) {
            const size_t act = max(x_rec, (size_t)dslots * lfm_act_slot_bytes(L.I));
            for (uint32_t w = kW; w >= 8; --w) {
                if (act >= kSmemBudget) continue;
                uint32_t s = (uint32_t)((kSmemBudget - act) / ((size_t)w * stage));
                if (s > kMaxS) s = kMaxS;
                if (s < want) continue;
                const size_t ring = (size_t)w * s * stage;
                /* the ring memory first holds x, ffn_norm, bias and the CTA's router rows, then the scores */
                const uint32_t dots = L.dense ? 0u : T * L.E;
                const uint32_t rows = dots ? (dots + grid - 1) / grid / T + 2 : 0u;
                const size_t head = ((size_t)T * L.D + L.D + ((L.E + 3) & ~3u)) * 4; /* x, ffn_norm, bias */
                if (ring < head + (size_t)rows * L.D * 4 || ring < head + (size_t)2 * T * L.E * 4) continue;
                return FusedPlan{w, s, dslots, ring + act};
            }
        }
    }
    return none;
}

}  // namespace

bool lfm_fused_ok(const MoeLayerDev &L, uint32_t T, int grid) { return fused_plan(L, T, (uint32_t)grid).warps != 0; }

cudaError_t lfm_launch_layer_fused(const MoeLayerDev &L, float *x, uint32_t T, const RouteTables &rt, float *h,
                                   float *y, unsigned *gbar, uint8_t *xrec, float *scores, int grid, cudaStream_t s) {
    const FusedPlan pl = fused_plan(L, T, (uint32_t)grid);
    if (pl.warps == 0) return cudaErrorInvalidValue;
    static size_t cache[16];
    cudaError_t e = lfm_smem_attr((const void *)k_moe_layer, pl.smem, cache);
    if (e != cudaSuccess) return e;
    LayerArgs a{L, x, T, rt, h, y, gbar, xrec, scores, pl.stages, pl.dslots};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(pl.warps * 32);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_moe_layer, a);
}
