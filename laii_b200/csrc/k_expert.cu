/*
 * K3 grouped Q4_K expert GEMVs and K4 combine (decode / verify path).
 *
 * Work: the dispatch tables list (active expert u, 8-token chunk c) pairs.
 * Each pair's weight rows are split in items of 8 rows; the flattened list of
 * (pair, item) is cut into one contiguous range per block of a persistent grid
 * (one block per SM).  Within a block:
 *   - a producer warp streams each item's rows (8 gate + 8 up rows for K3a,
 *     8 down rows for K3b: 1152 B / 1008 B per row at D=2048 / I=1792) into a
 *     ring of shared-memory stages with 1-D bulk copies (cp.async.bulk on the
 *     TMA engine, evict-first L2 policy) completing on mbarriers;
 *   - consumer warp w takes items w, w+8, ... of the block through stages it
 *     owns (consumed in order); one warp computes a whole item with lfm_q4k_rows8 (4 lanes per row, super-blocks in order,
 *     exact integer sub-block sums, the reference's fp32 update order), the
 *     chunk's activations read through the read-only cache;
 *   - gate|up: h = (g / (1 + exp(-g))) * u   (tools/lfm2_decode_1x4.c:976-985);
 *   - down: y[slot][r].
 * k_quant_rows then makes Q8_K(h) per 256 (tools/lfm2_cpuid_quants.c:584-631)
 * and k_combine applies x[t][r] = fma(w_k, y[slot(t,k)][r], x[t][r]) for
 * k = 0..K-1 in order (tools/lfm2_moe_checkpoint.c:266-269, :338-364); all
 * kernels chain with programmatic dependent launch.
 * Every mbarrier wait is bounded (lfm_mbar_wait); after a timeout the block
 * stops issuing copies, lets the ones in flight land, and leaves its range
 * with the device error word set.
 */
#include "moe_device.cuh"
#include "moe_internal.h"

namespace {

/* gate|up: 8 warp pairs (gate warp + up warp per item); down: 12 warps. */
template <int kMats> struct GemvShape {
    static constexpr int kConsumers = kMats == 2 ? 16 : 12;  /* consumer warps */
    static constexpr int kPerItem = kMats;                    /* warps sharing one item */
    static constexpr int kThreads = (kConsumers + 1) * 32;
    static constexpr int kActSlots = kMats == 2 ? 2 : 3;      /* (expert, chunk) pairs staged per phase */
};
constexpr int kRows = LFM_GEMV_ROWS; /* rows per item (8) */
constexpr int kCh = LFM_GEMV_CHUNK;
constexpr int kMaxStages = 32;

__device__ __forceinline__ int ld_volatile(const int *p) { return *reinterpret_cast<const volatile int *>(p); }

struct GemvShared {
    uint64_t full[kMaxStages];
    uint64_t empty[kMaxStages];
    float gx[8][kRows][kCh]; /* gate results handed from the gate warp to the up warp of a pair */
    int pair_ok[8][2];        /* per-pair go/no-go, written only by that pair's two warps */
    int abort;
};

struct GemvArgs {
    MoeLayerDev L;
    Q8Rows act;        /* activation rows: xq (token-indexed) or hq (slot-indexed) */
    RouteTables rt;
    float *out;        /* h [slots][I] or y [slots][D] */
    uint32_t stages;   /* stages in use = groups * depth */
    uint32_t groups;   /* active consumer groups (warp pairs for gate|up, warps for down) */
    uint32_t slots;    /* activation slots (pairs staged per phase), 1..kActSlots */
    int next_down;     /* gate|up: prefetch the down rows of the next kernel into L2 */
};

/* Dynamic shared memory: [stages][kMats][8 rows][row stride] weights, then
 * kActSlots activation slots. */

template <int kMats>
__global__ void __launch_bounds__(GemvShape<kMats>::kThreads, 1) k_gemv(GemvArgs A) {
    using Sh = GemvShape<kMats>;
    extern __shared__ __align__(128) uint8_t dsm[];
    __shared__ GemvShared sh;
    const MoeLayerDev &L = A.L;
    const uint32_t rows_total = kMats == 2 ? L.I : L.D;
    const uint32_t cols = kMats == 2 ? L.D : L.I;
    const uint32_t nb = cols / 256;
    const uint32_t row_bytes = nb * LFM_Q4K_BYTES;
    const uint32_t rs = lfm_stage_stride(row_bytes);
    const uint32_t stage_bytes = kMats * kRows * rs;
    const uint32_t G = A.groups;          /* consumer groups in use */
    const uint32_t depth = A.stages / G;  /* private stages per group */
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t K = lfm_layer_K(L);

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < A.stages; ++s) {
            lfm_mbar_init(&sh.full[s], 1);
            lfm_mbar_init(&sh.empty[s], 1);
        }
        sh.abort = 0;
        lfm_fence_mbar_init();
    }
    __syncthreads();
    lfm_pdl_launch_dependents();
    lfm_pdl_wait(); /* routing tables and activations come from the preceding kernels */

    const uint32_t gpp = rows_total / kRows; /* items per (expert, chunk) pair */
    const uint64_t n_items = (uint64_t)__ldcg(A.rt.summary + 3) * gpp;
    const uint64_t i0 = n_items * blockIdx.x / gridDim.x;
    const uint64_t i1 = n_items * (blockIdx.x + 1) / gridDim.x;
    const uint8_t *W0 = kMats == 2 ? L.gate : L.down;
    const uint8_t *W1 = L.up;

    /* Stage ownership: local item k belongs to group k%G, which owns stages
     * (k%G)*depth .. +depth-1 and consumes them strictly in order, so no wait
     * can target a phase two ahead of a barrier (parity waits would alias). */
    auto stage_of = [&](uint64_t k, uint32_t &ph) -> uint32_t {
        const uint64_t q = k / G;
        ph = (uint32_t)(q / depth);
        return (uint32_t)(k % G) * depth + (uint32_t)(q % depth);
    };

    if (warp == Sh::kConsumers) {
        /* ---------------- producer ---------------- */
        if (lane == 0) {
            const uint64_t policy = lfm_policy_evict_first();
            uint64_t k = 0, pj = ~0ull;
            int e = 0;
            for (uint64_t i = i0; i < i1; ++i, ++k) {
                if (i / gpp != pj) { /* the expert changes once per gpp items */
                    pj = i / gpp;
                    e = __ldcg(A.rt.act + __ldcg(A.rt.pairs + pj).x);
                }
                uint32_t ph;
                const uint32_t s = stage_of(k, ph);
                if (ph >= 1 && !lfm_mbar_wait(&sh.empty[s], (ph - 1) & 1u, A.rt.err)) {
                    atomicExch(&sh.abort, 1);
                    break;
                }
                if (ld_volatile(&sh.abort)) break;
                const size_t row0 = (size_t)e * rows_total + (size_t)(i % gpp) * kRows;
                uint8_t *dst = dsm + (size_t)s * stage_bytes;
                lfm_mbar_arrive_tx(&sh.full[s], kMats * kRows * row_bytes);
                for (int m = 0; m < kMats; ++m)
                    lfm_bulk_g2s(dst + (size_t)m * kRows * rs, (m == 0 ? W0 : W1) + row0 * row_bytes,
                                 kRows * row_bytes, &sh.full[s], policy);
                /* the item that refills this stage next round: start its HBM read now */
                const uint64_t ia = i + (uint64_t)G * depth;
                if (ia < i1) {
                    const uint64_t pa = ia / gpp;
                    const int ea = pa == pj ? e : __ldcg(A.rt.act + __ldcg(A.rt.pairs + pa).x);
                    const size_t rowa = (size_t)ea * rows_total + (size_t)(ia % gpp) * kRows;
                    for (int m = 0; m < kMats; ++m)
                        lfm_prefetch_l2((m == 0 ? W0 : W1) + rowa * row_bytes, kRows * row_bytes);
                }
            }
            if (kMats == 2 && A.next_down) {
                /* warm L2 with the rows this block will stream in the down kernel
                 * (same pair list and block partition there) */
                const uint32_t nbd = L.I / 256, dbytes = nbd * LFM_Q4K_BYTES;
                const uint64_t gd = L.D / kRows, nd = (uint64_t)__ldcg(A.rt.summary + 3) * gd;
                const uint64_t d0 = nd * blockIdx.x / gridDim.x, d1 = nd * (blockIdx.x + 1) / gridDim.x;
                uint64_t pd = ~0ull;
                int ed = 0;
                for (uint64_t q = d0; q < d1; ++q) {
                    if (q / gd != pd) { pd = q / gd; ed = __ldcg(A.rt.act + __ldcg(A.rt.pairs + pd).x); }
                    lfm_prefetch_l2(L.down + ((size_t)ed * L.D + (size_t)(q % gd) * kRows) * dbytes, kRows * dbytes);
                }
            }
            /* leave no copy in flight into this block's shared memory: the last
             * G*depth items issued cover every stage's newest phase */
            const uint64_t span = (uint64_t)G * depth;
            for (uint64_t q = k > span ? k - span : 0; q < k; ++q) {
                uint32_t ph;
                const uint32_t s = stage_of(q, ph);
                lfm_mbar_wait(&sh.full[s], ph & 1u, A.rt.err);
            }
        }
        return;
    }

    /* ---------------- consumers ---------------- */
    const uint32_t grp = (uint32_t)warp / Sh::kPerItem;  /* consumer group */
    const int mat = warp % Sh::kPerItem;                  /* gate|up: 0 gate, 1 up */
    if (grp >= G) return;
    const int r = lane >> 2, g = lane & 3;
    const int n_cons = (int)G * Sh::kPerItem * 32;        /* threads in the consumer barrier */
    const int ctid = threadIdx.x;
    uint8_t *act_base = dsm + (size_t)A.stages * stage_bytes;
    const size_t slot_bytes = lfm_act_slot_bytes(cols);
    __shared__ int s_rows[Sh::kActSlots][kCh]; /* A.slots <= kActSlots */
    __shared__ int s_nt[Sh::kActSlots], s_slot0[Sh::kActSlots];
    bool stop = false;
    if (i0 < i1) {
        const uint64_t j_first = i0 / gpp, j_last = (i1 - 1) / gpp;
        for (uint64_t jp = j_first; jp <= j_last; jp += A.slots) {
            const uint32_t np = (uint32_t)min((uint64_t)A.slots, j_last - jp + 1);
            /* stage this phase's pairs */
            lfm_bar_sync(15, n_cons); /* previous phase fully consumed */
            if (ctid < (int)np) {
                const int2 pr = __ldcg(A.rt.pairs + jp + ctid);
                const uint32_t e = (uint32_t)__ldcg(A.rt.act + pr.x);
                const int n_e = __ldcg(A.rt.counts + e);
                const int off_e = __ldcg(A.rt.offsets + e);
                s_slot0[ctid] = off_e + pr.y * kCh;
                s_nt[ctid] = min(kCh, n_e - pr.y * kCh);
            }
            lfm_bar_sync(15, n_cons);
            if (ctid < (int)np * kCh) {
                const int q = ctid / kCh, t = ctid % kCh;
                s_rows[q][t] = t < s_nt[q] ? (kMats == 2 ? __ldcg(A.rt.perm + s_slot0[q] + t) / (int)K : s_slot0[q] + t) : 0;
            }
            lfm_bar_sync(15, n_cons);
            for (uint32_t q = 0; q < np; ++q)
                lfm_stage_act(A.act, s_rows[q], s_nt[q], act_base + q * slot_bytes, ctid, n_cons);
            lfm_bar_sync(15, n_cons);

            /* this phase's items, round-robin over groups (k = local item index) */
            const uint64_t ia = max(i0, jp * gpp), ib = min(i1, (jp + np) * gpp);
            uint64_t k = ia - i0;
            k += (grp + G - (uint32_t)(k % G)) % G;
            for (; i0 + k < ib; k += G) {
                const uint64_t i = i0 + k;
                const uint32_t q = (uint32_t)(i / gpp - jp);
                const int nt = s_nt[q], slot0 = s_slot0[q];
                uint32_t ph;
                const uint32_t s = stage_of(k, ph);
                bool ok = !stop && !ld_volatile(&sh.abort) && lfm_mbar_wait(&sh.full[s], ph & 1u, A.rt.err);
                ok = __all_sync(LFM_FULL_MASK, ok); /* the row dots shuffle across the whole warp */
                if (kMats == 2) {
                    /* both warps of the pair decide together from slots only they write,
                     * so they always take the same number of pair barriers */
                    if (lane == 0) sh.pair_ok[grp][mat] = ok ? 1 : 0;
                    lfm_bar_sync(1 + (int)grp, 64);
                    ok = sh.pair_ok[grp][0] && sh.pair_ok[grp][1];
                    lfm_bar_sync(1 + (int)grp, 64); /* both read the slots before either rewrites them */
                }
                if (!ok) {
                    /* keep walking the phase (barriers stay balanced) but do no more work */
                    if (lane == 0) atomicExch(&sh.abort, 1);
                    stop = true;
                    continue;
                }
                const uint8_t *st = dsm + (size_t)s * stage_bytes + (size_t)mat * kRows * rs;
                const uint32_t row0 = (uint32_t)(i % gpp) * kRows;
                const ActSmem av = lfm_act_slot(act_base + q * slot_bytes, cols);
                float s0[kCh], s1[kCh];
                lfm_q4k_rows8<1, false>(st, nullptr, rs, av, nt, s0, s1, RowDebug{});
                if (kMats == 2) {
                    if (mat == 0) {
#pragma unroll
                        for (int t = 0; t < kCh; ++t)
                            if ((t & 3) == g && t < nt) sh.gx[grp][r][t] = s0[t];
                    }
                    lfm_bar_sync(1 + (int)grp, 64); /* gate results visible; both warps done with the stage */
                    if (mat == 1) {
                        if (lane == 0) lfm_mbar_arrive(&sh.empty[s]);
#pragma unroll
                        for (int t = 0; t < kCh; ++t) {
                            if ((t & 3) == g && t < nt) {
                                const float gv = sh.gx[grp][r][t];
                                const float silu = __fdiv_rn(gv, __fadd_rn(1.0f, lfm_expf(-gv)));
                                A.out[(size_t)(slot0 + t) * L.I + row0 + r] = __fmul_rn(silu, s0[t]);
                            }
                        }
                    }
                } else {
                    __syncwarp();
                    if (lane == 0) lfm_mbar_arrive(&sh.empty[s]);
#pragma unroll
                    for (int t = 0; t < kCh; ++t)
                        if ((t & 3) == g && t < nt) A.out[(size_t)(slot0 + t) * L.D + row0 + r] = s0[t];
                }
            }
        }
    }
}

/* Q8_K of fp32 rows: one warp per 256-element block. */
__global__ void __launch_bounds__(256) k_quant_rows(const float *__restrict__ src, uint32_t rows, uint32_t cols,
                                                    Q8Rows dst) {
    lfm_pdl_launch_dependents();
    lfm_pdl_wait();
    const uint32_t nb = cols / 256;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t gw = blockIdx.x * 8 + warp;
    if (gw >= rows * nb) return;
    const uint32_t r = gw / nb, b = gw % nb;
    const float4 *p = reinterpret_cast<const float4 *>(src + (size_t)r * cols + 256 * b + 8 * lane);
    const float4 a0 = __ldcg(p), a1 = __ldcg(p + 1);
    const float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    lfm_quant_block_warp(v, dst, r, b);
}

/* Combine: x[t][r] = fma chain over k in order.  Block (rb, t) covers 4
 * consecutive columns per thread (float4); all K loads are issued first. */
__global__ void __launch_bounds__(128) k_combine(float *__restrict__ x, uint32_t D, uint32_t K, RouteTables rt,
                                                 const float *__restrict__ y) {
    lfm_pdl_launch_dependents();
    lfm_pdl_wait();
    const uint32_t t = blockIdx.y;
    const uint32_t r = (blockIdx.x * 128 + threadIdx.x) * 4;
    if (r >= D) return;
    int sl[LFM_GPU_MAX_TOPK_DEV];
    float wk[LFM_GPU_MAX_TOPK_DEV];
    float4 yv[LFM_GPU_MAX_TOPK_DEV];
#pragma unroll
    for (int k = 0; k < LFM_GPU_MAX_TOPK_DEV; ++k) {
        if (k < (int)K) {
            sl[k] = __ldcg(rt.inv + (size_t)t * K + k);
            wk[k] = __ldcg(rt.w + (size_t)t * K + k);
        }
    }
#pragma unroll
    for (int k = 0; k < LFM_GPU_MAX_TOPK_DEV; ++k)
        if (k < (int)K && sl[k] >= 0) yv[k] = __ldcg(reinterpret_cast<const float4 *>(y + (size_t)sl[k] * D + r));
    float4 v = *reinterpret_cast<float4 *>(x + (size_t)t * D + r);
#pragma unroll
    for (int k = 0; k < LFM_GPU_MAX_TOPK_DEV; ++k) {
        if (k < (int)K && sl[k] >= 0) {
            v.x = __fmaf_rn(wk[k], yv[k].x, v.x);
            v.y = __fmaf_rn(wk[k], yv[k].y, v.y);
            v.z = __fmaf_rn(wk[k], yv[k].z, v.z);
            v.w = __fmaf_rn(wk[k], yv[k].w, v.w);
        }
    }
    *reinterpret_cast<float4 *>(x + (size_t)t * D + r) = v;
}

/* Debug: every (vector, 8-row block) through lfm_q4k_rows8 with its integer parts. */
__global__ void __launch_bounds__(256) k_debug_rows(const uint8_t *__restrict__ w, uint32_t n_rows, uint32_t n_cols,
                                                    Q8Rows xq, int32_t *sub_dots, int32_t *acc, int32_t *mins,
                                                    float *rows_out) {
    extern __shared__ __align__(128) uint8_t slot[];
    __shared__ int vrow[kCh];
    const uint32_t nb = n_cols / 256;
    const uint32_t v = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t row_bytes = (size_t)nb * LFM_Q4K_BYTES;
    if (threadIdx.x < kCh) vrow[threadIdx.x] = (int)v;
    __syncthreads();
    lfm_stage_act(xq, vrow, 1, slot, threadIdx.x, blockDim.x);
    __syncthreads();
    const ActSmem av = lfm_act_slot(slot, n_cols);
    for (uint32_t rb = (blockIdx.y * 8 + warp) * kRows; rb < n_rows; rb += gridDim.y * 8 * kRows) {
        const size_t o = (size_t)v * n_rows + rb;
        RowDebug dbg{sub_dots + o * nb * 8, acc + o * nb, mins + o * nb};
        float s0[kCh], s1[kCh];
        lfm_q4k_rows8<1, true, false>(w + rb * row_bytes, nullptr, (uint32_t)row_bytes, av, 1, s0, s1, dbg);
        if ((lane & 3) == 0) rows_out[o + (lane >> 2)] = s0[0];
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

cudaError_t launch_ex(const void *fn, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl, void **args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

constexpr size_t kSmemBudget = 220 * 1024;

/* Consumer groups and stages: as many groups as stages allow (at most the
 * kernel's), then a whole number of private stages per group. */
/* Activation slots, consumer groups and stages: the most slots that still
 * leave stages for at least 4 groups (else one slot), as many groups as the
 * remaining stages allow (at most the kernel's), then a whole number of
 * private stages per group. */
void gemv_plan(uint32_t cols, uint32_t mats, uint32_t &slots, uint32_t &groups, uint32_t &stages) {
    const size_t stage = (size_t)mats * kRows * lfm_stage_stride(cols / 256 * LFM_Q4K_BYTES);
    const uint32_t gmax = mats == 2 ? (uint32_t)GemvShape<2>::kConsumers / 2 : (uint32_t)GemvShape<1>::kConsumers;
    const uint32_t smax = mats == 2 ? (uint32_t)GemvShape<2>::kActSlots : (uint32_t)GemvShape<1>::kActSlots;
    size_t n = 0;
    for (slots = smax; slots >= 1; --slots) {
        const size_t fixed = sizeof(GemvShared) + 2048 + (size_t)slots * lfm_act_slot_bytes(cols);
        n = fixed < kSmemBudget ? (kSmemBudget - fixed) / stage : 0;
        if (n >= 4 || slots == 1) break;
    }
    if (n > kMaxStages) n = kMaxStages;
    groups = (uint32_t)(n < gmax ? n : gmax);
    stages = groups ? (uint32_t)(n / groups * groups) : 0;
}

}  // namespace

/* Raise a kernel's dynamic shared-memory limit once per device (host side). */
cudaError_t lfm_smem_attr(const void *fn, size_t smem, size_t *cache16) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    size_t &c = cache16[dev & 15];
    if (smem <= c) return cudaSuccess;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess) c = smem;
    return e;
}

size_t lfm_gemv_smem(uint32_t cols, uint32_t mats) {
    uint32_t slots, groups, stages;
    gemv_plan(cols, mats, slots, groups, stages);
    return (size_t)stages * mats * kRows * lfm_stage_stride(cols / 256 * LFM_Q4K_BYTES) +
           (size_t)slots * lfm_act_slot_bytes(cols);
}

static cudaError_t launch_gemv(const void *fn, uint32_t cols, uint32_t mats, GemvArgs &a, int grid, cudaStream_t s,
                               bool pdl) {
    static size_t cache[2][16];
    gemv_plan(cols, mats, a.slots, a.groups, a.stages);
    if (a.groups == 0 || a.slots == 0) return cudaErrorInvalidValue;
    const size_t smem = lfm_gemv_smem(cols, mats);
    cudaError_t e = lfm_smem_attr(fn, smem, cache[mats - 1]);
    if (e != cudaSuccess) return e;
    void *args[] = {&a};
    const int threads = mats == 2 ? GemvShape<2>::kThreads : GemvShape<1>::kThreads;
    return launch_ex(fn, dim3(grid), dim3(threads), smem, s, pdl, args);
}

cudaError_t lfm_launch_gateup(const MoeLayerDev &L, Q8Rows xq, const RouteTables &rt, float *h, int grid,
                              cudaStream_t s, bool pdl) {
    GemvArgs a{L, xq, rt, h, 0, 0, 0, 1};
    return launch_gemv((const void *)k_gemv<2>, L.D, 2, a, grid, s, pdl);
}

cudaError_t lfm_launch_down(const MoeLayerDev &L, Q8Rows hq, const RouteTables &rt, float *y, int grid,
                            cudaStream_t s, bool pdl) {
    GemvArgs a{L, hq, rt, y, 0, 0, 0, 0};
    return launch_gemv((const void *)k_gemv<1>, L.I, 1, a, grid, s, pdl);
}

cudaError_t lfm_launch_quant_rows(const float *h, uint32_t rows, uint32_t cols, Q8Rows hq, cudaStream_t s, bool pdl) {
    if (rows == 0) return cudaSuccess;
    const uint32_t warps = rows * (cols / 256);
    void *args[] = {(void *)&h, &rows, &cols, &hq};
    return launch_ex((const void *)k_quant_rows, dim3((warps + 7) / 8), dim3(256), 0, s, pdl, args);
}

cudaError_t lfm_launch_combine(const MoeLayerDev &L, float *x, uint32_t T, const RouteTables &rt, const float *y,
                               cudaStream_t s, bool pdl) {
    if (T == 0) return cudaSuccess;
    uint32_t D = L.D, K = lfm_layer_K(L);
    RouteTables r = rt;
    void *args[] = {&x, &D, &K, &r, (void *)&y};
    return launch_ex((const void *)k_combine, dim3((D / 4 + 127) / 128, T), dim3(128), 0, s, pdl, args);
}

cudaError_t lfm_launch_debug_q4k_rows(const uint8_t *w, uint32_t n_rows, uint32_t n_cols, Q8Rows xq,
                                      uint32_t n_vec, int32_t *sub_dots, int32_t *acc, int32_t *mins,
                                      float *rows_out, cudaStream_t s) {
    if (n_rows % kRows) return cudaErrorInvalidValue;
    static size_t cache[16];
    const size_t smem = lfm_act_slot_bytes(n_cols);
    cudaError_t e = lfm_smem_attr((const void *)k_debug_rows, smem, cache);
    if (e != cudaSuccess) return e;
    const uint32_t gy = min(64u, (n_rows / kRows + 7) / 8);
    k_debug_rows<<<dim3(n_vec, gy), 256, smem, s>>>(w, n_rows, n_cols, xq, sub_dots, acc, mins, rows_out);
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
