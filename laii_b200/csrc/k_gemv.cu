/*
 * K3 grouped Q4_K expert GEMVs (decode / verify path).
 *
 * Work list: the dispatch tables list (active expert u, 8-token chunk c)
 * pairs.  Each pair's weight rows are cut into items of R rows (gate|up: R = 2
 * rows of each of gate and up; down: R = 4 rows); the flattened list of
 * (pair, item) is split into one contiguous range per block of a persistent
 * grid (one block per SM).
 *
 * Within a block every warp computes and feeds itself: warp w takes the
 * block's items w, w+W, w+2W, ... and streams them through a private ring of
 * S shared-memory stages with 1-D bulk copies (cp.async.bulk on the TMA
 * engine, evict-first L2 policy) completing on its own mbarriers, keeping S-1
 * copies in flight while it computes.  No warp waits for another except at
 * activation phases (below), so a slow warp never stalls the copies of the
 * others.  A stage holds one "unit": the item's rows over 8 consecutive
 * super-blocks (a whole row when cols <= 2048, one bulk copy per matrix).
 *
 * Lane mapping inside a unit: lane = 8*g + h, g = (matrix, row) group (4 of
 * them), h = super-block 8p+h of pass p.  Each lane forms the exact integer
 * sums of its super-block for every token of the pair and the operands of
 * the fp32 update (lfm_q4k_sb, with the token count a template parameter so
 * tokens interleave without branches), writes them over the consumed stage,
 * and then lane 8*g + t runs the fp32 update chain of row g for token t over
 * the super-blocks in order (lfm_q4k_chain) -- the reference's evaluation
 * order.
 *   gate|up: h = (g / (1 + exp(-g))) * u   (tools/lfm2_decode_1x4.c:976-985)
 *   down:    y[slot][r]
 *
 * Activations: the Q8_K rows of up to `slots` pairs ("a phase") are staged in
 * shared memory by all warps together; phases are separated by block-wide
 * barriers.  Weight copies run ahead across phases.
 *
 * Every mbarrier wait is bounded (lfm_mbar_wait); after a timeout a warp stops
 * computing and copying, keeps taking the phase barriers, lets its copies in
 * flight land (bounded) and leaves with the device error word set.
 */
#include "moe_device.cuh"
#include "moe_internal.h"

namespace {

constexpr int kCh = LFM_GEMV_CHUNK;  /* tokens per pair (8) */
constexpr int kMaxWarps = 12;
constexpr int kMaxStages = 4;
constexpr int kMaxSlots = 2;
constexpr size_t kSmemBudget = 224 * 1024;
constexpr uint32_t kUnitSb = 8;       /* super-blocks per unit row */

template <int kMats> struct GemvRows { static constexpr int R = kMats == 2 ? 2 : 4; };

__device__ __forceinline__ int ld_volatile_int(const int *p) { return *reinterpret_cast<const volatile int *>(p); }



struct GemvShared {
    uint64_t full[kMaxWarps][kMaxStages];
    int p_slot0[kMaxSlots], p_nt[kMaxSlots];
    int p_rows[kMaxSlots][kCh];
    int abort;
};

struct GemvArgs {
    MoeLayerDev L;
    Q8Rows act;        /* activation rows: xq (token-indexed) or hq (slot-indexed) */
    RouteTables rt;
    float *out;        /* h [slots][I] or y [slots][D] */
    uint32_t stages;   /* S: stages per warp */
    uint32_t slots;    /* pairs staged per phase */
};

struct GemvPlan {
    uint32_t warps, stages, slots;
    size_t smem;
};

__host__ __device__ inline uint32_t unit_row_stride(uint32_t nb) { return (nb < kUnitSb ? nb : kUnitSb) * LFM_Q4K_BYTES; }

/* Largest configuration that fits: 2 activation slots if that still leaves
 * 3 stages for 12 warps, else 1; then the most warps (down to 4) with at least
 * 2 stages each, preferring 3-4 stages. */
GemvPlan gemv_plan(uint32_t cols, uint32_t mats) {
    const uint32_t nb = cols / 256;
    const size_t stage = (size_t)4 * unit_row_stride(nb); /* 4 (matrix, row) groups per unit */
    (void)mats;
    const size_t fixed0 = 1024;
    for (uint32_t slots = kMaxSlots; slots >= 1; --slots) {
        const size_t act = (size_t)slots * lfm_act_slot_bytes(cols);
        for (uint32_t want = 3; want >= 2; --want) {
            for (uint32_t w = kMaxWarps; w >= 4; --w) {
                const size_t fixed = fixed0 + act;
                if (fixed >= kSmemBudget) continue;
                uint32_t s = (uint32_t)((kSmemBudget - fixed) / ((size_t)w * stage));
                if (s > kMaxStages) s = kMaxStages;
                if (s < want) continue;
                if (slots == 2 && !(w == kMaxWarps && s >= 3)) continue;
                return GemvPlan{w, s, slots, (size_t)w * s * stage + act};
            }
        }
    }
    return GemvPlan{0, 0, 0, 0};
}

/* Integer phase of one unit for kNt tokens: lane (g, h) forms the update
 * operands of its super-block, then -- once every lane of the warp has read
 * its weights -- writes them over the stage it came from as entry (h, t, g)
 * (16 bytes at ((h*8 + t)*4 + g)*16; at most 512*nsb <= 576*nsb bytes, the
 * stage's size), so lane (g, t) later reads its 8 entries 512 bytes apart and
 * the warp's 32 chain lanes read 512 contiguous bytes per step. */
template <int kNt>
__device__ __forceinline__ void unit_ints(const uint8_t *wsb, const uint8_t *rec, uint32_t tstride, bool act,
                                          uint8_t *st, int g, int h) {
    float4 o[kNt];
    uint32_t toff[kNt];
#pragma unroll
    for (int t = 0; t < kNt; ++t) toff[t] = (uint32_t)t * tstride;
    if (act) lfm_q4k_sb<kNt, true, false>(wsb, rec, toff, o, nullptr);
    __syncwarp();
    if (act) {
#pragma unroll
        for (int t = 0; t < kNt; ++t) {
            const uint32_t a = lfm_smem_u32(st + (size_t)((h * 8 + t) * 4 + g) * 16);
            asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(a), "f"(o[t].x), "f"(o[t].y), "f"(o[t].z),
                         "f"(o[t].w)
                         : "memory");
        }
    }
    __syncwarp();
}

template <int kMats>
__global__ void __launch_bounds__(kMaxWarps * 32, 1) k_gemv(GemvArgs A) {
    constexpr int R = GemvRows<kMats>::R;
    extern __shared__ __align__(128) uint8_t dsm[];
    __shared__ GemvShared sh;
    const MoeLayerDev &L = A.L;
    const uint32_t rows_total = kMats == 2 ? L.I : L.D;
    const uint32_t cols = kMats == 2 ? L.D : L.I;
    const uint32_t nb = cols / 256;
    const uint32_t row_bytes = nb * LFM_Q4K_BYTES;
    const uint32_t rs = unit_row_stride(nb);
    const uint32_t stage_bytes = 4 * rs;
    const uint32_t npass = (nb + kUnitSb - 1) / kUnitSb;
    const uint32_t W = blockDim.x >> 5, S = A.stages;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t K = lfm_layer_K(L);

    if (lane == 0) {
        for (uint32_t s = 0; s < S; ++s) lfm_mbar_init(&sh.full[warp][s], 1);
        lfm_fence_mbar_init();
    }
    if (threadIdx.x == 0) sh.abort = 0;
    __syncthreads();
    lfm_pdl_launch_dependents();
    lfm_pdl_wait(); /* routing tables and activations come from the preceding kernels */

    const uint32_t gpp = rows_total / R; /* items per (expert, chunk) pair */
    const uint64_t n_items = (uint64_t)__ldcg(A.rt.summary + 3) * gpp;
    const uint64_t i0 = n_items * blockIdx.x / gridDim.x;
    const uint64_t i1 = n_items * (blockIdx.x + 1) / gridDim.x;
    if (i0 >= i1) return; /* whole block */
    const uint8_t *W0 = kMats == 2 ? L.gate : L.down;
    const uint8_t *W1 = L.up;
    uint8_t *my_stages = dsm + (size_t)warp * S * stage_bytes;
    uint8_t *act_base = dsm + (size_t)W * S * stage_bytes;
    const size_t slot_bytes = lfm_act_slot_bytes(cols);

    const uint64_t n_local = i1 - i0;
    const uint64_t my_items = n_local > (uint64_t)warp ? (n_local - warp + W - 1) / W : 0;
    const uint64_t my_units = my_items * npass;

    /* ---- copy issue (lane 0 of each warp, for its own ring) ---- */
    const uint64_t policy = lfm_policy_evict_first();
    uint64_t issued = 0;
    uint64_t pj = ~0ull;
    int pe = 0;
    auto issue = [&](uint64_t v) {
        const uint64_t i = i0 + warp + (v / npass) * W;
        const uint32_t p = (uint32_t)(v % npass);
        const uint64_t j = i / gpp;
        if (j != pj) { /* the expert changes once per gpp items */
            pj = j;
            pe = __ldcg(A.rt.act + __ldcg(A.rt.pairs + j).x);
        }
        const size_t row0 = (size_t)pe * rows_total + (size_t)(i % gpp) * R;
        const uint32_t nsb = min(kUnitSb, nb - kUnitSb * p);
        const uint32_t seg = nsb * LFM_Q4K_BYTES;
        uint64_t *bar = &sh.full[warp][v % S];
        uint8_t *dst = my_stages + (size_t)(v % S) * stage_bytes;
        lfm_mbar_arrive_tx(bar, 4u * seg);
        for (int m = 0; m < kMats; ++m) {
            const uint8_t *src = (m == 0 ? W0 : W1) + row0 * row_bytes + (size_t)p * kUnitSb * LFM_Q4K_BYTES;
            uint8_t *d = dst + (size_t)m * R * rs;
            if (npass == 1) {
                lfm_bulk_g2s(d, src, R * row_bytes, bar, policy); /* R whole rows are contiguous */
            } else {
                for (int r = 0; r < R; ++r) lfm_bulk_g2s(d + (size_t)r * rs, src + (size_t)r * row_bytes, seg, bar, policy);
            }
        }
    };
    if (lane == 0)
        for (; issued < my_units && issued < S; ++issued) issue(issued);

    /* ---- phases of `slots` pairs; this warp's items in each ---- */
    const int g = lane >> 3, h = lane & 7;     /* (matrix,row) group; super-block / token lane */
    const uint64_t j_first = i0 / gpp, j_last = (i1 - 1) / gpp;
    uint64_t v = 0;             /* next unit to consume */
    uint64_t k = (uint64_t)warp; /* next local item */
    bool stop = false;
    for (uint64_t jp = j_first; jp <= j_last; jp += A.slots) {
        const uint32_t np = (uint32_t)min((uint64_t)A.slots, j_last - jp + 1);
        __syncthreads(); /* the previous phase's activations are no longer read */
        if (threadIdx.x < np) {
            const int2 pr = __ldcg(A.rt.pairs + jp + threadIdx.x);
            const uint32_t e = (uint32_t)__ldcg(A.rt.act + pr.x);
            const int n_e = __ldcg(A.rt.counts + e);
            const int off_e = __ldcg(A.rt.offsets + e);
            sh.p_slot0[threadIdx.x] = off_e + pr.y * kCh;
            sh.p_nt[threadIdx.x] = min(kCh, n_e - pr.y * kCh);
        }
        __syncthreads();
        if (threadIdx.x < np * kCh) {
            const int q = threadIdx.x / kCh, t = threadIdx.x % kCh;
            sh.p_rows[q][t] = t < sh.p_nt[q]
                                  ? (kMats == 2 ? __ldcg(A.rt.perm + sh.p_slot0[q] + t) / (int)K : sh.p_slot0[q] + t)
                                  : 0;
        }
        __syncthreads();
        for (uint32_t q = 0; q < np; ++q)
            lfm_stage_act(A.act, sh.p_rows[q], sh.p_nt[q], act_base + q * slot_bytes, threadIdx.x, blockDim.x);
        __syncthreads();

        for (; k < n_local && (i0 + k) / gpp < jp + np; k += W) {
            if (stop) continue;
            const uint64_t i = i0 + k;
            const uint32_t q = (uint32_t)(i / gpp - jp);
            const int nt = sh.p_nt[q], slot0 = sh.p_slot0[q];
            const uint32_t row0 = (uint32_t)(i % gpp) * R;
            const ActSlot av = lfm_act_slot(act_base + q * slot_bytes, cols);
            const uint32_t tstride = nb * LFM_ACT_REC;
            float run = 0.0f; /* lane 8g+t: row g, token t */
            for (uint32_t p = 0; p < npass; ++p, ++v) {
                const uint32_t s = (uint32_t)(v % S);
                bool ok = !ld_volatile_int(&sh.abort) && lfm_mbar_wait(&sh.full[warp][s], (uint32_t)(v / S) & 1u, A.rt.err);
                ok = __all_sync(LFM_FULL_MASK, ok);
                if (!ok) {
                    if (lane == 0) atomicExch(&sh.abort, 1);
                    stop = true;
                    break;
                }
                uint8_t *st = my_stages + (size_t)s * stage_bytes;
                const uint32_t nsb = min(kUnitSb, nb - kUnitSb * p);
                const uint8_t *wsb = st + (size_t)g * rs + (size_t)h * LFM_Q4K_BYTES;
                const uint8_t *rec = av.rec + (size_t)(kUnitSb * p + h) * LFM_ACT_REC;
                const bool act = (uint32_t)h < nsb;
                if (nt <= 1) unit_ints<1>(wsb, rec, tstride, act, st, g, h);
                else if (nt <= 2) unit_ints<2>(wsb, rec, tstride, act, st, g, h);
                else if (nt <= 4) unit_ints<4>(wsb, rec, tstride, act, st, g, h);
                else unit_ints<8>(wsb, rec, tstride, act, st, g, h);
                if (h < nt) run = lfm_q4k_chain(run, st + (size_t)(h * 4 + g) * 16, 512, nsb);
                __syncwarp(); /* stage free again */
                if (lane == 0 && issued < my_units) {
                    issue(issued);
                    ++issued;
                }
            }
            if (stop) continue;
            if (kMats == 2) {
                const float u = __shfl_down_sync(LFM_FULL_MASK, run, 16);
                if (lane < 16 && h < nt) {
                    const float silu = __fdiv_rn(run, __fadd_rn(1.0f, lfm_silu_expf(-run)));
                    A.out[(size_t)(slot0 + h) * L.I + row0 + g] = __fmul_rn(silu, u);
                }
            } else {
                if (h < nt) A.out[(size_t)(slot0 + h) * L.D + row0 + g] = run;
            }
        }
    }
    /* leave no copy in flight into this block's shared memory */
    if (lane == 0)
        for (; v < issued; ++v) lfm_mbar_wait(&sh.full[warp][v % S], (uint32_t)(v / S) & 1u, A.rt.err);
}

/* Debug: vector v against rows [4*gy .. ) through the production integer and
 * fp32 routines; weights read from global memory.  Shared memory: the
 * vector's records, then 512 bytes of chain operands per warp. */
__global__ void __launch_bounds__(256) k_debug_rows(const uint8_t *__restrict__ w, uint32_t n_rows, uint32_t n_cols,
                                                    Q8Rows xq, int32_t *sub_dots, int32_t *acc_out, int32_t *mins_out,
                                                    float *rows_out) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int vrow[kCh];
    const uint32_t nb = n_cols / 256;
    const uint32_t v = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 3, h = lane & 7;
    const size_t row_bytes = (size_t)nb * LFM_Q4K_BYTES;
    uint8_t *slot = smem;
    uint8_t *scr = smem + lfm_act_slot_bytes(n_cols, 1) + (size_t)warp * 512;
    if (threadIdx.x < kCh) vrow[threadIdx.x] = (int)v;
    __syncthreads();
    lfm_stage_act(xq, vrow, 1, slot, threadIdx.x, blockDim.x);
    __syncthreads();
    for (uint32_t rb = (blockIdx.y * 8 + warp) * 4; rb < n_rows; rb += gridDim.y * 8 * 4) {
        const uint32_t row = rb + g;
        const size_t o = (size_t)v * n_rows + row;
        float run = 0.0f;
        for (uint32_t p = 0; p * kUnitSb < nb; ++p) {
            const uint32_t nsb = min(kUnitSb, nb - kUnitSb * p);
            const uint32_t b = kUnitSb * p + h;
            if ((uint32_t)h < nsb) {
                int32_t dbg[10];
                float4 e[1];
                const uint32_t toff[1] = {0};
                lfm_q4k_sb<1, false, true>(w + row * row_bytes + (size_t)b * LFM_Q4K_BYTES, slot + (size_t)b * LFM_ACT_REC,
                                           toff, e, dbg);
                for (int j = 0; j < 8; ++j) sub_dots[(o * nb + b) * 8 + j] = dbg[j];
                acc_out[o * nb + b] = dbg[8];
                mins_out[o * nb + b] = dbg[9];
                *reinterpret_cast<float4 *>(scr + (size_t)(h * 4 + g) * 16) = e[0];
            }
            __syncwarp();
            if (h == 0) run = lfm_q4k_chain(run, scr + (size_t)g * 16, 64, nsb);
            __syncwarp();
        }
        if (h == 0) rows_out[o] = run;
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
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

cudaError_t launch_gemv(const void *fn, uint32_t cols, uint32_t mats, GemvArgs &a, int grid, cudaStream_t s,
                        bool pdl) {
    static size_t cache[2][16];
    const GemvPlan pl = gemv_plan(cols, mats);
    if (pl.warps == 0) return cudaErrorInvalidValue;
    a.stages = pl.stages;
    a.slots = pl.slots;
    cudaError_t e = lfm_smem_attr(fn, pl.smem, cache[mats - 1]);
    if (e != cudaSuccess) return e;
    void *args[] = {&a};
    return launch_ex(fn, dim3(grid), dim3(pl.warps * 32), pl.smem, s, pdl, args);
}

}  // namespace

size_t lfm_gemv_smem(uint32_t cols, uint32_t mats) { return gemv_plan(cols, mats).smem; }

cudaError_t lfm_launch_gateup(const MoeLayerDev &L, Q8Rows xq, const RouteTables &rt, float *h, int grid,
                              cudaStream_t s, bool pdl) {
    GemvArgs a{L, xq, rt, h, 0, 0};
    return launch_gemv((const void *)k_gemv<2>, L.D, 2, a, grid, s, pdl);
}

cudaError_t lfm_launch_down(const MoeLayerDev &L, Q8Rows hq, const RouteTables &rt, float *y, int grid,
                            cudaStream_t s, bool pdl) {
    GemvArgs a{L, hq, rt, y, 0, 0};
    return launch_gemv((const void *)k_gemv<1>, L.I, 1, a, grid, s, pdl);
}

cudaError_t lfm_launch_debug_q4k_rows(const uint8_t *w, uint32_t n_rows, uint32_t n_cols, Q8Rows xq,
                                      uint32_t n_vec, int32_t *sub_dots, int32_t *acc, int32_t *mins,
                                      float *rows_out, cudaStream_t s) {
    if (n_rows % 4) return cudaErrorInvalidValue;
    static size_t cache[16];
    const size_t smem = lfm_act_slot_bytes(n_cols, 1) + 8 * 512;
    cudaError_t e = lfm_smem_attr((const void *)k_debug_rows, smem, cache);
    if (e != cudaSuccess) return e;
    const uint32_t gy = min(64u, (n_rows / 4 + 7) / 8);
    k_debug_rows<<<dim3(n_vec, gy), 256, smem, s>>>(w, n_rows, n_cols, xq, sub_dots, acc, mins, rows_out);
    return cudaGetLastError();
}
