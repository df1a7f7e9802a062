/*
 * Internal (non-exported) interfaces of liblfm_gpu_moe.so: device-side data
 * layouts of the MoE-FFN path and the kernel launchers each .cu provides.
 *
 * HBM layout (per layer, see lfm_gpu_moe.cu):
 *   gate/up  Q4_K [E][I][D/256]  144-byte GGUF blocks, uploaded as-is
 *   down     Q4_K [E][D][I/256]
 *   router   fp32 [E][D], bias fp32 [E], ffn_norm fp32 [D]
 * Activations are kept as split Q8_K rows (qs int8 [rows][cols], d fp32
 * [rows][cols/256], bsums int16 [rows][cols/256][16]): same numbers as
 * block_q8_K, but 16-byte aligned rows for vector and bulk loads.
 */
#ifndef LFM_MOE_INTERNAL_H
#define LFM_MOE_INTERNAL_H

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "lfm_formats.h"

#define LFM_GPU_MAX_TOPK_DEV 8
#define LFM_GPU_MAX_EXPERTS_DEV 256
#define LFM_GPU_MAX_D 8192      /* router stages 5*D fp32 in shared memory     */
#define LFM_GEMV_CHUNK 8        /* tokens per staged activation chunk (GEMV)   */
#define LFM_FUSED_MAX_T 16      /* largest T the fused decode layer handles    */

/* Device error word bits (read by lfm_gpu_moe_sync and the host-buffer forward). */
#define LFM_DEVERR_EXPERT_ID 0x1u   /* routing produced an expert id >= E     */
#define LFM_DEVERR_SEGMENT 0x2u     /* dispatch segment out of range           */
#define LFM_DEVERR_TIMEOUT 0x4u     /* a bounded device wait ran out           */

struct Q8Rows {
    int8_t *qs;      /* [rows][cols]      */
    float *d;        /* [rows][cols/256]  */
    int16_t *bs;     /* [rows][cols/256][16] */
    uint32_t cols;
};

/* tcgen05 GEMM work (k_umma.cu): a tile is weight rows [row0, row0 + 128) of
 * `expert` in matrix `mat` (0: gate or down, 1: up) against token block `tb`;
 * a token block is dispatch slots [slot0, slot0 + ntok), ntok <= nt. */
struct __align__(16) LfmUTile { /* one 16-byte store / load */
    int32_t expert, tb, row0, mat;
};
struct __align__(8) LfmUTokBlock {
    int32_t slot0, ntok;
};
/* Tile plans the dispatch step writes for the tcgen05 GEMMs (nt == 0: none):
 * token blocks of <= nt slots per active expert, then tiles (expert, 128-row
 * block, token block, matrix) with the matrix and then the token blocks
 * fastest: one plan covers gate and up together, one the down rows.
 * counts = {tiles gu, blocks, tiles dn, blocks}. */
struct UmmaPlanOut {
    LfmUTile *tiles_gu, *tiles_dn;
    LfmUTokBlock *tbs;
    int32_t *counts;
    uint32_t rows_gu, rows_dn, nt, max_gu, max_dn, max_tb;
};

/* Routing / dispatch tables for one forward (all device pointers). */
struct RouteTables {
    int32_t *idx;        /* [T*K] expert id of assignment a = t*K + k                   */
    float *w;            /* [T*K] combine weight                                        */
    int32_t *counts;     /* [E]   assignments per expert                                 */
    int32_t *offsets;    /* [E+1] exclusive prefix of counts (first slot of expert e)     */
    int32_t *perm;       /* [T*K] slot -> assignment (slots grouped by expert)           */
    int32_t *inv;        /* [T*K] assignment -> slot                                     */
    int32_t *act;        /* [E]   expert id of active expert u (experts with tokens)     */
    int2 *pairs;         /* [E + T*K/8] (u, chunk) work pairs, u-major                   */
    int32_t *summary;    /* [4]   active experts U, max segment, slots, pairs            */
    uint32_t *tok_count; /* [T]   per-token router-block arrival counters (kept at 0)     */
    uint32_t *done;      /* [1]   CTA arrival counter of the dispatch (kept at 0)          */
    int32_t *chunk;      /* [T*K/1024][E] per-chunk expert counts, then ranks (split dispatch; NULL: one block) */
    float *logits;       /* [T*E] router logits                                          */
    float *rms;          /* [T]   1/rms of x (the prefill router's two passes)            */
    uint32_t *err;       /* device error word                                            */
    unsigned long long *loads; /* [2] running sum of unique experts, MoE layer runs      */
    UmmaPlanOut plan;    /* tcgen05 GEMM tile plans to build with the dispatch (nt == 0: none) */
};

struct MoeLayerDev {
    uint32_t D, E, K, I, dense;
    float eps, routed_scale;
    int norm_topk;
    float *ffn_norm;
    float *router_w;
    float *bias;         /* NULL when the layer has no exp_probs_b */
    const uint8_t *gate; /* Q4_K blocks */
    const uint8_t *up;
    const uint8_t *down;
    uint32_t down_q6k;   /* 1: down is Q6_K [E][D][I/256] 210-byte blocks (k_q6k.cu), 0: Q4_K */
};

/* Expert-side geometry of a layer (dense layers are one expert, top-1). */
__host__ __device__ inline uint32_t lfm_layer_E(const MoeLayerDev &L) { return L.dense ? 1u : L.E; }
__host__ __device__ inline uint32_t lfm_layer_K(const MoeLayerDev &L) { return L.dense ? 1u : L.K; }

/* Raise a kernel's dynamic shared-memory limit once per device (cache16: 16 slots). */
cudaError_t lfm_smem_attr(const void *fn, size_t smem, size_t *cache16);

/* k_route.cu */
/* dispatch tables only, from rt.idx already filled (one block) */
cudaError_t lfm_launch_dispatch(const MoeLayerDev &L, uint32_t T, const RouteTables &rt, cudaStream_t s);
struct EpPublish;
/* pub (expert parallelism): the dispatch step also publishes the per-expert counts to every rank */
cudaError_t lfm_launch_route(const MoeLayerDev &L, const float *x, uint32_t T, Q8Rows xq, const RouteTables &rt,
                             cudaStream_t s, bool pdl, const EpPublish *pub = nullptr);
/* kernel launches lfm_launch_route makes for (L, T) */
uint32_t lfm_route_kernels(const MoeLayerDev &L, uint32_t T);

/* k_expert.cu */
size_t lfm_gemv_smem(uint32_t cols, uint32_t mats);

/* Fused decode layer (k_layer.cu): whether (layer, T) fits it, and its
 * cooperative launch on `grid` CTAs (one per SM). gbar: 2 zeroed words. */
bool lfm_fused_ok(const MoeLayerDev &L, uint32_t T, int grid);
cudaError_t lfm_launch_layer_fused(const MoeLayerDev &L, float *x, uint32_t T, const RouteTables &rt, float *h,
                                   float *y, unsigned *gbar, uint8_t *xrec, float *scores, int grid, cudaStream_t s);
cudaError_t lfm_launch_gateup(const MoeLayerDev &L, Q8Rows xq, const RouteTables &rt, float *h, int grid,
                              cudaStream_t s, bool pdl);
cudaError_t lfm_launch_quant_rows(const float *h, uint32_t rows, uint32_t cols, Q8Rows hq, cudaStream_t s, bool pdl);
cudaError_t lfm_launch_down(const MoeLayerDev &L, Q8Rows hq, const RouteTables &rt, float *y, int grid,
                            cudaStream_t s, bool pdl);
/* k_q6k.cu: down projection of a layer whose down tensor is Q6_K (pairs of the dispatch tables) */
cudaError_t lfm_launch_down_q6k(const MoeLayerDev &L, Q8Rows hq, const RouteTables &rt, float *y, int grid,
                                cudaStream_t s);
cudaError_t lfm_launch_combine(const MoeLayerDev &L, float *x, uint32_t T, const RouteTables &rt, const float *y,
                               cudaStream_t s, bool pdl);
cudaError_t lfm_launch_debug_q4k_rows(const uint8_t *w, uint32_t n_rows, uint32_t n_cols, Q8Rows xq,
                                      uint32_t n_vec, int32_t *sub_dots, int32_t *acc, int32_t *mins,
                                      float *rows_out, cudaStream_t s);
cudaError_t lfm_launch_q8_to_gguf(Q8Rows q, uint32_t rows, uint8_t *out, cudaStream_t s);
/* expert parallelism: given routing of received rows, and the (t, k)-ordered combine */
cudaError_t lfm_launch_ep_prepare(const int32_t *expert_ids, uint32_t n, uint32_t first, uint32_t count,
                                  const RouteTables &rt, cudaStream_t s);
cudaError_t lfm_launch_ep_combine(float *x, uint32_t T, uint32_t D, uint32_t K, const float *w, const float *y,
                                  cudaStream_t s);
cudaError_t lfm_launch_gguf_to_q8(const uint8_t *in, uint32_t rows, Q8Rows q, cudaStream_t s);

/* ---- expert parallelism over peer memory (k_ep.cu, k_route.cu, k_umma.cu) ----
 * Every rank's exchange arena has the same layout; the host maps the other
 * ranks' arenas (CUDA IPC) so kernels read and write them directly.  Flags
 * carry the epoch of the layer step (wrap-safe compare); the count table is
 * double-buffered by epoch parity.  The epoch lives in device memory (step:
 * the last finished step, advanced by the combine's last CTA), so a captured
 * CUDA graph replays step after step with the same kernel arguments. */
#define LFM_EP_MAX_RANKS 8
struct EpArena {
    uint32_t *cnt_flag; /* [LFM_EP_MAX_RANKS] epoch of home rank r's published counts (written by r)   */
    uint32_t *y_flag;   /* [LFM_EP_MAX_RANKS] epoch of expert rank r's stored outputs (written by r)    */
    uint32_t *done;     /* [1] output-store CTAs finished (this rank only; kept at 0)                    */
    int32_t *table;     /* [2][LFM_EP_MAX_RANKS][E] per-expert counts of every home rank                 */
    Q8Rows xq;          /* [max_tokens] this rank's Q8_K rows of x (read by the expert ranks)            */
    int32_t *perm;      /* [max_tokens*K] slot -> assignment t*K+k, slots grouped by expert (read by them)*/
    float *yhome;       /* [max_tokens*K][D] expert output of assignment t*K+k (written by them)         */
    uint32_t *rowmap;   /* [max_recv] received slot -> (home rank << 24) | home slot (this rank only)    */
    uint32_t *ret;      /* [max_recv] received slot -> (home rank << 24) | t*K+k     (this rank only)    */
    int32_t *n_recv;    /* [1] rows received in this step (this rank only)                               */
    uint32_t *step;     /* [1] epoch of this rank's last finished step (this rank only)                   */
    uint32_t *cdone;    /* [1] combine CTAs finished (this rank only; kept at 0)                          */
};
/* What the exchange kernels of one step need: this rank's arena and every rank's view of its own. */
struct EpStep {
    uint32_t rank, world, E, K, D;
    uint32_t ahead;      /* the step's epoch is *self.step + ahead (1; the wait check uses 2)   */
    uint32_t max_assign; /* T*K capacity of every home rank's yhome / perm */
    uint32_t max_recv;   /* received-slot capacity of this rank          */
    uint64_t wait_ns;
    uint32_t *err;
    EpArena self;
    int32_t *table[LFM_EP_MAX_RANKS];     /* peer views */
    uint32_t *cnt_flag[LFM_EP_MAX_RANKS];
    uint32_t *y_flag[LFM_EP_MAX_RANKS];
    float *yhome[LFM_EP_MAX_RANKS];
};
/* The received rows for k_xt_gather: slot -> home rank's Q8_K row (peer views). */
struct EpGather {
    const uint32_t *rowmap;
    uint32_t *ret;
    uint32_t *err;
    uint32_t K, world, max_assign; /* max_assign: T*K capacity of a home rank */
    const int32_t *perm[LFM_EP_MAX_RANKS];
    const int8_t *qs[LFM_EP_MAX_RANKS];
    const float *d[LFM_EP_MAX_RANKS];
    const int16_t *bs[LFM_EP_MAX_RANKS];
};
/* Owning rank of expert e when E experts are split over `world` ranks, the
 * first E % world ranks holding one more. */
__host__ __device__ inline uint32_t lfm_ep_owner(uint32_t e, uint32_t E, uint32_t world) {
    const uint32_t base = E / world, rem = E % world, big = rem * (base + 1);
    return e < big ? e / (base + 1) : rem + (e - big) / base;
}
__host__ __device__ inline uint32_t lfm_ep_first(uint32_t r, uint32_t E, uint32_t world) {
    const uint32_t base = E / world, rem = E % world;
    return r * base + (r < rem ? r : rem);
}
/* A home rank's per-expert counts of one step, into every rank's table, then
 * its cnt_flag there (release, after a system-scope fence of the writes that
 * precede it: the Q8_K rows and slots the expert ranks read next). */
struct EpPublish {
    int32_t *table[LFM_EP_MAX_RANKS];
    uint32_t *cnt_flag[LFM_EP_MAX_RANKS];
    const uint32_t *step;           /* epoch of the step = *step + 1 */
    uint32_t world, rank, E;        /* world == 0: nothing to publish */
};
/* publish rt.counts[E] on its own (a step with no tokens, where no dispatch runs) */
cudaError_t lfm_launch_ep_publish(const EpStep &st, const int32_t *counts, cudaStream_t s);
/* expert rank: wait for every rank's counts, then the received slots' layout
 * (rowmap, n_recv) and the tcgen05 tile plans of the local experts
 * [first, first + count) */
cudaError_t lfm_launch_ep_plan(const EpStep &st, uint32_t first, uint32_t count, const RouteTables &rt,
                               cudaStream_t s, bool pdl = false);
/* Where an expert rank's down GEMM stores its output rows: the row of slot j
 * goes to home rank (ret[j] >> 24)'s yhome row ret[j] & 0xffffff (a peer
 * store over NVLink, or local); the GEMM's last CTA then raises y_flag[rank]
 * on every rank (release, after a system-scope fence of every CTA's stores). */
struct UmmaEpOut {
    const uint32_t *ret;
    float *yhome[LFM_EP_MAX_RANKS];
    uint32_t *y_flag[LFM_EP_MAX_RANKS];
    uint32_t *done;
    const uint32_t *step;  /* epoch of the step = *step + 1 */
    uint32_t world, rank, max_assign;
};
/* home rank: wait for every expert rank's y_flag, then x[t] += w . yhome[t] in k order;
 * advance: then the rank's step counter moves to this step's epoch */
cudaError_t lfm_launch_ep_combine_wait(const EpStep &st, float *x, uint32_t T, const float *w, bool advance,
                                       cudaStream_t s, bool pdl = false);

/* k_gemm.cu: prefill grouped GEMM (tensor cores) */
size_t lfm_gemm_tiles_max(uint32_t rows, uint32_t slots, uint32_t experts);
size_t lfm_gemm_tile_bytes();
cudaError_t lfm_launch_gemm_plan(const RouteTables &rt, uint32_t rows, void *tiles, int32_t *n_tiles,
                                 uint32_t max_tiles, cudaStream_t s);
cudaError_t lfm_launch_q4k_gemm(const uint8_t *W, uint32_t rows, uint32_t cols, Q8Rows X, const int32_t *perm,
                                uint32_t K, const void *tiles, const int32_t *n_tiles, float *Y, uint32_t *err,
                                int grid, cudaStream_t s);
cudaError_t lfm_launch_swiglu_quant(const float *G, const float *U, uint32_t rows, uint32_t cols, Q8Rows dst,
                                    cudaStream_t s);

/* 2-D tiled tensor map (no swizzle, no interleave, zero fill) over a row-major
 * matrix [outer][inner] of elem_bytes elements with rows row_bytes apart, box
 * box_inner x box_outer; false when the driver refuses it (k_umma.cu). */
bool lfm_tmap_2d(CUtensorMap *tm, CUtensorMapDataType type, uint32_t elem_bytes, const void *base, uint64_t inner,
                 uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer);

/* k_umma.cu: grouped GEMM on tcgen05 (rows % 128 == 0), nt tokens per block (16..128) */
bool lfm_umma_ok(uint32_t rows);
uint32_t lfm_umma_nt(uint32_t slots, uint32_t experts);
size_t lfm_umma_tb_max(uint32_t slots, uint32_t experts, uint32_t nt);
size_t lfm_umma_tiles_max(uint32_t rows, uint32_t slots, uint32_t experts, uint32_t nt);
size_t lfm_umma_xt_bytes(size_t max_tb, uint32_t nb, uint32_t nt);
cudaError_t lfm_launch_xt_gather(Q8Rows X, const int32_t *perm, uint32_t K, const void *tbs, const int32_t *n_tb,
                                 uint32_t max_tb, uint32_t nt, uint8_t *xt, cudaStream_t s, bool pdl = false);
/* the same from other ranks' Q8_K rows (expert parallelism, g.rowmap set); X.cols gives D */
cudaError_t lfm_launch_xt_gather_ep(const EpGather &g, uint32_t cols, const void *tbs, const int32_t *n_tb,
                                    uint32_t max_tb, uint32_t nt, uint8_t *xt, cudaStream_t s, bool pdl = false);
/* SwiGLU of the gate|up outputs, Q8_K, written as the down GEMM's token blocks */
cudaError_t lfm_launch_swiglu_xt(const float *G, const float *U, uint32_t cols, const void *tbs, const int32_t *n_tb,
                                 uint32_t max_tb, uint32_t nt, uint8_t *xt, cudaStream_t s, bool pdl = false);
/* W0, W1: `experts` tensors [rows][cols/256] Q4_K back to back (tiles of
 * matrix m read Wm and write Ym; W1/Y1 may repeat W0/Y0 when every tile has m = 0).
 * ep (expert parallelism, down GEMM): store each row at its home rank instead of Y. */
struct UmmaEpOut;
cudaError_t lfm_launch_q4k_umma(const uint8_t *W0, const uint8_t *W1, uint32_t experts, uint32_t rows, uint32_t cols,
                                const uint8_t *xt, uint32_t nt, const void *tiles, const void *tbs,
                                const int32_t *n_tiles, float *Y0, float *Y1, uint32_t *err, int grid, cudaStream_t s,
                                const UmmaEpOut *ep = nullptr, bool pdl = false);

/* k_synth.cu */
/* blocks [first, first + n_blocks) of the tensor drawn from `seed` */
cudaError_t lfm_launch_synth_q4k(uint8_t *out, uint64_t n_blocks, uint64_t seed, float stddev, cudaStream_t s,
                                 uint64_t first = 0);
cudaError_t lfm_launch_synth_f32(float *out, uint64_t n, uint64_t seed, float mean, float stddev,
                                 cudaStream_t s);

#endif /* LFM_MOE_INTERNAL_H */
