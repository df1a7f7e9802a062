/*
 * C-ABI implementation of include/lfm_gpu_moe.h: handle lifecycle, weight
 * upload into HBM, scratch management and the forward orchestration
 *   K1 route -> K2 dispatch -> K3 gate|up+SwiGLU -> Q8_K(h) -> K3 down -> K4 combine
 * for one lfm2moe layer (tools/lfm2_moe_checkpoint.c:312-365, batched over T
 * tokens) or one dense SwiGLU layer (tools/lfm2_decode_1x4.c:1070-1104).
 * There is no CPU path: every failure is returned as a status.
 */
#include <cuda_runtime.h>
#include <new>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "lfm_gpu_moe.h"
#include "moe_internal.h"

#define LFM_API extern "C" __attribute__((visibility("default")))

namespace {

struct LayerSlot {
    bool present = false;
    MoeLayerDev dev{};
    uint32_t ep_first = 0, ep_count = 0; /* expert shard [first, first+count); count 0 = all experts */
    void *bufs[7] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
    size_t sizes[7] = {0, 0, 0, 0, 0, 0, 0};
};

struct Workspace {
    uint32_t T = 0, D = 0, E = 0, K = 0, I = 0;
    size_t TK = 0;            /* (token, expert) rows covered          */
    void *base = nullptr;
    size_t bytes = 0;
    size_t counters_bytes = 0; /* leading zero-kept counter region      */
    float *x = nullptr;       /* [T][D] staging for host x            */
    Q8Rows xq{};              /* [T] x D                              */
    RouteTables rt{};
    float *h = nullptr;       /* [T*K][I]                              */
    Q8Rows hq{};              /* [T*K] x I                             */
    float *y = nullptr;       /* [T*K][D]                              */
    unsigned *gbar = nullptr; /* [2] grid barrier of the fused layer (counter region) */
    uint8_t *xrec = nullptr;  /* [T][D/256] Q8_K records exchanged by the fused layer */
    float *scores = nullptr;  /* [T*E][2] router scores exchanged by the fused layer */
    float *u = nullptr;       /* [T*K][I] up projections of the prefill GEMM path (h holds gate) */
    void *tiles_gu = nullptr; /* GEMM tile plans: gate|up rows (I), down rows (D) */
    void *tiles_dn = nullptr;
    int32_t *n_tiles = nullptr; /* [2] */
    uint32_t max_tiles_gu = 0, max_tiles_dn = 0;
    /* tcgen05 GEMM path (k_umma.cu): 128-row tile plans, token blocks, pre-gathered tokens */
    LfmUTile *utiles_gu = nullptr, *utiles_dn = nullptr;
    LfmUTokBlock *utbs = nullptr;
    int32_t *ucounts = nullptr; /* [4]: tiles gu, blocks, tiles dn, blocks */
    uint8_t *xt = nullptr;
    uint32_t umax_gu = 0, umax_dn = 0, umax_tb = 0;
};

}  // namespace

namespace {
enum KernelId { K_ROUTE, K_GATEUP, K_QUANT_H, K_DOWN, K_COMBINE, K_LAYER, K_PLAN, K_GEMM_G, K_GEMM_U, K_SWIGLU, K_GEMM_D,
                K_XT, K_GEMM_GU, K_EP_PUBLISH, K_EP_PLAN, K_COUNT };
const char *const kKernelNames[K_COUNT] = {"route", "gateup", "quant_h", "down", "combine", "moe_layer",
                                           "gemm_plan", "gemm_gate", "gemm_up", "swiglu_q8", "gemm_down",
                                           "xt_gather", "gemm_gateup", "ep_publish", "ep_plan"};
struct ProfRec {
    int kid;
    cudaEvent_t a, b;
};
/* One captured forward: layers [first, first+n) on x for T tokens. */
struct GraphEntry {
    uint32_t first, n, T;
    bool ep;  /* MoE layers as expert-parallel steps over peer memory */
    float *x;
    uint32_t kernels;
    cudaGraphExec_t exec;
};
constexpr size_t kMaxGraphs = 64;
}  // namespace

namespace {
/* Expert parallelism over peer memory: this rank's exchange arena (CUDA IPC
 * exportable) and every rank's mapping of it. */
struct EpP2P {
    bool attached = false, connected = false;
    uint32_t rank = 0, world = 1, T_max = 0, D = 0, E = 0, K = 0, I = 0;
    uint64_t wait_ns = 0;
    uint8_t *arena = nullptr;
    size_t bytes = 0;
    uint8_t *peer[LFM_EP_MAX_RANKS] = {};  /* peer[rank] == arena */
    bool opened[LFM_EP_MAX_RANKS] = {};    /* mapped through cudaIpcOpenMemHandle */
    /* byte offsets of the arena's parts (the same on every rank) */
    size_t o_cnt = 0, o_y = 0, o_done = 0, o_tab = 0, o_qs = 0, o_qd = 0, o_qb = 0, o_perm = 0, o_yhome = 0,
           o_rowmap = 0, o_ret = 0, o_nrecv = 0, o_step = 0, o_cdone = 0;
    uint32_t max_recv() const { return world * T_max * K; }
};
}  // namespace

struct lfm_gpu_moe {
    int device = 0;
    cudaStream_t stream = nullptr;
    char err[512] = {0};
    LayerSlot layers[LFM_GPU_MOE_MAX_LAYERS];
    Workspace ws;
    uint32_t *dev_err = nullptr;  /* device error word, zeroed at creation */
    int sm_count = 148;
    unsigned long long *loads = nullptr;  /* device [2]: expert loads, MoE layer runs */
    lfm_gpu_moe_stats_t stats{};
    bool prof = false;
    std::vector<ProfRec> recs;
    bool use_graphs = true;
    bool use_fused = true;   /* fused decode layer for T <= LFM_FUSED_MAX_T */
    bool use_gemm = true;    /* tensor-core grouped GEMMs for prefill-sized T */
    bool use_umma = true;    /* ... on tcgen05 (k_umma.cu) where rows % 128 == 0, else mma.sync (k_gemm.cu) */
    bool use_pdl = true;     /* chain the kernels with programmatic dependent launch */
    std::vector<GraphEntry> graphs;
    EpP2P ep;
};

namespace {

lfm_gpu_status_t fail(lfm_gpu_moe_t *h, lfm_gpu_status_t st, const char *fmt, ...) {
    if (h) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(h->err, sizeof h->err, fmt, ap);
        va_end(ap);
    }
    return st;
}

lfm_gpu_status_t cuda_fail(lfm_gpu_moe_t *h, cudaError_t e, const char *what) {
    const lfm_gpu_status_t st = e == cudaErrorMemoryAllocation ? LFM_GPU_ERR_OOM : LFM_GPU_ERR_CUDA;
    return fail(h, st, "%s: %s", what, cudaGetErrorString(e));
}

#define LFM_CUDA(h, call)                                    \
    do {                                                     \
        cudaError_t e_ = (call);                             \
        if (e_ != cudaSuccess) return cuda_fail((h), e_, #call); \
    } while (0)

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

void free_layer(LayerSlot &L) {
    for (void *&p : L.bufs) {
        if (p) cudaFree(p);
        p = nullptr;
    }
    for (size_t &z : L.sizes) z = 0;
    L.present = false;
    L.ep_first = L.ep_count = 0;
    L.dev = MoeLayerDev{};
}

size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

/* Captured forwards hold device pointers (weights, workspace, x): drop them
 * whenever one of those can change. */
void drop_graphs(lfm_gpu_moe_t *h) {
    for (GraphEntry &g : h->graphs) cudaGraphExecDestroy(g.exec);
    h->graphs.clear();
}

/* Make sure the workspace covers T tokens for the given layer shape.  The
 * completion counters (tok_count, done) live in one zeroed
 * region; kernels return every counter to zero when they finish with it. */
lfm_gpu_status_t ensure_workspace(lfm_gpu_moe_t *h, uint32_t T, uint32_t D, uint32_t E, uint32_t K, uint32_t I) {
    Workspace &w = h->ws;
    /* tokens (T) and (token, expert) assignments (TK) are sized apart: the
     * expert-parallel step needs many rows at K = 1 next to few tokens at K */
    const size_t tk_req = (size_t)T * (K ? K : 1u);
    if (w.base && T <= w.T && tk_req <= w.TK && D <= w.D && E <= w.E && I <= w.I) return LFM_GPU_OK;
    T = T > w.T ? T : w.T; D = D > w.D ? D : w.D; E = E > w.E ? E : w.E;
    K = K > w.K ? K : w.K; I = I > w.I ? I : w.I;
    if (E < 1) E = 1;
    if (K < 1) K = 1;
    const size_t TK = tk_req > w.TK ? tk_req : w.TK;
    const size_t n_pairs = E + (TK + LFM_GEMV_CHUNK - 1) / LFM_GEMV_CHUNK + 1;
    size_t off = 0;
    auto take = [&](size_t bytes) { const size_t o = off; off += align256(bytes); return o; };
    /* counters first: one memset covers them */
    const size_t o_tc = take(sizeof(uint32_t) * T);
    const size_t o_done = take(sizeof(uint32_t));
    const size_t o_gbar = take(sizeof(uint32_t) * 2);
    const size_t counters_end = off;
    const size_t o_x = take(sizeof(float) * T * D);
    const size_t o_xq = take((size_t)T * D);
    const size_t o_xd = take(sizeof(float) * T * (D / 256));
    const size_t o_xb = take(sizeof(int16_t) * T * (D / 256) * 16);
    const size_t o_idx = take(sizeof(int32_t) * TK);
    const size_t o_w = take(sizeof(float) * TK);
    const size_t o_cnt = take(sizeof(int32_t) * E);
    const size_t o_off = take(sizeof(int32_t) * (E + 1));
    const size_t o_perm = take(sizeof(int32_t) * TK);
    const size_t o_inv = take(sizeof(int32_t) * TK);
    const size_t o_act = take(sizeof(int32_t) * E);
    const size_t o_pairs = take(sizeof(int2) * n_pairs);
    const size_t o_sum = take(sizeof(int32_t) * 4);
    const size_t o_log = take(sizeof(float) * T * E);
    const size_t o_rms = take(sizeof(float) * T);
    const size_t o_h = take(sizeof(float) * TK * I);
    const size_t o_hq = take(TK * I);
    const size_t o_hd = take(sizeof(float) * TK * (I / 256));
    const size_t o_hb = take(sizeof(int16_t) * TK * (I / 256) * 16);
    const size_t o_y = take(sizeof(float) * TK * D);
    const size_t o_xrec = take((size_t)T * (D / 256) * 304);
    const size_t o_scores = take(sizeof(float) * 2 * T * E);
    const size_t o_chunk = take(sizeof(int32_t) * ((TK + 1023) / 1024) * E);
    const size_t mt_gu = lfm_gemm_tiles_max(I, (uint32_t)TK, E), mt_dn = lfm_gemm_tiles_max(D, (uint32_t)TK, E);
    const size_t o_u = take(sizeof(float) * TK * I);
    const size_t o_tgu = take(lfm_gemm_tile_bytes() * mt_gu);
    const size_t o_tdn = take(lfm_gemm_tile_bytes() * mt_dn);
    const size_t o_nt = take(sizeof(int32_t) * 2);
    /* tcgen05 GEMM scratch for the smallest token block (the most blocks) and the largest (the most bytes) */
    const size_t umax_tb = lfm_umma_tb_max((uint32_t)TK, E, 16);
    const size_t umax_gu = 2 * lfm_umma_tiles_max(I, (uint32_t)TK, E, 16), umax_dn = lfm_umma_tiles_max(D, (uint32_t)TK, E, 16);
    const uint32_t nbx = (D > I ? D : I) / 256;
    const size_t xt16 = lfm_umma_xt_bytes(umax_tb, nbx, 16), xt128 = lfm_umma_xt_bytes(lfm_umma_tb_max((uint32_t)TK, E, 128), nbx, 128);
    const size_t o_utgu = take(sizeof(LfmUTile) * umax_gu);
    const size_t o_utdn = take(sizeof(LfmUTile) * umax_dn);
    const size_t o_utbs = take(sizeof(LfmUTokBlock) * umax_tb);
    const size_t o_ucnt = take(sizeof(int32_t) * 4);
    const size_t o_xt = take(xt16 > xt128 ? xt16 : xt128);
    void *base = nullptr;
    /* the old workspace may still be read by queued work on any stream */
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(h, e, "workspace sync");
    e = cudaMalloc(&base, off);
    if (e != cudaSuccess) return cuda_fail(h, e, "workspace cudaMalloc");
    e = cudaMemset(base, 0, counters_end);
    if (e != cudaSuccess) { cudaFree(base); return cuda_fail(h, e, "workspace memset"); }
    if (w.base) cudaFree(w.base);
    drop_graphs(h);
    uint8_t *b = static_cast<uint8_t *>(base);
    w.base = base; w.bytes = off; w.counters_bytes = counters_end;
    w.T = T; w.D = D; w.E = E; w.K = K; w.I = I; w.TK = TK;
    w.x = reinterpret_cast<float *>(b + o_x);
    w.xq = Q8Rows{reinterpret_cast<int8_t *>(b + o_xq), reinterpret_cast<float *>(b + o_xd),
                  reinterpret_cast<int16_t *>(b + o_xb), 0};
    w.rt.idx = reinterpret_cast<int32_t *>(b + o_idx);
    w.rt.w = reinterpret_cast<float *>(b + o_w);
    w.rt.counts = reinterpret_cast<int32_t *>(b + o_cnt);
    w.rt.offsets = reinterpret_cast<int32_t *>(b + o_off);
    w.rt.perm = reinterpret_cast<int32_t *>(b + o_perm);
    w.rt.inv = reinterpret_cast<int32_t *>(b + o_inv);
    w.rt.act = reinterpret_cast<int32_t *>(b + o_act);
    w.rt.pairs = reinterpret_cast<int2 *>(b + o_pairs);
    w.rt.summary = reinterpret_cast<int32_t *>(b + o_sum);
    w.rt.tok_count = reinterpret_cast<uint32_t *>(b + o_tc);
    w.rt.done = reinterpret_cast<uint32_t *>(b + o_done);
    w.rt.logits = reinterpret_cast<float *>(b + o_log);
    w.rt.chunk = reinterpret_cast<int32_t *>(b + o_chunk);
    w.rt.rms = reinterpret_cast<float *>(b + o_rms);
    w.rt.err = h->dev_err;
    w.rt.loads = h->loads;
    w.h = reinterpret_cast<float *>(b + o_h);
    w.hq = Q8Rows{reinterpret_cast<int8_t *>(b + o_hq), reinterpret_cast<float *>(b + o_hd),
                  reinterpret_cast<int16_t *>(b + o_hb), 0};
    w.y = reinterpret_cast<float *>(b + o_y);
    w.gbar = reinterpret_cast<unsigned *>(b + o_gbar);
    w.xrec = b + o_xrec;
    w.scores = reinterpret_cast<float *>(b + o_scores);
    w.u = reinterpret_cast<float *>(b + o_u);
    w.tiles_gu = b + o_tgu;
    w.tiles_dn = b + o_tdn;
    w.n_tiles = reinterpret_cast<int32_t *>(b + o_nt);
    w.max_tiles_gu = (uint32_t)mt_gu;
    w.max_tiles_dn = (uint32_t)mt_dn;
    w.utiles_gu = reinterpret_cast<LfmUTile *>(b + o_utgu);
    w.utiles_dn = reinterpret_cast<LfmUTile *>(b + o_utdn);
    w.utbs = reinterpret_cast<LfmUTokBlock *>(b + o_utbs);
    w.ucounts = reinterpret_cast<int32_t *>(b + o_ucnt);
    w.xt = b + o_xt;
    w.umax_gu = (uint32_t)umax_gu;
    w.umax_dn = (uint32_t)umax_dn;
    w.umax_tb = (uint32_t)umax_tb;
    return LFM_GPU_OK;
}

lfm_gpu_status_t check_layer_shape(lfm_gpu_moe_t *h, uint32_t layer, uint32_t D, uint32_t E, uint32_t K,
                                   uint32_t I) {
    if (layer >= LFM_GPU_MOE_MAX_LAYERS) return fail(h, LFM_GPU_ERR_INVALID_ARG, "layer %u out of range", layer);
    if (D == 0 || D % 256 || I == 0 || I % 256)
        return fail(h, LFM_GPU_ERR_INVALID_ARG, "D=%u and I=%u must be positive multiples of 256", D, I);
    if (D > LFM_GPU_MAX_D || I > 16384)
        return fail(h, LFM_GPU_ERR_UNSUPPORTED, "D=%u / I=%u above this build's limits (8192 / 16384)", D, I);
    if (E == 0 || E > LFM_GPU_MOE_MAX_EXPERTS) return fail(h, LFM_GPU_ERR_INVALID_ARG, "E=%u not in 1..256", E);
    if (K == 0 || K > LFM_GPU_MOE_MAX_TOP_K || K > E)
        return fail(h, LFM_GPU_ERR_INVALID_ARG, "K=%u not in 1..min(8,E)", K);
    return LFM_GPU_OK;
}

/* Launch one step (`kernels` kernel launches), bracketed by events when profiling is on. */
template <typename F>
cudaError_t timed(lfm_gpu_moe_t *h, int kid, cudaStream_t s, F &&launch, uint32_t kernels = 1) {
    if (!h->prof) {
        h->stats.kernels_launched += kernels;
        return launch();
    }
    ProfRec r{kid, nullptr, nullptr};
    cudaError_t e = cudaEventCreate(&r.a);
    if (e == cudaSuccess) e = cudaEventCreate(&r.b);
    if (e == cudaSuccess) e = cudaEventRecord(r.a, s);
    if (e == cudaSuccess) e = launch();
    if (e == cudaSuccess) e = cudaEventRecord(r.b, s);
    if (e == cudaSuccess) {
        h->recs.push_back(r);
        h->stats.kernels_launched += kernels;
    } else {
        if (r.a) cudaEventDestroy(r.a);
        if (r.b) cudaEventDestroy(r.b);
    }
    return e;
}

/* Everything after routing: gate|up + SwiGLU, Q8_K(h), down, combine into x.
 * T > 16: grouped GEMMs on the tensor cores -- tcgen05 (k_umma.cu, token
 * blocks sized to the tokens per expert) where rows % 128 == 0, else mma.sync
 * (k_gemm.cu) for prefill-sized loads; otherwise the grouped GEMVs. */
/* The tcgen05 tile plans a forward of T tokens on L needs, for the dispatch
 * step to build (nt == 0 when the tcgen05 GEMMs are not the path). */
UmmaPlanOut umma_plan_for(lfm_gpu_moe_t *h, const MoeLayerDev &L, uint32_t T) {
    UmmaPlanOut p{};
    if (!(h->use_gemm && h->use_umma && T > LFM_FUSED_MAX_T && lfm_umma_ok(L.I) && lfm_umma_ok(L.D)) || L.down_q6k)
        return p;
    Workspace &w = h->ws;
    const uint32_t TK = T * lfm_layer_K(L), E = lfm_layer_E(L);
    p.nt = lfm_umma_nt(TK, E);
    p.rows_gu = L.I;
    p.rows_dn = L.D;
    p.tiles_gu = w.utiles_gu;
    p.tiles_dn = w.utiles_dn;
    p.tbs = w.utbs;
    p.counts = w.ucounts;
    p.max_tb = (uint32_t)lfm_umma_tb_max(TK, E, p.nt);
    p.max_gu = 2 * (uint32_t)lfm_umma_tiles_max(L.I, TK, E, p.nt); /* gate and up */
    p.max_dn = (uint32_t)lfm_umma_tiles_max(L.D, TK, E, p.nt);
    return p;
}

lfm_gpu_status_t run_experts(lfm_gpu_moe_t *h, const MoeLayerDev &L, float *x, uint32_t T, Q8Rows xq,
                             cudaStream_t s, bool pdl, const UmmaPlanOut &plan) {
    Workspace &w = h->ws;
    Q8Rows hq = w.hq; hq.cols = L.I;
    const int grid = h->sm_count;
    const uint32_t K = lfm_layer_K(L);
    const bool prefill = h->use_gemm && T > LFM_FUSED_MAX_T && (uint64_t)T * K >= 32ull * lfm_layer_E(L);
    if (plan.nt) { /* the dispatch step built the tile plans */
        const uint32_t TK = T * K, E = lfm_layer_E(L), nt = plan.nt, mtb = plan.max_tb;
        /* chained with programmatic dependent launch: every kernel waits (griddepcontrol.wait) before it
         * touches what its predecessor writes, so only launch latency and prologues overlap */
        LFM_CUDA(h, timed(h, K_XT, s, [&] {
            return lfm_launch_xt_gather(xq, w.rt.perm, K, w.utbs, w.ucounts + 1, mtb, nt, w.xt, s, pdl);
        }));
        LFM_CUDA(h, timed(h, K_GEMM_GU, s, [&] { /* gate and up in one launch */
            return lfm_launch_q4k_umma(L.gate, L.up, E, L.I, L.D, w.xt, nt, w.utiles_gu, w.utbs, w.ucounts, w.h, w.u,
                                       w.rt.err, grid, s, nullptr, pdl);
        }));
        LFM_CUDA(h, timed(h, K_SWIGLU, s, [&] {
            return lfm_launch_swiglu_xt(w.h, w.u, L.I, w.utbs, w.ucounts + 3, mtb, nt, w.xt, s, pdl);
        }));
        LFM_CUDA(h, timed(h, K_GEMM_D, s, [&] {
            return lfm_launch_q4k_umma(L.down, L.down, E, L.D, L.I, w.xt, nt, w.utiles_dn, w.utbs, w.ucounts + 2, w.y, w.y,
                                       w.rt.err, grid, s, nullptr, pdl);
        }));
        LFM_CUDA(h, timed(h, K_COMBINE, s, [&] { return lfm_launch_combine(L, x, T, w.rt, w.y, s, pdl); }));
        return LFM_GPU_OK;
    }
    if (prefill) {
        LFM_CUDA(h, timed(h, K_PLAN, s, [&] {
            cudaError_t e = lfm_launch_gemm_plan(w.rt, L.I, w.tiles_gu, w.n_tiles, w.max_tiles_gu, s);
            return e == cudaSuccess ? lfm_launch_gemm_plan(w.rt, L.D, w.tiles_dn, w.n_tiles + 1, w.max_tiles_dn, s) : e;
        }, 2));
        LFM_CUDA(h, timed(h, K_GEMM_G, s, [&] {
            return lfm_launch_q4k_gemm(L.gate, L.I, L.D, xq, w.rt.perm, K, w.tiles_gu, w.n_tiles, w.h, w.rt.err, grid, s);
        }));
        LFM_CUDA(h, timed(h, K_GEMM_U, s, [&] {
            return lfm_launch_q4k_gemm(L.up, L.I, L.D, xq, w.rt.perm, K, w.tiles_gu, w.n_tiles, w.u, w.rt.err, grid, s);
        }));
        LFM_CUDA(h, timed(h, K_SWIGLU, s, [&] { return lfm_launch_swiglu_quant(w.h, w.u, T * K, L.I, hq, s); }));
        LFM_CUDA(h, timed(h, K_GEMM_D, s, [&] {
            if (L.down_q6k) return lfm_launch_down_q6k(L, hq, w.rt, w.y, grid, s);
            return lfm_launch_q4k_gemm(L.down, L.D, L.I, hq, nullptr, 1, w.tiles_dn, w.n_tiles + 1, w.y, w.rt.err, grid, s);
        }));
        LFM_CUDA(h, timed(h, K_COMBINE, s, [&] { return lfm_launch_combine(L, x, T, w.rt, w.y, s, false); }));
        return LFM_GPU_OK;
    }
    LFM_CUDA(h, timed(h, K_GATEUP, s, [&] { return lfm_launch_gateup(L, xq, w.rt, w.h, grid, s, pdl); }));
    LFM_CUDA(h, timed(h, K_QUANT_H, s, [&] { return lfm_launch_quant_rows(w.h, T * K, L.I, hq, s, pdl); }));
    LFM_CUDA(h, timed(h, K_DOWN, s, [&] {
        return L.down_q6k ? lfm_launch_down_q6k(L, hq, w.rt, w.y, grid, s) : lfm_launch_down(L, hq, w.rt, w.y, grid, s, pdl);
    }));
    LFM_CUDA(h, timed(h, K_COMBINE, s, [&] { return lfm_launch_combine(L, x, T, w.rt, w.y, s, pdl); }));
    return LFM_GPU_OK;
}

/* One layer forward on device x; `stream` already resolved.
 * T <= LFM_FUSED_MAX_T: one cooperative launch of the fused layer (k_layer.cu).
 * Otherwise route(+dispatch) -> gate|up(+SwiGLU) -> h->Q8_K -> down -> combine
 * chained with programmatic dependent launch.
 * Profiling brackets each launch with events, which breaks the PDL overlap,
 * so it is turned off while profiling. */
lfm_gpu_status_t forward_layer(lfm_gpu_moe_t *h, const LayerSlot &S, float *x, uint32_t T, cudaStream_t s) {
    const MoeLayerDev &L = S.dev;
    Workspace &w = h->ws;  /* sized for the whole call by forward_common */
    Q8Rows xq = w.xq; xq.cols = L.D;
    const bool pdl = !h->prof && h->use_pdl;
    const int grid = h->sm_count;
    if (h->use_fused && !L.down_q6k && lfm_fused_ok(L, T, grid)) {
        LFM_CUDA(h, timed(h, K_LAYER, s, [&] { return lfm_launch_layer_fused(L, x, T, w.rt, w.h, w.y, w.gbar, w.xrec, w.scores, grid, s); }));
        return LFM_GPU_OK;
    }
    RouteTables rt = w.rt;
    rt.plan = umma_plan_for(h, L, T);
    LFM_CUDA(h, timed(h, K_ROUTE, s, [&] { return lfm_launch_route(L, x, T, xq, rt, s, pdl); },
                      lfm_route_kernels(L, T)));
    return run_experts(h, L, x, T, xq, s, pdl, rt.plan);
}

lfm_gpu_status_t read_device_error(lfm_gpu_moe_t *h) {
    uint32_t e = 0;
    LFM_CUDA(h, cudaMemcpy(&e, h->dev_err, sizeof e, cudaMemcpyDeviceToHost));
    if (e == 0) return LFM_GPU_OK;
    LFM_CUDA(h, cudaMemset(h->dev_err, 0, sizeof(uint32_t)));
    /* an abandoned forward can leave completion counters part-way: clear them */
    if (h->ws.base) LFM_CUDA(h, cudaMemset(h->ws.base, 0, h->ws.counters_bytes));
    if (e & LFM_DEVERR_TIMEOUT) return fail(h, LFM_GPU_ERR_TIMEOUT, "device wait timed out (0x%x)", e);
    return fail(h, LFM_GPU_ERR_DEVICE_CHECK, "device bounds check tripped (0x%x)", e);
}

}  // namespace

LFM_API lfm_gpu_status_t lfm_gpu_moe_create(lfm_gpu_moe_t **out, int device_id) {
    if (!out) return LFM_GPU_ERR_INVALID_ARG;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device_id < 0 || device_id >= n) return LFM_GPU_ERR_INVALID_ARG;
    lfm_gpu_moe_t *h = new (std::nothrow) lfm_gpu_moe_t();
    if (!h) return LFM_GPU_ERR_OOM;
    h->device = device_id;
    {
        const char *nf = getenv("LFM_GPU_MOE_NO_FUSED"); /* force the separate-kernel path (A/B runs) */
        h->use_fused = !(nf && nf[0] && nf[0] != '0');
        const char *ng = getenv("LFM_GPU_MOE_NO_GEMM"); /* force the GEMV path for prefill (A/B runs) */
        h->use_gemm = !(ng && ng[0] && ng[0] != '0');
        const char *nu = getenv("LFM_GPU_MOE_NO_UMMA"); /* prefill GEMMs on mma.sync instead of tcgen05 (A/B runs) */
        h->use_umma = !(nu && nu[0] && nu[0] != '0');
        const char *np = getenv("LFM_GPU_MOE_NO_PDL"); /* plain stream order between kernels (A/B runs) */
        h->use_pdl = !(np && np[0] && np[0] != '0');
    }
    DeviceGuard g(device_id);
    if (cudaDeviceGetAttribute(&h->sm_count, cudaDevAttrMultiProcessorCount, device_id) != cudaSuccess ||
        h->sm_count <= 0)
        h->sm_count = 148;
    if (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&h->dev_err, sizeof(uint32_t)) != cudaSuccess ||
        cudaMemset(h->dev_err, 0, sizeof(uint32_t)) != cudaSuccess ||
        cudaMalloc(&h->loads, 2 * sizeof(unsigned long long)) != cudaSuccess ||
        cudaMemset(h->loads, 0, 2 * sizeof(unsigned long long)) != cudaSuccess) {
        lfm_gpu_moe_destroy(h);
        return LFM_GPU_ERR_CUDA;
    }
    *out = h;
    return LFM_GPU_OK;
}

namespace {
void ep_release(lfm_gpu_moe_t *h); /* expert-parallel arena and peer mappings (below) */
}  // namespace

LFM_API void lfm_gpu_moe_destroy(lfm_gpu_moe_t *h) {
    if (!h) return;
    DeviceGuard g(h->device);
    if (h->stream) cudaStreamSynchronize(h->stream);
    drop_graphs(h);
    for (LayerSlot &L : h->layers) free_layer(L);
    if (h->ws.base) cudaFree(h->ws.base);
    if (h->dev_err) cudaFree(h->dev_err);
    if (h->loads) cudaFree(h->loads);
    for (ProfRec &r : h->recs) { cudaEventDestroy(r.a); cudaEventDestroy(r.b); }
    if (h->ep.attached) {
        cudaDeviceSynchronize();
        ep_release(h);
    }
    if (h->stream) cudaStreamDestroy(h->stream);
    delete h;
}

LFM_API const char *lfm_gpu_moe_last_error(const lfm_gpu_moe_t *h) { return h ? h->err : "null handle"; }

/* Upload of a layer with experts [first, first + n) of E (all of them when n == E). */
static lfm_gpu_status_t upload_layer_impl(lfm_gpu_moe_t *h, uint32_t layer, uint32_t D, uint32_t E, uint32_t K,
                                          uint32_t I, float eps, const float *ffn_norm, const float *router_w,
                                          const float *exp_probs_b, const void *gate_exps, const void *up_exps,
                                          const void *down_exps, uint32_t w_type, uint32_t down_type,
                                          int norm_topk_prob, float routed_scale, uint32_t first, uint32_t n) {
    if (!h) return LFM_GPU_ERR_INVALID_ARG;
    lfm_gpu_status_t st = check_layer_shape(h, layer, D, E, K, I);
    if (st != LFM_GPU_OK) return st;
    if (n == 0 || first >= E || n > E - first)
        return fail(h, LFM_GPU_ERR_INVALID_ARG, "expert shard [%u, %u+%u) not inside 0..%u", first, first, n, E);
    if (w_type != LFM_GGML_TYPE_Q4_K) return fail(h, LFM_GPU_ERR_UNSUPPORTED, "expert weight type %u (only Q4_K=12)", w_type);
    if (down_type != LFM_GGML_TYPE_Q4_K && down_type != LFM_GGML_TYPE_Q6_K)
        return fail(h, LFM_GPU_ERR_UNSUPPORTED, "down weight type %u (Q4_K=12 or Q6_K=14)", down_type);
    const bool q6k = down_type == LFM_GGML_TYPE_Q6_K;
    if (q6k && I > 3072)
        return fail(h, LFM_GPU_ERR_UNSUPPORTED, "Q6_K down with I=%u (the Q6_K kernel stages rows of I <= 3072)", I);
    if (!router_w || !gate_exps || !up_exps || !down_exps) return fail(h, LFM_GPU_ERR_INVALID_ARG, "null tensor");
    DeviceGuard g(h->device);
    drop_graphs(h);
    LayerSlot &S = h->layers[layer];
    free_layer(S);
    const size_t nbd = D / 256, nbi = I / 256;
    const size_t sz[6] = {sizeof(float) * D, sizeof(float) * E * D, sizeof(float) * ((E + 3) / 4 * 4),
                          (size_t)n * I * nbd * LFM_Q4K_BYTES, (size_t)n * I * nbd * LFM_Q4K_BYTES,
                          (size_t)n * D * nbi * (q6k ? LFM_Q6K_BYTES : LFM_Q4K_BYTES)};
    const void *src[6] = {ffn_norm, router_w, exp_probs_b, gate_exps, up_exps, down_exps};
    for (int i = 0; i < 6; ++i) {
        if (i == 0 && !ffn_norm) continue;
        if (i == 2 && !exp_probs_b) continue;
        /* a Q6_K down tensor gets 16 bytes of slack: k_q6k.cu copies 16-byte aligned spans around its rows */
        cudaError_t e = cudaMalloc(&S.bufs[i], sz[i] + (i == 5 && q6k ? 16 : 0));
        if (e == cudaSuccess && i == 2) e = cudaMemset(S.bufs[i], 0, sz[i]); /* bias padded to 16 bytes */
        if (e == cudaSuccess)
            e = cudaMemcpy(S.bufs[i], src[i], i == 2 ? sizeof(float) * E : sz[i], cudaMemcpyHostToDevice);
        if (e != cudaSuccess) { free_layer(S); return cuda_fail(h, e, "layer upload"); }
        S.sizes[i] = sz[i];
    }
    S.dev = MoeLayerDev{D, E, K, I, 0, eps, routed_scale, norm_topk_prob ? 1 : 0,
                        static_cast<float *>(S.bufs[0]), static_cast<float *>(S.bufs[1]),
                        static_cast<float *>(S.bufs[2]), static_cast<const uint8_t *>(S.bufs[3]),
                        static_cast<const uint8_t *>(S.bufs[4]), static_cast<const uint8_t *>(S.bufs[5]),
                        q6k ? 1u : 0u};
    S.ep_first = first;
    S.ep_count = n;
    S.present = true;
    return LFM_GPU_OK;
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_upload_layer(lfm_gpu_moe_t *h, uint32_t layer, uint32_t D, uint32_t E,
                                                  uint32_t K, uint32_t I, float eps, const float *ffn_norm,
                                                  const float *router_w, const float *exp_probs_b,
                                                  const void *gate_exps, const void *up_exps,
                                                  const void *down_exps, uint32_t w_type, int norm_topk_prob,
                                                  float routed_scale) {
    return upload_layer_impl(h, layer, D, E, K, I, eps, ffn_norm, router_w, exp_probs_b, gate_exps, up_exps,
                             down_exps, w_type, w_type, norm_topk_prob, routed_scale, 0, E);
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_upload_layer_shard(lfm_gpu_moe_t *h, uint32_t layer, uint32_t D, uint32_t E,
                                                        uint32_t K, uint32_t I, float eps, const float *ffn_norm,
                                                        const float *router_w, const float *exp_probs_b,
                                                        const void *gate_local, const void *up_local,
                                                        const void *down_local, uint32_t w_type,
                                                        int norm_topk_prob, float routed_scale,
                                                        uint32_t expert_first, uint32_t n_local) {
    return upload_layer_impl(h, layer, D, E, K, I, eps, ffn_norm, router_w, exp_probs_b, gate_local, up_local,
                             down_local, w_type, w_type, norm_topk_prob, routed_scale, expert_first, n_local);
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_upload_layer_typed(lfm_gpu_moe_t *h, uint32_t layer, uint32_t D, uint32_t E,
                                                        uint32_t K, uint32_t I, float eps, const float *ffn_norm,
                                                        const float *router_w, const float *exp_probs_b,
                                                        const void *gate_exps, const void *up_exps,
                                                        const void *down_exps, uint32_t gate_up_type,
                                                        uint32_t down_type, int norm_topk_prob, float routed_scale) {
    return upload_layer_impl(h, layer, D, E, K, I, eps, ffn_norm, router_w, exp_probs_b, gate_exps, up_exps,
                             down_exps, gate_up_type, down_type, norm_topk_prob, routed_scale, 0, E);
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_upload_dense(lfm_gpu_moe_t *h, uint32_t layer, uint32_t D, uint32_t I,
                                                  float eps, const float *ffn_norm, const void *gate,
                                                  const void *up, const void *down, uint32_t w_type) {
    if (!h) return LFM_GPU_ERR_INVALID_ARG;
    lfm_gpu_status_t st = check_layer_shape(h, layer, D, 1, 1, I);
    if (st != LFM_GPU_OK) return st;
    if (w_type != LFM_GGML_TYPE_Q4_K) return fail(h, LFM_GPU_ERR_UNSUPPORTED, "dense weight type %u (only Q4_K=12)", w_type);
    if (!gate || !up || !down) return fail(h, LFM_GPU_ERR_INVALID_ARG, "null tensor");
    DeviceGuard g(h->device);
    drop_graphs(h);
    LayerSlot &S = h->layers[layer];
    free_layer(S);
    const size_t nbd = D / 256, nbi = I / 256;
    const size_t sz[4] = {sizeof(float) * D, (size_t)I * nbd * LFM_Q4K_BYTES, (size_t)I * nbd * LFM_Q4K_BYTES,
                          (size_t)D * nbi * LFM_Q4K_BYTES};
    const void *src[4] = {ffn_norm, gate, up, down};
    const int slot[4] = {0, 3, 4, 5};
    for (int i = 0; i < 4; ++i) {
        if (i == 0 && !ffn_norm) continue;
        cudaError_t e = cudaMalloc(&S.bufs[slot[i]], sz[i]);
        if (e == cudaSuccess) e = cudaMemcpy(S.bufs[slot[i]], src[i], sz[i], cudaMemcpyHostToDevice);
        if (e != cudaSuccess) { free_layer(S); return cuda_fail(h, e, "dense upload"); }
        S.sizes[slot[i]] = sz[i];
    }
    S.dev = MoeLayerDev{D, 0, 0, I, 1, eps, 1.0f, 0, static_cast<float *>(S.bufs[0]), nullptr, nullptr,
                        static_cast<const uint8_t *>(S.bufs[3]), static_cast<const uint8_t *>(S.bufs[4]),
                        static_cast<const uint8_t *>(S.bufs[5])};
    S.present = true;
    return LFM_GPU_OK;
}

static lfm_gpu_status_t synth_layer_impl(lfm_gpu_moe_t *h, uint32_t layer, uint32_t D, uint32_t E, uint32_t K,
                                         uint32_t I, float eps, const uint64_t seeds[5], float w_std,
                                         float router_std, float bias_std, const float *exp_probs_b,
                                         uint32_t first, uint32_t n) {
    if (!h || !seeds) return LFM_GPU_ERR_INVALID_ARG;
    lfm_gpu_status_t st = check_layer_shape(h, layer, D, E, K, I);
    if (st != LFM_GPU_OK) return st;
    if (n == 0 || first >= E || n > E - first)
        return fail(h, LFM_GPU_ERR_INVALID_ARG, "expert shard [%u, %u+%u) not inside 0..%u", first, first, n, E);
    DeviceGuard g(h->device);
    drop_graphs(h);
    LayerSlot &S = h->layers[layer];
    free_layer(S);
    const size_t nbd = D / 256, nbi = I / 256;
    const size_t sz[6] = {sizeof(float) * D, sizeof(float) * E * D, sizeof(float) * ((E + 3) / 4 * 4),
                          (size_t)n * I * nbd * LFM_Q4K_BYTES, (size_t)n * I * nbd * LFM_Q4K_BYTES,
                          (size_t)n * D * nbi * LFM_Q4K_BYTES};
    for (int i = 0; i < 6; ++i) {
        cudaError_t e = cudaMalloc(&S.bufs[i], sz[i]);
        if (e != cudaSuccess) { free_layer(S); return cuda_fail(h, e, "synth layer cudaMalloc"); }
        S.sizes[i] = sz[i];
    }
    cudaStream_t s = h->stream;
    cudaError_t e = lfm_launch_synth_f32(static_cast<float *>(S.bufs[0]), D, 0, 1.0f, 0.0f, s);
    if (e == cudaSuccess) e = lfm_launch_synth_f32(static_cast<float *>(S.bufs[1]), (uint64_t)E * D, seeds[3], 0.0f, router_std, s);
    if (e == cudaSuccess) {
        e = cudaMemsetAsync(S.bufs[2], 0, sz[2], s);
        if (e == cudaSuccess && exp_probs_b)
            e = cudaMemcpyAsync(S.bufs[2], exp_probs_b, sizeof(float) * E, cudaMemcpyHostToDevice, s);
        else if (e == cudaSuccess)
            e = lfm_launch_synth_f32(static_cast<float *>(S.bufs[2]), E, seeds[4], 0.0f, bias_std, s);
    }
    /* the shard's blocks are blocks [first*rows*nb, ...) of the full tensors */
    if (e == cudaSuccess)
        e = lfm_launch_synth_q4k(static_cast<uint8_t *>(S.bufs[3]), (uint64_t)n * I * nbd, seeds[0], w_std, s,
                                 (uint64_t)first * I * nbd);
    if (e == cudaSuccess)
        e = lfm_launch_synth_q4k(static_cast<uint8_t *>(S.bufs[4]), (uint64_t)n * I * nbd, seeds[1], w_std, s,
                                 (uint64_t)first * I * nbd);
    if (e == cudaSuccess)
        e = lfm_launch_synth_q4k(static_cast<uint8_t *>(S.bufs[5]), (uint64_t)n * D * nbi, seeds[2], w_std, s,
                                 (uint64_t)first * D * nbi);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) { free_layer(S); return cuda_fail(h, e, "synth layer"); }
    S.dev = MoeLayerDev{D, E, K, I, 0, eps, 1.0f, 1, static_cast<float *>(S.bufs[0]), static_cast<float *>(S.bufs[1]),
                        static_cast<float *>(S.bufs[2]), static_cast<const uint8_t *>(S.bufs[3]),
                        static_cast<const uint8_t *>(S.bufs[4]), static_cast<const uint8_t *>(S.bufs[5])};
    S.ep_first = first;
    S.ep_count = n;
    S.present = true;
    return LFM_GPU_OK;
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_synth_layer(lfm_gpu_moe_t *h, uint32_t layer, uint32_t D, uint32_t E,
                                                 uint32_t K, uint32_t I, float eps, const uint64_t seeds[5],
                                                 float w_std, float router_std, float bias_std,
                                                 const float *exp_probs_b) {
    return synth_layer_impl(h, layer, D, E, K, I, eps, seeds, w_std, router_std, bias_std, exp_probs_b, 0, E);
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_synth_layer_shard(lfm_gpu_moe_t *h, uint32_t layer, uint32_t D, uint32_t E,
                                                       uint32_t K, uint32_t I, float eps, const uint64_t seeds[5],
                                                       float w_std, float router_std, float bias_std,
                                                       const float *exp_probs_b, uint32_t expert_first,
                                                       uint32_t n_local) {
    return synth_layer_impl(h, layer, D, E, K, I, eps, seeds, w_std, router_std, bias_std, exp_probs_b,
                            expert_first, n_local);
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_reserve(lfm_gpu_moe_t *h, uint32_t max_tokens) {
    if (!h) return LFM_GPU_ERR_INVALID_ARG;
    if (max_tokens == 0 || max_tokens > 65535) return fail(h, LFM_GPU_ERR_INVALID_ARG, "max_tokens %u not in 1..65535", max_tokens);
    uint32_t D = 0, E = 1, K = 1, I = 0;
    for (const LayerSlot &S : h->layers) {
        if (!S.present) continue;
        D = S.dev.D > D ? S.dev.D : D;
        I = S.dev.I > I ? S.dev.I : I;
        E = S.dev.E > E ? S.dev.E : E;
        K = S.dev.K > K ? S.dev.K : K;
    }
    if (D == 0) return fail(h, LFM_GPU_ERR_NOT_READY, "reserve before any layer upload");
    DeviceGuard g(h->device);
    return ensure_workspace(h, max_tokens, D, E, K, I);
}

namespace {
lfm_gpu_status_t ep_forward_layer(lfm_gpu_moe_t *h, const LayerSlot &S, float *x, uint32_t T, cudaStream_t s);
}  // namespace

/* Layer l of a stack: expert-parallel step for a MoE shard when ep, else the regular forward. */
static lfm_gpu_status_t stack_layer(lfm_gpu_moe_t *h, uint32_t l, float *x, uint32_t T, cudaStream_t s, bool ep) {
    const LayerSlot &S = h->layers[l];
    if (ep && !S.dev.dense) return ep_forward_layer(h, S, x, T, s);
    if (T == 0) return LFM_GPU_OK;
    return forward_layer(h, S, x, T, s);
}

/* Replay (capturing on first use) the graph of layers [first, first+n) on x.
 * Capture runs on the handle's own stream (never the caller's, which may be
 * the legacy default stream); the replay is launched on the caller's stream. */
static lfm_gpu_status_t run_graph(lfm_gpu_moe_t *h, uint32_t first, uint32_t n, float *x, uint32_t T,
                                  cudaStream_t s, bool ep = false) {
    GraphEntry *hit = nullptr;
    for (GraphEntry &g : h->graphs)
        if (g.first == first && g.n == n && g.T == T && g.x == x && g.ep == ep) { hit = &g; break; }
    if (!hit) {
        /* first call with this key: run eagerly (kernel attributes get set
         * outside any capture), then capture the same launches for replay */
        for (uint32_t l = first; l < first + n; ++l) {
            lfm_gpu_status_t st = stack_layer(h, l, x, T, s, ep);
            if (st != LFM_GPU_OK) return st;
        }
        if (h->graphs.size() >= kMaxGraphs) {
            cudaGraphExecDestroy(h->graphs.front().exec);
            h->graphs.erase(h->graphs.begin());
        }
        LFM_CUDA(h, cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal));
        const uint32_t k0 = h->stats.kernels_launched;
        lfm_gpu_status_t st = LFM_GPU_OK;
        for (uint32_t l = first; l < first + n && st == LFM_GPU_OK; ++l)
            st = stack_layer(h, l, x, T, h->stream, ep);
        cudaGraph_t graph = nullptr;
        const cudaError_t ce = cudaStreamEndCapture(h->stream, &graph);
        if (st != LFM_GPU_OK) { if (graph) cudaGraphDestroy(graph); return st; }
        if (ce != cudaSuccess) return cuda_fail(h, ce, "cudaStreamEndCapture");
        cudaGraphExec_t exec = nullptr;
        const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        if (ie != cudaSuccess) return cuda_fail(h, ie, "cudaGraphInstantiate");
        h->graphs.push_back(GraphEntry{first, n, T, ep, x, h->stats.kernels_launched - k0, exec});
        h->stats.kernels_launched = k0;
        return LFM_GPU_OK;
    }
    LFM_CUDA(h, cudaGraphLaunch(hit->exec, s));
    h->stats.kernels_launched += hit->kernels;
    return LFM_GPU_OK;
}

static lfm_gpu_status_t forward_common(lfm_gpu_moe_t *h, uint32_t first, uint32_t n, float *x, uint32_t T,
                                       int x_on_device, void *stream) {
    if (!h || !x) return LFM_GPU_ERR_INVALID_ARG;
    if (T == 0) return LFM_GPU_OK;
    if (T > 65535) return fail(h, LFM_GPU_ERR_INVALID_ARG, "T=%u above 65535 tokens per call", T);
    if (x_on_device && (reinterpret_cast<uintptr_t>(x) & 15u))
        return fail(h, LFM_GPU_ERR_INVALID_ARG, "device x must be 16-byte aligned (bulk copies read it)");
    if (n == 0 || first >= LFM_GPU_MOE_MAX_LAYERS || n > LFM_GPU_MOE_MAX_LAYERS - first)
        return fail(h, LFM_GPU_ERR_INVALID_ARG, "layer range [%u, %u+%u) invalid", first, first, n);
    uint32_t D = 0, E = 1, K = 1, I = 0;
    for (uint32_t l = first; l < first + n; ++l) {
        const LayerSlot &S = h->layers[l];
        if (!S.present) return fail(h, LFM_GPU_ERR_NOT_READY, "layer %u not uploaded", l);
        if (S.ep_count && S.ep_count != S.dev.E)
            return fail(h, LFM_GPU_ERR_UNSUPPORTED, "layer %u holds an expert shard: use the lfm_gpu_moe_ep_* calls", l);
        if (D && S.dev.D != D) return fail(h, LFM_GPU_ERR_INVALID_ARG, "layers disagree on D");
        D = S.dev.D;
        E = S.dev.E > E ? S.dev.E : E;
        K = S.dev.K > K ? S.dev.K : K;
        I = S.dev.I > I ? S.dev.I : I;
    }
    DeviceGuard g(h->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);  /* NULL = the CUDA default stream */
    lfm_gpu_status_t st = ensure_workspace(h, T, D, E, K, I);
    if (st != LFM_GPU_OK) return st;
    h->stats = lfm_gpu_moe_stats_t{};
    h->stats.tokens = T;
    float *xd = x;
    if (!x_on_device) {
        xd = h->ws.x;
        LFM_CUDA(h, cudaMemcpyAsync(xd, x, sizeof(float) * T * D, cudaMemcpyHostToDevice, s));
    }
    if (h->use_graphs && !h->prof) {
        st = run_graph(h, first, n, xd, T, s);
        if (st != LFM_GPU_OK) return st;
    } else {
        for (uint32_t l = first; l < first + n; ++l) {
            st = forward_layer(h, h->layers[l], xd, T, s);
            if (st != LFM_GPU_OK) return st;
        }
    }
    if (!x_on_device) {
        LFM_CUDA(h, cudaMemcpyAsync(x, xd, sizeof(float) * T * D, cudaMemcpyDeviceToHost, s));
        LFM_CUDA(h, cudaStreamSynchronize(s));
        return read_device_error(h);
    }
    return LFM_GPU_OK;
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_forward(lfm_gpu_moe_t *h, uint32_t layer, float *x, uint32_t T,
                                             int x_on_device, void *stream) {
    return forward_common(h, layer, 1, x, T, x_on_device, stream);
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_forward_stack(lfm_gpu_moe_t *h, uint32_t first, uint32_t n, float *x,
                                                   uint32_t T, int x_on_device, void *stream) {
    return forward_common(h, first, n, x, T, x_on_device, stream);
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_debug_route(lfm_gpu_moe_t *h, uint32_t layer, const float *x, uint32_t T,
                                                 uint32_t *idx_out, float *w_out, void *q8_out) {
    if (!h || !x || !idx_out || !w_out) return LFM_GPU_ERR_INVALID_ARG;
    if (layer >= LFM_GPU_MOE_MAX_LAYERS || !h->layers[layer].present || h->layers[layer].dev.dense)
        return fail(h, LFM_GPU_ERR_NOT_READY, "layer %u is not an uploaded MoE layer", layer);
    if (T == 0 || T > 65535) return fail(h, LFM_GPU_ERR_INVALID_ARG, "T=%u not in 1..65535", T);
    const MoeLayerDev &L = h->layers[layer].dev;
    DeviceGuard g(h->device);
    lfm_gpu_status_t st = ensure_workspace(h, T, L.D, L.E, L.K, L.I);
    if (st != LFM_GPU_OK) return st;
    cudaStream_t s = h->stream;
    Workspace &w = h->ws;
    Q8Rows xq = w.xq; xq.cols = L.D;
    LFM_CUDA(h, cudaMemcpyAsync(w.x, x, sizeof(float) * T * L.D, cudaMemcpyHostToDevice, s));
    LFM_CUDA(h, lfm_launch_route(L, w.x, T, xq, w.rt, s, false));
    LFM_CUDA(h, cudaMemcpyAsync(idx_out, w.rt.idx, sizeof(int32_t) * T * L.K, cudaMemcpyDeviceToHost, s));
    LFM_CUDA(h, cudaMemcpyAsync(w_out, w.rt.w, sizeof(float) * T * L.K, cudaMemcpyDeviceToHost, s));
    if (q8_out) {
        /* pack into the y buffer (T*K*D*4 bytes >= T*(D/256)*292), then copy out */
        uint8_t *tmp = reinterpret_cast<uint8_t *>(w.y);
        LFM_CUDA(h, lfm_launch_q8_to_gguf(xq, T, tmp, s));
        LFM_CUDA(h, cudaMemcpyAsync(q8_out, tmp, (size_t)T * (L.D / 256) * LFM_Q8K_BYTES, cudaMemcpyDeviceToHost, s));
    }
    LFM_CUDA(h, cudaStreamSynchronize(s));
    return read_device_error(h);
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_debug_q4k_rows(lfm_gpu_moe_t *h, const void *w, uint32_t n_rows,
                                                    uint32_t n_cols, const void *xq, uint32_t n_vec,
                                                    int32_t *sub_dots, int32_t *acc, int32_t *mins,
                                                    float *rows_out) {
    if (!h || !w || !xq || !sub_dots || !acc || !mins || !rows_out) return LFM_GPU_ERR_INVALID_ARG;
    if (n_cols == 0 || n_cols % 256 || n_cols > 32768 || n_rows == 0 || n_rows % 8 || n_vec == 0 || n_vec > 65535)
        return fail(h, LFM_GPU_ERR_INVALID_ARG, "bad debug shape rows=%u cols=%u vecs=%u", n_rows, n_cols, n_vec);
    DeviceGuard g(h->device);
    const size_t nb = n_cols / 256;
    const size_t wb = (size_t)n_rows * nb * LFM_Q4K_BYTES, xb = (size_t)n_vec * nb * LFM_Q8K_BYTES;
    const size_t no = (size_t)n_vec * n_rows;
    size_t off = 0;
    auto take = [&](size_t b) { const size_t o = off; off += align256(b); return o; };
    const size_t o_w = take(wb), o_x = take(xb), o_qs = take((size_t)n_vec * n_cols), o_d = take(4 * n_vec * nb),
                 o_bs = take(32 * n_vec * nb), o_sd = take(4 * no * nb * 8), o_a = take(4 * no * nb),
                 o_m = take(4 * no * nb), o_r = take(4 * no);
    uint8_t *buf = nullptr;
    LFM_CUDA(h, cudaMalloc(&buf, off));
    cudaStream_t s = h->stream;
    Q8Rows q{reinterpret_cast<int8_t *>(buf + o_qs), reinterpret_cast<float *>(buf + o_d),
             reinterpret_cast<int16_t *>(buf + o_bs), n_cols};
    cudaError_t e = cudaMemcpyAsync(buf + o_w, w, wb, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(buf + o_x, xq, xb, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = lfm_launch_gguf_to_q8(buf + o_x, n_vec, q, s);
    if (e == cudaSuccess)
        e = lfm_launch_debug_q4k_rows(buf + o_w, n_rows, n_cols, q, n_vec, reinterpret_cast<int32_t *>(buf + o_sd),
                                      reinterpret_cast<int32_t *>(buf + o_a), reinterpret_cast<int32_t *>(buf + o_m),
                                      reinterpret_cast<float *>(buf + o_r), s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(sub_dots, buf + o_sd, 4 * no * nb * 8, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(acc, buf + o_a, 4 * no * nb, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(mins, buf + o_m, 4 * no * nb, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(rows_out, buf + o_r, 4 * no, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    cudaFree(buf);
    if (e != cudaSuccess) return cuda_fail(h, e, "debug_q4k_rows");
    return LFM_GPU_OK;
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_debug_read_layer_range(lfm_gpu_moe_t *h, uint32_t layer, uint32_t which,
                                                            size_t offset, void *out, size_t bytes) {
    if (!h || !out || which > 5) return LFM_GPU_ERR_INVALID_ARG;
    if (layer >= LFM_GPU_MOE_MAX_LAYERS || !h->layers[layer].present)
        return fail(h, LFM_GPU_ERR_NOT_READY, "layer %u not uploaded", layer);
    const LayerSlot &S = h->layers[layer];
    if (!S.bufs[which]) return fail(h, LFM_GPU_ERR_NOT_READY, "layer %u has no tensor %u", layer, which);
    if (bytes == 0 || offset > S.sizes[which] || bytes > S.sizes[which] - offset)
        return fail(h, LFM_GPU_ERR_INVALID_ARG, "tensor %u holds %zu bytes, asked for [%zu, %zu+%zu)", which,
                    S.sizes[which], offset, offset, bytes);
    DeviceGuard g(h->device);
    LFM_CUDA(h, cudaStreamSynchronize(h->stream));
    LFM_CUDA(h, cudaMemcpy(out, static_cast<const uint8_t *>(S.bufs[which]) + offset, bytes, cudaMemcpyDeviceToHost));
    return LFM_GPU_OK;
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_debug_read_layer(lfm_gpu_moe_t *h, uint32_t layer, uint32_t which, void *out,
                                                      size_t bytes) {
    return lfm_gpu_moe_debug_read_layer_range(h, layer, which, 0, out, bytes);
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_sync(lfm_gpu_moe_t *h) {
    if (!h) return LFM_GPU_ERR_INVALID_ARG;
    DeviceGuard g(h->device);
    LFM_CUDA(h, cudaStreamSynchronize(h->stream));
    LFM_CUDA(h, cudaDeviceSynchronize());
    return read_device_error(h);
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_last_stats(const lfm_gpu_moe_t *hc, lfm_gpu_moe_stats_t *out) {
    lfm_gpu_moe_t *h = const_cast<lfm_gpu_moe_t *>(hc);
    if (!h || !out) return LFM_GPU_ERR_INVALID_ARG;
    DeviceGuard g(h->device);
    *out = h->stats;
    LFM_CUDA(h, cudaDeviceSynchronize());
    unsigned long long ld[2] = {0, 0};
    LFM_CUDA(h, cudaMemcpy(ld, h->loads, sizeof ld, cudaMemcpyDeviceToHost));
    out->expert_loads = ld[0];
    out->layer_runs = ld[1];
    if (h->ws.base) {
        int32_t sm[4] = {0, 0, 0, 0};
        LFM_CUDA(h, cudaMemcpy(sm, h->ws.rt.summary, sizeof sm, cudaMemcpyDeviceToHost));
        out->unique_experts = (uint32_t)sm[0];
        out->max_segment = (uint32_t)sm[1];
    }
    return LFM_GPU_OK;
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_profile(lfm_gpu_moe_t *h, int enable) {
    if (!h) return LFM_GPU_ERR_INVALID_ARG;
    h->prof = enable != 0;
    return LFM_GPU_OK;
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_profile_read(lfm_gpu_moe_t *h, lfm_gpu_moe_kernel_time_t *out, uint32_t cap,
                                                  uint32_t *n_out) {
    if (!h || (!out && cap) || !n_out) return LFM_GPU_ERR_INVALID_ARG;
    DeviceGuard g(h->device);
    LFM_CUDA(h, cudaDeviceSynchronize());
    double ms[K_COUNT] = {0};
    uint32_t cnt[K_COUNT] = {0};
    cudaError_t err = cudaSuccess;
    for (ProfRec &r : h->recs) {
        float t = 0.0f;
        cudaError_t e = cudaEventElapsedTime(&t, r.a, r.b);
        if (e != cudaSuccess && err == cudaSuccess) err = e;
        ms[r.kid] += t;
        cnt[r.kid] += 1;
        cudaEventDestroy(r.a);
        cudaEventDestroy(r.b);
    }
    h->recs.clear();
    if (err != cudaSuccess) return cuda_fail(h, err, "profile events");
    uint32_t n = 0;
    for (int k = 0; k < K_COUNT; ++k) {
        if (!cnt[k]) continue;
        if (n < cap) {
            snprintf(out[n].name, sizeof out[n].name, "%s", kKernelNames[k]);
            out[n].launches = cnt[k];
            out[n].total_ms = ms[k];
        }
        ++n;
    }
    *n_out = n;
    return LFM_GPU_OK;
}

/* ---- forward without allocation -------------------------------------------
 * The regular forward grows the handle's scratch on demand, which calls
 * cudaMalloc after a device-wide synchronisation.  A caller that must not
 * allocate mid-step (a serving engine with a memory plan fixed at load time, or
 * one that cannot stall every stream of the device for an allocation) uses
 * lfm_gpu_moe_forward_noalloc instead: its scratch is the file-scope array
 * below, whose address is looked up once per device. */
namespace {
constexpr size_t kNoAllocBytes = LFM_GPU_MOE_NOALLOC_SCRATCH_BYTES;
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void *g_noalloc_base[kNoAllocMaxDevices] = {nullptr};
}  // namespace

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

/* Carve the scratch of one layer call (T tokens) out of `b` (nullptr: only
 * size it).  Returns the bytes used; *counters_end = the leading bytes that
 * must be zero when the route kernel starts. */
static size_t noalloc_layout(uint32_t T, const MoeLayerDev &L, uint8_t *b, Workspace *w, size_t *counters_end) {
    const size_t E = L.E ? L.E : 1, K = lfm_layer_K(L) ? lfm_layer_K(L) : 1;
    const size_t TK = (size_t)T * K, D = L.D, I = L.I;
    const size_t n_pairs = E + (TK + LFM_GEMV_CHUNK - 1) / LFM_GEMV_CHUNK + 1;
    size_t off = 0;
    auto take = [&](size_t bytes) { const size_t o = off; off += align256(bytes); return o; };
    const size_t o_tc = take(sizeof(uint32_t) * T), o_done = take(sizeof(uint32_t));
    if (counters_end) *counters_end = off;
    const size_t o_xq = take((size_t)T * D), o_xd = take(sizeof(float) * T * (D / 256)),
                 o_xb = take(sizeof(int16_t) * T * (D / 256) * 16);
    const size_t o_idx = take(sizeof(int32_t) * TK), o_w = take(sizeof(float) * TK),
                 o_cnt = take(sizeof(int32_t) * E), o_off = take(sizeof(int32_t) * (E + 1)),
                 o_perm = take(sizeof(int32_t) * TK), o_inv = take(sizeof(int32_t) * TK),
                 o_act = take(sizeof(int32_t) * E), o_pairs = take(sizeof(int2) * n_pairs),
                 o_sum = take(sizeof(int32_t) * 4), o_log = take(sizeof(float) * T * E),
                 o_rms = take(sizeof(float) * T);
    const size_t o_h = take(sizeof(float) * TK * I), o_hq = take(TK * I), o_hd = take(sizeof(float) * TK * (I / 256)),
                 o_hb = take(sizeof(int16_t) * TK * (I / 256) * 16), o_y = take(sizeof(float) * TK * D);
    if (!b) return off;
    w->T = T; w->D = L.D; w->E = (uint32_t)E; w->K = (uint32_t)K; w->I = L.I;
    w->base = b; w->bytes = off; w->counters_bytes = o_xq;
    w->x = nullptr;
    w->xq = Q8Rows{reinterpret_cast<int8_t *>(b + o_xq), reinterpret_cast<float *>(b + o_xd),
                   reinterpret_cast<int16_t *>(b + o_xb), L.D};
    w->rt.idx = reinterpret_cast<int32_t *>(b + o_idx);
    w->rt.w = reinterpret_cast<float *>(b + o_w);
    w->rt.counts = reinterpret_cast<int32_t *>(b + o_cnt);
    w->rt.offsets = reinterpret_cast<int32_t *>(b + o_off);
    w->rt.perm = reinterpret_cast<int32_t *>(b + o_perm);
    w->rt.inv = reinterpret_cast<int32_t *>(b + o_inv);
    w->rt.act = reinterpret_cast<int32_t *>(b + o_act);
    w->rt.pairs = reinterpret_cast<int2 *>(b + o_pairs);
    w->rt.summary = reinterpret_cast<int32_t *>(b + o_sum);
    w->rt.tok_count = reinterpret_cast<uint32_t *>(b + o_tc);
    w->rt.done = reinterpret_cast<uint32_t *>(b + o_done);
    w->rt.logits = reinterpret_cast<float *>(b + o_log);
    w->rt.rms = reinterpret_cast<float *>(b + o_rms);
    w->h = reinterpret_cast<float *>(b + o_h);
    w->hq = Q8Rows{reinterpret_cast<int8_t *>(b + o_hq), reinterpret_cast<float *>(b + o_hd),
                   reinterpret_cast<int16_t *>(b + o_hb), L.I};
    w->y = reinterpret_cast<float *>(b + o_y);
    return off;
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_forward_noalloc(lfm_gpu_moe_t *h, uint32_t layer, float *x, uint32_t T,
                                                     void *stream) {
    if (!h || !x) return LFM_GPU_ERR_INVALID_ARG;
    if (T == 0) return LFM_GPU_OK;
    if (reinterpret_cast<uintptr_t>(x) & 15u)
        return fail(h, LFM_GPU_ERR_INVALID_ARG, "device x must be 16-byte aligned (bulk copies read it)");
    if (layer >= LFM_GPU_MOE_MAX_LAYERS || !h->layers[layer].present)
        return fail(h, LFM_GPU_ERR_NOT_READY, "layer %u not uploaded", layer);
    const MoeLayerDev &L = h->layers[layer].dev;
    /* a shard holds only its experts' slabs while the router spans all E: routing
     * it here would read expert weights past the end of the shard's allocation */
    const uint32_t ep_count = h->layers[layer].ep_count;
    if (ep_count && ep_count != L.E)
        return fail(h, LFM_GPU_ERR_UNSUPPORTED,
                    "forward_noalloc: layer %u holds an expert shard: use the lfm_gpu_moe_ep_* calls", layer);
    if (L.down_q6k)
        return fail(h, LFM_GPU_ERR_UNSUPPORTED, "forward_noalloc: layer %u has a Q6_K down tensor (Q4_K only)", layer);
    const size_t need = noalloc_layout(T, L, nullptr, nullptr, nullptr);
    if (T > 65535 || need > kNoAllocBytes)
        return fail(h, LFM_GPU_ERR_UNSUPPORTED,
                    "forward_noalloc: T=%u on layer %u needs %zu bytes of scratch, above its fixed %zu bytes",
                    T, layer, need, kNoAllocBytes);
    if (h->device >= kNoAllocMaxDevices)
        return fail(h, LFM_GPU_ERR_UNSUPPORTED, "forward_noalloc: device %d above %d", h->device, kNoAllocMaxDevices);
    DeviceGuard g(h->device);
    uint8_t *base = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        if (!g_noalloc_base[h->device]) {
            void *p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
            if (e != cudaSuccess || !p) return cuda_fail(h, e, "cudaGetSymbolAddress(noalloc scratch)");
            g_noalloc_base[h->device] = p;
        }
        base = static_cast<uint8_t *>(g_noalloc_base[h->device]);
    }
    Workspace w;
    size_t counters_end = 0;
    noalloc_layout(T, L, base, &w, &counters_end);
    w.rt.err = h->dev_err;
    w.rt.loads = nullptr; /* leaves the handle's statistics alone */
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int grid = h->sm_count;
    const uint32_t K = lfm_layer_K(L);
    /* the completion counters start every layer at zero (an earlier call that
     * was abandoned on a device error may have left them part-way) */
    cudaError_t e = cudaMemsetAsync(base, 0, counters_end, s);
    if (e == cudaSuccess) e = lfm_launch_route(L, x, T, w.xq, w.rt, s, false);
    if (e == cudaSuccess) e = lfm_launch_gateup(L, w.xq, w.rt, w.h, grid, s, true);
    if (e == cudaSuccess) e = lfm_launch_quant_rows(w.h, T * K, L.I, w.hq, s, true);
    if (e == cudaSuccess) e = lfm_launch_down(L, w.hq, w.rt, w.y, grid, s, true);
    if (e == cudaSuccess) e = lfm_launch_combine(L, x, T, w.rt, w.y, s, true);
    if (e != cudaSuccess) return cuda_fail(h, e, "forward_noalloc launch");
    return LFM_GPU_OK;
}

/* ---- expert parallelism ---------------------------------------------------
 * One process per GPU; each holds the full router and an expert shard.  The
 * caller exchanges rows between ranks (e.g. NCCL all-to-all): route locally,
 * send each (token, k) row to the rank owning its expert, run the local
 * experts on the rows received, send the outputs back, combine at home. */

static lfm_gpu_status_t ep_layer(lfm_gpu_moe_t *h, uint32_t layer, const LayerSlot **out) {
    if (!h) return LFM_GPU_ERR_INVALID_ARG;
    if (layer >= LFM_GPU_MOE_MAX_LAYERS || !h->layers[layer].present || h->layers[layer].dev.dense)
        return fail(h, LFM_GPU_ERR_NOT_READY, "layer %u is not an uploaded MoE layer", layer);
    *out = &h->layers[layer];
    return LFM_GPU_OK;
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_ep_route(lfm_gpu_moe_t *h, uint32_t layer, const float *x, uint32_t T,
                                              int32_t *idx_out, float *w_out, void *q8_out, void *stream) {
    const LayerSlot *S = nullptr;
    lfm_gpu_status_t st = ep_layer(h, layer, &S);
    if (st != LFM_GPU_OK) return st;
    if (!x || !idx_out || !w_out || !q8_out) return fail(h, LFM_GPU_ERR_INVALID_ARG, "null buffer");
    if (T == 0) return LFM_GPU_OK;
    if (T > 65535) return fail(h, LFM_GPU_ERR_INVALID_ARG, "T=%u above 65535", T);
    if (reinterpret_cast<uintptr_t>(x) & 15u) return fail(h, LFM_GPU_ERR_INVALID_ARG, "device x must be 16-byte aligned");
    const MoeLayerDev &L = S->dev;
    DeviceGuard g(h->device);
    st = ensure_workspace(h, T, L.D, L.E, L.K, L.I);
    if (st != LFM_GPU_OK) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    Workspace &w = h->ws;
    Q8Rows xq = w.xq; xq.cols = L.D;
    RouteTables rt = w.rt;
    rt.loads = nullptr; /* expert loads are counted where the experts run (lfm_gpu_moe_ep_experts) */
    h->stats = lfm_gpu_moe_stats_t{};
    h->stats.tokens = T;
    h->stats.kernels_launched = lfm_route_kernels(L, T) + 1;
    LFM_CUDA(h, lfm_launch_route(L, x, T, xq, rt, s, false));
    LFM_CUDA(h, cudaMemcpyAsync(idx_out, w.rt.idx, sizeof(int32_t) * T * L.K, cudaMemcpyDeviceToDevice, s));
    LFM_CUDA(h, cudaMemcpyAsync(w_out, w.rt.w, sizeof(float) * T * L.K, cudaMemcpyDeviceToDevice, s));
    LFM_CUDA(h, lfm_launch_q8_to_gguf(xq, T, static_cast<uint8_t *>(q8_out), s));
    return LFM_GPU_OK;
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_ep_experts(lfm_gpu_moe_t *h, uint32_t layer, const void *q8_in, uint32_t n_rows,
                                                const int32_t *expert_ids, float *y_out, void *stream) {
    const LayerSlot *S = nullptr;
    lfm_gpu_status_t st = ep_layer(h, layer, &S);
    if (st != LFM_GPU_OK) return st;
    if (n_rows == 0) return LFM_GPU_OK;
    if (!q8_in || !expert_ids || !y_out) return fail(h, LFM_GPU_ERR_INVALID_ARG, "null buffer");
    if (n_rows > 65535) return fail(h, LFM_GPU_ERR_INVALID_ARG, "n_rows=%u above 65535 per call", n_rows);
    const uint32_t first = S->ep_first, count = S->ep_count ? S->ep_count : S->dev.E;
    /* the shard as a layer of its own: local experts 0..count-1, top-1, weight 1 */
    MoeLayerDev Lx = S->dev;
    Lx.E = count;
    Lx.K = 1;
    Lx.router_w = nullptr;
    Lx.bias = nullptr;
    Lx.norm_topk = 0;
    Lx.routed_scale = 1.0f;
    DeviceGuard g(h->device);
    st = ensure_workspace(h, n_rows, Lx.D, count, 1, Lx.I);
    if (st != LFM_GPU_OK) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    Workspace &w = h->ws;
    Q8Rows xq = w.xq; xq.cols = Lx.D;
    h->stats = lfm_gpu_moe_stats_t{};
    h->stats.tokens = n_rows;
    h->stats.kernels_launched = 3; /* + those of run_experts */
    LFM_CUDA(h, lfm_launch_gguf_to_q8(static_cast<const uint8_t *>(q8_in), n_rows, xq, s));
    LFM_CUDA(h, lfm_launch_ep_prepare(expert_ids, n_rows, first, count, w.rt, s));
    RouteTables rt = w.rt;
    rt.plan = umma_plan_for(h, Lx, n_rows);
    LFM_CUDA(h, lfm_launch_dispatch(Lx, n_rows, rt, s));
    LFM_CUDA(h, cudaMemsetAsync(y_out, 0, sizeof(float) * n_rows * Lx.D, s));
    return run_experts(h, Lx, y_out, n_rows, xq, s, false, rt.plan); /* y_out = fma(1, y, 0) = y */
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_ep_combine(lfm_gpu_moe_t *h, uint32_t layer, float *x, uint32_t T,
                                                const float *w, const float *y, void *stream) {
    const LayerSlot *S = nullptr;
    lfm_gpu_status_t st = ep_layer(h, layer, &S);
    if (st != LFM_GPU_OK) return st;
    if (T == 0) return LFM_GPU_OK;
    if (!x || !w || !y) return fail(h, LFM_GPU_ERR_INVALID_ARG, "null buffer");
    DeviceGuard g(h->device);
    h->stats = lfm_gpu_moe_stats_t{};
    h->stats.tokens = T;
    h->stats.kernels_launched = 1;
    LFM_CUDA(h, lfm_launch_ep_combine(x, T, S->dev.D, S->dev.K, w, y, static_cast<cudaStream_t>(stream)));
    return LFM_GPU_OK;
}

/* ---- expert parallelism over peer memory ----------------------------------
 * Home and expert roles of every rank in one call per layer; the exchange
 * kernels live in k_ep.cu (publish, push, combine), k_route.cu (plan) and
 * k_umma.cu (gather). */

namespace {

void ep_layout(EpP2P &p) {
    size_t off = 0;
    auto take = [&](size_t bytes) { const size_t o = off; off += align256(bytes); return o; };
    const size_t T = p.T_max, TK = (size_t)p.T_max * p.K, nb = p.D / 256, R = p.max_recv();
    p.o_cnt = take(sizeof(uint32_t) * LFM_EP_MAX_RANKS);
    p.o_y = take(sizeof(uint32_t) * LFM_EP_MAX_RANKS);
    p.o_done = take(sizeof(uint32_t));
    p.o_tab = take(sizeof(int32_t) * 2 * LFM_EP_MAX_RANKS * p.E);
    p.o_qs = take(T * p.D);
    p.o_qd = take(sizeof(float) * T * nb);
    p.o_qb = take(sizeof(int16_t) * T * nb * 16);
    p.o_perm = take(sizeof(int32_t) * TK);
    p.o_yhome = take(sizeof(float) * TK * p.D);
    p.o_rowmap = take(sizeof(uint32_t) * R);
    p.o_ret = take(sizeof(uint32_t) * R);
    p.o_nrecv = take(sizeof(int32_t));
    p.o_step = take(sizeof(uint32_t));
    p.o_cdone = take(sizeof(uint32_t));
    p.bytes = off;
}

/* What an exchanged handle carries besides the IPC handle: the attach
 * arguments every rank must share (the arena layout follows from them). */
struct EpSignature {
    uint32_t magic, rank, world, T_max, D, E, K, I;
    uint64_t bytes;
};
constexpr uint32_t kEpSigMagic = 0x5045464Cu; /* "LFEP" */
constexpr size_t kEpSigOffset = 64;
static_assert(sizeof(cudaIpcMemHandle_t) <= kEpSigOffset, "IPC handle size");
static_assert(kEpSigOffset + sizeof(EpSignature) <= LFM_GPU_MOE_IPC_HANDLE_BYTES, "exchanged handle size");

EpSignature ep_signature(const EpP2P &p, uint32_t rank) {
    EpSignature g{};
    g.magic = kEpSigMagic;
    g.rank = rank;
    g.world = p.world;
    g.T_max = p.T_max;
    g.D = p.D; g.E = p.E; g.K = p.K; g.I = p.I;
    g.bytes = p.bytes;
    return g;
}

EpArena ep_arena_view(const EpP2P &p, uint8_t *b) {
    EpArena a{};
    a.cnt_flag = reinterpret_cast<uint32_t *>(b + p.o_cnt);
    a.y_flag = reinterpret_cast<uint32_t *>(b + p.o_y);
    a.done = reinterpret_cast<uint32_t *>(b + p.o_done);
    a.table = reinterpret_cast<int32_t *>(b + p.o_tab);
    a.xq = Q8Rows{reinterpret_cast<int8_t *>(b + p.o_qs), reinterpret_cast<float *>(b + p.o_qd),
                  reinterpret_cast<int16_t *>(b + p.o_qb), p.D};
    a.perm = reinterpret_cast<int32_t *>(b + p.o_perm);
    a.yhome = reinterpret_cast<float *>(b + p.o_yhome);
    a.rowmap = reinterpret_cast<uint32_t *>(b + p.o_rowmap);
    a.ret = reinterpret_cast<uint32_t *>(b + p.o_ret);
    a.n_recv = reinterpret_cast<int32_t *>(b + p.o_nrecv);
    a.step = reinterpret_cast<uint32_t *>(b + p.o_step);
    a.cdone = reinterpret_cast<uint32_t *>(b + p.o_cdone);
    return a;
}

void ep_release(lfm_gpu_moe_t *h) {
    EpP2P &p = h->ep;
    for (uint32_t r = 0; r < LFM_EP_MAX_RANKS; ++r) {
        if (p.opened[r] && p.peer[r]) cudaIpcCloseMemHandle(p.peer[r]);
        p.opened[r] = false;
        p.peer[r] = nullptr;
    }
    if (p.arena) cudaFree(p.arena);
    p = EpP2P{};
}

}  // namespace

LFM_API lfm_gpu_status_t lfm_gpu_moe_ep_p2p_attach(lfm_gpu_moe_t *h, int rank, int world, uint32_t max_tokens,
                                                   uint32_t D, uint32_t E, uint32_t K, uint32_t I, uint32_t wait_ms,
                                                   void *ipc_handle_out) {
    if (!h || !ipc_handle_out) return LFM_GPU_ERR_INVALID_ARG;
    if (h->ep.attached) return fail(h, LFM_GPU_ERR_INVALID_ARG, "ep_p2p_attach: already attached (detach first)");
    if (world < 1 || world > LFM_EP_MAX_RANKS || rank < 0 || rank >= world)
        return fail(h, LFM_GPU_ERR_INVALID_ARG, "ep_p2p_attach: rank %d of world %d (1..%d ranks)", rank, world,
                    LFM_EP_MAX_RANKS);
    lfm_gpu_status_t st = check_layer_shape(h, 0, D, E, K, I);
    if (st != LFM_GPU_OK) return st;
    if ((uint32_t)world > E) return fail(h, LFM_GPU_ERR_INVALID_ARG, "ep_p2p_attach: %d ranks for %u experts", world, E);
    if (max_tokens == 0 || max_tokens > 65535)
        return fail(h, LFM_GPU_ERR_INVALID_ARG, "ep_p2p_attach: max_tokens=%u not in 1..65535", max_tokens);
    if (!(lfm_umma_ok(I) && lfm_umma_ok(D)))
        return fail(h, LFM_GPU_ERR_UNSUPPORTED, "ep_p2p_attach: D=%u, I=%u need multiples of 128 rows", D, I);
    DeviceGuard g(h->device);
    EpP2P &p = h->ep;
    p = EpP2P{};
    p.rank = (uint32_t)rank;
    p.world = (uint32_t)world;
    p.T_max = max_tokens;
    p.D = D; p.E = E; p.K = K; p.I = I;
    p.wait_ns = (uint64_t)(wait_ms ? wait_ms : 5000u) * 1000000ull;
    ep_layout(p);
    /* scratch for both roles now, so no forward reallocates it mid-step:
     * routing max_tokens tokens at K, and the shard's experts on every row
     * the ranks can send (at K = 1) */
    st = ensure_workspace(h, max_tokens, D, E, K, I);
    if (st == LFM_GPU_OK) st = ensure_workspace(h, p.max_recv(), D, E, 1, I);
    if (st != LFM_GPU_OK) { p = EpP2P{}; return st; }
    void *base = nullptr;
    cudaError_t e = cudaMalloc(&base, p.bytes);
    if (e != cudaSuccess) { p = EpP2P{}; return cuda_fail(h, e, "ep_p2p_attach: arena cudaMalloc"); }
    p.arena = static_cast<uint8_t *>(base);
    e = cudaMemset(base, 0, p.bytes);
    cudaIpcMemHandle_t ipc{};
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&ipc, base);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) { ep_release(h); return cuda_fail(h, e, "ep_p2p_attach: arena setup"); }
    memset(ipc_handle_out, 0, LFM_GPU_MOE_IPC_HANDLE_BYTES);
    memcpy(ipc_handle_out, &ipc, sizeof ipc);
    const EpSignature sig = ep_signature(p, p.rank);
    memcpy(static_cast<uint8_t *>(ipc_handle_out) + kEpSigOffset, &sig, sizeof sig);
    p.peer[p.rank] = p.arena;
    p.attached = true;
    return LFM_GPU_OK;
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_ep_p2p_connect(lfm_gpu_moe_t *h, const void *handles) {
    if (!h || !handles) return LFM_GPU_ERR_INVALID_ARG;
    EpP2P &p = h->ep;
    if (!p.attached) return fail(h, LFM_GPU_ERR_NOT_READY, "ep_p2p_connect: attach first");
    if (p.connected) return LFM_GPU_OK;
    DeviceGuard g(h->device);
    const uint8_t *hb = static_cast<const uint8_t *>(handles);
    /* every rank must have attached with the same shapes: the arenas' layouts are computed, not exchanged */
    for (uint32_t r = 0; r < p.world; ++r) {
        EpSignature theirs;
        memcpy(&theirs, hb + (size_t)r * LFM_GPU_MOE_IPC_HANDLE_BYTES + kEpSigOffset, sizeof theirs);
        const EpSignature want = ep_signature(p, r);
        if (memcmp(&theirs, &want, sizeof want) != 0)
            return fail(h, LFM_GPU_ERR_INVALID_ARG,
                        "ep_p2p_connect: handle %u is not rank %u of this world with this rank's shapes "
                        "(it has rank %u of %u, max_tokens %u, D %u, E %u, K %u, I %u; this rank %u of %u, "
                        "max_tokens %u, D %u, E %u, K %u, I %u)",
                        r, r, theirs.rank, theirs.world, theirs.T_max, theirs.D, theirs.E, theirs.K, theirs.I, p.rank,
                        p.world, p.T_max, p.D, p.E, p.K, p.I);
    }
    for (uint32_t r = 0; r < p.world; ++r) {
        if (r == p.rank) continue;
        cudaIpcMemHandle_t ipc;
        memcpy(&ipc, hb + (size_t)r * LFM_GPU_MOE_IPC_HANDLE_BYTES, sizeof ipc);
        void *ptr = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&ptr, ipc, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (uint32_t q = 0; q < r; ++q)
                if (p.opened[q]) { cudaIpcCloseMemHandle(p.peer[q]); p.opened[q] = false; p.peer[q] = nullptr; }
            return fail(h, LFM_GPU_ERR_COMM, "ep_p2p_connect: opening rank %u's arena: %s", r, cudaGetErrorString(e));
        }
        p.peer[r] = static_cast<uint8_t *>(ptr);
        p.opened[r] = true;
    }
    p.connected = true;
    return LFM_GPU_OK;
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_ep_p2p_detach(lfm_gpu_moe_t *h) {
    if (!h) return LFM_GPU_ERR_INVALID_ARG;
    if (!h->ep.attached) return LFM_GPU_OK;
    DeviceGuard g(h->device);
    const cudaError_t e = cudaDeviceSynchronize();
    drop_graphs(h); /* captured steps hold the peer mappings */
    ep_release(h);
    if (e != cudaSuccess) return cuda_fail(h, e, "ep_p2p_detach: sync");
    return LFM_GPU_OK;
}

namespace {

/* The layer must be this rank's shard of an arena-shaped MoE layer. */
lfm_gpu_status_t ep_check_layer(lfm_gpu_moe_t *h, uint32_t layer, const LayerSlot &S) {
    const EpP2P &p = h->ep;
    const MoeLayerDev &L = S.dev;
    const uint32_t first = lfm_ep_first(p.rank, p.E, p.world), count = lfm_ep_first(p.rank + 1, p.E, p.world) - first;
    if (L.dense || L.D != p.D || L.E != p.E || L.K != p.K || L.I != p.I)
        return fail(h, LFM_GPU_ERR_INVALID_ARG, "ep_p2p: layer %u is not a %ux%ux%ux%u MoE layer", layer, p.D, p.E,
                    p.K, p.I);
    if (L.down_q6k)
        return fail(h, LFM_GPU_ERR_UNSUPPORTED, "ep_p2p: layer %u has a Q6_K down tensor (the peer-memory path is Q4_K only)",
                    layer);
    if (S.ep_first != first || (S.ep_count ? S.ep_count : L.E) != count)
        return fail(h, LFM_GPU_ERR_INVALID_ARG, "ep_p2p: layer %u holds experts [%u, %u), rank %u owns [%u, %u)", layer,
                    S.ep_first, S.ep_first + (S.ep_count ? S.ep_count : L.E), p.rank, first, first + count);
    return LFM_GPU_OK;
}

/* This step's arguments: this rank's arena and every rank's mapping of its own. */
EpStep ep_step_args(lfm_gpu_moe_t *h, uint32_t ahead) {
    const EpP2P &p = h->ep;
    EpStep es{};
    es.rank = p.rank; es.world = p.world; es.E = p.E; es.K = p.K; es.D = p.D;
    es.ahead = ahead;
    es.max_assign = p.T_max * p.K;
    es.max_recv = p.max_recv();
    es.wait_ns = p.wait_ns;
    es.err = h->dev_err;
    es.self = ep_arena_view(p, p.arena);
    for (uint32_t r = 0; r < p.world; ++r) {
        const EpArena a = ep_arena_view(p, p.peer[r]);
        es.table[r] = a.table;
        es.cnt_flag[r] = a.cnt_flag;
        es.y_flag[r] = a.y_flag;
        es.yhome[r] = a.yhome;
    }
    return es;
}

/* One expert-parallel layer step on stream s: launches only (no host
 * synchronisation, no host-side step state), so it can be captured. */
lfm_gpu_status_t ep_forward_layer(lfm_gpu_moe_t *h, const LayerSlot &S, float *x, uint32_t T, cudaStream_t s) {
    const EpP2P &p = h->ep;
    const MoeLayerDev &L = S.dev;
    const uint32_t first = lfm_ep_first(p.rank, p.E, p.world), count = lfm_ep_first(p.rank + 1, p.E, p.world) - first;
    Workspace &w = h->ws;
    const int grid = h->sm_count;
    const EpStep es = ep_step_args(h, 1);
    /* chained with programmatic dependent launch like the single-GPU layer: every kernel waits
     * (griddepcontrol.wait) before it touches what its predecessor writes */
    const bool pdl = !h->prof && h->use_pdl;

    /* home role: route this rank's tokens into the arena (Q8_K rows, slots); the dispatch publishes the counts */
    RouteTables rt = w.rt;
    rt.perm = es.self.perm;
    rt.loads = nullptr;
    rt.plan = UmmaPlanOut{};
    if (T) {
        EpPublish pub{};
        for (uint32_t r = 0; r < p.world; ++r) {
            pub.table[r] = es.table[r];
            pub.cnt_flag[r] = es.cnt_flag[r];
        }
        pub.step = es.self.step;
        pub.world = p.world;
        pub.rank = p.rank;
        pub.E = p.E;
        LFM_CUDA(h, timed(h, K_ROUTE, s, [&] { return lfm_launch_route(L, x, T, es.self.xq, rt, s, pdl, &pub); },
                          lfm_route_kernels(L, T)));
    } else {
        LFM_CUDA(h, cudaMemsetAsync(rt.counts, 0, sizeof(int32_t) * p.E, s));
        LFM_CUDA(h, timed(h, K_EP_PUBLISH, s, [&] { return lfm_launch_ep_publish(es, rt.counts, s); }));
    }

    /* expert role: the rows every rank routed to this shard, token blocks sized to the expected load */
    UmmaPlanOut plan{};
    plan.nt = lfm_umma_nt(T ? T * p.K : p.K, count); /* T*K rows expected per shard on average */
    plan.rows_gu = L.I;
    plan.rows_dn = L.D;
    plan.tiles_gu = w.utiles_gu;
    plan.tiles_dn = w.utiles_dn;
    plan.tbs = w.utbs;
    plan.counts = w.ucounts;
    const uint32_t R = es.max_recv;
    plan.max_tb = (uint32_t)lfm_umma_tb_max(R, count, plan.nt);
    plan.max_gu = 2 * (uint32_t)lfm_umma_tiles_max(L.I, R, count, plan.nt);
    plan.max_dn = (uint32_t)lfm_umma_tiles_max(L.D, R, count, plan.nt);
    if (plan.max_tb > w.umax_tb || plan.max_gu > w.umax_gu || plan.max_dn > w.umax_dn)
        return fail(h, LFM_GPU_ERR_INVALID_ARG, "ep_p2p: tile plan capacity (internal)");
    RouteTables rx = w.rt;
    rx.plan = plan;
    const uint32_t nt = plan.nt, mtb = plan.max_tb;
    EpGather eg{};
    eg.rowmap = es.self.rowmap;
    eg.ret = es.self.ret;
    eg.err = h->dev_err;
    eg.K = p.K;
    eg.world = p.world;
    eg.max_assign = es.max_assign;
    for (uint32_t r = 0; r < p.world; ++r) {
        const EpArena a = ep_arena_view(p, p.peer[r]);
        eg.perm[r] = a.perm;
        eg.qs[r] = a.xq.qs;
        eg.d[r] = a.xq.d;
        eg.bs[r] = a.xq.bs;
    }
    LFM_CUDA(h, timed(h, K_EP_PLAN, s, [&] { return lfm_launch_ep_plan(es, first, count, rx, s, pdl); }));
    LFM_CUDA(h, timed(h, K_XT, s, [&] {
        return lfm_launch_xt_gather_ep(eg, L.D, w.utbs, w.ucounts + 1, mtb, nt, w.xt, s, pdl);
    }));
    LFM_CUDA(h, timed(h, K_GEMM_GU, s, [&] {
        return lfm_launch_q4k_umma(L.gate, L.up, count, L.I, L.D, w.xt, nt, w.utiles_gu, w.utbs, w.ucounts, w.h, w.u,
                                   h->dev_err, grid, s, nullptr, pdl);
    }));
    LFM_CUDA(h, timed(h, K_SWIGLU, s, [&] {
        return lfm_launch_swiglu_xt(w.h, w.u, L.I, w.utbs, w.ucounts + 3, mtb, nt, w.xt, s, pdl);
    }));
    /* down: every output row stored at its home rank from the epilogue (peer stores over NVLink),
     * y_flag raised on every rank by the last CTA */
    UmmaEpOut eo{};
    eo.ret = es.self.ret;
    for (uint32_t r = 0; r < p.world; ++r) {
        eo.yhome[r] = es.yhome[r];
        eo.y_flag[r] = es.y_flag[r];
    }
    eo.done = es.self.done;
    eo.step = es.self.step;
    eo.world = p.world;
    eo.rank = p.rank;
    eo.max_assign = es.max_assign;
    LFM_CUDA(h, timed(h, K_GEMM_D, s, [&] {
        return lfm_launch_q4k_umma(L.down, L.down, count, L.D, L.I, w.xt, nt, w.utiles_dn, w.utbs, w.ucounts + 2, w.y,
                                   w.y, h->dev_err, grid, s, &eo, pdl);
    }));

    /* home role: combine the outputs the expert ranks stored here; the step is done */
    LFM_CUDA(h, timed(h, K_COMBINE, s, [&] { return lfm_launch_ep_combine_wait(es, x, T, rt.w, true, s, pdl); }));
    return LFM_GPU_OK;
}

}  // namespace

LFM_API lfm_gpu_status_t lfm_gpu_moe_ep_p2p_forward(lfm_gpu_moe_t *h, uint32_t layer, float *x, uint32_t T,
                                                    void *stream) {
    const LayerSlot *S = nullptr;
    lfm_gpu_status_t st = ep_layer(h, layer, &S);
    if (st != LFM_GPU_OK) return st;
    if (!h->ep.connected) return fail(h, LFM_GPU_ERR_NOT_READY, "ep_p2p_forward: attach and connect first");
    st = ep_check_layer(h, layer, *S);
    if (st != LFM_GPU_OK) return st;
    if (T > h->ep.T_max) return fail(h, LFM_GPU_ERR_INVALID_ARG, "ep_p2p_forward: T=%u above max_tokens %u", T, h->ep.T_max);
    if (T && (!x || (reinterpret_cast<uintptr_t>(x) & 15u)))
        return fail(h, LFM_GPU_ERR_INVALID_ARG, "ep_p2p_forward: device x must be 16-byte aligned");
    DeviceGuard g(h->device);
    h->stats = lfm_gpu_moe_stats_t{};
    h->stats.tokens = T;
    return ep_forward_layer(h, *S, x, T, static_cast<cudaStream_t>(stream));
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_ep_p2p_wait_check(lfm_gpu_moe_t *h, void *stream) {
    if (!h) return LFM_GPU_ERR_INVALID_ARG;
    if (!h->ep.connected) return fail(h, LFM_GPU_ERR_NOT_READY, "ep_p2p_wait_check: attach and connect first");
    DeviceGuard g(h->device);
    const EpStep es = ep_step_args(h, 2); /* no rank signals a step beyond the next one */
    h->stats = lfm_gpu_moe_stats_t{};
    h->stats.kernels_launched = 1;
    LFM_CUDA(h, lfm_launch_ep_combine_wait(es, nullptr, 0, nullptr, false, static_cast<cudaStream_t>(stream)));
    return LFM_GPU_OK;
}

LFM_API lfm_gpu_status_t lfm_gpu_moe_ep_p2p_forward_stack(lfm_gpu_moe_t *h, uint32_t first, uint32_t n, float *x,
                                                          uint32_t T, void *stream) {
    if (!h) return LFM_GPU_ERR_INVALID_ARG;
    if (!h->ep.connected) return fail(h, LFM_GPU_ERR_NOT_READY, "ep_p2p_forward_stack: attach and connect first");
    if (n == 0 || first >= LFM_GPU_MOE_MAX_LAYERS || n > LFM_GPU_MOE_MAX_LAYERS - first)
        return fail(h, LFM_GPU_ERR_INVALID_ARG, "layer range [%u, %u+%u) invalid", first, first, n);
    if (T > h->ep.T_max)
        return fail(h, LFM_GPU_ERR_INVALID_ARG, "ep_p2p_forward_stack: T=%u above max_tokens %u", T, h->ep.T_max);
    if (T && (!x || (reinterpret_cast<uintptr_t>(x) & 15u)))
        return fail(h, LFM_GPU_ERR_INVALID_ARG, "ep_p2p_forward_stack: device x must be 16-byte aligned");
    uint32_t dI = 0;
    for (uint32_t l = first; l < first + n; ++l) {
        const LayerSlot &S = h->layers[l];
        if (!S.present) return fail(h, LFM_GPU_ERR_NOT_READY, "layer %u not uploaded", l);
        if (S.dev.D != h->ep.D) return fail(h, LFM_GPU_ERR_INVALID_ARG, "layer %u: D=%u, the arena's %u", l, S.dev.D, h->ep.D);
        if (S.dev.dense) {
            dI = S.dev.I > dI ? S.dev.I : dI;
            continue;
        }
        lfm_gpu_status_t st = ep_check_layer(h, l, S);
        if (st != LFM_GPU_OK) return st;
    }
    DeviceGuard g(h->device);
    if (dI && T) { /* dense layers run whole on every rank */
        lfm_gpu_status_t st = ensure_workspace(h, T, h->ep.D, 1, 1, dI);
        if (st != LFM_GPU_OK) return st;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    h->stats = lfm_gpu_moe_stats_t{};
    h->stats.tokens = T;
    if (h->use_graphs && !h->prof) return run_graph(h, first, n, x, T, s, true);
    for (uint32_t l = first; l < first + n; ++l) {
        lfm_gpu_status_t st = stack_layer(h, l, x, T, s, true);
        if (st != LFM_GPU_OK) return st;
    }
    return LFM_GPU_OK;
}
