/*
 * lfm_gpu_moe.h -- C-ABI of the B200 (sm_100a) lfm2moe sparse-MoE FFN.
 *
 * Drop-in boundary for laii's CPU MoE FFN.  The reference call it replaces is
 *
 *   void lfm2_forward_moe_ffn_1x4(LFM2ThreadPool *pool, float *x, float *xb,
 *        float *hb, block_q8_K_t *xq_scratch, const LFM2Layer *layer,
 *        const LFM2MoELayerExt *moe, uint32_t D, float eps);
 *                                    (tools/lfm2_moe_checkpoint.c:312-320)
 *
 * which updates one token's hidden state in place:
 *   x += sum_k w_k * Down_{e_k}( SwiGLU( Gate_{e_k} xq, Up_{e_k} xq ) )
 * with xq = Q8_K(RMSNorm(x) * ffn_norm), (e_k, w_k) = sigmoid + exp_probs_b
 * biased top-K with normalised unbiased weights.  This library does the same
 * for T tokens at once, on device-resident weights, with no CPU fallback:
 * every entry point either runs on the GPU or returns an error status.
 *
 * Conventions (from the reference's public C API, include/lfm2.h:40-48, and
 * its Vulkan offload, src/lfm_gpu/lfm_gpu_engine.h:37-44):
 *  - status codes: 0 = OK, negative = error; lfm_gpu_moe_last_error() has text;
 *  - caller-owned host buffers; the handle owns all device memory;
 *  - weights are copied to HBM once at upload (not per call, unlike the Vulkan path);
 *  - one host thread per handle; calls on a handle are not re-entrant
 *    (as the reference thread pool, tools/lfm2_threadpool.c:303-324);
 *  - tensors use GGUF layout: 3-D expert tensors [E][rows][cols/256] of
 *    144-byte Q4_K blocks (tools/lfm2_moe_checkpoint.c:54-58, :110-127).
 *
 * All functions are plain C (no CUDA or torch types); `stream` arguments are a
 * cudaStream_t passed as void* (NULL = the CUDA default stream, as in CUDA).
 */
#ifndef LFM_GPU_MOE_H
#define LFM_GPU_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct lfm_gpu_moe lfm_gpu_moe_t;

/* Mirrors lfm2_status_t (include/lfm2.h:40-48) for the codes they share. */
typedef enum {
    LFM_GPU_OK = 0,
    LFM_GPU_ERR_INVALID_ARG = -1,   /* bad shape, pointer, layer index          */
    LFM_GPU_ERR_UNSUPPORTED = -2,   /* weight type / shape this build lacks      */
    LFM_GPU_ERR_NOT_READY = -3,     /* layer not uploaded                        */
    LFM_GPU_ERR_OOM = -4,           /* cudaMalloc failed (same code as LFM2_ERR_OOM) */
    LFM_GPU_ERR_CUDA = -7,          /* CUDA runtime error                        */
    LFM_GPU_ERR_COMM = -8,          /* expert-parallel exchange failed           */
    LFM_GPU_ERR_TIMEOUT = -9,       /* a bounded device wait ran out             */
    LFM_GPU_ERR_DEVICE_CHECK = -10  /* a device-side bounds check tripped        */
} lfm_gpu_status_t;

#define LFM_GPU_MOE_MAX_EXPERTS 256
#define LFM_GPU_MOE_MAX_TOP_K 8
#define LFM_GPU_MOE_MAX_LAYERS 64

/* Create a handle bound to CUDA device `device_id` (its own stream, no layers).
 * Replaces: nothing in the reference (its CPU path needs no device handle);
 * the Vulkan analogue is lfm_gpu_engine_init (src/lfm_gpu/lfm_gpu_engine.h:37). */
lfm_gpu_status_t lfm_gpu_moe_create(lfm_gpu_moe_t **out, int device_id);

/* Free all device memory of the handle.  Replaces lfm_gpu_engine_free
 * (src/lfm_gpu/lfm_gpu_engine.h:38). */
void lfm_gpu_moe_destroy(lfm_gpu_moe_t *h);

/* Text of the last error on this handle ("" if none). */
const char *lfm_gpu_moe_last_error(const lfm_gpu_moe_t *h);

/* Upload one lfm2moe layer (copied into HBM).  Replaces the binding of
 * lfm2_bind_moe_layer (tools/lfm2_moe_checkpoint.c:70-102) plus the mmap'd
 * tensor data it points at:
 *   ffn_norm    fp32 [D]               blk.l.ffn_norm.weight (NULL = all ones)
 *   router_w    fp32 [E][D]            blk.l.ffn_gate_inp.weight
 *   exp_probs_b fp32 [E] or NULL       blk.l.exp_probs_b(.bias)
 *   gate_exps   Q4_K [E][I][D/256]     blk.l.ffn_gate_exps.weight
 *   up_exps     Q4_K [E][I][D/256]     blk.l.ffn_up_exps.weight
 *   down_exps   Q4_K [E][D][I/256]     blk.l.ffn_down_exps.weight
 * w_type must be 12 (GGML_TYPE_Q4_K).  D and I multiples of 256, E <= 256,
 * K <= 8.  norm_topk_prob / routed_scale as LFM2MoELayerExt (reference
 * defaults true / 1.0f, tools/lfm2_moe_checkpoint.c:98-100). */
lfm_gpu_status_t lfm_gpu_moe_upload_layer(lfm_gpu_moe_t *h, uint32_t layer, uint32_t D, uint32_t E,
                                          uint32_t K, uint32_t I, float eps, const float *ffn_norm,
                                          const float *router_w, const float *exp_probs_b,
                                          const void *gate_exps, const void *up_exps,
                                          const void *down_exps, uint32_t w_type,
                                          int norm_topk_prob, float routed_scale);

/* As lfm_gpu_moe_upload_layer, with the down tensor's own GGUF type: Q4_K_M
 * checkpoints store some blk.l.ffn_down_exps as Q6_K (the reference's
 * lfm2_compute_4rows_avx2 picks its Q6_K x Q8_K kernel by the tensor type,
 * tools/lfm2_decode_1x4.c:618-630; Q6_K block, tools/lfm2_cpuid_quants.c:101-106):
 *   gate_up_type 12 (Q4_K); down_type 12 (Q4_K) or 14 (Q6_K: [E][D][I/256]
 *   210-byte blocks; I <= 3072).
 * A Q6_K-down layer runs the route, the Q4_K gate|up GEMV (or GEMM) and a
 * dedicated Q6_K down kernel; the fused decode kernel, the tcgen05 GEMMs, the
 * peer-memory expert-parallel path and lfm_gpu_moe_forward_noalloc take Q4_K
 * layers only (they refuse a Q6_K layer with LFM_GPU_ERR_UNSUPPORTED). */
lfm_gpu_status_t lfm_gpu_moe_upload_layer_typed(lfm_gpu_moe_t *h, uint32_t layer, uint32_t D, uint32_t E,
                                                uint32_t K, uint32_t I, float eps, const float *ffn_norm,
                                                const float *router_w, const float *exp_probs_b,
                                                const void *gate_exps, const void *up_exps,
                                                const void *down_exps, uint32_t gate_up_type,
                                                uint32_t down_type, int norm_topk_prob, float routed_scale);

/* Upload a dense SwiGLU FFN layer (the leading layers of an lfm2moe stack,
 * run by lfm2_forward_ffn_fused_1x4, tools/lfm2_decode_1x4.c:1070-1104):
 * gate/up Q4_K [I][D/256], down Q4_K [D][I/256]. */
lfm_gpu_status_t lfm_gpu_moe_upload_dense(lfm_gpu_moe_t *h, uint32_t layer, uint32_t D, uint32_t I,
                                          float eps, const float *ffn_norm, const void *gate,
                                          const void *up, const void *down, uint32_t w_type);

/* Fill layer `layer` on the device from the seeded synthetic generator
 * (byte-identical to the host generator; no host copy of the weights).
 * Experts N(0, w_std) -> Q4_K, router N(0, router_std), exp_probs_b either
 * the given host array [E] or N(0, bias_std).  Seeds: see laii_b200/synth.py.
 * No counterpart in the reference (benchmark input generation). */
lfm_gpu_status_t lfm_gpu_moe_synth_layer(lfm_gpu_moe_t *h, uint32_t layer, uint32_t D, uint32_t E,
                                         uint32_t K, uint32_t I, float eps, const uint64_t seeds[5],
                                         float w_std, float router_std, float bias_std,
                                         const float *exp_probs_b);

/* Expert parallelism (one process per GPU, experts sharded across ranks): a
 * layer holding the full router (exp_probs_b, ffn_norm) but only experts
 * [expert_first, expert_first + n_local) of E.  gate/up/down_local are those
 * experts' slices of the GGUF tensors ([n_local][rows][cols/256] Q4_K), i.e.
 * lfm2_slice_expert_tensor_2d of each (tools/lfm2_moe_checkpoint.c:110-127).
 * A shard layer runs only through the lfm_gpu_moe_ep_* calls below. */
lfm_gpu_status_t lfm_gpu_moe_upload_layer_shard(lfm_gpu_moe_t *h, uint32_t layer, uint32_t D, uint32_t E,
                                                uint32_t K, uint32_t I, float eps, const float *ffn_norm,
                                                const float *router_w, const float *exp_probs_b,
                                                const void *gate_local, const void *up_local,
                                                const void *down_local, uint32_t w_type, int norm_topk_prob,
                                                float routed_scale, uint32_t expert_first, uint32_t n_local);

/* The seeded synthetic layer restricted to an expert shard: byte-identical to
 * the same experts of lfm_gpu_moe_synth_layer.  No counterpart in the reference. */
lfm_gpu_status_t lfm_gpu_moe_synth_layer_shard(lfm_gpu_moe_t *h, uint32_t layer, uint32_t D, uint32_t E,
                                               uint32_t K, uint32_t I, float eps, const uint64_t seeds[5],
                                               float w_std, float router_std, float bias_std,
                                               const float *exp_probs_b, uint32_t expert_first,
                                               uint32_t n_local);

/* EP step 1 (home rank): RMSNorm + Q8_K + router + top-K of device x[T][D]
 * (lfm2_rmsnorm_quantize_q8_K_simd + lfm2_moe_route_sigmoid_topk,
 * tools/lfm2_moe_checkpoint.c:328-333).  Device outputs: idx[T][K] global
 * expert ids, w[T][K] combine weights, q8[T][D/256] 292-byte block_q8_K.
 * Asynchronous on `stream`. */
lfm_gpu_status_t lfm_gpu_moe_ep_route(lfm_gpu_moe_t *h, uint32_t layer, const float *x, uint32_t T,
                                      int32_t *idx_out, float *w_out, void *q8_out, void *stream);

/* EP step 2 (expert rank): rows received from any rank -- row a is one
 * (token, k) assignment as q8_in[a][D/256] block_q8_K routed to global expert
 * expert_ids[a], which must lie in this rank's shard -- through gate/up,
 * SwiGLU, Q8_K(h) and down (tools/lfm2_moe_checkpoint.c:338-363 without the
 * weighting): y_out[a][D] fp32, unweighted.  n_rows <= 65535 per call.
 * Asynchronous on `stream`; a foreign expert id sets LFM_GPU_ERR_DEVICE_CHECK
 * at the next lfm_gpu_moe_sync. */
lfm_gpu_status_t lfm_gpu_moe_ep_experts(lfm_gpu_moe_t *h, uint32_t layer, const void *q8_in, uint32_t n_rows,
                                        const int32_t *expert_ids, float *y_out, void *stream);

/* EP step 3 (home rank): x[t] = fma(w[t][k], y[t*K + k], x[t]) for k = 0..K-1
 * in order (tools/lfm2_moe_checkpoint.c:266-269), y[T*K][D] in (t, k) order.
 * Asynchronous on `stream`. */
lfm_gpu_status_t lfm_gpu_moe_ep_combine(lfm_gpu_moe_t *h, uint32_t layer, float *x, uint32_t T, const float *w,
                                        const float *y, void *stream);

/* ---- expert parallelism over peer memory (NVLink / NVSwitch) -------------
 * The same layer step as ep_route -> exchange -> ep_experts -> exchange ->
 * ep_combine, with the two exchanges done by the library's own kernels
 * through CUDA IPC mappings of every rank's exchange arena: no host
 * synchronisation, no collective library call.  Per layer:
 *   home rank: route, publish its per-expert counts to every rank;
 *   expert rank: wait for every rank's counts (bounded), plan, gather the
 *     Q8_K rows of its experts from the home ranks' memory, gate/up, SwiGLU,
 *     down, store each output row into its home rank's arena, signal;
 *   home rank: wait for every expert rank's signal (bounded), combine in the
 *     reference's k order (tools/lfm2_moe_checkpoint.c:266-269).
 * Every rank calls lfm_gpu_moe_ep_p2p_forward for the same layers in the same
 * order (T may differ per rank, 0 included).  A wait that runs out sets
 * LFM_GPU_ERR_TIMEOUT at the next lfm_gpu_moe_sync; the ranks are then out of
 * step and must detach and attach again.  The layer must be the rank's shard:
 * experts [first, first + n) with (first, n) as in the host-side shard_of
 * (the first E % world ranks hold one expert more). */
#define LFM_GPU_MOE_EP_MAX_RANKS 8
#define LFM_GPU_MOE_IPC_HANDLE_BYTES 128

/* Step 1 (every rank): allocate this rank's exchange arena for up to
 * max_tokens tokens per rank and layers of shape D, E, K, I, and return its
 * IPC handle (LFM_GPU_MOE_IPC_HANDLE_BYTES opaque bytes) for the other ranks.
 * wait_ms bounds every device wait on another rank (0: 5000 ms).
 * No counterpart in the reference (its MoE runs on one host). */
lfm_gpu_status_t lfm_gpu_moe_ep_p2p_attach(lfm_gpu_moe_t *h, int rank, int world, uint32_t max_tokens, uint32_t D,
                                           uint32_t E, uint32_t K, uint32_t I, uint32_t wait_ms,
                                           void *ipc_handle_out);

/* Step 2 (every rank, after every rank's attach returned): map the other
 * ranks' arenas; handles[r] is rank r's handle from step 1, in rank order.
 * Every rank must have attached with the same world, max_tokens, D, E, K and
 * I (each handle carries them): otherwise LFM_GPU_ERR_INVALID_ARG and nothing
 * is mapped. */
lfm_gpu_status_t lfm_gpu_moe_ep_p2p_connect(lfm_gpu_moe_t *h, const void *handles);

/* x[T][D] += MoE(x) for this rank's tokens (device x), experts spread over
 * the ranks.  Asynchronous on `stream`. */
lfm_gpu_status_t lfm_gpu_moe_ep_p2p_forward(lfm_gpu_moe_t *h, uint32_t layer, float *x, uint32_t T, void *stream);

/* Layers [first, first + n) in order on the same device x[T][D]: MoE layers as
 * the step above, dense layers whole on this rank.  The launches of a (first,
 * n, T, x) are captured into a CUDA graph on first use and replayed after
 * (the step epoch lives in device memory, so a replay needs no new
 * arguments).  Asynchronous on `stream`. */
lfm_gpu_status_t lfm_gpu_moe_ep_p2p_forward_stack(lfm_gpu_moe_t *h, uint32_t first, uint32_t n, float *x,
                                                  uint32_t T, void *stream);

/* A check of the bounded-wait path: one device wait for a step that no rank
 * will ever signal, bounded by attach's wait_ms.  The next lfm_gpu_moe_sync
 * returns LFM_GPU_ERR_TIMEOUT and the handle stays usable (the step counter
 * does not move).  Asynchronous on `stream`.  No counterpart in the reference. */
lfm_gpu_status_t lfm_gpu_moe_ep_p2p_wait_check(lfm_gpu_moe_t *h, void *stream);

/* Unmap the peers and free the arena (after a device sync; every rank detaches
 * before any rank frees the memory another still reads: the caller puts a
 * barrier between the last forward and detach). */
lfm_gpu_status_t lfm_gpu_moe_ep_p2p_detach(lfm_gpu_moe_t *h);

/* ---- GGUF checkpoints -------------------------------------------------------
 * The FFN tensors of an lfm2moe GGUF v2/v3 file, bound as the reference binds
 * them (lfm2_bind_moe_layer, tools/lfm2_moe_checkpoint.c:70-102, on the
 * tensors and keys its loader reads, tools/lfm2_loader.c:359-366, :537-602):
 * block l is an lfm2moe layer when blk.l.ffn_gate_exps.weight exists (Q4_K
 * experts, ffn_down_exps Q4_K or Q6_K, F32 ffn_gate_inp router, optional exp_probs_b(.bias), top-K from
 * the ".expert_used_count" key, default 4), else a dense SwiGLU layer from
 * blk.l.ffn_{gate,up,down}.weight; both take blk.l.ffn_norm.weight and the
 * ".attention.layer_norm_rms_epsilon" key (default 1e-5). */
typedef struct {
    uint32_t kind;     /* 0: no FFN tensors, 1: dense SwiGLU, 2: lfm2moe */
    uint32_t D, E, K, I;
    float eps;
    int has_bias, has_norm;
    uint32_t down_type; /* GGUF type of the down tensor: 12 (Q4_K) or, lfm2moe only, 14 (Q6_K); 0: no FFN */
} lfm_gpu_moe_gguf_block_t;

/* Describe block `block` of the file (host only, no GPU needed); *n_blocks =
 * the ".block_count" key or one past the highest blk.N in the file. */
lfm_gpu_status_t lfm_gpu_moe_gguf_describe(const char *path, uint32_t block, lfm_gpu_moe_gguf_block_t *out,
                                           uint32_t *n_blocks);
/* Text of the calling thread's last GGUF error. */
const char *lfm_gpu_moe_gguf_last_error(void);

/* Upload blocks [first_block, first_block + n_blocks) (n_blocks 0: to the
 * end) into layer slots 0, 1, ...: lfm2moe blocks whole (n_local == 0) or as
 * the expert shard [expert_first, expert_first + n_local), dense blocks whole.
 * The file is mapped, not read into host memory first. *n_uploaded counts the
 * layers uploaded. */
lfm_gpu_status_t lfm_gpu_moe_upload_gguf(lfm_gpu_moe_t *h, const char *path, uint32_t first_block,
                                         uint32_t n_blocks, uint32_t expert_first, uint32_t n_local,
                                         uint32_t *n_uploaded);

/* Reserve scratch for up to max_tokens tokens per forward (forward grows it on
 * demand; reserve first when the forward is to be captured in a CUDA graph). */
lfm_gpu_status_t lfm_gpu_moe_reserve(lfm_gpu_moe_t *h, uint32_t max_tokens);

/* x[T][D] += MoE(x) for layer `layer` (or x += DenseFFN(x) for a dense layer),
 * the batched counterpart of lfm2_forward_moe_ffn_1x4 (tools/lfm2_moe_checkpoint.c:312).
 * x_on_device = 0: x is host memory; the call copies in, runs and copies back
 * before returning.  x_on_device = 1: x is device memory; the call is
 * asynchronous on `stream`. */
lfm_gpu_status_t lfm_gpu_moe_forward(lfm_gpu_moe_t *h, uint32_t layer, float *x, uint32_t T,
                                     int x_on_device, void *stream);

/* Layers [first, first + n) in order on the same x (an FFN-only stack). */
lfm_gpu_status_t lfm_gpu_moe_forward_stack(lfm_gpu_moe_t *h, uint32_t first, uint32_t n, float *x,
                                           uint32_t T, int x_on_device, void *stream);

/* Size of the fixed scratch that lfm_gpu_moe_forward_noalloc uses (per device). */
#define LFM_GPU_MOE_NOALLOC_SCRATCH_BYTES (4u << 20)

/* lfm_gpu_moe_forward for device-resident x on `stream` (NULL = the CUDA
 * default stream) that allocates nothing: no cudaMalloc/cudaFree, no growth of
 * the handle's scratch.  It exists for callers that must not allocate while a
 * step runs (an engine that plans all device memory at load time, or code that
 * cannot afford the device-wide synchronisation an allocation may cause).  Its
 * scratch is one fixed array of LFM_GPU_MOE_NOALLOC_SCRATCH_BYTES per device in
 * the library's static device memory; a (T, layer shape) whose scratch does not
 * fit is rejected with LFM_GPU_ERR_UNSUPPORTED before anything is launched
 * (the decode shape D=2048, E=32, K=4, I=1792 fits up to T=58 tokens).
 * The first call on a device looks the array up (cudaGetSymbolAddress) and
 * keeps its address for the life of the process; make that first call before
 * any stream capture, and do not call it again on a device whose primary
 * context was reset (cudaDeviceReset) in between.  Calls that can overlap on
 * one device -- on different streams, threads or handles -- race on the shared
 * scratch: serialise them.  A layer that holds an expert shard (uploaded with
 * the _shard calls) or a Q6_K down tensor is refused with
 * LFM_GPU_ERR_UNSUPPORTED.  Asynchronous; device-side errors are reported by
 * the next lfm_gpu_moe_sync.  Does not touch the handle's statistics or
 * profiling records.  No counterpart in the reference. */
lfm_gpu_status_t lfm_gpu_moe_forward_noalloc(lfm_gpu_moe_t *h, uint32_t layer, float *x, uint32_t T,
                                             void *stream);

/* Routing only, for parity checks: RMSNorm + Q8_K + router + top-K of host
 * x[T][D] -> expert ids [T][K], weights [T][K] and, if q8_out != NULL, the
 * Q8_K blocks of the normalised input [T][D/256] (292-byte GGUF layout).
 * Counterpart of lfm2_rmsnorm_quantize_q8_K_simd + lfm2_moe_route_sigmoid_topk
 * (tools/lfm2_moe_checkpoint.c:328-333).  Synchronous. */
lfm_gpu_status_t lfm_gpu_moe_debug_route(lfm_gpu_moe_t *h, uint32_t layer, const float *x, uint32_t T,
                                         uint32_t *idx_out, float *w_out, void *q8_out);

/* Integer partial sums of the Q4_K x Q8_K kernel used by the expert GEMVs, for
 * parity: host Q4_K rows w[n_rows][n_cols/256] (n_rows a multiple of 8, the
 * kernel's row group) against host Q8_K vectors
 * xq[n_vec][n_cols/256]; outputs (host) per (vec, row, super-block):
 * sub_dots[..][8] = sum over each 32-weight sub-block of q4*q8,
 * acc = sum_j sc_j*sub_dot_j, mins = sum_j m_j*(bsum pair j), and the fp32 row
 * results rows_out[n_vec][n_rows].  Counterpart of the Q4_K x Q8_K row kernels
 * (tools/lfm2_cpuid_quants.c:421-457, :1189-1257).  Synchronous. */
lfm_gpu_status_t lfm_gpu_moe_debug_q4k_rows(lfm_gpu_moe_t *h, const void *w, uint32_t n_rows,
                                            uint32_t n_cols, const void *xq, uint32_t n_vec,
                                            int32_t *sub_dots, int32_t *acc, int32_t *mins,
                                            float *rows_out);

/* Copy tensor `which` of an uploaded layer back to host memory, for checking
 * uploads and the device generator: 0 ffn_norm, 1 router_w, 2 exp_probs_b,
 * 3 gate, 4 up, 5 down; the first `bytes` bytes (at most the tensor's size;
 * exp_probs_b is stored padded to a multiple of 4 floats).  Synchronous.
 * No counterpart in the reference. */
lfm_gpu_status_t lfm_gpu_moe_debug_read_layer(lfm_gpu_moe_t *h, uint32_t layer, uint32_t which, void *out,
                                              size_t bytes);

/* As lfm_gpu_moe_debug_read_layer, bytes [offset, offset + bytes) of the tensor
 * (one expert's slab of a 3-D expert tensor, for a parity check that needs only
 * the experts its tokens were routed to).  Synchronous.  No counterpart in the
 * reference. */
lfm_gpu_status_t lfm_gpu_moe_debug_read_layer_range(lfm_gpu_moe_t *h, uint32_t layer, uint32_t which,
                                                    size_t offset, void *out, size_t bytes);

/* Wait for all work on the handle's stream and report any device-side error
 * (bounds check or timeout) raised since the last call. */
lfm_gpu_status_t lfm_gpu_moe_sync(lfm_gpu_moe_t *h);

/* Launch statistics of the last forward: kernels launched and the routing
 * summary (unique experts touched, largest expert segment). */
typedef struct {
    uint32_t kernels_launched;    /* kernels of the last forward call                 */
    uint32_t tokens;              /* T of the last forward call                       */
    uint32_t unique_experts;      /* experts touched by the last MoE layer run        */
    uint32_t max_segment;         /* largest per-expert token count of that layer     */
    uint64_t expert_loads;        /* sum of unique experts over all MoE layer runs
                                     since the handle was created (each is one pass
                                     over that expert's gate/up/down bytes)           */
    uint64_t layer_runs;          /* MoE layer runs counted in expert_loads           */
} lfm_gpu_moe_stats_t;

/* Synchronous (waits for the handle's stream).  The analogue of the reference's
 * lfm2_perf_stats_t (include/lfm2.h:99-107) for this path. */
lfm_gpu_status_t lfm_gpu_moe_last_stats(const lfm_gpu_moe_t *h, lfm_gpu_moe_stats_t *out);

/* Per-kernel device time: with profiling on, every kernel a forward launches
 * is bracketed by CUDA events on the launch stream; profile_read waits for the
 * stream, adds up the elapsed times per kernel name and clears the records.
 * No counterpart in the reference (its bench main uses wall clock,
 * tools/lfm2_moe_checkpoint.c:706-723). */
typedef struct {
    char name[32];
    uint32_t launches;
    double total_ms;
} lfm_gpu_moe_kernel_time_t;

lfm_gpu_status_t lfm_gpu_moe_profile(lfm_gpu_moe_t *h, int enable);
lfm_gpu_status_t lfm_gpu_moe_profile_read(lfm_gpu_moe_t *h, lfm_gpu_moe_kernel_time_t *out, uint32_t cap,
                                          uint32_t *n_out);

#ifdef __cplusplus
}
#endif

#endif /* LFM_GPU_MOE_H */
