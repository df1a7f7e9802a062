/*
 * TEST INFRASTRUCTURE ONLY -- the C shim of INTEGRATION.md, compiled as laii
 * would compile it: after the reference's own tools/lfm2_moe_checkpoint.c and
 * tools/lfm2_prefill_batch.c (included by path, nothing copied), linked with
 * liblfm_gpu_moe.so.  oracle/Makefile builds oracle/_ref/libshim_check.so from
 * this file and the shim block oracle/extract_shim.py lifts out of
 * INTEGRATION.md.  The exported calls build the reference's GGUFTensor /
 * LFM2Layer / LFM2MoELayerExt / LFM2BatchState around caller buffers and go
 * through the shim's entry points only:
 *   shim_bind          lfm2_gpu_moe_bind (an lfm2moe or dense layer)
 *   shim_forward_1x4   lfm2_forward_moe_ffn_gpu, one call per token (the
 *                      drop-in for lfm2_forward_moe_ffn_1x4)
 *   shim_forward_batch lfm2_forward_moe_ffn_batch_gpu on an LFM2BatchState
 *                      (lfm2_forward_ffn_batch's slot)
 */
#define _GNU_SOURCE 1
#define LFM2_LOADER_NO_MAIN 1
#define LFM2_THREADPOOL_NO_MAIN 1
#define LFM2_FORWARD_NO_MAIN 1
#define LFM2_DECODE_1X4_NO_MAIN 1
#define LFM2_KERNELS_FAST_NO_MAIN 1
#define LFM2_MOE_CHECKPOINT_NO_MAIN 1
#define LFM2_CPUID_QUANTS_NO_MAIN 1
#define LFM2_PREFILL_BATCH_NO_MAIN 1

#include "tools/lfm2_moe_checkpoint.c"
#include "tools/lfm2_prefill_batch.c"

#include "lfm_gpu_moe_shim.c" /* written by oracle/extract_shim.py from INTEGRATION.md */

#define SHIM_EXPORT __attribute__((visibility("default")))

/* Descriptors of each bound layer: the shim finds a layer by its LFM2Layer address. */
static struct {
    GGUFTensor norm, router, bias, gate, up, down;
    LFM2Layer layer;
    LFM2MoELayerExt moe;
} g_slot[LFM_GPU_MOE_MAX_LAYERS];

static GGUFTensor shim_tensor(uint32_t type, uint32_t n_dims, uint64_t ne0, uint64_t ne1, uint64_t ne2,
                              const void *data) {
    GGUFTensor t;
    memset(&t, 0, sizeof t);
    t.n_dims = n_dims;
    t.ne[0] = ne0; t.ne[1] = ne1; t.ne[2] = ne2; t.ne[3] = 1;
    t.type = type;
    t.data = data;
    return t;
}

/* E == 0: a dense SwiGLU layer (gate/up [I][D/256], down [D][I/256] Q4_K).
 * Otherwise an lfm2moe layer; down_type 12 (Q4_K) or 14 (Q6_K).  Returns 1 on success. */
SHIM_EXPORT int shim_bind(uint32_t l, uint32_t D, uint32_t E, uint32_t K, uint32_t I, float eps,
                          const float *ffn_norm, const float *router_w, const float *bias, const void *gate,
                          const void *up, const void *down, uint32_t down_type) {
    if (l >= LFM_GPU_MOE_MAX_LAYERS) return 0;
    memset(&g_slot[l], 0, sizeof g_slot[l]);
    g_slot[l].norm = shim_tensor(GGML_TYPE_F32, 1, D, 1, 1, ffn_norm);
    g_slot[l].layer.ffn_norm = ffn_norm ? &g_slot[l].norm : NULL;
    if (E == 0) {
        g_slot[l].gate = shim_tensor(GGML_TYPE_Q4_K, 2, D, I, 1, gate);
        g_slot[l].up = shim_tensor(GGML_TYPE_Q4_K, 2, D, I, 1, up);
        g_slot[l].down = shim_tensor(GGML_TYPE_Q4_K, 2, I, D, 1, down);
        g_slot[l].layer.ffn_gate = &g_slot[l].gate;
        g_slot[l].layer.ffn_up = &g_slot[l].up;
        g_slot[l].layer.ffn_down = &g_slot[l].down;
        g_slot[l].moe.is_moe_layer = false;
    } else {
        g_slot[l].router = shim_tensor(GGML_TYPE_F32, 2, D, E, 1, router_w);
        g_slot[l].bias = shim_tensor(GGML_TYPE_F32, 1, E, 1, 1, bias);
        g_slot[l].gate = shim_tensor(GGML_TYPE_Q4_K, 3, D, I, E, gate);
        g_slot[l].up = shim_tensor(GGML_TYPE_Q4_K, 3, D, I, E, up);
        g_slot[l].down = shim_tensor(down_type, 3, I, D, E, down);
        LFM2MoELayerExt *m = &g_slot[l].moe;
        m->is_moe_layer = true;
        m->n_experts = E;
        m->n_experts_used = K;
        m->norm_topk_prob = true;
        m->routed_scale = 1.0f;
        m->ffn_gate_inp = &g_slot[l].router;
        m->ffn_exp_probs_b = bias ? &g_slot[l].bias : NULL;
        m->ffn_gate_exps = &g_slot[l].gate;
        m->ffn_up_exps = &g_slot[l].up;
        m->ffn_down_exps = &g_slot[l].down;
    }
    return lfm2_gpu_moe_bind(l, &g_slot[l].layer, &g_slot[l].moe, D, eps);
}

/* x[T][D]: one drop-in call per token, as laii's decode loop makes them. */
SHIM_EXPORT void shim_forward_1x4(uint32_t l, float *x, uint32_t T, uint32_t D, float eps) {
    if (l >= LFM_GPU_MOE_MAX_LAYERS) return;
    for (uint32_t t = 0; t < T; ++t)
        lfm2_forward_moe_ffn_gpu(NULL, x + (size_t)t * D, NULL, NULL, NULL, &g_slot[l].layer, &g_slot[l].moe, D, eps);
}

/* x[B][D] as the batch state's residual stream, through the batched slot.  Returns 1 on success. */
SHIM_EXPORT int shim_forward_batch(uint32_t l, float *x, uint32_t B) {
    if (l >= LFM_GPU_MOE_MAX_LAYERS || B > LFM2_MAX_BATCH) return 0;
    LFM2BatchState s;
    memset(&s, 0, sizeof s);
    s.x = x;
    return lfm2_forward_moe_ffn_batch_gpu(&s, &g_slot[l].layer, B);
}

SHIM_EXPORT int shim_max_batch(void) { return LFM2_MAX_BATCH; }

SHIM_EXPORT void shim_release(void) { lfm2_gpu_moe_release(); }
