/*
 * TEST INFRASTRUCTURE ONLY -- C-ABI wrapper around the reference's own CPU
 * lfm2moe path, compiled from the reference sources where they lie (include by
 * path, nothing copied) into oracle/_ref/libref_moe.so by oracle/Makefile.
 *
 * It builds the reference's GGUFTensor / LFM2Layer / LFM2MoELayerExt
 * descriptors around caller buffers (the same way tests/test_moe_checkpoint.c
 * in the reference does) and calls, unmodified:
 *   lfm2_forward_moe_ffn_1x4          tools/lfm2_moe_checkpoint.c:312
 *   lfm2_moe_route_sigmoid_topk       tools/lfm2_moe_checkpoint.c:166
 *   lfm2_rmsnorm_quantize_q8_K_simd   tools/lfm2_decode_1x4.c:562
 *   lfm2_forward_ffn_fused_1x4        tools/lfm2_decode_1x4.c:1070
 *   lfm2_compute_4rows_avx2           tools/lfm2_decode_1x4.c:597
 *   kernel table quantize_q8_K        tools/lfm2_cpuid_quants.c:1797
 * with the reference's own thread pool (tools/lfm2_threadpool.c:382).
 * Used to pin the oracle restatement, to make golden fixtures, and as the
 * timed CPU baseline ("reference" arm of bench.py).
 */
#define _GNU_SOURCE 1
#define LFM2_LOADER_NO_MAIN 1
#define LFM2_THREADPOOL_NO_MAIN 1
#define LFM2_FORWARD_NO_MAIN 1
#define LFM2_DECODE_1X4_NO_MAIN 1
#define LFM2_KERNELS_FAST_NO_MAIN 1
#define LFM2_MOE_CHECKPOINT_NO_MAIN 1
#define LFM2_CPUID_QUANTS_NO_MAIN 1

#include <sched.h>
#include <xmmintrin.h>

#include "tools/lfm2_moe_checkpoint.c"

#define REF_EXPORT __attribute__((visibility("default")))

static LFM2ThreadPool g_pool;
static int g_pool_ready = 0;

/* The reference runs with FTZ/DAZ set on every thread; keep that for the
 * duration of each call and give the caller's MXCSR back afterwards. */
#define REF_FPENV_ENTER() const unsigned int ref_saved_csr = _mm_getcsr(); lfm2_set_denormals_zero_mode()
#define REF_FPENV_LEAVE() _mm_setcsr(ref_saved_csr)

/* Start (or restart) the reference thread pool; 0 = the reference's default
 * (N_phys - 1, or LFM_NUM_THREADS).  The pool pins the calling thread; the
 * caller's affinity mask is restored afterwards.  Returns the worker count. */
REF_EXPORT int ref_init(int n_threads) {
    cpu_set_t saved;
    const int have_mask = sched_getaffinity(0, sizeof saved, &saved) == 0;
    const unsigned int csr = _mm_getcsr();
    if (g_pool_ready) lfm2_threadpool_free(&g_pool);
    lfm2_threadpool_init(&g_pool, (uint32_t)(n_threads < 0 ? 0 : n_threads));
    g_pool_ready = 1;
    _mm_setcsr(csr);
    if (have_mask) sched_setaffinity(0, sizeof saved, &saved);
    return (int)g_pool.n_threads;
}

REF_EXPORT void ref_shutdown(void) {
    if (g_pool_ready) lfm2_threadpool_free(&g_pool);
    g_pool_ready = 0;
}

REF_EXPORT const char *ref_isa_name(void) { return lfm2_get_cpu_kernel_table()->isa_name; }

REF_EXPORT const char *ref_cpu_brand(void) { return lfm2_get_cpu_kernel_table()->cpu_brand; }

static GGUFTensor ref_tensor(uint32_t type, uint32_t n_dims, uint64_t ne0, uint64_t ne1, uint64_t ne2,
                             const void *data) {
    GGUFTensor t;
    memset(&t, 0, sizeof t);
    t.n_dims = n_dims;
    t.ne[0] = ne0; t.ne[1] = ne1; t.ne[2] = ne2; t.ne[3] = 1;
    t.type = type;
    t.data = data;
    return t;
}

/* Q8_K quantisation through the selected kernel table entry. */
REF_EXPORT void ref_quantize_q8k(const float *x, void *y, uint32_t n) {
    REF_FPENV_ENTER();
    lfm2_get_cpu_kernel_table()->quantize_q8_K(x, (block_q8_K_t *)y, n);
    REF_FPENV_LEAVE();
}

REF_EXPORT void ref_rmsnorm_q8k(const float *x, const float *norm_w, uint32_t D, float eps, float *xb,
                                void *xq) {
    REF_FPENV_ENTER();
    GGUFTensor tn = ref_tensor(GGML_TYPE_F32, 1, D, 1, 1, norm_w);
    lfm2_rmsnorm_quantize_q8_K_simd(xb, (block_q8_K_t *)xq, x, norm_w ? &tn : NULL, D, eps);
    REF_FPENV_LEAVE();
}

REF_EXPORT void ref_route(const float *router_w, const float *bias, const float *xb, uint32_t D,
                          uint32_t E, uint32_t K, uint32_t *idx, float *w) {
    REF_FPENV_ENTER();
    GGUFTensor tr = ref_tensor(GGML_TYPE_F32, 2, D, E, 1, router_w);
    GGUFTensor tb = ref_tensor(GGML_TYPE_F32, 1, E, 1, 1, bias);
    LFM2MoELayerExt moe;
    memset(&moe, 0, sizeof moe);
    moe.is_moe_layer = true;
    moe.n_experts = E;
    moe.n_experts_used = K;
    moe.norm_topk_prob = true;
    moe.routed_scale = 1.0f;
    moe.ffn_gate_inp = &tr;
    moe.ffn_exp_probs_b = bias ? &tb : NULL;
    uint32_t ii[LFM2_MAX_TOP_K];
    float ww[LFM2_MAX_TOP_K];
    lfm2_moe_route_sigmoid_topk(&moe, xb, NULL, ii, ww);
    for (uint32_t k = 0; k < K && k < LFM2_MAX_TOP_K; ++k) { idx[k] = ii[k]; w[k] = ww[k]; }
    REF_FPENV_LEAVE();
}

/* Rows [r0, r0+n_rows) of a Q4_K matrix (n_rows % 4 == 0) through the 4-row kernel. */
REF_EXPORT void ref_q4k_rows(const void *W, uint32_t n_cols, uint32_t total_rows, uint32_t r0,
                             uint32_t n_rows, const void *xq, float *out) {
    REF_FPENV_ENTER();
    GGUFTensor tw = ref_tensor(GGML_TYPE_Q4_K, 2, n_cols, total_rows, 1, W);
    for (uint32_t r = 0; r + 4 <= n_rows; r += 4)
        lfm2_compute_4rows_avx2(&tw, r0 + r, NULL, (const block_q8_K_t *)xq, out + r);
    REF_FPENV_LEAVE();
}

/* T tokens through lfm2_forward_moe_ffn_1x4, one call per token (the
 * reference has no batched MoE).  Optional per-token routing and Q8_K(x)
 * captured with the same calls the forward makes.  down_type: 12 (Q4_K) or 14 (Q6_K). */
REF_EXPORT int ref_moe_forward(float *x, uint32_t T, uint32_t D, uint32_t E, uint32_t K, uint32_t I,
                               float eps, const float *ffn_norm, const float *router_w, const float *bias,
                               const void *gate, const void *up, const void *down, uint32_t down_type,
                               uint32_t *idx_out, float *w_out, void *xq_out) {
    if (!g_pool_ready) ref_init(1);
    if (D % 256 || I % 256 || K > LFM2_MAX_TOP_K || E > LFM2_MAX_EXPERTS) return -1;
    REF_FPENV_ENTER();
    GGUFTensor tn = ref_tensor(GGML_TYPE_F32, 1, D, 1, 1, ffn_norm);
    GGUFTensor tr = ref_tensor(GGML_TYPE_F32, 2, D, E, 1, router_w);
    GGUFTensor tb = ref_tensor(GGML_TYPE_F32, 1, E, 1, 1, bias);
    GGUFTensor tg = ref_tensor(GGML_TYPE_Q4_K, 3, D, I, E, gate);
    GGUFTensor tu = ref_tensor(GGML_TYPE_Q4_K, 3, D, I, E, up);
    GGUFTensor td = ref_tensor(down_type, 3, I, D, E, down);
    LFM2Layer layer;
    memset(&layer, 0, sizeof layer);
    layer.ffn_norm = &tn;
    LFM2MoELayerExt moe;
    memset(&moe, 0, sizeof moe);
    moe.is_moe_layer = true;
    moe.n_experts = E;
    moe.n_experts_used = K;
    moe.norm_topk_prob = true;
    moe.routed_scale = 1.0f;
    moe.ffn_gate_inp = &tr;
    moe.ffn_exp_probs_b = bias ? &tb : NULL;
    moe.ffn_gate_exps = &tg;
    moe.ffn_up_exps = &tu;
    moe.ffn_down_exps = &td;

    float *xb = (float *)lfm2_aligned_alloc_64(sizeof(float) * D);
    float *hb = (float *)lfm2_aligned_alloc_64(sizeof(float) * I);
    block_q8_K_t *xq = (block_q8_K_t *)lfm2_aligned_alloc_64(sizeof(block_q8_K_t) * (D / 256 + I / 256));
    if (!xb || !hb || !xq) { free(xb); free(hb); free(xq); REF_FPENV_LEAVE(); return -2; }
    for (uint32_t t = 0; t < T; ++t) {
        float *xt = x + (size_t)t * D;
        if (idx_out || w_out || xq_out) {
            uint32_t ii[LFM2_MAX_TOP_K];
            float ww[LFM2_MAX_TOP_K];
            lfm2_rmsnorm_quantize_q8_K_simd(xb, xq, xt, &tn, D, eps);
            lfm2_moe_route_sigmoid_topk(&moe, xb, xq, ii, ww);
            for (uint32_t k = 0; k < K; ++k) {
                if (idx_out) idx_out[(size_t)t * K + k] = ii[k];
                if (w_out) w_out[(size_t)t * K + k] = ww[k];
            }
            if (xq_out) memcpy((block_q8_K_t *)xq_out + (size_t)t * (D / 256), xq, sizeof(block_q8_K_t) * (D / 256));
        }
        lfm2_forward_moe_ffn_1x4(&g_pool, xt, xb, hb, xq, &layer, &moe, D, eps);
    }
    free(xb); free(hb); free(xq);
    REF_FPENV_LEAVE();
    return 0;
}

/* Dense SwiGLU FFN (the leading non-MoE layers), one call per token. */
REF_EXPORT int ref_dense_ffn_forward(float *x, uint32_t T, uint32_t D, uint32_t I, float eps,
                                     const float *ffn_norm, const void *gate, const void *up,
                                     const void *down) {
    if (!g_pool_ready) ref_init(1);
    if (D % 256 || I % 256) return -1;
    REF_FPENV_ENTER();
    GGUFTensor tn = ref_tensor(GGML_TYPE_F32, 1, D, 1, 1, ffn_norm);
    GGUFTensor tg = ref_tensor(GGML_TYPE_Q4_K, 2, D, I, 1, gate);
    GGUFTensor tu = ref_tensor(GGML_TYPE_Q4_K, 2, D, I, 1, up);
    GGUFTensor td = ref_tensor(GGML_TYPE_Q4_K, 2, I, D, 1, down);
    LFM2Layer layer;
    memset(&layer, 0, sizeof layer);
    layer.ffn_norm = &tn;
    layer.ffn_gate = &tg;
    layer.ffn_up = &tu;
    layer.ffn_down = &td;
    float *xb = (float *)lfm2_aligned_alloc_64(sizeof(float) * D);
    float *hb = (float *)lfm2_aligned_alloc_64(sizeof(float) * I);
    block_q8_K_t *xq = (block_q8_K_t *)lfm2_aligned_alloc_64(sizeof(block_q8_K_t) * (D / 256 + I / 256));
    if (!xb || !hb || !xq) { free(xb); free(hb); free(xq); REF_FPENV_LEAVE(); return -2; }
    for (uint32_t t = 0; t < T; ++t)
        lfm2_forward_ffn_fused_1x4(&g_pool, x + (size_t)t * D, xb, hb, xq, &layer, D, eps);
    free(xb); free(hb); free(xq);
    REF_FPENV_LEAVE();
    return 0;
}
