/*
 * Small kernels around the grouped GEMVs (decode / verify path):
 *   k_quant_rows  Q8_K of h per 256 (tools/lfm2_cpuid_quants.c:584-631);
 *   k_combine     x[t][r] = fma(w_k, y[slot(t,k)][r], x[t][r]) for k = 0..K-1
 *                 in order (tools/lfm2_moe_checkpoint.c:266-269, :338-364);
 *   conversions between the internal Q8 rows and 292-byte GGUF block_q8_K.
 * All chain with programmatic dependent launch.
 */
#include "moe_device.cuh"
#include "moe_internal.h"

namespace {

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

/* Expert parallelism, received rows: row a goes to local expert
 * expert_ids[a] - first with weight 1 (out-of-shard ids are flagged and dropped). */
__global__ void k_ep_prepare(const int32_t *__restrict__ ids, uint32_t n, uint32_t first, uint32_t count,
                             RouteTables rt) {
    for (uint32_t a = blockIdx.x * blockDim.x + threadIdx.x; a < n; a += gridDim.x * blockDim.x) {
        const int32_t e = ids[a] - (int32_t)first;
        const bool ok = e >= 0 && (uint32_t)e < count;
        if (!ok) atomicOr(rt.err, LFM_DEVERR_EXPERT_ID);
        rt.idx[a] = ok ? e : -1;
        rt.w[a] = 1.0f;
    }
}

/* x[t][r] = fma(w[t][k], y[t*K+k][r], x[t][r]) for k = 0..K-1 in order
 * (tools/lfm2_moe_checkpoint.c:266-269), y already in (t, k) order. */
__global__ void __launch_bounds__(256) k_ep_combine(float *__restrict__ x, uint32_t T, uint32_t D, uint32_t K,
                                                    const float *__restrict__ w, const float *__restrict__ y) {
    const uint64_t n = (uint64_t)T * D;
    for (uint64_t q = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n; q += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t t = q / D, r = q - t * D;
        float acc = x[q];
        for (uint32_t k = 0; k < K; ++k) acc = __fmaf_rn(w[t * K + k], y[(t * K + k) * D + r], acc);
        x[q] = acc;
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

cudaError_t lfm_launch_ep_prepare(const int32_t *expert_ids, uint32_t n, uint32_t first, uint32_t count,
                                  const RouteTables &rt, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    k_ep_prepare<<<min(1184u, (n + 255) / 256), 256, 0, s>>>(expert_ids, n, first, count, rt);
    return cudaGetLastError();
}

cudaError_t lfm_launch_ep_combine(float *x, uint32_t T, uint32_t D, uint32_t K, const float *w, const float *y,
                                  cudaStream_t s) {
    const uint64_t n = (uint64_t)T * D;
    if (n == 0) return cudaSuccess;
    const uint64_t blocks = (n + 255) / 256;
    k_ep_combine<<<(unsigned)(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0, s>>>(x, T, D, K, w, y);
    return cudaGetLastError();
}
