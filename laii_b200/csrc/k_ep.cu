/*
 * Expert parallelism over peer memory: the exchange kernels.
 *
 * One process per GPU; every rank's exchange arena is mapped into every other
 * rank (CUDA IPC over NVLink / NVSwitch), so the two all-to-all steps of a
 * layer are loads and stores of the kernels themselves:
 *   k_ep_publish       home rank: its per-expert counts into every rank's
 *                      count table, then its cnt_flag there (release);
 *   (k_ep_plan, k_route.cu; k_xt_gather_ep, k_umma.cu: the expert rank lays
 *    out the received slots and gathers their Q8_K rows from the home ranks)
 *   (the down GEMM, k_umma.cu, stores each output row straight into its home
 *    rank's yhome[t*K + k] from its epilogue; its last CTA raises y_flag on
 *    every rank (release));
 *   k_ep_combine_wait  home rank: acquire every y_flag, then
 *                      x[t] = fma(w[t][k], yhome[t*K+k], x[t]) for k in order
 *                      (tools/lfm2_moe_checkpoint.c:266-269).
 * Flags hold the epoch of the layer step, read from the rank's device-side
 * step counter (the combine's last CTA advances it); waits compare wrap-safe
 * and are bounded by EpStep::wait_ns (LFM_DEVERR_TIMEOUT, then the kernel
 * returns).
 * Buffer reuse needs no further handshake: a home rank overwrites its Q8_K
 * rows, perm and count-table entries for step n+1 only after its combine of
 * step n saw every expert rank's y_flag, which each raises after it gathered
 * and computed step n; an expert rank writes yhome rows of step n+1 only after
 * every home rank published step n+1, i.e. after that rank's combine of step
 * n read them.  The count table alternates by epoch parity because a home rank
 * can publish step n+1 while a slower expert rank still plans step n.
 */
#include "moe_device.cuh"
#include "moe_internal.h"

namespace {

__global__ void __launch_bounds__(256) k_ep_publish(EpStep st, const int32_t *__restrict__ counts) {
    const uint32_t epoch = __ldcg(st.self.step) + st.ahead;
    const size_t row = ((size_t)(epoch & 1u) * LFM_EP_MAX_RANKS + st.rank) * st.E;
    for (uint32_t q = threadIdx.x; q < st.world * st.E; q += blockDim.x) {
        const uint32_t p = q / st.E, e = q - p * st.E;
        st.table[p][row + e] = __ldcg(counts + e);
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < st.world) lfm_st_release_sys(st.cnt_flag[threadIdx.x] + st.rank, epoch);
}

/* x[t][c..c+3] = fma(w[t][k], yhome[t*K+k][c..c+3], x) for k = 0..K-1 in order. */
__global__ void __launch_bounds__(256) k_ep_combine_wait(EpStep st, float *__restrict__ x, uint32_t T,
                                                         const float *__restrict__ w, int advance) {
    __shared__ int ok;
    lfm_pdl_launch_dependents();
    lfm_pdl_wait(); /* x and the routing tables belong to the preceding kernels */
    if (threadIdx.x == 0) {
        const uint32_t epoch = __ldcg(st.self.step) + st.ahead;
        ok = lfm_wait_flags(st.self.y_flag, st.world, epoch, st.wait_ns, st.err) ? 1 : 0;
        /* the step is over for this rank once every CTA has read its epoch: the last one advances it */
        __threadfence();
        if (advance && atomicAdd(st.self.cdone, 1u) == gridDim.x - 1) {
            atomicExch(st.self.cdone, 0u);
            atomicExch(st.self.step, epoch);
        }
    }
    __syncthreads();
    if (!ok) return;
    const uint32_t D4 = st.D / 4, K = st.K;
    const float *y = st.self.yhome;
    const uint64_t n = (uint64_t)T * D4;
    for (uint64_t q = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n; q += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t t = q / D4, c = q - t * D4;
        float4 acc = reinterpret_cast<float4 *>(x)[q];
        for (uint32_t k = 0; k < K; ++k) {
            const float wk = __ldg(w + t * K + k);
            const float4 v = __ldcg(reinterpret_cast<const float4 *>(y + (t * K + k) * st.D) + c);
            acc.x = __fmaf_rn(wk, v.x, acc.x);
            acc.y = __fmaf_rn(wk, v.y, acc.y);
            acc.z = __fmaf_rn(wk, v.z, acc.z);
            acc.w = __fmaf_rn(wk, v.w, acc.w);
        }
        reinterpret_cast<float4 *>(x)[q] = acc;
    }
}

}  // namespace

cudaError_t lfm_launch_ep_publish(const EpStep &st, const int32_t *counts, cudaStream_t s) {
    if (st.world == 0 || st.world > LFM_EP_MAX_RANKS) return cudaErrorInvalidValue;
    k_ep_publish<<<1, 256, 0, s>>>(st, counts);
    return cudaGetLastError();
}

cudaError_t lfm_launch_ep_combine_wait(const EpStep &st, float *x, uint32_t T, const float *w, bool advance,
                                       cudaStream_t s, bool pdl) {
    if (st.world == 0 || st.world > LFM_EP_MAX_RANKS || st.D % 4) return cudaErrorInvalidValue;
    const uint64_t n = (uint64_t)T * (st.D / 4);
    uint64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 8) blocks = 148 * 8;
    if (blocks == 0) blocks = 1; /* T == 0 still waits: no rank runs ahead of the step */
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)blocks);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_ep_combine_wait, st, x, T, w, advance ? 1 : 0);
}
