/*
 * Device-side seeded generator: fills multi-GB synthetic stacks directly in
 * HBM with the same arithmetic as the host generator (lfm_synth_core.h, built
 * here with -fmad=false), so both produce identical bytes.
 */
#include "lfm_synth_core.h"
#include "moe_internal.h"

namespace {

__global__ void k_synth_q4k(uint8_t *out, uint64_t n_blocks, uint64_t first, uint64_t seed, float stddev) {
    lfm_block_q4_K *o = reinterpret_cast<lfm_block_q4_K *>(out);
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_blocks;
         i += (uint64_t)gridDim.x * blockDim.x) {
        lfm_block_q4_K b;
        lfm_q4k_normal_block(seed, first + i, stddev, &b);
        o[i] = b;
    }
}

__global__ void k_synth_f32(float *out, uint64_t n, uint64_t seed, float mean, float stddev) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        out[i] = lfm_det_normal_f32(seed, i, mean, stddev);
}

}  // namespace

cudaError_t lfm_launch_synth_q4k(uint8_t *out, uint64_t n_blocks, uint64_t seed, float stddev, cudaStream_t s,
                                 uint64_t first) {
    if (n_blocks == 0) return cudaSuccess;
    uint64_t grid = (n_blocks + 127) / 128;
    if (grid > 148ull * 64) grid = 148ull * 64;
    k_synth_q4k<<<(unsigned)grid, 128, 0, s>>>(out, n_blocks, first, seed, stddev);
    return cudaGetLastError();
}

cudaError_t lfm_launch_synth_f32(float *out, uint64_t n, uint64_t seed, float mean, float stddev, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    uint64_t grid = (n + 255) / 256;
    if (grid > 148ull * 32) grid = 148ull * 32;
    k_synth_f32<<<(unsigned)grid, 256, 0, s>>>(out, n, seed, mean, stddev);
    return cudaGetLastError();
}
