/*
 * Host side of the seeded synthetic-input generator (liblfm_synth.so).
 * The arithmetic lives in lfm_synth_core.h and is shared bit-for-bit with
 * the device generator in lfm_gpu_synth.cu.  Large tensors are split over
 * POSIX threads; the result does not depend on the thread count.
 */
#define _GNU_SOURCE
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>

#include "lfm_synth_core.h"

#define LFM_EXPORT __attribute__((visibility("default")))

LFM_EXPORT uint64_t lfm_synth_u64(uint64_t seed, uint64_t ctr) { return lfm_rng_u64(seed, ctr); }

LFM_EXPORT double lfm_synth_normal(uint64_t seed, uint64_t idx) { return lfm_det_normal(seed, idx); }

LFM_EXPORT double lfm_synth_log(double x) { return lfm_det_log(x); }

LFM_EXPORT uint16_t lfm_synth_float_to_half(float f) { return lfm_float_to_half(f); }

LFM_EXPORT float lfm_synth_half_to_float(uint16_t h) { return lfm_half_to_float(h); }

typedef struct {
    int kind;            /* 0 = f32 normal, 1 = q4k normal */
    void *out;
    uint64_t seed, first, count;
    float mean, stddev;
} synth_job;

static void *synth_worker(void *arg) {
    synth_job *j = (synth_job *)arg;
    if (j->kind == 0) {
        float *o = (float *)j->out;
        for (uint64_t i = 0; i < j->count; ++i)
            o[i] = lfm_det_normal_f32(j->seed, j->first + i, j->mean, j->stddev);
    } else {
        lfm_block_q4_K *o = (lfm_block_q4_K *)j->out;
        for (uint64_t i = 0; i < j->count; ++i)
            lfm_q4k_normal_block(j->seed, j->first + i, j->stddev, &o[i]);
    }
    return NULL;
}

static void synth_run(int kind, void *out, size_t elem_bytes, uint64_t n, uint64_t first,
                      uint64_t seed, float mean, float stddev, int n_threads) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 64) n_threads = 64;
    if ((uint64_t)n_threads > n) n_threads = n ? (int)n : 1;
    pthread_t th[64];
    int joinable[64] = {0};
    synth_job jobs[64];
    const uint64_t per = (n + (uint64_t)n_threads - 1) / (uint64_t)n_threads;
    int n_jobs = 0;
    for (int t = 0; t < n_threads; ++t) {
        const uint64_t a = (uint64_t)t * per;
        if (a >= n) break;
        const uint64_t b = a + per < n ? a + per : n;
        jobs[t] = (synth_job){kind, (uint8_t *)out + a * elem_bytes, seed, first + a, b - a, mean, stddev};
        n_jobs = t + 1;
    }
    for (int t = 1; t < n_jobs; ++t) {
        if (pthread_create(&th[t], NULL, synth_worker, &jobs[t]) == 0) joinable[t] = 1;
        else synth_worker(&jobs[t]);   /* no thread available: run inline */
    }
    if (n_jobs > 0) synth_worker(&jobs[0]);
    for (int t = 1; t < n_jobs; ++t)
        if (joinable[t]) pthread_join(th[t], NULL);
}

/* out[i] = mean + stddev * N_(seed, first + i), i < n. */
LFM_EXPORT void lfm_synth_fill_normal_f32(float *out, uint64_t n, uint64_t first, uint64_t seed,
                                          float mean, float stddev, int n_threads) {
    synth_run(0, out, sizeof(float), n, first, seed, mean, stddev, n_threads);
}

/* Q4_K blocks [first_block, first_block + n_blocks) of an N(0, stddev) tensor. */
LFM_EXPORT void lfm_synth_fill_q4k_normal(void *out, uint64_t n_blocks, uint64_t first_block,
                                          uint64_t seed, float stddev, int n_threads) {
    synth_run(1, out, sizeof(lfm_block_q4_K), n_blocks, first_block, seed, 0.0f, stddev, n_threads);
}

/* Quantise n floats (n a multiple of 256) into n/256 Q4_K blocks. */
LFM_EXPORT int lfm_synth_quantize_q4k(const float *x, void *out, uint64_t n) {
    if (n % 256) return -1;
    lfm_block_q4_K *o = (lfm_block_q4_K *)out;
    for (uint64_t b = 0; b < n / 256; ++b) lfm_q4k_quantize_block(x + b * 256, &o[b]);
    return 0;
}

/* Dequantise Q4_K blocks to fp32 (w = d*sc*q - dmin*m, evaluated as two
 * products and a difference). */
LFM_EXPORT void lfm_synth_dequantize_q4k(const void *in, float *out, uint64_t n_blocks) {
    const lfm_block_q4_K *b = (const lfm_block_q4_K *)in;
    for (uint64_t i = 0; i < n_blocks; ++i) {
        const float d = lfm_half_to_float(b[i].d), dmin = lfm_half_to_float(b[i].dmin);
        for (int j = 0; j < 8; ++j) {
            int sc, m;
            lfm_q4k_scale_min(j, b[i].scales, &sc, &m);
            const int g = j >> 1, hi = j & 1;
            for (int l = 0; l < 32; ++l) {
                const int q = hi ? (b[i].qs[32 * g + l] >> 4) : (b[i].qs[32 * g + l] & 15);
                out[i * 256 + 32 * j + l] = d * (float)sc * (float)q - dmin * (float)m;
            }
        }
    }
}
