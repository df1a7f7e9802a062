/*
 * Seeded synthetic inputs for the MoE-FFN benchmarks and parity tests.
 *
 * Everything here uses only IEEE-754 basic operations (+ - * / sqrt and
 * round-to-nearest-even) with no fused multiply-add, so the host build
 * (gcc -std=c11, which does not contract) and the device build
 * (nvcc -fmad=false) produce bit-identical tensors.  That lets the device
 * generator fill multi-GB stacks while tests regenerate any slice on the host.
 *
 *  - counter RNG: splitmix64 (Steele, Lea & Flood, OOPSLA 2014) evaluated at
 *    an arbitrary position, so element i of a tensor depends only on (seed, i);
 *  - normals: Marsaglia's polar method on pairs of uniforms, with a bounded
 *    number of retries; log() is our own atanh-series evaluation in double;
 *  - Q4_K: a plain min/max quantiser of our own (6-bit per-32 scale and min,
 *    fp16 super-block scales).  The reference ships no fp32 -> Q4_K quantiser;
 *    parity is measured on identical Q4_K bytes, so its choice only shapes the
 *    inputs.
 */
#ifndef LFM_SYNTH_CORE_H
#define LFM_SYNTH_CORE_H

#include "lfm_formats.h"

#define LFM_SPLITMIX_GAMMA 0x9E3779B97F4A7C15ull

/* IEEE round-to-nearest division on both sides (the device compiler does not
 * always round a division by a constant correctly). */
#if defined(__CUDA_ARCH__)
#define LFM_FDIV(a, b) __fdiv_rn((a), (b))
#define LFM_DDIV(a, b) __ddiv_rn((a), (b))
#else
#define LFM_FDIV(a, b) ((a) / (b))
#define LFM_DDIV(a, b) ((a) / (b))
#endif

/* splitmix64 output number `ctr` (0-based) of the stream started at `seed`. */
LFM_HD uint64_t lfm_rng_u64(uint64_t seed, uint64_t ctr) {
    uint64_t z = seed + (ctr + 1ull) * LFM_SPLITMIX_GAMMA;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* natural log of a positive normal double: x = m * 2^e with m in [sqrt(1/2), sqrt(2)),
 * log(m) = 2 atanh(s), s = (m-1)/(m+1), |s| <= 0.1716, series to s^27. */
LFM_HD double lfm_det_log(double x) {
    uint64_t bits;
    memcpy(&bits, &x, sizeof bits);
    int e = (int)((bits >> 52) & 0x7FF) - 1023;
    bits = (bits & 0x000FFFFFFFFFFFFFull) | 0x3FF0000000000000ull;
    double m;
    memcpy(&m, &bits, sizeof m);
    if (m > 1.4142135623730951) { m = m * 0.5; e += 1; }
    const double s = LFM_DDIV(m - 1.0, m + 1.0);
    const double s2 = s * s;
    double term = s, sum = s;
    for (int k = 1; k <= 13; ++k) {
        term = term * s2;
        sum = sum + LFM_DDIV(term, (double)(2 * k + 1));
    }
    return 2.0 * sum + (double)e * 0.69314718055994530942;
}

/* Standard normal number `idx` of stream `seed` (polar method; pair idx/2 draws
 * up to 64 candidate points, the 2 coordinates give normals 2p and 2p+1). */
LFM_HD double lfm_det_normal(uint64_t seed, uint64_t idx) {
    const uint64_t pair = idx >> 1;
    for (uint64_t a = 0; a < 64; ++a) {
        const uint64_t c = (pair * 64ull + a) * 2ull;
        const double u = (double)(lfm_rng_u64(seed, c) >> 11) * (1.0 / 9007199254740992.0) * 2.0 - 1.0;
        const double v = (double)(lfm_rng_u64(seed, c + 1) >> 11) * (1.0 / 9007199254740992.0) * 2.0 - 1.0;
        const double s = u * u + v * v;
        if (s > 0.0 && s < 1.0) {
#if defined(__CUDA_ARCH__)
            const double f = __dsqrt_rn(LFM_DDIV(-2.0 * lfm_det_log(s), s));
#else
            const double f = sqrt(LFM_DDIV(-2.0 * lfm_det_log(s), s));
#endif
            return (idx & 1ull) ? v * f : u * f;
        }
    }
    return 0.0;
}

LFM_HD float lfm_det_normal_f32(uint64_t seed, uint64_t idx, float mean, float stddev) {
    return (float)lfm_det_normal(seed, idx) * stddev + mean;
}

LFM_HD float lfm_rne(float v) {
#if defined(__CUDA_ARCH__)
    return rintf(v);
#else
    return nearbyintf(v);
#endif
}

/* Quantise 256 floats into one Q4_K super-block (our own min/max scheme). */
LFM_HD void lfm_q4k_quantize_block(const float *x, lfm_block_q4_K *out) {
    float step[8], off[8];
    float max_step = 0.0f, max_off = 0.0f;
    for (int j = 0; j < 8; ++j) {
        float lo = x[32 * j], hi = x[32 * j];
        for (int i = 1; i < 32; ++i) {
            const float v = x[32 * j + i];
            lo = v < lo ? v : lo;
            hi = v > hi ? v : hi;
        }
        if (lo > 0.0f) lo = 0.0f;   /* the offset term -dmin*m is never positive */
        if (hi < lo) hi = lo;
        step[j] = LFM_FDIV(hi - lo, 15.0f);
        off[j] = -lo;
        max_step = step[j] > max_step ? step[j] : max_step;
        max_off = off[j] > max_off ? off[j] : max_off;
    }
    const uint16_t dh = lfm_float_to_half(LFM_FDIV(max_step, 63.0f));
    const uint16_t mh = lfm_float_to_half(LFM_FDIV(max_off, 63.0f));
    const float d = lfm_half_to_float(dh), dmin = lfm_half_to_float(mh);
    int sc[8], mn[8];
    for (int j = 0; j < 8; ++j) {
        float a = d > 0.0f ? lfm_rne(LFM_FDIV(step[j], d)) : 0.0f;
        float b = dmin > 0.0f ? lfm_rne(LFM_FDIV(off[j], dmin)) : 0.0f;
        sc[j] = a > 63.0f ? 63 : (int)a;
        mn[j] = b > 63.0f ? 63 : (int)b;
    }
    out->d = dh;
    out->dmin = mh;
    for (int j = 0; j < 4; ++j) {
        out->scales[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        out->scales[j + 4] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
        out->scales[j + 8] = (uint8_t)((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
    }
    uint8_t q[256];
    for (int j = 0; j < 8; ++j) {
        const float s = d * (float)sc[j];
        const float o = dmin * (float)mn[j];
        for (int i = 0; i < 32; ++i) {
            int v = 0;
            if (s > 0.0f) {
                const float r = lfm_rne(LFM_FDIV(x[32 * j + i] + o, s));
                v = r < 0.0f ? 0 : (r > 15.0f ? 15 : (int)r);
            }
            q[32 * j + i] = (uint8_t)v;
        }
    }
    for (int g = 0; g < 4; ++g)
        for (int l = 0; l < 32; ++l)
            out->qs[32 * g + l] = (uint8_t)(q[64 * g + l] | (q[64 * g + 32 + l] << 4));
}

/* Fill one Q4_K super-block with quantised N(0, stddev) weights: block `blk`
 * of the tensor covers normal numbers [256*blk, 256*blk + 256) of `seed`. */
LFM_HD void lfm_q4k_normal_block(uint64_t seed, uint64_t blk, float stddev, lfm_block_q4_K *out) {
    float x[256];
    for (int i = 0; i < 256; ++i)
        x[i] = lfm_det_normal_f32(seed, blk * 256ull + (uint64_t)i, 0.0f, stddev);
    lfm_q4k_quantize_block(x, out);
}

#endif /* LFM_SYNTH_CORE_H */
