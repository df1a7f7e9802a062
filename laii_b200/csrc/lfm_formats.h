/*
 * GGML K-quant block layouts on the lfm2moe MoE-FFN path, plus the scalar
 * helpers shared by host C, the CPU oracle and CUDA device code.
 *
 * The byte layouts are an interchange format (GGUF tensors are uploaded as-is),
 * so they must match the reference exactly:
 *   - Q4_K super-block, 256 weights in 144 bytes
 *     (reference: tools/lfm2_cpuid_quants.c:78-83, block_q4_K_t)
 *   - Q8_K activation super-block, 256 int8 + fp32 scale + 16 int16 partial sums
 *     in 292 bytes (reference: tools/lfm2_cpuid_quants.c:123-127, block_q8_K_t)
 *
 * Q4_K weight w[i] of sub-block j (32 weights) is  d*sc_j*q[i] - dmin*m_j,
 * with d, dmin fp16, sc_j/m_j 6-bit codes packed in scales[12] and q[i] a
 * 4-bit code.  qs[] stores 4 groups of 32 bytes; byte l of group g holds
 * element 64g+l in its low nibble and element 64g+32+l in its high nibble.
 */
#ifndef LFM_FORMATS_H
#define LFM_FORMATS_H

#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define LFM_HD __host__ __device__ __forceinline__
#else
#define LFM_HD static inline
#endif

#define LFM_QK_K 256          /* elements per K-quant super-block            */
#define LFM_Q4K_BYTES 144     /* sizeof(lfm_block_q4_K)                      */
#define LFM_Q8K_BYTES 292     /* sizeof(lfm_block_q8_K)                      */
#define LFM_Q6K_BYTES 210     /* block_q6_K: ql[128] qh[64] int8 scales[16] fp16 d */
#define LFM_GGML_TYPE_F32 0u
#define LFM_GGML_TYPE_Q4_K 12u
#define LFM_GGML_TYPE_Q6_K 14u

typedef struct {
    uint16_t d;          /* fp16 scale of the 6-bit sub-block scales        */
    uint16_t dmin;       /* fp16 scale of the 6-bit sub-block mins          */
    uint8_t  scales[12]; /* 8 x (6-bit scale, 6-bit min), packed            */
    uint8_t  qs[128];    /* 256 4-bit codes                                 */
} lfm_block_q4_K;

typedef struct {
    float   d;           /* max|x| / 127                                    */
    int8_t  qs[256];     /* round-to-nearest-even(x * 127 / max|x|)         */
    int16_t bsums[16];   /* sum of each run of 16 codes                     */
} lfm_block_q8_K;

#if !defined(__cplusplus)
_Static_assert(sizeof(lfm_block_q4_K) == LFM_Q4K_BYTES, "Q4_K block size");
_Static_assert(sizeof(lfm_block_q8_K) == LFM_Q8K_BYTES, "Q8_K block size");
#else
static_assert(sizeof(lfm_block_q4_K) == LFM_Q4K_BYTES, "Q4_K block size");
static_assert(sizeof(lfm_block_q8_K) == LFM_Q8K_BYTES, "Q8_K block size");
#endif

/* 6-bit scale / min codes of sub-block j (0..7) of a Q4_K super-block.
 * Sub-blocks 0..3 keep their 6 bits in the low bits of scales[j] (scale) and
 * scales[j+4] (min).  Sub-blocks 4..7 keep their low 4 bits in the two nibbles
 * of scales[j+4] and their top 2 bits in the top bits of scales[j-4] (scale)
 * and scales[j] (min).  Same unpacking as the reference's get_scale_min_k4
 * (tools/lfm2_cpuid_quants.c:182-191). */
LFM_HD void lfm_q4k_scale_min(int j, const uint8_t *s, int *sc, int *m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m  = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        *m  = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* Exact IEEE binary16 -> binary32 (normals, subnormals, inf, nan). */
LFM_HD float lfm_half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    uint32_t bits;
    if (e == 0x1Fu) {
        bits = sign | 0x7F800000u | (m << 13);
    } else if (e != 0) {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    } else if (m == 0) {
        bits = sign;
    } else {
        /* subnormal half: normalise the mantissa */
        int shift = 0;
        while ((m & 0x400u) == 0) { m <<= 1; ++shift; }
        m &= 0x3FFu;
        bits = sign | ((uint32_t)(113 - shift) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

/* IEEE binary32 -> binary16 with round-to-nearest-even. */
LFM_HD uint16_t lfm_float_to_half(float f) {
    uint32_t x;
    memcpy(&x, &f, sizeof x);
    const uint32_t sign = (x >> 16) & 0x8000u;
    x &= 0x7FFFFFFFu;
    if (x >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (x > 0x7F800000u ? 0x200u : 0u));
    if (x >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* >= 65520 rounds to inf */
    if (x < 0x38800000u) {                                   /* below 2^-14: subnormal */
        if (x < 0x33000000u) return (uint16_t)sign;           /* <= 2^-25 rounds to 0   */
        const uint32_t e = x >> 23;
        const uint32_t mant = (x & 0x7FFFFFu) | 0x800000u;
        const uint32_t shift = 126u - e;
        uint32_t h = mant >> shift;
        const uint32_t rem = mant & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (h & 1u))) ++h;
        return (uint16_t)(sign | h);
    }
    uint32_t h = (x >> 13) - (112u << 10);
    const uint32_t rem = x & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
}

#endif /* LFM_FORMATS_H */
