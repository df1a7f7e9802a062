/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for the lfm2moe MoE-FFN hot path.
 *
 * A scalar C11 restatement of the reference CPU path (laii, tools/
 * lfm2_moe_checkpoint.c:312-365 and the kernels it calls) that reproduces the
 * reference's floating-point evaluation order exactly, so its outputs can be
 * compared bit-for-bit with the reference built from source (oracle/_ref) and
 * with the CUDA path.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may load it.  The product library never calls into it.
 *
 * Pinning: tests/test_oracle_ref.py runs it against the reference itself
 * (oracle/_ref/libref_moe.so, built from the reference sources by
 * oracle/Makefile) on seeded inputs, bit-exact, and tests/test_oracle_golden.py
 * checks it against fixtures that the reference produced (tests/golden/).
 *
 * Evaluation-order notes (all from the AVX2/AVX-VNNI kernels the reference
 * selects at run time, tools/lfm2_cpuid_quants.c:1797-1917):
 *  - fp32 dot / sum-of-squares: 16 running lanes (two 8-wide FMA accumulators),
 *    then acc0+acc1, then the hsum tree (lo+hi, pairs, final pair),
 *    include/lfm2_simd_avx2.h:286-293 and :676-687;
 *  - Q8_K: d = max/127, codes = RNE(x * (127/max)), bsums from the unsaturated
 *    codes, tools/lfm2_cpuid_quants.c:584-631;
 *  - Q4_K x Q8_K, 4-row kernels: integer sums are exact; per super-block the
 *    fp32 update is  sum = fma(d*d8, acc, fma(-(dmin*d8), mins, sum))  for the
 *    AVX-VNNI kernel (:1189-1257) and  sum = sum + ((d*d8)*acc - (dmin*d8)*mins)
 *    for the AVX2 kernel (:978-1045).  `order` selects which one.
 *
 * Build: oracle/Makefile (gcc -std=c11 -O2 -mfma; ISO C mode, so gcc does
 * not contract a*b+c into an FMA on its own; every FMA below is explicit).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_EXPORT __attribute__((visibility("default")))

enum { ORC_ORDER_VNNI = 0, ORC_ORDER_AVX2 = 1 };

#pragma pack(push, 1)
typedef struct { uint16_t d, dmin; uint8_t scales[12]; uint8_t qs[128]; } orc_q4k;
typedef struct { float d; int8_t qs[256]; int16_t bsums[16]; } orc_q8k;
typedef struct { uint8_t ql[128]; uint8_t qh[64]; int8_t scales[16]; uint16_t d; } orc_q6k;
#pragma pack(pop)

_Static_assert(sizeof(orc_q4k) == 144, "q4k");
_Static_assert(sizeof(orc_q6k) == 210, "q6k");
_Static_assert(sizeof(orc_q8k) == 292, "q8k");

static float orc_h2f(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 31u, m = h & 1023u, bits;
    if (e == 31u) bits = sign | 0x7F800000u | (m << 13);
    else if (e) bits = sign | ((e + 112u) << 23) | (m << 13);
    else if (!m) bits = sign;
    else {
        int s = 0;
        while (!(m & 1024u)) { m <<= 1; ++s; }
        bits = sign | ((uint32_t)(113 - s) << 23) | ((m & 1023u) << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* tools/lfm2_cpuid_quants.c:182-191 */
static void orc_scale_min(int j, const uint8_t *q, int *sc, int *m) {
    if (j < 4) { *sc = q[j] & 63; *m = q[j + 4] & 63; }
    else {
        *sc = (q[j + 4] & 15) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

/* 8-lane horizontal sum as in include/lfm2_simd_avx2.h:286-293. */
static float orc_hsum8(const float v[8]) {
    float s[4];
    for (int i = 0; i < 4; ++i) s[i] = v[i] + v[i + 4];
    const float a = s[0] + s[2];
    const float b = s[1] + s[3];
    return a + b;
}

/* Sum of w[i]*x[i] in the order of include/lfm2_simd_avx2.h:676-687 (tail
 * elements, if n % 16 != 0, are added one by one with a separate multiply). */
ORC_EXPORT float orc_dot_f32(const float *w, const float *x, uint32_t n) {
    float acc[16] = {0};
    uint32_t i = 0;
    for (; i + 16 <= n; i += 16)
        for (int l = 0; l < 16; ++l) acc[l] = fmaf(w[i + l], x[i + l], acc[l]);
    float v[8];
    for (int l = 0; l < 8; ++l) v[l] = acc[l] + acc[l + 8];
    float sum = orc_hsum8(v);
    for (; i < n; ++i) sum = sum + w[i] * x[i];
    return sum;
}

static void orc_q8k_block(const float *x, orc_q8k *y) {
    float amax = 0.0f;
    for (int i = 0; i < 256; ++i) {
        const float a = fabsf(x[i]);
        if (a > amax) amax = a;
    }
    if (amax == 0.0f) { memset(y, 0, sizeof *y); return; }
    y->d = amax / 127.0f;
    const float s = 127.0f / amax;
    for (int j = 0; j < 16; ++j) {
        int32_t bs = 0;
        for (int l = 0; l < 16; ++l) {
            int32_t q = (int32_t)nearbyintf(x[16 * j + l] * s);
            bs += q;
            y->qs[16 * j + l] = (int8_t)(q > 127 ? 127 : (q < -128 ? -128 : q));
        }
        y->bsums[j] = (int16_t)bs;
    }
}

/* tools/lfm2_cpuid_quants.c:584-631 (the quantiser both x86 kernel tables use). */
ORC_EXPORT void orc_quantize_q8k(const float *x, void *y, uint32_t n) {
    for (uint32_t b = 0; b < n / 256; ++b) orc_q8k_block(x + 256 * b, (orc_q8k *)y + b);
}

/* RMSNorm + Q8_K, tools/lfm2_decode_1x4.c:93-196: sum of squares over 16
 * running lanes, inv = 1/sqrtf(ss/D + eps), xb = (x*inv)*w, then Q8_K per 256. */
ORC_EXPORT void orc_rmsnorm_q8k(const float *x, const float *norm_w, uint32_t D, float eps,
                                float *xb, void *xq) {
    float acc[16] = {0};
    uint32_t i = 0;
    for (; i + 16 <= D; i += 16)
        for (int l = 0; l < 16; ++l) acc[l] = fmaf(x[i + l], x[i + l], acc[l]);
    float v[8];
    for (int l = 0; l < 8; ++l) v[l] = acc[l] + acc[l + 8];
    float ss = orc_hsum8(v);
    for (; i < D; ++i) ss = ss + x[i] * x[i];
    const float inv = 1.0f / sqrtf(ss / (float)D + eps);
    for (uint32_t k = 0; k < D; ++k) {
        const float n = x[k] * inv;
        xb[k] = norm_w ? n * norm_w[k] : n;
    }
    if (xq) orc_quantize_q8k(xb, xq, D - D % 256);
}

/* Sigmoid + exp_probs_b-biased top-K, tools/lfm2_moe_checkpoint.c:166-240
 * (F32 router branch).  logits/sel (optional) receive z_e and s_e + b_e. */
ORC_EXPORT void orc_route(const float *router_w, const float *bias, const float *xb, uint32_t D,
                          uint32_t E, uint32_t K, int norm_topk, float routed_scale,
                          uint32_t *idx, float *w, float *logits, float *sel_out) {
    float sig[256], sel[256];
    for (uint32_t e = 0; e < E; ++e) {
        const float z = orc_dot_f32(router_w + (size_t)e * D, xb, D);
        sig[e] = 1.0f / (1.0f + expf(-z));
        sel[e] = bias ? sig[e] + bias[e] : sig[e];
        if (logits) logits[e] = z;
        if (sel_out) sel_out[e] = sel[e];
    }
    for (uint32_t k = 0; k < K; ++k) {
        uint32_t best = 0;
        float bv = -1e30f;
        for (uint32_t e = 0; e < E; ++e)
            if (sel[e] > bv) { bv = sel[e]; best = e; }
        idx[k] = best;
        w[k] = sig[best];
        sel[best] = -1e30f;
    }
    if (norm_topk) {
        float s = 0.0f;
        for (uint32_t k = 0; k < K; ++k) s = s + w[k];
        const float inv = routed_scale / (s + 1e-20f);
        for (uint32_t k = 0; k < K; ++k) w[k] = w[k] * inv;
    } else if (routed_scale != 1.0f) {
        for (uint32_t k = 0; k < K; ++k) w[k] = w[k] * routed_scale;
    }
}

/* Exact integer parts of one Q4_K x Q8_K super-block (tools/lfm2_cpuid_quants.c:
 * 421-457): per-sub-block dots, acc = sum sc_j*dot_j, mins = sum m_j*(bsum pair). */
static void orc_q4k_sb_ints(const orc_q4k *w, const orc_q8k *x, int32_t dots[8], int32_t *acc,
                            int32_t *mins) {
    int32_t a = 0, mn = 0;
    for (int j = 0; j < 8; ++j) {
        int sc, m;
        orc_scale_min(j, w->scales, &sc, &m);
        const int g = j >> 1, hi = j & 1;
        int32_t dot = 0;
        for (int l = 0; l < 32; ++l) {
            const int q = hi ? (w->qs[32 * g + l] >> 4) : (w->qs[32 * g + l] & 15);
            dot += q * (int32_t)x->qs[32 * j + l];
        }
        dots[j] = dot;
        a += sc * dot;
        mn += m * ((int32_t)x->bsums[2 * j] + (int32_t)x->bsums[2 * j + 1]);
    }
    *acc = a;
    *mins = mn;
}

static float orc_q4k_row(int order, const orc_q4k *row, const orc_q8k *x, uint32_t nb) {
    float sum = 0.0f;
    for (uint32_t b = 0; b < nb; ++b) {
        const float d8 = x[b].d;
        if (d8 == 0.0f) continue;
        int32_t dots[8], acc, mins;
        orc_q4k_sb_ints(&row[b], &x[b], dots, &acc, &mins);
        const float dd = d8 * orc_h2f(row[b].d);
        const float dm = d8 * orc_h2f(row[b].dmin);
        if (order == ORC_ORDER_VNNI) {
            sum = fmaf(dd, (float)acc, fmaf(-dm, (float)mins, sum));
        } else {
            sum = sum + (dd * (float)acc - dm * (float)mins);
        }
    }
    return sum;
}

/* out[r] = row r0+r of a Q4_K matrix [n_rows x n_cols] dotted with Q8_K xq. */
ORC_EXPORT void orc_q4k_rows(int order, const void *W, uint32_t n_cols, uint32_t r0, uint32_t n_rows,
                             const void *xq, float *out) {
    const uint32_t nb = n_cols / 256;
    const orc_q4k *w = (const orc_q4k *)W;
    for (uint32_t r = 0; r < n_rows; ++r)
        out[r] = orc_q4k_row(order, w + (size_t)(r0 + r) * nb, (const orc_q8k *)xq, nb);
}

/* Integer partial sums of one row: sub_dots[nb*8], acc[nb], mins[nb]. */
ORC_EXPORT void orc_q4k_row_ints(const void *row, const void *xq, uint32_t n_cols, int32_t *sub_dots,
                                 int32_t *acc, int32_t *mins) {
    const orc_q4k *w = (const orc_q4k *)row;
    const orc_q8k *x = (const orc_q8k *)xq;
    for (uint32_t b = 0; b < n_cols / 256; ++b)
        orc_q4k_sb_ints(&w[b], &x[b], sub_dots + 8 * b, &acc[b], &mins[b]);
}

/* Exact integer part of one Q6_K x Q8_K super-block (tools/lfm2_cpuid_quants.c:
 * 467-509 scalar, :1398-1540 AVX-VNNI): element i (half = i/128, m = (i/32)%4,
 * l = i%32) is  q = nibble m/2 of ql[64*half + 32*(m%2) + l]  |  bits 2m..2m+1 of
 * qh[32*half + l] << 4  (0..63), with the signed scale of sub-block i/16;
 * acc = sum sc*q*q8, off = sum sc_j*bsums_j, total = acc - 32*off. */
static int32_t orc_q6k_sb_int(const orc_q6k *w, const orc_q8k *x, int32_t *acc_out, int32_t *off_out) {
    int32_t acc = 0, off = 0;
    for (int j = 0; j < 16; ++j) off += (int32_t)w->scales[j] * (int32_t)x->bsums[j];
    for (int i = 0; i < 256; ++i) {
        const int half = i >> 7, m = (i >> 5) & 3, l = i & 31;
        const uint8_t lo = w->ql[64 * half + 32 * (m & 1) + l];
        const int q = ((m & 2) ? (lo >> 4) : (lo & 15)) | (((w->qh[32 * half + l] >> (2 * m)) & 3) << 4);
        acc += q * (int32_t)x->qs[i] * (int32_t)w->scales[i >> 4];
    }
    if (acc_out) *acc_out = acc;
    if (off_out) *off_out = off;
    return acc - 32 * off;
}

/* fp32 update per super-block, skipped where d8 == 0: AVX-VNNI 1x4 kernel
 * sum = fma(d8*d, total, sum) (:1534); AVX2 1x4 kernel
 * sum = sum + (d8*d)*total (tools/lfm2_cpuid_quants.c:1124). */
static float orc_q6k_row(int order, const orc_q6k *row, const orc_q8k *x, uint32_t nb) {
    float sum = 0.0f;
    for (uint32_t b = 0; b < nb; ++b) {
        const float d8 = x[b].d;
        if (d8 == 0.0f) continue;
        const int32_t tot = orc_q6k_sb_int(&row[b], &x[b], NULL, NULL);
        const float dd = d8 * orc_h2f(row[b].d);
        if (order == ORC_ORDER_VNNI) sum = fmaf(dd, (float)tot, sum);
        else sum = sum + dd * (float)tot;
    }
    return sum;
}

/* out[r] = row r0+r of a Q6_K matrix [n_rows x n_cols] dotted with Q8_K xq. */
ORC_EXPORT void orc_q6k_rows(int order, const void *W, uint32_t n_cols, uint32_t r0, uint32_t n_rows,
                             const void *xq, float *out) {
    const uint32_t nb = n_cols / 256;
    const orc_q6k *w = (const orc_q6k *)W;
    for (uint32_t r = 0; r < n_rows; ++r)
        out[r] = orc_q6k_row(order, w + (size_t)(r0 + r) * nb, (const orc_q8k *)xq, nb);
}

/* Integer parts of one Q6_K row: acc[nb], off[nb], total[nb] = acc - 32*off. */
ORC_EXPORT void orc_q6k_row_ints(const void *row, const void *xq, uint32_t n_cols, int32_t *acc, int32_t *off,
                                 int32_t *total) {
    const orc_q6k *w = (const orc_q6k *)row;
    const orc_q8k *x = (const orc_q8k *)xq;
    for (uint32_t b = 0; b < n_cols / 256; ++b) total[b] = orc_q6k_sb_int(&w[b], &x[b], &acc[b], &off[b]);
}

/* Bytes of one GGUF block of the down tensor's type (12: Q4_K, 14: Q6_K; 0 = unsupported). */
static size_t orc_block_bytes(uint32_t type) { return type == 12u ? sizeof(orc_q4k) : type == 14u ? sizeof(orc_q6k) : 0; }

/* Gate + Up + SwiGLU + Q8_K of h, tools/lfm2_decode_1x4.c:963-1065:
 * h = (g / (1 + expf(-g))) * u; then h quantised per 256. */
static void orc_swiglu(int order, const orc_q4k *gate, const orc_q4k *up, uint32_t D, uint32_t I,
                       const orc_q8k *xq, float *h, orc_q8k *hq) {
    const uint32_t nb = D / 256;
    for (uint32_t r = 0; r < I; ++r) {
        const float g = orc_q4k_row(order, gate + (size_t)r * nb, xq, nb);
        const float u = orc_q4k_row(order, up + (size_t)r * nb, xq, nb);
        h[r] = (g / (1.0f + expf(-g))) * u;
    }
    orc_quantize_q8k(h, hq, I);
}

/*
 * Full lfm2moe FFN for T tokens, one token at a time exactly as
 * lfm2_forward_moe_ffn_1x4 (tools/lfm2_moe_checkpoint.c:312-365):
 *   RMSNorm+Q8_K, route, then for k = 0..K-1 in order:
 *   h = SwiGLU(gate_e x, up_e x) -> Q8_K, x[r] = fma(w_k, down_e[r] . h, x[r]).
 * Expert tensors are GGUF 3-D [E][rows][cols/256]: gate/up Q4_K, down Q4_K
 * (down_type 12) or Q6_K (14, as Q4_K_M checkpoints store some ffn_down_exps,
 * tools/lfm2_decode_1x4.c:618-630 selects the kernel by type).  Optional outputs:
 * idx/w [T*K], xq [T*D/256] (Q8_K of the normalised input), h [T*K*I].
 * Returns 0, or -1 on a shape it does not support.
 */
ORC_EXPORT int orc_moe_forward(int order, float *x, uint32_t T, uint32_t D, uint32_t E, uint32_t K,
                               uint32_t I, float eps, const float *ffn_norm, const float *router_w,
                               const float *bias, const void *gate, const void *up, const void *down,
                               uint32_t down_type, int norm_topk, float routed_scale, uint32_t *idx_out,
                               float *w_out, void *xq_out, float *h_out) {
    if (D % 256 || I % 256 || E == 0 || E > 256 || K == 0 || K > E || K > 8) return -1;
    const size_t dn_bytes = orc_block_bytes(down_type);
    if (!dn_bytes) return -1;
    const uint32_t nbd = D / 256, nbi = I / 256;
    float *xb = (float *)malloc(sizeof(float) * D);
    float *h = (float *)malloc(sizeof(float) * I);
    float *dn = (float *)malloc(sizeof(float) * D);
    orc_q8k *xq = (orc_q8k *)malloc(sizeof(orc_q8k) * (nbd + nbi));
    if (!xb || !h || !dn || !xq) { free(xb); free(h); free(dn); free(xq); return -2; }
    const orc_q4k *G = (const orc_q4k *)gate, *U = (const orc_q4k *)up;
    const uint8_t *Dn = (const uint8_t *)down;
    for (uint32_t t = 0; t < T; ++t) {
        float *xt = x + (size_t)t * D;
        orc_rmsnorm_q8k(xt, ffn_norm, D, eps, xb, xq);
        if (xq_out) memcpy((orc_q8k *)xq_out + (size_t)t * nbd, xq, sizeof(orc_q8k) * nbd);
        uint32_t idx[8];
        float w[8];
        orc_route(router_w, bias, xb, D, E, K, norm_topk, routed_scale, idx, w, NULL, NULL);
        for (uint32_t k = 0; k < K; ++k) {
            const uint32_t e = idx[k];
            if (idx_out) idx_out[(size_t)t * K + k] = e;
            if (w_out) w_out[(size_t)t * K + k] = w[k];
            orc_swiglu(order, G + (size_t)e * I * nbd, U + (size_t)e * I * nbd, D, I, xq, h, xq + nbd);
            if (h_out) memcpy(h_out + ((size_t)t * K + k) * I, h, sizeof(float) * I);
            const uint8_t *De = Dn + (size_t)e * D * nbi * dn_bytes;
            if (down_type == 14u) orc_q6k_rows(order, De, I, 0, D, xq + nbd, dn);
            else orc_q4k_rows(order, De, I, 0, D, xq + nbd, dn);
            for (uint32_t r = 0; r < D; ++r) xt[r] = fmaf(w[k], dn[r], xt[r]);
        }
    }
    free(xb); free(h); free(dn); free(xq);
    return 0;
}

/* Expert-parallel pieces (for the host-logic tests of expert parallelism):
 * rows a = 0..n-1, each one (token, k) assignment given as its Q8_K blocks
 * xq[a][D/256] and its expert ids[a] (0-based within gate/up/down, which hold
 * the shard's experts): y[a] = Down_e(Q8_K(SwiGLU(Gate_e xq, Up_e xq))),
 * unweighted -- the inner loop of orc_moe_forward
 * (tools/lfm2_moe_checkpoint.c:338-363). */
ORC_EXPORT int orc_expert_rows(int order, uint32_t D, uint32_t I, const void *gate, const void *up,
                               const void *down, const void *xq_rows, const uint32_t *ids, uint32_t n,
                               float *y) {
    if (D % 256 || I % 256) return -1;
    const uint32_t nbd = D / 256, nbi = I / 256;
    float *h = (float *)malloc(sizeof(float) * I);
    orc_q8k *hq = (orc_q8k *)malloc(sizeof(orc_q8k) * nbi);
    if (!h || !hq) { free(h); free(hq); return -2; }
    const orc_q4k *G = (const orc_q4k *)gate, *U = (const orc_q4k *)up, *Dn = (const orc_q4k *)down;
    const orc_q8k *X = (const orc_q8k *)xq_rows;
    for (uint32_t a = 0; a < n; ++a) {
        const uint32_t e = ids[a];
        orc_swiglu(order, G + (size_t)e * I * nbd, U + (size_t)e * I * nbd, D, I, X + (size_t)a * nbd, h, hq);
        orc_q4k_rows(order, Dn + (size_t)e * D * nbi, I, 0, D, hq, y + (size_t)a * D);
    }
    free(h); free(hq);
    return 0;
}

/* x[t][r] = fmaf(w[t][k], y[t*K+k][r], x[t][r]) for k = 0..K-1 in order
 * (tools/lfm2_moe_checkpoint.c:266-269). */
ORC_EXPORT void orc_ep_combine(float *x, uint32_t T, uint32_t D, uint32_t K, const float *w, const float *y) {
    for (uint32_t t = 0; t < T; ++t)
        for (uint32_t k = 0; k < K; ++k)
            for (uint32_t r = 0; r < D; ++r)
                x[(size_t)t * D + r] = fmaf(w[(size_t)t * K + k], y[((size_t)t * K + k) * D + r], x[(size_t)t * D + r]);
}

/* Dense SwiGLU FFN (leading layers of an lfm2moe stack), tools/lfm2_decode_1x4.c:
 * 1070-1104: RMSNorm+Q8_K, SwiGLU -> Q8_K, down, then x[r] = x[r] + down[r]. */
ORC_EXPORT int orc_dense_ffn_forward(int order, float *x, uint32_t T, uint32_t D, uint32_t I, float eps,
                                     const float *ffn_norm, const void *gate, const void *up,
                                     const void *down) {
    if (D % 256 || I % 256) return -1;
    const uint32_t nbd = D / 256, nbi = I / 256;
    float *xb = (float *)malloc(sizeof(float) * D);
    float *h = (float *)malloc(sizeof(float) * I);
    float *dn = (float *)malloc(sizeof(float) * D);
    orc_q8k *xq = (orc_q8k *)malloc(sizeof(orc_q8k) * (nbd + nbi));
    if (!xb || !h || !dn || !xq) { free(xb); free(h); free(dn); free(xq); return -2; }
    for (uint32_t t = 0; t < T; ++t) {
        float *xt = x + (size_t)t * D;
        orc_rmsnorm_q8k(xt, ffn_norm, D, eps, xb, xq);
        orc_swiglu(order, (const orc_q4k *)gate, (const orc_q4k *)up, D, I, xq, h, xq + nbd);
        orc_q4k_rows(order, down, I, 0, D, xq + nbd, dn);
        for (uint32_t r = 0; r < D; ++r) xt[r] = xt[r] + dn[r];
    }
    free(xb); free(h); free(dn); free(xq);
    return 0;
}

/* Known-answer inputs of the reference's own tests, rebuilt exactly (same
 * float expressions) so the golden fixtures can pin the oracle to them:
 *  - router test, tests/test_moe_checkpoint.c:146-159 (xb, router weights,
 *    exp_probs_b with experts 9 and 25 forced to win);
 *  - Q8_K test, tests/test_cpuid_quants.c:80-82. */
ORC_EXPORT void orc_kat_router_inputs(float *xb, float *gate_inp, float *bias, uint32_t D, uint32_t E) {
    for (uint32_t i = 0; i < D; ++i) xb[i] = cosf((float)i * 0.013f);
    for (uint32_t e = 0; e < E; ++e) {
        bias[e] = (float)(e % 5) * 0.15f - 0.2f;
        for (uint32_t i = 0; i < D; ++i) gate_inp[(size_t)e * D + i] = sinf((float)(e * 17 + i) * 0.007f) * 0.04f;
    }
    if (E > 25) { bias[9] = 2.5f; bias[25] = 3.0f; }
}

ORC_EXPORT void orc_kat_q8k_inputs(float *x, uint32_t n) {
    for (uint32_t i = 0; i < n; ++i) x[i] = sinf((float)i * 0.031f) * ((i % 2 == 0) ? 2.5f : -1.8f);
}
