/*
 * Prefill: grouped Q4_K x Q8_K GEMM on the tensor cores (mma.sync IMMA,
 * m16n8k32, u8 x s8 -> s32), for T large enough that every active expert sees
 * tens of tokens.  The decode GEMV streams a weight row once per 8-token
 * pair; here a CTA keeps a 64-row weight tile and 128 tokens of one expert and
 * walks K one Q4_K super-block at a time.
 *
 * Exact integer super-block sums on the tensor cores.  For row r, token t,
 * super-block b the reference forms (tools/lfm2_cpuid_quants.c:421-457):
 *   acc  = sum_j sc_j * sum_{l<32} q4[32j+l] * q8[32j+l]
 *   mins = sum_j m_j  * (bsum[2j] + bsum[2j+1]) = sum_j m_j * sum_{l<32} q8[32j+l]
 * (the Q8_K codes never saturate, so the bsums are the sums of the codes).
 * With sc_j = 16*a_j + b_j (a_j <= 3, b_j <= 15) the operands
 *   A1 = b_j * q4 <= 225,  A2 = a_j * q4 <= 45,  A3 = m_j <= 63
 * fit unsigned 8 bits, so per k-step (= one 32-wide sub-block j)
 *   P = 16 * (A2 . X) + (A1 . X) = acc      (the A2 products, scaled, then A1 accumulated on top)
 *   Q = A3 . X                    = mins
 * are plain IMMA accumulations, exact in int32.  The fp32 update then follows
 * the reference's 4-row AVX-VNNI kernel per super-block, in order
 * (tools/lfm2_cpuid_quants.c:1189-1257):
 *   S = fma(d8*d, (float)acc, fma(-(d8*dmin), (float)mins, S)),  skipped when d8 == 0.
 *
 * CTA: 8 warps as 2 x 4, warp tile 32 rows x 32 tokens (2 x 4 m16n8 tiles).
 * Per super-block: the raw Q4_K rows and the tokens' Q8_K codes and scales
 * arrive by cp.async (double buffered); the CTA expands the nibbles into A1 and
 * A2 (row stride 272 bytes: ldmatrix conflict-free); warps load fragments with
 * ldmatrix and run 2*4*8*3 IMMAs, then the fp32 update.  Output: Y[slot][row]
 * fp32 for the tile's rows and tokens.
 *
 * Tiles come from a plan (k_gemm_plan): for every active expert, its 64-row
 * blocks x its 128-token blocks (tokens fastest, so the CTAs working on one
 * weight block run together and share it through L2).
 */
#include "moe_device.cuh"
#include "moe_internal.h"

namespace {

constexpr int kRowsT = 64;        /* weight rows per CTA tile */
constexpr int kTokT = 128;        /* tokens (dispatch slots) per CTA tile */
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kArow = 272;        /* bytes per expanded weight row / staged token row (256 + 16) */
constexpr int kWrow = LFM_Q4K_BYTES;

/* one stage: raw Q4_K rows, token codes, token scales */
constexpr int kStageW = kRowsT * kWrow;            /* 9216 */
constexpr int kStageX = kTokT * kArow;             /* 34816 */
constexpr int kStageD = kTokT * 4;                 /* 512 */
constexpr int kStage = kStageW + kStageX + kStageD;
constexpr int kAbytes = kRowsT * kArow;            /* 17408 each for A1, A2 */
constexpr int kSmem = 2 * kStage + 2 * kAbytes + kRowsT * 16;

struct GemmTile {
    int expert;  /* index into the expert tensors */
    int slot0;   /* first dispatch slot of the token block */
    int ntok;    /* tokens in the block (<= kTokT) */
    int row0;    /* first weight row */
};

struct GemmArgs {
    const uint8_t *W;    /* expert tensors [E][rows][nb] Q4_K */
    uint32_t rows;       /* rows per expert */
    uint32_t nb;         /* super-blocks per row */
    Q8Rows X;            /* activations: row of slot s is X row (tok_of_slot ? perm[s]/K : s) */
    const int32_t *perm; /* dispatch permutation (slot -> assignment), or NULL for slot-indexed X */
    uint32_t K;
    const GemmTile *tiles;
    const int32_t *n_tiles;
    float *Y;            /* [slots][rows] */
    uint32_t *err;
};

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(lfm_smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(lfm_smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(lfm_smem_u32(p)));
}

__device__ __forceinline__ void imma(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

/* Issue the cp.async copies of super-block b of a tile into stage `st`. */
__device__ __forceinline__ void load_stage(const GemmArgs &A, const GemmTile &tl, uint32_t b, uint8_t *st,
                                           const int *xrow) {
    uint8_t *sw = st, *sx = st + kStageW;
    float *sd = reinterpret_cast<float *>(st + kStageW + kStageX);
    const uint32_t row_bytes = A.nb * kWrow;
    const uint8_t *wsrc = A.W + ((size_t)tl.expert * A.rows + tl.row0) * row_bytes + (size_t)b * kWrow;
    /* weights: 64 rows x 144 bytes = 9 x 16-byte pieces per row */
    for (int q = threadIdx.x; q < kRowsT * 9; q += kThreads) {
        const int r = q / 9, c = q - r * 9;
        cp_async16(sw + r * kWrow + 16 * c, wsrc + (size_t)r * row_bytes + 16 * c);
    }
    /* token codes: 128 rows x 256 bytes (rows beyond ntok copy token 0's: never used) */
    for (int q = threadIdx.x; q < kTokT * 16; q += kThreads) {
        const int t = q >> 4, c = q & 15;
        cp_async16(sx + t * kArow + 16 * c, A.X.qs + (size_t)xrow[t] * A.X.cols + 256 * b + 16 * c);
    }
    for (int t = threadIdx.x; t < kTokT; t += kThreads) cp_async4(sd + t, A.X.d + (size_t)xrow[t] * A.nb + b);
}

__global__ void __launch_bounds__(kThreads, 1) k_q4k_gemm(GemmArgs A) {
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ int xrow[kTokT];
    uint8_t *stage[2] = {sm, sm + kStage};
    uint8_t *A1 = sm + 2 * kStage, *A2 = A1 + kAbytes;
    uint8_t *rowinfo = A2 + kAbytes; /* per row: d, dmin (floats), m bytes (2 words) */
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wm = warp >> 2, wn = warp & 3;  /* warp tile: rows 32*wm.., tokens 32*wn.. */
    const int gid = lane >> 2, tig = lane & 3;
    const int n_tiles = __ldcg(A.n_tiles);

    for (int ti = blockIdx.x; ti < n_tiles; ti += gridDim.x) {
        const GemmTile tl = A.tiles[ti];
        __syncthreads(); /* the previous tile is done with xrow and the stages */
        for (int t = threadIdx.x; t < kTokT; t += kThreads) {
            const int s = tl.slot0 + (t < tl.ntok ? t : 0);
            xrow[t] = A.perm ? __ldcg(A.perm + s) / (int)A.K : s;
        }
        __syncthreads();
        float S[2][4][4];
#pragma unroll
        for (int mi = 0; mi < 2; ++mi)
#pragma unroll
            for (int ni = 0; ni < 4; ++ni)
#pragma unroll
                for (int v = 0; v < 4; ++v) S[mi][ni][v] = 0.0f;

        load_stage(A, tl, 0, stage[0], xrow);
        cp_commit();
        for (uint32_t b = 0; b < A.nb; ++b) {
            uint8_t *st = stage[b & 1];
            if (b + 1 < A.nb) load_stage(A, tl, b + 1, stage[(b + 1) & 1], xrow);
            cp_commit();
            cp_wait<1>();
            __syncthreads(); /* stage b landed for every thread */

            /* expand the 64 Q4_K rows into A1 = b_j*q4 and A2 = a_j*q4 (row-major, 272-byte rows) */
            const uint8_t *sw = st;
            for (int q = threadIdx.x; q < kRowsT * 32; q += kThreads) {
                const int r = q >> 5, w = q & 31;      /* word w of the 128 nibble bytes */
                const uint8_t *blk = sw + r * kWrow;
                const uint32_t v = *reinterpret_cast<const uint32_t *>(blk + 16 + 4 * w);
                const int c = w >> 3, l4 = (w & 7) * 4; /* group c, bytes l4..l4+3 of its 32 */
                const uint32_t s0 = *reinterpret_cast<const uint32_t *>(blk + 4);
                const uint32_t s2 = *reinterpret_cast<const uint32_t *>(blk + 12);
                const uint32_t scA = s0 & 0x3F3F3F3Fu;
                const uint32_t scB = (s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u);
                const uint32_t scw = c < 2 ? scA : scB;
                const uint32_t sc_lo = (scw >> (16 * (c & 1))) & 0xFFu, sc_hi = (scw >> (16 * (c & 1) + 8)) & 0xFFu;
                const uint32_t lo = v & 0x0F0F0F0Fu, hi = (v >> 4) & 0x0F0F0F0Fu;
                /* bytes of a nibble word times a scalar <= 15 stay below 256: no carries */
                uint8_t *a1 = A1 + r * kArow, *a2 = A2 + r * kArow;
                *reinterpret_cast<uint32_t *>(a1 + 64 * c + l4) = lo * (sc_lo & 15u);
                *reinterpret_cast<uint32_t *>(a1 + 64 * c + 32 + l4) = hi * (sc_hi & 15u);
                *reinterpret_cast<uint32_t *>(a2 + 64 * c + l4) = lo * (sc_lo >> 4);
                *reinterpret_cast<uint32_t *>(a2 + 64 * c + 32 + l4) = hi * (sc_hi >> 4);
            }
            for (int r = threadIdx.x; r < kRowsT; r += kThreads) {
                const uint8_t *blk = sw + r * kWrow;
                const uint32_t hdr = *reinterpret_cast<const uint32_t *>(blk);
                const uint32_t s0 = *reinterpret_cast<const uint32_t *>(blk + 4);
                const uint32_t s1 = *reinterpret_cast<const uint32_t *>(blk + 8);
                const uint32_t s2 = *reinterpret_cast<const uint32_t *>(blk + 12);
                float *ri = reinterpret_cast<float *>(rowinfo + r * 16);
                ri[0] = lfm_h2f((uint16_t)(hdr & 0xFFFFu));
                ri[1] = lfm_h2f((uint16_t)(hdr >> 16));
                uint32_t *mi = reinterpret_cast<uint32_t *>(rowinfo + r * 16 + 8);
                mi[0] = s1 & 0x3F3F3F3Fu;                                        /* m0..m3 */
                mi[1] = ((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u);   /* m4..m7 */
                (void)s0;
            }
            __syncthreads(); /* A1, A2, row info ready */

            const uint8_t *sx = st + kStageW;
            const float *sd = reinterpret_cast<const float *>(st + kStageW + kStageX);
            int P[2][4][4], Q[2][4][4];
#pragma unroll
            for (int mi = 0; mi < 2; ++mi)
#pragma unroll
                for (int ni = 0; ni < 4; ++ni)
#pragma unroll
                    for (int v = 0; v < 4; ++v) { P[mi][ni][v] = 0; Q[mi][ni][v] = 0; }
            /* ldmatrix row addresses: lane l -> row (l & 15), 16-byte half (l >> 4) of a 32-byte k-step */
            const int lr = lane & 15, lh = lane >> 4;
            /* pass 0: A2 (scaled by 16 afterwards) and A3 (mins); pass 1: A1 */
#pragma unroll 1
            for (int pass = 0; pass < 2; ++pass) {
                const uint8_t *Aop = pass == 0 ? A2 : A1;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    uint32_t af[2][4];
#pragma unroll
                    for (int mi = 0; mi < 2; ++mi)
                        ldsm_x4(af[mi], Aop + (32 * wm + 16 * mi + lr) * kArow + 32 * j + 16 * lh);
                    /* matrices: (rows 0-7, k 0-15), (rows 8-15, k 0-15), (rows 0-7, k 16-31), (rows 8-15, k 16-31)
                     * -> exactly a0, a1, a2, a3 of the IMMA A fragment */
                    uint32_t bf[4][2];
#pragma unroll
                    for (int np = 0; np < 2; ++np) {
                        uint32_t r4[4];
                        /* tokens 16*np + (l & 15) of the warp's 32, k half (l >> 4) */
                        ldsm_x4(r4, sx + (32 * wn + 16 * np + lr) * kArow + 32 * j + 16 * lh);
                        /* r4: (tok 0-7, k0-15), (tok 8-15, k0-15), (tok 0-7, k16-31), (tok 8-15, k16-31) */
                        bf[2 * np][0] = r4[0];
                        bf[2 * np][1] = r4[2];
                        bf[2 * np + 1][0] = r4[1];
                        bf[2 * np + 1][1] = r4[3];
                    }
#pragma unroll
                    for (int mi = 0; mi < 2; ++mi) {
                        const uint32_t a[4] = {af[mi][0], af[mi][1], af[mi][2], af[mi][3]};
#pragma unroll
                        for (int ni = 0; ni < 4; ++ni) imma(P[mi][ni], a, bf[ni][0], bf[ni][1]);
                    }
                    if (pass == 0) {
                        /* A3: m_j of each row, replicated in all 4 bytes */
#pragma unroll
                        for (int mi = 0; mi < 2; ++mi) {
                            const int r0 = 32 * wm + 16 * mi + gid;
                            const uint32_t m0 = (reinterpret_cast<const uint32_t *>(rowinfo + r0 * 16 + 8)[j >> 2] >> (8 * (j & 3))) & 0xFFu;
                            const uint32_t m1 = (reinterpret_cast<const uint32_t *>(rowinfo + (r0 + 8) * 16 + 8)[j >> 2] >> (8 * (j & 3))) & 0xFFu;
                            const uint32_t a[4] = {m0 * 0x01010101u, m1 * 0x01010101u, m0 * 0x01010101u, m1 * 0x01010101u};
#pragma unroll
                            for (int ni = 0; ni < 4; ++ni) imma(Q[mi][ni], a, bf[ni][0], bf[ni][1]);
                        }
                    }
                }
                if (pass == 0) {
#pragma unroll
                    for (int mi = 0; mi < 2; ++mi)
#pragma unroll
                        for (int ni = 0; ni < 4; ++ni)
#pragma unroll
                            for (int v = 0; v < 4; ++v) P[mi][ni][v] *= 16;
                }
            }
            /* fp32 update of the reference, super-block b, for the warp's 32 x 32 (row, token) */
#pragma unroll
            for (int mi = 0; mi < 2; ++mi) {
#pragma unroll
                for (int hr = 0; hr < 2; ++hr) {
                    const int r = 32 * wm + 16 * mi + gid + 8 * hr;
                    const float d = reinterpret_cast<const float *>(rowinfo + r * 16)[0];
                    const float dmin = reinterpret_cast<const float *>(rowinfo + r * 16)[1];
#pragma unroll
                    for (int ni = 0; ni < 4; ++ni) {
#pragma unroll
                        for (int c = 0; c < 2; ++c) {
                            const int t = 32 * wn + 8 * ni + 2 * tig + c;
                            const float d8 = sd[t];
                            const int v = 2 * hr + c;
                            if (d8 != 0.0f)
                                S[mi][ni][v] = __fmaf_rn(__fmul_rn(d8, d), (float)P[mi][ni][v],
                                                         __fmaf_rn(-__fmul_rn(d8, dmin), (float)Q[mi][ni][v], S[mi][ni][v]));
                        }
                    }
                }
            }
            __syncthreads(); /* A1/A2/row info and stage b free for reuse */
        }
        /* Y[slot][row] for the tile's valid tokens */
#pragma unroll
        for (int mi = 0; mi < 2; ++mi)
#pragma unroll
            for (int hr = 0; hr < 2; ++hr) {
                const int r = 32 * wm + 16 * mi + gid + 8 * hr;
#pragma unroll
                for (int ni = 0; ni < 4; ++ni)
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        const int t = 32 * wn + 8 * ni + 2 * tig + c;
                        if (t < tl.ntok) A.Y[(size_t)(tl.slot0 + t) * A.rows + tl.row0 + r] = S[mi][ni][2 * hr + c];
                    }
            }
    }
}

/* Tile plan from the dispatch tables: every active expert's 64-row blocks x its
 * 128-token blocks.  One block; writes n_tiles and the tiles. */
__global__ void k_gemm_plan(RouteTables rt, uint32_t rows, GemmTile *tiles, int32_t *n_tiles, uint32_t max_tiles) {
    __shared__ int s_base[LFM_GPU_MAX_EXPERTS_DEV + 1];
    __shared__ int s_e[LFM_GPU_MAX_EXPERTS_DEV], s_cnt[LFM_GPU_MAX_EXPERTS_DEV], s_off[LFM_GPU_MAX_EXPERTS_DEV];
    const int U = __ldcg(rt.summary + 0);
    const int nrb = (int)rows / kRowsT;
    for (int u = threadIdx.x; u < U; u += blockDim.x) {
        const int e = __ldcg(rt.act + u);
        s_e[u] = e;
        s_cnt[u] = __ldcg(rt.counts + e);
        s_off[u] = __ldcg(rt.offsets + e);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int acc = 0;
        for (int u = 0; u < U; ++u) {
            s_base[u] = acc;
            acc += nrb * ((s_cnt[u] + kTokT - 1) / kTokT);
        }
        s_base[U] = acc;
        if ((uint32_t)acc > max_tiles) { atomicOr(rt.err, LFM_DEVERR_SEGMENT); acc = 0; }
        *n_tiles = acc;
    }
    __syncthreads();
    if ((uint32_t)s_base[U] > max_tiles) return;
    for (int u = 0; u < U; ++u) {
        const int e = s_e[u];
        const int cnt = s_cnt[u], off = s_off[u];
        const int ntb = (cnt + kTokT - 1) / kTokT;
        for (int q = threadIdx.x; q < nrb * ntb; q += blockDim.x) {
            const int rb = q / ntb, tb = q - rb * ntb;
            tiles[s_base[u] + q] = GemmTile{e, off + tb * kTokT, min(kTokT, cnt - tb * kTokT), rb * kRowsT};
        }
    }
}

/* h = (g / (1 + exp(-g))) * u, then Q8_K per 256 (tools/lfm2_decode_1x4.c:976-997);
 * one warp per 256-element block of a slot row. */
__global__ void __launch_bounds__(256) k_swiglu_quant(const float *__restrict__ G, const float *__restrict__ U,
                                                      uint32_t rows, uint32_t cols, Q8Rows dst) {
    const uint32_t nb = cols / 256;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t gw = blockIdx.x * 8 + warp;
    if (gw >= rows * nb) return;
    const uint32_t r = gw / nb, b = gw % nb;
    const size_t o = (size_t)r * cols + 256 * b + 8 * lane;
    const float4 g0 = __ldcg(reinterpret_cast<const float4 *>(G + o)), g1 = __ldcg(reinterpret_cast<const float4 *>(G + o) + 1);
    const float4 u0 = __ldcg(reinterpret_cast<const float4 *>(U + o)), u1 = __ldcg(reinterpret_cast<const float4 *>(U + o) + 1);
    const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    const float u[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(__fdiv_rn(g[i], __fadd_rn(1.0f, lfm_silu_expf(-g[i]))), u[i]);
    lfm_quant_block_warp(v, dst, r, b);
}

}  // namespace

size_t lfm_gemm_tiles_max(uint32_t rows, uint32_t slots, uint32_t experts) {
    return (size_t)(rows / kRowsT) * ((slots + kTokT - 1) / kTokT + experts);
}

cudaError_t lfm_launch_gemm_plan(const RouteTables &rt, uint32_t rows, void *tiles, int32_t *n_tiles,
                                 uint32_t max_tiles, cudaStream_t s) {
    k_gemm_plan<<<1, 256, 0, s>>>(rt, rows, static_cast<GemmTile *>(tiles), n_tiles, max_tiles);
    return cudaGetLastError();
}

size_t lfm_gemm_tile_bytes() { return sizeof(GemmTile); }

cudaError_t lfm_launch_q4k_gemm(const uint8_t *W, uint32_t rows, uint32_t cols, Q8Rows X, const int32_t *perm,
                                uint32_t K, const void *tiles, const int32_t *n_tiles, float *Y, uint32_t *err,
                                int grid, cudaStream_t s) {
    if (rows % kRowsT || cols % 256) return cudaErrorInvalidValue;
    static size_t cache[16];
    cudaError_t e = lfm_smem_attr((const void *)k_q4k_gemm, kSmem, cache);
    if (e != cudaSuccess) return e;
    GemmArgs a{W, rows, cols / 256, X, perm, K, static_cast<const GemmTile *>(tiles), n_tiles, Y, err};
    k_q4k_gemm<<<grid, kThreads, kSmem, s>>>(a);
    return cudaGetLastError();
}

cudaError_t lfm_launch_swiglu_quant(const float *G, const float *U, uint32_t rows, uint32_t cols, Q8Rows dst,
                                    cudaStream_t s) {
    const uint32_t warps = rows * (cols / 256);
    if (warps == 0) return cudaSuccess;
    k_swiglu_quant<<<(warps + 7) / 8, 256, 0, s>>>(G, U, rows, cols, dst);
    return cudaGetLastError();
}
