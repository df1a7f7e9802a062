/*
 * Prefill: grouped Q4_K x Q8_K GEMM on the 5th-generation tensor cores
 * (tcgen05.mma kind::i8, u8 x s8 -> s32, accumulators in tensor memory).
 *
 * Exact integer super-block sums.  For row r, token t, super-block b the
 * reference forms (tools/lfm2_cpuid_quants.c:421-457)
 *   acc  = sum_j sc_j * sum_{l<32} q4[32j+l] * q8[32j+l]
 *   mins = sum_j m_j  * (bsum[2j] + bsum[2j+1])
 * With sc_j = 16*a_j + b_j (a_j <= 3, b_j <= 15) the expanded weights
 *   A1 = b_j * q4 <= 225,  A2 = a_j * q4 <= 45     (unsigned bytes)
 * give acc = D1 + 16*D2 with D1 = A1 . X and D2 = A2 . X accumulated over the
 * whole super-block (K = 256) by the tensor core, exact in int32.  mins is
 * four dp2a per (row, token) from the tokens' sub-block sums.  The fp32 update
 * is the reference's, per super-block in order (tools/lfm2_cpuid_quants.c:1189-1257):
 *   S = fma(d8*d, (float)acc, fma(-(d8*dmin), (float)mins, S)),  skipped when d8 == 0.
 *
 * Tile: 128 weight rows (MMA M) x 128 tokens (MMA N) of one expert; K walked
 * in half super-blocks (128 bytes).  One CTA per SM, persistent over the tile
 * list, warp-specialised:
 *   warps 0-7   epilogue: TMEM -> registers (tcgen05.ld 32x32b), the fp32
 *               update above into 64 running sums per thread (thread = row,
 *               warp pair = the tile's two 64-token halves), Y at the end;
 *   warps 8-11  producers: thread p owns weight row p; its Q4_K bytes arrive
 *               by a 144-byte bulk copy per super-block (ring of 3), it expands
 *               the nibbles into A1/A2 in the UMMA canonical K-major layout
 *               (8-row x 16-byte core matrices) and publishes d, dmin, m_j;
 *   warp 12     TMEM allocation and the MMA issue (one thread): per half
 *               super-block 4 K-steps x (A1 -> D1, A2 -> D2), commits release
 *               the shared-memory stages and hand a finished accumulator pair
 *               to the epilogue.  D1/D2 are double buffered (2 x 256 columns),
 *               so super-block b+1 multiplies while b drains;
 *   warp 13     loader (one thread): the tokens' codes and scales for each
 *               half super-block, pre-gathered by k_xt_gather into the same
 *               canonical layout, one bulk copy each.
 * Every mbarrier wait is bounded; on a timeout the CTA raises the device error
 * word, every role leaves its loop, the CTA waits out copies and MMAs in
 * flight and frees its tensor memory before it exits.
 */
#include "moe_device.cuh"
#include "moe_internal.h"

namespace {

constexpr int kM = 128;                      /* weight rows per tile (MMA M)               */
constexpr int kN = 128;                      /* tokens per tile (MMA N)                    */
constexpr int kHalf = 128;                   /* K bytes per stage: half a super-block      */
constexpr int kCoreK = kM * 16;              /* bytes between K-adjacent core matrices     */
constexpr int kOp = kM * kHalf;              /* 16384: one operand stage (A1, A2 or B)     */
constexpr int kTokInfo = kN * 4 + kN * 16;   /* d8[128] fp32 + sub-block bsum pairs [128][4] */
constexpr int kXtSb = 2 * kOp + kTokInfo;    /* pre-gathered tokens per (block, super-block) */
constexpr int kRaw = LFM_Q4K_BYTES;
constexpr int kRawSlot = kM * kRaw;
constexpr int kRowInfo = kM * 16;            /* d, dmin, m0..3, m4..7 per row              */
constexpr int kSA = 3;                       /* A1/A2 and B stages                         */
constexpr int kSR = 3;                       /* raw weight ring (super-blocks)             */
constexpr int kEpiWarps = 8, kProdWarps = 4;
constexpr int kWarpMma = kEpiWarps + kProdWarps;
constexpr int kWarpLoad = kWarpMma + 1;
constexpr int kThreads = (kWarpLoad + 1) * 32;
constexpr uint32_t kTmemCols = 512;

constexpr int kOffA = 0;
constexpr int kOffB = kOffA + kSA * 2 * kOp;
constexpr int kOffR = kOffB + kSA * kOp;
constexpr int kOffT = kOffR + kSR * kRawSlot;
constexpr int kOffW = kOffT + 2 * kTokInfo;
constexpr int kSmem = kOffW + 2 * kRowInfo;
static_assert(kSmem <= 227 * 1024, "shared memory");

/* Instruction descriptor, kind::i8: D s32 (bits 4-5 = 2), A u8 (7-9 = 0),
 * B s8 (10-12 = 1), both K-major, N >> 3 at bits 17-22, M >> 4 at 24-28. */
constexpr uint32_t kIdesc = (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(kN >> 3) << 17) |
                            ((uint32_t)(kM >> 4) << 24);

struct UTile {
    int32_t expert, tb, row0, pad;
};
struct UTokBlock {
    int32_t slot0, ntok;
};

struct UmmaArgs {
    const uint8_t *W;     /* expert tensors [E][rows][nb] Q4_K */
    uint32_t rows, nb;
    const uint8_t *xt;    /* pre-gathered tokens [block][nb][kXtSb] */
    const UTile *tiles;
    const UTokBlock *tbs;
    const int32_t *n_tiles;
    float *Y;             /* [slots][rows] */
    uint32_t *err;
};

struct UmmaBars {
    uint64_t a_full[kSA], a_empty[kSA], b_full[kSA], b_empty[kSA], r_full[kSR];
    uint64_t t_full[2], t_empty[2], ti_full[2], ri_full[2], i_empty[2];
    uint32_t tmem;
    int abort;
};

/* Shared-memory matrix descriptor, K-major without swizzle: start address,
 * leading byte offset (K-adjacent core matrices) = kCoreK, stride byte offset
 * (8-row groups) = 128, version 1 at bit 46. */
__device__ __forceinline__ uint64_t udesc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(kCoreK >> 4) << 16) | ((uint64_t)(128 >> 4) << 32) |
           (1ull << 46);
}

__device__ __forceinline__ void umma_i8(uint32_t d, uint64_t a, uint64_t b, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     lfm_smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(lfm_smem_u32(dst)),
                 "r"(cols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

/* 16 consecutive 32-bit columns of this thread's TMEM lane. */
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}
/* Wait for this thread's TMEM loads; the registers are tied to the wait so no
 * use of them is scheduled before it. */
__device__ __forceinline__ void tmem_wait(uint32_t (&a)[16], uint32_t (&b)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]),
                   "+r"(a[8]), "+r"(a[9]), "+r"(a[10]), "+r"(a[11]), "+r"(a[12]), "+r"(a[13]), "+r"(a[14]),
                   "+r"(a[15])::"memory");
    asm volatile(""
                 : "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7]),
                   "+r"(b[8]), "+r"(b[9]), "+r"(b[10]), "+r"(b[11]), "+r"(b[12]), "+r"(b[13]), "+r"(b[14]),
                   "+r"(b[15])::"memory");
}

__device__ __forceinline__ void sts128(uint8_t *p, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(lfm_smem_u32(p)), "r"(x), "r"(y), "r"(z), "r"(w)
                 : "memory");
}

/* Bounded wait that also gives up once another role has aborted. */
__device__ __forceinline__ bool uwait(uint64_t *bar, uint32_t parity, volatile int *abort, uint32_t *err) {
    if (lfm_mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = lfm_globaltimer();
    while (!lfm_mbar_try_wait(bar, parity)) {
        if (*abort) return false;
        if (lfm_globaltimer() - t0 > LFM_WAIT_LIMIT_NS) {
            atomicOr(err, LFM_DEVERR_TIMEOUT);
            *abort = 1;
            return false;
        }
    }
    return true;
}

__global__ void __launch_bounds__(kThreads, 1) k_q4k_umma(UmmaArgs A) {
    extern __shared__ __align__(1024) uint8_t sm[];
    __shared__ UmmaBars bars;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int i = 0; i < kSA; ++i) {
            lfm_mbar_init(&bars.a_full[i], kProdWarps * 32);
            lfm_mbar_init(&bars.a_empty[i], 1);
            lfm_mbar_init(&bars.b_full[i], 1);
            lfm_mbar_init(&bars.b_empty[i], 1);
        }
        for (int i = 0; i < kSR; ++i) lfm_mbar_init(&bars.r_full[i], kProdWarps * 32);
        for (int i = 0; i < 2; ++i) {
            lfm_mbar_init(&bars.t_full[i], 1);
            lfm_mbar_init(&bars.t_empty[i], kEpiWarps);
            lfm_mbar_init(&bars.ti_full[i], 1);
            lfm_mbar_init(&bars.ri_full[i], kProdWarps * 32);
            lfm_mbar_init(&bars.i_empty[i], kEpiWarps);
        }
        bars.abort = 0;
        lfm_fence_mbar_init();
    }
    if (warp == kWarpMma) {
        tmem_alloc(&bars.tmem, kTmemCols);
        tmem_relinquish();
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars.tmem;
    volatile int *abort = &bars.abort;
    const int n_tiles = __ldcg(A.n_tiles);
    const uint32_t my_tiles =
        (int)blockIdx.x < n_tiles ? (uint32_t)(n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / gridDim.x : 0u;
    const uint32_t nb = A.nb;
    const uint32_t G = my_tiles * nb; /* super-blocks this CTA walks, tile-major */
    uint8_t *sA = sm + kOffA, *sB = sm + kOffB, *sR = sm + kOffR, *sT = sm + kOffT, *sW = sm + kOffW;

    if (warp < kEpiWarps) {
        /* ---------------- epilogue ---------------- */
        const int q4 = warp & 3, ch = warp >> 2;
        const int r = 32 * q4 + lane;
        const uint32_t tl = tmem + ((uint32_t)(32 * q4) << 16);
        uint32_t g = 0;
        bool ok = true;
        for (uint32_t it = 0; it < my_tiles && ok; ++it) {
            const UTile tile = A.tiles[blockIdx.x + it * gridDim.x];
            const UTokBlock blk = A.tbs[tile.tb];
            const int nv = blk.ntok - 64 * ch; /* valid tokens in this warp's half */
            float S[64];
#pragma unroll
            for (int i = 0; i < 64; ++i) S[i] = 0.0f;
            for (uint32_t sb = 0; sb < nb; ++sb, ++g) {
                const uint32_t buf = g & 1u, ph = (g >> 1) & 1u;
                ok = uwait(&bars.t_full[buf], ph, abort, A.err) && uwait(&bars.ti_full[buf], ph, abort, A.err) &&
                     uwait(&bars.ri_full[buf], ph, abort, A.err);
                if (!ok) break;
                tc_fence_after();
                const uint4 ri = *reinterpret_cast<const uint4 *>(sW + buf * kRowInfo + r * 16);
                const float d = __uint_as_float(ri.x), dmin = __uint_as_float(ri.y);
                const float *d8s = reinterpret_cast<const float *>(sT + buf * kTokInfo);
                const uint4 *bps = reinterpret_cast<const uint4 *>(sT + buf * kTokInfo + kN * 4);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    if (16 * c < nv) { /* warp-uniform */
                        uint32_t v1[16], v2[16];
                        const uint32_t col = buf * 256u + 64u * ch + 16u * c;
                        tmem_ld16(tl + col, v1);
                        tmem_ld16(tl + col + 128u, v2);
                        tmem_wait(v1, v2);
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            const int t = 64 * ch + 16 * c + i;
                            const float d8 = d8s[t];
                            const uint4 bp = bps[t];
                            const int acc = (int)v1[i] + 16 * (int)v2[i];
                            int mins = __dp2a_lo((int)bp.x, (int)ri.z, 0);
                            mins = __dp2a_hi((int)bp.y, (int)ri.z, mins);
                            mins = __dp2a_lo((int)bp.z, (int)ri.w, mins);
                            mins = __dp2a_hi((int)bp.w, (int)ri.w, mins);
                            if (d8 != 0.0f)
                                S[16 * c + i] = __fmaf_rn(__fmul_rn(d8, d), (float)acc,
                                                          __fmaf_rn(-__fmul_rn(d8, dmin), (float)mins, S[16 * c + i]));
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    lfm_mbar_arrive(&bars.t_empty[buf]);
                    lfm_mbar_arrive(&bars.i_empty[buf]);
                }
            }
            if (!ok) break;
            float *yb = A.Y + (size_t)(blk.slot0 + 64 * ch) * A.rows + tile.row0 + r;
#pragma unroll
            for (int t = 0; t < 64; ++t)
                if (t < nv) yb[(size_t)t * A.rows] = S[t];
        }
        if (!ok) *abort = 1;
    } else if (warp < kWarpMma) {
        /* ---------------- producers ---------------- */
        const int p = tid - kEpiWarps * 32;
        const uint32_t rowoff = (uint32_t)(p >> 3) * 128u + (uint32_t)(p & 7) * 16u;
        auto issue_raw = [&](uint32_t gg) {
            const UTile tile = A.tiles[blockIdx.x + (gg / nb) * gridDim.x];
            const uint8_t *src = A.W + (((size_t)tile.expert * A.rows + tile.row0 + p) * nb + gg % nb) * kRaw;
            uint64_t *bar = &bars.r_full[gg % kSR];
            lfm_mbar_arrive_tx(bar, kRaw);
            lfm_bulk_g2s_plain(sR + (gg % kSR) * kRawSlot + p * kRaw, src, kRaw, bar);
        };
        for (uint32_t gg = 0; gg < G && gg < kSR - 1; ++gg) issue_raw(gg);
        bool ok = true;
        for (uint32_t g = 0; g < G && ok; ++g) {
            /* slot (g + 2) % 3 held super-block g - 1, which this thread has finished reading */
            if (g + kSR - 1 < G) issue_raw(g + kSR - 1);
            if (!uwait(&bars.r_full[g % kSR], (g / kSR) & 1u, abort, A.err)) { ok = false; break; }
            const uint8_t *raw = sR + (g % kSR) * kRawSlot + p * kRaw;
            const uint4 hdr = lfm_ld16<true>(raw);
            const uint32_t s0 = hdr.y, s1 = hdr.z, s2 = hdr.w;
            const uint32_t scA = s0 & 0x3F3F3F3Fu;
            const uint32_t scB = (s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u);
            const uint32_t mA = s1 & 0x3F3F3F3Fu;
            const uint32_t mB = ((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u);
            const uint32_t buf = g & 1u;
            if (g >= 2 && !uwait(&bars.i_empty[buf], ((g >> 1) & 1u) ^ 1u, abort, A.err)) { ok = false; break; }
            sts128(sW + buf * kRowInfo + p * 16, __float_as_uint(lfm_h2f((uint16_t)(hdr.x & 0xFFFFu))),
                   __float_as_uint(lfm_h2f((uint16_t)(hdr.x >> 16))), mA, mB);
            lfm_mbar_arrive(&bars.ri_full[buf]);
            for (uint32_t h = 0; h < 2; ++h) {
                const uint32_t q = 2 * g + h, s = q % kSA;
                if (q >= kSA && !uwait(&bars.a_empty[s], ((q / kSA) & 1u) ^ 1u, abort, A.err)) { ok = false; break; }
                uint8_t *a1 = sA + s * 2 * kOp, *a2 = a1 + kOp;
                const uint32_t scw = h ? scB : scA; /* nibble groups 2h, 2h+1: sub-blocks 4h..4h+3 */
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    const uint32_t slo = (scw >> (16 * cc)) & 0xFFu, shi = (scw >> (16 * cc + 8)) & 0xFFu;
                    const uint32_t bl = slo & 15u, al = slo >> 4, bh = shi & 15u, ah = shi >> 4;
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf) {
                        /* bytes 16*hf.. of nibble group 2h+cc: elements 16*hf.. of sub-blocks 4h+2cc (low
                         * nibbles) and 4h+2cc+1 (high); their 16-byte K chunks within the half: 4cc+hf, 4cc+2+hf */
                        const uint4 w = lfm_ld16<true>(raw + 16 + 32 * (2 * h + cc) + 16 * hf);
                        const uint32_t l0 = w.x & 0x0F0F0F0Fu, l1 = w.y & 0x0F0F0F0Fu, l2 = w.z & 0x0F0F0F0Fu,
                                       l3 = w.w & 0x0F0F0F0Fu;
                        const uint32_t h0 = (w.x >> 4) & 0x0F0F0F0Fu, h1 = (w.y >> 4) & 0x0F0F0F0Fu,
                                       h2 = (w.z >> 4) & 0x0F0F0F0Fu, h3 = (w.w >> 4) & 0x0F0F0F0Fu;
                        const uint32_t klo = (4 * cc + hf) * kCoreK + rowoff, khi = (4 * cc + 2 + hf) * kCoreK + rowoff;
                        /* bytes of a nibble word times a scalar <= 15 stay below 256: no carries */
                        sts128(a1 + klo, l0 * bl, l1 * bl, l2 * bl, l3 * bl);
                        sts128(a2 + klo, l0 * al, l1 * al, l2 * al, l3 * al);
                        sts128(a1 + khi, h0 * bh, h1 * bh, h2 * bh, h3 * bh);
                        sts128(a2 + khi, h0 * ah, h1 * ah, h2 * ah, h3 * ah);
                    }
                }
                fence_async_smem(); /* generic-proxy writes -> the tensor core's reads */
                lfm_mbar_arrive(&bars.a_full[s]);
            }
        }
        if (!ok) *abort = 1;
    } else if (warp == kWarpMma) {
        /* ---------------- MMA issue ---------------- */
        if (lane == 0) {
            bool ok = true;
            for (uint32_t g = 0; g < G && ok; ++g) {
                const uint32_t buf = g & 1u;
                if (g >= 2 && !uwait(&bars.t_empty[buf], ((g >> 1) & 1u) ^ 1u, abort, A.err)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d1 = tmem + buf * 256u, d2 = d1 + 128u;
                for (uint32_t h = 0; h < 2; ++h) {
                    const uint32_t q = 2 * g + h, s = q % kSA, ph = (q / kSA) & 1u;
                    if (!uwait(&bars.a_full[s], ph, abort, A.err) || !uwait(&bars.b_full[s], ph, abort, A.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a1 = lfm_smem_u32(sA + s * 2 * kOp), a2 = a1 + kOp;
                    const uint32_t b = lfm_smem_u32(sB + s * kOp);
#pragma unroll
                    for (uint32_t k = 0; k < 4; ++k) {
                        const uint32_t en = (h | k) ? 1u : 0u;
                        umma_i8(d1, udesc(a1 + 2 * k * kCoreK), udesc(b + 2 * k * kCoreK), en);
                        umma_i8(d2, udesc(a2 + 2 * k * kCoreK), udesc(b + 2 * k * kCoreK), en);
                    }
                    umma_commit(&bars.a_empty[s]);
                    umma_commit(&bars.b_empty[s]);
                }
                if (ok) umma_commit(&bars.t_full[buf]);
            }
            if (!ok) *abort = 1;
        }
    } else {
        /* ---------------- loader ---------------- */
        if (lane == 0) {
            bool ok = true;
            for (uint32_t g = 0; g < G && ok; ++g) {
                const UTile tile = A.tiles[blockIdx.x + (g / nb) * gridDim.x];
                const uint8_t *src = A.xt + ((size_t)tile.tb * nb + g % nb) * kXtSb;
                const uint32_t buf = g & 1u;
                if (g >= 2 && !uwait(&bars.i_empty[buf], ((g >> 1) & 1u) ^ 1u, abort, A.err)) { ok = false; break; }
                lfm_mbar_arrive_tx(&bars.ti_full[buf], kTokInfo);
                lfm_bulk_g2s_plain(sT + buf * kTokInfo, src + 2 * kOp, kTokInfo, &bars.ti_full[buf]);
                for (uint32_t h = 0; h < 2; ++h) {
                    const uint32_t q = 2 * g + h, s = q % kSA;
                    if (q >= kSA && !uwait(&bars.b_empty[s], ((q / kSA) & 1u) ^ 1u, abort, A.err)) {
                        ok = false;
                        break;
                    }
                    lfm_mbar_arrive_tx(&bars.b_full[s], kOp);
                    lfm_bulk_g2s_plain(sB + s * kOp, src + h * kOp, kOp, &bars.b_full[s]);
                }
            }
            if (!ok) *abort = 1;
        }
    }

    __syncthreads();
    if (*abort) {
        /* copies and MMAs already issued complete within microseconds: let them land */
        const uint64_t t0 = lfm_globaltimer();
        while (lfm_globaltimer() - t0 < 2000000ull) {
        }
    }
    if (warp == kWarpMma) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

/* Tokens of every block, per super-block, in the MMA's canonical K-major
 * layout: half h (K bytes 128h..128h+127) is 8 chunks of 16 K bytes x 128
 * tokens, token t's 16 bytes at chunk*kCoreK + 16*t (= 8-token groups of 128
 * bytes); then d8 per token and the sub-block sums bsum[2j] + bsum[2j+1]
 * packed two per word (j = 0..7).  Tokens past the block's count are zero. */
__global__ void __launch_bounds__(256) k_xt_gather(Q8Rows X, const int32_t *perm, uint32_t K, const UTokBlock *tbs,
                                                   const int32_t *n_tb, uint32_t nb, uint8_t *xt) {
    __shared__ int xr[kN];
    const int tb = blockIdx.x;
    if (tb >= __ldcg(n_tb)) return;
    const uint32_t sb = blockIdx.y;
    const UTokBlock blk = tbs[tb];
    if (threadIdx.x < kN) {
        const int t = threadIdx.x;
        xr[t] = t < blk.ntok ? (perm ? __ldcg(perm + blk.slot0 + t) / (int)K : blk.slot0 + t) : -1;
    }
    __syncthreads();
    uint8_t *dst = xt + ((size_t)tb * nb + sb) * kXtSb;
    for (int q = threadIdx.x; q < kN * 16; q += blockDim.x) {
        const int c = q >> 7, t = q & (kN - 1);
        const int row = xr[t];
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (row >= 0) v = __ldcg(reinterpret_cast<const uint4 *>(X.qs + (size_t)row * X.cols + 256 * sb + 16 * c));
        *reinterpret_cast<uint4 *>(dst + (c >> 3) * kOp + (c & 7) * kCoreK + 16 * t) = v;
    }
    if (threadIdx.x < kN) {
        const int t = threadIdx.x, row = xr[t];
        float d8 = 0.0f;
        uint4 pr = make_uint4(0u, 0u, 0u, 0u);
        if (row >= 0) {
            d8 = __ldcg(X.d + (size_t)row * nb + sb);
            const int16_t *bs = X.bs + ((size_t)row * nb + sb) * 16;
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int lo = bs[4 * i] + bs[4 * i + 1], hi = bs[4 * i + 2] + bs[4 * i + 3];
                w[i] = (uint32_t)(uint16_t)lo | ((uint32_t)(uint16_t)hi << 16);
            }
            pr = make_uint4(w[0], w[1], w[2], w[3]);
        }
        reinterpret_cast<float *>(dst + 2 * kOp)[t] = d8;
        reinterpret_cast<uint4 *>(dst + 2 * kOp + kN * 4)[t] = pr;
    }
}

/* Tile plan from the dispatch tables: token blocks of <= 128 slots per active
 * expert, then tiles = (expert, 128-row block, token block) with the token
 * blocks fastest, so CTAs that share a weight block run together and share it
 * through L2.  One block; counts[0] = tiles, counts[1] = token blocks. */
__global__ void k_umma_plan(RouteTables rt, uint32_t rows, UTile *tiles, UTokBlock *tbs, int32_t *counts,
                            uint32_t max_tiles, uint32_t max_tb) {
    __shared__ int s_e[LFM_GPU_MAX_EXPERTS_DEV], s_cnt[LFM_GPU_MAX_EXPERTS_DEV], s_off[LFM_GPU_MAX_EXPERTS_DEV];
    __shared__ int s_tb[LFM_GPU_MAX_EXPERTS_DEV + 1], s_ti[LFM_GPU_MAX_EXPERTS_DEV + 1];
    __shared__ int s_bad;
    const int U = __ldcg(rt.summary + 0);
    const int nrb = (int)rows / kM;
    for (int u = threadIdx.x; u < U; u += blockDim.x) {
        const int e = __ldcg(rt.act + u);
        s_e[u] = e;
        s_cnt[u] = __ldcg(rt.counts + e);
        s_off[u] = __ldcg(rt.offsets + e);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int a = 0, b = 0;
        for (int u = 0; u < U; ++u) {
            const int n = (s_cnt[u] + kN - 1) / kN;
            s_tb[u] = a;
            s_ti[u] = b;
            a += n;
            b += n * nrb;
        }
        s_bad = (uint32_t)a > max_tb || (uint32_t)b > max_tiles;
        if (s_bad) {
            atomicOr(rt.err, LFM_DEVERR_SEGMENT);
            a = b = 0;
        }
        counts[0] = b;
        counts[1] = a;
    }
    __syncthreads();
    if (s_bad) return;
    for (int u = 0; u < U; ++u) {
        const int n = (s_cnt[u] + kN - 1) / kN;
        for (int q = threadIdx.x; q < n; q += blockDim.x)
            tbs[s_tb[u] + q] = UTokBlock{s_off[u] + q * kN, min(kN, s_cnt[u] - q * kN)};
        for (int q = threadIdx.x; q < n * nrb; q += blockDim.x) {
            const int rb = q / n, i = q - rb * n;
            tiles[s_ti[u] + q] = UTile{s_e[u], s_tb[u] + i, rb * kM, 0};
        }
    }
}

}  // namespace

bool lfm_umma_ok(uint32_t rows) { return rows % kM == 0; }
size_t lfm_umma_tb_max(uint32_t slots, uint32_t experts) { return (slots + kN - 1) / kN + experts; }
size_t lfm_umma_tiles_max(uint32_t rows, uint32_t slots, uint32_t experts) {
    return (size_t)(rows / kM) * lfm_umma_tb_max(slots, experts);
}
size_t lfm_umma_tile_bytes() { return sizeof(UTile); }
size_t lfm_umma_tb_bytes() { return sizeof(UTokBlock); }
size_t lfm_umma_xt_bytes(size_t max_tb, uint32_t nb) { return max_tb * nb * (size_t)kXtSb; }

cudaError_t lfm_launch_umma_plan(const RouteTables &rt, uint32_t rows, void *tiles, void *tbs, int32_t *counts,
                                 uint32_t max_tiles, uint32_t max_tb, cudaStream_t s) {
    k_umma_plan<<<1, 256, 0, s>>>(rt, rows, static_cast<UTile *>(tiles), static_cast<UTokBlock *>(tbs), counts,
                                  max_tiles, max_tb);
    return cudaGetLastError();
}

cudaError_t lfm_launch_xt_gather(Q8Rows X, const int32_t *perm, uint32_t K, const void *tbs, const int32_t *n_tb,
                                 uint32_t max_tb, uint8_t *xt, cudaStream_t s) {
    const uint32_t nb = X.cols / 256;
    if (max_tb == 0 || nb == 0) return cudaSuccess;
    k_xt_gather<<<dim3(max_tb, nb), 256, 0, s>>>(X, perm, K, static_cast<const UTokBlock *>(tbs), n_tb, nb, xt);
    return cudaGetLastError();
}

cudaError_t lfm_launch_q4k_umma(const uint8_t *W, uint32_t rows, uint32_t cols, const uint8_t *xt, const void *tiles,
                                const void *tbs, const int32_t *n_tiles, float *Y, uint32_t *err, int grid,
                                cudaStream_t s) {
    if (rows % kM || cols % 256) return cudaErrorInvalidValue;
    static size_t cache[16];
    cudaError_t e = lfm_smem_attr((const void *)k_q4k_umma, kSmem, cache);
    if (e != cudaSuccess) return e;
    UmmaArgs a{W, rows, cols / 256, xt, static_cast<const UTile *>(tiles), static_cast<const UTokBlock *>(tbs),
               n_tiles, Y, err};
    k_q4k_umma<<<grid, kThreads, kSmem, s>>>(a);
    return cudaGetLastError();
}
