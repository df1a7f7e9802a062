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
 * Tile: 128 weight rows (MMA M) x nt tokens (MMA N, nt = 16..128 chosen per
 * call from the tokens per expert) of one expert; K walked in half
 * super-blocks (128 bytes).  One CTA per SM, persistent over the tile
 * list, warp-specialised:
 *   warps 0-7   epilogue: TMEM -> registers (tcgen05.ld 32x32b), the fp32
 *               update above into <= 64 running sums per thread (thread =
 *               row, warp pair = the tile's two token halves), Y at the end;
 *   warps 8-11  producers: the tile's 128 Q4_K rows of a super-block arrive
 *               by one 2-D tensor copy (TMA tile 144 bytes x 128 rows, ring of
 *               3 super-blocks); thread p expands row p's nibbles into A1/A2 in
 *               the UMMA canonical K-major layout (8-row x 16-byte core
 *               matrices) and publishes d, dmin, m_j;
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
#include <cudaTypedefs.h>

#include <mutex>

#include "moe_device.cuh"
#include "moe_internal.h"

namespace {

constexpr int kM = 128;                      /* weight rows per tile (MMA M)               */
constexpr int kN = 128;                      /* most tokens per tile (MMA N)               */
constexpr int kHalf = 128;                   /* K bytes per stage: half a super-block      */
constexpr int kCoreK = kM * 16;              /* bytes between K-adjacent core matrices     */
constexpr int kOp = kM * kHalf;              /* 16384: one operand stage (A1, A2 or B)     */
constexpr int kTokInfo = kN * 4 + kN * 16;   /* d8[nt] fp32 + sub-block bsum pairs [nt][4]  */
/* pre-gathered tokens per (block, super-block) for nt tokens a block */
__host__ __device__ constexpr uint32_t xt_sb_bytes(uint32_t nt) { return nt * (2 * kHalf + 20); }
constexpr int kRaw = LFM_Q4K_BYTES;
constexpr int kRawSlot = kM * kRaw;
constexpr int kRowInfo = kM * 16;            /* d, dmin, m0..3, m4..7 per row              */
constexpr int kSA = 3;                       /* A1/A2 and B stages                         */
constexpr uint32_t kTmemCols = 512;

/* Two arrangements of the same pipeline.
 *  prefill (kTs = false, nt > 64): A1/A2 expanded into shared memory (SS MMA);
 *    8 epilogue warps (two per TMEM lane quarter, half of the tokens each), 4
 *    producer warps (one row each, both halves of a super-block); TMEM holds
 *    D1/D2 for nt <= 128 tokens, double buffered (4 x 128 columns).
 *  decode (kTs = true, nt <= 64): A1/A2 expanded into tensor memory with
 *    tcgen05.st (A-from-TMEM MMA), which spares shared memory the expanded
 *    rows -- at few tokens per expert that traffic, not the tensor core, is
 *    the limit; 4 epilogue warps, 8 producer warps (one row each, one half of
 *    the super-block), a deeper raw-weight ring.  TMEM: D1/D2 for nt <= 64
 *    double buffered (columns 0-255), then 3 stages of A1|A2 (64 columns each). */
template <bool kTs>
struct UCfg {
    static constexpr int kEpi = kTs ? 4 : 8;
    static constexpr int kProd = kTs ? 8 : 4;
    static constexpr int kSR = kTs ? 8 : 3;
    static constexpr int kWarpMma = kEpi + kProd;
    static constexpr int kWarpLoad = kWarpMma + 1;
    static constexpr int kThreads = (kWarpLoad + 1) * 32;
    static constexpr int kOffA = 0;
    static constexpr int kOffB = kOffA + (kTs ? 0 : kSA * 2 * kOp);
    static constexpr int kOffR = kOffB + kSA * kOp;
    static constexpr int kOffT = kOffR + kSR * kRawSlot;
    static constexpr int kOffW = kOffT + 2 * kTokInfo;
    static constexpr int kSmem = kOffW + 2 * kRowInfo;
    static constexpr uint32_t kDbuf = kTs ? 128u : 256u; /* TMEM columns of one D1|D2 buffer */
    static constexpr uint32_t kD2 = kTs ? 64u : 128u;    /* D2 after D1                      */
    static constexpr uint32_t kA0 = 256u;                /* first A stage (decode)           */
};
constexpr uint32_t kNtDecode = 64; /* largest token block of the decode arrangement */
static_assert(UCfg<false>::kSmem <= 227 * 1024 && UCfg<true>::kSmem <= 227 * 1024, "shared memory");
static_assert(UCfg<false>::kThreads == UCfg<true>::kThreads, "one block size");
constexpr int kThreads = UCfg<false>::kThreads;

/* Instruction descriptor, kind::i8: D s32 (bits 4-5 = 2), A u8 (7-9 = 0),
 * B s8 (10-12 = 1), both K-major, M >> 4 at bits 24-28; N >> 3 goes to 17-22. */
constexpr uint32_t kIdescBase = (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(kM >> 4) << 24);

struct UTile {
    int32_t expert, tb, row0, pad;
};
struct UTokBlock {
    int32_t slot0, ntok;
};

struct UmmaArgs {
    const uint8_t *W;     /* expert tensors [E][rows][nb] Q4_K */
    uint32_t rows, nb;
    const uint8_t *xt;    /* pre-gathered tokens [block][nb][xt_sb_bytes(nt)] */
    uint32_t nt;          /* tokens per block (MMA N): a multiple of 16, <= 128 */
    const UTile *tiles;
    const UTokBlock *tbs;
    const int32_t *n_tiles;
    float *Y;             /* [slots][rows] */
    uint32_t *err;
};

struct UmmaBars {
    uint64_t a_full[kSA], a_empty[kSA], b_full[kSA], b_empty[kSA], r_full[8], r_empty[8];
    uint64_t t_full[2], t_empty[2], ti_full[2], ri_full[2], i_empty[2];
    uint32_t tmem;
    int abort;
};

/* Shared-memory matrix descriptor, K-major without swizzle: start address,
 * leading byte offset (K-adjacent core matrices) `lbo`, stride byte offset
 * (8-row groups) = 128, version 1 at bit 46. */
__device__ __forceinline__ uint64_t udesc(uint32_t saddr, uint32_t lbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)(128 >> 4) << 32) | (1ull << 46);
}

__device__ __forceinline__ void umma_i8(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
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

/* 8 consecutive 32-bit columns of this thread's TMEM lane. */
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr));
}
/* Wait for this thread's TMEM loads; the registers are tied to the wait so no
 * use of them is scheduled before it. */
__device__ __forceinline__ void tmem_wait(uint32_t (&a)[8], uint32_t (&b)[8]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]),
                   "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7])::"memory");
}

/* 32 consecutive 32-bit columns of this thread's TMEM lane from registers. */
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
        "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
        "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

/* A from tensor memory: tcgen05.mma with the A operand's TMEM address. */
__device__ __forceinline__ void umma_i8_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d),
        "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
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

template <bool kTs>
__global__ void __launch_bounds__(kThreads, 1) k_q4k_umma(const __grid_constant__ CUtensorMap tmw, UmmaArgs A) {
    using C = UCfg<kTs>;
    extern __shared__ __align__(1024) uint8_t sm[];
    __shared__ UmmaBars bars;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int i = 0; i < kSA; ++i) {
            lfm_mbar_init(&bars.a_full[i], kM); /* one arrival per row of the half super-block */
            lfm_mbar_init(&bars.a_empty[i], 1);
            lfm_mbar_init(&bars.b_full[i], 1);
            lfm_mbar_init(&bars.b_empty[i], 1);
        }
        for (int i = 0; i < C::kSR; ++i) {
            lfm_mbar_init(&bars.r_full[i], 1);
            lfm_mbar_init(&bars.r_empty[i], C::kProd * 32);
        }
        for (int i = 0; i < 2; ++i) {
            lfm_mbar_init(&bars.t_full[i], 1);
            lfm_mbar_init(&bars.t_empty[i], C::kEpi);
            lfm_mbar_init(&bars.ti_full[i], 1);
            lfm_mbar_init(&bars.ri_full[i], kM);
            lfm_mbar_init(&bars.i_empty[i], C::kEpi);
        }
        bars.abort = 0;
        lfm_fence_mbar_init();
    }
    if (warp == C::kWarpMma) {
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
    uint8_t *sA = sm + C::kOffA, *sB = sm + C::kOffB, *sR = sm + C::kOffR, *sT = sm + C::kOffT, *sW = sm + C::kOffW;

    if (warp < C::kEpi) {
        /* ---------------- epilogue ---------------- */
        const int q4 = warp & 3, ch = warp >> 2;
        const int r = 32 * q4 + lane;
        const int half = (int)A.nt / (C::kEpi / 4); /* columns of this warp: [ch * half, ch * half + half) */
        const uint32_t tl = tmem + ((uint32_t)(32 * q4) << 16);
        uint32_t g = 0;
        bool ok = true;
        for (uint32_t it = 0; it < my_tiles && ok; ++it) {
            const UTile tile = A.tiles[blockIdx.x + it * gridDim.x];
            const UTokBlock blk = A.tbs[tile.tb];
            const int nv = min(blk.ntok - ch * half, half); /* valid tokens in this warp's columns */
            float S[64];
#pragma unroll
            for (int i = 0; i < 64; ++i) S[i] = 0.0f;
            for (uint32_t sb = 0; sb < nb; ++sb, ++g) {
                const uint32_t buf = g & 1u, ph = (g >> 1) & 1u;
                /* every decision that leaves a loop is warp-uniform: tcgen05.ld is .sync.aligned */
                ok = __all_sync(LFM_FULL_MASK, uwait(&bars.t_full[buf], ph, abort, A.err) &&
                                                   uwait(&bars.ti_full[buf], ph, abort, A.err) &&
                                                   uwait(&bars.ri_full[buf], ph, abort, A.err));
                if (!ok) break;
                tc_fence_after();
                const uint4 ri = *reinterpret_cast<const uint4 *>(sW + buf * kRowInfo + r * 16);
                const float d = __uint_as_float(ri.x), dmin = __uint_as_float(ri.y);
                const float *d8s = reinterpret_cast<const float *>(sT + buf * kTokInfo) + ch * half;
                const uint4 *bps = reinterpret_cast<const uint4 *>(sT + buf * kTokInfo + A.nt * 4) + ch * half;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    if (8 * c < nv) { /* warp-uniform */
                        uint32_t v1[8], v2[8];
                        const uint32_t col = buf * C::kDbuf + (uint32_t)(ch * half) + 8u * c;
                        tmem_ld8(tl + col, v1);
                        tmem_ld8(tl + col + C::kD2, v2);
                        tmem_wait(v1, v2);
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const int t = 8 * c + i;
                            const float d8 = d8s[t];
                            const uint4 bp = bps[t];
                            const int acc = (int)v1[i] + 16 * (int)v2[i];
                            int mins = __dp2a_lo((int)bp.x, (int)ri.z, 0);
                            mins = __dp2a_hi((int)bp.y, (int)ri.z, mins);
                            mins = __dp2a_lo((int)bp.z, (int)ri.w, mins);
                            mins = __dp2a_hi((int)bp.w, (int)ri.w, mins);
                            if (d8 != 0.0f)
                                S[8 * c + i] = __fmaf_rn(__fmul_rn(d8, d), (float)acc,
                                                         __fmaf_rn(-__fmul_rn(d8, dmin), (float)mins, S[8 * c + i]));
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
            float *yb = A.Y + (size_t)(blk.slot0 + ch * half) * A.rows + tile.row0 + r;
#pragma unroll
            for (int t = 0; t < 64; ++t)
                if (t < nv) yb[(size_t)t * A.rows] = S[t];
        }
        if (!ok) *abort = 1;
    } else if (warp < C::kWarpMma) {
        /* ---------------- producers ---------------- */
        const int pt = tid - C::kEpi * 32;
        const int p = pt & (kM - 1);             /* weight row of the tile                          */
        const int h0 = kTs ? pt / kM : 0;        /* decode: this thread's half of every super-block */
        const int nh = kTs ? 1 : 2;
        const uint32_t rowoff = (uint32_t)(p >> 3) * 128u + (uint32_t)(p & 7) * 16u;
        const uint32_t tla = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + C::kA0; /* decode: this lane quarter */
        /* producer 0 issues: the tile's 128 rows x super-block gg (144 bytes at x = 144 * sb) */
        auto issue_raw = [&](uint32_t gg) {
            const UTile tile = A.tiles[blockIdx.x + (gg / nb) * gridDim.x];
            uint64_t *bar = &bars.r_full[gg % C::kSR];
            lfm_mbar_arrive_tx(bar, kRawSlot);
            lfm_tma_load_2d(sR + (gg % C::kSR) * kRawSlot, &tmw, (gg % nb) * kRaw,
                            (uint32_t)tile.expert * A.rows + tile.row0, bar);
        };
        bool ok = true;
        if (pt == 0)
            for (uint32_t gg = 0; gg < G && gg < C::kSR - 1; ++gg) issue_raw(gg);
        /* every decision that leaves a loop is warp-uniform (tcgen05.st is .sync.aligned) */
        for (uint32_t g = 0; g < G && ok; ++g) {
            bool w = true;
            /* slot (g - 1) % kSR held super-block g - 1: reissue it once every producer has left it */
            if (pt == 0 && g + C::kSR - 1 < G) {
                if (g >= 1) w = uwait(&bars.r_empty[(g - 1) % C::kSR], ((g - 1) / C::kSR) & 1u, abort, A.err);
                if (w) issue_raw(g + C::kSR - 1);
            }
            w = w && uwait(&bars.r_full[g % C::kSR], (g / C::kSR) & 1u, abort, A.err);
            if (!__all_sync(LFM_FULL_MASK, w)) { ok = false; break; }
            const uint8_t *raw = sR + (g % C::kSR) * kRawSlot + p * kRaw;
            const uint4 hdr = lfm_ld16<true>(raw);
            const uint32_t s0 = hdr.y, s1 = hdr.z, s2 = hdr.w;
            const uint32_t scA = s0 & 0x3F3F3F3Fu;
            const uint32_t scB = (s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u);
            const uint32_t buf = g & 1u;
            if (h0 == 0) {
                const uint32_t mA = s1 & 0x3F3F3F3Fu;
                const uint32_t mB = ((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u);
                w = g < 2 || uwait(&bars.i_empty[buf], ((g >> 1) & 1u) ^ 1u, abort, A.err);
                if (!__all_sync(LFM_FULL_MASK, w)) { ok = false; break; }
                sts128(sW + buf * kRowInfo + p * 16, __float_as_uint(lfm_h2f((uint16_t)(hdr.x & 0xFFFFu))),
                       __float_as_uint(lfm_h2f((uint16_t)(hdr.x >> 16))), mA, mB);
                lfm_mbar_arrive(&bars.ri_full[buf]);
            }
            for (int hh = 0; hh < nh; ++hh) {
                const uint32_t h = (uint32_t)(h0 + hh);
                const uint32_t q = 2 * g + h, s = q % kSA;
                w = q < kSA || uwait(&bars.a_empty[s], ((q / kSA) & 1u) ^ 1u, abort, A.err);
                if (!__all_sync(LFM_FULL_MASK, w)) { ok = false; break; }
                const uint32_t scw = h ? scB : scA; /* nibble groups 2h, 2h+1: sub-blocks 4h..4h+3 */
                if constexpr (kTs) {
                    /* K byte 4j..4j+3 of the half in TMEM column j: word j of nibble group 2h + j/16 */
                    tc_fence_after();
                    uint32_t a1[32], a2[32];
#pragma unroll
                    for (int cc = 0; cc < 2; ++cc) {
                        const uint32_t slo = (scw >> (16 * cc)) & 0xFFu, shi = (scw >> (16 * cc + 8)) & 0xFFu;
                        const uint32_t bl = slo & 15u, al = slo >> 4, bh = shi & 15u, ah = shi >> 4;
#pragma unroll
                        for (int hf = 0; hf < 2; ++hf) {
                            const uint4 w = lfm_ld16<true>(raw + 16 + 32 * (2 * h + cc) + 16 * hf);
                            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                            for (int m = 0; m < 4; ++m) {
                                const uint32_t lo = ww[m] & 0x0F0F0F0Fu, hi = (ww[m] >> 4) & 0x0F0F0F0Fu;
                                /* bytes of a nibble word times a scalar <= 15 stay below 256: no carries */
                                a1[16 * cc + 4 * hf + m] = lo * bl;
                                a2[16 * cc + 4 * hf + m] = lo * al;
                                a1[16 * cc + 8 + 4 * hf + m] = hi * bh;
                                a2[16 * cc + 8 + 4 * hf + m] = hi * ah;
                            }
                        }
                    }
                    tmem_st32(tla + 64u * s, a1);
                    tmem_st32(tla + 64u * s + 32u, a2);
                    tmem_wait_st();
                    tc_fence_before();
                } else {
                    uint8_t *a1 = sA + s * 2 * kOp, *a2 = a1 + kOp;
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
                            const uint32_t x0 = (w.x >> 4) & 0x0F0F0F0Fu, x1 = (w.y >> 4) & 0x0F0F0F0Fu,
                                           x2 = (w.z >> 4) & 0x0F0F0F0Fu, x3 = (w.w >> 4) & 0x0F0F0F0Fu;
                            const uint32_t klo = (4 * cc + hf) * kCoreK + rowoff, khi = (4 * cc + 2 + hf) * kCoreK + rowoff;
                            /* bytes of a nibble word times a scalar <= 15 stay below 256: no carries */
                            sts128(a1 + klo, l0 * bl, l1 * bl, l2 * bl, l3 * bl);
                            sts128(a2 + klo, l0 * al, l1 * al, l2 * al, l3 * al);
                            sts128(a1 + khi, x0 * bh, x1 * bh, x2 * bh, x3 * bh);
                            sts128(a2 + khi, x0 * ah, x1 * ah, x2 * ah, x3 * ah);
                        }
                    }
                    fence_async_smem(); /* generic-proxy writes -> the tensor core's reads */
                }
                lfm_mbar_arrive(&bars.a_full[s]);
            }
            if (ok) lfm_mbar_arrive(&bars.r_empty[g % C::kSR]);
        }
        if (!ok) *abort = 1;
    } else if (warp == C::kWarpMma) {
        /* ---------------- MMA issue ---------------- */
        if (lane == 0) {
            bool ok = true;
            const uint32_t idesc = kIdescBase | ((A.nt >> 3) << 17), blbo = A.nt * 16u;
            for (uint32_t g = 0; g < G && ok; ++g) {
                const uint32_t buf = g & 1u;
                if (g >= 2 && !uwait(&bars.t_empty[buf], ((g >> 1) & 1u) ^ 1u, abort, A.err)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d1 = tmem + buf * C::kDbuf, d2 = d1 + C::kD2;
                for (uint32_t h = 0; h < 2; ++h) {
                    const uint32_t q = 2 * g + h, s = q % kSA, ph = (q / kSA) & 1u;
                    if (!uwait(&bars.a_full[s], ph, abort, A.err) || !uwait(&bars.b_full[s], ph, abort, A.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t b = lfm_smem_u32(sB + s * kOp);
#pragma unroll
                    for (uint32_t k = 0; k < 4; ++k) {
                        const uint32_t en = (h | k) ? 1u : 0u;
                        const uint64_t bd = udesc(b + 2 * k * blbo, blbo);
                        if constexpr (kTs) {
                            const uint32_t a1 = tmem + C::kA0 + 64u * s + 8u * k; /* 8 columns = 32 K bytes */
                            umma_i8_ts(d1, a1, bd, idesc, en);
                            umma_i8_ts(d2, a1 + 32u, bd, idesc, en);
                        } else {
                            const uint32_t a1 = lfm_smem_u32(sA + s * 2 * kOp), a2 = a1 + kOp;
                            umma_i8(d1, udesc(a1 + 2 * k * kCoreK, kCoreK), bd, idesc, en);
                            umma_i8(d2, udesc(a2 + 2 * k * kCoreK, kCoreK), bd, idesc, en);
                        }
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
                const uint32_t opb = A.nt * kHalf; /* one half super-block of the block's codes */
                const uint8_t *src = A.xt + ((size_t)tile.tb * nb + g % nb) * xt_sb_bytes(A.nt);
                const uint32_t buf = g & 1u;
                if (g >= 2 && !uwait(&bars.i_empty[buf], ((g >> 1) & 1u) ^ 1u, abort, A.err)) { ok = false; break; }
                lfm_mbar_arrive_tx(&bars.ti_full[buf], A.nt * 20u);
                lfm_bulk_g2s_plain(sT + buf * kTokInfo, src + 2 * opb, A.nt * 20u, &bars.ti_full[buf]);
                for (uint32_t h = 0; h < 2; ++h) {
                    const uint32_t q = 2 * g + h, s = q % kSA;
                    if (q >= kSA && !uwait(&bars.b_empty[s], ((q / kSA) & 1u) ^ 1u, abort, A.err)) {
                        ok = false;
                        break;
                    }
                    lfm_mbar_arrive_tx(&bars.b_full[s], opb);
                    lfm_bulk_g2s_plain(sB + s * kOp, src + h * opb, opb, &bars.b_full[s]);
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
    if (warp == C::kWarpMma) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

/* Tokens of every block, per super-block, in the MMA's canonical K-major
 * layout: half h (K bytes 128h..128h+127) is 8 chunks of 16 K bytes x nt
 * tokens, token t's 16 bytes at chunk*16*nt + 16*t (= 8-token groups of 128
 * bytes); then d8 per token and the sub-block sums bsum[2j] + bsum[2j+1]
 * packed two per word (j = 0..7).  Tokens past the block's count are zero. */
__global__ void __launch_bounds__(256) k_xt_gather(Q8Rows X, const int32_t *perm, uint32_t K, const UTokBlock *tbs,
                                                   const int32_t *n_tb, uint32_t nb, uint32_t nt, uint8_t *xt) {
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
    uint8_t *dst = xt + ((size_t)tb * nb + sb) * xt_sb_bytes(nt);
    for (uint32_t q = threadIdx.x; q < nt * 16; q += blockDim.x) {
        const uint32_t c = q / nt, t = q % nt;
        const int row = xr[t];
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (row >= 0) v = __ldcg(reinterpret_cast<const uint4 *>(X.qs + (size_t)row * X.cols + 256 * sb + 16 * c));
        *reinterpret_cast<uint4 *>(dst + (c >> 3) * nt * kHalf + (c & 7) * 16 * nt + 16 * t) = v;
    }
    if (threadIdx.x < nt) {
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
        reinterpret_cast<float *>(dst + 2 * nt * kHalf)[t] = d8;
        reinterpret_cast<uint4 *>(dst + 2 * nt * kHalf + nt * 4)[t] = pr;
    }
}

/* Tile plan from the dispatch tables: token blocks of <= nt slots per active
 * expert, then tiles = (expert, 128-row block, token block) with the token
 * blocks fastest, so CTAs that share a weight block run together and share it
 * through L2.  One block; counts[0] = tiles, counts[1] = token blocks. */
__global__ void k_umma_plan(RouteTables rt, uint32_t rows, uint32_t nt, UTile *tiles, UTokBlock *tbs,
                            int32_t *counts, uint32_t max_tiles, uint32_t max_tb) {
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
            const int n = (s_cnt[u] + (int)nt - 1) / (int)nt;
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
        const int n = (s_cnt[u] + (int)nt - 1) / (int)nt;
        for (int q = threadIdx.x; q < n; q += blockDim.x)
            tbs[s_tb[u] + q] = UTokBlock{s_off[u] + q * (int)nt, min((int)nt, s_cnt[u] - q * (int)nt)};
        for (int q = threadIdx.x; q < n * nrb; q += blockDim.x) {
            const int rb = q / n, i = q - rb * n;
            tiles[s_ti[u] + q] = UTile{s_e[u], s_tb[u] + i, rb * kM, 0};
        }
    }
}

}  // namespace

bool lfm_umma_ok(uint32_t rows) { return rows % kM == 0; }
uint32_t lfm_umma_nt(uint32_t slots, uint32_t experts) {
    /* about three times the mean tokens per expert, so most experts fit one block */
    const uint32_t mean = (slots + experts - 1) / (experts ? experts : 1u);
    const uint32_t nt = (3 * mean + 15) / 16 * 16;
    return nt < 16 ? 16u : nt > (uint32_t)kN ? (uint32_t)kN : nt;
}
size_t lfm_umma_tb_max(uint32_t slots, uint32_t experts, uint32_t nt) { return (slots + nt - 1) / nt + experts; }
size_t lfm_umma_tiles_max(uint32_t rows, uint32_t slots, uint32_t experts, uint32_t nt) {
    return (size_t)(rows / kM) * lfm_umma_tb_max(slots, experts, nt);
}
size_t lfm_umma_tile_bytes() { return sizeof(UTile); }
size_t lfm_umma_tb_bytes() { return sizeof(UTokBlock); }
size_t lfm_umma_xt_bytes(size_t max_tb, uint32_t nb, uint32_t nt) { return max_tb * nb * (size_t)xt_sb_bytes(nt); }

cudaError_t lfm_launch_umma_plan(const RouteTables &rt, uint32_t rows, uint32_t nt, void *tiles, void *tbs,
                                 int32_t *counts, uint32_t max_tiles, uint32_t max_tb, cudaStream_t s) {
    if (nt % 16 || nt == 0 || nt > (uint32_t)kN) return cudaErrorInvalidValue;
    k_umma_plan<<<1, 256, 0, s>>>(rt, rows, nt, static_cast<UTile *>(tiles), static_cast<UTokBlock *>(tbs), counts,
                                  max_tiles, max_tb);
    return cudaGetLastError();
}

cudaError_t lfm_launch_xt_gather(Q8Rows X, const int32_t *perm, uint32_t K, const void *tbs, const int32_t *n_tb,
                                 uint32_t max_tb, uint32_t nt, uint8_t *xt, cudaStream_t s) {
    const uint32_t nb = X.cols / 256;
    if (max_tb == 0 || nb == 0) return cudaSuccess;
    k_xt_gather<<<dim3(max_tb, nb), 256, 0, s>>>(X, perm, K, static_cast<const UTokBlock *>(tbs), n_tb, nb, nt, xt);
    return cudaGetLastError();
}

/* cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link). */
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

bool lfm_tmap_2d(CUtensorMap *tm, CUtensorMapDataType type, uint32_t elem_bytes, const void *base, uint64_t inner,
                 uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer) {
    const PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (!encode || (reinterpret_cast<uintptr_t>(base) & 15u) || row_bytes % 16 || (box_inner * elem_bytes) % 16)
        return false;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    return encode(tm, type, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t lfm_launch_q4k_umma(const uint8_t *W, uint32_t experts, uint32_t rows, uint32_t cols, const uint8_t *xt,
                                uint32_t nt, const void *tiles, const void *tbs, const int32_t *n_tiles, float *Y,
                                uint32_t *err, int grid, cudaStream_t s) {
    if (rows % kM || cols % 256 || experts == 0 || nt % 16 || nt == 0 || nt > (uint32_t)kN)
        return cudaErrorInvalidValue;
    /* the expert tensor as a 2-D byte matrix [experts * rows][nb * 144] */
    CUtensorMap tm;
    const uint64_t row_bytes = (uint64_t)(cols / 256) * kRaw;
    if (!lfm_tmap_2d(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, W, row_bytes, (uint64_t)experts * rows, row_bytes, kRaw, kM))
        return cudaErrorInvalidValue;
    UmmaArgs a{W, rows, cols / 256, xt, nt, static_cast<const UTile *>(tiles), static_cast<const UTokBlock *>(tbs),
               n_tiles, Y, err};
    if (nt <= kNtDecode) {
        static size_t cache[16];
        cudaError_t e = lfm_smem_attr((const void *)k_q4k_umma<true>, UCfg<true>::kSmem, cache);
        if (e != cudaSuccess) return e;
        k_q4k_umma<true><<<grid, kThreads, UCfg<true>::kSmem, s>>>(tm, a);
    } else {
        static size_t cache[16];
        cudaError_t e = lfm_smem_attr((const void *)k_q4k_umma<false>, UCfg<false>::kSmem, cache);
        if (e != cudaSuccess) return e;
        k_q4k_umma<false><<<grid, kThreads, UCfg<false>::kSmem, s>>>(tm, a);
    }
    return cudaGetLastError();
}
