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
 * list, warp-specialised (counts per arrangement in UCfg below):
 *   epilogue    TMEM -> registers (tcgen05.ld 32x32b), the fp32 update above
 *               into running sums (thread = row; the warps of a TMEM lane
 *               quarter split the tile's tokens), Y at the end;
 *   producers   the tile's 128 Q4_K rows of a super-block arrive by one 2-D
 *               tensor copy (TMA tile 144 bytes x 128 rows, a ring of
 *               super-blocks); a thread expands its row's nibbles into the
 *               UMMA canonical K-major layout (8-row x 16-byte core matrices)
 *               and publishes d, dmin and the 6-bit scales and mins;
 *   2 MMA warps TMEM allocation (the first) and the MMA issue (one thread
 *               each, independent accumulators); commits release the stages
 *               and hand a finished accumulator buffer to the epilogue.
 *               Accumulators are double buffered, so super-block b+1
 *               multiplies while b drains;
 *   loader      one thread: the tokens' codes and scales for each half
 *               super-block, pre-gathered (k_xt_gather, k_swiglu_xt) into the
 *               same canonical layout, one bulk copy each.
 * Every mbarrier wait is bounded; on a timeout the CTA raises the device error
 * word, every role leaves its loop, the CTA waits out copies and MMAs in
 * flight and frees its tensor memory before it exits.
 */
#include <cudaTypedefs.h>

#include <cstdlib>
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
constexpr uint32_t kSI = 4;                  /* super-blocks of row/token scales in flight */
constexpr uint32_t kCtaTiles = 96;           /* tiles of a CTA kept in shared memory       */
constexpr int kMaxSB = 16;                   /* most B (token) stages                      */
constexpr uint32_t kTmemCols = 512;

/* Two arrangements of the same pipeline.
 *  prefill (kDec = false, nt > 32): A1 = b*q4 and A2 = a*q4 in shared memory,
 *    acc = D1 + 16*D2 accumulated over the super-block by the tensor core
 *    (16 MMAs a super-block, the two MMA warps issuing A1 and A2); 16
 *    epilogue warps (four per TMEM lane quarter, a quarter of the tokens
 *    each), 4 producer warps (one row each, both halves of a super-block);
 *    TMEM: D1/D2 for nt <= 128, double buffered.
 *  decode (kDec = true, nt <= 32): A = the raw nibbles as bytes and one
 *    accumulator per sub-block, D_j = q4 . q8 over its 32 K, so a super-block
 *    takes 8 MMAs; the epilogue forms acc = sum_j sc_j * D_j (exact).  At few
 *    tokens per expert a tcgen05.mma costs about the same whatever N, so the
 *    instruction count, not the arithmetic, sets the pace.  4 epilogue warps,
 *    8 producer warps (one row each, one half of every super-block), a deeper
 *    raw-weight ring; TMEM: 8 accumulators x 32 columns, double buffered. */
template <bool kDec>
struct UCfg {
    static constexpr int kEpi = kDec ? 4 : 16;
    static constexpr int kProd = kDec ? 8 : 4;
    static constexpr int kSR = kDec ? 5 : 3;                   /* raw weight ring (super-blocks)      */
    static constexpr int kSA = kDec ? 4 : 3;  /* A stages: decode 2 per half super-block, prefill 3 shared */
    static constexpr int kAStage = kDec ? kOp : 2 * kOp;       /* A, or A1|A2                         */
    static constexpr int kBBytes = kDec ? 32 * 1024 : 48 * 1024; /* B ring: as many nt-token stages as fit */
    static constexpr int kRowInfo = kM * (kDec ? 32 : 16);    /* d, dmin, m0..3, m4..7 (, sc0..3, sc4..7) */
    static constexpr int kWarpMma = kEpi + kProd;  /* two MMA-issuing warps: kWarpMma, kWarpMma + 1 */
    static constexpr int kWarpLoad = kWarpMma + 2;
    static constexpr int kThreads = (kWarpLoad + 1) * 32;
    static constexpr int kOffA = 0;
    static constexpr int kOffB = kOffA + kSA * kAStage;
    static constexpr int kOffR = kOffB + kBBytes;
    static constexpr int kOffT = kOffR + kSR * kRawSlot;
    static constexpr int kOffW = kOffT + kSI * kTokInfo;
    static constexpr int kSmem = kOffW + kSI * kRowInfo;
    static constexpr uint32_t kDbuf = 256u;             /* TMEM columns of one accumulator buffer   */
    static constexpr uint32_t kDstep = kDec ? 32u : 128u; /* D_j (decode) / D2 (prefill) column step */
};
constexpr uint32_t kNtDecode = 32; /* largest token block of the decode arrangement */
static_assert(UCfg<false>::kSmem <= 227 * 1024 && UCfg<true>::kSmem <= 227 * 1024, "shared memory");

/* Instruction descriptor, kind::i8: D s32 (bits 4-5 = 2), A u8 (7-9 = 0),
 * B s8 (10-12 = 1), both K-major, M >> 4 at bits 24-28; N >> 3 goes to 17-22. */
constexpr uint32_t kIdescBase = (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(kM >> 4) << 24);

using UTile = LfmUTile;
using UTokBlock = LfmUTokBlock;

struct UmmaArgs {
    const uint8_t *W;     /* expert tensors [E][rows][nb] Q4_K */
    uint32_t rows, nb;
    const uint8_t *xt;    /* pre-gathered tokens [block][nb][xt_sb_bytes(nt)] */
    uint32_t nt;          /* tokens per block (MMA N): a multiple of 16, <= 128 */
    uint32_t nsb;         /* B stages of nt * 128 bytes in the B ring (<= kMaxSB) */
    const UTile *tiles;
    const UTokBlock *tbs;
    const int32_t *n_tiles;
    float *Y[2];          /* [slots][rows] per matrix */
    uint32_t *err;
};

struct UmmaBars {
    uint64_t a_full[4], a_empty[4], b_full[kMaxSB], b_empty[kMaxSB], r_full[8], r_empty[8];
    uint64_t t_full[2], t_empty[2], ti_full[kSI], ri_full[kSI], i_empty[kSI];
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
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t (&v)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "r"(taddr));
}
/* N = 4 or 8 consecutive 32-bit columns of this thread's TMEM lane. */
template <int N>
__device__ __forceinline__ void tmem_ldn(uint32_t taddr, uint32_t (&v)[N]) {
    if constexpr (N == 8) tmem_ld8(taddr, v);
    else tmem_ld4(taddr, v);
}
template <int N>
__device__ __forceinline__ void tmem_tien(uint32_t (&a)[N]) {
    if constexpr (N == 8)
        asm volatile("" : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7])::"memory");
    else
        asm volatile("" : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3])::"memory");
}
/* Wait for this thread's TMEM loads; the registers are tied to the wait so no
 * use of them is scheduled before it. */
__device__ __forceinline__ void tmem_wait(uint32_t (&a)[8], uint32_t (&b)[8]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]),
                   "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7])::"memory");
}

/* Tie registers to a completed tcgen05.wait::ld so no use is scheduled before it. */
__device__ __forceinline__ void tmem_tie(uint32_t (&a)[8]) {
    asm volatile("" : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7])::"memory");
}

/* Two fp32 lanes at once (fma/mul .rn.ftz .f32x2): the same IEEE operations
 * as the scalar forms, lane by lane. */
__device__ __forceinline__ uint64_t pk2(float x, float y) {
    return (uint64_t)__float_as_uint(x) | ((uint64_t)__float_as_uint(y) << 32);
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.ftz.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.ftz.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

/* mins = sum_j m_j * bsum_j from the token's sub-block sums (pairs) and the row's m bytes. */
__device__ __forceinline__ int mins_of(const uint4 bp, uint32_t mA, uint32_t mB) {
    int m = __dp2a_lo((int)bp.x, (int)mA, 0);
    m = __dp2a_hi((int)bp.y, (int)mA, m);
    m = __dp2a_lo((int)bp.z, (int)mB, m);
    return __dp2a_hi((int)bp.w, (int)mB, m);
}

__device__ __forceinline__ void sts128(uint8_t *p, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(lfm_smem_u32(p)), "r"(x), "r"(y), "r"(z), "r"(w)
                 : "memory");
}

/* Bounded wait that also gives up once another role has aborted. */
__device__ __forceinline__ bool uwait(uint64_t *bar, uint32_t parity, volatile int *abort, uint32_t *err) {
    if (lfm_mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = lfm_globaltimer();
    while (!lfm_mbar_try_wait_sleep(bar, parity, LFM_WAIT_SLEEP_NS)) {
        if (*abort) return false;
        if (lfm_globaltimer() - t0 > LFM_WAIT_LIMIT_NS) {
            atomicOr(err, LFM_DEVERR_TIMEOUT);
            *abort = 1;
            return false;
        }
    }
    return true;
}

template <bool kDec, bool kEp>
__global__ void __launch_bounds__(UCfg<kDec>::kThreads, 1) k_q4k_umma(const __grid_constant__ CUtensorMap tmw0,
                                                          const __grid_constant__ CUtensorMap tmw1, UmmaArgs A,
                                                          const __grid_constant__ UmmaEpOut ep) {
    using C = UCfg<kDec>;
    extern __shared__ __align__(1024) uint8_t sm[];
    __shared__ UmmaBars bars;
    __shared__ UTile s_tile[kCtaTiles];    /* this CTA's tiles, in walking order */
    __shared__ UTokBlock s_blk[kCtaTiles]; /* and their token blocks           */
    __shared__ float *s_yh[LFM_EP_MAX_RANKS];  /* home ranks' output rows (expert parallelism) */
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (kEp && tid < LFM_EP_MAX_RANKS) s_yh[tid] = ep.yhome[tid];
    if (tid == 0) {
        /* decode: each half super-block feeds one MMA stream; prefill: both streams read every stage */
        for (int i = 0; i < C::kSA; ++i) {
            lfm_mbar_init(&bars.a_full[i], kM); /* one arrival per row of the half super-block */
            lfm_mbar_init(&bars.a_empty[i], kDec ? 1 : 2);
        }
        for (uint32_t i = 0; i < A.nsb; ++i) {
            lfm_mbar_init(&bars.b_full[i], 1);
            lfm_mbar_init(&bars.b_empty[i], kDec ? 1 : 2);
        }
        for (int i = 0; i < C::kSR; ++i) {
            lfm_mbar_init(&bars.r_full[i], 1);
            lfm_mbar_init(&bars.r_empty[i], C::kProd * 32);
        }
        for (int i = 0; i < 2; ++i) {
            lfm_mbar_init(&bars.t_full[i], 2); /* one commit from each MMA stream */
            lfm_mbar_init(&bars.t_empty[i], C::kEpi);
        }
        for (uint32_t i = 0; i < kSI; ++i) {
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
    const int n_tiles = __ldcg(A.n_tiles);
    const uint32_t my_tiles =
        (int)blockIdx.x < n_tiles ? (uint32_t)(n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / gridDim.x : 0u;
    /* the tile list off the critical path: a dependent global load per super-block would serialise the issue */
    for (uint32_t it = tid; it < my_tiles && it < kCtaTiles; it += blockDim.x) {
        const UTile t = A.tiles[blockIdx.x + it * gridDim.x];
        s_tile[it] = t;
        s_blk[it] = A.tbs[t.tb];
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars.tmem;
    volatile int *abort = &bars.abort;
    const uint32_t nb = A.nb;
    const uint32_t G = my_tiles * nb; /* super-blocks this CTA walks, tile-major */
    auto tile_at = [&](uint32_t it) -> UTile {
        return it < kCtaTiles ? s_tile[it] : A.tiles[blockIdx.x + it * gridDim.x];
    };
    /* Stage slot and phase parity of half h of super-block g; true on a slot's first use.
     * prefill: one ring in half-super-block order (both MMA streams read every stage);
     * decode: one ring per half, so each MMA stream waits on its own barriers in order. */
    auto aslot = [&](uint32_t g, uint32_t h, uint32_t &idx, uint32_t &par) -> bool {
        if constexpr (kDec) {
            constexpr uint32_t n = C::kSA / 2;
            idx = h * n + g % n;
            par = (g / n) & 1u;
            return g < n;
        } else {
            const uint32_t q = 2 * g + h;
            idx = q % C::kSA;
            par = (q / C::kSA) & 1u;
            return q < (uint32_t)C::kSA;
        }
    };
    auto bslot = [&](uint32_t g, uint32_t h, uint32_t &idx, uint32_t &par) -> bool {
        if constexpr (kDec) {
            const uint32_t n = A.nsb / 2;
            idx = h * n + g % n;
            par = (g / n) & 1u;
            return g < n;
        } else {
            const uint32_t q = 2 * g + h;
            idx = q % A.nsb;
            par = (q / A.nsb) & 1u;
            return q < A.nsb;
        }
    };
    uint8_t *sA = sm + C::kOffA, *sB = sm + C::kOffB, *sR = sm + C::kOffR, *sT = sm + C::kOffT, *sW = sm + C::kOffW;

    if (warp < C::kEpi) {
        /* ---------------- epilogue ---------------- */
        constexpr int kCols = kDec ? (int)kNtDecode : kN / (C::kEpi / 4); /* most columns of one warp */
        const int q4 = warp & 3, ch = warp >> 2;
        const int r = 32 * q4 + lane;
        const int half = (int)A.nt / (C::kEpi / 4); /* columns of this warp: [ch * half, ch * half + half) */
        const uint32_t tl = tmem + ((uint32_t)(32 * q4) << 16);
        uint32_t g = 0;
        bool ok = true;
        for (uint32_t it = 0; it < my_tiles && ok; ++it) {
            const UTile tile = tile_at(it);
            const UTokBlock blk = it < kCtaTiles ? s_blk[it] : A.tbs[tile.tb];
            const int nv = min(blk.ntok - ch * half, half); /* valid tokens in this warp's columns */
            float S[kCols];
#pragma unroll
            for (int i = 0; i < kCols; ++i) S[i] = 0.0f;
            for (uint32_t sb = 0; sb < nb; ++sb, ++g) {
                const uint32_t buf = g & 1u, ph = (g >> 1) & 1u;
                /* every decision that leaves a loop is warp-uniform: tcgen05.ld is .sync.aligned */
                ok = __all_sync(LFM_FULL_MASK, uwait(&bars.t_full[buf], ph, abort, A.err) &&
                                                   uwait(&bars.ti_full[g % kSI], (g / kSI) & 1u, abort, A.err) &&
                                                   uwait(&bars.ri_full[g % kSI], (g / kSI) & 1u, abort, A.err));
                if (!ok) break;
                const uint32_t is = g % kSI;
                const uint4 ri = *reinterpret_cast<const uint4 *>(sW + is * C::kRowInfo + r * (kDec ? 32 : 16));
                const uint64_t dd = pk2(__uint_as_float(ri.x), __uint_as_float(ri.x));
                const uint64_t nm = pk2(-__uint_as_float(ri.y), -__uint_as_float(ri.y)); /* -dmin */
                const float *d8s = reinterpret_cast<const float *>(sT + is * kTokInfo) + ch * half;
                const uint4 *bps = reinterpret_cast<const uint4 *>(sT + is * kTokInfo + A.nt * 4) + ch * half;
                int sc[8];
                if constexpr (kDec) {
                    const uint4 r2 = *reinterpret_cast<const uint4 *>(sW + is * C::kRowInfo + r * 32 + 16);
#pragma unroll
                    for (int j = 0; j < 8; ++j) sc[j] = (int)(((j < 4 ? r2.x : r2.y) >> (8 * (j & 3))) & 0xFFu);
                }
                constexpr int kStep = 8; /* columns per TMEM round trip */
#pragma unroll
                for (int c = 0; c < kCols / kStep; ++c) {
                    if (kStep * c < nv) { /* warp-uniform */
                        const uint32_t col = buf * C::kDbuf + (uint32_t)(ch * half) + (uint32_t)(kStep * c);
                        int acc[kStep];
                        if constexpr (kDec) {
                            /* acc = sum_j sc_j * D_j, D_j at column block 32 j */
                            uint32_t v[8][8];
#pragma unroll
                            for (int j = 0; j < 8; ++j) tmem_ld8(tl + col + C::kDstep * j, v[j]);
                            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                            for (int j = 0; j < 8; ++j) tmem_tie(v[j]);
#pragma unroll
                            for (int i = 0; i < 8; ++i) {
                                int a = 0;
#pragma unroll
                                for (int j = 0; j < 8; ++j) a += sc[j] * (int)v[j][i];
                                acc[i] = a;
                            }
                        } else {
                            uint32_t v1[8], v2[8];
                            tmem_ld8(tl + col, v1);
                            tmem_ld8(tl + col + C::kDstep, v2);
                            tmem_wait(v1, v2);
#pragma unroll
                            for (int i = 0; i < 8; ++i) acc[i] = (int)v1[i] + 16 * (int)v2[i];
                        }
                        /* S = fma(d8*d, acc, fma(-(d8*dmin), mins, S)), two tokens a step; a d8 == 0
                         * block has acc = mins = 0 (all its codes are 0) and adds exact zeros */
#pragma unroll
                        for (int i = 0; i < kStep; i += 2) {
                            const int t = kStep * c + i;
                            const float2 d8 = *reinterpret_cast<const float2 *>(d8s + t);
                            const uint64_t d8p = pk2(d8.x, d8.y);
                            const int m0 = mins_of(bps[t], ri.z, ri.w), m1 = mins_of(bps[t + 1], ri.z, ri.w);
                            const uint64_t inner = fma2(mul2(d8p, nm), pk2((float)m0, (float)m1), pk2(S[t], S[t + 1]));
                            const uint64_t out = fma2(mul2(d8p, dd), pk2((float)acc[i], (float)acc[i + 1]), inner);
                            S[t] = __uint_as_float((uint32_t)out);
                            S[t + 1] = __uint_as_float((uint32_t)(out >> 32));
                        }
                    }
                }
                /* the loads above completed (tcgen05.wait::ld): the accumulator may be overwritten */
                __syncwarp();
                if (lane == 0) {
                    lfm_mbar_arrive(&bars.t_empty[buf]);
                    lfm_mbar_arrive(&bars.i_empty[is]);
                }
            }
            if (!ok) break;
            if constexpr (kEp) { /* the row of slot j belongs to a token of home rank ret[j] >> 24 */
                const uint32_t *rt = ep.ret + blk.slot0 + ch * half;
#pragma unroll
                for (int t = 0; t < kCols; ++t)
                    if (t < nv) {
                        const uint32_t v = __ldg(rt + t), hr = v >> 24, a = v & 0xffffffu;
                        if (hr < ep.world && a < ep.max_assign)
                            s_yh[hr][(size_t)a * A.rows + tile.row0 + r] = S[t];
                        else
                            atomicOr(A.err, LFM_DEVERR_SEGMENT);
                    }
            } else {
                float *yb = (tile.mat ? A.Y[1] : A.Y[0]) + (size_t)(blk.slot0 + ch * half) * A.rows + tile.row0 + r;
#pragma unroll
                for (int t = 0; t < kCols; ++t)
                    if (t < nv) yb[(size_t)t * A.rows] = S[t];
            }
        }
        if (!ok) *abort = 1;
    } else if (warp < C::kWarpMma) {
        /* ---------------- producers ---------------- */
        const int pt = tid - C::kEpi * 32;
        const int p = pt & (kM - 1);             /* weight row of the tile                          */
        const int h0 = kDec ? pt / kM : 0;       /* decode: this thread's half of every super-block */
        const int nh = kDec ? 1 : 2;
        const uint32_t rowoff = (uint32_t)(p >> 3) * 128u + (uint32_t)(p & 7) * 16u;
        /* producer 0 issues: the tile's 128 rows x super-block gg (144 bytes at x = 144 * sb) */
        auto issue_raw = [&](uint32_t gg) {
            const UTile tile = tile_at(gg / nb);
            uint64_t *bar = &bars.r_full[gg % C::kSR];
            lfm_mbar_arrive_tx(bar, kRawSlot);
            lfm_tma_load_2d_hint(sR + (gg % C::kSR) * kRawSlot, tile.mat ? &tmw1 : &tmw0, (gg % nb) * kRaw,
                                 (uint32_t)tile.expert * A.rows + tile.row0, bar, lfm_policy_evict_first());
        };
        bool ok = true;
        if (pt == 0)
            for (uint32_t gg = 0; gg < G && gg < C::kSR - 1; ++gg) issue_raw(gg);
        /* every decision that leaves a loop is warp-uniform */
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
            if (h0 == 0) {
                const uint32_t mA = s1 & 0x3F3F3F3Fu;
                const uint32_t mB = ((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u);
                w = g < kSI || uwait(&bars.i_empty[g % kSI], ((g / kSI) & 1u) ^ 1u, abort, A.err);
                if (!__all_sync(LFM_FULL_MASK, w)) { ok = false; break; }
                uint8_t *ri = sW + (g % kSI) * C::kRowInfo + p * (kDec ? 32 : 16);
                sts128(ri, __float_as_uint(lfm_h2f((uint16_t)(hdr.x & 0xFFFFu))),
                       __float_as_uint(lfm_h2f((uint16_t)(hdr.x >> 16))), mA, mB);
                if (kDec) sts128(ri + 16, scA, scB, 0u, 0u);
                lfm_mbar_arrive(&bars.ri_full[g % kSI]);
            }
            for (int hh = 0; hh < nh; ++hh) {
                const uint32_t h = (uint32_t)(h0 + hh);
                uint32_t s, ap;
                const bool first = aslot(g, h, s, ap);
                w = first || uwait(&bars.a_empty[s], ap ^ 1u, abort, A.err);
                if (!__all_sync(LFM_FULL_MASK, w)) { ok = false; break; }
                uint8_t *a1 = sA + s * C::kAStage, *a2 = a1 + kOp;
                const uint32_t scw = h ? scB : scA; /* nibble groups 2h, 2h+1: sub-blocks 4h..4h+3 */
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    const uint32_t slo = (scw >> (16 * cc)) & 0xFFu, shi = (scw >> (16 * cc + 8)) & 0xFFu;
                    const uint32_t bl = slo & 15u, al = slo >> 4, bh = shi & 15u, ah = shi >> 4;
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf) {
                        /* bytes 16*hf.. of nibble group 2h+cc: elements 16*hf.. of sub-blocks 4h+2cc (low
                         * nibbles) and 4h+2cc+1 (high); their 16-byte K chunks within the half: 4cc+hf, 4cc+2+hf */
                        const uint4 w4 = lfm_ld16<true>(raw + 16 + 32 * (2 * h + cc) + 16 * hf);
                        const uint32_t l0 = w4.x & 0x0F0F0F0Fu, l1 = w4.y & 0x0F0F0F0Fu, l2 = w4.z & 0x0F0F0F0Fu,
                                       l3 = w4.w & 0x0F0F0F0Fu;
                        const uint32_t x0 = (w4.x >> 4) & 0x0F0F0F0Fu, x1 = (w4.y >> 4) & 0x0F0F0F0Fu,
                                       x2 = (w4.z >> 4) & 0x0F0F0F0Fu, x3 = (w4.w >> 4) & 0x0F0F0F0Fu;
                        const uint32_t klo = (4 * cc + hf) * kCoreK + rowoff, khi = (4 * cc + 2 + hf) * kCoreK + rowoff;
                        if constexpr (kDec) {
                            /* the nibbles themselves; the scales are applied per sub-block in the epilogue */
                            sts128(a1 + klo, l0, l1, l2, l3);
                            sts128(a1 + khi, x0, x1, x2, x3);
                        } else {
                            /* bytes of a nibble word times a scalar <= 15 stay below 256: no carries */
                            sts128(a1 + klo, l0 * bl, l1 * bl, l2 * bl, l3 * bl);
                            sts128(a2 + klo, l0 * al, l1 * al, l2 * al, l3 * al);
                            sts128(a1 + khi, x0 * bh, x1 * bh, x2 * bh, x3 * bh);
                            sts128(a2 + khi, x0 * ah, x1 * ah, x2 * ah, x3 * ah);
                        }
                    }
                }
                fence_async_smem(); /* generic-proxy writes -> the tensor core's reads */
                lfm_mbar_arrive(&bars.a_full[s]);
            }
            if (ok) lfm_mbar_arrive(&bars.r_empty[g % C::kSR]);
        }
        if (!ok) *abort = 1;
    } else if (warp < C::kWarpLoad) {
        /* ---------------- MMA issue: two streams of independent accumulators ----------------
         * decode: stream h issues the K steps of half h (sub-blocks 4h..4h+3 -> D_4h..D_4h+3);
         * prefill: stream 0 issues A1 -> D1, stream 1 A2 -> D2, each over the whole super-block. */
        const uint32_t st = (uint32_t)(warp - C::kWarpMma);
        if (lane == 0) {
            bool ok = true;
            const uint32_t idesc = kIdescBase | ((A.nt >> 3) << 17), blbo = A.nt * 16u;
            for (uint32_t g = 0; g < G && ok; ++g) {
                const uint32_t buf = g & 1u;
                if (g >= 2 && !uwait(&bars.t_empty[buf], ((g >> 1) & 1u) ^ 1u, abort, A.err)) { ok = false; break; }
                const uint32_t d0 = tmem + buf * C::kDbuf;
                for (uint32_t h = kDec ? st : 0u; h < (kDec ? st + 1 : 2u); ++h) {
                    uint32_t s, ph, sb, pb;
                    aslot(g, h, s, ph);
                    bslot(g, h, sb, pb);
                    /* operands written by threads (fence.proxy.async before their arrival) or by bulk
                     * copies: the barrier alone orders them before the MMA's reads */
                    if (!uwait(&bars.a_full[s], ph, abort, A.err) || !uwait(&bars.b_full[sb], pb, abort, A.err)) {
                        ok = false;
                        break;
                    }
                    const uint32_t b = lfm_smem_u32(sB + sb * A.nt * kHalf);
                    const uint32_t a = lfm_smem_u32(sA + s * C::kAStage) + (kDec ? 0u : st * kOp);
#pragma unroll
                    for (uint32_t k = 0; k < 4; ++k) {
                        const uint64_t bd = udesc(b + 2 * k * blbo, blbo);
                        if constexpr (kDec) {
                            /* K step k of half h = sub-block 4h + k, into its own accumulator */
                            umma_i8(d0 + C::kDstep * (4 * h + k), udesc(a + 2 * k * kCoreK, kCoreK), bd, idesc, 0u);
                        } else {
                            umma_i8(d0 + C::kDstep * st, udesc(a + 2 * k * kCoreK, kCoreK), bd, idesc, (h | k) ? 1u : 0u);
                        }
                    }
                    umma_commit(&bars.a_empty[s]);
                    umma_commit(&bars.b_empty[sb]);
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
                const UTile tile = tile_at(g / nb);
                const uint32_t opb = A.nt * kHalf; /* one half super-block of the block's codes */
                const uint8_t *src = A.xt + ((size_t)tile.tb * nb + g % nb) * xt_sb_bytes(A.nt);
                const uint32_t is = g % kSI;
                if (g >= kSI && !uwait(&bars.i_empty[is], ((g / kSI) & 1u) ^ 1u, abort, A.err)) { ok = false; break; }
                lfm_mbar_arrive_tx(&bars.ti_full[is], A.nt * 20u);
                lfm_bulk_g2s_plain(sT + is * kTokInfo, src + 2 * opb, A.nt * 20u, &bars.ti_full[is]);
                for (uint32_t h = 0; h < 2; ++h) {
                    uint32_t s, bp;
                    const bool first = bslot(g, h, s, bp);
                    if (!first && !uwait(&bars.b_empty[s], bp ^ 1u, abort, A.err)) {
                        ok = false;
                        break;
                    }
                    lfm_mbar_arrive_tx(&bars.b_full[s], opb);
                    lfm_bulk_g2s_plain(sB + s * opb, src + h * opb, opb, &bars.b_full[s]);
                }
            }
            if (!ok) *abort = 1;
        }
    }

    if (kEp) __threadfence_system(); /* this thread's peer stores, before the CTA counts itself done */
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
    if (kEp && tid == 0 && atomicAdd(ep.done, 1u) == gridDim.x - 1) {
        /* the last CTA: every row of this rank is stored at its home rank */
        atomicExch(ep.done, 0u);
        __threadfence_system();
        const uint32_t epoch = __ldcg(ep.step) + 1u;
        for (uint32_t p = 0; p < ep.world; ++p) lfm_st_release_sys(ep.y_flag[p] + ep.rank, epoch);
    }
}

/* ---------------------------------------------------------------------------
 * The same GEMM with the weight operand in tensor memory.
 *
 * Expander warps (one thread per weight row = TMEM lane) unpack each super-
 * block straight from the raw Q4_K tile into TMEM with tcgen05.st:
 * A1 = b_j * q4 and A2 = a_j * q4 (sc_j = 16 a_j + b_j), so acc = D1 + 16 D2
 * over the super-block exactly as above, and the MMA reads A from TMEM
 * (tcgen05.mma ... [a-tmem]).  Shared memory then carries only the raw
 * weights (TMA), their one read by the expanders and the token operand: the
 * nibble-to-byte operand never makes a shared-memory round trip.
 *
 * Input ring: slot s holds one super-block's A operand (TMEM columns
 * 128 s .. 128 s + 127: per half h, A1 in 64 h + 0..31 and A2 in 64 h + 32..63,
 * the half's K bytes 4c..4c+3 in column c, i.e. the element order of the
 * token operand: 32-byte chunk 2h low nibbles, its high nibbles, chunk 2h+1
 * low, high) and its token operand (both halves, one bulk copy).  The
 * expanders and the token loader fill a slot together (one in_full
 * barrier); one commit per MMA stream releases it (in_empty).  So per
 * super-block each MMA thread waits twice, issues 8 MMAs back to back and
 * commits twice.
 *
 * TMEM: the A slots (as many as the accumulator buffers leave room for: two
 * buffers of 2*nt columns, D1 | D2, leave 3 slots for nt <= 32 and 2 for
 * nt <= 64), then the accumulators.
 *
 * Decode variant (kDec, token blocks of 16): A is the raw nibbles (64 TMEM
 * columns a super-block, no scale multiply) and every 32-wide sub-block j gets
 * its own accumulator D_j = q4 . q8 (8 x 16 columns a buffer), so a super-block
 * takes 8 MMAs instead of 16; MMA stream s issues the four sub-blocks of half
 * s, so the streams never share an accumulator.  The epilogue forms
 * acc = sum_j sc_j * D_j exactly.  At a few tokens per expert the round trip
 * MMA -> epilogue -> free buffer and the issue slots the warps share set the
 * pace; every wait therefore suspends the warp (mbarrier try_wait with a
 * time hint) instead of spinning.
 * Warps: epilogue (8 for the decode variant, else 16: two or four per TMEM
 * lane quarter, splitting the tokens), 4 expanders, two MMA-issuing warps (one
 * thread each: A1 -> D1 and A2 -> D2; the first also allocates TMEM), then one
 * warp each for the weight TMA and the token loader.
 * --------------------------------------------------------------------------- */
template <bool kDec>
struct TCfg {
    static constexpr int kEpi = kDec ? 8 : 16;       /* epilogue warps: 2 / 4 per TMEM lane quarter */
    static constexpr int kExp = 4;                   /* expander warps: lane quarter = warp & 3 (with 8,
                                                        two a quarter each taking half of every
                                                        super-block's chunks, the decode GEMM ran
                                                        1.6x slower) */
    static constexpr int kWarpExp = kEpi;
    static constexpr int kWarpMma = kEpi + kExp;     /* two MMA-issuing warps: A1 -> D1, A2 -> D2 */
    static constexpr int kWarpTma = kWarpMma + 2;
    static constexpr int kWarpLoad = kWarpMma + 3;
    static constexpr int kThreads = (kWarpLoad + 1) * 32;
    static constexpr int kSR = 6;                    /* raw weight ring (super-blocks)  */
    static constexpr int kBBytes = 64 * 1024;        /* token operand slots             */
    static constexpr int kRowInfo = kM * (kDec ? 32 : 16); /* d, dmin, m0..3, m4..7 (, sc0..3, sc4..7) per row */
    static constexpr uint32_t kSlotCols = kDec ? 64 : 128; /* TMEM columns of one A slot (a super-block)  */
    static constexpr uint32_t kAccTok = kDec ? 8 : 2;      /* accumulator columns per token in a buffer   */
    static constexpr uint32_t kAccBufs = 2;                /* accumulator buffers (a third measured no
                                                              faster in the decode variant) */
    static constexpr uint32_t kMaxSlotsC = kDec ? 4 : 3;
    static constexpr int kOffB = 0;
    static constexpr int kOffR = kOffB + kBBytes;
    static constexpr int kOffT = kOffR + kSR * kRawSlot;
    static constexpr int kOffW = kOffT + kSI * kTokInfo;
    static constexpr int kSmem = kOffW + kSI * kRowInfo;
};
static_assert(TCfg<false>::kSmem <= 227 * 1024 && TCfg<true>::kSmem <= 227 * 1024, "shared memory");
constexpr uint32_t kNtTm = 64;      /* most tokens per block: two A slots + two 2*nt buffers = 512 columns */
constexpr uint32_t kNtTmDec = 16;   /* token block of the decode variant: four A slots + two 8*16 buffers */
constexpr uint32_t kMaxSlots = 4;
constexpr uint32_t kMaxAccBufs = 3;
static_assert(2 * 128 + 4 * kNtTm <= kTmemCols && 2 * 64 + 3 * 8 * kNtTmDec <= kTmemCols, "tensor memory");
/* input ring slots for nt tokens a block: TMEM (A) and the shared-memory token slots (B) */
template <bool kDec>
__host__ __device__ constexpr uint32_t tm_slots(uint32_t nt) {
    using C = TCfg<kDec>;
    const uint32_t a = (kTmemCols - C::kAccBufs * C::kAccTok * nt) / C::kSlotCols,
                   b = (uint32_t)C::kBBytes / (2 * nt * kHalf);
    const uint32_t n = a < b ? a : b;
    return n < C::kMaxSlotsC ? n : C::kMaxSlotsC;
}

struct TmBars {
    uint64_t in_full[kMaxSlots], in_empty[kMaxSlots], r_full[8], r_empty[8];
    uint64_t t_full[kMaxAccBufs], t_empty[kMaxAccBufs], ti_full[kSI], ri_full[kSI], i_empty[kSI];
    uint32_t tmem;
    int abort;
};

__device__ __forceinline__ void umma_i8_ta(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d),
        "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

/* 16 consecutive 32-bit columns of this thread's TMEM lane. */
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
                 "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
                 "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
                 : "memory");
}

/* 8 consecutive 32-bit columns of this thread's TMEM lane. */
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
                 "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}

template <bool kDec, bool kEp>
__global__ void __launch_bounds__(TCfg<kDec>::kThreads, 1) k_q4k_tm(const __grid_constant__ CUtensorMap tmw0,
                                                         const __grid_constant__ CUtensorMap tmw1, UmmaArgs A,
                                                         const __grid_constant__ UmmaEpOut ep) {
    using C = TCfg<kDec>;
    extern __shared__ __align__(1024) uint8_t sm[];
    __shared__ TmBars bars;
    __shared__ UTile s_tile[kCtaTiles];
    __shared__ UTokBlock s_blk[kCtaTiles];
    __shared__ float *s_yh[LFM_EP_MAX_RANKS];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t nt = A.nt;
    const uint32_t ns = tm_slots<kDec>(nt);
    if (kEp && tid < LFM_EP_MAX_RANKS) s_yh[tid] = ep.yhome[tid];
    if (tid == 0) {
        for (uint32_t i = 0; i < ns; ++i) {
            lfm_mbar_init(&bars.in_full[i], C::kExp + 1); /* the expander warps and the loader's expect_tx */
            lfm_mbar_init(&bars.in_empty[i], 2); /* one commit per MMA stream */
        }
        for (uint32_t i = 0; i < C::kAccBufs; ++i) {
            lfm_mbar_init(&bars.t_full[i], 2);
            lfm_mbar_init(&bars.t_empty[i], C::kEpi);
        }
        for (int i = 0; i < C::kSR; ++i) {
            lfm_mbar_init(&bars.r_full[i], 1);
            lfm_mbar_init(&bars.r_empty[i], C::kExp);
        }
        for (uint32_t i = 0; i < kSI; ++i) {
            lfm_mbar_init(&bars.ti_full[i], 1);
            lfm_mbar_init(&bars.ri_full[i], 4); /* the first expander warp of each lane quarter */
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
    lfm_pdl_launch_dependents();
    lfm_pdl_wait(); /* tile lists, token blocks and outputs belong to the preceding kernels */
    const int n_tiles = __ldcg(A.n_tiles);
    const uint32_t my_tiles =
        (int)blockIdx.x < n_tiles ? (uint32_t)(n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / gridDim.x : 0u;
    for (uint32_t it = tid; it < my_tiles && it < kCtaTiles; it += blockDim.x) {
        const UTile t = A.tiles[blockIdx.x + it * gridDim.x];
        s_tile[it] = t;
        s_blk[it] = A.tbs[t.tb];
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars.tmem;
    volatile int *abort = &bars.abort;
    const uint32_t nb = A.nb;
    const uint32_t G = my_tiles * nb;
    auto tile_at = [&](uint32_t it) -> UTile {
        return it < kCtaTiles ? s_tile[it] : A.tiles[blockIdx.x + it * gridDim.x];
    };
    const uint32_t acc0 = ns * C::kSlotCols;  /* first accumulator column         */
    const uint32_t abuf = C::kAccTok * nt;     /* columns of one accumulator buffer */
    const uint32_t opb = nt * kHalf;    /* one half super-block of the token operand */
    uint8_t *sB = sm + C::kOffB, *sR = sm + C::kOffR, *sT = sm + C::kOffT, *sW = sm + C::kOffW;

    if (warp < C::kEpi) {
        /* ---------------- epilogue ---------------- */
        constexpr int kCols = (kDec ? (int)kNtTmDec : (int)kNtTm) / (C::kEpi / 4);
        const int q4 = warp & 3, ch = warp >> 2;
        const int r = 32 * q4 + lane;
        const int half = (int)nt / (C::kEpi / 4);
        const uint32_t tl = tmem + ((uint32_t)(32 * q4) << 16);
        uint32_t g = 0, buf = 0, ph = 0; /* accumulator buffer ring position and phase */
        bool ok = true;
        for (uint32_t it = 0; it < my_tiles && ok; ++it) {
            const UTile tile = tile_at(it);
            const UTokBlock blk = it < kCtaTiles ? s_blk[it] : A.tbs[tile.tb];
            const int nv = min(blk.ntok - ch * half, half);
            float S[kCols];
#pragma unroll
            for (int i = 0; i < kCols; ++i) S[i] = 0.0f;
            for (uint32_t sb = 0; sb < nb; ++sb, ++g) {
                ok = __all_sync(LFM_FULL_MASK, uwait(&bars.t_full[buf], ph, abort, A.err) &&
                                                   uwait(&bars.ti_full[g % kSI], (g / kSI) & 1u, abort, A.err) &&
                                                   uwait(&bars.ri_full[g % kSI], (g / kSI) & 1u, abort, A.err));
                if (!ok) break;
                tc_fence_after();
                const uint32_t is = g % kSI;
                const uint4 ri = *reinterpret_cast<const uint4 *>(sW + is * C::kRowInfo + r * (kDec ? 32 : 16));
                int sc[8];
                if constexpr (kDec) {
                    const uint4 r2 = *reinterpret_cast<const uint4 *>(sW + is * C::kRowInfo + r * 32 + 16);
#pragma unroll
                    for (int j = 0; j < 8; ++j) sc[j] = (int)(((j < 4 ? r2.x : r2.y) >> (8 * (j & 3))) & 0xFFu);
                }
                const uint64_t dd = pk2(__uint_as_float(ri.x), __uint_as_float(ri.x));
                const uint64_t nm = pk2(-__uint_as_float(ri.y), -__uint_as_float(ri.y)); /* -dmin */
                const float *d8s = reinterpret_cast<const float *>(sT + is * kTokInfo) + ch * half;
                const uint4 *bps = reinterpret_cast<const uint4 *>(sT + is * kTokInfo + nt * 4) + ch * half;
                constexpr int kStep = kCols < 8 ? kCols : 8; /* columns per TMEM round trip */
#pragma unroll
                for (int c = 0; c < kCols / kStep; ++c) {
                    if (kStep * c < nv) { /* warp-uniform */
                        const uint32_t col = acc0 + buf * abuf + (uint32_t)(ch * half) + (uint32_t)(kStep * c);
                        int acc[kStep];
                        if constexpr (kDec) {
                            /* acc = sum_j sc_j * D_j, D_j at column block j * nt */
                            uint32_t v[8][kStep];
#pragma unroll
                            for (int j = 0; j < 8; ++j) tmem_ldn<kStep>(tl + col + (uint32_t)j * nt, v[j]);
                            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                            for (int j = 0; j < 8; ++j) tmem_tien<kStep>(v[j]);
#pragma unroll
                            for (int i = 0; i < kStep; ++i) {
                                int a = 0;
#pragma unroll
                                for (int j = 0; j < 8; ++j) a += sc[j] * (int)v[j][i];
                                acc[i] = a;
                            }
                        } else {
                            uint32_t v1[8], v2[8];
                            tmem_ld8(tl + col, v1);
                            tmem_ld8(tl + col + nt, v2);
                            tmem_wait(v1, v2);
#pragma unroll
                            for (int i = 0; i < 8; ++i) acc[i] = (int)v1[i] + 16 * (int)v2[i];
                        }
#pragma unroll
                        for (int i = 0; i < kStep; i += 2) {
                            const int t = kStep * c + i;
                            const float2 d8 = *reinterpret_cast<const float2 *>(d8s + t);
                            const uint64_t d8p = pk2(d8.x, d8.y);
                            const int m0 = mins_of(bps[t], ri.z, ri.w), m1 = mins_of(bps[t + 1], ri.z, ri.w);
                            const uint64_t inner = fma2(mul2(d8p, nm), pk2((float)m0, (float)m1), pk2(S[t], S[t + 1]));
                            const uint64_t out = fma2(mul2(d8p, dd), pk2((float)acc[i], (float)acc[i + 1]), inner);
                            S[t] = __uint_as_float((uint32_t)out);
                            S[t + 1] = __uint_as_float((uint32_t)(out >> 32));
                        }
                    }
                }
                /* the loads above completed (tcgen05.wait::ld): the buffer may be overwritten */
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    lfm_mbar_arrive(&bars.t_empty[buf]);
                    lfm_mbar_arrive(&bars.i_empty[is]);
                }
                if (++buf == C::kAccBufs) { buf = 0; ph ^= 1u; }
            }
            if (!ok) break;
            if constexpr (kEp) {
                const uint32_t *rt = ep.ret + blk.slot0 + ch * half;
#pragma unroll
                for (int t = 0; t < kCols; ++t)
                    if (t < nv) {
                        const uint32_t v = __ldg(rt + t), hr = v >> 24, a = v & 0xffffffu;
                        if (hr < ep.world && a < ep.max_assign)
                            s_yh[hr][(size_t)a * A.rows + tile.row0 + r] = S[t];
                        else
                            atomicOr(A.err, LFM_DEVERR_SEGMENT);
                    }
            } else {
                float *yb = (tile.mat ? A.Y[1] : A.Y[0]) + (size_t)(blk.slot0 + ch * half) * A.rows + tile.row0 + r;
#pragma unroll
                for (int t = 0; t < kCols; ++t)
                    if (t < nv) yb[(size_t)t * A.rows] = S[t];
            }
        }
        if (!ok) *abort = 1;
    } else if (warp < C::kWarpMma) {
        /* ---------------- expanders: raw Q4_K rows -> A1 | A2 in TMEM ---------------- */
        const int q4 = warp & 3;
        const int eh = C::kExp > 4 ? (warp - C::kWarpExp) >> 2 : 0; /* which expander of the lane quarter */
        const int p = 32 * q4 + lane;                     /* weight row of the tile = TMEM lane */
        const uint32_t tl = tmem + ((uint32_t)(32 * q4) << 16);
        bool ok = true;
        uint32_t slot = 0, spar = 0, rs = 0, rpar = 0;
        for (uint32_t g = 0; g < G && ok; ++g) {
            ok = __all_sync(LFM_FULL_MASK, uwait(&bars.r_full[rs], rpar, abort, A.err));
            if (!ok) break;
            const uint8_t *raw = sR + rs * kRawSlot + p * kRaw;
            const uint4 hdr = lfm_ld16<true>(raw);
            const uint32_t s0 = hdr.y, s1 = hdr.z, s2 = hdr.w;
            const uint32_t scA = s0 & 0x3F3F3F3Fu;
            const uint32_t scB = (s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u);
            const uint32_t mA = s1 & 0x3F3F3F3Fu;
            const uint32_t mB = ((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u);
            if (eh == 0) { /* the row's scales for the epilogue */
                ok = __all_sync(LFM_FULL_MASK,
                                g < kSI || uwait(&bars.i_empty[g % kSI], ((g / kSI) & 1u) ^ 1u, abort, A.err));
                if (!ok) break;
                uint8_t *rinfo = sW + (g % kSI) * C::kRowInfo + p * (kDec ? 32 : 16);
                sts128(rinfo, __float_as_uint(lfm_h2f((uint16_t)(hdr.x & 0xFFFFu))),
                       __float_as_uint(lfm_h2f((uint16_t)(hdr.x >> 16))), mA, mB);
                if (kDec) sts128(rinfo + 16, scA, scB, 0u, 0u);
                __syncwarp();
                if (lane == 0) lfm_mbar_arrive(&bars.ri_full[g % kSI]);
            }
            ok = __all_sync(LFM_FULL_MASK, g < ns || uwait(&bars.in_empty[slot], spar ^ 1u, abort, A.err));
            if (!ok) break;
            tc_fence_after();
            const uint32_t abase = tl + slot * C::kSlotCols;
            if constexpr (kDec) {
                /* the nibbles themselves: chunk hc's low nibbles in columns 16hc.., high in 16hc+8..;
                 * expander eh of the quarter takes its share of the four chunks */
                constexpr int kHc = 4 / (C::kExp / 4); /* chunks per expander warp */
#pragma unroll
                for (int hc = kHc * eh; hc < kHc * eh + kHc; ++hc) {
                    const uint4 w0 = lfm_ld16<true>(raw + 16 + 32 * hc);
                    const uint4 w1 = lfm_ld16<true>(raw + 16 + 32 * hc + 16);
                    const uint32_t wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
                    uint32_t v[16]; /* low nibbles, then high nibbles: 16 columns, one store */
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        v[i] = wv[i] & 0x0F0F0F0Fu;
                        v[8 + i] = (wv[i] >> 4) & 0x0F0F0F0Fu;
                    }
                    tmem_st16(abase + 16 * hc, v);
                }
            } else
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t scw = h ? scB : scA; /* sub-blocks 4h..4h+3 */
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) { /* 32-byte chunk 2h + cc: sub-blocks 4h+2cc (low), 4h+2cc+1 (high) */
                    const uint32_t slo = (scw >> (16 * cc)) & 0xFFu, shi = (scw >> (16 * cc + 8)) & 0xFFu;
                    const uint32_t bl = slo & 15u, al = slo >> 4, bh = shi & 15u, ah = shi >> 4;
                    const uint4 w0 = lfm_ld16<true>(raw + 16 + 32 * (2 * h + cc));
                    const uint4 w1 = lfm_ld16<true>(raw + 16 + 32 * (2 * h + cc) + 16);
                    const uint32_t wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
                    const uint32_t c0 = abase + 64 * h + 16 * cc;
                    uint32_t v1[16], v2[16]; /* A1, A2: low-nibble columns then high-nibble columns */
                    /* bytes of a nibble word times a scalar <= 15 stay below 256: no carries */
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const uint32_t lo = wv[i] & 0x0F0F0F0Fu, hi = (wv[i] >> 4) & 0x0F0F0F0Fu;
                        v1[i] = lo * bl;
                        v2[i] = lo * al;
                        v1[8 + i] = hi * bh;
                        v2[8 + i] = hi * ah;
                    }
                    tmem_st16(c0, v1);
                    tmem_st16(c0 + 32, v2);
                }
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                lfm_mbar_arrive(&bars.in_full[slot]);
                lfm_mbar_arrive(&bars.r_empty[rs]);
            }
            if (++slot == ns) { slot = 0; spar ^= 1u; }
            if (++rs == (uint32_t)C::kSR) { rs = 0; rpar ^= 1u; }
        }
        if (!ok) *abort = 1;
    } else if (warp < C::kWarpTma) {
        /* ---------------- MMA issue: stream 0 A1 -> D1, stream 1 A2 -> D2 ----------------
         * Ring positions advance by counters (no runtime division in these
         * single-thread loops), and the operand descriptors are a base plus
         * constant offsets. */
        const uint32_t stream = (uint32_t)(warp - C::kWarpMma);
        if (lane == 0) {
            bool ok = true;
            const uint32_t idesc = kIdescBase | ((nt >> 3) << 17), blbo = nt * 16u;
            const uint64_t bdesc0 = udesc(lfm_smem_u32(sB), blbo);
            const uint32_t dstep = (2 * blbo) >> 4;      /* one K step (32 bytes) in descriptor address units */
            const uint32_t hstep = opb >> 4;             /* one half super-block                              */
            const uint32_t aoff = tmem + stream * 32u;   /* A1 or A2 columns of a half                         */
            uint32_t slot = 0, spar = 0, g = 0, buf = 0, bpar = 0;
            for (uint32_t it = 0; it < my_tiles && ok; ++it) {
                for (uint32_t sbk = 0; sbk < nb; ++sbk, ++g) {
                    if ((g >= C::kAccBufs && !uwait(&bars.t_empty[buf], bpar ^ 1u, abort, A.err)) ||
                        !uwait(&bars.in_full[slot], spar, abort, A.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t bd = bdesc0 + (uint64_t)(slot * 2 * hstep);
                    if constexpr (kDec) {
                        /* half `stream`: sub-block 4 s + k into its own accumulator */
                        const uint32_t d = tmem + acc0 + buf * abuf + 4 * stream * nt;
                        const uint32_t a = tmem + slot * C::kSlotCols + 32 * stream;
                        const uint64_t bh = bd + stream * hstep;
#pragma unroll
                        for (uint32_t k = 0; k < 4; ++k) umma_i8_ta(d + k * nt, a + 8 * k, bh + k * dstep, idesc, 0u);
                    } else {
                        const uint32_t d = tmem + acc0 + buf * abuf + stream * nt;
                        const uint32_t a = aoff + slot * C::kSlotCols;
#pragma unroll
                        for (uint32_t h = 0; h < 2; ++h)
#pragma unroll
                            for (uint32_t k = 0; k < 4; ++k)
                                umma_i8_ta(d, a + 64 * h + 8 * k, bd + h * hstep + k * dstep, idesc, (h | k) ? 1u : 0u);
                    }
                    umma_commit(&bars.in_empty[slot]);
                    umma_commit(&bars.t_full[buf]);
                    if (++slot == ns) { slot = 0; spar ^= 1u; }
                    if (++buf == C::kAccBufs) { buf = 0; bpar ^= 1u; }
                }
            }
            if (!ok) *abort = 1;
        }
    } else if (warp == C::kWarpTma) {
        /* ---------------- weight TMA: the tile's 128 rows x super-block ---------------- */
        if (lane == 0) {
            bool ok = true;
            uint32_t rs = 0, rpar = 0, g = 0;
            const uint64_t policy = lfm_policy_evict_first(); /* weights are read once a layer */
            for (uint32_t it = 0; it < my_tiles && ok; ++it) {
                const UTile tile = tile_at(it);
                const CUtensorMap *tm = tile.mat ? &tmw1 : &tmw0;
                const uint32_t row = (uint32_t)tile.expert * A.rows + tile.row0;
                for (uint32_t sbk = 0; sbk < nb; ++sbk, ++g) {
                    if (g >= (uint32_t)C::kSR && !uwait(&bars.r_empty[rs], rpar ^ 1u, abort, A.err)) { ok = false; break; }
                    lfm_mbar_arrive_tx(&bars.r_full[rs], kRawSlot);
                    lfm_tma_load_2d_hint(sR + rs * kRawSlot, tm, sbk * kRaw, row, &bars.r_full[rs], policy);
                    if (++rs == (uint32_t)C::kSR) { rs = 0; rpar ^= 1u; }
                }
            }
            if (!ok) *abort = 1;
        }
    } else {
        /* ---------------- loader: the token operand (both halves, one copy) and scales ---------------- */
        if (lane == 0) {
            bool ok = true;
            uint32_t slot = 0, spar = 0, g = 0;
            for (uint32_t it = 0; it < my_tiles && ok; ++it) {
                const UTile tile = tile_at(it);
                const uint8_t *src0 = A.xt + (size_t)tile.tb * nb * xt_sb_bytes(nt);
                for (uint32_t sbk = 0; sbk < nb; ++sbk, ++g) {
                    const uint8_t *src = src0 + (size_t)sbk * xt_sb_bytes(nt);
                    const uint32_t is = g % kSI;
                    if ((g >= kSI && !uwait(&bars.i_empty[is], ((g / kSI) & 1u) ^ 1u, abort, A.err)) ||
                        (g >= ns && !uwait(&bars.in_empty[slot], spar ^ 1u, abort, A.err))) {
                        ok = false;
                        break;
                    }
                    lfm_mbar_arrive_tx(&bars.ti_full[is], nt * 20u);
                    lfm_bulk_g2s_plain(sT + is * kTokInfo, src + 2 * opb, nt * 20u, &bars.ti_full[is]);
                    lfm_mbar_arrive_tx(&bars.in_full[slot], 2 * opb);
                    lfm_bulk_g2s_plain(sB + slot * 2 * opb, src, 2 * opb, &bars.in_full[slot]);
                    if (++slot == ns) { slot = 0; spar ^= 1u; }
                }
            }
            if (!ok) *abort = 1;
        }
    }

    if (kEp) __threadfence_system();
    tc_fence_before();
    __syncthreads();
    if (*abort) {
        const uint64_t t0 = lfm_globaltimer();
        while (lfm_globaltimer() - t0 < 2000000ull) {
        }
    }
    if (warp == C::kWarpMma) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
    if (kEp && tid == 0 && atomicAdd(ep.done, 1u) == gridDim.x - 1) {
        atomicExch(ep.done, 0u);
        __threadfence_system();
        const uint32_t epoch = __ldcg(ep.step) + 1u;
        for (uint32_t p = 0; p < ep.world; ++p) lfm_st_release_sys(ep.y_flag[p] + ep.rank, epoch);
    }
}

/* Launch `fn` with the programmatic-dependent-launch attribute when pdl is set. */
template <typename... Args>
static cudaError_t launch_pdl(void (*fn)(Args...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, fn, args...);
}

/* Tokens of every block, per super-block, in the MMA's canonical K-major
 * layout: half h (K bytes 128h..128h+127) is 8 chunks of 16 K bytes x nt
 * tokens, token t's 16 bytes at chunk*16*nt + 16*t (= 8-token groups of 128
 * bytes); then d8 per token and the sub-block sums bsum[2j] + bsum[2j+1]
 * packed two per word (j = 0..7).  Tokens past the block's count are zero. */
struct XtRow {
    const int8_t *qs; /* the token's Q8_K row: values, scales, sums */
    const float *d;
    const int16_t *bs;
};

/* Copy super-block sb of the block's ntok tokens (row pointers in shared
 * memory) into the block's pre-gathered layout. */
constexpr uint32_t kXtThreads = 256;
__device__ __forceinline__ void xt_copy_block(const XtRow *rows, int ntok, uint32_t sb, uint32_t nt, uint8_t *dst) {
    /* all loads first, then the stores: the rows may sit on another GPU, where
     * a load takes microseconds, so every thread keeps all of its in flight */
    constexpr uint32_t kIt = kN * 16 / kXtThreads;
    uint4 v[kIt];
#pragma unroll
    for (uint32_t i = 0; i < kIt; ++i) {
        const uint32_t q = threadIdx.x + i * kXtThreads, c = q / nt, t = q % nt;
        v[i] = make_uint4(0u, 0u, 0u, 0u);
        if (q < nt * 16 && (int)t < ntok) v[i] = __ldcg(reinterpret_cast<const uint4 *>(rows[t].qs + 256 * sb + 16 * c));
    }
#pragma unroll
    for (uint32_t i = 0; i < kIt; ++i) {
        const uint32_t q = threadIdx.x + i * kXtThreads, c = q / nt, t = q % nt;
        if (q < nt * 16) *reinterpret_cast<uint4 *>(dst + (c >> 3) * nt * kHalf + (c & 7) * 16 * nt + 16 * t) = v[i];
    }
    if (threadIdx.x < nt) {
        const int t = threadIdx.x;
        float d8 = 0.0f;
        uint4 pr = make_uint4(0u, 0u, 0u, 0u);
        if (t < ntok) {
            d8 = __ldcg(rows[t].d + sb);
            const uint4 *bp = reinterpret_cast<const uint4 *>(rows[t].bs + 16 * sb);
            const uint4 b0 = __ldcg(bp), b1 = __ldcg(bp + 1);
            const uint32_t bw[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) { /* bsum pairs (4i, 4i+1) and (4i+2, 4i+3) */
                const int lo = (int)(int16_t)(bw[2 * i] & 0xffffu) + (int)(int16_t)(bw[2 * i] >> 16);
                const int hi = (int)(int16_t)(bw[2 * i + 1] & 0xffffu) + (int)(int16_t)(bw[2 * i + 1] >> 16);
                w[i] = (uint32_t)(uint16_t)lo | ((uint32_t)(uint16_t)hi << 16);
            }
            pr = make_uint4(w[0], w[1], w[2], w[3]);
        }
        reinterpret_cast<float *>(dst + 2 * nt * kHalf)[t] = d8;
        reinterpret_cast<uint4 *>(dst + 2 * nt * kHalf + nt * 4)[t] = pr;
    }
}

__global__ void __launch_bounds__(kXtThreads) k_xt_gather(Q8Rows X, const int32_t *perm, uint32_t K, const UTokBlock *tbs,
                                                   const int32_t *n_tb, uint32_t nb, uint32_t nt, uint8_t *xt) {
    __shared__ XtRow rows[kN];
    lfm_pdl_launch_dependents();
    lfm_pdl_wait();
    const int tb = blockIdx.x;
    if (tb >= __ldcg(n_tb)) return;
    const uint32_t sb = blockIdx.y;
    const UTokBlock blk = tbs[tb];
    if (threadIdx.x < kN && (int)threadIdx.x < blk.ntok) {
        const int t = threadIdx.x;
        const size_t row = perm ? (size_t)(__ldcg(perm + blk.slot0 + t) / (int)K) : (size_t)(blk.slot0 + t);
        rows[t] = XtRow{X.qs + row * X.cols, X.d + row * nb, X.bs + row * nb * 16};
    }
    __syncthreads();
    xt_copy_block(rows, blk.ntok, sb, nt, xt + ((size_t)tb * nb + sb) * xt_sb_bytes(nt));
}

/* Expert parallelism: the block's received slots name their home rank and
 * the home rank's slot; the Q8_K rows are read from the home rank's memory
 * (over NVLink) with one bulk copy per token and super-block (256 code bytes,
 * 32 bytes of sums) into shared memory, then laid out like k_xt_gather.  The
 * sb == 0 CTAs also record each slot's assignment t*K+k at home, where the
 * down GEMM stores the output row. */
constexpr uint32_t kGxRow = 256 + 16; /* padded smem row: 16-byte chunks of consecutive tokens hit distinct banks */
struct GatherSmem {
    uint8_t qs[kN * kGxRow];
    int16_t bs[kN * 16];
    float d8[kN];
    uint64_t bar;
    int ok;
};
__global__ void __launch_bounds__(kXtThreads) k_xt_gather_ep(EpGather g, const UTokBlock *tbs, const int32_t *n_tb,
                                                             uint32_t nb, uint32_t nt, uint8_t *xt) {
    extern __shared__ __align__(128) uint8_t gx_raw[];
    GatherSmem &S = *reinterpret_cast<GatherSmem *>(gx_raw);
    lfm_pdl_launch_dependents();
    lfm_pdl_wait(); /* the plan (token blocks, rowmap) belongs to the preceding kernel */
    const int tb = blockIdx.x;
    if (tb >= __ldcg(n_tb)) return;
    const uint32_t sb = blockIdx.y, cols = nb * 256;
    const UTokBlock blk = tbs[tb];
    const int ntok = blk.ntok;
    if (threadIdx.x == 0) {
        lfm_mbar_init(&S.bar, 1);
        lfm_fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x < kN && (int)threadIdx.x < ntok) {
        const int t = threadIdx.x;
        const uint32_t v = __ldcg(g.rowmap + blk.slot0 + t);
        uint32_t r = v >> 24, a = 0;
        if (r < g.world && (v & 0xffffffu) < g.max_assign) a = (uint32_t)__ldcg(g.perm[r] + (v & 0xffffffu));
        if (r >= g.world || a >= g.max_assign) { /* a plan or perm entry out of range: read row 0 of rank 0 */
            atomicOr(g.err, LFM_DEVERR_SEGMENT);
            r = 0;
            a = 0;
        }
        const size_t row = a / g.K;
        if (sb == 0) g.ret[blk.slot0 + t] = (r << 24) | a;
        if (t == 0) lfm_mbar_arrive_tx(&S.bar, (uint32_t)ntok * (256u + 32u));
        __syncwarp(__activemask()); /* the expected bytes are posted before any copy of warp 0 lands */
        lfm_bulk_g2s_plain(S.qs + t * kGxRow, g.qs[r] + row * cols + 256 * sb, 256u, &S.bar);
        lfm_bulk_g2s_plain(S.bs + t * 16, g.bs[r] + (row * nb + sb) * 16, 32u, &S.bar);
        S.d8[t] = __ldcg(g.d[r] + row * nb + sb);
    }
    if (threadIdx.x == 0) S.ok = ntok <= 0 || lfm_mbar_wait(&S.bar, 0, g.err) ? 1 : 0;
    __syncthreads();
    if (!S.ok) { /* copies in flight land within microseconds: let them before the CTA's memory goes */
        const uint64_t t0 = lfm_globaltimer();
        while (lfm_globaltimer() - t0 < 2000000ull) {
        }
        return;
    }
    uint8_t *dst = xt + ((size_t)tb * nb + sb) * xt_sb_bytes(nt);
    for (uint32_t q = threadIdx.x; q < nt * 16; q += kXtThreads) {
        const uint32_t c = q / nt, t = q % nt;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if ((int)t < ntok) v = *reinterpret_cast<const uint4 *>(S.qs + t * kGxRow + 16 * c);
        *reinterpret_cast<uint4 *>(dst + (c >> 3) * nt * kHalf + (c & 7) * 16 * nt + 16 * t) = v;
    }
    if (threadIdx.x < nt) {
        const int t = threadIdx.x;
        float d8 = 0.0f;
        uint4 pr = make_uint4(0u, 0u, 0u, 0u);
        if (t < ntok) {
            d8 = S.d8[t];
            const int16_t *bs = S.bs + t * 16;
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

/* Q8_K of one 256-value block held 8 per lane (elements 8*lane..) -- the
 * quantiser of lfm_quant_block_warp, value for value -- written as token t of
 * a pre-gathered block (the layout k_xt_gather writes). */
__device__ __forceinline__ void quant_block_xt(const float v[8], uint8_t *dst, uint32_t nt, uint32_t t) {
    const int lane = threadIdx.x & 31;
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = lfm_warp_max(amax);
    int q[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int part = 0;
    if (amax != 0.0f) {
        const float s = __fdiv_rn(127.0f, amax);
#pragma unroll
        for (int i = 0; i < 8; ++i) { q[i] = __float2int_rn(__fmul_rn(v[i], s)); part += q[i]; }
    }
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        lo |= (uint32_t)(uint8_t)(int8_t)max(-128, min(127, q[i])) << (8 * i);
        hi |= (uint32_t)(uint8_t)(int8_t)max(-128, min(127, q[4 + i])) << (8 * i);
    }
    /* elements 8*lane..8*lane+7: half (8*lane)/128, 16-byte K chunk ((8*lane) % 128) / 16, bytes 8*(lane & 1).. */
    const uint32_t k = 8u * lane;
    *reinterpret_cast<uint2 *>(dst + (k >> 7) * nt * kHalf + ((k & 127) >> 4) * 16 * nt + 16 * t + (k & 15)) =
        make_uint2(lo, hi);
    /* sub-block sums (32 codes, unsaturated): lanes 4j..4j+3; pairs (2i, 2i+1) packed per word */
    int sum4 = part + __shfl_xor_sync(LFM_FULL_MASK, part, 1);
    sum4 += __shfl_xor_sync(LFM_FULL_MASK, sum4, 2);
    const int odd = __shfl_down_sync(LFM_FULL_MASK, sum4, 4);
    if ((lane & 7) == 0)
        reinterpret_cast<uint32_t *>(dst + 2 * nt * kHalf + nt * 4 + 16 * t)[lane >> 3] =
            (uint32_t)(uint16_t)sum4 | ((uint32_t)(uint16_t)odd << 16);
    if (lane == 0) reinterpret_cast<float *>(dst + 2 * nt * kHalf)[t] = amax == 0.0f ? 0.0f : __fdiv_rn(amax, 127.0f);
}

/* h = (g / (1 + exp(-g))) * u (tools/lfm2_decode_1x4.c:976-985), quantised to
 * Q8_K per 256 and written straight into the down GEMM's pre-gathered token
 * blocks (the slots of a block are consecutive); one warp per (token, 256
 * block), eight tokens of a token block per CTA. */
__global__ void __launch_bounds__(256) k_swiglu_xt(const float *__restrict__ G, const float *__restrict__ U,
                                                   uint32_t cols, const UTokBlock *tbs, const int32_t *n_tb,
                                                   uint32_t nt, uint8_t *xt) {
    lfm_pdl_launch_dependents();
    lfm_pdl_wait();
    const int tb = blockIdx.x / (nt / 8);
    if (tb >= __ldcg(n_tb)) return;
    const uint32_t sb = blockIdx.y, nb = cols / 256;
    const UTokBlock blk = tbs[tb];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t *dst = xt + ((size_t)tb * nb + sb) * xt_sb_bytes(nt);
    {
        const uint32_t t = (blockIdx.x % (nt / 8)) * 8 + warp;
        float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if ((int)t < blk.ntok) {
            const size_t o = (size_t)(blk.slot0 + t) * cols + 256 * sb + 8 * lane;
            const float4 g0 = __ldcg(reinterpret_cast<const float4 *>(G + o)), g1 = __ldcg(reinterpret_cast<const float4 *>(G + o) + 1);
            const float4 u0 = __ldcg(reinterpret_cast<const float4 *>(U + o)), u1 = __ldcg(reinterpret_cast<const float4 *>(U + o) + 1);
            const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
            const float u[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(__fdiv_rn(g[i], __fadd_rn(1.0f, lfm_silu_expf(-g[i]))), u[i]);
        }
        quant_block_xt(v, dst, nt, t);
    }
}

}  // namespace

bool lfm_umma_ok(uint32_t rows) { return rows % kM == 0; }
uint32_t lfm_umma_nt(uint32_t slots, uint32_t experts) {
    /* about three times the mean tokens per expert, so most experts fit one block;
     * at decode sizes (a mean of up to 8) blocks of 16 for the per-sub-block variant */
    const uint32_t mean = (slots + experts - 1) / (experts ? experts : 1u);
    if (mean <= 8) return kNtTmDec;
    const uint32_t nt = (3 * mean + 15) / 16 * 16;
    return nt < 16 ? 16u : nt > kNtTm ? kNtTm : nt;
}
size_t lfm_umma_tb_max(uint32_t slots, uint32_t experts, uint32_t nt) { return (slots + nt - 1) / nt + experts; }
size_t lfm_umma_tiles_max(uint32_t rows, uint32_t slots, uint32_t experts, uint32_t nt) {
    return (size_t)(rows / kM) * lfm_umma_tb_max(slots, experts, nt);
}
size_t lfm_umma_xt_bytes(size_t max_tb, uint32_t nb, uint32_t nt) { return max_tb * nb * (size_t)xt_sb_bytes(nt); }

cudaError_t lfm_launch_xt_gather(Q8Rows X, const int32_t *perm, uint32_t K, const void *tbs, const int32_t *n_tb,
                                 uint32_t max_tb, uint32_t nt, uint8_t *xt, cudaStream_t s, bool pdl) {
    const uint32_t nb = X.cols / 256;
    if (max_tb == 0 || nb == 0) return cudaSuccess;
    return launch_pdl(k_xt_gather, dim3(max_tb, nb), dim3(kXtThreads), 0, s, pdl, X, perm, K,
                      static_cast<const UTokBlock *>(tbs), n_tb, nb, nt, xt);
}

cudaError_t lfm_launch_xt_gather_ep(const EpGather &g, uint32_t cols, const void *tbs, const int32_t *n_tb,
                                    uint32_t max_tb, uint32_t nt, uint8_t *xt, cudaStream_t s, bool pdl) {
    const uint32_t nb = cols / 256;
    if (max_tb == 0 || nb == 0) return cudaSuccess;
    static size_t cache[16];
    const cudaError_t e = lfm_smem_attr((const void *)k_xt_gather_ep, sizeof(GatherSmem), cache);
    if (e != cudaSuccess) return e;
    return launch_pdl(k_xt_gather_ep, dim3(max_tb, nb), dim3(kXtThreads), sizeof(GatherSmem), s, pdl, g,
                      static_cast<const UTokBlock *>(tbs), n_tb, nb, nt, xt);
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

cudaError_t lfm_launch_swiglu_xt(const float *G, const float *U, uint32_t cols, const void *tbs, const int32_t *n_tb,
                                 uint32_t max_tb, uint32_t nt, uint8_t *xt, cudaStream_t s, bool pdl) {
    const uint32_t nb = cols / 256;
    if (max_tb == 0 || nb == 0) return cudaSuccess;
    return launch_pdl(k_swiglu_xt, dim3(max_tb * (nt / 8), nb), dim3(256), 0, s, pdl, G, U, cols,
                      static_cast<const UTokBlock *>(tbs), n_tb, nt, xt);
}

template <bool kDec, bool kEp>
static cudaError_t launch_tm(const CUtensorMap &tm0, const CUtensorMap &tm1, const UmmaArgs &a, const UmmaEpOut &ep,
                             int grid, cudaStream_t s, bool pdl) {
    using C = TCfg<kDec>;
    static size_t cache[16];
    const cudaError_t e = lfm_smem_attr((const void *)k_q4k_tm<kDec, kEp>, C::kSmem, cache);
    if (e != cudaSuccess) return e;
    return launch_pdl(k_q4k_tm<kDec, kEp>, dim3(grid), dim3(C::kThreads), C::kSmem, s, pdl, tm0, tm1, a, ep);
}

template <bool kDec, bool kEp>
static cudaError_t launch_umma(const CUtensorMap &tm0, const CUtensorMap &tm1, const UmmaArgs &a,
                               const UmmaEpOut &ep, int grid, cudaStream_t s) {
    using C = UCfg<kDec>;
    static size_t cache[16];
    const cudaError_t e = lfm_smem_attr((const void *)k_q4k_umma<kDec, kEp>, C::kSmem, cache);
    if (e != cudaSuccess) return e;
    k_q4k_umma<kDec, kEp><<<grid, C::kThreads, C::kSmem, s>>>(tm0, tm1, a, ep);
    return cudaGetLastError();
}

cudaError_t lfm_launch_q4k_umma(const uint8_t *W0, const uint8_t *W1, uint32_t experts, uint32_t rows, uint32_t cols,
                                const uint8_t *xt, uint32_t nt, const void *tiles, const void *tbs,
                                const int32_t *n_tiles, float *Y0, float *Y1, uint32_t *err, int grid, cudaStream_t s,
                                const UmmaEpOut *ep, bool pdl) {
    if (rows % kM || cols % 256 || experts == 0 || nt % 16 || nt == 0 || nt > (uint32_t)kN)
        return cudaErrorInvalidValue;
    if (ep && (!ep->ret || !ep->done || !ep->step || ep->world == 0 || ep->world > LFM_EP_MAX_RANKS)) return cudaErrorInvalidValue;
    /* each expert tensor as a 2-D byte matrix [experts * rows][nb * 144] */
    CUtensorMap tm0, tm1;
    const uint64_t row_bytes = (uint64_t)(cols / 256) * kRaw;
    if (!lfm_tmap_2d(&tm0, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, W0, row_bytes, (uint64_t)experts * rows, row_bytes, kRaw, kM) ||
        !lfm_tmap_2d(&tm1, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, W1, row_bytes, (uint64_t)experts * rows, row_bytes, kRaw, kM))
        return cudaErrorInvalidValue;
    const bool dec = nt <= kNtDecode;
    const UmmaEpOut eo = ep ? *ep : UmmaEpOut{};
    static const bool smem_a = [] { /* the shared-memory A operand version, for A/B runs */
        const char *v = getenv("LFM_GPU_MOE_UMMA_SMEM_A");
        return v && v[0] == '1';
    }();
    if (!smem_a) {
        const bool tdec = nt <= kNtTmDec;
        if (nt > kNtTm || (tdec ? tm_slots<true>(nt) : tm_slots<false>(nt)) < 2) return cudaErrorInvalidValue;
        UmmaArgs a{W0, rows, cols / 256, xt, nt, 0u, static_cast<const UTile *>(tiles),
                   static_cast<const UTokBlock *>(tbs), n_tiles, {Y0, Y1}, err};
        if (tdec)
            return ep ? launch_tm<true, true>(tm0, tm1, a, eo, grid, s, pdl)
                      : launch_tm<true, false>(tm0, tm1, a, eo, grid, s, pdl);
        return ep ? launch_tm<false, true>(tm0, tm1, a, eo, grid, s, pdl)
                  : launch_tm<false, false>(tm0, tm1, a, eo, grid, s, pdl);
    }
    uint32_t nsb = min((uint32_t)kMaxSB, (uint32_t)(dec ? UCfg<true>::kBBytes : UCfg<false>::kBBytes) / (nt * kHalf));
    if (dec) nsb &= ~1u; /* one B ring per half super-block */
    UmmaArgs a{W0, rows, cols / 256, xt, nt, nsb, static_cast<const UTile *>(tiles), static_cast<const UTokBlock *>(tbs),
               n_tiles, {Y0, Y1}, err};
    if (dec)
        return ep ? launch_umma<true, true>(tm0, tm1, a, eo, grid, s) : launch_umma<true, false>(tm0, tm1, a, eo, grid, s);
    return ep ? launch_umma<false, true>(tm0, tm1, a, eo, grid, s) : launch_umma<false, false>(tm0, tm1, a, eo, grid, s);
}
