/*
 * mla_tc.cu -- paged absorbed-MLA decode on the 5th-generation tensor cores
 * (tcgen05 + TMEM + TMA) for the DeepSeek shape: 128 query heads sharing one
 * cache entry of 576 bf16 values (512 latent + 64 rope), V = the 512 latent
 * values, 64-token pages.
 *
 * Work: the plan's chunks (sequence, page range) are split evenly over
 * n_workers; a worker is a cluster of two CTAs on two SMs that split the
 * entry dimension: CTA r owns latent values [256r, 256r+256) and rope values
 * [512+32r, 544+32r).  Per 64-token page ("tile"):
 *   GEMM1  S_r = Q[:, own 288 dims] . KV[:, own 288 dims]^T  (M=128 heads,
 *          N=64 tokens, K=288) -> TMEM, double-buffered.  The 256 latent dims
 *          of Q are an A operand in TMEM, the 32 rope dims in shared memory;
 *   the two partial S are exchanged: each CTA stages its partial in shared
 *          memory and bulk copies, one per TMEM lane quadrant (32 heads,
 *          8 KB), move it into the peer's receive buffer (the SM-to-SM
 *          network moves ~20 B/clk this way, twice what per-thread remote
 *          stores reach).  a + b is the same float in both
 *          CTAs, so both run the identical softmax on identical scores;
 *   softmax in the log2 domain with a lazily updated row maximum (O is
 *          rescaled only when a row's maximum grows by more than 2^8);
 *          P = bf16 probabilities, written into the shared-memory slot the
 *          peer's partial scores arrived in;
 *   GEMM2  O_r += P . V[:, own 256 latent dims]  (M=128, N=256, K=64), A = P
 *          from that slot, V read MN-major from the same page tile.
 * Four staging warps (one per lane quadrant) copy each tile's partial scores
 * to the exchange buffer as soon as GEMM1 has written them and issue their
 * quadrant's copy themselves, so the exchange of tile j+1 runs while the
 * softmax warps finish tile j, and the softmax warps of a quadrant start
 * when that quadrant's 8 KB have landed; a score buffer is free once the staging
 * and softmax warps have read it, and the MMA warp issues GEMM1 up to two
 * tiles ahead of GEMM2.  The peer's partial scores
 * land in one of two receive slots; a slot is handed back to the peer by the
 * commit of the GEMM2 that read P from it, which arrives on the peer's
 * barrier directly.
 *
 * Roles per CTA (480 threads): warp 0 issues TMA loads, warp 1 owns TMEM and
 * issues the GEMM1s, warp 2 the GEMM2s (one elected thread each; on int8 /
 * e4m3 pages warp 1 issues both and warp 2 is idle), warps 3-10
 * finish scores, softmax and epilogue: two threads per head row (TMEM lane),
 * one per 32-token half of a tile; warps 11-14 stage the partial scores and
 * copy them to the peer (one TMEM lane quadrant each).
 *
 * Shared memory (per CTA): Q rope dims 8 KB (SW64 [128x32]), 3 page stages of
 * 36 KB, an exchange out buffer and two in slots of 32 KB (partial scores,
 * then P), a 3 KB row-statistics buffer, per stage the token scales (256 B)
 * and rope codes (2 KB) of quantised pools, barriers.  TMEM: S at columns 0
 * and 64, Q at 128, O at 256..511.
 *
 * Every wait is bounded (about two seconds of clock); on expiry the kernel
 * records an error word, drains its own TMA loads, copies and MMAs, frees
 * TMEM and returns.  No load uses cluster multicast, and no CTA reads another
 * GPU's memory.
 */
#include "../../include/attention.h"
#include "../../include/hal.h"
#include "../../include/kv_cache.h"
#include "ct_internal.h"
#include "tc_ptx.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

namespace {

constexpr int kH = 128, kE = 576, kDv = 512, kP = 64;
constexpr int kSoftmaxWarps = 8;             /* two per TMEM lane quadrant: 20 warps keep 128 registers */
constexpr int kParts = kSoftmaxWarps / 4;               /* threads per head row (one per TMEM lane quadrant warp) */
constexpr int kTPT = 64 / kParts;                       /* tokens of a page per thread */
constexpr int kOCols = 256 / kParts;                    /* O columns (value dims) per thread */
constexpr int kFirstSoftmaxWarp = 3;
constexpr int kFirstStageWarp = kFirstSoftmaxWarp + kSoftmaxWarps;   /* 4 warps, one per TMEM lane quadrant */
constexpr int kThreads = 32 * (kFirstStageWarp + 4);   /* 480 */
constexpr int kConvWarps = 4;                           /* int8 / e4m3 pools: codes -> bf16 in shared memory */
constexpr int kFirstConvWarp = kFirstStageWarp + 4;
constexpr int kThreadsQ = kThreads + 32 * kConvWarps;   /* 608 */
constexpr int kStages = 3;
constexpr uint32_t kQBytes = 8192;                      /* the rope dims of the half: SW64 [128 x 32] */
constexpr uint32_t kCodeBytes = 4 * 4096 + 2048 + 256;  /* quantised page half: codes + 64 scales */
constexpr uint32_t kKvBytes = 4 * 8192 + 4096;          /* 36,864 per stage */
constexpr uint32_t kXBytes = 32768;                     /* one tile's partial scores, 128 x 64 fp32 */
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffKv = kOffQ + kQBytes;
constexpr uint32_t kOffOut = kOffKv + kStages * kKvBytes;
constexpr uint32_t kOffIn = kOffOut + kXBytes;         /* two receive slots */
constexpr uint32_t kOffRed = kOffIn + 2 * kXBytes;
constexpr uint32_t kRedBytes = 3 * kParts * kH * 4;     /* row max [2 parities][parts], row sum [parts] */
constexpr uint32_t kOffScale = kOffRed + kRedBytes;    /* per stage: 64 fp32 token scales (quantised pools) */
constexpr uint32_t kOffRc = kOffScale + kStages * 256;  /* per stage: the rope codes, 64 x 32 bytes (quantised pools) */
constexpr uint32_t kOffBar = kOffRc + kStages * 2048;
constexpr uint32_t kNumBars = 48;
constexpr uint32_t kOffTmem = kOffBar + kNumBars * 8;
constexpr uint32_t kSmemUsed = kOffTmem + 16;
constexpr uint32_t kSmemAlloc = kSmemUsed + 1024;       /* slack to align the base to 1024 B */
static_assert(kSmemAlloc <= 232448, "shared memory per CTA");
static_assert(kOffKv % 1024 == 0 && kOffOut % 1024 == 0 && kOffIn % 1024 == 0, "swizzle atoms need 1 KB alignment");
static_assert(kOffRc % 128 == 0, "TMA destination alignment");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemS = 0;      /* 2 x 64 columns: fp32 scores */
constexpr uint32_t kTmemQ = 128;    /* 128 columns, bf16 query latent dims of the half */
constexpr uint32_t kTmemO = 256;    /* 256 columns, fp32 output accumulator */
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;
constexpr long long kWaitCycles = 4000000000LL;         /* ~2 s at 2 GHz */

/* barrier slots */
enum : uint32_t {
    B_KV_FULL = 0, B_KV_EMPTY = 3, B_Q_FULL = 6, B_Q_EMPTY = 7, B_QT_FULL = 8, B_S_FULL = 9, B_P_FULL = 11,
    B_O_READY = 13, B_O_FINAL = 14, B_O_FREE = 15, B_X_EMPTY = 16 /* [slot] */, B_DRAIN = 18,
    B_RED = 19 /* [parity][quad] */, B_RED_L = 27 /* [quad] */,
    B_CONV_FULL = 31 /* [stage]: page converted to bf16 (quantised pools) */,
    B_S_EMPTY = 34 /* [score buffer]: the softmax warps have read the scores */,
    B_X_FULL = 36 /* [slot][quad]: the peer's partial scores of a quadrant's rows have landed */,
    B_DRAIN2 = 44 /* the GEMM2 thread's MMAs (bf16 pages) */
};

/* instruction descriptors: f32 accumulate, bf16 A and B, M = 128 */
constexpr uint32_t kIdescS = (1u << 4) | (1u << 7) | (1u << 10) | ((64u >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t kIdescO = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((256u >> 3) << 17) | ((128u >> 4) << 24);

__device__ int g_mla_tc_error;                          /* 0 = ok; else the code of the first failed wait */

using namespace ct_tc;

/* ---- shared state of one CTA ------------------------------------------- */

struct Ctx {
    uint8_t *smem;          /* 1024-aligned base */
    uint32_t s;             /* its shared address */
    uint32_t peer;          /* the other CTA's rank */
    volatile int *abort;    /* set by a thread whose wait expired */
};

__device__ __forceinline__ uint32_t bar(const Ctx &c, uint32_t i) { return c.s + kOffBar + 8 * i; }

/* Bounded wait; returns false (and raises the abort flag) on expiry. */
__device__ bool wait_bar(const Ctx &c, uint32_t b, uint32_t parity, bool cluster_scope, int code) {
    long long t0 = clock64();
    for (;;) {
        if (cluster_scope ? mbar_try_cluster(b, parity) : mbar_try(b, parity)) return true;
        if (*c.abort) return false;
        if (clock64() - t0 > kWaitCycles) {
            atomicCAS(&g_mla_tc_error, 0, code);
            *c.abort = 1;
            return false;
        }
    }
}

struct Params {
    const ct_mla_chunk_t *chunks;
    const int32_t *worker_begin;
    const int32_t *bt;
    const int32_t *lens;
    const uint16_t *q;
    uint16_t *out;
    float *lse;
    float *part_o;
    float *part_ml;
    const float *scales;     /* quantised pools: fp32 per token, [n_pages][64] */
    uint32_t maxp;
    uint32_t n_pages;
    float qk_scale;          /* scale * log2(e) */
    int out32;               /* out is 32-B aligned: the epilogue writes whole sectors */
};

/* Warp-cooperative walk over the pages of a chunk that hold tokens: lanes
 * read 32 consecutive block-table entries with one coalesced load, a ballot
 * marks the usable pages (page id in [0, n_pages), at least one token), and
 * next() hands them out in order.  All 32 lanes call it together; every
 * role walks the same list. */
struct WarpTiles {
    const int32_t *bt_row;
    int32_t len, next_lp, end, base, my_pg;
    uint32_t n_pages, mask;
    __device__ __forceinline__ void init(const ct_mla_chunk_t &ch, const Params &p) {
        bt_row = p.bt + (size_t)ch.row * p.maxp;
        len = p.lens[ch.row];
        next_lp = ch.page_begin;
        end = ch.page_end;
        n_pages = p.n_pages;
        mask = 0;
        base = 0;
        my_pg = -1;
    }
    __device__ __forceinline__ bool next(int32_t &pg, int32_t &ntok) {
        const int32_t lane = (int32_t)(threadIdx.x & 31);
        while (mask == 0) {
            if (next_lp >= end) return false;
            base = next_lp;
            const int32_t cur = base + lane;
            int32_t v = -1, n = 0;
            if (cur < end) {
                v = __ldg(bt_row + cur);
                n = min(kP, len - cur * kP);
            }
            my_pg = v;
            mask = __ballot_sync(0xFFFFFFFFu, cur < end && n > 0 && v >= 0 && (uint32_t)v < n_pages);
            next_lp = base + 32;
        }
        const int i = __ffs(mask) - 1;
        mask &= mask - 1;
        pg = __shfl_sync(0xFFFFFFFFu, my_pg, i);
        ntok = min(kP, len - (base + i) * kP);
        return true;
    }
};

__device__ __forceinline__ ct_mla_chunk_t load_chunk(const Params &p, int ci) {
    const int4 *src = reinterpret_cast<const int4 *>(p.chunks + ci);
    const int4 a = __ldg(src), b = __ldg(src + 1);
    ct_mla_chunk_t ch;
    ch.seq = a.x; ch.row = a.y; ch.page_begin = a.z; ch.page_end = a.w;
    ch.part = b.x; ch.pad[0] = b.y; ch.pad[1] = b.z; ch.pad[2] = b.w;
    return ch;
}

/* Tiles of a chunk (warp-collective): the pages WarpTiles would hand out,
 * counted with all of the chunk's block-table loads in flight at once (16
 * per lane), so that a role starting a chunk of hundreds of pages does not
 * wait for one load per 32 pages in turn. */
__device__ __forceinline__ uint32_t count_tiles(const ct_mla_chunk_t &ch, const Params &p) {
    const int32_t *row = p.bt + (size_t)ch.row * p.maxp;
    const int32_t len = p.lens[ch.row];
    const int32_t lim = len > 0 ? (int32_t)min((int64_t)ch.page_end, ((int64_t)len + kP - 1) / kP) : 0;
    const int32_t lane = (int32_t)(threadIdx.x & 31);
    uint32_t cnt = 0;
    for (int32_t b = ch.page_begin + lane; b < lim; b += 32 * 16) {
        int32_t v[16];
        #pragma unroll
        for (int k = 0; k < 16; k++) v[k] = b + 32 * k < lim ? __ldg(row + b + 32 * k) : -1;
        #pragma unroll
        for (int k = 0; k < 16; k++) cnt += (v[k] >= 0 && (uint32_t)v[k] < p.n_pages) ? 1u : 0u;
    }
    return __reduce_add_sync(0xFFFFFFFFu, cnt);
}

/* ---- warp 0: TMA producer (lane 0 issues) -------------------------------- */

template <int KV>
__device__ void producer(const Ctx &c, const Params &p, const CUtensorMap *kv_lat, const CUtensorMap *kv_rope,
                         const CUtensorMap *q_rope, int wbeg, int wend, uint32_t rank) {
    constexpr bool kQuant = KV != CT_KV_BF16;
    const bool leader = (threadIdx.x & 31) == 0;
    uint32_t g = 0;
    bool ok = true;
    /* The queries of a chunk (128 heads x 576 values) go into L2 ahead of
     * the staging warps, which load them into TMEM when the previous chunk's
     * GEMM1s are done; the first chunk's as early as possible. */
    if (leader && wbeg < wend) bulk_prefetch_l2(p.q + (size_t)load_chunk(p, wbeg).seq * kH * kE, kH * kE * 2);
    for (int ci = wbeg; ci < wend && ok; ci++) {
        const ct_mla_chunk_t ch = load_chunk(p, ci);
        WarpTiles it;
        it.init(ch, p);
        int32_t pg, ntok;
        if (!it.next(pg, ntok)) continue;               /* nothing readable in this chunk */
        /* L2 prefetch three pages ahead of the page being loaded: a load waits
         * for its stage until GEMM2 frees it, ~2 tiles later, and then reads
         * from L2 instead of paying the HBM latency in that loop */
        WarpTiles ah;
        ah.init(ch, p);
        int32_t apg, antok;
        bool ah_ok = ah.next(apg, antok);
        auto prefetch = [&](int32_t pgx) {
            if ((threadIdx.x & 31) == 0) {
                for (int b = 0; b < 4; b++) tma_prefetch_2d(kv_lat, rank * 256 + b * 64, pgx * kP);
                tma_prefetch_2d(kv_rope, 512 + rank * 32, pgx * kP);
            }
        };
        for (int a = 0; a < 2 && ah_ok; a++) {
            ah_ok = ah.next(apg, antok);
            if (ah_ok) prefetch(apg);
        }
        /* the next chunk's queries when the look-ahead reaches the end of
         * this chunk, ~6 tiles before the staging warps load them: earlier,
         * a long chunk's page stream would evict them from L2 again (the
         * staging warps also issue the rope dims' TMA load, so this loop
         * never waits for the previous chunk's GEMM1s) */
        bool q_next = ci + 1 < wend;
        auto prefetch_q_next = [&]() {
            if (!q_next) return;
            const int32_t nseq = load_chunk(p, ci + 1).seq;
            if (leader) bulk_prefetch_l2(p.q + (size_t)nseq * kH * kE, kH * kE * 2);
            q_next = false;
        };
        if (!ah_ok) prefetch_q_next();
        do {
            const uint32_t st = g % kStages;
            if (leader) {
                ok = wait_bar(c, bar(c, B_KV_EMPTY + st), ((g / kStages) & 1) ^ 1, false, 2);
                if (ok) {
                    const uint32_t dst = c.s + kOffKv + st * kKvBytes, fb = bar(c, B_KV_FULL + st);
                    const int y = pg * kP;
                    if (!kQuant) {
                        mbar_expect_tx(fb, kKvBytes);
                        for (int b = 0; b < 4; b++) tma_load_2d(dst + b * 8192, kv_lat, rank * 256 + b * 64, y, fb);
                        tma_load_2d(dst + 4 * 8192, kv_rope, 512 + rank * 32, y, fb);
                    } else {
                        /* 8-bit latent codes into the upper half of each bf16 box
                         * (the converter widens them in place), the rope codes
                         * beside the stages, and the page's scales */
                        mbar_expect_tx(fb, kCodeBytes);
                        for (int b = 0; b < 4; b++)
                            tma_load_2d(dst + b * 8192 + 4096, kv_lat, rank * 256 + b * 64, y, fb);
                        tma_load_2d(c.s + kOffRc + st * 2048, kv_rope, 512 + rank * 32, y, fb);
                        bulk_load(c.s + kOffScale + st * 256, p.scales + (size_t)pg * kP, 256, fb);
                    }
                }
            }
            ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
            if (!ok) break;
            if (ah_ok) {
                ah_ok = ah.next(apg, antok);
                if (ah_ok) prefetch(apg);
                else prefetch_q_next();
            }
            g++;
        } while (it.next(pg, ntok));
    }
    if (!leader) return;
    /* Drain: every issued load must have landed before the CTA may exit. */
    for (uint32_t k = 0; k < (uint32_t)kStages && k < g; k++) {
        const uint32_t last = g - 1 - k;
        const uint32_t st = last % kStages;
        long long t0 = clock64();
        while (!mbar_try(bar(c, B_KV_FULL + st), (last / kStages) & 1) && clock64() - t0 < kWaitCycles) {}
    }
}

/* ---- warp 1: MMA issuer (lane 0 issues) ---------------------------------- */

__device__ void issue_gemm1(const Ctx &c, uint32_t tmem, uint32_t st, uint32_t sbuf, int i0, int i1) {
    const uint32_t q = c.s + kOffQ, kv = c.s + kOffKv + st * kKvBytes;
    const uint32_t d = tmem + kTmemS + sbuf * 64;
    /* the 256 latent dims of the half: A from TMEM */
    for (int i = i0; i < i1; i++)
        mma_ts(d, tmem + kTmemQ + i * 8, sdesc(kv + (i >> 2) * 8192 + (i & 3) * 32, 1, 64, kSw128), kIdescS,
               i > 0 ? 1u : 0u);
    if (i1 < 16) return;
    /* rope dims: A from shared memory */
    #pragma unroll
    for (int k = 0; k < 2; k++)
        mma_ss(d, sdesc(q + k * 32, 1, 32, kSw64), sdesc(kv + 4 * 8192 + k * 32, 1, 32, kSw64), kIdescS, 1);
}

/* P of a tile sits in the receive slot its peer scores came in: rows of 8
 * heads (8 x 128 B, SW128 K-major) every 2048 B, so that the rows a TMEM
 * lane quadrant writes lie over partial scores that quadrant has read. */
__device__ void issue_gemm2(const Ctx &c, uint32_t tmem, uint32_t st, uint32_t slot, bool first) {
    const uint32_t v = c.s + kOffKv + st * kKvBytes, pa = c.s + kOffIn + slot * kXBytes;
    #pragma unroll
    for (int k = 0; k < 4; k++)
        mma_ss(tmem + kTmemO, sdesc(pa + k * 32, 1, 2048 / 16, kSw128), sdesc(v + k * 2048, 512, 64, kSw128), kIdescO,
               (first && k == 0) ? 0u : 1u);
}

template <int KV>
__device__ void mma_issuer(const Ctx &c, const Params &p, uint32_t tmem, int wbeg, int wend) {
    constexpr uint32_t kPageReady = KV == CT_KV_BF16 ? B_KV_FULL : B_CONV_FULL;
    const bool leader = (threadIdx.x & 31) == 0;
    uint32_t g = 0, nchunk = 0;
    bool ok = true;
    for (int ci = wbeg; ci < wend && ok; ci++) {
        const ct_mla_chunk_t ch = load_chunk(p, ci);
        const uint32_t n = count_tiles(ch, p);
        if (n == 0) continue;
        if (leader) {
            /* both parts of this chunk's Q: the TMA half and the TMEM half */
            ok = wait_bar(c, bar(c, B_Q_FULL), nchunk & 1, false, 3) &&
                 wait_bar(c, bar(c, B_QT_FULL), nchunk & 1, false, 3);
            tc_fence_after();
            /* Issue whichever GEMM is ready, GEMM2 first (it frees a page
             * stage and the peer's copy into a receive slot).  GEMM1 of tile
             * t+2 reuses the score columns of tile t once the softmax warps
             * have read them, and runs at most two tiles ahead of GEMM2. */
            uint32_t n1 = 0, n2 = 0;
            long long t0 = clock64();
            auto try_g2 = [&]() -> bool {
                if (n2 < n1) {
                    const uint32_t gt = g + n2;
                    if (mbar_test(bar(c, B_P_FULL + (gt & 1)), (gt >> 1) & 1) &&
                        (n2 > 0 || mbar_test(bar(c, B_O_FREE), (nchunk & 1) ^ 1))) {
                        tc_fence_after();
                        issue_gemm2(c, tmem, gt % kStages, gt & 1, n2 == 0);
                        mma_commit(bar(c, B_KV_EMPTY + gt % kStages));
                        mma_commit(bar(c, B_O_READY));
                        mma_commit_to(bar(c, B_X_EMPTY + (gt & 1)), (uint16_t)(1u << c.peer));   /* P read */
                        n2++;
                        return true;
                    }
                }
                return false;
            };
            while (ok && n2 < n) {
                bool did = try_g2();
                if (n1 < n && n1 <= n2 + 2) {
                    const uint32_t gt = g + n1;
                    if (mbar_test(bar(c, kPageReady + gt % kStages), (gt / kStages) & 1) &&
                        mbar_test(bar(c, B_S_EMPTY + (gt & 1)), ((gt >> 1) & 1) ^ 1)) {
                        tc_fence_after();
                        /* in two halves: the issuing thread is held at the MMA
                         * rate, so a P that becomes ready meanwhile gets its
                         * GEMM2 between them instead of after all 18 MMAs */
                        issue_gemm1(c, tmem, gt % kStages, gt & 1, 0, 8);
                        try_g2();
                        issue_gemm1(c, tmem, gt % kStages, gt & 1, 8, 16);
                        mma_commit(bar(c, B_S_FULL + (gt & 1)));
                        if (n1 == n - 1) mma_commit(bar(c, B_Q_EMPTY));
                        n1++;
                        did = true;
                    }
                }
                if (did) {
                    t0 = clock64();
                } else if (*c.abort) {
                    ok = false;
                } else if (clock64() - t0 > kWaitCycles) {
                    atomicCAS(&g_mla_tc_error, 0, n2 < n1 ? 7 : 5);
                    *c.abort = 1;
                    ok = false;
                }
            }
            if (ok) mma_commit(bar(c, B_O_FINAL));
        }
        ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
        g += n;
        nchunk++;
    }
    if (!leader) return;
    /* Drain the tensor pipe before TMEM is released. */
    mma_commit(bar(c, B_DRAIN));
    long long t0 = clock64();
    while (!mbar_try(bar(c, B_DRAIN), 0) && clock64() - t0 < kWaitCycles) {}
}

/* GEMM1 of every tile, in order, as soon as its page is in shared memory
 * and its score buffer has been read (warp 1, one elected thread). */
template <int KV>
__device__ void gemm1_issuer(const Ctx &c, const Params &p, uint32_t tmem, int wbeg, int wend) {
    constexpr uint32_t kPageReady = KV == CT_KV_BF16 ? B_KV_FULL : B_CONV_FULL;
    const bool leader = (threadIdx.x & 31) == 0;
    uint32_t g = 0, nchunk = 0;
    bool ok = true;
    for (int ci = wbeg; ci < wend && ok; ci++) {
        const ct_mla_chunk_t ch = load_chunk(p, ci);
        const uint32_t n = count_tiles(ch, p);
        if (n == 0) continue;
        if (leader) {
            /* both parts of this chunk's Q: the TMA half and the TMEM half */
            ok = wait_bar(c, bar(c, B_Q_FULL), nchunk & 1, false, 3) &&
                 wait_bar(c, bar(c, B_QT_FULL), nchunk & 1, false, 3);
            for (uint32_t j = 0; j < n && ok; j++) {
                const uint32_t gt = g + j;
                ok = wait_bar(c, bar(c, kPageReady + gt % kStages), (gt / kStages) & 1, false, 5) &&
                     wait_bar(c, bar(c, B_S_EMPTY + (gt & 1)), ((gt >> 1) & 1) ^ 1, false, 5);
                if (!ok) break;
                tc_fence_after();
                issue_gemm1(c, tmem, gt % kStages, gt & 1, 0, 16);
                mma_commit(bar(c, B_S_FULL + (gt & 1)));
                if (j == n - 1) mma_commit(bar(c, B_Q_EMPTY));
            }
        }
        ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
        g += n;
        nchunk++;
    }
    if (!leader) return;
    /* Drain this thread's MMAs before TMEM is released. */
    mma_commit(bar(c, B_DRAIN));
    long long t0 = clock64();
    while (!mbar_try(bar(c, B_DRAIN), 0) && clock64() - t0 < kWaitCycles) {}
}

/* GEMM2 of every tile, in order, as soon as its P is written (warp 2, one
 * elected thread): a thread of its own, so that a ready P never waits
 * behind the issue of a GEMM1, which the tensor pipe holds back at its
 * execution rate.  The first GEMM2 of a chunk also waits until the
 * epilogue has read the previous chunk's O. */
__device__ void gemm2_issuer(const Ctx &c, const Params &p, uint32_t tmem, int wbeg, int wend) {
    const bool leader = (threadIdx.x & 31) == 0;
    uint32_t g = 0, nchunk = 0;
    bool ok = true;
    for (int ci = wbeg; ci < wend && ok; ci++) {
        const ct_mla_chunk_t ch = load_chunk(p, ci);
        const uint32_t n = count_tiles(ch, p);
        if (n == 0) continue;
        if (leader) {
            for (uint32_t j = 0; j < n && ok; j++) {
                const uint32_t gt = g + j;
                ok = wait_bar(c, bar(c, B_P_FULL + (gt & 1)), (gt >> 1) & 1, false, 7) &&
                     (j > 0 || wait_bar(c, bar(c, B_O_FREE), (nchunk & 1) ^ 1, false, 7));
                if (!ok) break;
                tc_fence_after();
                issue_gemm2(c, tmem, gt % kStages, gt & 1, j == 0);
                mma_commit(bar(c, B_KV_EMPTY + gt % kStages));
                mma_commit(bar(c, B_O_READY));
                mma_commit_to(bar(c, B_X_EMPTY + (gt & 1)), (uint16_t)(1u << c.peer));   /* P read */
            }
            if (ok) mma_commit(bar(c, B_O_FINAL));
        }
        ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
        g += n;
        nchunk++;
    }
    if (!leader) return;
    mma_commit(bar(c, B_DRAIN2));
    long long t0 = clock64();
    while (!mbar_try(bar(c, B_DRAIN2), 0) && clock64() - t0 < kWaitCycles) {}
}

/* ---- warps 3-10: scores, softmax, epilogue -------------------------------- */

/* A wait all 32 lanes of a softmax warp leave together (the tcgen05 loads
 * and stores that follow are warp-collective). */
__device__ __forceinline__ bool wait_warp(const Ctx &c, uint32_t b, uint32_t parity, bool cluster_scope, int code) {
    const bool r = wait_bar(c, b, parity, cluster_scope, code);
    return __all_sync(0xFFFFFFFFu, r);
}

/* One arrive per warp, after every lane's preceding work. */
__device__ __forceinline__ void warp_arrive(uint32_t b) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(b);
}

/* 2^x by the hardware approximation (relative error ~2^-22; the result is
 * rounded to bf16 for the tensor cores anyway); -inf gives 0. */
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

/* Two floats -> packed bf16 pair (lo in the low half), round to nearest even. */
__device__ __forceinline__ uint32_t bf16x2_rn(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}

/* Swizzled position of 16-byte chunk `c` (0..15) of exchange row `row`. */
__device__ __forceinline__ uint32_t xoff(uint32_t row, uint32_t c) { return row * 256 + ((c ^ (row & 15)) << 4); }

struct Row {
    uint32_t row, part, quad, lane_base, tid;
    float m_used, l;
};

/* Finishes global tile t (index jj in its chunk): adds the peer's partial
 * scores, updates the running maximum, rescales O if needed, writes P. */
template <int KV>
__device__ bool finish_tile(const Ctx &c, const Params &p, uint32_t tmem, Row &r, uint32_t t, uint32_t jj,
                            int32_t ntok) {
    constexpr bool kQuant = KV != CT_KV_BF16;
    const float *tok_scale = reinterpret_cast<const float *>(c.smem + kOffScale + (t % kStages) * 256) + r.part * kTPT;
    float *red = reinterpret_cast<float *>(c.smem + kOffRed);
    const uint32_t slot = t & 1;
    /* this CTA's partial scores of the thread's 16 tokens */
    float s[kTPT];
    if (!wait_warp(c, bar(c, B_S_FULL + slot), (t >> 1) & 1, false, 12)) return false;
    tc_fence_after();
    if constexpr (kTPT == 16) tmem_ld16(tmem + r.lane_base + kTmemS + slot * 64 + r.part * kTPT, s);
    else tmem_ld32(tmem + r.lane_base + kTmemS + slot * 64 + r.part * kTPT, s);
    tmem_wait_ld();
    tc_fence_before();
    warp_arrive(bar(c, B_S_EMPTY + slot));            /* with the stagers': GEMM1 of tile t+2 may overwrite */
    if (!wait_warp(c, bar(c, B_X_FULL + slot * 4 + r.quad), (t >> 1) & 1, true, 10)) return false;
    const float4 *xin = reinterpret_cast<const float4 *>(c.smem + kOffIn + slot * kXBytes);
    #pragma unroll
    for (int q4 = 0; q4 < kTPT / 4; q4++) {
        const float4 w = xin[xoff(r.row, r.part * (kTPT / 4) + q4) >> 4];
        s[4 * q4] += w.x; s[4 * q4 + 1] += w.y; s[4 * q4 + 2] += w.z; s[4 * q4 + 3] += w.w;
    }
    /* arm this quadrant's barrier of the slot for tile t + 2 (8 KB) */
    if (r.part == 0 && (r.tid & 31) == 0) mbar_expect_tx(bar(c, B_X_FULL + slot * 4 + r.quad), kXBytes / 4);
    /* quantised pages: the scores are code dot products; times the token's scale */
    if constexpr (kQuant) {                         /* packed pairs (f32x2), same roundings */
        const float2 *sc2 = reinterpret_cast<const float2 *>(tok_scale);
        #pragma unroll
        for (int k = 0; k < kTPT / 2; k++) {
            const float2 m = __fmul2_rn(make_float2(s[2 * k], s[2 * k + 1]), sc2[k]);
            s[2 * k] = m.x;
            s[2 * k + 1] = m.y;
        }
    }
    /* the last page of a sequence masks the slots past its end (warp-uniform) */
    const bool partial = ntok < kP;
    if (partial) {
        #pragma unroll
        for (int i = 0; i < kTPT; i++)
            if ((int32_t)(r.part * kTPT + i) >= ntok) s[i] = -INFINITY;
    }
    /* row maximum over all parts, of the unscaled scores (the softmax scale is
     * positive, so it commutes with the maximum) */
    float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    #pragma unroll
    for (int i = 0; i < kTPT; i++) m4[i & 3] = fmaxf(m4[i & 3], s[i]);
    float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
    /* the other parts of each row are in the other warps of this quadrant */
    float *rm = red + (t & 1) * kParts * kH;
    rm[r.part * kH + r.row] = mx;
    const uint32_t rb = bar(c, B_RED + (t & 1) * 4 + r.quad);
    warp_arrive(rb);        /* also: the other parts may now write P over the partials this thread read */
    if (!wait_warp(c, rb, (t >> 1) & 1, false, 16)) return false;
    #pragma unroll
    for (int k = 1; k < kParts; k++) mx = fmaxf(mx, rm[((r.part + k) % kParts) * kH + r.row]);
    mx *= p.qk_scale;                                       /* log2 domain */
    const bool grow = mx > r.m_used + kRescaleThreshold;   /* also true for the first tile */
    const float m_new = grow ? mx : r.m_used;
    const float alpha = grow ? ex2_approx(r.m_used - m_new) : 1.0f;   /* 0 on the first tile */
    if (__any_sync(0xFFFFFFFFu, grow && jj > 0)) {
        /* O holds tiles before t: wait for GEMM2(t-1), rescale this thread's part of the row */
        if (!wait_warp(c, bar(c, B_O_READY), (t - 1) & 1, false, 11)) return false;
        tc_fence_after();
        const float a = grow ? alpha : 1.0f;
        #pragma unroll 1
        for (int cc = 0; cc < kOCols / 16; cc++) {
            float o[16];
            uint32_t u[16];
            tmem_ld16(tmem + r.lane_base + kTmemO + r.part * kOCols + cc * 16, o);
            tmem_wait_ld();
            #pragma unroll
            for (int i = 0; i < 16; i++) u[i] = __float_as_uint(o[i] * a);
            tmem_st16(tmem + r.lane_base + kTmemO + r.part * kOCols + cc * 16, u);
        }
        tmem_wait_st();
        tc_fence_before();
    }
    r.l *= alpha;
    r.m_used = m_new;
    /* P = bf16(2^(scale * s - m)) into the receive slot, over partial
     * scores of this quadrant's rows (all four parts have read theirs: the
     * maximum exchange above).  The normaliser sums the fp32 probabilities. */
    uint32_t w[kTPT / 2];
    float l4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const float qk = p.qk_scale, nm = -r.m_used;
    #pragma unroll
    for (int k = 0; k < kTPT / 2; k++) {
        const float p0 = ex2_approx(fmaf(s[2 * k], qk, nm)), p1 = ex2_approx(fmaf(s[2 * k + 1], qk, nm));
        l4[k & 3] += p0 + p1;
        if (!kQuant) {
            w[k] = bf16x2_rn(p0, p1);
        } else if (!partial) {
            /* V = scale x codes: the scale folds into P */
            const float2 ps = __fmul2_rn(make_float2(p0, p1), reinterpret_cast<const float2 *>(tok_scale)[k]);
            w[k] = bf16x2_rn(ps.x, ps.y);
        } else {
            const bool in0 = (int32_t)(r.part * kTPT + 2 * k) < ntok, in1 = (int32_t)(r.part * kTPT + 2 * k + 1) < ntok;
            w[k] = bf16x2_rn(in0 ? p0 * tok_scale[2 * k] : 0.0f, in1 ? p1 * tok_scale[2 * k + 1] : 0.0f);
        }
    }
    r.l += (l4[0] + l4[1]) + (l4[2] + l4[3]);
    {
        uint8_t *pr = c.smem + kOffIn + slot * kXBytes + (r.row >> 3) * 2048 + (r.row & 7) * 128;
        const uint32_t c0 = (kTPT / 8) * r.part, sw = r.row & 7;      /* 16-byte chunks of 8 tokens */
        #pragma unroll
        for (int k = 0; k < kTPT / 8; k++)
            *reinterpret_cast<uint4 *>(pr + (((c0 + k) ^ sw) << 4)) =
                make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
    }
    /* a partial page: zero the V rows past its tokens (stale slots may hold
     * anything; the converter already wrote zeros there for quantised pages) */
    if (!kQuant && ntok < kP) {
        uint8_t *kvs = c.smem + kOffKv + (t % kStages) * kKvBytes;
        const uint32_t per_blk = (uint32_t)(kP - ntok) * 8;          /* 16-B words per box */
        for (uint32_t i = r.tid; i < 4 * per_blk; i += 32 * kSoftmaxWarps) {
            const uint32_t blk = i / per_blk, rem = i % per_blk;
            const uint32_t rr = (uint32_t)ntok + rem / 8, w16 = rem % 8;
            *reinterpret_cast<uint4 *>(kvs + blk * 8192 + rr * 128 + w16 * 16) = make_uint4(0, 0, 0, 0);
        }
    }
    proxy_fence();                                  /* P and zeroed rows -> the tensor core's view */
    tc_fence_before();
    warp_arrive(bar(c, B_P_FULL + (t & 1)));
    return true;
}

/* ---- warps 11-14: staging -------------------------------------------------- */

/* Copies each tile's partial scores (this warp's 32 head rows, all 64
 * tokens) from TMEM to the exchange buffer as soon as GEMM1 has written them,
 * independently of the softmax warps, and sends those 8 KB into the peer's
 * receive slot (one bulk copy, completing on the peer's barrier of this
 * quadrant and slot), so that the exchange of tile t+1 runs while tile t is
 * being finished.  The quadrant's out rows are rewritten only after its
 * previous copy has read them (the issuing lane's bulk group). */
__device__ void stager(const Ctx &c, const Params &p, const CUtensorMap *q_rope, uint32_t tmem, int wbeg, int wend,
                       uint32_t rank) {
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t quad = warp & 3, row = quad * 32 + lane, lane_base = (quad * 32) << 16;
    uint32_t t = 0, nq = 0;
    bool ok = true;
    const uint32_t in_peer = mapa(c.s + kOffIn, c.peer);
    const uint32_t xf_peer = mapa(bar(c, B_X_FULL), c.peer);
    for (int ci = wbeg; ci < wend && ok; ci++) {
        const ct_mla_chunk_t ch = load_chunk(p, ci);
        /* this CTA's 256 latent dims of the chunk's Q (this thread: head
         * `row`) into TMEM as soon as the previous chunk's GEMM1s are done,
         * while the softmax warps may still be finishing that chunk.  The
         * producer prefetched the chunk's queries into L2; the first quarter
         * is loaded before the chunk's pages are counted (a block-table walk)
         * and before that wait.  Quadrant 0 issues the rope dims' TMA load
         * into shared memory. */
        const uint4 *src = reinterpret_cast<const uint4 *>(p.q + ((size_t)ch.seq * kH + row) * kE + rank * 256);
        uint32_t u[32];
        auto load8 = [&](int q64) {
            if (q64 < 3) prefetch_l1(src + (q64 + 1) * 8);     /* the next quarter's 128 bytes */
            #pragma unroll
            for (int k = 0; k < 8; k++) {
                const uint4 x = __ldg(src + q64 * 8 + k);
                u[4 * k] = x.x; u[4 * k + 1] = x.y; u[4 * k + 2] = x.z; u[4 * k + 3] = x.w;
            }
        };
        load8(0);
        const uint32_t n = count_tiles(ch, p);
        if (n == 0) continue;
        if (!(ok = wait_warp(c, bar(c, B_Q_EMPTY), (nq & 1) ^ 1, false, 17))) break;
        tc_fence_after();
        if (quad == 0 && lane == 0) {
            mbar_expect_tx(bar(c, B_Q_FULL), kQBytes);
            tma_load_2d(c.s + kOffQ, q_rope, 512 + rank * 32, ch.seq * kH, bar(c, B_Q_FULL));
        }
        tmem_st32(tmem + lane_base + kTmemQ, u);
        #pragma unroll 1
        for (int q64 = 1; q64 < 4; q64++) {
            load8(q64);
            tmem_st32(tmem + lane_base + kTmemQ + q64 * 32, u);
        }
        tmem_wait_st();
        tc_fence_before();
        warp_arrive(bar(c, B_QT_FULL));
        nq++;
        for (uint32_t j = 0; j < n && ok; j++, t++) {
            const uint32_t sb = t & 1;
            if (!(ok = wait_warp(c, bar(c, B_S_FULL + sb), (t >> 1) & 1, false, 8))) break;
            tc_fence_after();
            float s[64];
            tmem_ld32(tmem + lane_base + kTmemS + sb * 64, s);
            tmem_ld32(tmem + lane_base + kTmemS + sb * 64 + 32, s + 32);
            tmem_wait_ld();
            tc_fence_before();
            warp_arrive(bar(c, B_S_EMPTY + sb));
            /* this quadrant's rows of the out buffer: its previous copy has read them */
            if (lane == 0) bulk_wait_read();
            __syncwarp();
            float4 *xout = reinterpret_cast<float4 *>(c.smem + kOffOut);
            #pragma unroll
            for (int q4 = 0; q4 < 16; q4++)
                xout[xoff(row, q4) >> 4] = make_float4(s[4 * q4], s[4 * q4 + 1], s[4 * q4 + 2], s[4 * q4 + 3]);
            proxy_fence();
            __syncwarp();
            if (lane == 0) {
                /* the peer has consumed tile t-2 from receive slot sb */
                ok = wait_bar(c, bar(c, B_X_EMPTY + sb), ((t >> 1) & 1) ^ 1, true, 15);
                if (ok) bulk_copy_to_peer(in_peer + sb * kXBytes + quad * 8192, c.s + kOffOut + quad * 8192, 8192,
                                          xf_peer + (sb * 4 + quad) * 8);
            }
            ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
        }
    }
    if (lane == 0) {
        bulk_wait_all();
        /* the peer's GEMM2 of the last two tiles releases their slots here by
         * a remote arrive; wait for it so none lands after exit */
        if (quad == 0)
            for (uint32_t u = t >= 2 ? t - 2 : 0; u < t && ok; u++)
                ok = wait_bar(c, bar(c, B_X_EMPTY + (u & 1)), (u >> 1) & 1, true, 20);
        /* and the last rope load this warp issued has landed */
        if (quad == 0 && nq) {
            long long t0 = clock64();
            while (!mbar_try(bar(c, B_Q_FULL), (nq - 1) & 1) && clock64() - t0 < kWaitCycles) {}
        }
    }
}

template <int KV>
__device__ void softmax_warps(const Ctx &c, const Params &p, uint32_t tmem, int wbeg, int wend, uint32_t rank) {
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t quad = warp & 3;                     /* TMEM lane quadrant this warp may access */
    Row r;
    r.part = (warp - kFirstSoftmaxWarp) >> 2;           /* tokens [16k, 16k+16) of a tile, O columns [64k, +64) */
    r.row = quad * 32 + lane;                           /* head */
    r.quad = quad;
    r.lane_base = (quad * 32) << 16;
    r.tid = (warp - kFirstSoftmaxWarp) * 32 + lane;
    float *red = reinterpret_cast<float *>(c.smem + kOffRed);
    uint32_t g = 0, nchunk = 0;
    bool ok = true;
    for (int ci = wbeg; ci < wend && ok; ci++) {
        const ct_mla_chunk_t ch = load_chunk(p, ci);
        WarpTiles it;
        it.init(ch, p);
        int32_t pg, ntok;
        const size_t oh = (size_t)ch.seq * kH + r.row;
        const uint32_t d_base = rank * 256 + r.part * kOCols;
        if (!it.next(pg, ntok)) {
            /* nothing readable: zero output */
            if (ch.part < 0) {
                uint4 *dst = reinterpret_cast<uint4 *>(p.out + oh * kDv + d_base);
                for (int k = 0; k < kOCols / 8; k++) dst[k] = make_uint4(0, 0, 0, 0);
            } else {
                float4 *dst = reinterpret_cast<float4 *>(p.part_o + ((size_t)ch.part * kH + r.row) * kDv + d_base);
                for (int k = 0; k < kOCols / 4; k++) dst[k] = make_float4(0, 0, 0, 0);
            }
            if (rank == 0 && r.part == 0) {
                if (ch.part < 0) {
                    if (p.lse) p.lse[oh] = -INFINITY;
                } else {
                    float *ml = p.part_ml + 4 * ((size_t)ch.part * kH + r.row);     /* (m, l_lo, l_hi, -) */
                    ml[0] = -INFINITY;
                    ml[1] = ml[2] = 0.0f;
                }
            }
            continue;
        }
        r.m_used = -INFINITY;
        r.l = 0.0f;
        uint32_t j = 0;
        do {
            if (!finish_tile<KV>(c, p, tmem, r, g + j, j, ntok)) { ok = false; break; }
            j++;
        } while (it.next(pg, ntok));
        if (!ok) break;
        g += j;
        /* epilogue: the row sum over all parts, then O of this CTA's 256 value dims */
        float *rl = red + 2 * kParts * kH;
        rl[r.part * kH + r.row] = r.l;
        warp_arrive(bar(c, B_RED_L + r.quad));
        if (!wait_warp(c, bar(c, B_RED_L + r.quad), nchunk & 1, false, 18)) { ok = false; break; }
        float l_tot = r.l;
        #pragma unroll
        for (int k = 1; k < kParts; k++) l_tot += rl[((r.part + k) % kParts) * kH + r.row];
        if (!wait_warp(c, bar(c, B_O_FINAL), nchunk & 1, false, 13)) { ok = false; break; }
        tc_fence_after();
        const float inv = l_tot > 0.0f ? 1.0f / l_tot : 0.0f;
        #pragma unroll 1
        for (int cc = 0; cc < kOCols / 32; cc++) {
            float o[32];
            tmem_ld32(tmem + r.lane_base + kTmemO + r.part * kOCols + cc * 32, o);
            tmem_wait_ld();
            const uint32_t d0 = d_base + cc * 32;
            /* a lane writes 32 consecutive values of its head row: whole
             * 32-byte sectors (the split-KV partials always, the bf16 output
             * when it is 32-B aligned) */
            if (ch.part < 0) {
                uint32_t w[16];
                #pragma unroll
                for (int e = 0; e < 16; e++)
                    w[e] = (uint32_t)ct_f32_to_bf16(o[2 * e] * inv) | ((uint32_t)ct_f32_to_bf16(o[2 * e + 1] * inv) << 16);
                uint4 *dst = reinterpret_cast<uint4 *>(p.out + oh * kDv + d0);
                if (p.out32) {
                    st_global_v8(dst, w);
                    st_global_v8(dst + 2, w + 8);
                } else {
                    #pragma unroll
                    for (int k = 0; k < 4; k++) dst[k] = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
                }
            } else {
                float *dst = p.part_o + ((size_t)ch.part * kH + r.row) * kDv + d0;
                #pragma unroll
                for (int k = 0; k < 4; k++) st_global_v8(dst + 8 * k, reinterpret_cast<const uint32_t *>(o + 8 * k));
            }
        }
        tc_fence_before();
        warp_arrive(bar(c, B_O_FREE));
        /* statistics that one thread per row writes */
        if (rank == 0 && r.part == 0) {
            if (ch.part < 0) {
                if (p.lse) p.lse[oh] = l_tot > 0.0f ? r.m_used * kLn2 + logf(l_tot) : -INFINITY;
            } else {
                /* both CTAs use the same probabilities: one sum for both halves of the dims */
                float *ml = p.part_ml + 4 * ((size_t)ch.part * kH + r.row);     /* (m, l_lo, l_hi, -) */
                ml[0] = r.m_used;
                ml[1] = ml[2] = l_tot;
            }
        }
        nchunk++;
    }
}

/* ---- warps 15-18 (int8 / e4m3 pools): codes -> bf16 in place -------------- */

/* 16 codes (one 16-byte chunk) -> 16 bf16 values as two 16-byte chunks.
 * Every int8 and e4m3 value is exactly representable in bf16, so a value's
 * bf16 is the upper half of its fp32.  int8 without a conversion
 * instruction: the code + 128 (its byte xor 0x80) becomes the low byte of
 * the fp32 2^23 (bits 0x4B000000), and subtracting 2^23 + 128 leaves the
 * code exactly (integers below 2^24).  e4m3 by the paired conversion to
 * f16x2 and f32. */
template <int KV>
__device__ __forceinline__ void widen16(const uint4 &c, uint4 &lo, uint4 &hi) {
    uint32_t o[8];
    if (KV == CT_KV_INT8) {
        const uint32_t w[4] = {c.x, c.y, c.z, c.w};
        #pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t pair = (w[i >> 1] >> (16 * (i & 1))) & 0xFFFFu;
            const float f0 = (float)(int8_t)(pair & 0xFF), f1 = (float)(int8_t)(pair >> 8);
            o[i] = __byte_perm(__float_as_uint(f0), __float_as_uint(f1), 0x7632u);
        }
    } else {
        const uint32_t w[4] = {c.x, c.y, c.z, c.w};
        #pragma unroll
        for (int i = 0; i < 8; i++) {
            const float2 f = ct_e4m3x2_to_f32x2((uint16_t)((w[i >> 1] >> (16 * (i & 1))) & 0xFFFFu));
            o[i] = __byte_perm(__float_as_uint(f.x), __float_as_uint(f.y), 0x7632u);
        }
    }
    lo = make_uint4(o[0], o[1], o[2], o[3]);
    hi = make_uint4(o[4], o[5], o[6], o[7]);
}

/* The TMA put each latent box's codes in the upper half of its bf16 box
 * (64 rows x 64 codes at +4 KB of an 8 KB SW128 box) and the rope codes
 * (64 rows x 32) in a 2 KB area of their own.  Warp w owns latent box w: it
 * loads all of the box's codes into registers, then writes the bf16 rows
 * over them, so no other warp's codes are overwritten; it also converts rope
 * rows [16w, 16w+16) into the SW64 rope box.  Latent rows past the page's
 * tokens become zeros (they are V rows of GEMM2). */
template <int KV>
__device__ void converter(const Ctx &c, const Params &p, int wbeg, int wend) {
    static_assert(kConvWarps == 4, "one latent box and a quarter of the rope box per warp");
    const uint32_t lane = threadIdx.x & 31, cw = (threadIdx.x >> 5) - kFirstConvWarp;
    uint32_t g = 0;
    bool ok = true;
    for (int ci = wbeg; ci < wend && ok; ci++) {
        const ct_mla_chunk_t ch = load_chunk(p, ci);
        WarpTiles it;
        it.init(ch, p);
        int32_t pg, ntok;
        while (it.next(pg, ntok)) {
            const uint32_t st = g % kStages;
            if (!wait_warp(c, bar(c, B_KV_FULL + st), (g / kStages) & 1, false, 19)) { ok = false; break; }
            uint8_t *kv = c.smem + kOffKv + st * kKvBytes;
            uint8_t *box = kv + cw * 8192;
            uint4 code[8];
            #pragma unroll
            for (int k = 0; k < 8; k++) code[k] = reinterpret_cast<const uint4 *>(box + 4096)[lane + 32 * k];
            const uint4 rc = reinterpret_cast<const uint4 *>(c.smem + kOffRc + st * 2048)[32 * cw + lane];
            __syncwarp();
            #pragma unroll
            for (int k = 0; k < 8; k++) {
                const uint32_t idx = lane + 32 * k, row = idx >> 2, cc = idx & 3;
                uint4 lo = make_uint4(0, 0, 0, 0), hi = lo;
                if ((int32_t)row < ntok) widen16<KV>(code[k], lo, hi);
                *reinterpret_cast<uint4 *>(box + row * 128 + (((2 * cc) ^ (row & 7)) << 4)) = lo;
                *reinterpret_cast<uint4 *>(box + row * 128 + (((2 * cc + 1) ^ (row & 7)) << 4)) = hi;
            }
            {
                uint8_t *rbox = kv + 4 * 8192;
                const uint32_t idx = 32 * cw + lane, row = idx >> 1, cc = idx & 1, sw = (row >> 1) & 3;
                uint4 lo, hi;
                widen16<KV>(rc, lo, hi);
                *reinterpret_cast<uint4 *>(rbox + row * 64 + (((2 * cc) ^ sw) << 4)) = lo;
                *reinterpret_cast<uint4 *>(rbox + row * 64 + (((2 * cc + 1) ^ sw) << 4)) = hi;
            }
            proxy_fence();                             /* generic writes -> the tensor core's view */
            warp_arrive(bar(c, B_CONV_FULL + st));
            g++;
        }
    }
}

/* ---- the kernel ----------------------------------------------------------- */

template <int KV>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(KV == CT_KV_BF16 ? kThreads : kThreadsQ, 1)
    k_mla_tc(const __grid_constant__ CUtensorMap kv_lat, const __grid_constant__ CUtensorMap kv_rope,
             const __grid_constant__ CUtensorMap q_rope, Params p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ int s_abort;
    const uint32_t raw = smem_addr(smem_raw);
    const uint32_t pad = (1024u - (raw & 1023u)) & 1023u;
    Ctx c;
    c.smem = smem_raw + pad;
    c.s = raw + pad;
    const uint32_t rank = cluster_rank();
    c.peer = rank ^ 1u;
    c.abort = &s_abort;
    const uint32_t warp = threadIdx.x >> 5;
    const int w = blockIdx.x >> 1;

    if (threadIdx.x == 0) {
        s_abort = 0;
        for (int i = 0; i < kStages; i++) {
            mbar_init(bar(c, B_KV_FULL + i), 1);
            mbar_init(bar(c, B_KV_EMPTY + i), 1);
        }
        mbar_init(bar(c, B_Q_FULL), 1); mbar_init(bar(c, B_Q_EMPTY), 1); mbar_init(bar(c, B_QT_FULL), 4);
        for (int i = 0; i < 2; i++) {
            mbar_init(bar(c, B_S_FULL + i), 1);
            mbar_init(bar(c, B_P_FULL + i), kSoftmaxWarps);
            mbar_init(bar(c, B_X_EMPTY + i), 1);            /* the peer's GEMM2 commit */
            mbar_init(bar(c, B_S_EMPTY + i), kSoftmaxWarps + 4);   /* softmax and staging warps */
        }
        for (int i = 0; i < 8; i++) mbar_init(bar(c, B_RED + i), kParts);     /* the warps of a quadrant */
        for (int i = 0; i < 8; i++) mbar_init(bar(c, B_X_FULL + i), 1);       /* 8 KB each */
        for (int i = 0; i < 4; i++) mbar_init(bar(c, B_RED_L + i), kParts);
        mbar_init(bar(c, B_O_READY), 1); mbar_init(bar(c, B_O_FINAL), 1);
        mbar_init(bar(c, B_O_FREE), kSoftmaxWarps);
        mbar_init(bar(c, B_DRAIN), 1);
        mbar_init(bar(c, B_DRAIN2), 1);
        for (int i = 0; i < kStages; i++) mbar_init(bar(c, B_CONV_FULL + i), kConvWarps);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int i = 0; i < 8; i++) mbar_expect_tx(bar(c, B_X_FULL + i), kXBytes / 4);   /* the first two tiles */
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(c.s + kOffTmem), "r"(kTmemCols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();                                 /* both CTAs' barriers exist before any remote arrive or copy */
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(c.smem + kOffTmem);
    const int wbeg = p.worker_begin[w], wend = p.worker_begin[w + 1];

    if (warp == 0) {
        producer<KV>(c, p, &kv_lat, &kv_rope, &q_rope, wbeg, wend, rank);
    } else if (warp == 1) {
        /* bf16 pages: one thread per GEMM; the int8 / e4m3 kernels, whose
         * converter warps share the SM, measured faster with one thread
         * issuing both (GEMM2 first when ready) */
        if constexpr (KV == CT_KV_BF16) gemm1_issuer<KV>(c, p, tmem, wbeg, wend);
        else mma_issuer<KV>(c, p, tmem, wbeg, wend);
    } else if (warp == 2) {
        if constexpr (KV == CT_KV_BF16) gemm2_issuer(c, p, tmem, wbeg, wend);
    } else if (warp < (uint32_t)kFirstStageWarp) {
        softmax_warps<KV>(c, p, tmem, wbeg, wend, rank);
    } else if (warp < (uint32_t)kFirstConvWarp) {
        stager(c, p, &q_rope, tmem, wbeg, wend, rank);
    } else if (KV != CT_KV_BF16) {
        converter<KV>(c, p, wbeg, wend);
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    cluster_sync();                                 /* no CTA leaves while its peer may still write its smem */
}

/* ---- host side ------------------------------------------------------------ */

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void *p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        else
            cudaGetLastError();
    }
    return fn;
}

/* 2-D map over [rows][576] values (bf16, or 1-byte codes) with a
 * (box_cols x box_rows) box. */
bool make_map(CUtensorMap *m, const void *base, uint64_t rows, uint32_t box_cols, uint32_t box_rows,
              CUtensorMapSwizzle sw, bool bytes = false) {
    auto fn = encode_fn();
    if (!fn) return false;
    const uint32_t elt = bytes ? 1 : 2;
    cuuint64_t dims[2] = {(cuuint64_t)kE, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)kE * elt};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, bytes ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base),
              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool shape_ok(const ct_mla_dims_t *d) {
    return d->n_heads == (uint32_t)kH && d->entry_dim == (uint32_t)kE && d->v_dim == (uint32_t)kDv &&
           d->page_tokens == (uint32_t)kP && d->scale > 0.0f &&
           (d->kv_dtype == CT_KV_BF16 || d->kv_dtype == CT_KV_INT8 || d->kv_dtype == CT_KV_E4M3);
}

const void *kernel_for(uint32_t kv) {
    switch (kv) {
        case CT_KV_INT8: return (const void *)k_mla_tc<CT_KV_INT8>;
        case CT_KV_E4M3: return (const void *)k_mla_tc<CT_KV_E4M3>;
        default: return (const void *)k_mla_tc<CT_KV_BF16>;
    }
}

int threads_for(uint32_t kv) { return kv == CT_KV_BF16 ? kThreads : kThreadsQ; }

}  // namespace

extern "C" int ct__mla_tc_workers(const ct_mla_dims_t *dims, int device) {
    if (!dims || !shape_ok(dims)) return 0;
    int major = 0, minor = 0, sms = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (major != 10 || minor != 0 || !encode_fn()) return 0;
    /* One worker per co-resident cluster, so every worker runs in one wave. */
    static int cached[64][4];
    if (device < 0 || device >= 64) return 0;
    const uint32_t kv = dims->kv_dtype;
    if (cached[device][kv] == 0) {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(device);
        int n = 0;
        const void *fn = kernel_for(kv);
        if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemAlloc) == cudaSuccess) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(2 * (sms / 2), 1, 1);
            cfg.blockDim = dim3(threads_for(kv), 1, 1);
            cfg.dynamicSmemBytes = kSmemAlloc;
            if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) n = 0;
        }
        cudaGetLastError();
        cudaSetDevice(prev);
        cached[device][kv] = n > 0 ? n : -1;
    }
    return cached[device][kv] > 0 ? cached[device][kv] : 0;
}

/* Error word of the tensor-core kernel (0 = no wait expired), for tests. */
extern "C" int ct_mla_tc_error(int clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_mla_tc_error, sizeof v) != cudaSuccess) { cudaGetLastError(); return -1; }
    if (clear && v) {
        int z = 0;
        cudaMemcpyToSymbol(g_mla_tc_error, &z, sizeof z);
    }
    return v;
}

extern "C" int ct__launch_mla_tc(const ct_mla_dims_t *dims, const ct_mla_chunk_t *chunks, uint32_t n_chunks,
                                 const int32_t *worker_begin, uint32_t n_workers, const void *q,
                                 const void *pool, const float *scales, const int32_t *block_table,
                                 const int32_t *seq_lens, void *out, float *lse, float *part_o, float *part_ml,
                                 void *stream) {
    (void)n_chunks;
    if (!shape_ok(dims)) return CT_ERR_UNSUPPORTED;
    const uint32_t kv = dims->kv_dtype;
    const bool quant = kv != CT_KV_BF16;
    if (quant && (!scales || ((uintptr_t)scales & 15u))) return CT_ERR_UNSUPPORTED;
    int dev = 0;
    cudaGetDevice(&dev);
    if (ct__mla_tc_workers(dims, dev) <= 0 || n_workers == 0) return CT_ERR_UNSUPPORTED;
    if (((uintptr_t)pool & 15u) || ((uintptr_t)q & 15u) || ((uintptr_t)out & 15u)) return CT_ERR_UNSUPPORTED;
    /* Maps cover exactly the pool and q: a page id beyond the pool reads
     * zeros (TMA out-of-bounds fill) rather than foreign memory. */
    CUtensorMap kv_lat, kv_rope, q_rope;
    if (dims->n_pages == 0 || dims->n_seq == 0) return CT_ERR_ARG;
    const uint64_t pool_rows = (uint64_t)dims->n_pages * kP;
    const uint64_t q_rows = (uint64_t)dims->n_seq * kH;
    const bool maps_ok =
        quant ? make_map(&kv_lat, pool, pool_rows, 64, 64, CU_TENSOR_MAP_SWIZZLE_NONE, true) &&
                    make_map(&kv_rope, pool, pool_rows, 32, 64, CU_TENSOR_MAP_SWIZZLE_NONE, true)
              : make_map(&kv_lat, pool, pool_rows, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B) &&
                    make_map(&kv_rope, pool, pool_rows, 32, 64, CU_TENSOR_MAP_SWIZZLE_64B);
    if (!maps_ok || !make_map(&q_rope, q, q_rows, 32, 128, CU_TENSOR_MAP_SWIZZLE_64B)) {
        ct__set_error("mla_tc: cuTensorMapEncodeTiled failed");
        return CT_ERR_CUDA;
    }
    Params p;
    p.chunks = chunks;
    p.worker_begin = worker_begin;
    p.bt = block_table;
    p.lens = seq_lens;
    p.q = static_cast<const uint16_t *>(q);
    p.out = static_cast<uint16_t *>(out);
    p.lse = lse;
    p.part_o = part_o;
    p.part_ml = part_ml;
    p.scales = scales;
    p.maxp = dims->max_pages_per_seq;
    p.n_pages = dims->n_pages;
    p.qk_scale = dims->scale * kLog2e;
    p.out32 = ((uintptr_t)out & 31u) == 0;
    static bool attr_set[4] = {false, false, false, false};
    if (!attr_set[kv]) {
        int rc = ct__cuda_status(cudaFuncSetAttribute(kernel_for(kv), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                      (int)kSmemAlloc), "mla_tc attribute");
        if (rc) return rc;
        attr_set[kv] = true;
    }
    cudaStream_t st = (cudaStream_t)stream;
    const dim3 grid(2 * n_workers);
    switch (kv) {
        case CT_KV_INT8: k_mla_tc<CT_KV_INT8><<<grid, kThreadsQ, kSmemAlloc, st>>>(kv_lat, kv_rope, q_rope, p); break;
        case CT_KV_E4M3: k_mla_tc<CT_KV_E4M3><<<grid, kThreadsQ, kSmemAlloc, st>>>(kv_lat, kv_rope, q_rope, p); break;
        default: k_mla_tc<CT_KV_BF16><<<grid, kThreads, kSmemAlloc, st>>>(kv_lat, kv_rope, q_rope, p); break;
    }
    return ct__cuda_status(cudaGetLastError(), "mla_tc launch");
}
