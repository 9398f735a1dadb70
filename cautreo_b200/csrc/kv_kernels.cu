/*
 * kv_kernels.cu -- HBM-bound kernels of the paged KV cache:
 *   write_slots   append / quantise-on-append (eight lanes per token up to
 *                 768 values, one warp per token beyond; block pools: a
 *                 CTA per 64 tokens staged in shared memory)
 *   gather        block-table gather with dequantise-on-gather (64-token CTA
 *                 tiles; block pools: page runs staged in shared memory)
 *   move_pages    page-granular gather used by defragmenting compaction
 *   compress      contiguous every-k-th token compaction (ct_kv_compress)
 *
 * Layout in HBM.  Pool: [n_pages][page_tokens][dim] values of the pool dtype
 * (bf16 / fp32 / int8 / e4m3); quantised pools add scales
 * [n_pages][page_tokens] fp32.  A token entry of the MLA cache is 576 bf16
 * = 1152 B (9 x 128 B lines); int8/e4m3 entries are 576 B + a 4 B scale.
 * Block-quantised pools (Q8_0 / Q4_0 / Q2_0 / Q1_0) hold dim/32 blocks per
 * token (612 / 324 / 180 / 108 B for 576 values) and no scales array.
 * Element pools move data in 16-byte vectors and require dim % 16 == 0;
 * block pools require dim % 32 == 0 and stage tiles of entries in shared
 * memory.
 */
#include "../../include/hal.h"
#include "../../include/kv_cache.h"
#include "../../include/quant.h"
#include "ct_internal.h"

#include <algorithm>

namespace {

constexpr int kWarps = 8;          /* tokens per 256-thread block */

/* Two floats -> packed bf16 pair (lo in the low half), round to nearest even
 * (one cvt; equal to ct_f32_to_bf16 for every non-NaN input). */
__device__ __forceinline__ uint32_t bf16x2_rn(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}

/* 16 consecutive source values of a token as raw words: bf16 -> 8 words
 * (two per word, low half first), fp32 -> 16 words. */
template <bool SrcBf16>
struct Chunk {
    uint32_t w[SrcBf16 ? 8 : 16];
    __device__ __forceinline__ void load(const void *src, size_t tok, uint32_t dim, uint32_t c) {
        const uint4 *p = SrcBf16 ? reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(src) + tok * dim + c * 16)
                                 : reinterpret_cast<const uint4 *>(static_cast<const float *>(src) + tok * dim + c * 16);
        #pragma unroll
        for (int i = 0; i < (SrcBf16 ? 2 : 4); i++) {
            const uint4 v = __ldg(p + i);
            w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
        }
    }
    __device__ __forceinline__ float val(int i) const {
        if (SrcBf16) return __uint_as_float((i & 1) ? (w[i >> 1] & 0xFFFF0000u) : (w[i >> 1] << 16));
        return __uint_as_float(w[i]);
    }
};

/* K1 / K2: one warp per token.  Lane l owns 16-value chunks l, l+32, ...
 * (MaxChunks per lane), kept as raw words so a 576-value token costs few
 * registers and many warps stay resident; quantised pools need the token's
 * absmax, reduced with warp shuffles, before any code is written. */
template <bool SrcBf16, int PoolDtype, int MaxChunks>
__global__ void __launch_bounds__(256) k_write_slots(void *pool, float *scales, const void *src,
                                                     const int32_t *dest, uint32_t n, uint32_t dim) {
    const uint32_t warp = blockIdx.x * kWarps + (threadIdx.x >> 5);
    const uint32_t lane = threadIdx.x & 31;
    if (warp >= n) return;
    const int32_t slot = dest ? dest[warp] : (int32_t)warp;      /* no dest: slot = token */
    if (slot < 0) return;
    const uint32_t n_chunks = dim / 16;
    Chunk<SrcBf16> v[MaxChunks];
    #pragma unroll
    for (int k = 0; k < MaxChunks; k++) {
        const uint32_t c = lane + 32u * k;
        if (c < n_chunks) v[k].load(src, warp, dim, c);
    }
    const size_t base = (size_t)slot * dim;
    if (PoolDtype == CT_KV_BF16) {
        #pragma unroll
        for (int k = 0; k < MaxChunks; k++) {
            const uint32_t c = lane + 32u * k;
            if (c >= n_chunks) continue;
            uint32_t w[8];
            if (SrcBf16) {
                #pragma unroll
                for (int i = 0; i < 8; i++) w[i] = v[k].w[i];
            } else {
                #pragma unroll
                for (int i = 0; i < 8; i++)
                    w[i] = (uint32_t)ct_f32_to_bf16(v[k].val(2 * i)) | ((uint32_t)ct_f32_to_bf16(v[k].val(2 * i + 1)) << 16);
            }
            uint4 *p = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(pool) + base + c * 16);
            __stcs(p, make_uint4(w[0], w[1], w[2], w[3]));
            __stcs(p + 1, make_uint4(w[4], w[5], w[6], w[7]));
        }
    } else if (PoolDtype == CT_KV_F32) {
        #pragma unroll
        for (int k = 0; k < MaxChunks; k++) {
            const uint32_t c = lane + 32u * k;
            if (c >= n_chunks) continue;
            float4 *p = reinterpret_cast<float4 *>(static_cast<float *>(pool) + base + c * 16);
            #pragma unroll
            for (int i = 0; i < 4; i++)
                __stcs(p + i, make_float4(v[k].val(4 * i), v[k].val(4 * i + 1), v[k].val(4 * i + 2), v[k].val(4 * i + 3)));
        }
    } else {
        float amax = 0.0f;
        #pragma unroll
        for (int k = 0; k < MaxChunks; k++) {
            if (lane + 32u * k >= n_chunks) continue;
            #pragma unroll
            for (int i = 0; i < 16; i++) amax = fmaxf(amax, fabsf(v[k].val(i)));
        }
        amax = ct_warp_max(amax);
        const float d = __fdiv_rn(amax, PoolDtype == CT_KV_INT8 ? 127.0f : 448.0f);
        const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        #pragma unroll
        for (int k = 0; k < MaxChunks; k++) {
            const uint32_t c = lane + 32u * k;
            if (c >= n_chunks) continue;
            uint32_t w[4] = {0, 0, 0, 0};
            if (PoolDtype == CT_KV_INT8) {
                #pragma unroll
                for (int i = 0; i < 16; i++)
                    w[i >> 2] |= (uint32_t)(uint8_t)(int8_t)ct_q8_code(v[k].val(i), id) << (8 * (i & 3));
            } else {
                #pragma unroll
                for (int i = 0; i < 16; i += 2)
                    w[i >> 2] |= (uint32_t)ct_e4m3x2_code(v[k].val(i), v[k].val(i + 1), id) << (8 * (i & 3));
            }
            __stcs(reinterpret_cast<uint4 *>(static_cast<uint8_t *>(pool) + base + c * 16), make_uint4(w[0], w[1], w[2], w[3]));
        }
        if (lane == 0) scales[slot] = d;
    }
}

/* Eight lanes per token, four tokens per warp: lane g of a token's group owns
 * the 8-value units g, g+8, ... (UPL per lane), so every lane does the same
 * work for entries whose unit count is a multiple of 8 (576 values = 72
 * units, 9 per lane), a load instruction reads 128 contiguous bytes of bf16
 * source per token, and the absmax is a 3-step shuffle within the group.
 * Same codes as k_write_slots: floor(x * id + 0.5) is one round-down
 * conversion of the rounded sum (NaN -> 0, as the float -> int conversion of
 * floorf gives), then the clamp. */
template <bool SrcBf16, int PoolDtype, int UPL>
__global__ void __launch_bounds__(256) k_write_grouped(void *pool, float *scales, const void *src,
                                                       const int32_t *dest, uint32_t n, uint32_t dim) {
    const uint32_t g = threadIdx.x & 7;
    const uint32_t tok = blockIdx.x * 32 + (threadIdx.x >> 3);
    const int32_t slot = tok < n ? (dest ? dest[tok] : (int32_t)tok) : -1;   /* no dest: slot = token */
    const uint32_t n_units = dim / 8;
    constexpr int kW = SrcBf16 ? 4 : 8;                 /* source words per unit */
    uint32_t w[UPL][kW];
    if (slot >= 0) {
        #pragma unroll
        for (int i = 0; i < UPL; i++) {
            const uint32_t u = i * 8 + g;
            if (u >= n_units) continue;
            const uint4 *p = SrcBf16 ? reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(src) + (size_t)tok * dim + u * 8)
                                     : reinterpret_cast<const uint4 *>(static_cast<const float *>(src) + (size_t)tok * dim + u * 8);
            #pragma unroll
            for (int k = 0; k < kW / 4; k++) {
                const uint4 v = __ldg(p + k);
                w[i][4 * k] = v.x; w[i][4 * k + 1] = v.y; w[i][4 * k + 2] = v.z; w[i][4 * k + 3] = v.w;
            }
        }
    }
    auto val = [&](int i, int e) -> float {
        if (SrcBf16) return __uint_as_float((e & 1) ? (w[i][e >> 1] & 0xFFFF0000u) : (w[i][e >> 1] << 16));
        return __uint_as_float(w[i][e]);
    };
    const size_t base = (size_t)(slot < 0 ? 0 : slot) * dim;
    if (PoolDtype == CT_KV_BF16 || PoolDtype == CT_KV_F32) {
        if (slot < 0) return;
        #pragma unroll
        for (int i = 0; i < UPL; i++) {
            const uint32_t u = i * 8 + g;
            if (u >= n_units) continue;
            if (PoolDtype == CT_KV_BF16) {
                uint32_t o[4];
                #pragma unroll
                for (int k = 0; k < 4; k++)
                    o[k] = SrcBf16 ? w[i][k]
                                   : (uint32_t)ct_f32_to_bf16(val(i, 2 * k)) | ((uint32_t)ct_f32_to_bf16(val(i, 2 * k + 1)) << 16);
                __stcs(reinterpret_cast<uint4 *>(static_cast<uint16_t *>(pool) + base + u * 8), make_uint4(o[0], o[1], o[2], o[3]));
            } else {
                float4 *p = reinterpret_cast<float4 *>(static_cast<float *>(pool) + base + u * 8);
                __stcs(p, make_float4(val(i, 0), val(i, 1), val(i, 2), val(i, 3)));
                __stcs(p + 1, make_float4(val(i, 4), val(i, 5), val(i, 6), val(i, 7)));
            }
        }
        return;
    }
    float amax = 0.0f;
    if (slot >= 0) {
        #pragma unroll
        for (int i = 0; i < UPL; i++) {
            if (i * 8 + g >= n_units) continue;
            #pragma unroll
            for (int e = 0; e < 8; e++) amax = fmaxf(amax, fabsf(val(i, e)));
        }
    }
    #pragma unroll
    for (int o = 1; o < 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
    if (slot < 0) return;
    const float d = __fdiv_rn(amax, PoolDtype == CT_KV_INT8 ? 127.0f : 448.0f);
    const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    #pragma unroll
    for (int i = 0; i < UPL; i++) {
        const uint32_t u = i * 8 + g;
        if (u >= n_units) continue;
        uint32_t c[2];
        if (PoolDtype == CT_KV_INT8) {
            int q[8];
            #pragma unroll
            for (int e = 0; e < 8; e++) {
                const int r = __float2int_rd(__fadd_rn(__fmul_rn(val(i, e), id), 0.5f));
                q[e] = max(-127, min(127, r));
            }
            #pragma unroll
            for (int k = 0; k < 2; k++)
                c[k] = __byte_perm(__byte_perm(q[4 * k], q[4 * k + 1], 0x0040), __byte_perm(q[4 * k + 2], q[4 * k + 3], 0x0040),
                                   0x5410);
        } else {
            #pragma unroll
            for (int k = 0; k < 2; k++)
                c[k] = (uint32_t)ct_e4m3x2_code(val(i, 4 * k), val(i, 4 * k + 1), id) |
                       ((uint32_t)ct_e4m3x2_code(val(i, 4 * k + 2), val(i, 4 * k + 3), id) << 16);
        }
        __stcs(reinterpret_cast<uint2 *>(static_cast<uint8_t *>(pool) + base + u * 8), make_uint2(c[0], c[1]));
    }
    if (g == 0) scales[slot] = d;
}

/* Tiles of the gathers below: 64 tokens per CTA, up to 9 (token, 16-value
 * chunk) pairs per thread (entries of at most 576 values). */
constexpr int kTileTok = 64, kTileK = 9;

template <bool SrcBf16, int PoolDtype>
int launch_write(void *pool, float *scales, const void *src, const int32_t *dest, uint32_t n,
                 uint32_t dim, cudaStream_t st) {
    const uint32_t chunks = dim / 16, units = dim / 8;
    if (units <= 96) {
        const int gb = (int)((n + 31) / 32);
        if (units <= 16) k_write_grouped<SrcBf16, PoolDtype, 2><<<gb, 256, 0, st>>>(pool, scales, src, dest, n, dim);
        else if (units <= 32) k_write_grouped<SrcBf16, PoolDtype, 4><<<gb, 256, 0, st>>>(pool, scales, src, dest, n, dim);
        else if (units <= 64) k_write_grouped<SrcBf16, PoolDtype, 8><<<gb, 256, 0, st>>>(pool, scales, src, dest, n, dim);
        else if (units <= 72) k_write_grouped<SrcBf16, PoolDtype, 9><<<gb, 256, 0, st>>>(pool, scales, src, dest, n, dim);
        else k_write_grouped<SrcBf16, PoolDtype, 12><<<gb, 256, 0, st>>>(pool, scales, src, dest, n, dim);
        ct__count_launches(1);
        return ct__cuda_status(cudaGetLastError(), "write_slots");
    }
    const int blocks = (int)((n + kWarps - 1) / kWarps);
    if (chunks <= 32) k_write_slots<SrcBf16, PoolDtype, 1><<<blocks, 256, 0, st>>>(pool, scales, src, dest, n, dim);
    else if (chunks <= 64) k_write_slots<SrcBf16, PoolDtype, 2><<<blocks, 256, 0, st>>>(pool, scales, src, dest, n, dim);
    else if (chunks <= 128) k_write_slots<SrcBf16, PoolDtype, 4><<<blocks, 256, 0, st>>>(pool, scales, src, dest, n, dim);
    else return CT_ERR_UNSUPPORTED;
    ct__count_launches(1);
    return ct__cuda_status(cudaGetLastError(), "write_slots");
}

/* One token of a gather (whole warp): pool slot -> output row, dequantising
 * to fp32 or bf16.  Lanes own 16-value chunks; every load is issued before
 * any store. */
template <int PoolDtype, bool OutBf16, int MaxChunks>
__device__ __forceinline__ void gather_token(const void *pool, const float *scales, size_t slot, uint32_t dim,
                                             void *out_row) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t n_chunks = dim / 16;
    constexpr int kWords = (PoolDtype == CT_KV_F32) ? 16 : (PoolDtype == CT_KV_BF16 ? 8 : 4);
    uint32_t w[MaxChunks][kWords];
    #pragma unroll
    for (int k = 0; k < MaxChunks; k++) {
        const uint32_t c = lane + 32u * k;
        if (c >= n_chunks) continue;
        const size_t byte = (slot * dim + c * 16) * (PoolDtype == CT_KV_F32 ? 4 : PoolDtype == CT_KV_BF16 ? 2 : 1);
        const uint4 *p = reinterpret_cast<const uint4 *>(static_cast<const uint8_t *>(pool) + byte);
        #pragma unroll
        for (int i = 0; i < kWords / 4; i++) {
            const uint4 v = __ldcs(p + i);
            w[k][4 * i] = v.x; w[k][4 * i + 1] = v.y; w[k][4 * i + 2] = v.z; w[k][4 * i + 3] = v.w;
        }
    }
    const float sc = (PoolDtype == CT_KV_INT8 || PoolDtype == CT_KV_E4M3) ? scales[slot] : 1.0f;
    #pragma unroll
    for (int k = 0; k < MaxChunks; k++) {
        const uint32_t c = lane + 32u * k;
        if (c >= n_chunks) continue;
        if constexpr (PoolDtype == CT_KV_BF16 && OutBf16) {
            uint4 *p = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(out_row) + c * 16);
            __stcs(p, make_uint4(w[k][0], w[k][1], w[k][2], w[k][3]));
            __stcs(p + 1, make_uint4(w[k][4], w[k][5], w[k][6], w[k][7]));
            continue;
        } else {
        float v[16];
        #pragma unroll
        for (int i = 0; i < 16; i++) {
            if (PoolDtype == CT_KV_BF16) v[i] = __uint_as_float((i & 1) ? (w[k][i >> 1] & 0xFFFF0000u) : (w[k][i >> 1] << 16));
            else if (PoolDtype == CT_KV_F32) v[i] = __uint_as_float(w[k][i]);
            else if (PoolDtype == CT_KV_INT8) {
                v[i] = (float)(int8_t)(uint8_t)(w[k][i >> 2] >> (8 * (i & 3))) * sc;
            } else if ((i & 1) == 0) {
                const float2 f = ct_e4m3x2_to_f32x2((uint16_t)(w[k][i >> 2] >> (8 * (i & 3))));
                v[i] = f.x * sc;
                v[i + 1] = f.y * sc;
            }
        }
        if (OutBf16) {
            uint32_t o[8];
            #pragma unroll
            for (int i = 0; i < 8; i++) o[i] = (uint32_t)ct_f32_to_bf16(v[2 * i]) | ((uint32_t)ct_f32_to_bf16(v[2 * i + 1]) << 16);
            uint4 *p = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(out_row) + c * 16);
            __stcs(p, make_uint4(o[0], o[1], o[2], o[3]));
            __stcs(p + 1, make_uint4(o[4], o[5], o[6], o[7]));
        } else {
            float4 *p = reinterpret_cast<float4 *>(static_cast<float *>(out_row) + c * 16);
            #pragma unroll
            for (int i = 0; i < 4; i++) __stcs(p + i, make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]));
        }
        }
    }
}

/* K3: tokens [start, start+n) of one sequence, one warp per token. */
template <int PoolDtype, bool OutBf16, int MaxChunks>
__global__ void __launch_bounds__(256) k_gather(const void *pool, const float *scales,
                                                const int32_t *bt_row, uint32_t page_tokens,
                                                uint32_t dim, uint32_t start, uint32_t n, void *out) {
    const uint32_t t = blockIdx.x * kWarps + (threadIdx.x >> 5);
    if (t >= n) return;
    const uint32_t pos = start + t;
    const int32_t pg = bt_row[pos / page_tokens];
    const size_t slot = (size_t)pg * page_tokens + pos % page_tokens;
    const size_t out_elt = (size_t)t * dim * (OutBf16 ? 2 : 4);
    gather_token<PoolDtype, OutBf16, MaxChunks>(pool, scales, slot, dim, static_cast<uint8_t *>(out) + out_elt);
}

/* K3b: several sequences in one launch; desc[y] = (seq, start, count,
 * first output row) and blockIdx.y selects it. */
template <int PoolDtype, bool OutBf16, int MaxChunks>
__global__ void __launch_bounds__(256) k_gather_batch(const void *pool, const float *scales, const int32_t *bt,
                                                      uint32_t max_pages, uint32_t page_tokens, uint32_t dim,
                                                      const int4 *desc, void *out) {
    const int4 d = desc[blockIdx.y];
    const uint32_t t = blockIdx.x * kWarps + (threadIdx.x >> 5);
    if (t >= (uint32_t)d.z) return;
    const uint32_t pos = (uint32_t)d.y + t;
    const int32_t pg = bt[(size_t)d.x * max_pages + pos / page_tokens];
    const size_t slot = (size_t)pg * page_tokens + pos % page_tokens;
    const size_t out_elt = ((size_t)(uint32_t)d.w + t) * dim * (OutBf16 ? 2 : 4);
    gather_token<PoolDtype, OutBf16, MaxChunks>(pool, scales, slot, dim, static_cast<uint8_t *>(out) + out_elt);
}

/* K1b / K3c: block-quantised pools (Q8_0 / Q4_0 / Q2_0 / Q1_0).
 * Append: a CTA takes a tile of up to 64 consecutive source tokens; a thread
 * encodes a whole block (32 values, so the per-block scale arithmetic is
 * paid once per 32 values) and loads its next block while it encodes this
 * one, and several CTAs per SM keep the loads in flight.  The tile's entries
 * are built in shared memory and go out as 16-byte vectors when its slots
 * are consecutive.
 * Gather: persistent CTAs (four per SM) stride over runs of one page's
 * entries, double-buffered in shared memory with cp.async, so the copy of
 * the next run is in flight while one is decoded; a block is decoded by kL
 * adjacent lanes (4 for bf16 output, 8 for fp32), each storing its values as
 * one 16-byte vector, so a warp writes 512 consecutive bytes per
 * instruction. */
constexpr int kMaxBlocks = 128;                 /* dim <= 4096 */
constexpr uint32_t kBlkOut = 47 * 1024;         /* append: entry bytes of a tile (+16 within 48 KB) */
constexpr uint32_t kBlkStage = 18 * 1024;       /* gather: code bytes per buffer */
constexpr int kBlkCtasPerSm = 4;                /* gather */

/* Tokens per tile or item: the largest power of two whose bytes fit the
 * budget (1..64), so that a tile of a 64-token page never straddles two
 * pages. */
__host__ __device__ inline uint32_t blk_tile(uint32_t bytes_per_token, uint32_t budget) {
    uint32_t t = budget / bytes_per_token;
    t = t > 64 ? 64 : (t < 1 ? 1 : t);
    while (t & (t - 1)) t &= t - 1;
    return t;
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                 ::"r"((uint32_t)__cvta_generic_to_shared(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
/* every group of this thread except the newest has landed */
__device__ __forceinline__ void cp_async_wait_prev() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

/* max that propagates NaN (IEEE maximum, not maxNum) */
__device__ __forceinline__ float fmax_nan(float a, float b) {
    float d;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
    return d;
}

template <int Type> struct BlockCode {
    static constexpr int kBits = Type == CT_QUANT_Q8_0 ? 8 : Type == CT_QUANT_Q4_0 ? 4 : Type == CT_QUANT_Q2_0 ? 2 : 1;
    static constexpr int kMax = Type == CT_QUANT_Q8_0 ? 127 : Type == CT_QUANT_Q4_0 ? 7 : 1;
};

/* One block's fp16 scale and packed codes, ct_block_encode's bit for bit,
 * into blk (2-byte aligned, shared memory).  Fast path: the block's |x|
 * maximum, taken NaN-propagating, is finite, and d = amax / qmax is 0 or a
 * normal float.  Then |x id| <= qmax (1 + 2^-22), so floor(x id + 0.5) lies
 * in [-qmax, qmax] without a clamp, and the floor is taken by adding
 * 1.5 * 2^23 (plus 1 for Q2_0's code + 1) rounding down: the low bits of that
 * sum are the two's-complement code.  Otherwise (a NaN, an Inf, a subnormal
 * scale) every value goes through ct_block_code, and the maximum skips NaNs
 * as the reference's does. */
template <int Type>
__device__ __forceinline__ void block_encode_thread(const float *x, uint8_t *blk) {
    constexpr int kW = (CtBlock<Type>::kBytes - 2) / 4;
    uint16_t *h = reinterpret_cast<uint16_t *>(blk);
    float amax = 0.0f;
    #pragma unroll
    for (int i = 0; i < 32; i++) amax = fmax_nan(amax, fabsf(x[i]));
    const bool finite = amax <= 3.40282347e38f;                /* false for NaN and Inf */
    if (amax != amax) {
        amax = 0.0f;
        #pragma unroll
        for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(x[i]));
    }
    uint32_t w[kW];
    if (Type == CT_QUANT_Q1_0) {
        h[0] = ct_ref_f32_to_fp16(amax);
        uint32_t bits = 0;
        #pragma unroll
        for (int i = 0; i < 32; i++) bits |= (x[i] >= 0.0f ? 1u : 0u) << i;
        w[0] = bits;
    } else {
        constexpr int qm = BlockCode<Type>::kMax;
        constexpr float magic = Type == CT_QUANT_Q2_0 ? 12582913.0f : 12582912.0f;
        const float d = __fdiv_rn(amax, (float)qm);
        h[0] = ct_ref_f32_to_fp16(d);
        const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        uint32_t r[32];
        if (finite && (d == 0.0f || d >= 1.17549435e-38f)) {
            #pragma unroll
            for (int i = 0; i < 32; i++) r[i] = __float_as_uint(__fadd_rd(__fadd_rn(__fmul_rn(x[i], id), 0.5f), magic));
        } else {
            #pragma unroll
            for (int i = 0; i < 32; i++) r[i] = (uint32_t)(ct_block_code(x[i], id, qm) + (Type == CT_QUANT_Q2_0 ? 1 : 0));
        }
        if (Type == CT_QUANT_Q8_0) {
            #pragma unroll
            for (int j = 0; j < kW; j++)
                w[j] = __byte_perm(__byte_perm(r[4 * j], r[4 * j + 1], 0x0040), __byte_perm(r[4 * j + 2], r[4 * j + 3], 0x0040),
                                   0x5410);
        } else {
            constexpr int cb = BlockCode<Type>::kBits, per = 32 / cb;
            #pragma unroll
            for (int j = 0; j < kW; j++) {
                uint32_t v = 0;
                #pragma unroll
                for (int k = 0; k < per; k++) v |= (r[per * j + k] & ((1u << cb) - 1u)) << (cb * k);
                w[j] = v;
            }
        }
    }
    #pragma unroll
    for (int j = 0; j < kW; j++) {
        h[1 + 2 * j] = (uint16_t)w[j];
        h[2 + 2 * j] = (uint16_t)(w[j] >> 16);
    }
}

/* Lane q's kV values of a block in shared memory, ct_block_decode's exactly
 * (code x d in fp32, exact: at most 8 + 11 significant bits).  A code becomes
 * a float by placing it, offset to be non-negative, in the low bits of
 * 1.5 * 2^23 (one byte permute for Q8_0) and subtracting that float's base;
 * Q1_0 sets d's sign from the bit.  No conversion instructions. */
template <int Type, int kV>
__device__ __forceinline__ void block_decode_lane(const uint8_t *blk, uint32_t q, float *x) {
    constexpr int cb = BlockCode<Type>::kBits, LB = kV * cb;    /* this lane's code bits */
    const uint16_t *h = reinterpret_cast<const uint16_t *>(blk);
    const float d = ct_ref_fp16_to_f32(h[0]);
    uint32_t w0, w1 = 0;
    if (LB == 64) {
        const uint16_t *c = h + 1 + 4 * q;
        w0 = (uint32_t)c[0] | ((uint32_t)c[1] << 16);
        w1 = (uint32_t)c[2] | ((uint32_t)c[3] << 16);
    } else if (LB == 32) {
        const uint16_t *c = h + 1 + 2 * q;
        w0 = (uint32_t)c[0] | ((uint32_t)c[1] << 16);
    } else if (LB == 16) {
        w0 = h[1 + q];
    } else {
        constexpr uint32_t S = LB < 16 ? 16 / LB : 1;
        w0 = (uint32_t)h[1 + q / S] >> ((q % S) * LB);
    }
    #pragma unroll
    for (int i = 0; i < kV; i++) {
        if (Type == CT_QUANT_Q1_0) {
            x[i] = __uint_as_float(__float_as_uint(d) ^ ((((w0 >> i) & 1u) ^ 1u) << 31));
            continue;
        }
        float f;
        if (Type == CT_QUANT_Q8_0)
            f = __uint_as_float(__byte_perm((i < 4 ? w0 : w1) ^ 0x80808080u, 0x4B400000u, 0x7650u + (i & 3))) - 12583040.0f;
        else if (Type == CT_QUANT_Q4_0)
            f = __uint_as_float((((w0 >> (4 * i)) & 0xFu) ^ 8u) | 0x4B400000u) - 12582920.0f;
        else
            f = __uint_as_float(((w0 >> (2 * i)) & 3u) | 0x4B400000u) - 12582913.0f;
        x[i] = __fmul_rn(f, d);
    }
}

int blk_sm_count() {
    static int cached[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (cached[dev] <= 0) {
        int c = 0;
        if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || c <= 0) c = 148;
        cached[dev] = c;
    }
    return cached[dev];
}

/* The 32 source values of one block as raw 16-byte vectors (bf16: 4, fp32:
 * 8), from a 16-byte aligned source, or with 2-byte loads from one that is
 * not. */
template <bool SrcBf16>
struct BlockSrc {
    static constexpr int kVec = SrcBf16 ? 4 : 8;
    uint4 v[kVec];
    template <bool Aligned>
    __device__ __forceinline__ void load(const uint8_t *q) {
        if (Aligned) {
            #pragma unroll
            for (int i = 0; i < kVec; i++) v[i] = __ldcs(reinterpret_cast<const uint4 *>(q) + i);
        } else {
            uint16_t *h = reinterpret_cast<uint16_t *>(v);
            #pragma unroll
            for (int i = 0; i < 8 * kVec; i++) h[i] = __ldcs(reinterpret_cast<const unsigned short *>(q) + i);
        }
    }
    __device__ __forceinline__ void values(float *x) const {
        #pragma unroll
        for (int i = 0; i < kVec; i++) {
            const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
            #pragma unroll
            for (int j = 0; j < 4; j++) {
                if (SrcBf16) {
                    x[8 * i + 2 * j] = __uint_as_float(w[j] << 16);
                    x[8 * i + 2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
                } else {
                    x[4 * i + j] = __uint_as_float(w[j]);
                }
            }
        }
    }
};

/* Append: tokens [tile x, tile x + tile) of the source, whose blocks are
 * back to back (64 or 128 bytes each).  When the tile's slots are
 * consecutive (a run of one page, the usual bulk append) its entries are one
 * byte run of the pool: they are encoded into shared memory at the run's
 * offset modulo 16 and stored as 16-byte vectors (2-byte pieces at the two
 * ragged ends); otherwise each token's entry is stored as 4- or 2-byte
 * words.  Tokens with a negative slot are skipped. */
template <bool SrcBf16, int Type, bool Aligned>
__global__ void __launch_bounds__(256, 4) k_write_blocks(uint8_t *pool, const void *src, const int32_t *dest, uint32_t n,
                                                      uint32_t dim, uint32_t tile) {
    constexpr int kB = CtBlock<Type>::kBytes;
    constexpr uint32_t kBlkBytes = SrcBf16 ? 64 : 128;
    extern __shared__ __align__(16) uint8_t outs[];            /* tile * eb + 16 bytes */
    const uint32_t nb = dim / 32, eb = nb * kB;
    const uint32_t t0 = blockIdx.x * tile, cnt = min(tile, n - t0), nblk = cnt * nb;
    const uint8_t *s8 = static_cast<const uint8_t *>(src) + (size_t)t0 * nb * kBlkBytes;
    BlockSrc<SrcBf16> cur;
    if (threadIdx.x < nblk) cur.template load<Aligned>(s8 + (size_t)threadIdx.x * kBlkBytes);
    /* no dest: the entries go to slots 0, 1, 2, ... */
    const uint32_t d0 = dest ? (uint32_t)dest[t0] : t0;
    const bool mine = !dest || threadIdx.x >= cnt || (uint32_t)dest[t0 + threadIdx.x] == d0 + threadIdx.x;
    const bool contig = __syncthreads_and(mine) && (int32_t)d0 >= 0 && ((uintptr_t)pool & 15) == 0;
    const size_t g0 = contig ? (size_t)d0 * eb : 0;
    const uint32_t mis = (uint32_t)(g0 & 15);                   /* even: eb is */
    for (uint32_t p = threadIdx.x; p < nblk; p += 256) {
        float x[32];
        if (!SrcBf16 && p != threadIdx.x) cur.template load<Aligned>(s8 + (size_t)p * kBlkBytes);
        cur.values(x);
        /* bf16: the next block's 64 bytes are in flight during this encode
         * (fp32 sources, 128 bytes a block, would not fit the registers) */
        if (SrcBf16 && p + 256 < nblk) cur.template load<Aligned>(s8 + (size_t)(p + 256) * kBlkBytes);
        block_encode_thread<Type>(x, outs + mis + p * kB);
    }
    __syncthreads();
    if (contig) {
        const uint32_t end = mis + cnt * eb, nv = (end + 15) / 16;
        uint8_t *g = pool + (g0 - mis);
        for (uint32_t v = threadIdx.x; v < nv; v += 256) {
            const uint32_t a = 16 * v;
            if (a >= mis && a + 16 <= end) {
                *reinterpret_cast<uint4 *>(g + a) = *reinterpret_cast<const uint4 *>(outs + a);
            } else {
                for (uint32_t c = max(a, mis); c < min(a + 16, end); c += 2)
                    *reinterpret_cast<uint16_t *>(g + c) = *reinterpret_cast<const uint16_t *>(outs + c);
            }
        }
    } else if ((eb & 3) == 0) {
        const uint32_t W = eb / 4;
        for (uint32_t p = threadIdx.x; p < cnt * W; p += 256) {
            const uint32_t t = p / W, w = p - t * W;
            const int32_t slot = dest[t0 + t];
            if (slot >= 0)
                reinterpret_cast<uint32_t *>(pool + (size_t)slot * eb)[w] = reinterpret_cast<const uint32_t *>(outs + t * eb)[w];
        }
    } else {
        const uint32_t W = eb / 2;
        for (uint32_t p = threadIdx.x; p < cnt * W; p += 256) {
            const uint32_t t = p / W, w = p - t * W;
            const int32_t slot = dest[t0 + t];
            if (slot >= 0)
                reinterpret_cast<uint16_t *>(pool + (size_t)slot * eb)[w] = reinterpret_cast<const uint16_t *>(outs + t * eb)[w];
        }
    }
}

/* One gather item: tokens [lo, hi) of one page, at most `tile` of them. */
struct BlkItem {
    const uint8_t *page;
    uint32_t lo, hi, a, nvec, off;
    size_t row0;
};

/* Gather: tokens [start, start+n) of one sequence (desc == nullptr), or of
 * desc[y] = (seq, start, count, first output row) for each y.  Item i =
 * (y, x): x = page index within the range x tiles per page + tile within the
 * page, items_x of them per y.  An item's entries are one contiguous run of
 * its page, copied as 16-byte vectors (rounded out to 16-byte boundaries
 * inside the page); each lane then decodes its kV values and stores them as
 * one 16-byte vector of the output row. */
template <int Type, bool OutBf16>
__global__ void __launch_bounds__(256, kBlkCtasPerSm) k_gather_blocks(const uint8_t *pool, const int32_t *bt,
                                                                      uint32_t max_pages, uint32_t page_tokens,
                                                                      uint32_t dim, uint32_t start, uint32_t n,
                                                                      const int4 *desc, uint64_t items_x,
                                                                      uint64_t n_items, void *out, uint32_t tile) {
    constexpr int kB = CtBlock<Type>::kBytes, kL = OutBf16 ? 4 : 8, kV = 32 / kL;
    extern __shared__ __align__(16) uint8_t smem[];
    const uint32_t nb = dim / 32, eb = nb * kB, P = page_tokens, per_page = (P + tile - 1) / tile;
    const uint32_t stage = (tile * eb + 32 + 15) & ~15u;
    auto find = [&](uint64_t i, BlkItem &w) -> uint64_t {
        for (; i < n_items; i += gridDim.x) {
            const uint64_t y = i / items_x;
            const uint32_t x = (uint32_t)(i - y * items_x);
            const int32_t *bt_row = bt;
            uint32_t s0 = start, cn = n;
            size_t r0 = 0;
            if (desc) {
                const int4 d = desc[y];
                bt_row = bt + (size_t)d.x * max_pages;
                s0 = (uint32_t)d.y;
                cn = (uint32_t)d.z;
                r0 = (uint32_t)d.w;
            }
            if (cn == 0) continue;
            const uint32_t lp = s0 / P + x / per_page, sub = x % per_page;
            const uint32_t lo = max(s0, lp * P + sub * tile);
            const uint32_t hi = min(min(s0 + cn, lp * P + P), lp * P + sub * tile + tile);
            if (lo >= hi) continue;
            const uint32_t b_lo = (lo - lp * P) * eb, b_hi = (hi - lp * P) * eb;
            w.page = pool + (size_t)bt_row[lp] * P * eb;
            w.a = b_lo & ~15u;
            w.nvec = (((b_hi + 15u) & ~15u) - w.a) / 16;
            w.off = b_lo - w.a;
            w.lo = lo;
            w.hi = hi;
            w.row0 = r0 + (lo - s0);
            return i;
        }
        return n_items;
    };
    auto issue = [&](const BlkItem &w, uint8_t *buf) {
        const uint8_t *s = w.page + w.a;
        for (uint32_t v = threadIdx.x; v < w.nvec; v += 256) cp_async16(buf + 16 * v, s + 16 * v);
    };
    BlkItem cur, nxt;
    uint64_t i = find(blockIdx.x, cur);
    if (i < n_items) issue(cur, smem);
    cp_async_commit();
    for (uint32_t k = 0; i < n_items; k++) {
        const uint64_t j = find(i + gridDim.x, nxt);
        if (j < n_items) issue(nxt, smem + ((k + 1) & 1) * stage);
        cp_async_commit();
        cp_async_wait_prev();
        __syncthreads();
        const uint8_t *buf = smem + (k & 1) * stage + cur.off;
        const uint32_t units = (cur.hi - cur.lo) * nb * kL;
        const size_t e0 = cur.row0 * dim;
        for (uint32_t u = threadIdx.x; u < units; u += 256) {
            const uint32_t blk = u / kL, q = u % kL;
            float x[kV];
            block_decode_lane<Type, kV>(buf + blk * kB, q, x);
            const size_t e = e0 + (size_t)blk * 32 + q * kV;    /* token t, block b: t dim + 32 b = 32 blk */
            if (OutBf16) {
                __stcs(reinterpret_cast<uint4 *>(static_cast<uint16_t *>(out) + e),
                       make_uint4(bf16x2_rn(x[0], x[1]), bf16x2_rn(x[2], x[3]), bf16x2_rn(x[4], x[5]),
                                  bf16x2_rn(x[6], x[7])));
            } else {
                __stcs(reinterpret_cast<float4 *>(static_cast<float *>(out) + e), make_float4(x[0], x[1], x[2], x[3]));
            }
        }
        __syncthreads();                          /* this buffer is refilled next */
        cur = nxt;
        i = j;
    }
}

template <bool SrcBf16, int Type>
void launch_write_blocks_t(uint8_t *pool, const void *src, const int32_t *dest, uint32_t n, uint32_t dim,
                           cudaStream_t st) {
    const uint32_t eb = dim / 32 * CtBlock<Type>::kBytes, tile = blk_tile(eb, kBlkOut);
    const int grid = (int)((n + tile - 1) / tile);
    const size_t sm = (size_t)tile * eb + 16;
    if (((uintptr_t)src & 15) == 0)
        k_write_blocks<SrcBf16, Type, true><<<grid, 256, sm, st>>>(pool, src, dest, n, dim, tile);
    else
        k_write_blocks<SrcBf16, Type, false><<<grid, 256, sm, st>>>(pool, src, dest, n, dim, tile);
}

template <bool SrcBf16>
int launch_write_blocks(uint32_t type, void *pool, const void *src, const int32_t *dest, uint32_t n, uint32_t dim,
                        cudaStream_t st) {
    uint8_t *p = static_cast<uint8_t *>(pool);
    switch (type) {
        case CT_KV_Q8_0: launch_write_blocks_t<SrcBf16, CT_QUANT_Q8_0>(p, src, dest, n, dim, st); break;
        case CT_KV_Q4_0: launch_write_blocks_t<SrcBf16, CT_QUANT_Q4_0>(p, src, dest, n, dim, st); break;
        case CT_KV_Q2_0: launch_write_blocks_t<SrcBf16, CT_QUANT_Q2_0>(p, src, dest, n, dim, st); break;
        default:         launch_write_blocks_t<SrcBf16, CT_QUANT_Q1_0>(p, src, dest, n, dim, st); break;
    }
    ct__count_launches(1);
    return ct__cuda_status(cudaGetLastError(), "write_slots");
}

template <int Type>
void launch_gather_blocks(bool ob, const void *pool, const int32_t *bt, uint32_t maxp, uint32_t P, uint32_t dim,
                          uint32_t start, uint32_t n, const int4 *desc, uint32_t n_desc, void *out, cudaStream_t st) {
    const uint32_t eb = dim / 32 * CtBlock<Type>::kBytes, tile = blk_tile(eb, kBlkStage);
    const uint32_t per_page = (P + tile - 1) / tile;
    /* n tokens starting anywhere in a page span at most n / P + 2 pages */
    const uint64_t items_x = (uint64_t)(n / P + 2) * per_page, n_items = items_x * (desc ? n_desc : 1);
    const uint64_t cap = (uint64_t)blk_sm_count() * kBlkCtasPerSm;
    const int grid = (int)(n_items < cap ? n_items : cap);
    const size_t sm = 2 * (size_t)((tile * eb + 32 + 15) & ~15u);
    const uint8_t *p = static_cast<const uint8_t *>(pool);
    if (ob) k_gather_blocks<Type, true><<<grid, 256, sm, st>>>(p, bt, maxp, P, dim, start, n, desc, items_x, n_items, out, tile);
    else    k_gather_blocks<Type, false><<<grid, 256, sm, st>>>(p, bt, maxp, P, dim, start, n, desc, items_x, n_items, out, tile);
}

/* The reference block codecs on flat device arrays (ct_quant_q*_0 /
 * ct_quant_deq*_0 on the device): decode with eight lanes per block, each
 * storing its four fp32 values as one 16-byte vector (a warp writes 512
 * consecutive bytes); the block bytes are read straight from global memory. */
template <int Type>
__global__ void __launch_bounds__(256) k_decode_blocks_flat(const uint8_t *src, float *dst, int64_t nb) {
    constexpr int kB = CtBlock<Type>::kBytes;
    const int64_t units = nb * 8;
    for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < units; u += (int64_t)gridDim.x * blockDim.x) {
        const int64_t blk = u >> 3;
        const uint32_t q = (uint32_t)(u & 7);
        float x[4];
        block_decode_lane<Type, 4>(src + blk * kB, q, x);
        __stcs(reinterpret_cast<float4 *>(dst + blk * 32 + q * 4), make_float4(x[0], x[1], x[2], x[3]));
    }
}

/* K3t: the gathers from bf16 / int8 / e4m3 pools for entries of at most 576
 * values, as CTA tiles of 64 output rows: (row, 16-value chunk) pairs spread
 * evenly over the 256 threads (9 each for 576 values, where a warp per token
 * leaves 28 of 32 lanes idle half the time), all of a thread's loads issued
 * before any store.  Rows
 * [64 x, 64 x + 64) of tokens [start, start+n) of one sequence (desc null),
 * or of desc[y] = (seq, start, count, first output row). */
template <int PoolDtype, bool OutBf16>
__global__ void __launch_bounds__(256) k_gather_tiled(const void *pool, const float *scales, const int32_t *bt,
                                                      uint32_t max_pages, uint32_t page_tokens, uint32_t dim,
                                                      uint32_t start, uint32_t n, const int4 *desc, void *out) {
    constexpr int kW = PoolDtype == CT_KV_BF16 ? 8 : 4;      /* words per 16-value chunk */
    const int32_t *bt_row = bt;
    size_t row0 = 0;
    if (desc) {
        const int4 d = desc[blockIdx.y];
        bt_row = bt + (size_t)d.x * max_pages;
        start = (uint32_t)d.y;
        n = (uint32_t)d.z;
        row0 = (uint32_t)d.w;
    }
    const uint32_t r0 = blockIdx.x * kTileTok;
    if (r0 >= n) return;
    const uint32_t C = dim / 16, cnt = min((uint32_t)kTileTok, n - r0), pairs = cnt * C;
    uint32_t w[kTileK][kW];
    float sc[kTileK];
    #pragma unroll
    for (int k = 0; k < kTileK; k++) {
        const uint32_t q = threadIdx.x + 256u * k;
        if (q >= pairs) continue;
        const uint32_t t = q / C, c = q - t * C, pos = start + r0 + t;
        const size_t slot = (size_t)bt_row[pos / page_tokens] * page_tokens + pos % page_tokens;
        const uint4 *p = reinterpret_cast<const uint4 *>(static_cast<const uint8_t *>(pool) +
                                                         (slot * dim + c * 16) * (PoolDtype == CT_KV_BF16 ? 2 : 1));
        const uint4 a = __ldcs(p);
        w[k][0] = a.x; w[k][1] = a.y; w[k][2] = a.z; w[k][3] = a.w;
        if (kW == 8) {
            const uint4 b = __ldcs(p + 1);
            w[k][kW == 8 ? 4 : 0] = b.x; w[k][kW == 8 ? 5 : 1] = b.y; w[k][kW == 8 ? 6 : 2] = b.z; w[k][kW == 8 ? 7 : 3] = b.w;
        }
        sc[k] = PoolDtype == CT_KV_BF16 ? 1.0f : scales[slot];
    }
    #pragma unroll
    for (int k = 0; k < kTileK; k++) {
        const uint32_t q = threadIdx.x + 256u * k;
        if (q >= pairs) continue;
        const uint32_t t = q / C, c = q - t * C;
        uint8_t *orow = static_cast<uint8_t *>(out) + (row0 + r0 + t) * dim * (OutBf16 ? 2 : 4);
        if constexpr (PoolDtype == CT_KV_BF16 && OutBf16) {
            uint4 *o = reinterpret_cast<uint4 *>(reinterpret_cast<uint16_t *>(orow) + c * 16);
            __stcs(o, make_uint4(w[k][0], w[k][1], w[k][2], w[k][3]));
            __stcs(o + 1, make_uint4(w[k][kW - 4], w[k][kW - 3], w[k][kW - 2], w[k][kW - 1]));
        } else {
            float v[16];
            #pragma unroll
            for (int i = 0; i < 16; i++) {
                if (PoolDtype == CT_KV_BF16) {
                    v[i] = __uint_as_float((i & 1) ? (w[k][(i >> 1) % kW] & 0xFFFF0000u) : (w[k][(i >> 1) % kW] << 16));
                } else if (PoolDtype == CT_KV_INT8) {
                    v[i] = (float)(int8_t)(uint8_t)(w[k][(i >> 2) % kW] >> (8 * (i & 3))) * sc[k];
                } else if ((i & 1) == 0) {
                    const float2 f = ct_e4m3x2_to_f32x2((uint16_t)(w[k][(i >> 2) % kW] >> (8 * (i & 3))));
                    v[i] = f.x * sc[k];
                    v[i + 1] = f.y * sc[k];
                }
            }
            if (OutBf16) {
                uint32_t o[8];
                #pragma unroll
                for (int i = 0; i < 8; i++)
                    o[i] = (uint32_t)ct_f32_to_bf16(v[2 * i]) | ((uint32_t)ct_f32_to_bf16(v[2 * i + 1]) << 16);
                uint4 *po = reinterpret_cast<uint4 *>(reinterpret_cast<uint16_t *>(orow) + c * 16);
                __stcs(po, make_uint4(o[0], o[1], o[2], o[3]));
                __stcs(po + 1, make_uint4(o[4], o[5], o[6], o[7]));
            } else {
                float4 *po = reinterpret_cast<float4 *>(reinterpret_cast<float *>(orow) + c * 16);
                #pragma unroll
                for (int i = 0; i < 4; i++) __stcs(po + i, make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]));
            }
        }
    }
}

/* K4 (pages): block b copies whole page map[b] -> b; 16-byte vectors with
 * four loads in flight per thread. */
__global__ void __launch_bounds__(256) k_move_pages(const uint4 *src, const float *src_sc, uint4 *dst,
                                                    float *dst_sc, const int32_t *map,
                                                    size_t vec_per_page, uint32_t page_tokens) {
    const size_t from = (size_t)map[blockIdx.x];
    const uint4 *s = src + from * vec_per_page;
    uint4 *d = dst + (size_t)blockIdx.x * vec_per_page;
    size_t i = threadIdx.x;
    for (; i + 3 * 256 < vec_per_page; i += 4 * 256) {
        uint4 a = __ldcs(s + i), b = __ldcs(s + i + 256), c = __ldcs(s + i + 512), e = __ldcs(s + i + 768);
        __stcs(d + i, a); __stcs(d + i + 256, b); __stcs(d + i + 512, c); __stcs(d + i + 768, e);
    }
    for (; i < vec_per_page; i += 256) __stcs(d + i, __ldcs(s + i));
    if (src_sc && threadIdx.x < page_tokens)
        dst_sc[(size_t)blockIdx.x * page_tokens + threadIdx.x] = src_sc[from * page_tokens + threadIdx.x];
}

/* ct_kv_compress: row j of the kept set is row j*step (per layer), copied
 * through a scratch buffer because rows overlap in place. */
__global__ void k_compress_out(const float4 *k, const float4 *v, float4 *scratch, uint32_t max_ctx,
                               uint32_t stride4, uint32_t new_len, uint32_t step, uint32_t n_layers) {
    const size_t total = (size_t)n_layers * new_len * stride4;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        size_t e = i % stride4, r = (i / stride4) % new_len, l = i / ((size_t)stride4 * new_len);
        size_t src = (l * max_ctx + r * step) * stride4 + e;
        scratch[i] = k[src];
        scratch[total + i] = v[src];
    }
}

__global__ void k_compress_in(float4 *k, float4 *v, const float4 *scratch, uint32_t max_ctx,
                              uint32_t stride4, uint32_t new_len, uint32_t n_layers) {
    const size_t total = (size_t)n_layers * new_len * stride4;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        size_t e = i % stride4, r = (i / stride4) % new_len, l = i / ((size_t)stride4 * new_len);
        size_t dst = (l * max_ctx + r) * stride4 + e;
        k[dst] = scratch[i];
        v[dst] = scratch[total + i];
    }
}

/* Scalar variant for strides that are not a multiple of 4 floats. */
__global__ void k_compress_scalar(float *k, float *v, float *scratch, uint32_t max_ctx, uint32_t stride,
                                  uint32_t new_len, uint32_t step, uint32_t n_layers, int phase) {
    const size_t total = (size_t)n_layers * new_len * stride;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        size_t e = i % stride, r = (i / stride) % new_len, l = i / ((size_t)stride * new_len);
        if (phase == 0) {
            size_t src = (l * max_ctx + r * step) * stride + e;
            scratch[i] = k[src]; scratch[total + i] = v[src];
        } else {
            size_t dst = (l * max_ctx + r) * stride + e;
            k[dst] = scratch[i]; v[dst] = scratch[total + i];
        }
    }
}

}  // namespace

/* Flat block codecs: n fp32 values (a multiple of 32) <-> n / 32 blocks.
 * The encode runs the append kernel with the blocks as consecutive slots of
 * "tokens" of up to 128 blocks.  Returns CT_ERR_UNSUPPORTED for arrays of
 * 2^32 tokens or more (the callers then use their per-block kernels). */
extern "C" int ct__launch_encode_blocks(int type, const float *x, void *blocks, int64_t n, void *stream) {
    const int64_t nb = n / 32;
    if (((uintptr_t)blocks & 15) != 0) return CT_ERR_UNSUPPORTED;      /* the kernel stores 4- and 16-byte words */
    uint32_t f = 128;
    while (f > 1 && nb % f) f >>= 1;
    if (nb / f >= (int64_t)0xFFFFFFFF) return CT_ERR_UNSUPPORTED;
    const uint32_t dim = 32 * f, n_tok = (uint32_t)(nb / f);
    if (n_tok == 0) return CT_OK;
    static const uint32_t kPool[5] = {0, CT_KV_Q8_0, CT_KV_Q4_0, CT_KV_Q2_0, CT_KV_Q1_0};
    if (type < 1 || type > 4) return CT_ERR_ARG;
    return launch_write_blocks<false>(kPool[type], blocks, x, nullptr, n_tok, dim, (cudaStream_t)stream);
}

extern "C" int ct__launch_decode_blocks(int type, const void *blocks, float *x, int64_t n, void *stream) {
    const int64_t nb = n / 32;
    if (nb == 0) return CT_OK;
    if (((uintptr_t)x & 15) != 0 || ((uintptr_t)blocks & 1) != 0) return CT_ERR_UNSUPPORTED;
    const int grid = (int)std::min<int64_t>((nb * 8 + 255) / 256, (int64_t)148 * 16);
    const uint8_t *src = static_cast<const uint8_t *>(blocks);
    cudaStream_t st = (cudaStream_t)stream;
    switch (type) {
        case CT_QUANT_Q8_0: k_decode_blocks_flat<CT_QUANT_Q8_0><<<grid, 256, 0, st>>>(src, x, nb); break;
        case CT_QUANT_Q4_0: k_decode_blocks_flat<CT_QUANT_Q4_0><<<grid, 256, 0, st>>>(src, x, nb); break;
        case CT_QUANT_Q2_0: k_decode_blocks_flat<CT_QUANT_Q2_0><<<grid, 256, 0, st>>>(src, x, nb); break;
        case CT_QUANT_Q1_0: k_decode_blocks_flat<CT_QUANT_Q1_0><<<grid, 256, 0, st>>>(src, x, nb); break;
        default: return CT_ERR_ARG;
    }
    ct__count_launches(1);
    return ct__cuda_status(cudaGetLastError(), "decode_blocks");
}

/* Per-token int8 / e4m3 codes of n_tok consecutive entries (dim a multiple
 * of 16, at most 2048) into consecutive rows: the append kernels with the
 * rows as slots. */
extern "C" int ct__launch_quant_tokens(int int8, const void *x, int src_is_bf16, uint32_t n_tok, uint32_t dim,
                                       void *codes, float *scales, void *stream) {
    if (dim % 16 != 0 || dim > 2048) return CT_ERR_UNSUPPORTED;
    if (n_tok == 0) return CT_OK;
    cudaStream_t st = (cudaStream_t)stream;
    if (int8)
        return src_is_bf16 ? launch_write<true, CT_KV_INT8>(codes, scales, x, nullptr, n_tok, dim, st)
                           : launch_write<false, CT_KV_INT8>(codes, scales, x, nullptr, n_tok, dim, st);
    return src_is_bf16 ? launch_write<true, CT_KV_E4M3>(codes, scales, x, nullptr, n_tok, dim, st)
                       : launch_write<false, CT_KV_E4M3>(codes, scales, x, nullptr, n_tok, dim, st);
}

extern "C" int ct_kv_paged_write_slots(void *pool, float *scales, uint32_t pool_dtype, const void *entries,
                                       uint32_t src_dtype, const int32_t *dest_slot, uint32_t n,
                                       uint32_t dim, void *stream) {
    if (!pool || !entries || !dest_slot || dim == 0 || dim % 16 != 0) return CT_ERR_ARG;
    if ((pool_dtype == CT_KV_INT8 || pool_dtype == CT_KV_E4M3) && !scales) return CT_ERR_ARG;
    const bool blocks = pool_dtype >= CT_KV_Q8_0 && pool_dtype <= CT_KV_Q1_0;
    if (blocks && (dim % 32 != 0 || dim / 32 > (uint32_t)kMaxBlocks)) return CT_ERR_ARG;
    if (n == 0) return CT_OK;
    cudaStream_t st = (cudaStream_t)stream;
    const bool bf = src_dtype == CT_KV_BF16;
    if (!bf && src_dtype != CT_KV_F32) return CT_ERR_ARG;
    if (blocks)
        return bf ? launch_write_blocks<true>(pool_dtype, pool, entries, dest_slot, n, dim, st)
                  : launch_write_blocks<false>(pool_dtype, pool, entries, dest_slot, n, dim, st);
    switch (pool_dtype) {
        case CT_KV_BF16: return bf ? launch_write<true, CT_KV_BF16>(pool, scales, entries, dest_slot, n, dim, st)
                                   : launch_write<false, CT_KV_BF16>(pool, scales, entries, dest_slot, n, dim, st);
        case CT_KV_F32:  return bf ? launch_write<true, CT_KV_F32>(pool, scales, entries, dest_slot, n, dim, st)
                                   : launch_write<false, CT_KV_F32>(pool, scales, entries, dest_slot, n, dim, st);
        case CT_KV_INT8: return bf ? launch_write<true, CT_KV_INT8>(pool, scales, entries, dest_slot, n, dim, st)
                                   : launch_write<false, CT_KV_INT8>(pool, scales, entries, dest_slot, n, dim, st);
        case CT_KV_E4M3: return bf ? launch_write<true, CT_KV_E4M3>(pool, scales, entries, dest_slot, n, dim, st)
                                   : launch_write<false, CT_KV_E4M3>(pool, scales, entries, dest_slot, n, dim, st);
        default: return CT_ERR_ARG;
    }
}

extern "C" int ct_kv_paged_move_pages(const void *src_pool, const float *src_scales, void *dst_pool,
                                      float *dst_scales, const int32_t *map, uint32_t n_pages,
                                      size_t page_bytes, uint32_t page_tokens, void *stream) {
    if (!src_pool || !dst_pool || !map || page_bytes % 16 != 0 || page_tokens > 256) return CT_ERR_ARG;
    if ((src_scales == NULL) != (dst_scales == NULL)) return CT_ERR_ARG;
    if (n_pages == 0) return CT_OK;
    k_move_pages<<<n_pages, 256, 0, (cudaStream_t)stream>>>(
        static_cast<const uint4 *>(src_pool), src_scales, static_cast<uint4 *>(dst_pool), dst_scales, map,
        page_bytes / 16, page_tokens);
    ct__count_launches(1);
    return ct__cuda_status(cudaGetLastError(), "move_pages");
}

namespace {

template <int D, bool Ob, int MC>
void gather_one(const void *pool, const float *scales, const int32_t *bt_row, uint32_t P, uint32_t dim, uint32_t start,
                uint32_t n, void *out, cudaStream_t st) {
    k_gather<D, Ob, MC><<<(n + kWarps - 1) / kWarps, 256, 0, st>>>(pool, scales, bt_row, P, dim, start, n, out);
}
template <int D, bool Ob, int MC>
void gather_many(const void *pool, const float *scales, const int32_t *bt, uint32_t maxp, uint32_t P, uint32_t dim,
                 const int4 *desc, uint32_t n_desc, uint32_t max_n, void *out, cudaStream_t st) {
    k_gather_batch<D, Ob, MC><<<dim3((max_n + kWarps - 1) / kWarps, n_desc), 256, 0, st>>>(pool, scales, bt, maxp, P,
                                                                                          dim, desc, out);
}

template <int D>
int gather_dispatch(bool ob, uint32_t chunks, const void *pool, const float *scales, const int32_t *bt, uint32_t maxp,
                    uint32_t P, uint32_t dim, uint32_t start, uint32_t n, const int4 *desc, uint32_t n_desc,
                    void *out, cudaStream_t st) {
    if (D != CT_KV_F32 && chunks * kTileTok <= 256u * kTileK) {
        const dim3 grid((n + kTileTok - 1) / kTileTok, desc ? n_desc : 1);
        if (ob) k_gather_tiled<D, true><<<grid, 256, 0, st>>>(pool, scales, bt, maxp, P, dim, start, n, desc, out);
        else    k_gather_tiled<D, false><<<grid, 256, 0, st>>>(pool, scales, bt, maxp, P, dim, start, n, desc, out);
        return CT_OK;
    }
    const int mc = chunks <= 32 ? 1 : chunks <= 64 ? 2 : chunks <= 128 ? 4 : 0;
    if (!mc) return CT_ERR_UNSUPPORTED;
#define CT_G(OB, MC) (desc ? gather_many<D, OB, MC>(pool, scales, bt, maxp, P, dim, desc, n_desc, n, out, st) \
                           : gather_one<D, OB, MC>(pool, scales, bt, P, dim, start, n, out, st))
    if (ob) { if (mc == 1) CT_G(true, 1); else if (mc == 2) CT_G(true, 2); else CT_G(true, 4); }
    else    { if (mc == 1) CT_G(false, 1); else if (mc == 2) CT_G(false, 2); else CT_G(false, 4); }
#undef CT_G
    return CT_OK;
}

int gather_any(uint32_t pool_dtype, bool ob, const void *pool, const float *scales, const int32_t *bt, uint32_t maxp,
               uint32_t P, uint32_t dim, uint32_t start, uint32_t n, const int4 *desc, uint32_t n_desc, void *out,
               cudaStream_t st) {
    const uint32_t chunks = dim / 16;
    int rc = CT_OK;
    if (pool_dtype >= CT_KV_Q8_0 && pool_dtype <= CT_KV_Q1_0) {
        if (dim % 32 != 0 || dim / 32 > (uint32_t)kMaxBlocks) return CT_ERR_ARG;
        switch (pool_dtype) {
            case CT_KV_Q8_0: launch_gather_blocks<CT_QUANT_Q8_0>(ob, pool, bt, maxp, P, dim, start, n, desc, n_desc, out, st); break;
            case CT_KV_Q4_0: launch_gather_blocks<CT_QUANT_Q4_0>(ob, pool, bt, maxp, P, dim, start, n, desc, n_desc, out, st); break;
            case CT_KV_Q2_0: launch_gather_blocks<CT_QUANT_Q2_0>(ob, pool, bt, maxp, P, dim, start, n, desc, n_desc, out, st); break;
            default:         launch_gather_blocks<CT_QUANT_Q1_0>(ob, pool, bt, maxp, P, dim, start, n, desc, n_desc, out, st); break;
        }
        ct__count_launches(1);
        return ct__cuda_status(cudaGetLastError(), "gather");
    }
    switch (pool_dtype) {
        case CT_KV_BF16: rc = gather_dispatch<CT_KV_BF16>(ob, chunks, pool, scales, bt, maxp, P, dim, start, n, desc, n_desc, out, st); break;
        case CT_KV_F32:  rc = gather_dispatch<CT_KV_F32>(ob, chunks, pool, scales, bt, maxp, P, dim, start, n, desc, n_desc, out, st); break;
        case CT_KV_INT8: rc = gather_dispatch<CT_KV_INT8>(ob, chunks, pool, scales, bt, maxp, P, dim, start, n, desc, n_desc, out, st); break;
        case CT_KV_E4M3: rc = gather_dispatch<CT_KV_E4M3>(ob, chunks, pool, scales, bt, maxp, P, dim, start, n, desc, n_desc, out, st); break;
        default: return CT_ERR_ARG;
    }
    if (rc) return rc;
    ct__count_launches(1);
    return ct__cuda_status(cudaGetLastError(), "gather");
}

}  // namespace

extern "C" int ct__launch_kv_gather(const void *pool, const float *scales, uint32_t pool_dtype,
                                    const int32_t *bt_row, uint32_t page_tokens, uint32_t dim,
                                    uint32_t start, uint32_t n, void *out, uint32_t out_dtype,
                                    void *stream) {
    if (n == 0) return CT_OK;
    if (dim % 16 != 0) return CT_ERR_ARG;
    return gather_any(pool_dtype, out_dtype == CT_KV_BF16, pool, scales, bt_row, 0, page_tokens, dim, start, n,
                      nullptr, 0, out, (cudaStream_t)stream);
}

extern "C" int ct__launch_kv_gather_batch(const void *pool, const float *scales, uint32_t pool_dtype,
                                          const int32_t *bt, uint32_t max_pages, uint32_t page_tokens,
                                          uint32_t dim, const void *desc, uint32_t n_desc, uint32_t max_count,
                                          void *out, uint32_t out_dtype, void *stream) {
    if (n_desc == 0 || max_count == 0) return CT_OK;
    if (dim % 16 != 0 || n_desc > 65535) return CT_ERR_ARG;
    return gather_any(pool_dtype, out_dtype == CT_KV_BF16, pool, scales, bt, max_pages, page_tokens, dim, 0, max_count,
                      static_cast<const int4 *>(desc), n_desc, out, (cudaStream_t)stream);
}

extern "C" int ct__launch_kv_compress(float *k, float *v, float *scratch, uint32_t n_layers,
                                      uint32_t max_ctx, uint32_t stride, uint32_t new_len,
                                      uint32_t step, void *stream) {
    if (new_len == 0 || stride == 0 || n_layers == 0) return CT_OK;
    cudaStream_t st = (cudaStream_t)stream;
    const size_t total = (size_t)n_layers * new_len * stride;
    const int grid = ct__grid_for(total / 4 + 1, 256, 148 * 16);
    if (stride % 4 == 0 && ((uintptr_t)k % 16 == 0) && ((uintptr_t)v % 16 == 0)) {
        k_compress_out<<<grid, 256, 0, st>>>((const float4 *)k, (const float4 *)v, (float4 *)scratch, max_ctx,
                                             stride / 4, new_len, step, n_layers);
        k_compress_in<<<grid, 256, 0, st>>>((float4 *)k, (float4 *)v, (const float4 *)scratch, max_ctx,
                                            stride / 4, new_len, n_layers);
    } else {
        k_compress_scalar<<<grid, 256, 0, st>>>(k, v, scratch, max_ctx, stride, new_len, step, n_layers, 0);
        k_compress_scalar<<<grid, 256, 0, st>>>(k, v, scratch, max_ctx, stride, new_len, step, n_layers, 1);
    }
    ct__count_launches(2);
    return ct__cuda_status(cudaGetLastError(), "compress");
}

/* Block-table / length mirror update: dst[pairs[2i]] = pairs[2i+1]. */
__global__ void k_scatter_i32(int32_t *dst, const int32_t *pairs, uint32_t n) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        dst[pairs[2 * i]] = pairs[2 * i + 1];
}

extern "C" int ct__launch_scatter_i32(int32_t *dst, const int32_t *pairs, uint32_t n_pairs, void *stream) {
    if (n_pairs == 0) return CT_OK;
    /* The host stages the final value for every index, so pairs repeating an
     * index carry the same value and may land in any order. */
    k_scatter_i32<<<ct__grid_for(n_pairs, 256, 148 * 4), 256, 0, (cudaStream_t)stream>>>(dst, pairs, n_pairs);
    ct__count_launches(1);
    return ct__cuda_status(cudaGetLastError(), "scatter_i32");
}

/* Gathered rows to their places: dst[ids[i]] = src[i] for n rows of
 * row_bytes (a multiple of 4).  A warp takes a 4 KB segment of a row (long
 * rows spread over many warps), its lanes' eight 16-byte loads in flight
 * before their stores; 4-byte words where the row or a pointer is not
 * 16-byte aligned. */
__global__ void k_scatter_rows(uint8_t *dst, const uint8_t *src, const uint32_t *ids, uint32_t n, size_t row_bytes) {
    const uint32_t lane = threadIdx.x & 31;
    const size_t seg_per_row = (row_bytes + 4095) / 4096, n_seg = (size_t)n * seg_per_row;
    const size_t warps = (size_t)gridDim.x * (blockDim.x / 32);
    for (size_t w = blockIdx.x * (size_t)(blockDim.x / 32) + (threadIdx.x >> 5); w < n_seg; w += warps) {
        const size_t r = w / seg_per_row, off = (w - r * seg_per_row) * 4096;
        const size_t len = row_bytes - off < 4096 ? row_bytes - off : 4096;
        const uint8_t *s = src + r * row_bytes + off;
        uint8_t *d = dst + (size_t)ids[r] * row_bytes + off;
        if (len % 16 == 0 && ((uintptr_t)s & 15) == 0 && ((uintptr_t)d & 15) == 0) {
            const uint4 *s4 = reinterpret_cast<const uint4 *>(s);
            uint4 *d4 = reinterpret_cast<uint4 *>(d);
            const uint32_t nv = (uint32_t)(len / 16);
            uint4 v[8];
            #pragma unroll
            for (int j = 0; j < 8; j++)
                if (lane + 32u * j < nv) v[j] = __ldcs(s4 + lane + 32 * j);
            #pragma unroll
            for (int j = 0; j < 8; j++)
                if (lane + 32u * j < nv) d4[lane + 32 * j] = v[j];
        } else {
            for (size_t i = lane; i < len / 4; i += 32)
                reinterpret_cast<uint32_t *>(d)[i] = reinterpret_cast<const uint32_t *>(s)[i];
        }
    }
}

extern "C" int ct__launch_scatter_rows(void *dst, const void *src, const uint32_t *ids, uint32_t n, size_t row_bytes,
                                       void *stream) {
    if (n == 0) return CT_OK;
    if (!dst || !src || !ids || row_bytes % 4 != 0) return CT_ERR_ARG;
    const size_t segs = (size_t)n * ((row_bytes + 4095) / 4096);
    k_scatter_rows<<<ct__grid_for(segs * 32, 256, 148 * 16), 256, 0, (cudaStream_t)stream>>>(
        static_cast<uint8_t *>(dst), static_cast<const uint8_t *>(src), ids, n, row_bytes);
    ct__count_launches(1);
    return ct__cuda_status(cudaGetLastError(), "scatter_rows");
}
