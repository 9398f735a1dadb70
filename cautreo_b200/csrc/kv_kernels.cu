/*
 * kv_kernels.cu -- HBM-bound kernels of the paged KV cache:
 *   write_slots   append / quantise-on-append (one warp per token)
 *   gather        block-table gather with dequantise-on-gather
 *   move_pages    page-granular gather used by defragmenting compaction
 *   compress      contiguous every-k-th token compaction (ct_kv_compress)
 *
 * Layout in HBM.  Pool: [n_pages][page_tokens][dim] values of the pool dtype
 * (bf16 / fp32 / int8 / e4m3); quantised pools add scales
 * [n_pages][page_tokens] fp32.  A token entry of the MLA cache is 576 bf16
 * = 1152 B (9 x 128 B lines); int8/e4m3 entries are 576 B + a 4 B scale.
 * Every kernel moves data in 16-byte vectors and requires dim % 16 == 0.
 */
#include "../../include/hal.h"
#include "../../include/kv_cache.h"
#include "ct_internal.h"

namespace {

constexpr int kWarps = 8;          /* tokens per 256-thread block */

/* Loads 16 consecutive source values of token `tok`, chunk `c` (16 values). */
template <bool SrcBf16>
__device__ __forceinline__ void load16(const void *src, size_t tok, uint32_t dim, uint32_t c, float v[16]) {
    if (SrcBf16) {
        const uint4 *p = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(src) + tok * dim + c * 16);
        uint4 a = __ldg(p), b = __ldg(p + 1);
        const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        #pragma unroll
        for (int i = 0; i < 8; i++) { v[2 * i] = __uint_as_float(w[i] << 16); v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u); }
    } else {
        const float4 *p = reinterpret_cast<const float4 *>(static_cast<const float *>(src) + tok * dim + c * 16);
        #pragma unroll
        for (int i = 0; i < 4; i++) { float4 f = __ldg(p + i); v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w; }
    }
}

/* K1 / K2: one warp per token.  Lane l owns 16-value chunks l, l+32, ...
 * (MaxChunks per lane); quantised pools need the token's absmax, reduced
 * with warp shuffles, before any code is written. */
template <bool SrcBf16, int PoolDtype, int MaxChunks>
__global__ void __launch_bounds__(256) k_write_slots(void *pool, float *scales, const void *src,
                                                     const int32_t *dest, uint32_t n, uint32_t dim) {
    const uint32_t warp = blockIdx.x * kWarps + (threadIdx.x >> 5);
    const uint32_t lane = threadIdx.x & 31;
    if (warp >= n) return;
    const int32_t slot = dest[warp];
    if (slot < 0) return;
    const uint32_t n_chunks = dim / 16;
    float v[MaxChunks][16];
    float amax = 0.0f;
    #pragma unroll
    for (int k = 0; k < MaxChunks; k++) {
        uint32_t c = lane + 32u * k;
        if (c < n_chunks) {
            load16<SrcBf16>(src, warp, dim, c, v[k]);
            #pragma unroll
            for (int i = 0; i < 16; i++) amax = fmaxf(amax, fabsf(v[k][i]));
        }
    }
    const size_t base = (size_t)slot * dim;
    if (PoolDtype == CT_KV_BF16) {
        #pragma unroll
        for (int k = 0; k < MaxChunks; k++) {
            uint32_t c = lane + 32u * k;
            if (c >= n_chunks) continue;
            uint32_t w[8];
            #pragma unroll
            for (int i = 0; i < 8; i++) w[i] = (uint32_t)ct_f32_to_bf16(v[k][2 * i]) | ((uint32_t)ct_f32_to_bf16(v[k][2 * i + 1]) << 16);
            uint4 *p = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(pool) + base + c * 16);
            p[0] = make_uint4(w[0], w[1], w[2], w[3]);
            p[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
    } else if (PoolDtype == CT_KV_F32) {
        #pragma unroll
        for (int k = 0; k < MaxChunks; k++) {
            uint32_t c = lane + 32u * k;
            if (c >= n_chunks) continue;
            float4 *p = reinterpret_cast<float4 *>(static_cast<float *>(pool) + base + c * 16);
            #pragma unroll
            for (int i = 0; i < 4; i++) p[i] = make_float4(v[k][4 * i], v[k][4 * i + 1], v[k][4 * i + 2], v[k][4 * i + 3]);
        }
    } else {
        amax = ct_warp_max(amax);
        const float d = __fdiv_rn(amax, PoolDtype == CT_KV_INT8 ? 127.0f : 448.0f);
        const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        #pragma unroll
        for (int k = 0; k < MaxChunks; k++) {
            uint32_t c = lane + 32u * k;
            if (c >= n_chunks) continue;
            uint32_t w[4] = {0, 0, 0, 0};
            #pragma unroll
            for (int i = 0; i < 16; i++) {
                uint32_t b = PoolDtype == CT_KV_INT8 ? (uint32_t)(uint8_t)(int8_t)ct_q8_code(v[k][i], id)
                                                     : (uint32_t)ct_e4m3_code(v[k][i], id);
                w[i >> 2] |= b << (8 * (i & 3));
            }
            *reinterpret_cast<uint4 *>(static_cast<uint8_t *>(pool) + base + c * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        if (lane == 0) scales[slot] = d;
    }
}

template <bool SrcBf16, int PoolDtype>
int launch_write(void *pool, float *scales, const void *src, const int32_t *dest, uint32_t n,
                 uint32_t dim, cudaStream_t st) {
    const uint32_t chunks = dim / 16;
    const int blocks = (int)((n + kWarps - 1) / kWarps);
    if (chunks <= 32) k_write_slots<SrcBf16, PoolDtype, 1><<<blocks, 256, 0, st>>>(pool, scales, src, dest, n, dim);
    else if (chunks <= 64) k_write_slots<SrcBf16, PoolDtype, 2><<<blocks, 256, 0, st>>>(pool, scales, src, dest, n, dim);
    else if (chunks <= 128) k_write_slots<SrcBf16, PoolDtype, 4><<<blocks, 256, 0, st>>>(pool, scales, src, dest, n, dim);
    else return CT_ERR_UNSUPPORTED;
    ct__count_launches(1);
    return ct__cuda_status(cudaGetLastError(), "write_slots");
}

/* K3: one warp per token, dequantising to fp32 or bf16. */
template <int PoolDtype, bool OutBf16>
__global__ void __launch_bounds__(256) k_gather(const void *pool, const float *scales,
                                                const int32_t *bt_row, uint32_t page_tokens,
                                                uint32_t dim, uint32_t start, uint32_t n, void *out) {
    const uint32_t t = blockIdx.x * kWarps + (threadIdx.x >> 5);
    const uint32_t lane = threadIdx.x & 31;
    if (t >= n) return;
    const uint32_t pos = start + t;
    const int32_t pg = bt_row[pos / page_tokens];
    const size_t slot = (size_t)pg * page_tokens + pos % page_tokens;
    const float sc = (PoolDtype == CT_KV_INT8 || PoolDtype == CT_KV_E4M3) ? scales[slot] : 1.0f;
    for (uint32_t c = lane; c < dim / 16; c += 32) {
        float v[16];
        if (PoolDtype == CT_KV_BF16) load16<true>(pool, slot, dim, c, v);
        else if (PoolDtype == CT_KV_F32) load16<false>(pool, slot, dim, c, v);
        else {
            uint4 w = __ldg(reinterpret_cast<const uint4 *>(static_cast<const uint8_t *>(pool) + slot * dim + c * 16));
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
            #pragma unroll
            for (int i = 0; i < 16; i++) {
                uint8_t b = (uint8_t)(ws[i >> 2] >> (8 * (i & 3)));
                v[i] = (PoolDtype == CT_KV_INT8 ? (float)(int8_t)b : ct_e4m3_to_f32(b)) * sc;
            }
        }
        if (OutBf16) {
            uint32_t w[8];
            #pragma unroll
            for (int i = 0; i < 8; i++) w[i] = (uint32_t)ct_f32_to_bf16(v[2 * i]) | ((uint32_t)ct_f32_to_bf16(v[2 * i + 1]) << 16);
            uint4 *p = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(out) + (size_t)t * dim + c * 16);
            p[0] = make_uint4(w[0], w[1], w[2], w[3]);
            p[1] = make_uint4(w[4], w[5], w[6], w[7]);
        } else {
            float4 *p = reinterpret_cast<float4 *>(static_cast<float *>(out) + (size_t)t * dim + c * 16);
            #pragma unroll
            for (int i = 0; i < 4; i++) p[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
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

extern "C" int ct_kv_paged_write_slots(void *pool, float *scales, uint32_t pool_dtype, const void *entries,
                                       uint32_t src_dtype, const int32_t *dest_slot, uint32_t n,
                                       uint32_t dim, void *stream) {
    if (!pool || !entries || !dest_slot || dim == 0 || dim % 16 != 0) return CT_ERR_ARG;
    if ((pool_dtype == CT_KV_INT8 || pool_dtype == CT_KV_E4M3) && !scales) return CT_ERR_ARG;
    if (n == 0) return CT_OK;
    cudaStream_t st = (cudaStream_t)stream;
    const bool bf = src_dtype == CT_KV_BF16;
    if (!bf && src_dtype != CT_KV_F32) return CT_ERR_ARG;
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

extern "C" int ct__launch_kv_gather(const void *pool, const float *scales, uint32_t pool_dtype,
                                    const int32_t *bt_row, uint32_t page_tokens, uint32_t dim,
                                    uint32_t start, uint32_t n, void *out, uint32_t out_dtype,
                                    void *stream) {
    if (n == 0) return CT_OK;
    if (dim % 16 != 0) return CT_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    const int blocks = (int)((n + kWarps - 1) / kWarps);
    const bool ob = out_dtype == CT_KV_BF16;
#define CT_GATHER(D) (ob ? (k_gather<D, true><<<blocks, 256, 0, st>>>(pool, scales, bt_row, page_tokens, dim, start, n, out), 0) \
                         : (k_gather<D, false><<<blocks, 256, 0, st>>>(pool, scales, bt_row, page_tokens, dim, start, n, out), 0))
    switch (pool_dtype) {
        case CT_KV_BF16: CT_GATHER(CT_KV_BF16); break;
        case CT_KV_F32:  CT_GATHER(CT_KV_F32); break;
        case CT_KV_INT8: CT_GATHER(CT_KV_INT8); break;
        case CT_KV_E4M3: CT_GATHER(CT_KV_E4M3); break;
        default: return CT_ERR_ARG;
    }
#undef CT_GATHER
    ct__count_launches(1);
    return ct__cuda_status(cudaGetLastError(), "gather");
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
