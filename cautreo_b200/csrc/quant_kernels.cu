/*
 * quant_kernels.cu -- block codecs of src/quant/quant.c on the device, and
 * the per-token KV codecs.
 *
 * Block codecs (Q8_0 / Q4_0 / Q2_0 / Q1_0, 32 values per block): one thread
 * per block, the reference's arithmetic step for step (quant.c:77-249):
 * d = amax / qmax in fp32, the fp16 scale from the reference's truncating
 * encoder, codes from the fp32 d via floor(x * (1/d) + 0.5) with every
 * operation individually rounded, and decode with the fp16-rounded scale.
 * Block layout: u16 scale followed by the packed codes (34 / 18 / 10 / 6 B).
 *
 * The block codecs and the per-token encoders run on the paged cache's
 * append and gather kernels where the shapes allow (kv_kernels.cu:
 * ct__launch_encode_blocks / _decode_blocks / _quant_tokens: the same
 * arithmetic, coalesced); the kernels here cover the rest.
 *
 * Per-token codecs: one warp per token, absmax by warp shuffle; decode by
 * 16-code vectors when the entry is a multiple of 16 codes.
 */
#include "../../include/hal.h"
#include "../../include/quant.h"
#include "ct_internal.h"

namespace {

/* One thread per block; the arithmetic is ct_block_encode / ct_block_decode,
 * shared with the block-quantised page pools of the paged cache. */
template <int Type>
__global__ void k_quant_blocks(const float *src, uint8_t *dst, int64_t nb) {
    constexpr int kBytes = CtBlock<Type>::kBytes;
    for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < nb; b += (int64_t)gridDim.x * blockDim.x) {
        float x[32];
        #pragma unroll
        for (int i = 0; i < 32; i++) x[i] = src[b * 32 + i];
        ct_block_encode<Type>(x, dst + b * kBytes);
    }
}

template <int Type>
__global__ void k_dequant_blocks(const uint8_t *src, float *dst, int64_t nb) {
    constexpr int kBytes = CtBlock<Type>::kBytes;
    for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < nb; b += (int64_t)gridDim.x * blockDim.x) {
        float x[32];
        ct_block_decode<Type>(src + b * kBytes, x);
        #pragma unroll
        for (int i = 0; i < 32; i++) dst[b * 32 + i] = x[i];
    }
}

/* Per-token codecs: one warp per token, values strided by lane. */
template <bool Int8, bool SrcBf16>
__global__ void __launch_bounds__(256) k_quant_tokens(const void *x, uint32_t n_tok, uint32_t dim,
                                                      uint8_t *codes, float *scales) {
    const uint32_t t = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (t >= n_tok) return;
    auto val = [&](uint32_t i) -> float {
        return SrcBf16 ? ct_bf16_to_f32(static_cast<const uint16_t *>(x)[(size_t)t * dim + i])
                       : static_cast<const float *>(x)[(size_t)t * dim + i];
    };
    float amax = 0.0f;
    for (uint32_t i = lane; i < dim; i += 32) amax = fmaxf(amax, fabsf(val(i)));
    amax = ct_warp_max(amax);
    const float d = __fdiv_rn(amax, Int8 ? 127.0f : 448.0f);
    const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    for (uint32_t i = lane; i < dim; i += 32)
        codes[(size_t)t * dim + i] = Int8 ? (uint8_t)(int8_t)ct_q8_code(val(i), id) : ct_e4m3_code(val(i), id);
    if (lane == 0) scales[t] = d;
}

/* 16 codes (one 16-byte vector) of a token per thread -> four float4. */
template <bool Int8>
__global__ void __launch_bounds__(256) k_dequant_tokens16(const uint8_t *codes, const float *scales, uint32_t n_tok,
                                                          uint32_t dim, float *x) {
    const uint32_t per = dim / 16;
    const size_t total = (size_t)n_tok * per;
    for (size_t c = blockIdx.x * (size_t)blockDim.x + threadIdx.x; c < total; c += (size_t)gridDim.x * blockDim.x) {
        const float sc = __ldg(scales + (total <= 0xFFFFFFFFu ? (size_t)((uint32_t)c / per) : c / per));
        const uint4 v = __ldcs(reinterpret_cast<const uint4 *>(codes) + c);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        float4 *o = reinterpret_cast<float4 *>(x) + 4 * c;
        #pragma unroll
        for (int j = 0; j < 4; j++) {
            float f[4];
            #pragma unroll
            for (int b = 0; b < 4; b++) {
                const uint8_t u = (uint8_t)(w[j] >> (8 * b));
                f[b] = __fmul_rn(Int8 ? (float)(int8_t)u : ct_e4m3_to_f32(u), sc);
            }
            __stcs(o + j, make_float4(f[0], f[1], f[2], f[3]));
        }
    }
}

template <bool Int8>
__global__ void k_dequant_tokens(const uint8_t *codes, const float *scales, uint32_t n_tok, uint32_t dim, float *x) {
    const size_t total = (size_t)n_tok * dim;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const float sc = scales[i / dim];
        const uint8_t b = codes[i];
        x[i] = __fmul_rn(Int8 ? (float)(int8_t)b : ct_e4m3_to_f32(b), sc);
    }
}

}  // namespace

extern "C" int ct__launch_q_blocks(int type, const float *x, void *blocks, int64_t n, void *stream) {
    if (n <= 0) return CT_OK;
    if (type < CT_QUANT_Q8_0 || type > CT_QUANT_Q1_0) return CT_ERR_ARG;
    const int fast = ct__launch_encode_blocks(type, x, blocks, n, stream);
    if (fast != CT_ERR_UNSUPPORTED) return fast;
    const int64_t nb = n / 32;
    const int grid = ct__grid_for((size_t)nb, 128, 148 * 8);
    cudaStream_t st = (cudaStream_t)stream;
    uint8_t *dst = static_cast<uint8_t *>(blocks);
    switch (type) {
        case CT_QUANT_Q8_0: k_quant_blocks<CT_QUANT_Q8_0><<<grid, 128, 0, st>>>(x, dst, nb); break;
        case CT_QUANT_Q4_0: k_quant_blocks<CT_QUANT_Q4_0><<<grid, 128, 0, st>>>(x, dst, nb); break;
        case CT_QUANT_Q2_0: k_quant_blocks<CT_QUANT_Q2_0><<<grid, 128, 0, st>>>(x, dst, nb); break;
        case CT_QUANT_Q1_0: k_quant_blocks<CT_QUANT_Q1_0><<<grid, 128, 0, st>>>(x, dst, nb); break;
        default: return CT_ERR_ARG;
    }
    ct__count_launches(1);
    return ct__cuda_status(cudaGetLastError(), "quant_blocks");
}

extern "C" int ct__launch_deq_blocks(int type, const void *blocks, float *x, int64_t n, void *stream) {
    if (n <= 0) return CT_OK;
    if (type < CT_QUANT_Q8_0 || type > CT_QUANT_Q1_0) return CT_ERR_ARG;
    const int fast = ct__launch_decode_blocks(type, blocks, x, n, stream);
    if (fast != CT_ERR_UNSUPPORTED) return fast;
    const int64_t nb = n / 32;
    const int grid = ct__grid_for((size_t)nb, 128, 148 * 8);
    cudaStream_t st = (cudaStream_t)stream;
    const uint8_t *src = static_cast<const uint8_t *>(blocks);
    switch (type) {
        case CT_QUANT_Q8_0: k_dequant_blocks<CT_QUANT_Q8_0><<<grid, 128, 0, st>>>(src, x, nb); break;
        case CT_QUANT_Q4_0: k_dequant_blocks<CT_QUANT_Q4_0><<<grid, 128, 0, st>>>(src, x, nb); break;
        case CT_QUANT_Q2_0: k_dequant_blocks<CT_QUANT_Q2_0><<<grid, 128, 0, st>>>(src, x, nb); break;
        case CT_QUANT_Q1_0: k_dequant_blocks<CT_QUANT_Q1_0><<<grid, 128, 0, st>>>(src, x, nb); break;
        default: return CT_ERR_ARG;
    }
    ct__count_launches(1);
    return ct__cuda_status(cudaGetLastError(), "dequant_blocks");
}

extern "C" int ct_quant_q8_0_dev(const float *x, void *blocks, int64_t n, void *stream) {
    if (!x || !blocks || n < 0 || n % 32 != 0) return CT_ERR_ARG;
    return ct__launch_q_blocks(CT_QUANT_Q8_0, x, blocks, n, stream);
}

extern "C" int ct_dequant_q8_0_dev(const void *blocks, float *x, int64_t n, void *stream) {
    if (!x || !blocks || n < 0 || n % 32 != 0) return CT_ERR_ARG;
    return ct__launch_deq_blocks(CT_QUANT_Q8_0, blocks, x, n, stream);
}

static int quant_tokens(bool int8, const void *x, int src_is_bf16, uint32_t n_tok, uint32_t dim,
                        uint8_t *codes, float *scales, void *stream) {
    if (!x || !codes || !scales || dim == 0) return CT_ERR_ARG;
    if (n_tok == 0) return CT_OK;
    const bool aligned = ((uintptr_t)x & 15) == 0 && ((uintptr_t)codes & 15) == 0;
    if (aligned) {
        const int fast = ct__launch_quant_tokens(int8, x, src_is_bf16, n_tok, dim, codes, scales, stream);
        if (fast != CT_ERR_UNSUPPORTED) return fast;
    }
    const int grid = (int)((n_tok + 7) / 8);
    cudaStream_t st = (cudaStream_t)stream;
    if (int8) {
        if (src_is_bf16) k_quant_tokens<true, true><<<grid, 256, 0, st>>>(x, n_tok, dim, codes, scales);
        else k_quant_tokens<true, false><<<grid, 256, 0, st>>>(x, n_tok, dim, codes, scales);
    } else {
        if (src_is_bf16) k_quant_tokens<false, true><<<grid, 256, 0, st>>>(x, n_tok, dim, codes, scales);
        else k_quant_tokens<false, false><<<grid, 256, 0, st>>>(x, n_tok, dim, codes, scales);
    }
    ct__count_launches(1);
    return ct__cuda_status(cudaGetLastError(), "quant_tokens");
}

extern "C" int ct_quant_kv_int8(const void *x, int src_is_bf16, uint32_t n_tok, uint32_t dim,
                                int8_t *codes, float *scales, void *stream) {
    return quant_tokens(true, x, src_is_bf16, n_tok, dim, reinterpret_cast<uint8_t *>(codes), scales, stream);
}

extern "C" int ct_quant_kv_e4m3(const void *x, int src_is_bf16, uint32_t n_tok, uint32_t dim,
                                uint8_t *codes, float *scales, void *stream) {
    return quant_tokens(false, x, src_is_bf16, n_tok, dim, codes, scales, stream);
}

extern "C" int ct_dequant_kv_int8(const int8_t *codes, const float *scales, uint32_t n_tok, uint32_t dim,
                                  float *x, void *stream) {
    if (!codes || !scales || !x) return CT_ERR_ARG;
    if ((size_t)n_tok * dim == 0) return CT_OK;
    if (dim % 16 == 0 && ((uintptr_t)codes & 15) == 0 && ((uintptr_t)x & 15) == 0) {
        const int g16 = ct__grid_for((size_t)n_tok * (dim / 16), 256, 148 * 16);
        k_dequant_tokens16<true><<<g16, 256, 0, (cudaStream_t)stream>>>(reinterpret_cast<const uint8_t *>(codes), scales,
                                                                         n_tok, dim, x);
        ct__count_launches(1);
        return ct__cuda_status(cudaGetLastError(), "dequant_int8");
    }
    const int grid = ct__grid_for((size_t)n_tok * dim, 256, 148 * 8);
    k_dequant_tokens<true><<<grid, 256, 0, (cudaStream_t)stream>>>(reinterpret_cast<const uint8_t *>(codes), scales, n_tok, dim, x);
    ct__count_launches(1);
    return ct__cuda_status(cudaGetLastError(), "dequant_int8");
}

extern "C" int ct_dequant_kv_e4m3(const uint8_t *codes, const float *scales, uint32_t n_tok, uint32_t dim,
                                  float *x, void *stream) {
    if (!codes || !scales || !x) return CT_ERR_ARG;
    if ((size_t)n_tok * dim == 0) return CT_OK;
    if (dim % 16 == 0 && ((uintptr_t)codes & 15) == 0 && ((uintptr_t)x & 15) == 0) {
        const int g16 = ct__grid_for((size_t)n_tok * (dim / 16), 256, 148 * 16);
        k_dequant_tokens16<false><<<g16, 256, 0, (cudaStream_t)stream>>>(codes, scales, n_tok, dim, x);
        ct__count_launches(1);
        return ct__cuda_status(cudaGetLastError(), "dequant_e4m3");
    }
    const int grid = ct__grid_for((size_t)n_tok * dim, 256, 148 * 8);
    k_dequant_tokens<false><<<grid, 256, 0, (cudaStream_t)stream>>>(codes, scales, n_tok, dim, x);
    ct__count_launches(1);
    return ct__cuda_status(cudaGetLastError(), "dequant_e4m3");
}
