/*
 * ct_internal.h -- internal interface between the C11 host layer
 * (cautreo_b200/host) and the CUDA kernels (cautreo_b200/csrc).
 * Plain C declarations; device helpers only when compiled by nvcc.
 */
#ifndef CT_INTERNAL_H
#define CT_INTERNAL_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* fp32 -> bf16 bits on the host, the same round-to-nearest-even integer rule
 * as the device's ct_f32_to_bf16 (ds4_forward.c:60-66). */
static inline uint16_t ct_f32_to_bf16_host(float f) {
    union { float f; uint32_t u; } v;
    v.f = f;
    return (uint16_t)((v.u + 0x7FFFu + ((v.u >> 16) & 1u)) >> 16);
}

/* ---- bookkeeping shared by every launcher (host/runtime.c) ------------- */
/* Records a CUDA error (code from cudaError_t) with a location; returns
 * CT_ERR_CUDA (or CT_OK when code == 0). */
int  ct__cuda_status(int code, const char *where);
void ct__count_launches(uint32_t n);
/* Sets the last-error message without a CUDA code. */
void ct__set_error(const char *msg);
/* Stream-ordered temporary device memory from a memory pool private to the
 * library (one per device, keeping up to 1 GiB cached between calls, so a
 * call repeated every step neither maps nor unmaps memory).  Free on the
 * same stream. */
int  ct__scratch_alloc(void **p, size_t bytes, void *stream);
void ct__scratch_free(void *p, void *stream);

/* ---- MLA decode work plan (shared by host/attention.c and the kernels) -- */
typedef struct {
    int32_t seq;         /* output row */
    int32_t row;         /* block-table row */
    int32_t page_begin;  /* first logical page of the chunk */
    int32_t page_end;    /* one past the last */
    int32_t part;        /* partial-result slot, or -1: write the final output */
    int32_t pad[3];
} ct_mla_chunk_t;

typedef struct {
    int32_t seq;         /* output row */
    int32_t first_part;  /* first partial-result slot */
    int32_t n_parts;
    int32_t pad;
} ct_mla_combine_t;

typedef struct {
    uint32_t n_heads, entry_dim, v_dim, page_tokens, max_pages_per_seq, kv_dtype;
    float    scale;
    uint32_t n_pages;    /* pool pages: bounds every page read */
    uint32_t n_seq;      /* rows of q / out */
} ct_mla_dims_t;

/* ---- launchers (csrc); all return a ct_status_t ------------------------- */
int ct__launch_kv_gather(const void *pool, const float *scales, uint32_t pool_dtype,
                         const int32_t *bt_row, uint32_t page_tokens, uint32_t dim,
                         uint32_t start, uint32_t n, void *out, uint32_t out_dtype,
                         void *stream);
/* Several (seq, start, count, first output row) ranges in one launch; desc is
 * a device array of n_desc int4, max_count the largest count. */
int ct__launch_kv_gather_batch(const void *pool, const float *scales, uint32_t pool_dtype, const int32_t *bt,
                               uint32_t max_pages, uint32_t page_tokens, uint32_t dim, const void *desc,
                               uint32_t n_desc, uint32_t max_count, void *out, uint32_t out_dtype, void *stream);
int ct__launch_kv_compress(float *k, float *v, float *scratch, uint32_t n_layers,
                           uint32_t max_ctx, uint32_t stride, uint32_t new_len,
                           uint32_t step, void *stream);

int ct__launch_q_blocks(int type, const float *x, void *blocks, int64_t n, void *stream);
int ct__launch_deq_blocks(int type, const void *blocks, float *x, int64_t n, void *stream);
/* The same on the paged cache's kernels (kv_kernels.cu); CT_ERR_UNSUPPORTED
 * when the shape or alignment does not suit them. */
int ct__launch_encode_blocks(int type, const float *x, void *blocks, int64_t n, void *stream);
int ct__launch_decode_blocks(int type, const void *blocks, float *x, int64_t n, void *stream);
int ct__launch_quant_tokens(int int8, const void *x, int src_is_bf16, uint32_t n_tok, uint32_t dim, void *codes,
                            float *scales, void *stream);

/* ct_attn_forward / ct_attn_softmax on device buffers; scratch of the size
 * the _scratch_bytes functions give (long inputs run split over CTAs). */
size_t ct__attn_scratch_bytes(uint32_t n_tokens, uint32_t n_heads, uint32_t head_dim);
int ct__launch_attn_shared(const float *q, const float *k, const float *v, uint32_t n_tokens,
                           uint32_t n_heads, uint32_t head_dim, float scale, float *out,
                           float *scratch, void *stream);
size_t ct__softmax_scratch_bytes(uint32_t n);
int ct__launch_softmax(float *x, uint32_t n, void *scratch, void *stream);
/* dst[ids[i]] = src[i] for n rows of row_bytes (a multiple of 4). */
int ct__launch_scatter_rows(void *dst, const void *src, const uint32_t *ids, uint32_t n, size_t row_bytes,
                            void *stream);

/* Work list of n_seq sequences from the device lengths (mla_plan.cu):
 * chunks [n_seq + n_workers], worker_begin [n_workers + 1], combines,
 * counts[2] = (chunks, combines) written. */
int ct__launch_mla_plan(const uint32_t *rows, const int32_t *seq_lens, uint32_t n_seq, uint32_t page_tokens,
                        uint32_t max_pages, uint32_t n_workers, ct_mla_chunk_t *chunks, int32_t *worker_begin,
                        ct_mla_combine_t *combines, int32_t *counts, void *stream);
/* counts (device, may be NULL): how many of the n_chunks / n_combines
 * entries are in use (the CUDA-core and combine launches cover n_chunks /
 * n_combines blocks and skip the rest). */
int ct__launch_mla_decode(const ct_mla_dims_t *dims, const ct_mla_chunk_t *chunks,
                          uint32_t n_chunks, const int32_t *worker_begin, uint32_t n_workers,
                          const ct_mla_combine_t *combines,
                          uint32_t n_combines, const int32_t *counts, const void *q, const void *pool,
                          const float *scales, const int32_t *block_table,
                          const int32_t *seq_lens, void *out, float *lse, float *part_o,
                          float *part_ml, void *stream, uint32_t *n_launches);

#ifdef __cplusplus
}
#endif

/* ------------------------------------------------------------------------ */
#ifdef __CUDACC__
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#define CT_DEV __device__ __forceinline__

/* bf16 bits -> fp32 (exact). */
CT_DEV float ct_bf16_to_f32(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }

/* fp32 -> bf16 bits, round to nearest even on the dropped 16 bits; the same
 * integer rule as the reference's f32_to_bf16 (ds4_forward.c:60-66). */
CT_DEV uint16_t ct_f32_to_bf16(float f) {
    uint32_t u = __float_as_uint(f);
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

/* The reference fp16 scale encoder (quant.c:16-45), including its
 * truncation and the unsigned exponent wrap that turns |x| < 2^-15 into Inf. */
CT_DEV uint16_t ct_ref_f32_to_fp16(float f) {
    uint32_t u = __float_as_uint(f);
    uint32_t sgn = (u >> 31) & 1u, e = (u >> 23) & 0xFFu, m = u & 0x7FFFFFu;
    if (e == 0) return (uint16_t)(sgn << 15);
    if (e == 0xFF) return (uint16_t)((sgn << 15) | 0x7C00u | (m >> 13));
    uint32_t ne = e - 112u;
    if (ne >= 31u) return (uint16_t)((sgn << 15) | 0x7C00u);
    if (ne == 0u) return (uint16_t)((sgn << 15) | (((m | 0x800000u) >> 1) >> 13));
    return (uint16_t)((sgn << 15) | (ne << 10) | (m >> 13));
}

/* The reference fp16 decoder (quant.c:47-75), subnormal rule included. */
CT_DEV float ct_ref_fp16_to_f32(uint16_t h) {
    uint32_t sgn = (h >> 15) & 1u, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, u;
    if (e == 0) {
        if (m == 0) u = sgn << 31;
        else {
            uint32_t ex = 112u;
            while (!(m & 0x400u)) { m <<= 1; ex--; }
            u = (sgn << 31) | (ex << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (e == 31) {
        u = (sgn << 31) | 0x7F800000u | (m << 13);
    } else {
        u = (sgn << 31) | ((e + 112u) << 23) | (m << 13);
    }
    return __uint_as_float(u);
}

/* int8 code with the Q8_0 rounding: floor(x*id + 0.5), clamp +/-127, every
 * operation individually rounded (no FMA contraction). */
CT_DEV int ct_q8_code(float x, float id) {
    int q = (int)floorf(__fadd_rn(__fmul_rn(x, id), 0.5f));
    return q > 127 ? 127 : (q < -127 ? -127 : q);
}

/* ---- block codecs of quant.c (32 values per block) ---------------------
 * Type: 1 = Q8_0 (34 B), 2 = Q4_0 (18 B), 3 = Q2_0 (10 B), 4 = Q1_0 (6 B),
 * the ct_quant_type_t values.  Block = u16 reference-fp16 scale, then the
 * packed codes (quant.c:77-249): d = amax / qmax in fp32 (qmax 127 / 7 / 1),
 * codes floor(x * (1/d) + 0.5) clamped to +/-qmax from the fp32 d, Q4_0 two
 * 4-bit two's-complement codes per byte (low nibble first), Q2_0 four
 * (code + 1) per byte (low bits first), Q1_0 the sign bits (x >= 0) with the
 * fp16 of amax as the scale.  Decoding multiplies by the fp16-rounded d. */
template <int Type> struct CtBlock {
    static constexpr int kBytes = Type == 1 ? 34 : Type == 2 ? 18 : Type == 3 ? 10 : 6;
};

/* The reference converts floorf(v) with a C (int) cast, which on x86-64
 * (cvttss2si) gives INT_MIN for NaN and for values outside the int range;
 * the clamp then turns INT_MIN into -lim.  So v NaN or >= 2^31 codes -lim
 * here too (a CUDA cast would give 0 for NaN and saturate at INT_MAX), and
 * v < -2^31 saturates to INT_MIN, also -lim. */
CT_DEV int ct_block_code(float x, float id, int lim) {
    const float v = __fadd_rn(__fmul_rn(x, id), 0.5f);
    if (!(v < 2147483648.0f)) return -lim;
    const int q = (int)floorf(v);
    return q > lim ? lim : (q < -lim ? -lim : q);
}

template <int Type>
CT_DEV void ct_block_encode(const float *x, uint8_t *blk) {
    float amax = 0.0f;
    #pragma unroll
    for (int i = 0; i < 32; i++) { const float a = fabsf(x[i]); if (a > amax) amax = a; }
    if (Type == 4) {
        const uint16_t h = ct_ref_f32_to_fp16(amax);
        blk[0] = (uint8_t)h; blk[1] = (uint8_t)(h >> 8);
        #pragma unroll
        for (int i = 0; i < 32; i += 8) {
            uint32_t byte = 0;
            #pragma unroll
            for (int j = 0; j < 8; j++) if (x[i + j] >= 0) byte |= 1u << j;
            blk[2 + i / 8] = (uint8_t)byte;
        }
        return;
    }
    const float qmax = Type == 1 ? 127.0f : Type == 2 ? 7.0f : 1.0f;
    const float d = __fdiv_rn(amax, qmax);
    const uint16_t h = ct_ref_f32_to_fp16(d);
    blk[0] = (uint8_t)h; blk[1] = (uint8_t)(h >> 8);
    const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    if (Type == 1) {
        #pragma unroll
        for (int i = 0; i < 32; i++) blk[2 + i] = (uint8_t)(int8_t)ct_block_code(x[i], id, 127);
    } else if (Type == 2) {
        #pragma unroll
        for (int i = 0; i < 32; i += 2) {
            const int q0 = ct_block_code(x[i], id, 7), q1 = ct_block_code(x[i + 1], id, 7);
            blk[2 + i / 2] = (uint8_t)((q0 & 0xF) | ((q1 & 0xF) << 4));
        }
    } else {
        #pragma unroll
        for (int i = 0; i < 32; i += 4) {
            uint32_t byte = 0;
            #pragma unroll
            for (int j = 0; j < 4; j++) byte |= (uint32_t)((ct_block_code(x[i + j], id, 1) + 1) & 3) << (2 * j);
            blk[2 + i / 4] = (uint8_t)byte;
        }
    }
}

template <int Type>
CT_DEV void ct_block_decode(const uint8_t *blk, float *x) {
    const float d = ct_ref_fp16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
    #pragma unroll
    for (int i = 0; i < 32; i++) {
        int q;
        if (Type == 1) q = (int8_t)blk[2 + i];
        else if (Type == 2) { q = (blk[2 + i / 2] >> (4 * (i & 1))) & 0xF; if (q >= 8) q -= 16; }
        else if (Type == 3) q = (int)((blk[2 + i / 4] >> (2 * (i & 3))) & 3) - 1;
        else { x[i] = (blk[2 + i / 8] >> (i & 7)) & 1 ? d : -d; continue; }
        x[i] = __fmul_rn((float)q, d);
    }
}

/* e4m3 code of x * id, round-to-nearest-even, saturating to +/-448. */
CT_DEV uint8_t ct_e4m3_code(float x, float id) {
    return (uint8_t)__nv_cvt_float_to_fp8(__fmul_rn(x, id), __NV_SATFINITE, __NV_E4M3);
}

CT_DEV float ct_e4m3_to_f32(uint8_t v) {
    __half_raw hr = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)v, __NV_E4M3);
    return __half2float(__half(hr));
}

/* Two e4m3 codes (low byte first) -> two floats, one conversion per pair. */
CT_DEV float2 ct_e4m3x2_to_f32x2(uint16_t v) {
    __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)v, __NV_E4M3);
    return __half22float2(__half2(hr));
}

/* e4m3 codes of (x0 * id, x1 * id) packed low byte first, RNE, saturating. */
CT_DEV uint16_t ct_e4m3x2_code(float x0, float x1, float id) {
    return (uint16_t)__nv_cvt_float2_to_fp8x2(make_float2(__fmul_rn(x0, id), __fmul_rn(x1, id)), __NV_SATFINITE,
                                              __NV_E4M3);
}

CT_DEV float ct_warp_max(float v) {
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    return v;
}

CT_DEV float ct_warp_sum(float v) {
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

static inline int ct__grid_for(size_t items, int per_block, int cap) {
    size_t g = (items + per_block - 1) / per_block;
    if (g < 1) g = 1;
    if ((size_t)cap < g) g = cap;
    return (int)g;
}
#endif /* __CUDACC__ */

#endif /* CT_INTERNAL_H */
