#ifndef CT_QUANT_H
#define CT_QUANT_H

/*
 * quant.h -- block and per-token quantisation codecs on B200.
 *
 * Part 1 keeps the reference interface of src/quant/quant.h:18-110 unchanged
 * (same block structs, enum values and signatures).  The encoders and
 * decoders run as CUDA kernels on copies of the caller's host buffers and are
 * bit-exact with the reference CPU code, including its fp16-scale quirks
 * (the encoder truncates, maps |d| < 2^-15 to Inf, and the decoder halves
 * subnormals).
 *
 * Part 2 adds the per-token KV codecs used by the paged cache: one fp32
 * absmax scale per token, int8 (d = amax/127, codes floor(x/d + 0.5) clamped
 * to +/-127, the Q8_0 rounding) or fp8 e4m3 (d = amax/448, round to nearest
 * even, saturating).  Device pointers.
 */

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ======================================================================== */
/* Part 1 -- reference interface (src/quant/quant.h:18-110)                 */
/* ======================================================================== */

#define CT_QUANT_BLOCK_SIZE 32

typedef struct { uint16_t d; int8_t  q[CT_QUANT_BLOCK_SIZE];     } ct_q8_0_block_t; /* 34 B */
typedef struct { uint16_t d; uint8_t q[CT_QUANT_BLOCK_SIZE / 2]; } ct_q4_0_block_t; /* 18 B */
typedef struct { uint16_t d; uint8_t q[CT_QUANT_BLOCK_SIZE / 4]; } ct_q2_0_block_t; /* 10 B */
typedef struct { uint16_t d; uint8_t q[CT_QUANT_BLOCK_SIZE / 8]; } ct_q1_0_block_t; /*  6 B */

typedef enum {
    CT_QUANT_FP16 = 0,
    CT_QUANT_Q8_0 = 1,
    CT_QUANT_Q4_0 = 2,
    CT_QUANT_Q2_0 = 3,
    CT_QUANT_Q1_0 = 4,
} ct_quant_type_t;

/* quant.h:57-66, integer division kept (Q8_0 -> 1, the others -> 0). */
static inline size_t ct_quant_bytes_per_float(ct_quant_type_t t) {
    switch (t) {
        case CT_QUANT_FP16: return 2;
        case CT_QUANT_Q8_0: return sizeof(ct_q8_0_block_t) / CT_QUANT_BLOCK_SIZE;
        case CT_QUANT_Q4_0: return sizeof(ct_q4_0_block_t) / CT_QUANT_BLOCK_SIZE;
        case CT_QUANT_Q2_0: return sizeof(ct_q2_0_block_t) / CT_QUANT_BLOCK_SIZE;
        case CT_QUANT_Q1_0: return sizeof(ct_q1_0_block_t) / CT_QUANT_BLOCK_SIZE;
        default: return 4;
    }
}

/* quant.h:71-80: n floats (a multiple of 32) -> n/32 blocks. */
void ct_quant_q8_0(const float *src, ct_q8_0_block_t *dst, int64_t n);
void ct_quant_q4_0(const float *src, ct_q4_0_block_t *dst, int64_t n);
void ct_quant_q2_0(const float *src, ct_q2_0_block_t *dst, int64_t n);
void ct_quant_q1_0(const float *src, ct_q1_0_block_t *dst, int64_t n);

/* quant.h:85-94 */
void ct_quant_deq8_0(const ct_q8_0_block_t *src, float *dst, int64_t n);
void ct_quant_deq4_0(const ct_q4_0_block_t *src, float *dst, int64_t n);
void ct_quant_deq2_0(const ct_q2_0_block_t *src, float *dst, int64_t n);
void ct_quant_deq1_0(const ct_q1_0_block_t *src, float *dst, int64_t n);

/* quant.h:99-102: returns bytes written, 0 on NULL / n % 32 != 0 / FP16. */
size_t ct_quant_do(const float *src, void *dst, int64_t n, ct_quant_type_t type);
void   ct_quant_undo(const void *src, float *dst, int64_t n, ct_quant_type_t type);

/* quant.h:107-110 */
uint16_t ct_quant_f32_to_fp16(float f);
float    ct_quant_fp16_to_f32(uint16_t h);

/* ======================================================================== */
/* Part 2 -- per-token KV codecs on device buffers (new)                    */
/* ======================================================================== */

/* x: device [n_tok][dim] (src_is_bf16: bf16 bits, else fp32);
 * codes: device [n_tok][dim] int8; scales: device [n_tok] fp32. */
int ct_quant_kv_int8(const void *x, int src_is_bf16, uint32_t n_tok, uint32_t dim,
                     int8_t *codes, float *scales, void *stream);
int ct_quant_kv_e4m3(const void *x, int src_is_bf16, uint32_t n_tok, uint32_t dim,
                     uint8_t *codes, float *scales, void *stream);
/* Decoders to fp32 (device). */
int ct_dequant_kv_int8(const int8_t *codes, const float *scales, uint32_t n_tok, uint32_t dim,
                       float *x, void *stream);
int ct_dequant_kv_e4m3(const uint8_t *codes, const float *scales, uint32_t n_tok, uint32_t dim,
                       float *x, void *stream);

/* Q8_0 on device buffers: x [n] fp32 -> n/32 blocks of 34 B, and back. */
int ct_quant_q8_0_dev(const float *x, void *blocks, int64_t n, void *stream);
int ct_dequant_q8_0_dev(const void *blocks, float *x, int64_t n, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* CT_QUANT_H */
