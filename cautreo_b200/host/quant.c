/*
 * quant.c -- the reference ct_quant_* interface (src/quant/quant.c) over the
 * device codecs of quant_kernels.cu.  Arguments, defaults and return values
 * as in the reference: n floats (a multiple of 32; trailing values beyond the
 * last whole block are ignored) -> n/32 blocks; ct_quant_do returns the bytes
 * written or 0; FP16 has no block codec and writes nothing.
 */
#include "../../include/hal.h"
#include "../../include/quant.h"
#include "../csrc/ct_internal.h"

#include <cuda_runtime_api.h>
#include <string.h>

static size_t block_bytes(int type) {
    switch (type) {
        case CT_QUANT_Q8_0: return sizeof(ct_q8_0_block_t);
        case CT_QUANT_Q4_0: return sizeof(ct_q4_0_block_t);
        case CT_QUANT_Q2_0: return sizeof(ct_q2_0_block_t);
        case CT_QUANT_Q1_0: return sizeof(ct_q1_0_block_t);
        default: return 0;
    }
}

/* Host -> device -> kernel -> host, on the legacy stream. */
static int run_codec(int type, int encode, const void *src, void *dst, int64_t n) {
    const int64_t nb = n / 32;
    if (nb <= 0) return CT_OK;
    const size_t fb = (size_t)nb * 32 * sizeof(float), bb = (size_t)nb * block_bytes(type);
    char *buf = NULL;
    int rc = ct__cuda_status(cudaMallocAsync((void **)&buf, fb + bb + 16, 0), "ct_quant");
    if (rc) return rc;
    float *df = (float *)buf;
    void *db = buf + fb;
    if (encode) {
        rc = ct__cuda_status(cudaMemcpyAsync(df, src, fb, cudaMemcpyHostToDevice, 0), "ct_quant");
        if (!rc) rc = ct__launch_q_blocks(type, df, db, nb * 32, NULL);
        if (!rc) rc = ct__cuda_status(cudaMemcpyAsync(dst, db, bb, cudaMemcpyDeviceToHost, 0), "ct_quant");
    } else {
        rc = ct__cuda_status(cudaMemcpyAsync(db, src, bb, cudaMemcpyHostToDevice, 0), "ct_quant");
        if (!rc) rc = ct__launch_deq_blocks(type, db, df, nb * 32, NULL);
        if (!rc) rc = ct__cuda_status(cudaMemcpyAsync(dst, df, fb, cudaMemcpyDeviceToHost, 0), "ct_quant");
    }
    cudaFreeAsync(buf, 0);
    int rc2 = ct__cuda_status(cudaStreamSynchronize(0), "ct_quant");
    return rc ? rc : rc2;
}

void ct_quant_q8_0(const float *src, ct_q8_0_block_t *dst, int64_t n) { run_codec(CT_QUANT_Q8_0, 1, src, dst, n); }
void ct_quant_q4_0(const float *src, ct_q4_0_block_t *dst, int64_t n) { run_codec(CT_QUANT_Q4_0, 1, src, dst, n); }
void ct_quant_q2_0(const float *src, ct_q2_0_block_t *dst, int64_t n) { run_codec(CT_QUANT_Q2_0, 1, src, dst, n); }
void ct_quant_q1_0(const float *src, ct_q1_0_block_t *dst, int64_t n) { run_codec(CT_QUANT_Q1_0, 1, src, dst, n); }
void ct_quant_deq8_0(const ct_q8_0_block_t *src, float *dst, int64_t n) { run_codec(CT_QUANT_Q8_0, 0, src, dst, n); }
void ct_quant_deq4_0(const ct_q4_0_block_t *src, float *dst, int64_t n) { run_codec(CT_QUANT_Q4_0, 0, src, dst, n); }
void ct_quant_deq2_0(const ct_q2_0_block_t *src, float *dst, int64_t n) { run_codec(CT_QUANT_Q2_0, 0, src, dst, n); }
void ct_quant_deq1_0(const ct_q1_0_block_t *src, float *dst, int64_t n) { run_codec(CT_QUANT_Q1_0, 0, src, dst, n); }

size_t ct_quant_do(const float *src, void *dst, int64_t n, ct_quant_type_t type) {
    if (!src || !dst || n % CT_QUANT_BLOCK_SIZE != 0) return 0;
    if (block_bytes(type) == 0) return 0;
    if (run_codec(type, 1, src, dst, n) != CT_OK) return 0;
    return (size_t)(n / CT_QUANT_BLOCK_SIZE) * block_bytes(type);
}

void ct_quant_undo(const void *src, float *dst, int64_t n, ct_quant_type_t type) {
    if (!src || !dst || n % CT_QUANT_BLOCK_SIZE != 0) return;
    if (block_bytes(type) == 0) return;
    run_codec(type, 0, src, dst, n);
}

/* Scalar conversions: the reference's bit rules (quant.c:16-75), as in the
 * device helpers ct_ref_f32_to_fp16 / ct_ref_fp16_to_f32 that the codecs use.
 * Pure integer work on one value: no device round trip. */
uint16_t ct_quant_f32_to_fp16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    uint32_t sgn = (u >> 31) & 1u, e = (u >> 23) & 0xFFu, m = u & 0x7FFFFFu;
    if (e == 0) return (uint16_t)(sgn << 15);
    if (e == 0xFF) return (uint16_t)((sgn << 15) | 0x7C00u | (m >> 13));
    uint32_t ne = e - 112u;
    if (ne >= 31u) return (uint16_t)((sgn << 15) | 0x7C00u);
    if (ne == 0u) return (uint16_t)((sgn << 15) | (((m | 0x800000u) >> 1) >> 13));
    return (uint16_t)((sgn << 15) | (ne << 10) | (m >> 13));
}

float ct_quant_fp16_to_f32(uint16_t h) {
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
    float f;
    memcpy(&f, &u, 4);
    return f;
}
