/*
 * mla_tc.cu -- paged absorbed-MLA decode on the 5th-generation tensor cores
 * (tcgen05 + TMEM + TMA) for the DeepSeek shape: 128 query heads, 576-value
 * entries (512 latent + 64 rope), 512 value dims, 64-token bf16 pages.
 */
#include "../../include/attention.h"
#include "../../include/hal.h"
#include "../../include/kv_cache.h"
#include "ct_internal.h"

extern "C" int ct__mla_tc_workers(const ct_mla_dims_t *dims, int device) {
    (void)dims; (void)device;
    return 0;
}

extern "C" int ct__launch_mla_tc(const ct_mla_dims_t *dims, const ct_mla_chunk_t *chunks, uint32_t n_chunks,
                                 const int32_t *worker_begin, uint32_t n_workers, const void *q,
                                 const void *pool, const int32_t *block_table, const int32_t *seq_lens,
                                 void *out, float *lse, float *part_o, float *part_ml, void *stream) {
    (void)dims; (void)chunks; (void)n_chunks; (void)worker_begin; (void)n_workers; (void)q; (void)pool;
    (void)block_table; (void)seq_lens; (void)out; (void)lse; (void)part_o; (void)part_ml; (void)stream;
    return CT_ERR_UNSUPPORTED;
}
