#ifndef CT_SYNTH_H
#define CT_SYNTH_H

/*
 * synth.h -- seeded synthetic KV-cache contents generated on the device
 * (new; no reference counterpart).  Used to fill large caches without a host
 * round trip.
 *
 * Generator: element i of stream `key` is SplitMix64 output i
 * (mix64(key + (i+1) * 0x9E3779B97F4A7C15)); a normal value uses draws 2i
 * and 2i+1 through Box-Muller (cosine branch, double precision, rounded to
 * fp32); an element is an outlier (multiplied by outlier_mul) when draw i of
 * the derived stream mix64(key ^ 0xA0761D6478BD642F) is below outlier_bp
 * modulo 10000.  Keys: ct_synth_key(seed, stream).
 */

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

uint64_t ct_synth_key(uint64_t seed, uint64_t stream);

/* out[j] = value(start + j) for j < n, as bf16 (dtype 0) or fp32 (dtype 1). */
int ct_synth_fill(void *out, uint32_t dtype, uint64_t key, uint64_t start, uint64_t n,
                  uint32_t outlier_bp, float outlier_mul, void *stream);

/* Fills every token t < seq_lens[i] of sequence rows[i] (i < n_seq) in a paged
 * pool through its block table: entry value e of (row, t) is
 * value(((uint64)row << 24 | t) * entry_dim + e).  Quantised pools (int8 /
 * e4m3) get per-token codes and scales as on append. */
int ct_synth_fill_paged(void *pool, float *scales, uint32_t pool_dtype, const int32_t *block_table,
                        uint32_t max_pages_per_seq, const uint32_t *rows_dev, const int32_t *seq_lens_dev,
                        uint32_t n_seq, uint32_t max_len, uint32_t page_tokens, uint32_t entry_dim,
                        uint64_t key, uint32_t outlier_bp, float outlier_mul, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* CT_SYNTH_H */
