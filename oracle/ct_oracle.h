/*
 * ct_oracle.h -- CPU oracle for the KV-cache / decode-attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load this library, and only as the checker
 * (or the timed CPU baseline); the product library never links or calls it.
 *
 * This is a C11 restatement, in the reference's numerics, of the parts of the
 * path that have no code in the reference (paging, block tables, window/LRU
 * eviction, compaction, absorbed-MLA decode, per-token int8/fp8 codecs, LPT
 * sharding).  The parts that DO exist in the reference (ct_kv_*, ct_attn_*,
 * ct_quant_*) are taken from the reference objects themselves
 * (oracle/_ref/libctref.so, built by oracle/Makefile), and the tests pin each
 * restated function against them where they overlap:
 *   - orc_attn_forward / orc_mla_decode   follow src/attention/attention.c:11-53
 *   - orc_ct_f32_to_fp16 / fp16_to_f32    follow src/quant/quant.c:16-75
 *   - orc_q8_0_quantize / dequantize      follow src/quant/quant.c:77-111
 *   - orc_f32_to_bf16 / bf16_to_f32       follow src/transformer/ds4_forward.c:52-66
 *   - orc_kv_compress_every_kth           follows src/kv_cache/kv_cache.c:113-137
 *   - LRU tie rule                         follows src/streaming/streaming.c:86-96
 */
#ifndef CT_ORACLE_H
#define CT_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- seeded synthetic inputs: counter-based SplitMix64 + Box-Muller ----- */
uint64_t orc_mix64(uint64_t z);
uint64_t orc_key(uint64_t seed, uint64_t stream);
uint64_t orc_u64(uint64_t key, uint64_t i);
double   orc_unit(uint64_t key, uint64_t i);
float    orc_normal(uint64_t key, uint64_t i);
/* out[j] = normal(key, start + j), multiplied by outlier_mul where
 * orc_outlier(key, start + j, outlier_bp) says so (bp = basis points). */
int      orc_outlier(uint64_t key, uint64_t i, uint32_t outlier_bp);
void     orc_fill_normal_f32(uint64_t key, uint64_t start, uint64_t n, uint32_t outlier_bp,
                             float outlier_mul, float *out);
void     orc_fill_normal_bf16(uint64_t key, uint64_t start, uint64_t n, uint32_t outlier_bp,
                              float outlier_mul, uint16_t *out);
void     orc_permutation(uint64_t key, uint32_t n, int32_t *perm);
void     orc_lengths_loguniform(uint64_t key, uint32_t n, uint32_t lo, uint32_t hi, uint32_t *len);

/* ---- scalar conversions ------------------------------------------------ */
uint16_t orc_f32_to_bf16(float f);
float    orc_bf16_to_f32(uint16_t h);
uint16_t orc_ct_f32_to_fp16(float f);
float    orc_ct_fp16_to_f32(uint16_t h);
uint8_t  orc_f32_to_e4m3_satfinite(float f);
float    orc_e4m3_to_f32(uint8_t v);

/* ---- codecs --------------------------------------------------------------- */
/* Q8_0 block (34 B: u16 fp16 scale + 32 int8), n multiple of 32. */
void orc_q8_0_quantize(const float *src, uint8_t *dst_blocks, int64_t n);
void orc_q8_0_dequantize(const uint8_t *src_blocks, float *dst, int64_t n);
/* Per-token codecs: one fp32 scale per token over `dim` values. */
void orc_kv_quant_int8(const float *x, uint32_t n_tok, uint32_t dim, int8_t *codes, float *scales);
void orc_kv_dequant_int8(const int8_t *codes, const float *scales, uint32_t n_tok, uint32_t dim, float *x);
void orc_kv_quant_e4m3(const float *x, uint32_t n_tok, uint32_t dim, uint8_t *codes, float *scales);
void orc_kv_dequant_e4m3(const uint8_t *codes, const float *scales, uint32_t n_tok, uint32_t dim, float *x);

/* ---- attention ------------------------------------------------------------ */
void orc_attn_softmax(float *x, uint32_t n);
int  orc_attn_forward(const float *q, const float *k, const float *v, uint32_t n_tokens,
                      uint32_t n_heads, uint32_t head_dim, float scale, float *out);
/* Absorbed-MLA decode for one sequence: all H heads read the same [n][E]
 * entries; scores use all E dims, the output uses the first Dv dims. */
int  orc_mla_decode(const float *q, const float *kv, uint32_t n, uint32_t H, uint32_t E,
                    uint32_t Dv, float scale, float *out);
/* Gather n tokens of one sequence out of a bf16 page pool through its block
 * table row into fp32 [n][E].  Returns -1 if a needed page is unmapped. */
int  orc_paged_gather_bf16_f32(const uint16_t *pool, const int32_t *bt_row, uint32_t n,
                               uint32_t page_tokens, uint32_t E, float *out);
/* Batched paged MLA decode over n_seq sequences (OpenMP over sequences).
 * q [n_seq][H][E] bf16 bits, out [n_seq][H][Dv] fp32. */
int  orc_mla_decode_paged_bf16(const uint16_t *pool, const int32_t *bt, uint32_t max_pages,
                               const int32_t *seq_lens, uint32_t n_seq, const uint16_t *q,
                               uint32_t H, uint32_t E, uint32_t Dv, uint32_t page_tokens,
                               float scale, int n_threads, float *out);

/* ---- contiguous cache compaction (ct_kv_compress semantics) -------------- */
uint32_t orc_kv_compress_every_kth(float *k, float *v, uint32_t n_layers, uint32_t max_ctx,
                                   uint32_t stride, uint32_t n_tokens, float ratio);

/* ---- paged allocator with sliding-window + LRU eviction ------------------ */
typedef struct {
    uint32_t n_seqs, page_tokens, n_pages, max_pages_per_seq, window_tokens;
} orc_alloc_cfg_t;

typedef struct {
    uint32_t round, seq, lpage; int32_t phys; uint32_t reason; /* 1 = window, 2 = LRU */
} orc_evict_event_t;

/* Replays rounds r = 0..max(len)-1 appending token r of every sequence with
 * r < len[s] in seq-id order.  Outputs:
 *   bt           [n_seqs][max_pages_per_seq]  final block tables (-1 = none)
 *   slot_owner   [n_pages][page_tokens]        (seq << 32 | token) last written
 *                                              into each slot, or ~0 if never
 *   events       eviction log (capacity max_events), *n_events its length
 *   last_access  [n_seqs] round each sequence was last read
 * Returns 0, or -1 if a sequence needs more than max_pages_per_seq pages or
 * the log overflows. */
int orc_alloc_replay(const orc_alloc_cfg_t *cfg, const uint32_t *len, int32_t *bt,
                     uint64_t *slot_owner, orc_evict_event_t *events, uint32_t max_events,
                     uint32_t *n_events, uint32_t *last_access, uint32_t *n_free_out);

/* Defragmenting compaction: live pages get new ids 0..n_live-1 in (seq, lpage)
 * order.  Rewrites bt in place and fills map_new_to_old[n_live]. */
uint32_t orc_compact_plan(int32_t *bt, uint32_t n_seqs, uint32_t max_pages_per_seq,
                          int32_t *map_new_to_old);

/* ---- sequence sharding ---------------------------------------------------- */
/* Longest-processing-time assignment: lengths descending (ties: lower seq id
 * first), each to the rank with the least assigned tokens (ties: lower rank). */
void orc_lpt_assign(const uint32_t *len, uint32_t n, uint32_t n_ranks, int32_t *rank_of);

#ifdef __cplusplus
}
#endif
#endif
