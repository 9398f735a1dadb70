#ifndef CAUTREO_KV_CACHE_H
#define CAUTREO_KV_CACHE_H

/*
 * kv_cache.h -- KV cache, backed by B200 device memory.
 *
 * Part 1 keeps the reference interface of src/kv_cache/kv_cache.h:22-66
 * byte-for-byte (same struct layouts, same signatures, same return
 * conventions), so src/transformer/transformer.c and src/engine link against
 * this library unchanged.  The K/V arrays live in HBM; every call copies
 * between the caller's host buffers and the device.
 *
 * Part 2 adds the paged cache the reference does not have: a pool of
 * fixed-size pages, per-sequence block tables, a sliding window, LRU
 * eviction, per-token int8 / fp8-e4m3 codecs applied on append, and
 * defragmenting compaction.  Device pointers, status codes (0 = success,
 * negative = error, see ct_status_t in hal.h), one handle per host thread.
 */

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ======================================================================== */
/* Part 1 -- reference interface (src/kv_cache/kv_cache.h:22-66)            */
/* ======================================================================== */

/* Replaces src/kv_cache/kv_cache.h:22-28; 20 bytes, same field order. */
typedef struct {
    uint32_t n_layers;
    uint32_t n_kv_heads;
    uint32_t head_dim;
    uint32_t max_ctx;         /* token capacity; 0 selects 2048 */
    float    compress_ratio;  /* 1.0 = none; 0 selects 1.0 */
} ct_kv_config_t;

typedef struct ct_kv_cache ct_kv_cache_t;

/* kv_cache.h:33 -- allocates zeroed [n_layers][max_ctx][n_kv_heads*head_dim]
 * fp32 K and V in device memory; NULL on failure. */
ct_kv_cache_t *ct_kv_create(const ct_kv_config_t *cfg);
/* kv_cache.h:34 */
void           ct_kv_destroy(ct_kv_cache_t *c);

/* kv_cache.h:37 -- copies one token's K and V row (n_kv_heads*head_dim fp32
 * each, host pointers) into (layer, token_pos).  false on NULL, layer out of
 * range or token_pos >= max_ctx.  len becomes max(len, token_pos + 1). */
bool ct_kv_append(ct_kv_cache_t *c, uint32_t layer, uint32_t token_pos,
                  const float *k, const float *v);

/* kv_cache.h:41 -- copies the row back to host buffers; false if
 * token_pos >= len.  Does not count as a read in the stats (as in the
 * reference). */
bool ct_kv_get(const ct_kv_cache_t *c, uint32_t layer, uint32_t token_pos,
               float *k_out, float *v_out);

/* kv_cache.h:45-46 */
uint32_t ct_kv_len(const ct_kv_cache_t *c);
uint32_t ct_kv_capacity(const ct_kv_cache_t *c);

/* kv_cache.h:49 -- zeroes the counters, keeps the data. */
void ct_kv_reset(ct_kv_cache_t *c);

/* kv_cache.h:52-53 -- the reference's raw file format: the 20-byte config,
 * u32 len, u32 n_compressed, then all of K and all of V (full capacity). */
bool ct_kv_save(const ct_kv_cache_t *c, const char *path);
bool ct_kv_load(ct_kv_cache_t *c, const char *path);

/* kv_cache.h:56 -- keeps tokens 0, step, 2*step, ... (step = max(2, (int)
 * ratio)) packed to the front of every layer, on the device. */
bool ct_kv_compress(ct_kv_cache_t *c, float ratio);

/* kv_cache.h:59-66 */
typedef struct {
    uint64_t n_appends;
    uint64_t n_reads;
    uint64_t bytes_used;
    uint32_t n_tokens;
} ct_kv_stats_t;

ct_kv_stats_t ct_kv_stats(const ct_kv_cache_t *c);

/* Device addresses of the K / V arrays (for kernels that read the cache in
 * place, e.g. ct_attn_decode_contig in attention.h).  New; no reference
 * counterpart. */
float *ct_kv_device_k(ct_kv_cache_t *c);
float *ct_kv_device_v(ct_kv_cache_t *c);

/* ======================================================================== */
/* Part 2 -- paged cache (new; no reference counterpart)                    */
/* ======================================================================== */

/* Storage type of the page pool. */
typedef enum {
    CT_KV_BF16 = 0,   /* 2 B per value */
    CT_KV_F32  = 1,   /* 4 B per value */
    CT_KV_INT8 = 2,   /* int8 codes + one fp32 scale per token (amax/127) */
    CT_KV_E4M3 = 3,   /* fp8 e4m3 codes + one fp32 scale per token (amax/448) */
    /* Cold-tier block codecs of quant.h (src/quant/quant.c:77-249): a token's
     * entry is entry_dim/32 blocks, byte for byte what ct_quant_q8_0 / _q4_0 /
     * _q2_0 / _q1_0 write for the token's values (a fp16 scale per 32 values
     * inside each block, no separate scales array).  entry_dim must be a
     * multiple of 32 (at most 4096) and page_tokens x entry bytes a multiple
     * of 16.  Append quantises, gather dequantises to bf16 or fp32 exactly as
     * ct_quant_deq*_0 (then rounds to bf16); compaction, fork and checkpoints
     * move the bytes.  The decode kernels do not read these pools (gather
     * them to bf16 first): ct_attn_mla_decode_paged over one returns
     * CT_ERR_UNSUPPORTED. */
    CT_KV_Q8_0 = 4,   /* 34 B per 32 values */
    CT_KV_Q4_0 = 5,   /* 18 B per 32 values */
    CT_KV_Q2_0 = 6,   /* 10 B per 32 values */
    CT_KV_Q1_0 = 7,   /*  6 B per 32 values */
} ct_kv_dtype_t;

typedef struct {
    uint32_t n_seqs;             /* block-table rows */
    uint32_t max_pages_per_seq;  /* block-table columns */
    uint32_t n_pages;            /* physical pages in the pool */
    uint32_t page_tokens;        /* tokens per page; 0 selects 64 */
    uint32_t entry_dim;          /* values per token; 0 selects 576 (512 latent + 64 rope) */
    uint32_t window_tokens;      /* sliding window; 0 keeps every token */
    uint32_t dtype;              /* ct_kv_dtype_t */
    int32_t  device;             /* CUDA ordinal */
} ct_kv_paged_config_t;

typedef struct ct_kv_paged ct_kv_paged_t;

typedef struct {
    uint64_t n_appends;          /* tokens appended */
    uint64_t n_evict_window;     /* pages freed by the sliding window */
    uint64_t n_evict_lru;        /* pages taken by LRU eviction */
    uint64_t n_compactions;
    uint64_t bytes_compacted;    /* page bytes moved by compaction */
    uint32_t n_pages_live;
    uint32_t n_pages_free;
    uint64_t clock;              /* allocator rounds so far */
} ct_kv_paged_stats_t;

typedef struct {
    uint32_t round, seq, lpage;
    int32_t  phys;
    uint32_t reason;             /* 1 = sliding window, 2 = LRU */
} ct_kv_evict_event_t;

ct_kv_paged_t *ct_kv_paged_create(const ct_kv_paged_config_t *cfg);
void           ct_kv_paged_destroy(ct_kv_paged_t *h);
/* Stream (cudaStream_t) used by every later call on h; NULL = legacy. */
int  ct_kv_paged_set_stream(ct_kv_paged_t *h, void *stream);

/* Order in which free pages are handed out: order[i] = physical id with
 * rank i (a permutation of 0..n_pages-1).  Default: ascending ids. */
int  ct_kv_paged_set_free_order(ct_kv_paged_t *h, const int32_t *order_host);

/* Appends counts[i] tokens to sequence seq_ids[i] (host arrays).  Tokens are
 * taken in rounds: round k appends token k of every i with k < counts[i], in
 * array order; each round advances the allocator clock.  Per token:
 *   1. opening a page when the pool is empty first evicts the least recently
 *      used full page, minimising (last_access, seq, lpage);
 *   2. the lowest-ranked free page is taken;
 *   3. the token is written (quantised on the way if the pool is int8/e4m3);
 *   4. last_access[seq] = clock;
 *   5. pages wholly outside the sliding window are freed.
 * entries: device [sum(counts)][entry_dim] in src_dtype (CT_KV_BF16 or
 * CT_KV_F32), ordered sequence by sequence (all tokens of seq_ids[0] first);
 * NULL reserves the slots and writes nothing. */
int  ct_kv_paged_append(ct_kv_paged_t *h, const uint32_t *seq_ids, const uint32_t *counts,
                        uint32_t n, const void *entries, uint32_t src_dtype);

/* Releases every page of a sequence and sets its length to 0. */
/* The same allocation as ct_kv_paged_append, with each new token's entry
 * produced on the device from its hidden state by ct_kv_project_write_slots
 * (x: device bf16 [sum(counts)][n_in], ordered like `entries`; W: device
 * bf16 [entry_dim][n_in]; norm_w NULL skips the norm).  No counterpart in
 * the reference. */
int  ct_kv_paged_append_projected(ct_kv_paged_t *h, const uint32_t *seq_ids, const uint32_t *counts,
                                  uint32_t n, const void *x, const void *w, uint32_t n_in,
                                  const float *norm_w, float eps, uint32_t norm_dim);
int  ct_kv_paged_free_seq(ct_kv_paged_t *h, uint32_t seq);
/* Frees up to n pages by LRU order; returns the number freed (>= 0). */
int  ct_kv_paged_evict_lru(ct_kv_paged_t *h, uint32_t n);
/* Renumbers live pages to 0..n_live-1 in (seq, lpage) order and moves their
 * bytes to match (device gather into a fresh pool). */
int  ct_kv_paged_compact(ct_kv_paged_t *h);

/* Copies n tokens [start, start+n) of a sequence to out (device) as
 * contiguous [n][entry_dim] values of out_dtype (CT_KV_BF16 or CT_KV_F32),
 * dequantising int8/e4m3 pages.  Fails if a page in the range is unmapped. */
int  ct_kv_paged_gather(ct_kv_paged_t *h, uint32_t seq, uint32_t start, uint32_t n,
                        void *out, uint32_t out_dtype);

/* Prefix sharing (new; the reference's ct_engine_kv_reuse is a no-op,
 * engine.c:653-657): sequence dst (empty) takes the first n_tokens of src.
 * Full pages are shared -- both block tables map them and a page returns to
 * the free set only when no sequence maps it -- and a partial last page is
 * copied into a page of dst's own, so appends never write a shared page.
 * Shared pages are not LRU victims; a sequence's window releases its
 * references; compaction keeps them shared.  CT_ERR_UNMAPPED if the window
 * already dropped part of src's prefix. */
int      ct_kv_paged_fork(ct_kv_paged_t *h, uint32_t src, uint32_t dst, uint32_t n_tokens);
/* Number of sequences mapping a physical page (0 = free). */
uint32_t ct_kv_paged_page_refs(const ct_kv_paged_t *h, int32_t page);

/* Token ids of cached positions, for KV reuse across turns (the reference's
 * engine persists only the ids, engine.c:634-651, and its ct_engine_kv_reuse
 * is a no-op, engine.c:653-657).  set_tokens records ids for positions
 * [start, start+n) of seq (start <= the ids recorded so far, start+n <= the
 * sequence's length); a fork copies the prefix's ids, free_seq drops them,
 * checkpoints carry them.  match_prefix finds the sequence whose recorded ids
 * share the longest prefix with ids[0:n] among sequences still mapped from
 * position 0 (ties: the lowest seq); *len_out = 0 when none matches.  Fork
 * that many tokens to reuse them. */
int      ct_kv_paged_set_tokens(ct_kv_paged_t *h, uint32_t seq, uint32_t start, const int32_t *ids, uint32_t n);
uint32_t ct_kv_paged_tokens(const ct_kv_paged_t *h, uint32_t seq, int32_t *ids_out, uint32_t max);
int      ct_kv_paged_match_prefix(const ct_kv_paged_t *h, const int32_t *ids, uint32_t n, uint32_t *seq_out,
                                  uint32_t *len_out);

/* Checkpoint of a paged cache (new; no reference counterpart -- it extends
 * the raw format of kv_cache.c:82-111, which ct_kv_save / ct_kv_load keep
 * unchanged): a versioned header ("CTKVPAGE", version 1), the configuration,
 * statistics, lengths, page ranges, LRU clocks, block table, free order, free
 * set and eviction log, then the bytes (and scales) of every live page, and a
 * checksum.  Loading restores the same state: later appends, evictions and
 * reads behave exactly as on the saved handle.  A handle with device < 0
 * saves tables only, which load with device -1. */
int            ct_kv_paged_save(ct_kv_paged_t *h, const char *path);
ct_kv_paged_t *ct_kv_paged_load(const char *path, int device);   /* NULL on failure */

/* The same for n ranges at once (host arrays): tokens [starts[i],
 * starts[i] + counts[i]) of sequence seqs[i], written back to back in range
 * order into out (device).  One launch per 65,535 ranges.  New; no reference
 * counterpart (the reference reads one row at a time, kv_cache.c:63-71). */
int  ct_kv_paged_gather_batch(ct_kv_paged_t *h, const uint32_t *seqs, const uint32_t *starts,
                              const uint32_t *counts, uint32_t n, void *out, uint32_t out_dtype);

/* Host mirrors / device views. */
int  ct_kv_paged_block_table(const ct_kv_paged_t *h, int32_t *out_host);  /* [n_seqs][max_pages] */
int  ct_kv_paged_seq_lens(const ct_kv_paged_t *h, uint32_t *out_host);    /* [n_seqs] */
int  ct_kv_paged_last_access(const ct_kv_paged_t *h, uint64_t *out_host); /* [n_seqs] */
uint32_t ct_kv_paged_evict_log(const ct_kv_paged_t *h, ct_kv_evict_event_t *out_host, uint32_t max);
ct_kv_paged_stats_t ct_kv_paged_stats(const ct_kv_paged_t *h);
const ct_kv_paged_config_t *ct_kv_paged_config(const ct_kv_paged_t *h);
void          *ct_kv_paged_pool(ct_kv_paged_t *h);          /* [n_pages][page_tokens][entry_dim] */
float         *ct_kv_paged_scales(ct_kv_paged_t *h);        /* [n_pages][page_tokens], NULL for bf16/f32 */
const int32_t *ct_kv_paged_block_table_dev(const ct_kv_paged_t *h);
const int32_t *ct_kv_paged_seq_lens_dev(const ct_kv_paged_t *h);

/* ---- stateless device kernels under the paged API ----------------------- */

/* Writes n token entries (device [n][dim], src_dtype BF16 or F32) to
 * dest_slot[i] = phys_page*page_tokens + slot (device int32; < 0 skips),
 * converting / quantising into the pool's dtype. */
int ct_kv_paged_write_slots(void *pool, float *scales, uint32_t pool_dtype, const void *entries,
                            uint32_t src_dtype, const int32_t *dest_slot, uint32_t n,
                            uint32_t dim, void *stream);

/* Fused producer (no counterpart in the reference, which projects one token
 * at a time with matvec_bf16 and copies the fp32 result into the cache,
 * ds4_forward.c:248-272 and 1548-1570): for n new tokens,
 *   entry[t] = W . x[t]          x: device bf16 [n][n_in], W: device bf16
 *                                [dim][n_in]; fp32 accumulation on the tensor
 *                                cores (the reference's fp32 hidden state is
 *                                rounded to bf16 first);
 *   optional RMS norm of entry[t][0:norm_dim] as rmsnorm_ip
 *   (ds4_forward.c:206-211): x * (1/sqrt(mean(x^2) + eps)) * norm_w;
 *   then written / quantised into dest_slot as ct_kv_paged_write_slots.
 * n_in % 64 == 0, dim % 64 == 0, norm_dim % 4 == 0 (norm_w NULL skips the
 * norm); x and W 16-byte aligned.  Uses stream-ordered scratch of
 * (ksplit + 1) x n x dim fp32 (ksplit <= 16).  sm_100 only. */
int ct_kv_project_write_slots(const void *x, const void *w, const float *norm_w, float eps,
                              uint32_t norm_dim, uint32_t n, uint32_t n_in, uint32_t dim, void *pool,
                              float *scales, uint32_t pool_dtype, const int32_t *dest_slot,
                              void *stream);
/* Error word of the projection kernel (0 = every bounded wait completed);
 * clear != 0 resets it.  Synchronises with the device. */
int ct_kv_project_error(int clear);

/* Page-level gather: dst page i <- src page map[i] (device int32), whole
 * pages of page_bytes (codes) and page_tokens scales (if scales != NULL). */
int ct_kv_paged_move_pages(const void *src_pool, const float *src_scales, void *dst_pool,
                           float *dst_scales, const int32_t *map, uint32_t n_pages,
                           size_t page_bytes, uint32_t page_tokens, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* CAUTREO_KV_CACHE_H */
