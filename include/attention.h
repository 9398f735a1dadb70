#ifndef CAUTREO_ATTENTION_H
#define CAUTREO_ATTENTION_H

/*
 * attention.h -- decode attention on B200.
 *
 * Part 1 keeps the reference interface of src/attention/attention.h:22-32
 * unchanged (host pointers, bool / void returns).  Each call copies its
 * inputs to the device, runs a CUDA kernel and copies the result back.
 *
 * Part 2 adds device-pointer entry points: plain decode over a contiguous
 * cache (the loop of src/transformer/transformer.c:185-214) and paged
 * absorbed-MLA decode (the latent cache of src/transformer/ds4_forward.c:
 * 1567-1636 extended with a 64-d RoPE key, paging and split-KV).
 */

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ======================================================================== */
/* Part 1 -- reference interface (src/attention/attention.h:22-32)          */
/* ======================================================================== */

/* attention.h:22 -- single-query scaled dot-product attention.  q and out are
 * [n_kv_heads][head_dim]; k and v are ONE [n_tokens][head_dim] block that
 * every head reads (attention.c:37,47).  scale 0 selects 1/sqrt(head_dim).
 * false on NULL pointers, n_tokens == 0 or a CUDA failure. */
bool ct_attn_forward(const float *q, const float *k, const float *v,
                     uint32_t n_tokens, uint32_t n_kv_heads, uint32_t head_dim,
                     float scale, float *out);

/* attention.h:26 -- same as ct_attn_forward. */
bool ct_attn_forward_kv(const float *q, const float *kv_k, const float *kv_v,
                        uint32_t n_tokens, uint32_t n_kv_heads, uint32_t head_dim,
                        float scale, float *out);

/* attention.h:31 -- in-place softmax of n floats (fp32 max, exp, double sum). */
void ct_attn_softmax(float *x, uint32_t n);

/* ======================================================================== */
/* Part 2 -- device entry points (new; no reference counterpart)            */
/* ======================================================================== */

/* Plain decode over a contiguous fp32 cache laid out as ct_kv_cache_t
 * ([n_layers][max_ctx][n_kv_heads*head_dim]), for n_layers layers at once.
 * q, out: device [n_layers][n_q_heads][head_dim]; query head h reads KV head
 * h % n_kv_heads (transformer.c:187); scores = q.k * scale, scale 0 selects
 * 1/sqrt(head_dim).  Attends tokens [0, n_tokens). */
int ct_attn_decode_contig(const float *q, const float *k_cache, const float *v_cache,
                          uint32_t n_layers, uint32_t max_ctx, uint32_t n_kv_heads,
                          uint32_t n_q_heads, uint32_t head_dim, uint32_t n_tokens,
                          float scale, float *out, void *stream);

/* One decode step of the same cache: writes k_new / v_new (device
 * [n_layers][n_kv_heads*head_dim]) at token pos, then attends [0, pos].
 * One launch for all layers and heads. */
int ct_attn_decode_step_contig(const float *q, const float *k_new, const float *v_new,
                               float *k_cache, float *v_cache, uint32_t n_layers,
                               uint32_t max_ctx, uint32_t n_kv_heads, uint32_t n_q_heads,
                               uint32_t head_dim, uint32_t pos, float scale, float *out,
                               void *stream);

/* ---- paged absorbed-MLA decode ------------------------------------------ */

/* Shape of one MLA decode problem. */
typedef struct {
    uint32_t n_heads;        /* query heads sharing one latent entry (128) */
    uint32_t entry_dim;      /* latent + rope values per token (576) */
    uint32_t v_dim;          /* leading values of an entry used as V (512) */
    uint32_t page_tokens;    /* 64 */
    uint32_t max_pages_per_seq;
    uint32_t kv_dtype;       /* ct_kv_dtype_t of the pool */
    float    scale;          /* softmax scale, e.g. 1/sqrt(192) */
    uint32_t n_pages;        /* pages in the pool; block-table entries >= n_pages are skipped */
} ct_mla_shape_t;

/* A work plan: device buffers for the split of every sequence's pages into
 * chunks across the SMs, and the scratch for partial results of sequences
 * that are split.  Each ct_attn_mla_decode_paged first recomputes the split
 * on the device from the CURRENT device lengths (pages laid end to end, the
 * same number of pages per worker), so one plan serves any lengths up to
 * max_pages_per_seq pages: a serving loop whose sequences grow reuses it,
 * without host planning or allocation, and a whole step can be replayed as
 * one CUDA graph. */
typedef struct ct_mla_plan ct_mla_plan_t;

/* seq_rows (host, may be NULL = 0..n_seq-1): block-table row of each output
 * sequence.  seq_lens_host: the sequences' lengths now (checked against
 * max_pages_per_seq; ct_mla_plan_chunks reports their split). */
ct_mla_plan_t *ct_mla_plan_create(const ct_mla_shape_t *shape, const uint32_t *seq_rows,
                                  const int32_t *seq_lens_host, uint32_t n_seq, int device);
void   ct_mla_plan_destroy(ct_mla_plan_t *p);
/* Number of work chunks the creation lengths split into, and the split-KV
 * scratch bytes the plan holds (sized for any lengths). */
uint32_t ct_mla_plan_chunks(const ct_mla_plan_t *p);
/* Workers the plan balances over, and whether it runs the tensor-core kernel
 * (1: 128 heads x 576 bf16 entries x 64-token pages on sm_100; 0: the
 * CUDA-core kernel for every other shape). */
uint32_t ct_mla_plan_workers(const ct_mla_plan_t *p);
int      ct_mla_plan_tensor_cores(const ct_mla_plan_t *p);
size_t   ct_mla_plan_scratch_bytes(const ct_mla_plan_t *p);

/* out[s][h][0:v_dim] = sum_t softmax_t(scale * q[s][h] . e_t) * e_t[0:v_dim]
 * over the entries e_t of sequence s in mapped pages (t < seq_lens[row]).
 * q: device [n_seq][n_heads][entry_dim] bf16.  pool / scales / block_table /
 * seq_lens: device, as held by ct_kv_paged_t.  out: device
 * [n_seq][n_heads][v_dim] bf16.  lse (optional, device [n_seq][n_heads] fp32)
 * receives the natural-log softmax normaliser.  Sequences of length 0 give 0. */
int ct_attn_mla_decode_paged(const ct_mla_plan_t *plan, const void *q, const void *pool,
                             const float *scales, const int32_t *block_table,
                             const int32_t *seq_lens, void *out, float *lse, void *stream);

/* Number of kernel launches the last ct_attn_mla_decode_paged issued
 * (planning, decode, and the combine when a sequence was split). */
uint32_t ct_mla_plan_launches(const ct_mla_plan_t *p);

/* Error word of the tensor-core MLA kernel on the current device: 0 when no
 * bounded wait expired, else the code of the first wait that did (the kernel
 * then returned early and its outputs are invalid).  clear != 0 resets it.
 * Reading it synchronises with the device.  -1 if it cannot be read. */
int ct_mla_tc_error(int clear);

/* One serving step with host I/O, for callers that keep inputs and outputs
 * in host memory: copies q_host ([n_seq][n_heads][entry_dim] bf16) and
 * entries_host ([n_seq][entry_dim] bf16, the token appended to each sequence)
 * to the device, writes the new tokens to dest_slot (device int32, as
 * ct_kv_paged_write_slots; NULL skips the append), decodes, and copies
 * out_host ([n_seq][n_heads][v_dim] bf16) back.  Returns when out_host is
 * filled.  The plan keeps the device staging buffers between calls; pinned
 * host buffers give the fastest copies.  Large steps are cut into sequence
 * groups whose copies overlap the decode of other groups, on streams the
 * plan owns (ordered after the work already queued on `stream`); all of
 * them have finished when the call returns.  Calls on one plan must not
 * overlap. */
int ct_attn_mla_decode_step_host(ct_mla_plan_t *plan, const void *q_host, const void *entries_host,
                                 const int32_t *dest_slot, void *pool, float *scales,
                                 const int32_t *block_table, const int32_t *seq_lens, void *out_host,
                                 void *stream);

/* ---- the same decode without any allocation ---------------------------- */

/* No counterpart in the reference.  For callers that cannot allocate device
 * memory on their decode path -- an engine that reserved nearly all of HBM
 * for its KV pool at start-up, where a later cudaMalloc would fail, or a
 * latency-bound serving loop that bans allocator calls (and the
 * synchronisation they bring) once running.  Computes what
 * ct_mla_plan_create + ct_attn_mla_decode_paged compute, but plans on the host
 * into static arrays and keeps its work list and split-KV partials in one
 * fixed device array of CT_MLA_NOALLOC_SCRATCH_BYTES inside the library, which
 * every GPU that loads the library holds until the process exits.  It calls
 * no cudaMalloc / cudaFree and no allocating library routine.
 *
 * Sequence s reads block-table row s.  seq_lens_host and seq_lens (device)
 * hold the same lengths.  Limits: n_seq <= CT_MLA_NOALLOC_MAX_SEQS, and the
 * split-KV partials (at most 2 x 59 sequences' worth of n_heads x v_dim fp32)
 * must fit the array; beyond either limit the call returns CT_ERR_ARG and
 * ct_hal_cuda_last_error() says which.  The first call on each device looks
 * up the array's device address with that device current, so make it before
 * any stream capture.  All calls share the array and leave their contents in
 * it; calls that overlap on the GPU race, so serialise them.  To bound the
 * split partials it spreads a batch over at most 60 workers (2-SM clusters),
 * i.e. 120 of the B200's 148 SMs, so a large batch decodes at up to
 * ~19 % lower throughput than through a plan, which uses every SM. */
#define CT_MLA_NOALLOC_SCRATCH_BYTES (32u << 20)
#define CT_MLA_NOALLOC_MAX_SEQS 4096u
int ct_attn_mla_decode_paged_noalloc(const ct_mla_shape_t *shape, const int32_t *seq_lens_host,
                                     uint32_t n_seq, const void *q, const void *pool,
                                     const float *scales, const int32_t *block_table,
                                     const int32_t *seq_lens, void *out, float *lse, void *stream);

/* ======================================================================== */
/* Part 3 -- the MLA-lite cache of ds4_forward.c on the device               */
/* ======================================================================== */

/* Replaces the per-layer latent cache and attention of ds4_forward.c
 * (store at :1565-1570, attention at :1572-1627; the reference's cache is a
 * calloc'ed fp32 [n_layers][ctx][kv_dim] array) for an engine that keeps its
 * hidden state on the host.  One handle holds every layer's cache (fp32
 * pages on the device).  Not thread-safe, like the reference engine. */
typedef struct ct_ds4_cache ct_ds4_cache_t;
ct_ds4_cache_t *ct_ds4_cache_create(uint32_t n_layers, uint32_t ctx, uint32_t kv_dim, int device);
void            ct_ds4_cache_destroy(ct_ds4_cache_t *c);
/* Positions stored for `layer`. */
uint32_t        ct_ds4_cache_len(const ct_ds4_cache_t *c, uint32_t layer);
/* One layer, one token: when pos < ctx stores kv_a (host, kv_dim fp32) at
 * pos (pos <= the stored length: positions arrive in order, or overwrite);
 * then out (host, kv_dim fp32) = sum_p softmax_p(q . k_p / sqrt(kv_dim)) k_p
 * over the first min(pos + 1, ctx) positions, q = the first kv_dim values of
 * q_b (host fp32).  q is rounded to bf16 and out comes from bf16 (the
 * attention tolerance of the MLA decode). */
int ct_ds4_attend(ct_ds4_cache_t *c, uint32_t layer, uint32_t pos, const float *kv_a, const float *q,
                  float *out);

#ifdef __cplusplus
}
#endif

#endif /* CAUTREO_ATTENTION_H */
