/*
 * kv_paged.c -- paged KV cache handle (kv_cache.h Part 2).
 *
 * Host side: block tables, free list, sliding window and LRU eviction, the
 * eviction log.  Device side (kv_kernels.cu): token writes with
 * quantise-on-append, gathers with dequantise-on-gather, page moves for
 * compaction.  The reference has no paged cache; its precedents are
 * ct_kv_compress for moving tokens down (src/kv_cache/kv_cache.c:113-137)
 * and the streamer's LRU, which picks the minimum last-access time with the
 * lowest index winning ties (src/streaming/streaming.c:86-96).
 *
 * Event order for each appended token (rounds across the sequences of one
 * call, see ct_kv_paged_append):
 *   1. a token at position r with r % P == 0 opens logical page r / P; if no
 *      page is free, the least recently used FULL page is evicted first,
 *      minimising (last_access[seq], seq, lpage);
 *   2. the free page of lowest rank is taken (rank = position in the free
 *      order, ascending ids by default);
 *   3. the token goes to slot r % P;
 *   4. last_access[seq] = the allocator clock of this round;
 *   5. pages lying wholly below len - window are freed.
 * A sequence's mapped pages form one run [lo, hi) of logical pages: new
 * pages open at hi; the window and LRU free from lo.
 *
 * Device mirrors (block table, lengths) are updated by scattering only the
 * changed entries, staged with the token slots in one pinned buffer.
 */
#include "../../include/hal.h"
#include "../../include/kv_cache.h"
#include "../csrc/ct_internal.h"

#include <cuda_runtime_api.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* Device helper in kv_kernels.cu: dst[idx[i]] = val[i]. */
int ct__launch_scatter_i32(int32_t *dst, const int32_t *pairs, uint32_t n_pairs, void *stream);

struct ct_kv_paged {
    ct_kv_paged_config_t cfg;
    int host_only;              /* device < 0: tables only, no device memory */
    cudaStream_t stream;
    size_t entry_bytes;         /* bytes of one token's entry in the pool */
    size_t page_bytes;          /* page_tokens * entry_dim * elt */
    /* device */
    void *pool;
    float *scales;
    int pool_async;             /* pool / scales came from cudaMallocAsync (a compaction) */
    int32_t *bt_dev;
    int32_t *len_dev;
    int32_t *stage_dev;         /* staged dest slots + (index, value) pairs */
    size_t stage_cap;           /* int32 elements */
    /* pinned staging and the event guarding its reuse */
    int32_t *stage_host;
    cudaEvent_t stage_ev;
    int stage_pending;
    /* host state */
    int32_t *bt;                /* [n_seqs][max_pages] */
    uint32_t *len, *lo, *hi;
    uint64_t *last_access;
    uint32_t *rank;             /* free-order rank of each physical page */
    uint32_t *refc;             /* sequences mapping each physical page (prefix sharing) */
    int32_t *heap;              /* free pages, min-heap by rank */
    uint32_t heap_n;
    ct_kv_evict_event_t *log;
    uint32_t log_n, log_cap;
    uint8_t *claimed;           /* per-call slot bitmap for last-writer-wins */
    ct_kv_paged_stats_t st;
    /* token ids of each sequence's cached positions [0, tok_n), for prefix
     * reuse (allocated per sequence on first use) */
    int32_t **tok;
    uint32_t *tok_n, *tok_cap;
    /* pending device updates of this call */
    int32_t *pairs;             /* (index, value) for bt_dev then len_dev */
    uint32_t n_bt_pairs, n_len_pairs, pairs_cap;
};

/* ---- free list ----------------------------------------------------------- */

static int heap_less(const ct_kv_paged_t *h, int32_t a, int32_t b) { return h->rank[a] < h->rank[b]; }

static void heap_push(ct_kv_paged_t *h, int32_t p) {
    uint32_t i = h->heap_n++;
    h->heap[i] = p;
    while (i > 0) {
        uint32_t up = (i - 1) / 2;
        if (!heap_less(h, h->heap[i], h->heap[up])) break;
        int32_t t = h->heap[up]; h->heap[up] = h->heap[i]; h->heap[i] = t; i = up;
    }
}

static int32_t heap_pop(ct_kv_paged_t *h) {
    int32_t top = h->heap[0];
    h->heap[0] = h->heap[--h->heap_n];
    uint32_t i = 0;
    for (;;) {
        uint32_t l = 2 * i + 1, r = l + 1, m = i;
        if (l < h->heap_n && heap_less(h, h->heap[l], h->heap[m])) m = l;
        if (r < h->heap_n && heap_less(h, h->heap[r], h->heap[m])) m = r;
        if (m == i) break;
        int32_t t = h->heap[m]; h->heap[m] = h->heap[i]; h->heap[i] = t; i = m;
    }
    return top;
}

static void heap_rebuild(ct_kv_paged_t *h, int32_t *pages, uint32_t n) {
    h->heap_n = 0;
    for (uint32_t i = 0; i < n; i++) heap_push(h, pages[i]);
}

/* ---- pending device updates ---------------------------------------------- */

static int pairs_reserve(ct_kv_paged_t *h, uint32_t extra) {
    uint32_t need = 2 * (h->n_bt_pairs + h->n_len_pairs + extra);
    if (need <= h->pairs_cap) return CT_OK;
    uint32_t cap = h->pairs_cap ? h->pairs_cap : 1024;
    while (cap < need) cap *= 2;
    int32_t *p = (int32_t *)realloc(h->pairs, (size_t)cap * sizeof(int32_t));
    if (!p) return CT_ERR_NOMEM;
    h->pairs = p;
    h->pairs_cap = cap;
    return CT_OK;
}

/* bt pairs are stored from the front, len pairs are appended after the call
 * by flush (lengths are final only then). */
static int set_bt(ct_kv_paged_t *h, uint32_t s, uint32_t lp, int32_t v) {
    size_t idx = (size_t)s * h->cfg.max_pages_per_seq + lp;
    h->bt[idx] = v;
    if (pairs_reserve(h, 1)) return CT_ERR_NOMEM;
    h->pairs[2 * h->n_bt_pairs] = (int32_t)idx;
    h->pairs[2 * h->n_bt_pairs + 1] = v;
    h->n_bt_pairs++;
    return CT_OK;
}

static int log_event(ct_kv_paged_t *h, uint32_t s, uint32_t lp, int32_t ph, uint32_t reason) {
    if (h->log_n == h->log_cap) {
        uint32_t cap = h->log_cap ? 2 * h->log_cap : 1024;
        ct_kv_evict_event_t *p = (ct_kv_evict_event_t *)realloc(h->log, (size_t)cap * sizeof *p);
        if (!p) return CT_ERR_NOMEM;
        h->log = p;
        h->log_cap = cap;
    }
    ct_kv_evict_event_t ev = { (uint32_t)h->st.clock, s, lp, ph, reason };
    h->log[h->log_n++] = ev;
    if (reason == 1) h->st.n_evict_window++; else h->st.n_evict_lru++;
    return CT_OK;
}

/* Unmaps logical page lo[s] of sequence s; the physical page returns to the
 * free set when no other sequence maps it. */
static int free_low_page(ct_kv_paged_t *h, uint32_t s, uint32_t reason) {
    uint32_t lp = h->lo[s];
    int32_t ph = h->bt[(size_t)s * h->cfg.max_pages_per_seq + lp];
    if (reason && log_event(h, s, lp, ph, reason)) return CT_ERR_NOMEM;
    if (set_bt(h, s, lp, -1)) return CT_ERR_NOMEM;
    h->lo[s]++;
    if (--h->refc[ph] == 0) {
        heap_push(h, ph);
        h->st.n_pages_live--;
    }
    return CT_OK;
}

/* LRU victim: sequence with a full lowest page that no other sequence maps
 * (evicting it frees memory), minimising (last_access, seq). */
static int64_t lru_victim(const ct_kv_paged_t *h) {
    int64_t best = -1;
    const uint32_t P = h->cfg.page_tokens, MP = h->cfg.max_pages_per_seq;
    for (uint32_t c = 0; c < h->cfg.n_seqs; c++) {
        if (h->lo[c] >= h->hi[c]) continue;
        if ((uint64_t)(h->lo[c] + 1) * P > h->len[c]) continue;      /* partial tail page */
        if (h->refc[h->bt[(size_t)c * MP + h->lo[c]]] > 1) continue;   /* shared prefix page */
        if (best < 0 || h->last_access[c] < h->last_access[best]) best = c;
    }
    return best;
}

/* ---- lifecycle ------------------------------------------------------------ */

void ct_kv_paged_destroy(ct_kv_paged_t *h) {
    if (!h) return;
    if (!h->host_only) {
        if (h->stage_pending) cudaEventSynchronize(h->stage_ev);
        cudaStreamSynchronize(h->stream);         /* no access to the buffers may be in flight */
        if (h->stage_ev) cudaEventDestroy(h->stage_ev);
        cudaFree(h->pool); cudaFree(h->scales); cudaFree(h->bt_dev); cudaFree(h->len_dev); cudaFree(h->stage_dev);
        if (h->stage_host) cudaFreeHost(h->stage_host);
    }
    free(h->bt); free(h->len); free(h->lo); free(h->hi); free(h->last_access); free(h->rank); free(h->refc);
    free(h->heap); free(h->log); free(h->claimed); free(h->pairs);
    if (h->tok) for (uint32_t s = 0; s < h->cfg.n_seqs; s++) free(h->tok[s]);
    free(h->tok); free(h->tok_n); free(h->tok_cap);
    free(h);
}

ct_kv_paged_t *ct_kv_paged_create(const ct_kv_paged_config_t *cfg) {
    if (!cfg || cfg->n_seqs == 0 || cfg->n_pages == 0 || cfg->max_pages_per_seq == 0 || cfg->dtype > CT_KV_Q1_0) {
        ct__set_error("ct_kv_paged_create: bad config");
        return NULL;
    }
    ct_kv_paged_t *h = (ct_kv_paged_t *)calloc(1, sizeof *h);
    if (!h) return NULL;
    h->cfg = *cfg;
    if (h->cfg.page_tokens == 0) h->cfg.page_tokens = 64;
    if (h->cfg.entry_dim == 0) h->cfg.entry_dim = 576;
    if (h->cfg.entry_dim % 16 != 0) { ct__set_error("ct_kv_paged_create: entry_dim % 16 != 0"); free(h); return NULL; }
    h->host_only = cfg->device < 0;
    if (!h->host_only && ct__cuda_status(cudaSetDevice(cfg->device), "ct_kv_paged_create")) { free(h); return NULL; }
    const uint32_t S = h->cfg.n_seqs, MP = h->cfg.max_pages_per_seq, NP = h->cfg.n_pages, P = h->cfg.page_tokens;
    const uint32_t dt = h->cfg.dtype, D = h->cfg.entry_dim;
    if (dt >= CT_KV_Q8_0) {
        /* block codecs: D/32 blocks of 34 / 18 / 10 / 6 bytes per token */
        static const uint32_t blk[4] = {34, 18, 10, 6};
        h->entry_bytes = (size_t)(D / 32) * blk[dt - CT_KV_Q8_0];
        if (D % 32 != 0 || D > 4096 || ((size_t)P * h->entry_bytes) % 16 != 0) {
            ct__set_error("ct_kv_paged_create: block pools need entry_dim % 32 == 0, <= 4096, and 16-byte pages");
            free(h);
            return NULL;
        }
    } else {
        h->entry_bytes = (size_t)D * (dt == CT_KV_BF16 ? 2 : dt == CT_KV_F32 ? 4 : 1);
    }
    h->page_bytes = (size_t)P * h->entry_bytes;
    const size_t bt_n = (size_t)S * MP;
    h->bt = (int32_t *)malloc(bt_n * sizeof(int32_t));
    h->len = (uint32_t *)calloc(S, sizeof(uint32_t));
    h->lo = (uint32_t *)calloc(S, sizeof(uint32_t));
    h->hi = (uint32_t *)calloc(S, sizeof(uint32_t));
    h->last_access = (uint64_t *)calloc(S, sizeof(uint64_t));
    h->rank = (uint32_t *)malloc((size_t)NP * sizeof(uint32_t));
    h->refc = (uint32_t *)calloc(NP, sizeof(uint32_t));
    h->heap = (int32_t *)malloc((size_t)NP * sizeof(int32_t));
    h->claimed = (uint8_t *)calloc(((size_t)NP * P + 7) / 8, 1);
    h->tok = (int32_t **)calloc(S, sizeof(int32_t *));
    h->tok_n = (uint32_t *)calloc(S, sizeof(uint32_t));
    h->tok_cap = (uint32_t *)calloc(S, sizeof(uint32_t));
    if (!h->bt || !h->len || !h->lo || !h->hi || !h->last_access || !h->rank || !h->refc || !h->heap || !h->claimed ||
        !h->tok || !h->tok_n || !h->tok_cap) {
        ct_kv_paged_destroy(h);
        return NULL;
    }
    for (size_t i = 0; i < bt_n; i++) h->bt[i] = -1;
    for (uint32_t p = 0; p < NP; p++) { h->rank[p] = p; h->heap[p] = (int32_t)p; }
    h->heap_n = NP;                      /* ascending ids already form a heap */
    h->st.n_pages_free = NP;
    if (h->host_only) return h;
    int rc = ct__cuda_status(cudaMalloc(&h->pool, (size_t)NP * h->page_bytes), "ct_kv_paged_create pool");
    if (!rc && (h->cfg.dtype == CT_KV_INT8 || h->cfg.dtype == CT_KV_E4M3))
        rc = ct__cuda_status(cudaMalloc((void **)&h->scales, (size_t)NP * P * sizeof(float)), "ct_kv_paged_create scales");
    if (!rc) rc = ct__cuda_status(cudaMalloc((void **)&h->bt_dev, bt_n * sizeof(int32_t)), "ct_kv_paged_create bt");
    if (!rc) rc = ct__cuda_status(cudaMalloc((void **)&h->len_dev, (size_t)S * sizeof(int32_t)), "ct_kv_paged_create len");
    if (!rc) rc = ct__cuda_status(cudaMemset(h->bt_dev, 0xFF, bt_n * sizeof(int32_t)), "ct_kv_paged_create");
    if (!rc) rc = ct__cuda_status(cudaMemset(h->len_dev, 0, (size_t)S * sizeof(int32_t)), "ct_kv_paged_create");
    if (!rc && h->scales) rc = ct__cuda_status(cudaMemset(h->scales, 0, (size_t)NP * P * sizeof(float)), "ct_kv_paged_create");
    if (!rc) rc = ct__cuda_status(cudaEventCreateWithFlags(&h->stage_ev, cudaEventDisableTiming), "ct_kv_paged_create");
    if (rc) { ct_kv_paged_destroy(h); return NULL; }
    return h;
}

int ct_kv_paged_set_stream(ct_kv_paged_t *h, void *stream) {
    if (!h) return CT_ERR_ARG;
    h->stream = (cudaStream_t)stream;
    return CT_OK;
}

int ct_kv_paged_set_free_order(ct_kv_paged_t *h, const int32_t *order) {
    if (!h || !order) return CT_ERR_ARG;
    const uint32_t NP = h->cfg.n_pages;
    uint8_t *seen = (uint8_t *)calloc(NP, 1);
    if (!seen) return CT_ERR_NOMEM;
    for (uint32_t i = 0; i < NP; i++) {
        if (order[i] < 0 || (uint32_t)order[i] >= NP || seen[order[i]]) { free(seen); return CT_ERR_ARG; }
        seen[order[i]] = 1;
    }
    free(seen);
    for (uint32_t i = 0; i < NP; i++) h->rank[order[i]] = i;
    int32_t *pages = (int32_t *)malloc((size_t)h->heap_n * sizeof(int32_t));
    if (!pages) return CT_ERR_NOMEM;
    memcpy(pages, h->heap, (size_t)h->heap_n * sizeof(int32_t));
    heap_rebuild(h, pages, h->heap_n);
    free(pages);
    return CT_OK;
}

/* ---- staging to the device ------------------------------------------------ */

static int stage_reserve(ct_kv_paged_t *h, size_t n) {
    if (h->stage_pending) {
        int rc = ct__cuda_status(cudaEventSynchronize(h->stage_ev), "stage");
        if (rc) return rc;
        h->stage_pending = 0;
    }
    if (n <= h->stage_cap) return CT_OK;
    size_t cap = h->stage_cap ? h->stage_cap : 4096;
    while (cap < n) cap *= 2;
    if (h->stage_host) cudaFreeHost(h->stage_host);
    if (h->stage_dev) cudaFree(h->stage_dev);
    h->stage_host = NULL; h->stage_dev = NULL; h->stage_cap = 0;
    int rc = ct__cuda_status(cudaMallocHost((void **)&h->stage_host, cap * sizeof(int32_t)), "stage host");
    if (!rc) rc = ct__cuda_status(cudaMalloc((void **)&h->stage_dev, cap * sizeof(int32_t)), "stage dev");
    if (rc) return rc;
    h->stage_cap = cap;
    return CT_OK;
}

/* Inputs of ct_kv_paged_append_projected: the entries are W . x[t]. */
typedef struct {
    const void *x, *w;
    const float *norm_w;
    float eps;
    uint32_t norm_dim, n_in;
} proj_args_t;

/* Uploads n_dest token slots plus the pending bt / len (index, value) pairs
 * in one pinned staging copy, then runs the scatters and the token writes
 * (entries copied, or projected when pj is set). */
static int flush(ct_kv_paged_t *h, const int32_t *dest, uint32_t n_dest, const void *entries, uint32_t src_dtype,
                 const proj_args_t *pj) {
    const size_t n_pairs = (size_t)h->n_bt_pairs + h->n_len_pairs;
    const size_t total = n_dest + 2 * n_pairs;
    if (h->host_only) {
        h->n_bt_pairs = h->n_len_pairs = 0;
        return entries || pj ? CT_ERR_UNSUPPORTED : CT_OK;
    }
    if (total == 0) return CT_OK;
    int rc = stage_reserve(h, total);
    if (rc) return rc;
    if (n_dest) memcpy(h->stage_host, dest, (size_t)n_dest * sizeof(int32_t));
    /* Stage the final host value of every touched index: an index touched
     * twice in one call then carries one value, and the scatter needs no order. */
    int32_t *pr = h->stage_host + n_dest;
    for (uint32_t i = 0; i < h->n_bt_pairs; i++) {
        pr[2 * i] = h->pairs[2 * i];
        pr[2 * i + 1] = h->bt[h->pairs[2 * i]];
    }
    for (uint32_t i = h->n_bt_pairs; i < h->n_bt_pairs + h->n_len_pairs; i++) {
        pr[2 * i] = h->pairs[2 * i];
        pr[2 * i + 1] = (int32_t)h->len[h->pairs[2 * i]];
    }
    rc = ct__cuda_status(cudaMemcpyAsync(h->stage_dev, h->stage_host, total * sizeof(int32_t),
                                         cudaMemcpyHostToDevice, h->stream), "stage upload");
    if (!rc) rc = ct__cuda_status(cudaEventRecord(h->stage_ev, h->stream), "stage event");
    if (rc) return rc;
    h->stage_pending = 1;
    if (h->n_bt_pairs) rc = ct__launch_scatter_i32(h->bt_dev, h->stage_dev + n_dest, h->n_bt_pairs, h->stream);
    if (!rc && h->n_len_pairs)
        rc = ct__launch_scatter_i32(h->len_dev, h->stage_dev + n_dest + 2 * (size_t)h->n_bt_pairs, h->n_len_pairs, h->stream);
    if (!rc && pj && n_dest)
        rc = ct_kv_project_write_slots(pj->x, pj->w, pj->norm_w, pj->eps, pj->norm_dim, n_dest, pj->n_in,
                                       h->cfg.entry_dim, h->pool, h->scales, h->cfg.dtype, h->stage_dev, h->stream);
    else if (!rc && entries && n_dest)
        rc = ct_kv_paged_write_slots(h->pool, h->scales, h->cfg.dtype, entries, src_dtype, h->stage_dev, n_dest,
                                     h->cfg.entry_dim, h->stream);
    h->n_bt_pairs = h->n_len_pairs = 0;
    return rc;
}

static int push_len(ct_kv_paged_t *h, uint32_t s) {
    if (pairs_reserve(h, 1)) return CT_ERR_NOMEM;
    uint32_t i = h->n_bt_pairs + h->n_len_pairs;
    h->pairs[2 * i] = (int32_t)s;
    h->pairs[2 * i + 1] = (int32_t)h->len[s];
    h->n_len_pairs++;
    return CT_OK;
}

/* ---- append --------------------------------------------------------------- */

static int append_impl(ct_kv_paged_t *h, const uint32_t *seq_ids, const uint32_t *counts, uint32_t n,
                       const void *entries, uint32_t src_dtype, const proj_args_t *pj) {
    if (!h || (n && (!seq_ids || !counts))) return CT_ERR_ARG;
    if (pj && h->host_only) return CT_ERR_UNSUPPORTED;
    if (entries && h->host_only) return CT_ERR_UNSUPPORTED;
    if (entries && src_dtype != CT_KV_BF16 && src_dtype != CT_KV_F32) return CT_ERR_ARG;
    const uint32_t P = h->cfg.page_tokens, MP = h->cfg.max_pages_per_seq, W = h->cfg.window_tokens;
    size_t total = 0;
    uint32_t maxc = 0;
    for (uint32_t i = 0; i < n; i++) {
        if (seq_ids[i] >= h->cfg.n_seqs) return CT_ERR_ARG;
        total += counts[i];
        if (counts[i] > maxc) maxc = counts[i];
    }
    if (total > 0x7FFFFFFFu) return CT_ERR_ARG;
    int rc = CT_OK;
    size_t *off = (size_t *)malloc((n ? n : 1) * sizeof(size_t));
    int32_t *dest = (int32_t *)malloc((total ? total : 1) * sizeof(int32_t));
    if (!off || !dest) { free(off); free(dest); return CT_ERR_NOMEM; }
    for (uint32_t i = 0, acc = 0; i < n; i++) { off[i] = acc; acc += counts[i]; }
    h->n_bt_pairs = h->n_len_pairs = 0;

    for (uint32_t k = 0; k < maxc && rc == CT_OK; k++) {
        for (uint32_t i = 0; i < n; i++) {
            if (k >= counts[i]) continue;
            const uint32_t s = seq_ids[i];
            const uint32_t r = h->len[s];
            const uint32_t lp = r / P;
            if (r % P == 0) {
                if (lp >= MP) { rc = CT_ERR_FULL; ct__set_error("append: block table row full"); break; }
                if (h->heap_n == 0) {
                    int64_t c = lru_victim(h);
                    if (c < 0) { rc = CT_ERR_FULL; ct__set_error("append: no evictable page"); break; }
                    if ((rc = free_low_page(h, (uint32_t)c, 2))) break;
                }
                int32_t ph = heap_pop(h);
                h->refc[ph] = 1;
                if ((rc = set_bt(h, s, lp, ph))) break;
                if (h->lo[s] == h->hi[s]) h->lo[s] = lp;
                h->hi[s] = lp + 1;
                h->st.n_pages_live++;
            }
            const int32_t ph = h->bt[(size_t)s * MP + lp];
            dest[off[i] + k] = ph * (int32_t)P + (int32_t)(r % P);
            h->len[s] = r + 1;
            h->last_access[s] = h->st.clock;
            h->st.n_appends++;
            if (W > 0 && r + 1 > W) {
                const uint64_t below = (uint64_t)r + 1 - W;
                while (h->lo[s] < h->hi[s] && (uint64_t)(h->lo[s] + 1) * P <= below)
                    if ((rc = free_low_page(h, s, 1))) break;
                if (rc) break;
            }
        }
        h->st.clock++;
    }
    if (rc == CT_OK && total > 1) {
        /* Last writer wins when a page was freed and reused inside the call:
         * walk the writes backwards in time (rounds descending, then array
         * order descending) and keep only the final write of each slot. */
        for (uint32_t k = maxc; k-- > 0;) {
            for (uint32_t i = n; i-- > 0;) {
                if (k >= counts[i]) continue;
                int32_t *d = &dest[off[i] + k];
                int32_t sl = *d;
                if (sl < 0) continue;
                if (h->claimed[sl >> 3] & (1u << (sl & 7))) *d = -1;
                else h->claimed[sl >> 3] |= (uint8_t)(1u << (sl & 7));
            }
        }
        for (size_t t = 0; t < total; t++) {
            int32_t sl = dest[t];
            if (sl >= 0) h->claimed[sl >> 3] = 0;
        }
        /* the clearing above zeroes whole bytes; bytes holding a discarded
         * duplicate were already set by its winner and are cleared with it */
    }
    if (rc == CT_OK)
        for (uint32_t i = 0; i < n; i++) if ((rc = push_len(h, seq_ids[i]))) break;
    free(off);
    h->st.n_pages_free = h->heap_n;
    if (rc != CT_OK) {
        /* Host state already advanced: publish what changed so the device
         * mirrors stay consistent, but write no token data. */
        flush(h, NULL, 0, NULL, 0, NULL);
        free(dest);
        return rc;
    }
    /* Without entries only the tables change: the slots need not travel. */
    rc = flush(h, dest, entries || pj ? (uint32_t)total : 0u, entries, src_dtype, pj);
    free(dest);
    return rc;
}

int ct_kv_paged_append(ct_kv_paged_t *h, const uint32_t *seq_ids, const uint32_t *counts, uint32_t n,
                       const void *entries, uint32_t src_dtype) {
    return append_impl(h, seq_ids, counts, n, entries, src_dtype, NULL);
}

int ct_kv_paged_append_projected(ct_kv_paged_t *h, const uint32_t *seq_ids, const uint32_t *counts, uint32_t n,
                                 const void *x, const void *w, uint32_t n_in, const float *norm_w, float eps,
                                 uint32_t norm_dim) {
    if (!x || !w) return CT_ERR_ARG;
    const proj_args_t pj = {x, w, norm_w, eps, norm_dim, n_in};
    return append_impl(h, seq_ids, counts, n, NULL, 0, &pj);
}

int ct_kv_paged_free_seq(ct_kv_paged_t *h, uint32_t s) {
    if (!h || s >= h->cfg.n_seqs) return CT_ERR_ARG;
    int rc = CT_OK;
    while (h->lo[s] < h->hi[s]) if ((rc = free_low_page(h, s, 0))) return rc;
    h->lo[s] = h->hi[s] = 0;
    h->len[s] = 0;
    h->tok_n[s] = 0;
    if ((rc = push_len(h, s))) return rc;
    h->st.n_pages_free = h->heap_n;
    return flush(h, NULL, 0, NULL, 0, NULL);
}

int ct_kv_paged_evict_lru(ct_kv_paged_t *h, uint32_t n) {
    if (!h) return CT_ERR_ARG;
    int rc = CT_OK;
    uint32_t done = 0;
    for (; done < n; done++) {
        int64_t c = lru_victim(h);
        if (c < 0) break;
        if ((rc = free_low_page(h, (uint32_t)c, 2))) return rc;
    }
    h->st.n_pages_free = h->heap_n;
    rc = flush(h, NULL, 0, NULL, 0, NULL);
    return rc ? rc : (int)done;
}

/* ---- prefix sharing ------------------------------------------------------ */

static int tok_reserve(ct_kv_paged_t *h, uint32_t s, uint32_t n) {
    if (n <= h->tok_cap[s]) return CT_OK;
    uint32_t cap = h->tok_cap[s] ? h->tok_cap[s] : 256;
    while (cap < n) cap *= 2;
    int32_t *t = (int32_t *)realloc(h->tok[s], (size_t)cap * sizeof(int32_t));
    if (!t) return CT_ERR_NOMEM;
    h->tok[s] = t;
    h->tok_cap[s] = cap;
    return CT_OK;
}

int ct_kv_paged_fork(ct_kv_paged_t *h, uint32_t src, uint32_t dst, uint32_t n_tokens) {
    if (!h || src >= h->cfg.n_seqs || dst >= h->cfg.n_seqs || src == dst) return CT_ERR_ARG;
    if (h->len[dst] != 0 || h->lo[dst] != h->hi[dst] || n_tokens > h->len[src]) return CT_ERR_ARG;
    const uint32_t P = h->cfg.page_tokens, MP = h->cfg.max_pages_per_seq;
    const uint32_t full = n_tokens / P, rem = n_tokens % P;
    if (n_tokens && h->lo[src] != 0) {                /* the window already dropped part of the prefix */
        ct__set_error("ct_kv_paged_fork: the prefix is no longer mapped");
        return CT_ERR_UNMAPPED;
    }
    h->n_bt_pairs = h->n_len_pairs = 0;
    int rc = CT_OK;
    for (uint32_t lp = 0; lp < full && !rc; lp++) {   /* full pages: shared, never written again */
        const int32_t ph = h->bt[(size_t)src * MP + lp];
        h->refc[ph]++;
        rc = set_bt(h, dst, lp, ph);
    }
    int32_t copy_from = -1, copy_to = -1;
    if (!rc && rem) {                                 /* the partial page: dst's own copy */
        if (h->heap_n == 0) {
            int64_t c = lru_victim(h);
            if (c < 0) { ct__set_error("fork: no evictable page"); rc = CT_ERR_FULL; }
            else rc = free_low_page(h, (uint32_t)c, 2);
        }
        if (!rc) {
            copy_from = h->bt[(size_t)src * MP + full];
            copy_to = heap_pop(h);
            h->refc[copy_to] = 1;
            h->st.n_pages_live++;
            rc = set_bt(h, dst, full, copy_to);
        }
    }
    if (rc) {                                         /* undo the shared references, publish any eviction */
        for (uint32_t lp = 0; lp < full; lp++) {
            const int32_t ph = h->bt[(size_t)dst * MP + lp];
            if (ph >= 0) { h->refc[ph]--; set_bt(h, dst, lp, -1); }
        }
        h->st.n_pages_free = h->heap_n;
        flush(h, NULL, 0, NULL, 0, NULL);
        return rc;
    }
    h->lo[dst] = 0;
    h->hi[dst] = full + (rem ? 1 : 0);
    h->len[dst] = n_tokens;
    {                                                 /* the prefix's token ids come along */
        const uint32_t nt = h->tok_n[src] < n_tokens ? h->tok_n[src] : n_tokens;
        h->tok_n[dst] = 0;
        if (nt && tok_reserve(h, dst, nt) == CT_OK) {
            memcpy(h->tok[dst], h->tok[src], (size_t)nt * sizeof(int32_t));
            h->tok_n[dst] = nt;
        }
    }
    h->last_access[dst] = h->st.clock++;
    if ((rc = push_len(h, dst))) return rc;
    h->st.n_pages_free = h->heap_n;
    if (!h->host_only && copy_to >= 0) {             /* first rem slots of the page, and their scales */
        const size_t tok_bytes = h->page_bytes / P;
        rc = ct__cuda_status(cudaMemcpyAsync((uint8_t *)h->pool + (size_t)copy_to * h->page_bytes,
                                             (const uint8_t *)h->pool + (size_t)copy_from * h->page_bytes,
                                             rem * tok_bytes, cudaMemcpyDeviceToDevice, h->stream), "fork copy");
        if (!rc && h->scales)
            rc = ct__cuda_status(cudaMemcpyAsync(h->scales + (size_t)copy_to * P, h->scales + (size_t)copy_from * P,
                                                 rem * sizeof(float), cudaMemcpyDeviceToDevice, h->stream), "fork copy");
        if (rc) return rc;
    }
    return flush(h, NULL, 0, NULL, 0, NULL);
}

uint32_t ct_kv_paged_page_refs(const ct_kv_paged_t *h, int32_t page) {
    if (!h || page < 0 || (uint32_t)page >= h->cfg.n_pages) return 0;
    return h->refc[page];
}

int ct_kv_paged_set_tokens(ct_kv_paged_t *h, uint32_t seq, uint32_t start, const int32_t *ids, uint32_t n) {
    if (!h || seq >= h->cfg.n_seqs || (n && !ids)) return CT_ERR_ARG;
    if (start > h->tok_n[seq] || (uint64_t)start + n > h->len[seq]) return CT_ERR_ARG;
    int rc = tok_reserve(h, seq, start + n);
    if (rc) return rc;
    memcpy(h->tok[seq] + start, ids, (size_t)n * sizeof(int32_t));
    if (start + n > h->tok_n[seq]) h->tok_n[seq] = start + n;
    return CT_OK;
}

uint32_t ct_kv_paged_tokens(const ct_kv_paged_t *h, uint32_t seq, int32_t *ids, uint32_t max) {
    if (!h || seq >= h->cfg.n_seqs) return 0;
    const uint32_t n = h->tok_n[seq] < max ? h->tok_n[seq] : max;
    if (ids && n) memcpy(ids, h->tok[seq], (size_t)n * sizeof(int32_t));
    return h->tok_n[seq];
}

int ct_kv_paged_match_prefix(const ct_kv_paged_t *h, const int32_t *ids, uint32_t n, uint32_t *seq_out,
                             uint32_t *len_out) {
    if (!h || (n && !ids) || !seq_out || !len_out) return CT_ERR_ARG;
    uint32_t best = 0, best_s = 0;
    for (uint32_t s = 0; s < h->cfg.n_seqs; s++) {
        if (h->lo[s] != 0 || h->lo[s] == h->hi[s]) continue;      /* nothing mapped from position 0 */
        const uint32_t lim = h->tok_n[s] < n ? h->tok_n[s] : n;
        uint32_t m = 0;
        while (m < lim && h->tok[s][m] == ids[m]) m++;
        if (m > best) { best = m; best_s = s; }
    }
    *seq_out = best_s;
    *len_out = best;
    return CT_OK;
}

/* ---- compaction ----------------------------------------------------------- */

int ct_kv_paged_compact(ct_kv_paged_t *h) {
    if (!h) return CT_ERR_ARG;
    const uint32_t S = h->cfg.n_seqs, MP = h->cfg.max_pages_per_seq, NP = h->cfg.n_pages, P = h->cfg.page_tokens;
    int32_t *map;
    int rc = CT_OK;
    if (h->host_only) {
        map = h->heap;                            /* scratch: rebuilt below */
    } else {
        rc = stage_reserve(h, (size_t)S * MP + NP + 64);
        if (rc) return rc;
        map = h->stage_host;                      /* [n_live] new -> old, then the bt image */
    }
    /* a page shared by several sequences gets one new id, at its first use */
    int32_t *new_id = (int32_t *)malloc((size_t)NP * sizeof(int32_t));
    uint32_t *refc2 = (uint32_t *)calloc(NP, sizeof(uint32_t));
    if (!new_id || !refc2) { free(new_id); free(refc2); return CT_ERR_NOMEM; }
    for (uint32_t p = 0; p < NP; p++) new_id[p] = -1;
    uint32_t n_live = 0;
    for (uint32_t s = 0; s < S; s++)
        for (uint32_t lp = h->lo[s]; lp < h->hi[s]; lp++) {
            int32_t *e = h->bt + (size_t)s * MP + lp;
            if (new_id[*e] < 0) {
                new_id[*e] = (int32_t)n_live;
                refc2[n_live] = h->refc[*e];
                map[n_live++] = *e;
            }
            *e = new_id[*e];
        }
    memcpy(h->refc, refc2, (size_t)NP * sizeof(uint32_t));
    free(new_id);
    free(refc2);
    if (h->host_only) goto renumbered;
    void *new_pool = NULL;
    float *new_scales = NULL;
    /* stream-ordered allocations: after the first compaction the pool's
     * memory comes back from the driver's cache without a device sync */
    rc = ct__cuda_status(cudaMallocAsync(&new_pool, (size_t)NP * h->page_bytes, h->stream), "compact pool");
    if (!rc && h->scales)
        rc = ct__cuda_status(cudaMallocAsync((void **)&new_scales, (size_t)NP * P * sizeof(float), h->stream),
                             "compact scales");
    if (!rc && new_scales) rc = ct__cuda_status(cudaMemsetAsync(new_scales, 0, (size_t)NP * P * sizeof(float), h->stream), "compact");
    /* bt image follows the map in the staging buffer */
    memcpy(map + n_live, h->bt, (size_t)S * MP * sizeof(int32_t));
    if (!rc) rc = ct__cuda_status(cudaMemcpyAsync(h->stage_dev, map, ((size_t)n_live + (size_t)S * MP) * sizeof(int32_t),
                                                  cudaMemcpyHostToDevice, h->stream), "compact upload");
    if (!rc) rc = ct_kv_paged_move_pages(h->pool, h->scales, new_pool, new_scales, h->stage_dev, n_live,
                                         h->page_bytes, P, h->stream);
    if (!rc) rc = ct__cuda_status(cudaMemcpyAsync(h->bt_dev, h->stage_dev + n_live, (size_t)S * MP * sizeof(int32_t),
                                                  cudaMemcpyDeviceToDevice, h->stream), "compact bt");
    if (rc) {
        if (new_pool) cudaFreeAsync(new_pool, h->stream);
        if (new_scales) cudaFreeAsync(new_scales, h->stream);
        cudaStreamSynchronize(h->stream);
        return rc;
    }
    if (h->pool_async) {                          /* from an earlier compaction: back to the cache */
        cudaFreeAsync(h->pool, h->stream);
        if (h->scales) cudaFreeAsync(h->scales, h->stream);
    }
    /* the staging buffer is reused by the next call on the host */
    rc = ct__cuda_status(cudaStreamSynchronize(h->stream), "compact sync");
    if (rc) return rc;
    if (!h->pool_async) {                         /* the create-time buffers */
        cudaFree(h->pool);
        cudaFree(h->scales);
    }
    h->pool_async = 1;
    h->pool = new_pool;
    h->scales = new_scales;
renumbered:
    /* Free pages are now n_live..NP-1, handed out in ascending order. */
    for (uint32_t p = 0; p < NP; p++) h->rank[p] = p;
    h->heap_n = 0;
    for (uint32_t p = n_live; p < NP; p++) h->heap[h->heap_n++] = (int32_t)p;
    h->st.n_pages_free = h->heap_n;
    h->st.n_compactions++;
    h->st.bytes_compacted += 2ull * n_live * h->page_bytes;
    return CT_OK;
}

/* ---- reads ------------------------------------------------------------------ */

int ct_kv_paged_gather(ct_kv_paged_t *h, uint32_t seq, uint32_t start, uint32_t n, void *out, uint32_t out_dtype) {
    if (!h || !out || seq >= h->cfg.n_seqs) return CT_ERR_ARG;
    if (h->host_only) return CT_ERR_UNSUPPORTED;
    if (out_dtype != CT_KV_BF16 && out_dtype != CT_KV_F32) return CT_ERR_ARG;
    if ((uint64_t)start + n > h->len[seq]) return CT_ERR_ARG;
    if (n == 0) return CT_OK;
    const uint32_t P = h->cfg.page_tokens;
    for (uint32_t lp = start / P; lp <= (start + n - 1) / P; lp++)
        if (h->bt[(size_t)seq * h->cfg.max_pages_per_seq + lp] < 0) return CT_ERR_UNMAPPED;
    return ct__launch_kv_gather(h->pool, h->scales, h->cfg.dtype, h->bt_dev + (size_t)seq * h->cfg.max_pages_per_seq,
                                P, h->cfg.entry_dim, start, n, out, out_dtype, h->stream);
}

int ct_kv_paged_gather_batch(ct_kv_paged_t *h, const uint32_t *seqs, const uint32_t *starts,
                             const uint32_t *counts, uint32_t n, void *out, uint32_t out_dtype) {
    if (!h || (n && (!seqs || !starts || !counts || !out))) return CT_ERR_ARG;
    if (h->host_only) return CT_ERR_UNSUPPORTED;
    if (out_dtype != CT_KV_BF16 && out_dtype != CT_KV_F32) return CT_ERR_ARG;
    const uint32_t P = h->cfg.page_tokens, MP = h->cfg.max_pages_per_seq;
    for (uint32_t i = 0; i < n; i++) {
        if (seqs[i] >= h->cfg.n_seqs || (uint64_t)starts[i] + counts[i] > h->len[seqs[i]]) return CT_ERR_ARG;
        if (counts[i] == 0) continue;
        for (uint32_t lp = starts[i] / P; lp <= (starts[i] + counts[i] - 1) / P; lp++)
            if (h->bt[(size_t)seqs[i] * MP + lp] < 0) return CT_ERR_UNMAPPED;
    }
    const size_t row_bytes = (size_t)h->cfg.entry_dim * (out_dtype == CT_KV_BF16 ? 2 : 4);
    uint64_t row = 0;
    for (uint32_t b = 0; b < n; b += 65535u) {                /* one launch per 65535 ranges */
        const uint32_t m = n - b < 65535u ? n - b : 65535u;
        int rc = stage_reserve(h, (size_t)4 * m);
        if (rc) return rc;
        uint32_t max_count = 0;
        const uint64_t row0 = row;
        for (uint32_t i = 0; i < m; i++) {
            int32_t *d = h->stage_host + 4 * (size_t)i;
            d[0] = (int32_t)seqs[b + i];
            d[1] = (int32_t)starts[b + i];
            d[2] = (int32_t)counts[b + i];
            d[3] = (int32_t)(row - row0);
            row += counts[b + i];
            if (counts[b + i] > max_count) max_count = counts[b + i];
        }
        if (row - row0 > 0x7FFFFFFFu) return CT_ERR_ARG;
        rc = ct__cuda_status(cudaMemcpyAsync(h->stage_dev, h->stage_host, (size_t)4 * m * sizeof(int32_t),
                                             cudaMemcpyHostToDevice, h->stream), "gather_batch upload");
        if (!rc) rc = ct__cuda_status(cudaEventRecord(h->stage_ev, h->stream), "gather_batch event");
        if (rc) return rc;
        h->stage_pending = 1;
        rc = ct__launch_kv_gather_batch(h->pool, h->scales, h->cfg.dtype, h->bt_dev, MP, P, h->cfg.entry_dim,
                                        h->stage_dev, m, max_count, (uint8_t *)out + row0 * row_bytes, out_dtype,
                                        h->stream);
        if (rc) return rc;
    }
    return CT_OK;
}

int ct_kv_paged_block_table(const ct_kv_paged_t *h, int32_t *out) {
    if (!h || !out) return CT_ERR_ARG;
    memcpy(out, h->bt, (size_t)h->cfg.n_seqs * h->cfg.max_pages_per_seq * sizeof(int32_t));
    return CT_OK;
}

int ct_kv_paged_seq_lens(const ct_kv_paged_t *h, uint32_t *out) {
    if (!h || !out) return CT_ERR_ARG;
    memcpy(out, h->len, (size_t)h->cfg.n_seqs * sizeof(uint32_t));
    return CT_OK;
}

int ct_kv_paged_last_access(const ct_kv_paged_t *h, uint64_t *out) {
    if (!h || !out) return CT_ERR_ARG;
    memcpy(out, h->last_access, (size_t)h->cfg.n_seqs * sizeof(uint64_t));
    return CT_OK;
}

uint32_t ct_kv_paged_evict_log(const ct_kv_paged_t *h, ct_kv_evict_event_t *out, uint32_t max) {
    if (!h) return 0;
    if (!out) return h->log_n;
    uint32_t n = h->log_n < max ? h->log_n : max;
    memcpy(out, h->log, (size_t)n * sizeof *out);
    return n;
}

ct_kv_paged_stats_t ct_kv_paged_stats(const ct_kv_paged_t *h) {
    ct_kv_paged_stats_t s;
    memset(&s, 0, sizeof s);
    if (h) s = h->st;
    return s;
}

const ct_kv_paged_config_t *ct_kv_paged_config(const ct_kv_paged_t *h) { return h ? &h->cfg : NULL; }
void *ct_kv_paged_pool(ct_kv_paged_t *h) { return h ? h->pool : NULL; }
float *ct_kv_paged_scales(ct_kv_paged_t *h) { return h ? h->scales : NULL; }
const int32_t *ct_kv_paged_block_table_dev(const ct_kv_paged_t *h) { return h ? h->bt_dev : NULL; }
const int32_t *ct_kv_paged_seq_lens_dev(const ct_kv_paged_t *h) { return h ? h->len_dev : NULL; }

/* ---- checkpoint --------------------------------------------------------- */

/* File layout (little-endian, no padding): "CTKVPAGE", u32 version (1),
 * u32 flags (bit 0: page bytes present); the 8 config words; the statistics
 * (5 x u64, 2 x u32, u64); per sequence len, lo, hi (u32) and last_access
 * (u64); the block table (i32, n_seqs x max_pages); the free-order rank of
 * every page (u32); the free set (u32 count, i32 ids); the eviction log (u32
 * count, 5 x u32 each); the live pages (u32 count, then per page its id (i32),
 * page bytes, and page_tokens fp32 scales for int8 / e4m3 pools); version 2
 * then the token ids (per sequence a u32 count and that many i32); last an
 * FNV-1a 64 of everything before it.  Version 1 files (no token ids) load. */

#define CKPT_MAGIC "CTKVPAGE"
#define CKPT_VERSION 2u

typedef struct {
    FILE *f;
    uint64_t fnv;
    int err;
} ckpt_io_t;

static void fnv_feed(ckpt_io_t *io, const void *p, size_t n) {
    const uint8_t *b = (const uint8_t *)p;
    for (size_t i = 0; i < n; i++) { io->fnv ^= b[i]; io->fnv *= 0x100000001B3ull; }
}
static void ck_write(ckpt_io_t *io, const void *p, size_t n) {
    if (io->err || n == 0) return;
    if (fwrite(p, 1, n, io->f) != n) { io->err = 1; return; }
    fnv_feed(io, p, n);
}
static void ck_read(ckpt_io_t *io, void *p, size_t n) {
    if (io->err || n == 0) return;
    if (fread(p, 1, n, io->f) != n) { io->err = 1; return; }
    fnv_feed(io, p, n);
}

int ct_kv_paged_save(ct_kv_paged_t *h, const char *path) {
    if (!h || !path) return CT_ERR_ARG;
    const uint32_t S = h->cfg.n_seqs, MP = h->cfg.max_pages_per_seq, NP = h->cfg.n_pages, P = h->cfg.page_tokens;
    if (!h->host_only) {                               /* every queued write has landed */
        int rc = ct__cuda_status(cudaStreamSynchronize(h->stream), "ct_kv_paged_save");
        if (rc) return rc;
    }
    FILE *f = fopen(path, "wb");
    if (!f) { ct__set_error("ct_kv_paged_save: cannot open the file"); return CT_ERR_IO; }
    ckpt_io_t io = {f, 0xCBF29CE484222325ull, 0};
    const uint32_t ver = CKPT_VERSION, flags = h->host_only ? 0u : 1u;
    ck_write(&io, CKPT_MAGIC, 8);
    ck_write(&io, &ver, 4);
    ck_write(&io, &flags, 4);
    const uint32_t cfgw[8] = {h->cfg.n_seqs, h->cfg.max_pages_per_seq, h->cfg.n_pages, h->cfg.page_tokens,
                              h->cfg.entry_dim, h->cfg.window_tokens, h->cfg.dtype, (uint32_t)h->cfg.device};
    ck_write(&io, cfgw, sizeof cfgw);
    const uint64_t st64[5] = {h->st.n_appends, h->st.n_evict_window, h->st.n_evict_lru, h->st.n_compactions,
                              h->st.bytes_compacted};
    const uint32_t st32[2] = {h->st.n_pages_live, h->st.n_pages_free};
    ck_write(&io, st64, sizeof st64);
    ck_write(&io, st32, sizeof st32);
    ck_write(&io, &h->st.clock, 8);
    ck_write(&io, h->len, (size_t)S * 4);
    ck_write(&io, h->lo, (size_t)S * 4);
    ck_write(&io, h->hi, (size_t)S * 4);
    ck_write(&io, h->last_access, (size_t)S * 8);
    ck_write(&io, h->bt, (size_t)S * MP * 4);
    ck_write(&io, h->rank, (size_t)NP * 4);
    ck_write(&io, &h->heap_n, 4);
    ck_write(&io, h->heap, (size_t)h->heap_n * 4);
    ck_write(&io, &h->log_n, 4);
    for (uint32_t i = 0; i < h->log_n && !io.err; i++) {
        const uint32_t e[5] = {h->log[i].round, h->log[i].seq, h->log[i].lpage, (uint32_t)h->log[i].phys,
                               h->log[i].reason};
        ck_write(&io, e, sizeof e);
    }
    uint32_t n_live = 0;                              /* distinct mapped pages (shared ones once) */
    uint8_t *seen = (uint8_t *)calloc(NP, 1);
    if (!seen) { fclose(f); return CT_ERR_NOMEM; }
    for (size_t i = 0; i < (size_t)S * MP; i++)
        if (h->bt[i] >= 0 && !seen[h->bt[i]]) { seen[h->bt[i]] = 1; n_live++; }
    memset(seen, 0, NP);
    ck_write(&io, &n_live, 4);
    int rc = CT_OK;
    if (!h->host_only && n_live) {
        const size_t sc_bytes = h->scales ? (size_t)P * sizeof(float) : 0;
        uint8_t *buf = (uint8_t *)malloc(h->page_bytes + sc_bytes);
        if (!buf) { free(seen); fclose(f); return CT_ERR_NOMEM; }
        for (size_t i = 0; i < (size_t)S * MP && !rc && !io.err; i++) {
            const int32_t pg = h->bt[i];
            if (pg < 0 || seen[pg]) continue;
            seen[pg] = 1;
            rc = ct__cuda_status(cudaMemcpy(buf, (const uint8_t *)h->pool + (size_t)pg * h->page_bytes,
                                            h->page_bytes, cudaMemcpyDeviceToHost), "ct_kv_paged_save page");
            if (!rc && sc_bytes)
                rc = ct__cuda_status(cudaMemcpy(buf + h->page_bytes, h->scales + (size_t)pg * P, sc_bytes,
                                                cudaMemcpyDeviceToHost), "ct_kv_paged_save scales");
            ck_write(&io, &pg, 4);
            ck_write(&io, buf, h->page_bytes + sc_bytes);
        }
        free(buf);
    }
    free(seen);
    for (uint32_t s = 0; s < S && !io.err; s++) {
        ck_write(&io, &h->tok_n[s], 4);
        ck_write(&io, h->tok[s], (size_t)h->tok_n[s] * 4);
    }
    const uint64_t sum = io.fnv;
    if (!io.err && fwrite(&sum, 8, 1, f) != 1) io.err = 1;
    if (fclose(f) != 0) io.err = 1;
    if (rc) return rc;
    if (io.err) { ct__set_error("ct_kv_paged_save: write failed"); return CT_ERR_IO; }
    return CT_OK;
}

ct_kv_paged_t *ct_kv_paged_load(const char *path, int device) {
    if (!path) return NULL;
    FILE *f = fopen(path, "rb");
    if (!f) { ct__set_error("ct_kv_paged_load: cannot open the file"); return NULL; }
    ckpt_io_t io = {f, 0xCBF29CE484222325ull, 0};
    char magic[8];
    uint32_t ver = 0, flags = 0, cfgw[8];
    ck_read(&io, magic, 8);
    ck_read(&io, &ver, 4);
    ck_read(&io, &flags, 4);
    ck_read(&io, cfgw, sizeof cfgw);
    if (io.err || memcmp(magic, CKPT_MAGIC, 8) != 0 || ver < 1 || ver > CKPT_VERSION) {
        fclose(f);
        ct__set_error("ct_kv_paged_load: not a paged KV checkpoint of version 1 or 2");
        return NULL;
    }
    ct_kv_paged_config_t cfg = {cfgw[0], cfgw[1], cfgw[2], cfgw[3], cfgw[4], cfgw[5], cfgw[6], device};
    if ((flags & 1u) == 0 && device >= 0) {
        fclose(f);
        ct__set_error("ct_kv_paged_load: the checkpoint holds tables only (load it with device -1)");
        return NULL;
    }
    ct_kv_paged_t *h = ct_kv_paged_create(&cfg);
    if (!h) { fclose(f); return NULL; }
    const uint32_t S = h->cfg.n_seqs, MP = h->cfg.max_pages_per_seq, NP = h->cfg.n_pages, P = h->cfg.page_tokens;
    uint64_t st64[5];
    uint32_t st32[2];
    ck_read(&io, st64, sizeof st64);
    ck_read(&io, st32, sizeof st32);
    ck_read(&io, &h->st.clock, 8);
    h->st.n_appends = st64[0]; h->st.n_evict_window = st64[1]; h->st.n_evict_lru = st64[2];
    h->st.n_compactions = st64[3]; h->st.bytes_compacted = st64[4];
    h->st.n_pages_live = st32[0]; h->st.n_pages_free = st32[1];
    ck_read(&io, h->len, (size_t)S * 4);
    ck_read(&io, h->lo, (size_t)S * 4);
    ck_read(&io, h->hi, (size_t)S * 4);
    ck_read(&io, h->last_access, (size_t)S * 8);
    ck_read(&io, h->bt, (size_t)S * MP * 4);
    ck_read(&io, h->rank, (size_t)NP * 4);
    uint32_t free_n = 0, log_n = 0, n_live = 0;
    ck_read(&io, &free_n, 4);
    int bad = io.err || free_n > NP;
    for (uint32_t i = 0; i < S && !bad; i++)
        bad = (uint64_t)h->len[i] > (uint64_t)MP * P || h->lo[i] > h->hi[i] || h->hi[i] > MP;
    for (uint32_t p = 0; p < NP && !bad; p++) bad = h->rank[p] >= NP;
    for (size_t i = 0; i < (size_t)S * MP && !bad; i++) bad = h->bt[i] < -1 || h->bt[i] >= (int32_t)NP;
    if (!bad) {                                        /* reference counts follow from the table */
        memset(h->refc, 0, (size_t)NP * sizeof(uint32_t));
        for (size_t i = 0; i < (size_t)S * MP; i++) if (h->bt[i] >= 0) h->refc[h->bt[i]]++;
        ck_read(&io, h->heap, (size_t)free_n * 4);
        for (uint32_t i = 0; i < free_n && !bad; i++) bad = h->heap[i] < 0 || h->heap[i] >= (int32_t)NP;
        /* every page is either free (once) or mapped, never both: a free id
         * that is also in the table, or listed twice, would let the
         * allocator hand a live page to another sequence */
        uint32_t distinct_live = 0;
        for (uint32_t p = 0; p < NP && !bad; p++) distinct_live += h->refc[p] > 0;
        for (uint32_t i = 0; i < free_n && !bad; i++) {
            const int32_t id = h->heap[i];
            bad = h->refc[id] != 0;
            h->refc[id] = UINT32_MAX;                  /* marks a free id seen */
        }
        for (uint32_t i = 0; i < free_n; i++)          /* undo the marks */
            if (h->heap[i] >= 0 && h->heap[i] < (int32_t)NP && h->refc[h->heap[i]] == UINT32_MAX) h->refc[h->heap[i]] = 0;
        bad = bad || (uint64_t)free_n + distinct_live != NP;
    }
    if (!bad) {                                        /* the free set back into rank order */
        int32_t *ids = (int32_t *)malloc((size_t)(free_n ? free_n : 1) * 4);
        bad = !ids;
        if (ids) {
            memcpy(ids, h->heap, (size_t)free_n * 4);
            heap_rebuild(h, ids, free_n);
            free(ids);
        }
        ck_read(&io, &log_n, 4);
        bad = bad || io.err;
    }
    for (uint32_t i = 0; i < log_n && !bad; i++) {
        uint32_t e[5];
        ck_read(&io, e, sizeof e);
        if (io.err) { bad = 1; break; }
        if (h->log_n == h->log_cap) {
            uint32_t cap = h->log_cap ? 2 * h->log_cap : 1024;
            ct_kv_evict_event_t *nl = (ct_kv_evict_event_t *)realloc(h->log, (size_t)cap * sizeof *nl);
            if (!nl) { bad = 1; break; }
            h->log = nl;
            h->log_cap = cap;
        }
        h->log[h->log_n++] = (ct_kv_evict_event_t){e[0], e[1], e[2], (int32_t)e[3], e[4]};
    }
    if (!bad) {
        ck_read(&io, &n_live, 4);
        bad = io.err || n_live > NP;
    }
    if (!bad && (flags & 1u) && n_live) {
        const size_t sc_bytes = h->scales ? (size_t)P * sizeof(float) : 0;
        uint8_t *buf = (uint8_t *)malloc(h->page_bytes + sc_bytes);
        bad = !buf;
        for (uint32_t i = 0; i < n_live && !bad; i++) {
            int32_t pg = -1;
            ck_read(&io, &pg, 4);
            ck_read(&io, buf, h->page_bytes + sc_bytes);
            if (io.err || pg < 0 || pg >= (int32_t)NP) { bad = 1; break; }
            if (!h->host_only) {
                bad = ct__cuda_status(cudaMemcpy((uint8_t *)h->pool + (size_t)pg * h->page_bytes, buf, h->page_bytes,
                                                 cudaMemcpyHostToDevice), "ct_kv_paged_load page") != CT_OK;
                if (!bad && sc_bytes)
                    bad = ct__cuda_status(cudaMemcpy(h->scales + (size_t)pg * P, buf + h->page_bytes, sc_bytes,
                                                     cudaMemcpyHostToDevice), "ct_kv_paged_load scales") != CT_OK;
            }
        }
        free(buf);
    }
    for (uint32_t s = 0; s < S && !bad && ver >= 2; s++) {
        uint32_t nt = 0;
        ck_read(&io, &nt, 4);
        bad = io.err || nt > h->len[s] || tok_reserve(h, s, nt) != CT_OK;
        if (!bad) {
            ck_read(&io, h->tok[s], (size_t)nt * 4);
            h->tok_n[s] = nt;
            bad = io.err;
        }
    }
    if (!bad) {
        const uint64_t want = io.fnv;
        uint64_t sum = 0;
        bad = fread(&sum, 8, 1, f) != 1 || sum != want;
        if (bad) ct__set_error("ct_kv_paged_load: checksum mismatch");
    } else {
        ct__set_error("ct_kv_paged_load: truncated or inconsistent checkpoint");
    }
    fclose(f);
    if (!bad && !h->host_only) {                       /* device mirrors of the tables */
        int32_t *len32 = (int32_t *)malloc((size_t)S * 4);
        bad = !len32;
        if (len32) {
            for (uint32_t i = 0; i < S; i++) len32[i] = (int32_t)h->len[i];
            bad = ct__cuda_status(cudaMemcpy(h->bt_dev, h->bt, (size_t)S * MP * 4, cudaMemcpyHostToDevice), "load bt") ||
                  ct__cuda_status(cudaMemcpy(h->len_dev, len32, (size_t)S * 4, cudaMemcpyHostToDevice), "load len");
            free(len32);
        }
    }
    if (bad) { ct_kv_paged_destroy(h); return NULL; }
    return h;
}
