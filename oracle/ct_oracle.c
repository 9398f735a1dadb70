/*
 * ct_oracle.c -- CPU oracle (test infrastructure only; see ct_oracle.h).
 *
 * Numerics follow the reference's own CPU code: fp64 dot and PV
 * accumulation, fp32 scores and expf, a double softmax sum and an fp32
 * divide (src/attention/attention.c:11-53); Q8_0 block rounding
 * floorf(x*id + 0.5f) with a truncating fp16 scale (src/quant/quant.c:16-111).
 * Compiled with -std=c11 -ffp-contract=off so no product is fused into an FMA.
 */
#include "ct_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* SplitMix64 (Steele, Lea, Flood 2014): the i-th output of a generator      */
/* seeded with `key` is mix64(key + (i + 1) * golden).  Counter based, so    */
/* any element of a stream can be produced independently (CPU or GPU).       */
/* ------------------------------------------------------------------------ */
#define ORC_GOLDEN 0x9E3779B97F4A7C15ull

uint64_t orc_mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t orc_key(uint64_t seed, uint64_t stream) {
    return orc_mix64(seed * ORC_GOLDEN + orc_mix64(stream + 0x632BE59BD9B4E019ull));
}

uint64_t orc_u64(uint64_t key, uint64_t i) { return orc_mix64(key + (i + 1) * ORC_GOLDEN); }

double orc_unit(uint64_t key, uint64_t i) {
    return (double)(orc_u64(key, i) >> 11) * (1.0 / 9007199254740992.0);
}

/* Box-Muller (1958), cosine branch only: element i uses draws 2i and 2i+1. */
float orc_normal(uint64_t key, uint64_t i) {
    double u1 = 1.0 - orc_unit(key, 2 * i);          /* (0, 1] */
    double u2 = orc_unit(key, 2 * i + 1);            /* [0, 1) */
    double r = sqrt(-2.0 * log(u1));
    return (float)(r * cos(6.283185307179586 * u2));
}

int orc_outlier(uint64_t key, uint64_t i, uint32_t outlier_bp) {
    if (outlier_bp == 0) return 0;
    uint64_t okey = orc_mix64(key ^ 0xA0761D6478BD642Full);
    return (orc_u64(okey, i) % 10000u) < outlier_bp;
}

void orc_fill_normal_f32(uint64_t key, uint64_t start, uint64_t n, uint32_t outlier_bp,
                         float outlier_mul, float *out) {
    #pragma omp parallel for schedule(static)
    for (int64_t j = 0; j < (int64_t)n; j++) {
        float x = orc_normal(key, start + (uint64_t)j);
        if (orc_outlier(key, start + (uint64_t)j, outlier_bp)) x *= outlier_mul;
        out[j] = x;
    }
}

void orc_fill_normal_bf16(uint64_t key, uint64_t start, uint64_t n, uint32_t outlier_bp,
                          float outlier_mul, uint16_t *out) {
    #pragma omp parallel for schedule(static)
    for (int64_t j = 0; j < (int64_t)n; j++) {
        float x = orc_normal(key, start + (uint64_t)j);
        if (orc_outlier(key, start + (uint64_t)j, outlier_bp)) x *= outlier_mul;
        out[j] = orc_f32_to_bf16(x);
    }
}

/* Fisher-Yates, drawing j uniformly in [0, i] from the stream. */
void orc_permutation(uint64_t key, uint32_t n, int32_t *perm) {
    for (uint32_t i = 0; i < n; i++) perm[i] = (int32_t)i;
    for (uint32_t i = n; i-- > 1;) {
        uint32_t j = (uint32_t)(orc_u64(key, i) % (uint64_t)(i + 1));
        int32_t t = perm[i]; perm[i] = perm[j]; perm[j] = t;
    }
}

/* len = floor(lo * (hi/lo)^u), u uniform in [0,1), clamped to [lo, hi]. */
void orc_lengths_loguniform(uint64_t key, uint32_t n, uint32_t lo, uint32_t hi, uint32_t *len) {
    double lr = log((double)hi / (double)lo);
    for (uint32_t s = 0; s < n; s++) {
        double t = floor((double)lo * exp(orc_unit(key, s) * lr));
        if (t < lo) t = lo;
        if (t > hi) t = hi;
        len[s] = (uint32_t)t;
    }
}

/* ------------------------------------------------------------------------ */
/* Scalar conversions                                                        */
/* ------------------------------------------------------------------------ */

/* bf16: top 16 bits; from fp32 by round-to-nearest-even on the dropped half
 * (ds4_forward.c:52-66 does the same, with no NaN special case). */
uint16_t orc_f32_to_bf16(float f) {
    uint32_t u; memcpy(&u, &f, 4);
    uint32_t bias = 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)((u + bias) >> 16);
}

float orc_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16; float f; memcpy(&f, &u, 4); return f;
}

/* The reference's fp16 encoder (quant.c:16-45), quirks included: the
 * mantissa is truncated, not rounded; the rebased exponent is held in an
 * unsigned int, so a biased fp32 exponent below 112 wraps round and lands in
 * the overflow branch (+/-Inf); exponent 112 becomes a subnormal. */
uint16_t orc_ct_f32_to_fp16(float f) {
    uint32_t u; memcpy(&u, &f, 4);
    uint32_t sgn = (u >> 31) & 1u, e = (u >> 23) & 0xFFu, m = u & 0x7FFFFFu;
    if (e == 0) return (uint16_t)(sgn << 15);
    if (e == 0xFF) return (uint16_t)((sgn << 15) | 0x7C00u | (m >> 13));
    uint32_t ne = e - 112u;                       /* unsigned on purpose */
    if (ne >= 31u) return (uint16_t)((sgn << 15) | 0x7C00u);
    if (ne == 0u) return (uint16_t)((sgn << 15) | (((m | 0x800000u) >> 1) >> 13));
    return (uint16_t)((sgn << 15) | (ne << 10) | (m >> 13));
}

float orc_ct_fp16_to_f32(uint16_t h) {
    uint32_t sgn = (h >> 15) & 1u, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, u;
    if (e == 0) {
        if (m == 0) u = sgn << 31;
        else {
            /* The reference normalises with a start exponent of 112 and one
             * decrement per shift (quant.c:57-63), which yields half the true
             * subnormal value m*2^-24.  Kept as is: decode must match it. */
            uint32_t ex = 112u;
            while (!(m & 0x400u)) { m <<= 1; ex--; }
            u = (sgn << 31) | (ex << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (e == 31) {
        u = (sgn << 31) | 0x7F800000u | (m << 13);
    } else {
        u = (sgn << 31) | ((e + 112u) << 23) | (m << 13);
    }
    float f; memcpy(&f, &u, 4); return f;
}

/* OCP 8-bit floating point E4M3 (bias 7, no infinities, S.1111.111 = NaN,
 * largest finite 448), round-to-nearest-even, saturating to +/-448. */
uint8_t orc_f32_to_e4m3_satfinite(float f) {
    uint32_t u; memcpy(&u, &f, 4);
    uint8_t sgn = (uint8_t)((u >> 24) & 0x80u);
    float a = fabsf(f);
    if (isnan(f)) return (uint8_t)(sgn | 0x7F);
    if (a >= 448.0f) return (uint8_t)(sgn | 0x7E);
    if (a < 0.015625f) {                          /* below 2^-6: subnormal grid m*2^-9 */
        float q = nearbyintf(a * 512.0f);         /* exact scale, RNE (default mode) */
        return (uint8_t)(sgn | (uint8_t)q);       /* q == 8 encodes 2^-6 exactly */
    }
    int e; (void)frexpf(a, &e); e -= 1;          /* a in [2^e, 2^(e+1)), e in [-6, 8] */
    float q = nearbyintf(ldexpf(a, 3 - e));      /* [8, 16] */
    if (q >= 16.0f) { q = 8.0f; e += 1; }
    uint32_t code = ((uint32_t)(e + 7) << 3) | ((uint32_t)q - 8u);
    if (code > 0x7Eu) code = 0x7Eu;
    return (uint8_t)(sgn | code);
}

float orc_e4m3_to_f32(uint8_t v) {
    uint32_t e = (v >> 3) & 0xFu, m = v & 7u;
    float r;
    if (e == 15 && m == 7) r = NAN;
    else if (e == 0) r = ldexpf((float)m, -9);
    else r = ldexpf((float)(8u + m), (int)e - 10);
    return (v & 0x80u) ? -r : r;
}

/* ------------------------------------------------------------------------ */
/* Codecs                                                                     */
/* ------------------------------------------------------------------------ */

/* Q8_0 (quant.c:77-111): per 32-value block, d = amax/127 stored as the
 * truncating fp16 above; codes use the fp32 d; decode uses the fp16 d. */
void orc_q8_0_quantize(const float *src, uint8_t *dst, int64_t n) {
    for (int64_t b = 0; b < n / 32; b++) {
        const float *x = src + b * 32;
        uint8_t *blk = dst + b * 34;
        float amax = 0.0f;
        for (int i = 0; i < 32; i++) { float a = fabsf(x[i]); if (a > amax) amax = a; }
        float d = amax / 127.0f;
        uint16_t h = orc_ct_f32_to_fp16(d);
        memcpy(blk, &h, 2);
        float id = d > 0 ? 1.0f / d : 0.0f;
        for (int i = 0; i < 32; i++) {
            int q = (int)floorf(x[i] * id + 0.5f);
            if (q > 127) q = 127;
            if (q < -127) q = -127;
            blk[2 + i] = (uint8_t)(int8_t)q;
        }
    }
}

void orc_q8_0_dequantize(const uint8_t *src, float *dst, int64_t n) {
    for (int64_t b = 0; b < n / 32; b++) {
        uint16_t h; memcpy(&h, src + b * 34, 2);
        float d = orc_ct_fp16_to_f32(h);
        for (int i = 0; i < 32; i++) dst[b * 32 + i] = (float)(int8_t)src[b * 34 + 2 + i] * d;
    }
}

/* Per-token int8: one fp32 scale d = amax/127 per token, codes rounded as in
 * Q8_0 (floor(x*id + 0.5), clamp +/-127), decode q*d. */
void orc_kv_quant_int8(const float *x, uint32_t n_tok, uint32_t dim, int8_t *codes, float *scales) {
    for (uint32_t t = 0; t < n_tok; t++) {
        const float *xt = x + (size_t)t * dim;
        float amax = 0.0f;
        for (uint32_t i = 0; i < dim; i++) { float a = fabsf(xt[i]); if (a > amax) amax = a; }
        float d = amax / 127.0f;
        float id = d > 0 ? 1.0f / d : 0.0f;
        for (uint32_t i = 0; i < dim; i++) {
            int q = (int)floorf(xt[i] * id + 0.5f);
            if (q > 127) q = 127;
            if (q < -127) q = -127;
            codes[(size_t)t * dim + i] = (int8_t)q;
        }
        scales[t] = d;
    }
}

void orc_kv_dequant_int8(const int8_t *codes, const float *scales, uint32_t n_tok, uint32_t dim, float *x) {
    for (uint32_t t = 0; t < n_tok; t++)
        for (uint32_t i = 0; i < dim; i++)
            x[(size_t)t * dim + i] = (float)codes[(size_t)t * dim + i] * scales[t];
}

/* Per-token e4m3: d = amax/448, code = e4m3_rn_satfinite(x * (1/d)). */
void orc_kv_quant_e4m3(const float *x, uint32_t n_tok, uint32_t dim, uint8_t *codes, float *scales) {
    for (uint32_t t = 0; t < n_tok; t++) {
        const float *xt = x + (size_t)t * dim;
        float amax = 0.0f;
        for (uint32_t i = 0; i < dim; i++) { float a = fabsf(xt[i]); if (a > amax) amax = a; }
        float d = amax / 448.0f;
        float id = d > 0 ? 1.0f / d : 0.0f;
        for (uint32_t i = 0; i < dim; i++) codes[(size_t)t * dim + i] = orc_f32_to_e4m3_satfinite(xt[i] * id);
        scales[t] = d;
    }
}

void orc_kv_dequant_e4m3(const uint8_t *codes, const float *scales, uint32_t n_tok, uint32_t dim, float *x) {
    for (uint32_t t = 0; t < n_tok; t++)
        for (uint32_t i = 0; i < dim; i++)
            x[(size_t)t * dim + i] = orc_e4m3_to_f32(codes[(size_t)t * dim + i]) * scales[t];
}

/* ------------------------------------------------------------------------ */
/* Attention (attention.c:11-53 numerics)                                    */
/* ------------------------------------------------------------------------ */

void orc_attn_softmax(float *x, uint32_t n) {
    if (!x || n == 0) return;
    float mx = x[0];
    for (uint32_t i = 1; i < n; i++) if (x[i] > mx) mx = x[i];
    double sum = 0.0;
    for (uint32_t i = 0; i < n; i++) { x[i] = expf(x[i] - mx); sum += x[i]; }
    if (sum > 0) for (uint32_t i = 0; i < n; i++) x[i] = (float)(x[i] / sum);
}

int orc_mla_decode(const float *q, const float *kv, uint32_t n, uint32_t H, uint32_t E,
                   uint32_t Dv, float scale, float *out) {
    if (!q || !kv || !out || n == 0 || Dv > E) return -1;
    float *p = (float *)malloc((size_t)n * sizeof(float));
    if (!p) return -1;
    for (uint32_t h = 0; h < H; h++) {
        const float *qh = q + (size_t)h * E;
        for (uint32_t t = 0; t < n; t++) {
            const float *kt = kv + (size_t)t * E;
            double dot = 0.0;
            for (uint32_t i = 0; i < E; i++) dot += (double)qh[i] * (double)kt[i];
            p[t] = scale * (float)dot;
        }
        orc_attn_softmax(p, n);
        for (uint32_t i = 0; i < Dv; i++) {
            double acc = 0.0;
            for (uint32_t t = 0; t < n; t++) acc += (double)p[t] * (double)kv[(size_t)t * E + i];
            out[(size_t)h * Dv + i] = (float)acc;
        }
    }
    free(p);
    return 0;
}

/* Same contract as the reference ct_attn_forward: every head reads the same
 * [n][head_dim] K and V (attention.c:37,47), scale 0 means 1/sqrt(head_dim). */
int orc_attn_forward(const float *q, const float *k, const float *v, uint32_t n_tokens,
                     uint32_t n_heads, uint32_t head_dim, float scale, float *out) {
    if (!q || !k || !v || !out || n_tokens == 0) return -1;
    if (scale == 0.0f) scale = 1.0f / sqrtf((float)head_dim);
    float *p = (float *)malloc((size_t)n_tokens * sizeof(float));
    if (!p) return -1;
    for (uint32_t h = 0; h < n_heads; h++) {
        const float *qh = q + (size_t)h * head_dim;
        for (uint32_t t = 0; t < n_tokens; t++) {
            double dot = 0.0;
            for (uint32_t i = 0; i < head_dim; i++) dot += (double)qh[i] * (double)k[(size_t)t * head_dim + i];
            p[t] = scale * (float)dot;
        }
        orc_attn_softmax(p, n_tokens);
        for (uint32_t i = 0; i < head_dim; i++) {
            double acc = 0.0;
            for (uint32_t t = 0; t < n_tokens; t++) acc += (double)p[t] * (double)v[(size_t)t * head_dim + i];
            out[(size_t)h * head_dim + i] = (float)acc;
        }
    }
    free(p);
    return 0;
}

int orc_paged_gather_bf16_f32(const uint16_t *pool, const int32_t *bt_row, uint32_t n,
                              uint32_t page_tokens, uint32_t E, float *out) {
    for (uint32_t t = 0; t < n; t++) {
        int32_t pg = bt_row[t / page_tokens];
        if (pg < 0) return -1;
        const uint16_t *src = pool + ((size_t)pg * page_tokens + t % page_tokens) * E;
        for (uint32_t i = 0; i < E; i++) out[(size_t)t * E + i] = orc_bf16_to_f32(src[i]);
    }
    return 0;
}

/* Attention reads the tokens t < len whose page is mapped; evicted pages
 * (block-table entry < 0) drop out of the softmax.  A sequence with no
 * readable token gets a zero output. */
int orc_mla_decode_paged_bf16(const uint16_t *pool, const int32_t *bt, uint32_t max_pages,
                              const int32_t *seq_lens, uint32_t n_seq, const uint16_t *q,
                              uint32_t H, uint32_t E, uint32_t Dv, uint32_t page_tokens,
                              float scale, int n_threads, float *out) {
    int bad = 0;
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#else
    (void)n_threads;
#endif
    #pragma omp parallel for schedule(dynamic, 1) reduction(|:bad)
    for (int64_t s = 0; s < (int64_t)n_seq; s++) {
        uint32_t n = (uint32_t)seq_lens[s];
        float *kv = (float *)malloc((size_t)(n ? n : 1) * E * sizeof(float));
        float *qf = (float *)malloc((size_t)H * E * sizeof(float));
        if (!kv || !qf) { bad |= 1; free(kv); free(qf); continue; }
        for (size_t i = 0; i < (size_t)H * E; i++) qf[i] = orc_bf16_to_f32(q[(size_t)s * H * E + i]);
        uint32_t m = 0;                      /* readable tokens, gathered in order */
        const int32_t *row = bt + (size_t)s * max_pages;
        for (uint32_t t = 0; t < n; t++) {
            int32_t pg = row[t / page_tokens];
            if (pg < 0) continue;
            const uint16_t *src = pool + ((size_t)pg * page_tokens + t % page_tokens) * E;
            for (uint32_t i = 0; i < E; i++) kv[(size_t)m * E + i] = orc_bf16_to_f32(src[i]);
            m++;
        }
        if (m == 0) memset(out + (size_t)s * H * Dv, 0, (size_t)H * Dv * sizeof(float));
        else if (orc_mla_decode(qf, kv, m, H, E, Dv, scale, out + (size_t)s * H * Dv) != 0) bad |= 1;
        free(kv); free(qf);
    }
    return bad ? -1 : 0;
}

/* ------------------------------------------------------------------------ */
/* ct_kv_compress semantics (kv_cache.c:113-137): keep tokens t = 0, step,   */
/* 2*step, ... with step = max(2, (uint32)ratio), moved down in every layer.  */
/* ------------------------------------------------------------------------ */
uint32_t orc_kv_compress_every_kth(float *k, float *v, uint32_t n_layers, uint32_t max_ctx,
                                   uint32_t stride, uint32_t n_tokens, float ratio) {
    uint32_t step = (uint32_t)ratio;
    if (step < 2) step = 2;
    uint32_t kept = 0;
    for (uint32_t t = 0; t < n_tokens; t += step, kept++) {
        if (t == kept) continue;
        for (uint32_t l = 0; l < n_layers; l++) {
            size_t base = (size_t)l * max_ctx * stride;
            memmove(k + base + (size_t)kept * stride, k + base + (size_t)t * stride, stride * sizeof(float));
            memmove(v + base + (size_t)kept * stride, v + base + (size_t)t * stride, stride * sizeof(float));
        }
    }
    return kept;
}

/* ------------------------------------------------------------------------ */
/* Paged allocator replay                                                     */
/* ------------------------------------------------------------------------ */

/* Binary min-heap of free physical page ids: "pop" always yields the lowest. */
typedef struct { int32_t *a; uint32_t n; } orc_heap_t;

static void heap_push(orc_heap_t *h, int32_t v) {
    uint32_t i = h->n++;
    h->a[i] = v;
    while (i > 0) {
        uint32_t p = (i - 1) / 2;
        if (h->a[p] <= h->a[i]) break;
        int32_t t = h->a[p]; h->a[p] = h->a[i]; h->a[i] = t; i = p;
    }
}

static int32_t heap_pop(orc_heap_t *h) {
    int32_t top = h->a[0];
    h->a[0] = h->a[--h->n];
    uint32_t i = 0;
    for (;;) {
        uint32_t l = 2 * i + 1, r = l + 1, m = i;
        if (l < h->n && h->a[l] < h->a[m]) m = l;
        if (r < h->n && h->a[r] < h->a[m]) m = r;
        if (m == i) break;
        int32_t t = h->a[m]; h->a[m] = h->a[i]; h->a[i] = t; i = m;
    }
    return top;
}

/*
 * Event order, per append of token r of sequence s (rounds ascending, and
 * sequences in id order inside a round):
 *   1. r % P == 0 opens logical page r/P.  If no page is free, one LRU victim
 *      is evicted first: among every sequence's lowest mapped page, those
 *      that are full (all P slots written) compete on
 *      (last_access[owner], owner); the lower sequence id wins a tie, as the
 *      first (lowest) index wins in the reference's LRU (streaming.c:86-96).
 *      Then the lowest free id is taken.
 *   2. The token is written to slot r % P of that page.
 *   3. last_access[s] = r  (a decode step reads every live page of s).
 *   4. Sliding window W: every mapped page lying wholly below len - W
 *      (len = r + 1) is freed.
 * A sequence's mapped pages always form one contiguous run [lo, hi) of
 * logical pages (new pages open at hi, the window and LRU take from lo), so
 * its lowest mapped page is lo and only that page can be its LRU victim.
 */
int orc_alloc_replay(const orc_alloc_cfg_t *cfg, const uint32_t *len, int32_t *bt,
                     uint64_t *slot_owner, orc_evict_event_t *events, uint32_t max_events,
                     uint32_t *n_events, uint32_t *last_access, uint32_t *n_free_out) {
    const uint32_t S = cfg->n_seqs, P = cfg->page_tokens, NP = cfg->n_pages, MP = cfg->max_pages_per_seq;
    const uint32_t W = cfg->window_tokens;
    int rc = 0;
    uint32_t *lo = (uint32_t *)calloc(S, sizeof(uint32_t));
    uint32_t *hi = (uint32_t *)calloc(S, sizeof(uint32_t));
    uint32_t *cur = (uint32_t *)calloc(S, sizeof(uint32_t));   /* tokens written so far */
    orc_heap_t heap = { (int32_t *)malloc((size_t)NP * sizeof(int32_t)), 0 };
    if (!lo || !hi || !cur || !heap.a) { rc = -1; goto done; }
    for (size_t i = 0; i < (size_t)S * MP; i++) bt[i] = -1;
    for (size_t i = 0; i < (size_t)NP * P; i++) slot_owner[i] = ~0ull;
    for (uint32_t s = 0; s < S; s++) last_access[s] = 0;
    for (uint32_t p = 0; p < NP; p++) heap_push(&heap, (int32_t)p);
    *n_events = 0;
    uint32_t max_len = 0;
    for (uint32_t s = 0; s < S; s++) if (len[s] > max_len) max_len = len[s];

    for (uint32_t r = 0; r < max_len && rc == 0; r++) {
        for (uint32_t s = 0; s < S; s++) {
            if (r >= len[s]) continue;
            uint32_t lp = r / P;
            if (r % P == 0) {
                if (lp >= MP) { rc = -1; break; }
                if (heap.n == 0) {
                    int64_t best = -1;
                    for (uint32_t c = 0; c < S; c++) {
                        if (lo[c] >= hi[c]) continue;
                        if ((uint64_t)(lo[c] + 1) * P > cur[c]) continue;     /* not full */
                        if (best < 0 || last_access[c] < last_access[best]) best = c;
                    }
                    if (best < 0) { rc = -2; break; }
                    uint32_t c = (uint32_t)best;
                    int32_t ph = bt[(size_t)c * MP + lo[c]];
                    if (*n_events >= max_events) { rc = -1; break; }
                    events[(*n_events)++] = (orc_evict_event_t){ r, c, lo[c], ph, 2u };
                    bt[(size_t)c * MP + lo[c]] = -1;
                    lo[c]++;
                    heap_push(&heap, ph);
                }
                int32_t ph = heap_pop(&heap);
                bt[(size_t)s * MP + lp] = ph;
                if (lo[s] == hi[s]) lo[s] = lp;
                hi[s] = lp + 1;
            }
            int32_t ph = bt[(size_t)s * MP + lp];
            slot_owner[(size_t)ph * P + r % P] = ((uint64_t)s << 32) | r;
            cur[s] = r + 1;
            last_access[s] = r;
            if (W > 0 && r + 1 > W) {
                uint32_t below = r + 1 - W;          /* tokens [0, below) are outside */
                while (lo[s] < hi[s] && (lo[s] + 1) * P <= below) {
                    int32_t fp = bt[(size_t)s * MP + lo[s]];
                    if (*n_events >= max_events) { rc = -1; break; }
                    events[(*n_events)++] = (orc_evict_event_t){ r, s, lo[s], fp, 1u };
                    bt[(size_t)s * MP + lo[s]] = -1;
                    lo[s]++;
                    heap_push(&heap, fp);
                }
                if (rc) break;
            }
        }
    }
    if (n_free_out) *n_free_out = heap.n;
done:
    free(lo); free(hi); free(cur); free(heap.a);
    return rc;
}

uint32_t orc_compact_plan(int32_t *bt, uint32_t n_seqs, uint32_t max_pages_per_seq,
                          int32_t *map_new_to_old) {
    uint32_t n = 0;
    for (uint32_t s = 0; s < n_seqs; s++)
        for (uint32_t lp = 0; lp < max_pages_per_seq; lp++) {
            int32_t *e = bt + (size_t)s * max_pages_per_seq + lp;
            if (*e < 0) continue;
            map_new_to_old[n] = *e;
            *e = (int32_t)n++;
        }
    return n;
}

/* ------------------------------------------------------------------------ */
/* LPT sharding                                                               */
/* ------------------------------------------------------------------------ */
static const uint32_t *g_lpt_len;
static int lpt_cmp(const void *a, const void *b) {
    uint32_t x = *(const uint32_t *)a, y = *(const uint32_t *)b;
    if (g_lpt_len[x] != g_lpt_len[y]) return g_lpt_len[x] > g_lpt_len[y] ? -1 : 1;
    return x < y ? -1 : (x > y);
}

void orc_lpt_assign(const uint32_t *len, uint32_t n, uint32_t n_ranks, int32_t *rank_of) {
    uint32_t *idx = (uint32_t *)malloc((size_t)n * sizeof(uint32_t));
    uint64_t *load = (uint64_t *)calloc(n_ranks, sizeof(uint64_t));
    for (uint32_t i = 0; i < n; i++) idx[i] = i;
    g_lpt_len = len;
    qsort(idx, n, sizeof(uint32_t), lpt_cmp);
    for (uint32_t k = 0; k < n; k++) {
        uint32_t best = 0;
        for (uint32_t r = 1; r < n_ranks; r++) if (load[r] < load[best]) best = r;
        rank_of[idx[k]] = (int32_t)best;
        load[best] += len[idx[k]];
    }
    free(idx); free(load);
}
