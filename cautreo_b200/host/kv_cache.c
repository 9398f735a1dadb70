/*
 * kv_cache.c -- the reference ct_kv_* interface (src/kv_cache/kv_cache.c)
 * over device memory.
 *
 * Semantics kept from the reference, line for line in behaviour:
 *   create   defaults max_ctx 2048 / compress_ratio 1, zeroed storage (:24-40)
 *   append   false on NULL, layer >= n_layers, pos >= max_ctx; len is one
 *            counter shared by all layers (:49-61)
 *   get      false if pos >= len; reads are not counted (:63-71)
 *   reset    counters only (:76-80)
 *   save/load  raw format, load ignores the saved config, short reads leave
 *            the rest of the storage unchanged (:82-111)
 *   compress keep every step-th token, step = max(2, (u32)ratio) (:113-137)
 *   stats    bytes_used = len * L * H * D * 4 * 2 (:139-147)
 * The K and V arrays live in HBM ([layer][max_ctx][n_kv_heads*head_dim] fp32)
 * so the device kernels (ct_attn_decode_contig) read them in place.
 */
#include "../../include/hal.h"
#include "../../include/kv_cache.h"
#include "../csrc/ct_internal.h"

#include <cuda_runtime_api.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

struct ct_kv_cache {
    ct_kv_config_t cfg;
    float *k, *v;              /* device */
    uint32_t n_tokens;
    uint32_t n_compressed;
    ct_kv_stats_t stats;
};

static size_t kv_stride(const ct_kv_cache_t *c) { return (size_t)c->cfg.n_kv_heads * c->cfg.head_dim; }
static size_t kv_total(const ct_kv_cache_t *c) { return (size_t)c->cfg.n_layers * c->cfg.max_ctx * kv_stride(c); }
static size_t kv_row(const ct_kv_cache_t *c, uint32_t layer, uint32_t pos) {
    return ((size_t)layer * c->cfg.max_ctx + pos) * kv_stride(c);
}

ct_kv_cache_t *ct_kv_create(const ct_kv_config_t *cfg) {
    ct_kv_cache_t *c = (ct_kv_cache_t *)calloc(1, sizeof *c);
    if (!c) return NULL;
    if (cfg) c->cfg = *cfg;
    if (c->cfg.max_ctx == 0) c->cfg.max_ctx = 2048;
    if (c->cfg.compress_ratio == 0.0f) c->cfg.compress_ratio = 1.0f;
    size_t total = kv_total(c);
    size_t bytes = (total ? total : 1) * sizeof(float);
    if (ct__cuda_status(cudaMalloc((void **)&c->k, bytes), "ct_kv_create") ||
        ct__cuda_status(cudaMalloc((void **)&c->v, bytes), "ct_kv_create") ||
        ct__cuda_status(cudaMemset(c->k, 0, bytes), "ct_kv_create") ||
        ct__cuda_status(cudaMemset(c->v, 0, bytes), "ct_kv_create")) {
        if (c->k) cudaFree(c->k);
        if (c->v) cudaFree(c->v);
        free(c);
        return NULL;
    }
    return c;
}

void ct_kv_destroy(ct_kv_cache_t *c) {
    if (!c) return;
    cudaFree(c->k);
    cudaFree(c->v);
    free(c);
}

bool ct_kv_append(ct_kv_cache_t *c, uint32_t layer, uint32_t token_pos, const float *k, const float *v) {
    if (!c || !k || !v) return false;
    if (layer >= c->cfg.n_layers) return false;
    if (token_pos >= c->cfg.max_ctx) return false;
    size_t off = kv_row(c, layer, token_pos), bytes = kv_stride(c) * sizeof(float);
    if (ct__cuda_status(cudaMemcpy(c->k + off, k, bytes, cudaMemcpyHostToDevice), "ct_kv_append") ||
        ct__cuda_status(cudaMemcpy(c->v + off, v, bytes, cudaMemcpyHostToDevice), "ct_kv_append"))
        return false;
    if (token_pos >= c->n_tokens) c->n_tokens = token_pos + 1;
    c->stats.n_appends++;
    return true;
}

bool ct_kv_get(const ct_kv_cache_t *c, uint32_t layer, uint32_t token_pos, float *k_out, float *v_out) {
    if (!c || !k_out || !v_out) return false;
    if (layer >= c->cfg.n_layers || token_pos >= c->n_tokens) return false;
    size_t off = kv_row(c, layer, token_pos), bytes = kv_stride(c) * sizeof(float);
    if (ct__cuda_status(cudaMemcpy(k_out, c->k + off, bytes, cudaMemcpyDeviceToHost), "ct_kv_get") ||
        ct__cuda_status(cudaMemcpy(v_out, c->v + off, bytes, cudaMemcpyDeviceToHost), "ct_kv_get"))
        return false;
    return true;
}

uint32_t ct_kv_len(const ct_kv_cache_t *c) { return c ? c->n_tokens : 0; }
uint32_t ct_kv_capacity(const ct_kv_cache_t *c) { return c ? c->cfg.max_ctx : 0; }

void ct_kv_reset(ct_kv_cache_t *c) {
    if (!c) return;
    c->n_tokens = 0;
    c->n_compressed = 0;
}

bool ct_kv_save(const ct_kv_cache_t *c, const char *path) {
    if (!c || !path) return false;
    size_t total = kv_total(c);
    float *h = (float *)malloc((total ? total : 1) * sizeof(float));
    if (!h) return false;
    FILE *f = fopen(path, "wb");
    if (!f) { free(h); return false; }
    bool ok = true;
    fwrite(&c->cfg, sizeof c->cfg, 1, f);
    fwrite(&c->n_tokens, sizeof(uint32_t), 1, f);
    fwrite(&c->n_compressed, sizeof(uint32_t), 1, f);
    if (ct__cuda_status(cudaMemcpy(h, c->k, total * sizeof(float), cudaMemcpyDeviceToHost), "ct_kv_save")) ok = false;
    else fwrite(h, sizeof(float), total, f);
    if (ok && ct__cuda_status(cudaMemcpy(h, c->v, total * sizeof(float), cudaMemcpyDeviceToHost), "ct_kv_save")) ok = false;
    else if (ok) fwrite(h, sizeof(float), total, f);
    fclose(f);
    free(h);
    return ok;
}

bool ct_kv_load(ct_kv_cache_t *c, const char *path) {
    if (!c || !path) return false;
    FILE *f = fopen(path, "rb");
    if (!f) return false;
    ct_kv_config_t cfg;
    if (fread(&cfg, sizeof cfg, 1, f) != 1) { fclose(f); return false; }
    if (fread(&c->n_tokens, sizeof(uint32_t), 1, f) != 1) { fclose(f); return false; }
    if (fread(&c->n_compressed, sizeof(uint32_t), 1, f) != 1) { fclose(f); return false; }
    size_t total = kv_total(c);
    float *h = (float *)malloc((total ? total : 1) * sizeof(float));
    bool ok = h != NULL;
    /* Start from the current contents so a short file leaves the tail as it
     * was, as the reference's unchecked fread does. */
    for (int arr = 0; ok && arr < 2; arr++) {
        float *dev = arr == 0 ? c->k : c->v;
        if (ct__cuda_status(cudaMemcpy(h, dev, total * sizeof(float), cudaMemcpyDeviceToHost), "ct_kv_load")) { ok = false; break; }
        size_t got = fread(h, sizeof(float), total, f);
        (void)got;
        if (ct__cuda_status(cudaMemcpy(dev, h, total * sizeof(float), cudaMemcpyHostToDevice), "ct_kv_load")) ok = false;
    }
    free(h);
    fclose(f);
    return ok;
}

bool ct_kv_compress(ct_kv_cache_t *c, float ratio) {
    if (!c || ratio <= 1.0f) return false;
    uint32_t step = (uint32_t)ratio;
    if (step < 2) step = 2;
    if (c->n_tokens < 2) return false;
    uint32_t new_len = (c->n_tokens + step - 1) / step;
    size_t bytes = 2 * (size_t)c->cfg.n_layers * new_len * kv_stride(c) * sizeof(float);
    float *scratch = NULL;
    if (ct__cuda_status(cudaMalloc((void **)&scratch, bytes ? bytes : 16), "ct_kv_compress")) return false;
    int rc = ct__launch_kv_compress(c->k, c->v, scratch, c->cfg.n_layers, c->cfg.max_ctx, (uint32_t)kv_stride(c),
                                    new_len, step, NULL);
    if (rc == CT_OK) rc = ct__cuda_status(cudaDeviceSynchronize(), "ct_kv_compress");
    cudaFree(scratch);
    if (rc != CT_OK) return false;
    c->n_compressed += c->n_tokens - new_len;
    c->n_tokens = new_len;
    return true;
}

ct_kv_stats_t ct_kv_stats(const ct_kv_cache_t *c) {
    ct_kv_stats_t s;
    memset(&s, 0, sizeof s);
    if (!c) return s;
    s.n_appends = c->stats.n_appends;
    s.n_reads = c->stats.n_reads;
    s.n_tokens = c->n_tokens;
    s.bytes_used = (uint64_t)c->n_tokens * c->cfg.n_layers * kv_stride(c) * sizeof(float) * 2;
    return s;
}

float *ct_kv_device_k(ct_kv_cache_t *c) { return c ? c->k : NULL; }
float *ct_kv_device_v(ct_kv_cache_t *c) { return c ? c->v : NULL; }
