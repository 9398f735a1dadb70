/*
 * ds4.c -- the MLA-lite latent cache of ds4_forward.c on the device, with the
 * per-layer call shape of the reference engine (host buffers in and out).
 *
 * ds4_forward.c:1565-1570 stores kv_a (kv_dim fp32 values) in the layer's
 * cache slot `pos` when pos < ctx; :1572-1627 scores the q_b[0:kv_dim] query
 * against every cached position p < min(pos + 1, ctx) with scale
 * 1/sqrt(kv_dim), takes a softmax, and sums the cached latents (V = the
 * latent).  Here the layers' caches are the rows of one paged fp32 cache
 * (ct_kv_paged_t, 64-token pages) and the attention is the MLA decode with
 * one head (ct_attn_mla_decode_paged_noalloc), so a call costs three small
 * copies, an append and one decode.
 */
#include "../../include/attention.h"
#include "../../include/hal.h"
#include "../../include/kv_cache.h"
#include "../csrc/ct_internal.h"

#include <cuda_runtime_api.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

struct ct_ds4_cache {
    ct_kv_paged_t *kv;
    uint32_t n_layers, ctx, dim, max_pages;
    int device;
    cudaStream_t stream;
    float *e_dev;            /* kv_a staged on the device */
    uint16_t *q_dev, *o_dev; /* bf16 query and output */
    int32_t *i_dev;          /* [0] slot, [1] attended length */
    float *e_host;           /* pinned staging */
    uint16_t *q_host, *o_host;
    int32_t *i_host;
};

void ct_ds4_cache_destroy(ct_ds4_cache_t *c) {
    if (!c) return;
    if (c->stream) cudaStreamSynchronize(c->stream);
    ct_kv_paged_destroy(c->kv);
    cudaFree(c->e_dev); cudaFree(c->q_dev); cudaFree(c->o_dev); cudaFree(c->i_dev);
    cudaFreeHost(c->e_host); cudaFreeHost(c->q_host); cudaFreeHost(c->o_host); cudaFreeHost(c->i_host);
    if (c->stream) cudaStreamDestroy(c->stream);
    free(c);
}

ct_ds4_cache_t *ct_ds4_cache_create(uint32_t n_layers, uint32_t ctx, uint32_t kv_dim, int device) {
    if (n_layers == 0 || ctx == 0 || kv_dim == 0 || kv_dim % 16 != 0) {
        ct__set_error("ct_ds4_cache_create: bad shape");
        return NULL;
    }
    ct_ds4_cache_t *c = (ct_ds4_cache_t *)calloc(1, sizeof *c);
    if (!c) return NULL;
    c->n_layers = n_layers;
    c->ctx = ctx;
    c->dim = kv_dim;
    c->device = device;
    c->max_pages = (ctx + 63) / 64;
    int rc = ct__cuda_status(cudaSetDevice(device), "ct_ds4_cache_create");
    if (!rc) rc = ct__cuda_status(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "ds4 stream");
    if (!rc) {
        const ct_kv_paged_config_t cfg = {n_layers, c->max_pages, n_layers * c->max_pages, 64, kv_dim, 0,
                                          CT_KV_F32, device};
        c->kv = ct_kv_paged_create(&cfg);
        if (!c->kv) rc = CT_ERR_CUDA;
        else rc = ct_kv_paged_set_stream(c->kv, c->stream);
    }
    if (!rc) rc = ct__cuda_status(cudaMalloc((void **)&c->e_dev, kv_dim * sizeof(float)), "ds4 staging");
    if (!rc) rc = ct__cuda_status(cudaMalloc((void **)&c->q_dev, kv_dim * sizeof(uint16_t)), "ds4 staging");
    if (!rc) rc = ct__cuda_status(cudaMalloc((void **)&c->o_dev, kv_dim * sizeof(uint16_t)), "ds4 staging");
    if (!rc) rc = ct__cuda_status(cudaMalloc((void **)&c->i_dev, 2 * sizeof(int32_t)), "ds4 staging");
    if (!rc) rc = ct__cuda_status(cudaMallocHost((void **)&c->e_host, kv_dim * sizeof(float)), "ds4 staging");
    if (!rc) rc = ct__cuda_status(cudaMallocHost((void **)&c->q_host, kv_dim * sizeof(uint16_t)), "ds4 staging");
    if (!rc) rc = ct__cuda_status(cudaMallocHost((void **)&c->o_host, kv_dim * sizeof(uint16_t)), "ds4 staging");
    if (!rc) rc = ct__cuda_status(cudaMallocHost((void **)&c->i_host, 2 * sizeof(int32_t)), "ds4 staging");
    if (rc) { ct_ds4_cache_destroy(c); return NULL; }
    return c;
}

uint32_t ct_ds4_cache_len(const ct_ds4_cache_t *c, uint32_t layer) {
    if (!c || layer >= c->n_layers) return 0;
    uint32_t *lens = (uint32_t *)malloc(c->n_layers * sizeof(uint32_t));
    if (!lens) return 0;
    uint32_t n = ct_kv_paged_seq_lens(c->kv, lens) == CT_OK ? lens[layer] : 0;
    free(lens);
    return n;
}

int ct_ds4_attend(ct_ds4_cache_t *c, uint32_t layer, uint32_t pos, const float *kv_a, const float *q,
                  float *out) {
    if (!c || !q || !out || layer >= c->n_layers) return CT_ERR_ARG;
    const uint32_t D = c->dim, P = 64;
    uint32_t *lens = (uint32_t *)malloc(c->n_layers * sizeof(uint32_t));
    if (!lens) return CT_ERR_NOMEM;
    int rc = ct_kv_paged_seq_lens(c->kv, lens);
    const uint32_t len = lens[layer];
    free(lens);
    if (rc) return rc;
    /* the store of ds4_forward.c:1567-1570 */
    if (pos < c->ctx) {
        if (!kv_a) return CT_ERR_ARG;
        if (pos > len) {
            ct__set_error("ct_ds4_attend: positions are stored in order (pos > cached length)");
            return CT_ERR_ARG;
        }
        memcpy(c->e_host, kv_a, D * sizeof(float));
        rc = ct__cuda_status(cudaMemcpyAsync(c->e_dev, c->e_host, D * sizeof(float), cudaMemcpyHostToDevice,
                                             c->stream), "ds4 kv_a");
        if (!rc && pos == len) {
            rc = ct_kv_paged_append(c->kv, &layer, (const uint32_t[]){1u}, 1, c->e_dev, CT_KV_F32);
        } else if (!rc) {                      /* a position stored before: overwrite its slot */
            int32_t *bt = (int32_t *)malloc((size_t)c->n_layers * c->max_pages * sizeof(int32_t));
            if (!bt) return CT_ERR_NOMEM;
            rc = ct_kv_paged_block_table(c->kv, bt);
            const int32_t pg = bt[(size_t)layer * c->max_pages + pos / P];
            free(bt);
            if (!rc) {
                c->i_host[0] = pg * (int32_t)P + (int32_t)(pos % P);
                rc = ct__cuda_status(cudaMemcpyAsync(c->i_dev, c->i_host, sizeof(int32_t), cudaMemcpyHostToDevice,
                                                     c->stream), "ds4 slot");
                if (!rc) rc = ct_kv_paged_write_slots(ct_kv_paged_pool(c->kv), NULL, CT_KV_F32, c->e_dev, CT_KV_F32,
                                                      c->i_dev, 1, D, c->stream);
            }
        }
        if (rc) return rc;
    }
    /* the attention of ds4_forward.c:1572-1627 over min(pos + 1, ctx) positions */
    const uint32_t n_pos = pos < c->ctx ? pos + 1 : c->ctx;
    const uint32_t have = pos < c->ctx ? (pos == len ? len + 1 : len) : len;
    if (n_pos > have) {
        ct__set_error("ct_ds4_attend: fewer positions cached than the attention reads");
        return CT_ERR_ARG;
    }
    for (uint32_t i = 0; i < D; i++) c->q_host[i] = ct_f32_to_bf16_host(q[i]);
    c->i_host[1] = (int32_t)n_pos;
    rc = ct__cuda_status(cudaMemcpyAsync(c->q_dev, c->q_host, D * sizeof(uint16_t), cudaMemcpyHostToDevice, c->stream),
                         "ds4 q");
    if (!rc) rc = ct__cuda_status(cudaMemcpyAsync(c->i_dev + 1, c->i_host + 1, sizeof(int32_t), cudaMemcpyHostToDevice,
                                                  c->stream), "ds4 len");
    const ct_mla_shape_t shape = {1, D, D, P, c->max_pages, CT_KV_F32, 1.0f / sqrtf((float)D),
                                  c->n_layers * c->max_pages};
    const int32_t n_host = (int32_t)n_pos;
    if (!rc) rc = ct_attn_mla_decode_paged_noalloc(&shape, &n_host, 1, c->q_dev, ct_kv_paged_pool(c->kv), NULL,
                                                   ct_kv_paged_block_table_dev(c->kv) + (size_t)layer * c->max_pages,
                                                   c->i_dev + 1, c->o_dev, NULL, c->stream);
    if (!rc) rc = ct__cuda_status(cudaMemcpyAsync(c->o_host, c->o_dev, D * sizeof(uint16_t), cudaMemcpyDeviceToHost,
                                                  c->stream), "ds4 out");
    if (!rc) rc = ct__cuda_status(cudaStreamSynchronize(c->stream), "ds4 sync");
    if (rc) return rc;
    for (uint32_t i = 0; i < D; i++) {
        const uint32_t u = (uint32_t)c->o_host[i] << 16;
        memcpy(&out[i], &u, sizeof u);
    }
    return CT_OK;
}
