/*
 * distributed.c -- distributed.h.
 *
 * Part 1 mirrors src/distributed/distributed.c: a context holding the config
 * (n_devices defaults to 1), rank queries, and in-process collectives that
 * are identities on one device (the reference's placeholders, :37-58).  The
 * cross-GPU exchange of the sharded decode -- gathering per-rank outputs and
 * stats -- is issued over NCCL by the host process that owns each GPU.
 * ct_dist_available_memory returns the device's free bytes.
 *
 * Part 2: longest-processing-time sharding of sequences over ranks.
 */
#include "../../include/distributed.h"

#include <cuda_runtime_api.h>
#include <stdlib.h>

struct ct_dist_ctx { ct_dist_config_t cfg; };

ct_dist_ctx_t *ct_dist_init(const ct_dist_config_t *cfg) {
    ct_dist_ctx_t *ctx = (ct_dist_ctx_t *)calloc(1, sizeof *ctx);
    if (!ctx) return NULL;
    if (cfg) ctx->cfg = *cfg;
    if (ctx->cfg.n_devices == 0) ctx->cfg.n_devices = 1;
    return ctx;
}

void ct_dist_destroy(ct_dist_ctx_t *ctx) { free(ctx); }
uint32_t ct_dist_n_devices(const ct_dist_ctx_t *ctx) { return ctx ? ctx->cfg.n_devices : 1; }
uint32_t ct_dist_device_id(const ct_dist_ctx_t *ctx) { return ctx ? ctx->cfg.device_id : 0; }
bool ct_dist_is_leader(const ct_dist_ctx_t *ctx) { return !ctx || ctx->cfg.device_id == 0; }

bool ct_dist_allreduce(ct_dist_ctx_t *ctx, float *buf, size_t n) {
    (void)ctx; (void)n;
    return buf != NULL;
}

bool ct_dist_broadcast(ct_dist_ctx_t *ctx, float *buf, size_t n, uint32_t root) {
    (void)ctx; (void)buf; (void)n; (void)root;
    return true;
}

bool ct_dist_send(ct_dist_ctx_t *ctx, const float *buf, size_t n, uint32_t dest) {
    (void)ctx; (void)buf; (void)n; (void)dest;
    return true;
}

bool ct_dist_recv(ct_dist_ctx_t *ctx, float *buf, size_t n, uint32_t src) {
    (void)ctx; (void)buf; (void)n; (void)src;
    return true;
}

uint64_t ct_dist_available_memory(const ct_dist_ctx_t *ctx, uint32_t device_id) {
    (void)ctx;
    int prev = 0;
    size_t free_b = 0, total_b = 0;
    if (cudaGetDevice(&prev) != cudaSuccess) { cudaGetLastError(); return 0; }
    if (cudaSetDevice((int)device_id) != cudaSuccess) { cudaGetLastError(); return 0; }
    if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) { cudaGetLastError(); free_b = 0; }
    cudaSetDevice(prev);
    return (uint64_t)free_b;
}

/* ---- Part 2 ------------------------------------------------------------- */

static const uint32_t *g_len;
static int by_len_desc(const void *a, const void *b) {
    uint32_t x = *(const uint32_t *)a, y = *(const uint32_t *)b;
    if (g_len[x] != g_len[y]) return g_len[x] > g_len[y] ? -1 : 1;
    return (x > y) - (x < y);
}

int ct_dist_shard_lpt(const uint32_t *lengths, uint32_t n, uint32_t n_ranks, int32_t *rank_of) {
    if ((n && (!lengths || !rank_of)) || n_ranks == 0) return -1;
    uint32_t *order = (uint32_t *)malloc((n ? n : 1) * sizeof(uint32_t));
    uint64_t *load = (uint64_t *)calloc(n_ranks, sizeof(uint64_t));
    if (!order || !load) { free(order); free(load); return -3; }
    for (uint32_t i = 0; i < n; i++) order[i] = i;
    g_len = lengths;
    qsort(order, n, sizeof(uint32_t), by_len_desc);
    for (uint32_t k = 0; k < n; k++) {
        uint32_t r = 0;
        for (uint32_t j = 1; j < n_ranks; j++) if (load[j] < load[r]) r = j;
        rank_of[order[k]] = (int32_t)r;
        load[r] += lengths[order[k]];
    }
    free(order);
    free(load);
    return 0;
}

uint32_t ct_dist_rank_sequences(const int32_t *rank_of, uint32_t n, uint32_t rank, uint32_t *seq_ids_out) {
    uint32_t c = 0;
    for (uint32_t s = 0; s < n; s++)
        if (rank_of[s] == (int32_t)rank) { if (seq_ids_out) seq_ids_out[c] = s; c++; }
    return c;
}
