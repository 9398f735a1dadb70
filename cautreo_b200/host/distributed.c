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
 *
 * Part 3: the NCCL backend.  libnccl.so.2 is opened at run time (dlopen
 * returns the copy a process already holds, e.g. the one its framework
 * loaded), so the library has no link-time NCCL dependency and single-GPU
 * users never load it.  A context created by ct_dist_init_nccl owns a
 * communicator, a stream on its device and the device buffers of the
 * gathers; its collectives are issued on that stream and waited for.
 */
#include "../../include/distributed.h"
#include "../../include/hal.h"
#include "../csrc/ct_internal.h"

#include <cuda_runtime_api.h>
#include <dlfcn.h>
#include <nccl.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---- the NCCL entry points this file uses, resolved once ------------------ */

typedef struct {
    ncclResult_t (*get_unique_id)(ncclUniqueId *);
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*comm_destroy)(ncclComm_t);
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*broadcast)(const void *, void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*group_start)(void);
    ncclResult_t (*group_end)(void);
    const char *(*error_string)(ncclResult_t);
} nccl_api_t;

static nccl_api_t g_nccl;
static int g_nccl_state;                 /* 0 untried, 1 loaded, -1 unavailable */
static pthread_once_t g_nccl_once = PTHREAD_ONCE_INIT;

static void nccl_load(void) {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) { g_nccl_state = -1; return; }
#define CT_NCCL_SYM(field, name) *(void **)&g_nccl.field = dlsym(h, name)
    CT_NCCL_SYM(get_unique_id, "ncclGetUniqueId");
    CT_NCCL_SYM(comm_init_rank, "ncclCommInitRank");
    CT_NCCL_SYM(comm_destroy, "ncclCommDestroy");
    CT_NCCL_SYM(all_reduce, "ncclAllReduce");
    CT_NCCL_SYM(broadcast, "ncclBroadcast");
    CT_NCCL_SYM(all_gather, "ncclAllGather");
    CT_NCCL_SYM(send, "ncclSend");
    CT_NCCL_SYM(recv, "ncclRecv");
    CT_NCCL_SYM(group_start, "ncclGroupStart");
    CT_NCCL_SYM(group_end, "ncclGroupEnd");
    CT_NCCL_SYM(error_string, "ncclGetErrorString");
#undef CT_NCCL_SYM
    g_nccl_state = g_nccl.get_unique_id && g_nccl.comm_init_rank && g_nccl.comm_destroy && g_nccl.all_reduce &&
                           g_nccl.broadcast && g_nccl.all_gather && g_nccl.send && g_nccl.recv && g_nccl.group_start &&
                           g_nccl.group_end && g_nccl.error_string
                       ? 1 : -1;
}

static int nccl_ready(void) {
    pthread_once(&g_nccl_once, nccl_load);
    if (g_nccl_state != 1) {
        ct__set_error("distributed: libnccl.so.2 could not be loaded");
        return CT_ERR_UNSUPPORTED;
    }
    return CT_OK;
}

static int nccl_status(ncclResult_t r, const char *where) {
    if (r == ncclSuccess) return CT_OK;
    char msg[256];
    snprintf(msg, sizeof msg, "%s: %s", where, g_nccl.error_string ? g_nccl.error_string(r) : "NCCL error");
    ct__set_error(msg);
    return CT_ERR_CUDA;
}

struct ct_dist_ctx {
    ct_dist_config_t cfg;
    /* NCCL backend (comm != NULL) */
    ncclComm_t comm;
    cudaStream_t stream;
    int device;
    int32_t *counts_dev;                  /* [n_devices] rows per rank, then one more slot */
    uint32_t *ids_dev;                    /* this rank's global ids */
    size_t ids_cap;
    uint8_t *stage_rows;                  /* rank 0: every rank's rows, rank by rank */
    uint32_t *stage_ids;                  /* rank 0: their global ids */
    size_t stage_rows_cap, stage_ids_cap;
    uint8_t *stats_dev;                   /* [1 + n_devices] ct_dist_stats_t */
};

ct_dist_ctx_t *ct_dist_init(const ct_dist_config_t *cfg) {
    ct_dist_ctx_t *ctx = (ct_dist_ctx_t *)calloc(1, sizeof *ctx);
    if (!ctx) return NULL;
    if (cfg) ctx->cfg = *cfg;
    if (ctx->cfg.n_devices == 0) ctx->cfg.n_devices = 1;
    return ctx;
}

void ct_dist_destroy(ct_dist_ctx_t *ctx) {
    if (!ctx) return;
    if (ctx->comm) {
        cudaSetDevice(ctx->device);
        cudaStreamSynchronize(ctx->stream);
        g_nccl.comm_destroy(ctx->comm);
        cudaStreamDestroy(ctx->stream);
        cudaFree(ctx->counts_dev); cudaFree(ctx->ids_dev); cudaFree(ctx->stage_rows); cudaFree(ctx->stage_ids);
        cudaFree(ctx->stats_dev);
    }
    free(ctx);
}
uint32_t ct_dist_n_devices(const ct_dist_ctx_t *ctx) { return ctx ? ctx->cfg.n_devices : 1; }
uint32_t ct_dist_device_id(const ct_dist_ctx_t *ctx) { return ctx ? ctx->cfg.device_id : 0; }
bool ct_dist_is_leader(const ct_dist_ctx_t *ctx) { return !ctx || ctx->cfg.device_id == 0; }

/* Runs on the context's stream and waits for it. */
static int finish(ct_dist_ctx_t *ctx, int rc) {
    const int rs = ct__cuda_status(cudaStreamSynchronize(ctx->stream), "distributed");
    return rc ? rc : rs;
}

/* With the reference's single-process contexts these are identities, as in
 * distributed.c:37-58; with an NCCL context they move device buffers. */
bool ct_dist_allreduce(ct_dist_ctx_t *ctx, float *buf, size_t n) {
    if (!buf) return false;
    if (!ctx || !ctx->comm) return true;
    if (cudaSetDevice(ctx->device) != cudaSuccess) return false;
    return finish(ctx, nccl_status(g_nccl.all_reduce(buf, buf, n, ncclFloat32, ncclSum, ctx->comm, ctx->stream),
                                   "ct_dist_allreduce")) == CT_OK;
}

bool ct_dist_broadcast(ct_dist_ctx_t *ctx, float *buf, size_t n, uint32_t root) {
    if (!ctx || !ctx->comm) return true;
    if (!buf || root >= ctx->cfg.n_devices || cudaSetDevice(ctx->device) != cudaSuccess) return false;
    return finish(ctx, nccl_status(g_nccl.broadcast(buf, buf, n, ncclFloat32, (int)root, ctx->comm, ctx->stream),
                                   "ct_dist_broadcast")) == CT_OK;
}

bool ct_dist_send(ct_dist_ctx_t *ctx, const float *buf, size_t n, uint32_t dest) {
    if (!ctx || !ctx->comm) return true;
    if (!buf || dest >= ctx->cfg.n_devices || cudaSetDevice(ctx->device) != cudaSuccess) return false;
    return finish(ctx, nccl_status(g_nccl.send(buf, n, ncclFloat32, (int)dest, ctx->comm, ctx->stream),
                                   "ct_dist_send")) == CT_OK;
}

bool ct_dist_recv(ct_dist_ctx_t *ctx, float *buf, size_t n, uint32_t src) {
    if (!ctx || !ctx->comm) return true;
    if (!buf || src >= ctx->cfg.n_devices || cudaSetDevice(ctx->device) != cudaSuccess) return false;
    return finish(ctx, nccl_status(g_nccl.recv(buf, n, ncclFloat32, (int)src, ctx->comm, ctx->stream),
                                   "ct_dist_recv")) == CT_OK;
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

/* ---- Part 3 ------------------------------------------------------------- */

int ct_dist_nccl_unique_id(uint8_t id_out[CT_DIST_ID_BYTES]) {
    if (!id_out) return CT_ERR_ARG;
    int rc = nccl_ready();
    if (rc) return rc;
    ncclUniqueId id;
    rc = nccl_status(g_nccl.get_unique_id(&id), "ct_dist_nccl_unique_id");
    if (!rc) memcpy(id_out, id.internal, CT_DIST_ID_BYTES);
    return rc;
}

ct_dist_ctx_t *ct_dist_init_nccl(const ct_dist_config_t *cfg, const uint8_t id[CT_DIST_ID_BYTES], int device) {
    if (!cfg || !id || cfg->n_devices == 0 || cfg->device_id >= cfg->n_devices) {
        ct__set_error("ct_dist_init_nccl: bad config");
        return NULL;
    }
    if (nccl_ready()) return NULL;
    if (ct__cuda_status(cudaSetDevice(device), "ct_dist_init_nccl")) return NULL;
    ct_dist_ctx_t *ctx = ct_dist_init(cfg);
    if (!ctx) return NULL;
    ctx->device = device;
    const uint32_t W = cfg->n_devices;
    int rc = ct__cuda_status(cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking), "ct_dist_init_nccl");
    if (!rc) rc = ct__cuda_status(cudaMalloc((void **)&ctx->counts_dev, (W + 1) * sizeof(int32_t)), "ct_dist_init_nccl");
    if (!rc) rc = ct__cuda_status(cudaMalloc((void **)&ctx->stats_dev, (W + 1) * sizeof(ct_dist_stats_t)), "ct_dist_init_nccl");
    if (!rc) {
        ncclUniqueId uid;
        memcpy(uid.internal, id, CT_DIST_ID_BYTES);
        rc = nccl_status(g_nccl.comm_init_rank(&ctx->comm, (int)W, uid, (int)cfg->device_id), "ncclCommInitRank");
    }
    if (rc) {
        if (ctx->stream) cudaStreamDestroy(ctx->stream);
        cudaFree(ctx->counts_dev); cudaFree(ctx->stats_dev);
        ctx->comm = NULL;
        free(ctx);
        return NULL;
    }
    return ctx;
}

/* Grows a device buffer to hold `need` bytes. */
static int reserve(void **buf, size_t *cap, size_t need) {
    if (*cap >= need && *buf) return CT_OK;
    cudaFree(*buf);
    *buf = NULL;
    *cap = 0;
    int rc = ct__cuda_status(cudaMalloc(buf, need ? need : 16), "distributed staging");
    if (!rc) *cap = need;
    return rc;
}

int ct_dist_gather_rows(ct_dist_ctx_t *ctx, const void *rows, uint32_t n_rows, size_t row_bytes,
                        const uint32_t *global_ids, uint32_t n_global, void *out, void *stream) {
    if (!ctx || !ctx->comm || row_bytes == 0 || row_bytes % 4 != 0 || (n_rows && (!rows || !global_ids)))
        return CT_ERR_ARG;
    const uint32_t W = ctx->cfg.n_devices, me = ctx->cfg.device_id;
    if (me == 0 && !out) return CT_ERR_ARG;
    for (uint32_t i = 0; i < n_rows; i++)
        if (global_ids[i] >= n_global) { ct__set_error("ct_dist_gather_rows: global id out of range"); return CT_ERR_ARG; }
    int rc = ct__cuda_status(cudaSetDevice(ctx->device), "ct_dist_gather_rows");
    if (rc) return rc;
    /* the gather starts after the caller's work on `stream` */
    cudaEvent_t ev = NULL;
    rc = ct__cuda_status(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "ct_dist_gather_rows");
    if (!rc) rc = ct__cuda_status(cudaEventRecord(ev, (cudaStream_t)stream), "ct_dist_gather_rows");
    if (!rc) rc = ct__cuda_status(cudaStreamWaitEvent(ctx->stream, ev, 0), "ct_dist_gather_rows");
    if (ev) cudaEventDestroy(ev);
    if (rc) return rc;
    /* every rank's row count */
    int32_t *counts = (int32_t *)malloc(W * sizeof(int32_t));
    if (!counts) return CT_ERR_NOMEM;
    const int32_t mine = (int32_t)n_rows;
    rc = ct__cuda_status(cudaMemcpyAsync(ctx->counts_dev + W, &mine, sizeof mine, cudaMemcpyHostToDevice, ctx->stream),
                         "ct_dist_gather_rows");
    if (!rc) rc = nccl_status(g_nccl.all_gather(ctx->counts_dev + W, ctx->counts_dev, 1, ncclInt32, ctx->comm, ctx->stream),
                              "ct_dist_gather_rows counts");
    if (!rc) rc = ct__cuda_status(cudaMemcpyAsync(counts, ctx->counts_dev, W * sizeof(int32_t), cudaMemcpyDeviceToHost,
                                                  ctx->stream), "ct_dist_gather_rows");
    if (!rc) rc = finish(ctx, CT_OK);
    uint64_t total = 0;
    for (uint32_t r = 0; r < W && !rc; r++) total += (uint64_t)(counts[r] > 0 ? counts[r] : 0);
    if (!rc && total > n_global) { ct__set_error("ct_dist_gather_rows: more rows than n_global"); rc = CT_ERR_ARG; }
    /* this rank's ids on the device */
    if (!rc) rc = reserve((void **)&ctx->ids_dev, &ctx->ids_cap, (size_t)n_rows * sizeof(uint32_t));
    if (!rc && n_rows)
        rc = ct__cuda_status(cudaMemcpyAsync(ctx->ids_dev, global_ids, (size_t)n_rows * sizeof(uint32_t),
                                             cudaMemcpyHostToDevice, ctx->stream), "ct_dist_gather_rows");
    if (!rc && me == 0) {
        rc = reserve((void **)&ctx->stage_rows, &ctx->stage_rows_cap, (size_t)total * row_bytes);
        if (!rc) rc = reserve((void **)&ctx->stage_ids, &ctx->stage_ids_cap, (size_t)total * sizeof(uint32_t));
    }
    if (!rc) {
        /* rank 0 keeps its own rows where they are and receives the others' */
        rc = nccl_status(g_nccl.group_start(), "ct_dist_gather_rows");
        uint64_t off = 0;
        for (uint32_t r = 0; r < W && !rc; r++) {
            const size_t n = (size_t)(counts[r] > 0 ? counts[r] : 0);
            if (me == 0 && r != 0 && n) {
                rc = nccl_status(g_nccl.recv(ctx->stage_ids + off, n, ncclUint32, (int)r, ctx->comm, ctx->stream), "recv ids");
                if (!rc) rc = nccl_status(g_nccl.recv(ctx->stage_rows + off * row_bytes, n * row_bytes, ncclUint8, (int)r,
                                                      ctx->comm, ctx->stream), "recv rows");
            }
            if (r == me && me != 0 && n) {
                rc = nccl_status(g_nccl.send(ctx->ids_dev, n, ncclUint32, 0, ctx->comm, ctx->stream), "send ids");
                if (!rc) rc = nccl_status(g_nccl.send(rows, n * row_bytes, ncclUint8, 0, ctx->comm, ctx->stream), "send rows");
            }
            if (r != 0) off += n;
        }
        const int re = nccl_status(g_nccl.group_end(), "ct_dist_gather_rows");
        if (!rc) rc = re;
        if (!rc && me == 0) {
            if (n_rows) rc = ct__launch_scatter_rows(out, rows, ctx->ids_dev, n_rows, row_bytes, ctx->stream);
            if (!rc && off) rc = ct__launch_scatter_rows(out, ctx->stage_rows, ctx->stage_ids, (uint32_t)off, row_bytes,
                                                         ctx->stream);
        }
    }
    free(counts);
    return finish(ctx, rc);
}

int ct_dist_gather_stats(ct_dist_ctx_t *ctx, const ct_dist_stats_t *mine, ct_dist_stats_t *all) {
    if (!ctx || !ctx->comm || !mine || (ctx->cfg.device_id == 0 && !all)) return CT_ERR_ARG;
    const uint32_t W = ctx->cfg.n_devices;
    int rc = ct__cuda_status(cudaSetDevice(ctx->device), "ct_dist_gather_stats");
    uint8_t *send = ctx->stats_dev + (size_t)W * sizeof(ct_dist_stats_t);
    if (!rc) rc = ct__cuda_status(cudaMemcpyAsync(send, mine, sizeof *mine, cudaMemcpyHostToDevice, ctx->stream),
                                  "ct_dist_gather_stats");
    if (!rc) rc = nccl_status(g_nccl.all_gather(send, ctx->stats_dev, sizeof *mine, ncclUint8, ctx->comm, ctx->stream),
                              "ct_dist_gather_stats");
    if (!rc && all) rc = ct__cuda_status(cudaMemcpyAsync(all, ctx->stats_dev, (size_t)W * sizeof *mine,
                                                         cudaMemcpyDeviceToHost, ctx->stream), "ct_dist_gather_stats");
    return finish(ctx, rc);
}
