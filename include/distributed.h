#ifndef CAUTREO_DISTRIBUTED_H
#define CAUTREO_DISTRIBUTED_H

/*
 * distributed.h -- multi-GPU support for the KV hot path.
 *
 * Part 1 keeps the reference interface of src/distributed/distributed.h:19-52
 * unchanged.  As in the reference (distributed.c:37-58) the in-process
 * collectives are single-device identities; the real exchange of this path --
 * gathering per-rank decode outputs and stats after a sequence-sharded step --
 * runs over NCCL from the host process (one rank per GPU), see Part 2.
 * ct_dist_available_memory reports free device memory from the CUDA runtime.
 *
 * Part 2 adds the sequence-sharding rule: longest-processing-time (LPT)
 * assignment of sequences to ranks by token count.
 *
 * Part 3 is the NCCL backend the reference reserves a place for
 * (distributed.c:41, "Real backends ... plug in here"): one process per GPU,
 * a communicator per context, and the two exchanges of the sharded decode --
 * every rank's output rows gathered to rank 0 at their global positions, and
 * every rank's statistics gathered to rank 0.  With it, the Part-1
 * collectives move device buffers between the processes.
 */

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* distributed.h:19-24 */
typedef enum {
    CT_DIST_NONE = 0,
    CT_DIST_TENSOR_PARALLEL,
    CT_DIST_PIPELINE_PARALLEL,
    CT_DIST_RDMA,
} ct_dist_mode_t;

/* distributed.h:26-31 */
typedef struct {
    ct_dist_mode_t mode;
    uint32_t       n_devices;
    uint32_t       device_id;
    const char   **device_names;
} ct_dist_config_t;

typedef struct ct_dist_ctx ct_dist_ctx_t;

/* distributed.h:36-52 */
ct_dist_ctx_t *ct_dist_init(const ct_dist_config_t *cfg);
void           ct_dist_destroy(ct_dist_ctx_t *ctx);
uint32_t ct_dist_n_devices(const ct_dist_ctx_t *ctx);
uint32_t ct_dist_device_id(const ct_dist_ctx_t *ctx);
bool     ct_dist_is_leader(const ct_dist_ctx_t *ctx);
bool ct_dist_allreduce(ct_dist_ctx_t *ctx, float *buf, size_t n);
bool ct_dist_broadcast(ct_dist_ctx_t *ctx, float *buf, size_t n, uint32_t root);
bool ct_dist_send(ct_dist_ctx_t *ctx, const float *buf, size_t n, uint32_t dest);
bool ct_dist_recv(ct_dist_ctx_t *ctx, float *buf, size_t n, uint32_t src);
uint64_t ct_dist_available_memory(const ct_dist_ctx_t *ctx, uint32_t device_id);

/* ---- Part 2: sequence sharding (new) ------------------------------------ */

/* rank_of[s] for each of n sequences: visit sequences by token count,
 * longest first (ties: lower sequence id first), and give each to the rank
 * holding the fewest tokens so far (ties: lower rank).  Returns 0. */
int ct_dist_shard_lpt(const uint32_t *lengths, uint32_t n, uint32_t n_ranks, int32_t *rank_of);

/* The sequences of one rank in ascending id order; returns their count. */
uint32_t ct_dist_rank_sequences(const int32_t *rank_of, uint32_t n, uint32_t rank,
                                uint32_t *seq_ids_out);

/* ---- Part 3: NCCL backend (new) --------------------------------------------- */

/* NCCL is loaded at run time (libnccl.so.2, the copy already in the process
 * if one is); these return CT_ERR_UNSUPPORTED when it cannot be loaded. */
#define CT_DIST_ID_BYTES 128

/* Rank 0 creates the communicator id; the launcher passes its 128 bytes to
 * every rank (a file, a socket, the process launcher's own store). */
int ct_dist_nccl_unique_id(uint8_t id_out[CT_DIST_ID_BYTES]);

/* A context whose collectives run over NCCL between cfg->n_devices
 * processes: this one is rank cfg->device_id and uses CUDA device `device`.
 * Every rank calls it with the same id; it returns when all have joined,
 * NULL on failure (ct_hal_cuda_last_error says why).  ct_dist_destroy
 * releases the communicator.  With such a context, ct_dist_allreduce (sum),
 * ct_dist_broadcast, ct_dist_send and ct_dist_recv take DEVICE fp32 buffers
 * and return once the transfer is complete; the contexts of ct_dist_init
 * keep the reference's single-process behaviour. */
ct_dist_ctx_t *ct_dist_init_nccl(const ct_dist_config_t *cfg, const uint8_t id[CT_DIST_ID_BYTES], int device);

/* Output rows of a sequence-sharded step, gathered to rank 0 in global
 * sequence order.  Every rank passes its n_rows rows (device, row_bytes
 * each, a multiple of 4), their global positions global_ids (host,
 * n_rows), and the same n_global; rank 0 passes out (device,
 * [n_global][row_bytes]), which receives every rank's rows at their
 * positions (rows no rank sends are left as they were).  The rows travel
 * with NCCL point-to-point sends into a staging buffer on rank 0 that one
 * kernel scatters to their places.  Enqueued on `stream`; returns CT_OK
 * once the gather is complete.  All ranks must call it. */
int ct_dist_gather_rows(ct_dist_ctx_t *ctx, const void *rows, uint32_t n_rows, size_t row_bytes,
                        const uint32_t *global_ids, uint32_t n_global, void *out, void *stream);

/* Per-rank statistics of a step. */
typedef struct {
    uint64_t kv_tokens;      /* KV tokens attended */
    uint64_t bytes;          /* algorithmic bytes moved */
    double   decode_us;      /* device time of the decode */
    int32_t  error;          /* the decode kernels' error word */
    uint32_t n_seqs;         /* sequences of the rank */
} ct_dist_stats_t;

/* all (rank 0: host [n_devices]) receives every rank's `mine`; the other
 * ranks may pass NULL.  All ranks must call it. */
int ct_dist_gather_stats(ct_dist_ctx_t *ctx, const ct_dist_stats_t *mine, ct_dist_stats_t *all);

#ifdef __cplusplus
}
#endif

#endif /* CAUTREO_DISTRIBUTED_H */
