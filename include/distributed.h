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

#ifdef __cplusplus
}
#endif

#endif /* CAUTREO_DISTRIBUTED_H */
