/*
 * attention.c -- attention.h on the device.
 *
 * Part 1: the reference's ct_attn_forward / ct_attn_forward_kv /
 * ct_attn_softmax (src/attention/attention.c:11-59) with the same
 * arguments, defaults and return values; inputs are copied to the device, the
 * kernels of attn_plain.cu run, the result is copied back.
 *
 * Part 2: MLA decode plans.  A plan holds the device buffers of the work
 * split for a fixed number of sequences: every decode first runs the
 * planning kernel (csrc/mla_plan.cu), which lays the sequences' pages end to
 * end from the CURRENT device lengths and gives each worker (a pair of SMs
 * for the tensor-core kernel, one block per chunk and head group for the
 * CUDA-core kernel) the same number of pages; chunks of a split sequence
 * write partial (o, m, l) to the plan's scratch and one combine launch
 * merges them.  So a plan stays valid while the sequences grow, and a
 * serving step needs no host planning and no allocation.
 */
#include "../../include/attention.h"
#include "../../include/hal.h"
#include "../../include/kv_cache.h"
#include "../csrc/ct_internal.h"

#include <cuda_runtime_api.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ---- Part 1 --------------------------------------------------------------- */

bool ct_attn_forward(const float *q, const float *k, const float *v, uint32_t n_tokens, uint32_t n_kv_heads,
                     uint32_t head_dim, float scale, float *out) {
    if (!q || !k || !v || !out || n_tokens == 0) return false;
    if (scale == 0.0f) scale = 1.0f / sqrtf((float)head_dim);
    if (n_kv_heads == 0 || head_dim == 0) return true;
    const size_t qb = (size_t)n_kv_heads * head_dim * sizeof(float);
    const size_t kb = (size_t)n_tokens * head_dim * sizeof(float);
    const size_t sb = ct__attn_scratch_bytes(n_tokens, n_kv_heads, head_dim);
    char *buf = NULL;
    const size_t total = 2 * qb + 2 * kb + sb;
    if (ct__scratch_alloc((void **)&buf, total, NULL)) return false;
    float *dq = (float *)buf, *dout = (float *)(buf + qb), *dk = (float *)(buf + 2 * qb);
    float *dv = (float *)(buf + 2 * qb + kb), *dsc = (float *)(buf + 2 * qb + 2 * kb);
    int rc = ct__cuda_status(cudaMemcpyAsync(dq, q, qb, cudaMemcpyHostToDevice, 0), "ct_attn_forward");
    if (!rc) rc = ct__cuda_status(cudaMemcpyAsync(dk, k, kb, cudaMemcpyHostToDevice, 0), "ct_attn_forward");
    if (!rc) rc = ct__cuda_status(cudaMemcpyAsync(dv, v, kb, cudaMemcpyHostToDevice, 0), "ct_attn_forward");
    if (!rc) rc = ct__launch_attn_shared(dq, dk, dv, n_tokens, n_kv_heads, head_dim, scale, dout, dsc, NULL);
    if (!rc) rc = ct__cuda_status(cudaMemcpyAsync(out, dout, qb, cudaMemcpyDeviceToHost, 0), "ct_attn_forward");
    ct__scratch_free(buf, NULL);
    if (!rc) rc = ct__cuda_status(cudaStreamSynchronize(0), "ct_attn_forward");
    return rc == CT_OK;
}

bool ct_attn_forward_kv(const float *q, const float *kv_k, const float *kv_v, uint32_t n_tokens,
                        uint32_t n_kv_heads, uint32_t head_dim, float scale, float *out) {
    return ct_attn_forward(q, kv_k, kv_v, n_tokens, n_kv_heads, head_dim, scale, out);
}

void ct_attn_softmax(float *x, uint32_t n) {
    if (!x || n == 0) return;
    float *d = NULL;
    const size_t b = (size_t)n * sizeof(float);
    const size_t extra = ct__softmax_scratch_bytes(n);
    if (ct__scratch_alloc((void **)&d, b + extra + 16, NULL)) return;
    void *sx = (char *)d + ((b + 15) & ~(size_t)15);
    int rc = ct__cuda_status(cudaMemcpyAsync(d, x, b, cudaMemcpyHostToDevice, 0), "ct_attn_softmax");
    if (!rc) rc = ct__launch_softmax(d, n, sx, NULL);
    if (!rc) rc = ct__cuda_status(cudaMemcpyAsync(x, d, b, cudaMemcpyDeviceToHost, 0), "ct_attn_softmax");
    ct__scratch_free(d, NULL);
    cudaStreamSynchronize(0);
}

/* ---- Part 2: MLA plans ---------------------------------------------------- */

/* ct_attn_mla_decode_step_host splits a step into up to this many sequence
 * groups, so that the copies of one group overlap the decode of another.
 * Each group costs one more set of decode launches, worth it while the
 * group's copies (~3 MB, ~60 us over PCIe) are longer than their fill and
 * drain; so a step gets one group per CT_STEP_GROUP_BYTES of copies. */
#define CT_STEP_GROUPS 8
#define CT_STEP_GROUP_BYTES (3u << 20)

struct ct_mla_plan {
    ct_mla_dims_t dims;
    uint32_t n_seq, n_workers, n_chunks, n_combines, n_parts;   /* the split of the creation lengths */
    uint32_t cap_chunks, cap_combines, cap_parts;
    int device;
    int tensor_cores;
    ct_mla_chunk_t *chunks;      /* device [cap_chunks], worker-major, written by the planning kernel */
    int32_t *worker_begin;       /* device [n_workers + 1] */
    ct_mla_combine_t *combines;  /* device [cap_combines] */
    int32_t *counts;             /* device: chunks and combines of the last decode */
    uint32_t *rows_dev;          /* device [n_seq] block-table rows, or NULL for 0..n_seq-1 */
    float *part_o, *part_ml;     /* device scratch: [cap_parts][n_heads][v_dim], [cap_parts][n_heads][4] */
    size_t scratch_bytes;
    void *stage_q, *stage_e, *stage_o;   /* device staging of ct_attn_mla_decode_step_host */
    uint32_t last_launches;
    /* Host copies of the inputs the plan was made from, so that
     * ct_attn_mla_decode_step_host can re-plan sequence groups. */
    ct_mla_shape_t shape;
    uint32_t *rows_h;
    int32_t *lens_h;
    /* ct_attn_mla_decode_step_host's pipeline: sequence groups
     * [group_begin[g], group_begin[g + 1]) with one sub-plan each, a copy-in
     * and a copy-out stream, a second decode stream for the odd groups, and
     * the events that order them. */
    uint32_t n_groups;
    uint32_t group_begin[CT_STEP_GROUPS + 1];
    ct_mla_plan_t *group_plan[CT_STEP_GROUPS];
    cudaStream_t copy_in, copy_out, dec2;
    cudaEvent_t ev_in[CT_STEP_GROUPS], ev_dec[CT_STEP_GROUPS], ev_go, ev_done2;
};

/* Declared in mla_tc.cu: whether the tensor-core kernel takes these dims on
 * this device, and the number of workers it runs. */
int ct__mla_tc_workers(const ct_mla_dims_t *dims, int device);

void ct_mla_plan_destroy(ct_mla_plan_t *p) {
    if (!p) return;
    cudaFree(p->chunks); cudaFree(p->worker_begin); cudaFree(p->combines); cudaFree(p->counts); cudaFree(p->rows_dev);
    cudaFree(p->part_o); cudaFree(p->part_ml);
    cudaFree(p->stage_q); cudaFree(p->stage_e); cudaFree(p->stage_o);
    for (uint32_t g = 0; g < CT_STEP_GROUPS; g++) {
        ct_mla_plan_destroy(p->group_plan[g]);
        if (p->ev_in[g]) cudaEventDestroy(p->ev_in[g]);
        if (p->ev_dec[g]) cudaEventDestroy(p->ev_dec[g]);
    }
    if (p->ev_go) cudaEventDestroy(p->ev_go);
    if (p->ev_done2) cudaEventDestroy(p->ev_done2);
    if (p->copy_in) cudaStreamDestroy(p->copy_in);
    if (p->copy_out) cudaStreamDestroy(p->copy_out);
    if (p->dec2) cudaStreamDestroy(p->dec2);
    free(p->rows_h); free(p->lens_h);
    free(p);
}

ct_mla_plan_t *ct_mla_plan_create(const ct_mla_shape_t *shape, const uint32_t *seq_rows,
                                  const int32_t *seq_lens, uint32_t n_seq, int device) {
    if (!shape || !seq_lens || shape->n_heads == 0 || shape->page_tokens == 0 || shape->v_dim > shape->entry_dim ||
        shape->entry_dim == 0 || shape->max_pages_per_seq == 0 || shape->n_pages == 0) {
        ct__set_error("ct_mla_plan_create: bad shape");
        return NULL;
    }
    ct_mla_plan_t *p = (ct_mla_plan_t *)calloc(1, sizeof *p);
    if (!p) return NULL;
    p->dims.n_heads = shape->n_heads;
    p->dims.entry_dim = shape->entry_dim;
    p->dims.v_dim = shape->v_dim;
    p->dims.page_tokens = shape->page_tokens;
    p->dims.max_pages_per_seq = shape->max_pages_per_seq;
    p->dims.kv_dtype = shape->kv_dtype;
    p->dims.scale = shape->scale;
    p->dims.n_pages = shape->n_pages;
    p->dims.n_seq = n_seq;
    p->n_seq = n_seq;
    p->device = device;
    p->shape = *shape;
    const uint32_t P = shape->page_tokens;

    int n_sms = 148;
    if (cudaDeviceGetAttribute(&n_sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) {
        cudaGetLastError();
        n_sms = 148;
    }
    int tc_workers = ct__mla_tc_workers(&p->dims, device);
    p->n_workers = tc_workers > 0 ? (uint32_t)tc_workers : (uint32_t)n_sms;
    p->tensor_cores = tc_workers > 0;

    for (uint32_t s = 0; s < n_seq; s++) {
        if (seq_lens[s] < 0 || (uint64_t)(seq_lens[s] + P - 1) / P > shape->max_pages_per_seq) {
            ct__set_error("ct_mla_plan_create: sequence longer than its block-table row");
            free(p);
            return NULL;
        }
    }
    p->rows_h = (uint32_t *)malloc((size_t)(n_seq ? n_seq : 1) * sizeof(uint32_t));
    p->lens_h = (int32_t *)malloc((size_t)(n_seq ? n_seq : 1) * sizeof(int32_t));
    if (!p->rows_h || !p->lens_h) {
        ct__set_error("ct_mla_plan_create: out of memory");
        free(p->rows_h); free(p->lens_h); free(p);
        return NULL;
    }
    for (uint32_t s = 0; s < n_seq; s++) {
        p->rows_h[s] = seq_rows ? seq_rows[s] : s;
        p->lens_h[s] = seq_lens[s];
    }
    const uint32_t W = p->n_workers;
    /* The split the planning kernel makes for the creation lengths (the same
     * rule, for ct_mla_plan_chunks): pages end to end, W equal page ranges. */
    uint64_t total = 0;
    for (uint32_t s = 0; s < n_seq; s++) total += ((uint32_t)seq_lens[s] + P - 1) / P;
    const uint64_t Q = total ? (total + W - 1) / W : 1;
    uint64_t cp = 0;
    for (uint32_t s = 0; s < n_seq; s++) {
        const uint64_t np = ((uint32_t)seq_lens[s] + P - 1) / P;
        const uint32_t n = np ? (uint32_t)((cp + np - 1) / Q - cp / Q + 1) : 1;
        p->n_chunks += n;
        if (n > 1) { p->n_parts += n; p->n_combines++; }
        cp += np;
    }
    /* Capacities for any lengths: every interior cut adds one chunk, and
     * split sequences hold at most 2 (W - 1) parts and W - 1 combines. */
    p->cap_chunks = n_seq + W;
    p->cap_combines = W < n_seq ? W : (n_seq ? n_seq : 1);
    p->cap_parts = 2 * W < n_seq + W ? 2 * W : n_seq + W;
    int rc = ct__cuda_status(cudaSetDevice(device), "ct_mla_plan_create");
    if (!rc) rc = ct__cuda_status(cudaMalloc((void **)&p->chunks, (size_t)p->cap_chunks * sizeof(ct_mla_chunk_t)), "plan chunks");
    if (!rc) rc = ct__cuda_status(cudaMalloc((void **)&p->worker_begin, ((size_t)W + 1) * sizeof(int32_t)), "plan workers");
    if (!rc) rc = ct__cuda_status(cudaMalloc((void **)&p->combines, (size_t)p->cap_combines * sizeof(ct_mla_combine_t)), "plan combines");
    if (!rc) rc = ct__cuda_status(cudaMalloc((void **)&p->counts, 2 * sizeof(int32_t)), "plan counts");
    if (!rc && seq_rows) {
        rc = ct__cuda_status(cudaMalloc((void **)&p->rows_dev, (size_t)(n_seq ? n_seq : 1) * sizeof(uint32_t)), "plan rows");
        if (!rc && n_seq)
            rc = ct__cuda_status(cudaMemcpy(p->rows_dev, seq_rows, (size_t)n_seq * sizeof(uint32_t), cudaMemcpyHostToDevice),
                                 "plan rows");
    }
    const size_t po = (size_t)p->cap_parts * shape->n_heads * shape->v_dim * sizeof(float);
    const size_t pm = (size_t)p->cap_parts * shape->n_heads * 4 * sizeof(float);   /* (m, l_lo, l_hi, -) */
    if (!rc) rc = ct__cuda_status(cudaMalloc((void **)&p->part_o, po), "plan scratch");
    if (!rc) rc = ct__cuda_status(cudaMalloc((void **)&p->part_ml, pm), "plan scratch");
    p->scratch_bytes = po + pm;
    if (rc) { ct_mla_plan_destroy(p); return NULL; }
    return p;
}

uint32_t ct_mla_plan_chunks(const ct_mla_plan_t *p) { return p ? p->n_chunks : 0; }
size_t ct_mla_plan_scratch_bytes(const ct_mla_plan_t *p) { return p ? p->scratch_bytes : 0; }
uint32_t ct_mla_plan_launches(const ct_mla_plan_t *p) { return p ? p->last_launches : 0; }
uint32_t ct_mla_plan_workers(const ct_mla_plan_t *p) { return p ? p->n_workers : 0; }
int ct_mla_plan_tensor_cores(const ct_mla_plan_t *p) { return p ? p->tensor_cores : 0; }

int ct_attn_mla_decode_paged(const ct_mla_plan_t *plan, const void *q, const void *pool, const float *scales,
                             const int32_t *block_table, const int32_t *seq_lens, void *out, float *lse,
                             void *stream) {
    if (!plan || !q || !pool || !block_table || !seq_lens || !out) return CT_ERR_ARG;
    if ((plan->dims.kv_dtype == CT_KV_INT8 || plan->dims.kv_dtype == CT_KV_E4M3) && !scales) return CT_ERR_ARG;
    ct_mla_plan_t *p = (ct_mla_plan_t *)plan;
    uint32_t launches = 0;
    int rc = ct__launch_mla_plan(p->rows_dev, seq_lens, p->n_seq, p->dims.page_tokens, p->dims.max_pages_per_seq,
                                 p->n_workers, p->chunks, p->worker_begin, p->combines, p->counts, stream);
    if (!rc) rc = ct__launch_mla_decode(&p->dims, p->chunks, p->cap_chunks, p->worker_begin, p->n_workers, p->combines,
                                        p->cap_combines, p->counts, q, pool, scales, block_table, seq_lens, out, lse,
                                        p->part_o, p->part_ml, stream, &launches);
    if (!rc) { launches++; ct__count_launches(1); }
    p->last_launches = launches;
    return rc;
}

/* Split p's sequences into contiguous groups and give each its own plan,
 * copy streams and events.  Called once per plan.  Nothing overlaps the
 * copy-in of the first groups or the copy-out of the last ones (the two
 * decode streams finish their last groups together), so the groups at
 * either end are smaller: group g of G gets a share of the step's KV tokens
 * proportional to min(1, 2^(min(g, G-1-g) - 2)), i.e. 1/4, 1/2, 1, ..., 1,
 * 1/2, 1/4; a group's copy time follows its sequence count, its decode time
 * its tokens. */
static int step_host_pipeline(ct_mla_plan_t *p, size_t step_bytes) {
    uint32_t G = (uint32_t)(step_bytes / CT_STEP_GROUP_BYTES);
    if (G > CT_STEP_GROUPS) G = CT_STEP_GROUPS;
    if (G > p->n_seq / 2) G = p->n_seq / 2;             /* at least two sequences a group */
    if (G < 1) G = 1;
    uint32_t w4[CT_STEP_GROUPS], wsum = 0;             /* weights in quarters */
    for (uint32_t g = 0; g < G; g++) {
        const uint32_t e = g < G - 1 - g ? g : G - 1 - g;
        w4[g] = e >= 2 ? 4 : 1u << e;
        wsum += w4[g];
    }
    uint64_t total = 0;
    for (uint32_t s = 0; s < p->n_seq; s++) total += (uint64_t)p->lens_h[s];
    p->group_begin[0] = 0;
    uint32_t g = 0, wacc = w4[0];
    uint64_t acc = 0;
    for (uint32_t s = 0; s < p->n_seq && g + 1 < G; s++) {
        acc += (uint64_t)p->lens_h[s];
        if (acc * wsum >= total * wacc) {               /* group g holds its share of the tokens */
            p->group_begin[++g] = s + 1;
            wacc += w4[g];
        }
    }
    while (g < G) p->group_begin[++g] = p->n_seq;
    p->n_groups = G;
    if (G == 1) return CT_OK;
    int rc = ct__cuda_status(cudaStreamCreateWithFlags(&p->copy_in, cudaStreamNonBlocking), "step_host streams");
    if (!rc) rc = ct__cuda_status(cudaStreamCreateWithFlags(&p->copy_out, cudaStreamNonBlocking), "step_host streams");
    if (!rc) rc = ct__cuda_status(cudaStreamCreateWithFlags(&p->dec2, cudaStreamNonBlocking), "step_host streams");
    if (!rc) rc = ct__cuda_status(cudaEventCreateWithFlags(&p->ev_go, cudaEventDisableTiming), "step_host events");
    if (!rc) rc = ct__cuda_status(cudaEventCreateWithFlags(&p->ev_done2, cudaEventDisableTiming), "step_host events");
    for (g = 0; g < G && !rc; g++) {
        const uint32_t a = p->group_begin[g], b = p->group_begin[g + 1];
        rc = ct__cuda_status(cudaEventCreateWithFlags(&p->ev_in[g], cudaEventDisableTiming), "step_host events");
        if (!rc) rc = ct__cuda_status(cudaEventCreateWithFlags(&p->ev_dec[g], cudaEventDisableTiming), "step_host events");
        if (!rc && b > a) {
            p->group_plan[g] = ct_mla_plan_create(&p->shape, p->rows_h + a, p->lens_h + a, b - a, p->device);
            if (!p->group_plan[g]) rc = CT_ERR_CUDA;
        }
    }
    if (rc) p->n_groups = 0;             /* the next call retries */
    return rc;
}

int ct_attn_mla_decode_step_host(ct_mla_plan_t *p, const void *q_host, const void *entries_host,
                                 const int32_t *dest_slot, void *pool, float *scales,
                                 const int32_t *block_table, const int32_t *seq_lens, void *out_host,
                                 void *stream) {
    if (!p || !q_host || !out_host || !pool || !block_table || !seq_lens) return CT_ERR_ARG;
    if (dest_slot && !entries_host) return CT_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    const size_t n = p->n_seq, H = p->dims.n_heads, E = p->dims.entry_dim, Dv = p->dims.v_dim;
    const size_t qr = H * E * 2, er = E * 2, orow = H * Dv * 2;   /* bytes per sequence */
    int rc = CT_OK;
    if (!p->stage_q) {
        rc = ct__cuda_status(cudaMalloc(&p->stage_q, n ? n * qr : 16), "step_host staging");
        if (!rc) rc = ct__cuda_status(cudaMalloc(&p->stage_e, n ? n * er : 16), "step_host staging");
        if (!rc) rc = ct__cuda_status(cudaMalloc(&p->stage_o, n ? n * orow : 16), "step_host staging");
        if (rc) return rc;
    }
    if (p->n_groups == 0 && (rc = step_host_pipeline(p, n * (qr + er + orow)))) return rc;

    if (p->n_groups == 1) {              /* one group: everything in order on the caller's stream */
        rc = ct__cuda_status(cudaMemcpyAsync(p->stage_q, q_host, n * qr, cudaMemcpyHostToDevice, st), "step_host q");
        if (!rc && dest_slot) {
            rc = ct__cuda_status(cudaMemcpyAsync(p->stage_e, entries_host, n * er, cudaMemcpyHostToDevice, st),
                                 "step_host e");
            if (!rc) rc = ct_kv_paged_write_slots(pool, scales, p->dims.kv_dtype, p->stage_e, CT_KV_BF16, dest_slot,
                                                  (uint32_t)n, (uint32_t)E, stream);
        }
        if (!rc) rc = ct_attn_mla_decode_paged(p, p->stage_q, pool, scales, block_table, seq_lens, p->stage_o, NULL,
                                               stream);
        if (!rc) rc = ct__cuda_status(cudaMemcpyAsync(out_host, p->stage_o, n * orow, cudaMemcpyDeviceToHost, st),
                                      "step_host out");
        if (!rc) rc = ct__cuda_status(cudaStreamSynchronize(st), "step_host sync");
        return rc;
    }

    /* Groups: the copy-in of group g+1 runs during the decode of group g, and
     * the copy-out of group g during the decode of group g+1.  All new tokens
     * (n_seq x entry_dim bf16, small) are copied and appended before the
     * first decode, as in the one-group order.  The groups' decodes are
     * independent (own sub-plan, own rows of the staging buffers), so even
     * groups run on the caller's stream and odd ones on a second stream: the
     * next group's kernels take the SMs its predecessor's last workers leave,
     * and the planning and combine launches of one group overlap the decode
     * of its neighbour. */
    uint32_t launches = 0;
    char *oh = (char *)out_host, *sq = (char *)p->stage_q, *so = (char *)p->stage_o;
    const char *qh = (const char *)q_host;
    /* The copies start after the work already queued on the caller's stream. */
    rc = ct__cuda_status(cudaEventRecord(p->ev_dec[0], st), "step_host");
    if (!rc) rc = ct__cuda_status(cudaStreamWaitEvent(p->copy_in, p->ev_dec[0], 0), "step_host");
    if (!rc && dest_slot) {
        rc = ct__cuda_status(cudaMemcpyAsync(p->stage_e, entries_host, n * er, cudaMemcpyHostToDevice, p->copy_in),
                             "step_host e");
        if (!rc) rc = ct__cuda_status(cudaEventRecord(p->ev_in[0], p->copy_in), "step_host");
        if (!rc) rc = ct__cuda_status(cudaStreamWaitEvent(st, p->ev_in[0], 0), "step_host");
        if (!rc) rc = ct_kv_paged_write_slots(pool, scales, p->dims.kv_dtype, p->stage_e, CT_KV_BF16, dest_slot,
                                              (uint32_t)n, (uint32_t)E, stream);
    }
    /* the second decode stream starts after the append (and everything
     * queued before this call) */
    if (!rc) rc = ct__cuda_status(cudaEventRecord(p->ev_go, st), "step_host");
    if (!rc) rc = ct__cuda_status(cudaStreamWaitEvent(p->dec2, p->ev_go, 0), "step_host");
    uint32_t g = 0;
    for (; g < p->n_groups && !rc; g++) {
        const size_t a = p->group_begin[g], m = p->group_begin[g + 1] - a;
        if (m == 0) continue;
        cudaStream_t sg = (g & 1) ? p->dec2 : st;
        rc = ct__cuda_status(cudaMemcpyAsync(sq + a * qr, qh + a * qr, m * qr, cudaMemcpyHostToDevice, p->copy_in),
                             "step_host q");
        if (!rc) rc = ct__cuda_status(cudaEventRecord(p->ev_in[g], p->copy_in), "step_host");
        if (!rc) rc = ct__cuda_status(cudaStreamWaitEvent(sg, p->ev_in[g], 0), "step_host");
        if (!rc) {
            rc = ct_attn_mla_decode_paged(p->group_plan[g], sq + a * qr, pool, scales, block_table, seq_lens,
                                          so + a * orow, NULL, (void *)sg);
            launches += p->group_plan[g]->last_launches;
        }
        if (!rc) rc = ct__cuda_status(cudaEventRecord(p->ev_dec[g], sg), "step_host");
        if (!rc) rc = ct__cuda_status(cudaStreamWaitEvent(p->copy_out, p->ev_dec[g], 0), "step_host");
        if (!rc) rc = ct__cuda_status(cudaMemcpyAsync(oh + a * orow, so + a * orow, m * orow, cudaMemcpyDeviceToHost,
                                                      p->copy_out), "step_host out");
    }
    /* the caller's stream ends after the second stream's work too */
    int rj = ct__cuda_status(cudaEventRecord(p->ev_done2, p->dec2), "step_host");
    if (!rj) rj = ct__cuda_status(cudaStreamWaitEvent(st, p->ev_done2, 0), "step_host");
    if (!rc) rc = rj;
    p->last_launches = launches;
    /* On an error part of the work may be queued: wait for all of it, so no
     * copy is still reading or writing the caller's buffers on return. */
    int rs = ct__cuda_status(cudaStreamSynchronize(p->copy_in), "step_host sync");
    int r2 = ct__cuda_status(cudaStreamSynchronize(p->dec2), "step_host sync");
    int rt = ct__cuda_status(cudaStreamSynchronize(st), "step_host sync");
    int ro = ct__cuda_status(cudaStreamSynchronize(p->copy_out), "step_host sync");
    if (!rc) rc = rs ? rs : r2 ? r2 : rt ? rt : ro;
    return rc;
}
