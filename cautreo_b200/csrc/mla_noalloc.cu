/*
 * mla_noalloc.cu -- paged MLA decode for callers that must not allocate.
 *
 * ct_attn_mla_decode_paged needs a plan (ct_mla_plan_create), which
 * cudaMallocs its work list and its split-KV scratch.  Some callers cannot do
 * that on their decode path: an inference engine that reserves nearly all
 * device memory for its KV pool at start-up (a later cudaMalloc would fail
 * with out-of-memory), or a serving loop with a hard per-token latency budget
 * that forbids allocator calls and their implicit synchronisation once it is
 * running.  ct_attn_mla_decode_paged_noalloc plans on the host into static
 * arrays and keeps its device-side work list and partial results in
 * g_mla_noalloc_scratch, a file-scope device array of
 * CT_MLA_NOALLOC_SCRATCH_BYTES that every GPU loading this library holds until
 * the process exits.  It then runs the same kernels as
 * ct_attn_mla_decode_paged.
 *
 * Host code cannot use the array's name as a device address, so each device
 * resolves it once with cudaGetSymbolAddress (with that device current) on
 * its first call, which should therefore come before any stream capture.
 * Every call shares the array and finds the previous call's contents there;
 * nothing in it has to start at zero, because each call writes every work
 * item and partial slot before reading it.  Calls that overlap on the GPU
 * (two streams, or two host threads) race on the array and on the static
 * host staging, so callers must serialise them.
 */
#include "../../include/attention.h"
#include "../../include/hal.h"
#include "../../include/kv_cache.h"
#include "ct_internal.h"

#include <string.h>

namespace {

constexpr size_t kScratchBytes = CT_MLA_NOALLOC_SCRATCH_BYTES;
constexpr uint32_t kMaxSeqs = CT_MLA_NOALLOC_MAX_SEQS;
constexpr uint32_t kMaxWorkers = 60;                 /* bounds the split sequences, hence the partials */
constexpr uint32_t kMaxChunks = kMaxSeqs + kMaxWorkers + 8;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_mla_noalloc_scratch[kScratchBytes];

void *g_scratch_addr[kMaxDevices];                    /* device address of the array, per device */

/* Host staging of the work list (static: no host allocation either). */
ct_mla_chunk_t g_chunks[kMaxChunks];
int32_t g_worker_begin[kMaxWorkers + 1];
ct_mla_combine_t g_combines[kMaxSeqs];
int32_t g_first_chunk[kMaxSeqs];
int32_t g_n_of[kMaxSeqs];

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

/* Resolves the array's device address for the current device, once. */
int scratch_for_current_device(void **out) {
    int dev = 0;
    int rc = ct__cuda_status(cudaGetDevice(&dev), "mla_noalloc: cudaGetDevice");
    if (rc) return rc;
    if (dev < 0 || dev >= kMaxDevices) {
        ct__set_error("ct_attn_mla_decode_paged_noalloc: device ordinal beyond 63");
        return CT_ERR_UNSUPPORTED;
    }
    if (!g_scratch_addr[dev]) {
        void *p = nullptr;
        rc = ct__cuda_status(cudaGetSymbolAddress(&p, g_mla_noalloc_scratch), "mla_noalloc: cudaGetSymbolAddress");
        if (rc) return rc;
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return CT_OK;
}

}  // namespace

extern "C" int ct__mla_tc_workers(const ct_mla_dims_t *dims, int device);

extern "C" int ct_attn_mla_decode_paged_noalloc(const ct_mla_shape_t *shape, const int32_t *seq_lens_host,
                                                uint32_t n_seq, const void *q, const void *pool,
                                                const float *scales, const int32_t *block_table,
                                                const int32_t *seq_lens, void *out, float *lse, void *stream) {
    if (!shape || !seq_lens_host || !q || !pool || !block_table || !seq_lens || !out) return CT_ERR_ARG;
    if (shape->n_heads == 0 || shape->page_tokens == 0 || shape->entry_dim == 0 || shape->v_dim > shape->entry_dim ||
        shape->max_pages_per_seq == 0 || shape->n_pages == 0) {
        ct__set_error("ct_attn_mla_decode_paged_noalloc: bad shape");
        return CT_ERR_ARG;
    }
    if ((shape->kv_dtype == CT_KV_INT8 || shape->kv_dtype == CT_KV_E4M3) && !scales) return CT_ERR_ARG;
    if (n_seq > kMaxSeqs) {
        ct__set_error("ct_attn_mla_decode_paged_noalloc: more than CT_MLA_NOALLOC_MAX_SEQS sequences");
        return CT_ERR_ARG;
    }
    ct_mla_dims_t dims;
    dims.n_heads = shape->n_heads;
    dims.entry_dim = shape->entry_dim;
    dims.v_dim = shape->v_dim;
    dims.page_tokens = shape->page_tokens;
    dims.max_pages_per_seq = shape->max_pages_per_seq;
    dims.kv_dtype = shape->kv_dtype;
    dims.scale = shape->scale;
    dims.n_pages = shape->n_pages;
    dims.n_seq = n_seq;
    const uint32_t P = shape->page_tokens;

    void *scratch = nullptr;
    int rc = scratch_for_current_device(&scratch);
    if (rc) return rc;
    int dev = 0, n_sms = 148;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        cudaGetLastError();
        n_sms = 148;
    }
    const int tc = ct__mla_tc_workers(&dims, dev);
    uint32_t W = tc > 0 ? (uint32_t)tc : (uint32_t)n_sms;
    if (W > kMaxWorkers) W = kMaxWorkers;

    /* Balanced split: sequences end to end, cut into W equal token ranges at
     * page boundaries (the same rule as ct_mla_plan_create, fewer workers). */
    uint64_t total = 0;
    for (uint32_t s = 0; s < n_seq; s++) {
        if (seq_lens_host[s] < 0 || (uint64_t)(seq_lens_host[s] + P - 1) / P > shape->max_pages_per_seq) {
            ct__set_error("ct_attn_mla_decode_paged_noalloc: sequence longer than its block-table row");
            return CT_ERR_ARG;
        }
        total += (uint64_t)seq_lens_host[s];
    }
    const uint64_t quota = total / W + 1;
    uint32_t nc = 0, w = 0;
    uint64_t filled = 0;
    g_worker_begin[0] = 0;
    for (uint32_t s = 0; s < n_seq; s++) {
        const uint32_t pages = ((uint32_t)seq_lens_host[s] + P - 1) / P;
        g_first_chunk[s] = (int32_t)nc;
        g_n_of[s] = 0;
        if (pages == 0) {
            g_chunks[nc++] = ct_mla_chunk_t{(int32_t)s, (int32_t)s, 0, 0, -1, {0, 0, 0}};
            g_n_of[s] = 1;
            continue;
        }
        uint32_t pg = 0;
        while (pg < pages) {
            uint64_t room = quota > filled ? quota - filled : 0;
            uint32_t take = (uint32_t)((room + P / 2) / P);
            if (take == 0) take = 1;
            if (w + 1 >= W || take > pages - pg) take = pages - pg;
            if (nc >= kMaxChunks) {
                ct__set_error("ct_attn_mla_decode_paged_noalloc: work list exceeds its static capacity");
                return CT_ERR_ARG;
            }
            g_chunks[nc++] = ct_mla_chunk_t{(int32_t)s, (int32_t)s, (int32_t)pg, (int32_t)(pg + take), 0, {0, 0, 0}};
            g_n_of[s]++;
            uint64_t tok = (uint64_t)take * P;
            if (pg + take == pages) tok = (uint64_t)seq_lens_host[s] - (uint64_t)pg * P;
            pg += take;
            filled += tok;
            if (filled + P / 2 >= quota && w + 1 < W) { g_worker_begin[++w] = (int32_t)nc; filled = 0; }
        }
    }
    while (w < W) g_worker_begin[++w] = (int32_t)nc;
    uint32_t parts = 0, ncb = 0;
    for (uint32_t s = 0; s < n_seq; s++) {
        if (g_n_of[s] <= 1) { g_chunks[g_first_chunk[s]].part = -1; continue; }
        g_combines[ncb++] = ct_mla_combine_t{(int32_t)s, (int32_t)parts, g_n_of[s], 0};
        for (int32_t i = 0; i < g_n_of[s]; i++) g_chunks[g_first_chunk[s] + i].part = (int32_t)(parts++);
    }

    /* Scratch layout: chunks | worker_begin | combines | (m, l) | partial o. */
    const size_t off_wb = align256((size_t)nc * sizeof(ct_mla_chunk_t));
    const size_t off_cb = off_wb + align256((size_t)(W + 1) * sizeof(int32_t));
    const size_t off_ml = off_cb + align256((size_t)(ncb ? ncb : 1) * sizeof(ct_mla_combine_t));
    const size_t off_o = off_ml + align256((size_t)(parts ? parts : 1) * shape->n_heads * 4 * sizeof(float));
    const size_t need = off_o + (size_t)(parts ? parts : 1) * shape->n_heads * shape->v_dim * sizeof(float);
    if (need > kScratchBytes) {
        ct__set_error("ct_attn_mla_decode_paged_noalloc: this batch needs more than CT_MLA_NOALLOC_SCRATCH_BYTES "
                      "of scratch (too many heads x value dims for its split sequences)");
        return CT_ERR_ARG;
    }
    unsigned char *base = static_cast<unsigned char *>(scratch);
    cudaStream_t st = (cudaStream_t)stream;
    /* From pageable host memory: each copy returns once the source has been
     * taken, so the static staging may be reused by the next call. */
    rc = ct__cuda_status(cudaMemcpyAsync(base, g_chunks, (size_t)nc * sizeof(ct_mla_chunk_t), cudaMemcpyHostToDevice, st),
                         "mla_noalloc: work list");
    if (!rc) rc = ct__cuda_status(cudaMemcpyAsync(base + off_wb, g_worker_begin, (size_t)(W + 1) * sizeof(int32_t),
                                                  cudaMemcpyHostToDevice, st), "mla_noalloc: workers");
    if (!rc && ncb)
        rc = ct__cuda_status(cudaMemcpyAsync(base + off_cb, g_combines, (size_t)ncb * sizeof(ct_mla_combine_t),
                                             cudaMemcpyHostToDevice, st), "mla_noalloc: combines");
    if (rc) return rc;
    uint32_t launches = 0;
    return ct__launch_mla_decode(&dims, reinterpret_cast<const ct_mla_chunk_t *>(base), nc,
                                 reinterpret_cast<const int32_t *>(base + off_wb), W,
                                 reinterpret_cast<const ct_mla_combine_t *>(base + off_cb), ncb, nullptr, q, pool, scales,
                                 block_table, seq_lens, out, lse, reinterpret_cast<float *>(base + off_o),
                                 reinterpret_cast<float *>(base + off_ml), stream, &launches);
}
