/*
 * mla_plan.cu -- the MLA decode work list, built on the device from the
 * current sequence lengths at every decode.
 *
 * Every page of every sequence costs one tile of the decode kernels, so the
 * work is balanced by pages: the sequences' pages are laid end to end
 * (sequence order), and worker w takes the global pages [w*Q, (w+1)*Q) with
 * Q = ceil(total / W).  Each sequence becomes one chunk per worker its pages
 * meet; a sequence met by several workers writes partial results (one slot
 * per chunk) that the combine merges.  An empty sequence is one chunk of no
 * pages, given to the worker its position falls in, which writes zeros.
 *
 * One block of 1024 threads scans the lengths (each thread a contiguous run
 * of sequences; two block scans, the second over chunk, part and split
 * counts at once), so a plan never depends on host-side lengths: a serving
 * loop whose sequences grow by a token per step reuses one plan, and the
 * step (plan + decode + combine) can be replayed as one CUDA graph.
 */
#include "../../include/attention.h"
#include "../../include/hal.h"
#include "ct_internal.h"

namespace {

constexpr int kPlanThreads = 1024;
constexpr uint32_t kCache = 4;                  /* page counts a thread keeps in registers */

/* Block-wide exclusive scan of N values per thread at once (one set of
 * barriers for all N); the block totals go to total[]. */
template <int N>
__device__ __forceinline__ void block_exclusive_scan(const uint32_t (&v)[N], uint32_t (&before)[N],
                                                     uint32_t (&total)[N], uint32_t (*warp_sums)[32]) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t x[N];
    #pragma unroll
    for (int i = 0; i < N; i++) x[i] = v[i];
    #pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        #pragma unroll
        for (int i = 0; i < N; i++) {
            const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, x[i], o);
            if (lane >= (uint32_t)o) x[i] += y;
        }
    }
    if (lane == 31) {
        #pragma unroll
        for (int i = 0; i < N; i++) warp_sums[i][warp] = x[i];
    }
    __syncthreads();
    if (warp < (uint32_t)N) {                   /* warp i scans the warp totals of value i */
        uint32_t w = lane < kPlanThreads / 32 ? warp_sums[warp][lane] : 0;
        #pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, w, o);
            if (lane >= (uint32_t)o) w += y;
        }
        warp_sums[warp][lane] = w;              /* inclusive warp totals */
    }
    __syncthreads();
    #pragma unroll
    for (int i = 0; i < N; i++) {
        before[i] = (warp ? warp_sums[i][warp - 1] : 0) + x[i] - v[i];
        total[i] = warp_sums[i][kPlanThreads / 32 - 1];
    }
    __syncthreads();                            /* warp_sums may be reused */
}

__global__ void __launch_bounds__(kPlanThreads) k_mla_plan(const uint32_t *rows, const int32_t *seq_lens,
                                                           uint32_t n_seq, uint32_t page_tokens, uint32_t max_pages,
                                                           uint32_t n_workers, ct_mla_chunk_t *chunks,
                                                           int32_t *worker_begin, ct_mla_combine_t *combines,
                                                           int32_t *counts) {
    __shared__ uint32_t warp_sums[3][32];
    __shared__ int32_t last_worker[kPlanThreads];       /* worker of each thread's last chunk */
    const uint32_t per = (n_seq + kPlanThreads - 1) / kPlanThreads;
    const uint32_t s0 = min(n_seq, threadIdx.x * per), s1 = min(n_seq, s0 + per);
    auto pages_of = [&](uint32_t s) -> uint32_t {
        const int32_t len = seq_lens[rows ? rows[s] : s];
        if (len <= 0) return 0;
        return min(max_pages, ((uint32_t)len + page_tokens - 1) / page_tokens);
    };
    /* this thread's sequences' page counts (the first kCache kept) */
    uint32_t cached[kCache];
    #pragma unroll
    for (uint32_t k = 0; k < kCache; k++) cached[k] = s0 + k < s1 ? pages_of(s0 + k) : 0;
    auto np_of = [&](uint32_t s) -> uint32_t {
        const uint32_t k = s - s0;
        if (k < kCache) {
            uint32_t r = cached[0];
            #pragma unroll
            for (uint32_t j = 1; j < kCache; j++) r = k == j ? cached[j] : r;
            return r;
        }
        return pages_of(s);
    };
    uint32_t my[1] = {0}, page0[1], total_pages[1];
    for (uint32_t s = s0; s < s1; s++) my[0] += np_of(s);
    block_exclusive_scan<1>(my, page0, total_pages, warp_sums);
    const uint32_t W = n_workers;
    const uint32_t Q = total_pages[0] ? (total_pages[0] + W - 1) / W : 1;
    /* chunks, parts and combines of this thread's sequences */
    uint32_t cnt[3] = {0, 0, 0};                /* chunks, parts, split sequences */
    {
        uint32_t cp = page0[0];
        for (uint32_t s = s0; s < s1; s++) {
            const uint32_t np = np_of(s);
            const uint32_t n = np ? (cp + np - 1) / Q - cp / Q + 1 : 1;
            cnt[0] += n;
            if (n > 1) { cnt[1] += n; cnt[2]++; }
            cp += np;
        }
    }
    uint32_t first[3], tot[3];
    block_exclusive_scan<3>(cnt, first, tot, warp_sums);
    /* write them; pad[0] of a chunk holds its worker */
    int32_t wlast = -1;
    {
        uint32_t cp = page0[0], ci = first[0], pi = first[1], bi = first[2];
        for (uint32_t s = s0; s < s1; s++) {
            const uint32_t np = np_of(s);
            const int32_t row = rows ? (int32_t)rows[s] : (int32_t)s;
            if (np == 0) {
                const uint32_t w = min(W - 1, cp / Q);
                chunks[ci++] = ct_mla_chunk_t{(int32_t)s, row, 0, 0, -1, {(int32_t)w, 0, 0}};
                wlast = (int32_t)w;
                continue;
            }
            const uint32_t w0 = cp / Q, w1 = (cp + np - 1) / Q, n = w1 - w0 + 1;
            if (n > 1) combines[bi++] = ct_mla_combine_t{(int32_t)s, (int32_t)pi, (int32_t)n, 0};
            for (uint32_t w = w0; w <= w1; w++) {
                const uint32_t g0 = max(cp, w * Q), g1 = min(cp + np, (w + 1) * Q);
                chunks[ci++] = ct_mla_chunk_t{(int32_t)s, row, (int32_t)(g0 - cp), (int32_t)(g1 - cp),
                                              n > 1 ? (int32_t)pi++ : -1, {(int32_t)w, 0, 0}};
            }
            wlast = (int32_t)w1;
            cp += np;
        }
    }
    last_worker[threadIdx.x] = wlast;
    __syncthreads();
    /* worker_begin[w] = the first chunk whose worker is >= w: each thread
     * fills the workers from its previous chunk's (the previous thread's
     * last, for its first chunk) to each of its chunks' */
    {
        int32_t wprev = threadIdx.x ? last_worker[threadIdx.x - 1] : -1;
        uint32_t cp = page0[0], ci = first[0];
        for (uint32_t s = s0; s < s1; s++) {
            const uint32_t np = np_of(s);
            const uint32_t w0 = np ? cp / Q : min(W - 1, cp / Q), w1 = np ? (cp + np - 1) / Q : w0;
            for (uint32_t w = w0; w <= w1; w++, ci++) {
                for (int32_t v = wprev + 1; v <= (int32_t)w; v++) worker_begin[v] = (int32_t)ci;
                wprev = (int32_t)w;
            }
            cp += np;
        }
    }
    if (threadIdx.x == 0) {
        const int32_t wl = n_seq ? last_worker[(n_seq - 1) / per] : -1;
        for (int32_t v = wl + 1; v <= (int32_t)W; v++) worker_begin[v] = (int32_t)tot[0];
        counts[0] = (int32_t)tot[0];
        counts[1] = (int32_t)tot[2];
    }
}

}  // namespace

extern "C" int ct__launch_mla_plan(const uint32_t *rows, const int32_t *seq_lens, uint32_t n_seq, uint32_t page_tokens,
                                   uint32_t max_pages, uint32_t n_workers, ct_mla_chunk_t *chunks,
                                   int32_t *worker_begin, ct_mla_combine_t *combines, int32_t *counts, void *stream) {
    if (!seq_lens || !chunks || !worker_begin || !combines || !counts || page_tokens == 0 || n_workers == 0)
        return CT_ERR_ARG;
    k_mla_plan<<<1, kPlanThreads, 0, (cudaStream_t)stream>>>(rows, seq_lens, n_seq, page_tokens, max_pages, n_workers,
                                                            chunks, worker_begin, combines, counts);
    return ct__cuda_status(cudaGetLastError(), "mla_plan");
}
