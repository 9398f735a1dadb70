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
 * of sequences), so a plan never depends on host-side lengths: a serving
 * loop whose sequences grow by a token per step reuses one plan, and the
 * step (plan + decode + combine) can be replayed as one CUDA graph.
 */
#include "../../include/attention.h"
#include "../../include/hal.h"
#include "ct_internal.h"

namespace {

constexpr int kPlanThreads = 1024;

/* Block-wide exclusive scan of one value per thread (inclusive result in
 * the returned pair's second member's place: total via *total). */
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t *warp_sums, uint32_t *total) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t x = v;
    #pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, x, o);
        if (lane >= (uint32_t)o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        uint32_t w = lane < kPlanThreads / 32 ? warp_sums[lane] : 0;
        #pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, w, o);
            if (lane >= (uint32_t)o) w += y;
        }
        warp_sums[lane] = w;                     /* inclusive warp totals */
    }
    __syncthreads();
    const uint32_t before = (warp ? warp_sums[warp - 1] : 0) + x - v;
    *total = warp_sums[kPlanThreads / 32 - 1];
    __syncthreads();
    return before;
}

__global__ void __launch_bounds__(kPlanThreads) k_mla_plan(const uint32_t *rows, const int32_t *seq_lens,
                                                           uint32_t n_seq, uint32_t page_tokens, uint32_t max_pages,
                                                           uint32_t n_workers, ct_mla_chunk_t *chunks,
                                                           int32_t *worker_begin, ct_mla_combine_t *combines,
                                                           int32_t *counts) {
    __shared__ uint32_t warp_sums[32];
    const uint32_t per = (n_seq + kPlanThreads - 1) / kPlanThreads;
    const uint32_t s0 = min(n_seq, threadIdx.x * per), s1 = min(n_seq, s0 + per);
    auto pages_of = [&](uint32_t s) -> uint32_t {
        const int32_t len = seq_lens[rows ? rows[s] : s];
        if (len <= 0) return 0;
        return min(max_pages, ((uint32_t)len + page_tokens - 1) / page_tokens);
    };
    /* pass 1: this thread's pages */
    uint32_t my_pages = 0;
    for (uint32_t s = s0; s < s1; s++) my_pages += pages_of(s);
    uint32_t total_pages;
    const uint32_t page0 = block_exclusive_scan(my_pages, warp_sums, &total_pages);
    const uint32_t W = n_workers;
    const uint32_t Q = total_pages ? (total_pages + W - 1) / W : 1;
    /* pass 2: chunks, parts and combines of this thread's sequences */
    uint32_t my_chunks = 0, my_parts = 0, my_split = 0;
    {
        uint32_t cp = page0;
        for (uint32_t s = s0; s < s1; s++) {
            const uint32_t np = pages_of(s);
            const uint32_t n = np ? (cp + np - 1) / Q - cp / Q + 1 : 1;
            my_chunks += n;
            if (n > 1) { my_parts += n; my_split++; }
            cp += np;
        }
    }
    uint32_t total_chunks, total_parts, total_split;
    const uint32_t chunk0 = block_exclusive_scan(my_chunks, warp_sums, &total_chunks);
    const uint32_t part0 = block_exclusive_scan(my_parts, warp_sums, &total_parts);
    const uint32_t comb0 = block_exclusive_scan(my_split, warp_sums, &total_split);
    /* pass 3: write them; pad[0] of a chunk holds its worker */
    {
        uint32_t cp = page0, ci = chunk0, pi = part0, bi = comb0;
        for (uint32_t s = s0; s < s1; s++) {
            const uint32_t np = pages_of(s);
            const int32_t row = rows ? (int32_t)rows[s] : (int32_t)s;
            if (np == 0) {
                const uint32_t w = min(W - 1, cp / Q);
                chunks[ci++] = ct_mla_chunk_t{(int32_t)s, row, 0, 0, -1, {(int32_t)w, 0, 0}};
                continue;
            }
            const uint32_t w0 = cp / Q, w1 = (cp + np - 1) / Q, n = w1 - w0 + 1;
            if (n > 1) combines[bi++] = ct_mla_combine_t{(int32_t)s, (int32_t)pi, (int32_t)n, 0};
            for (uint32_t w = w0; w <= w1; w++) {
                const uint32_t g0 = max(cp, w * Q), g1 = min(cp + np, (w + 1) * Q);
                chunks[ci++] = ct_mla_chunk_t{(int32_t)s, row, (int32_t)(g0 - cp), (int32_t)(g1 - cp),
                                              n > 1 ? (int32_t)pi++ : -1, {(int32_t)w, 0, 0}};
            }
            cp += np;
        }
    }
    __syncthreads();                            /* chunks written: their workers are readable */
    /* worker_begin[w] = the first chunk whose worker is >= w */
    for (uint32_t c = threadIdx.x; c < total_chunks; c += kPlanThreads) {
        const int32_t w = chunks[c].pad[0];
        const int32_t wprev = c ? chunks[c - 1].pad[0] : -1;
        for (int32_t v = wprev + 1; v <= w; v++) worker_begin[v] = (int32_t)c;
    }
    if (threadIdx.x == 0) {
        const int32_t wlast = total_chunks ? chunks[total_chunks - 1].pad[0] : -1;
        for (int32_t v = wlast + 1; v <= (int32_t)W; v++) worker_begin[v] = (int32_t)total_chunks;
        counts[0] = (int32_t)total_chunks;
        counts[1] = (int32_t)total_split;
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
