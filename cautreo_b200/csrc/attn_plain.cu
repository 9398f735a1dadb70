/*
 * attn_plain.cu -- single-query decode attention over contiguous K/V.
 *
 *  k_attn_shared     the reference's ct_attn_forward contract
 *                    (attention.c:23-53): every head reads one shared
 *                    [n][D] K and V; fp64 dot and PV, fp32 scores, expf,
 *                    double softmax sum, probabilities normalised before PV.
 *  k_softmax         ct_attn_softmax (attention.c:11-21).
 *  k_decode_contig   the engine's per-layer loop (transformer.c:185-214) for
 *                    all layers and heads in one launch, over the
 *                    ct_kv_cache_t layout [L][max_ctx][Hkv*D], online
 *                    softmax in fp32 with FMA; optional fused append.
 */
#include "../../include/attention.h"
#include "../../include/hal.h"
#include "ct_internal.h"

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ double block_sum_d(double v, double *red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    double s = 0.0;
    if (threadIdx.x == 0) { for (int i = 0; i < (int)(blockDim.x >> 5); i++) s += red[i]; red[0] = s; }
    __syncthreads();
    return red[0];
}

__device__ __forceinline__ float block_max_f(float v, float *red) {
    v = ct_warp_max(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    if (threadIdx.x == 0) { float m = red[0]; for (int i = 1; i < (int)(blockDim.x >> 5); i++) m = fmaxf(m, red[i]); red[0] = m; }
    __syncthreads();
    return red[0];
}

/* One block per head.  scores: global scratch [H][n]. */
__global__ void __launch_bounds__(kThreads) k_attn_shared(const float *q, const float *k, const float *v,
                                                          uint32_t n, uint32_t D, float scale,
                                                          float *out, float *scores) {
    __shared__ double red_d[kThreads / 32];
    __shared__ float red_f[kThreads / 32];
    extern __shared__ double pv[];                   /* [groups][D] partial PV sums */
    const uint32_t h = blockIdx.x;
    const float *qh = q + (size_t)h * D;
    float *sc = scores + (size_t)h * n;
    float mx = -INFINITY;
    for (uint32_t t = threadIdx.x; t < n; t += kThreads) {
        double dot = 0.0;
        for (uint32_t i = 0; i < D; i++) dot += (double)qh[i] * (double)k[(size_t)t * D + i];
        const float s = __fmul_rn(scale, (float)dot);
        sc[t] = s;
        if (s > mx) mx = s;
    }
    /* The reference seeds its max with x[0] and keeps it unless a later score is larger. */
    mx = block_max_f(mx, red_f);
    double sum = 0.0;
    for (uint32_t t = threadIdx.x; t < n; t += kThreads) {
        const float e = expf(__fsub_rn(sc[t], mx));
        sc[t] = e;
        sum += (double)e;
    }
    sum = block_sum_d(sum, red_d);
    __syncthreads();
    if (sum > 0) for (uint32_t t = threadIdx.x; t < n; t += kThreads) sc[t] = (float)((double)sc[t] / sum);
    __syncthreads();
    /* PV: threads split over (token group, dim); partial sums combined in a fixed order. */
    const uint32_t nd = D < (uint32_t)kThreads ? D : (uint32_t)kThreads;
    const uint32_t groups = kThreads / nd;
    const uint32_t g = threadIdx.x / nd, i0 = threadIdx.x % nd;
    if (g < groups) {
        for (uint32_t i = i0; i < D; i += nd) {
            double acc = 0.0;
            for (uint32_t t = g; t < n; t += groups) acc += (double)sc[t] * (double)v[(size_t)t * D + i];
            pv[(size_t)g * D + i] = acc;
        }
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < D; i += kThreads) {
        double acc = 0.0;
        for (uint32_t gg = 0; gg < groups; gg++) acc += pv[(size_t)gg * D + i];
        out[(size_t)h * D + i] = (float)acc;
    }
}

__global__ void __launch_bounds__(kThreads) k_softmax(float *x, uint32_t n) {
    __shared__ double red_d[kThreads / 32];
    __shared__ float red_f[kThreads / 32];
    float mx = -INFINITY;
    for (uint32_t i = threadIdx.x; i < n; i += kThreads) mx = fmaxf(mx, x[i]);
    mx = block_max_f(mx, red_f);
    double sum = 0.0;
    for (uint32_t i = threadIdx.x; i < n; i += kThreads) { float e = expf(__fsub_rn(x[i], mx)); x[i] = e; sum += e; }
    sum = block_sum_d(sum, red_d);
    if (sum > 0) for (uint32_t i = threadIdx.x; i < n; i += kThreads) x[i] = (float)((double)x[i] / sum);
}

/* One block per (q head, layer).  Tokens in tiles of 256: one score per
 * thread (fp32 dot), block max, rescale, then PV with the block split into
 * token groups x head_dim lanes.  head_dim <= 256.  With k_new/v_new set the
 * block first stores token `pos` of its KV head and uses it directly. */
__global__ void __launch_bounds__(kThreads) k_decode_contig(const float *q, const float *k_new, const float *v_new,
                                                            float *k_cache, float *v_cache, uint32_t max_ctx,
                                                            uint32_t hkv, uint32_t hq, uint32_t D, uint32_t n,
                                                            float scale, float *out) {
    extern __shared__ float sm[];
    float *qs = sm;                      /* [D] */
    float *ps = qs + D;                  /* [256] probabilities of the tile */
    float *part = ps + kThreads;         /* [groups][D] */
    __shared__ float red_f[kThreads / 32];
    __shared__ float s_alpha;
    const uint32_t qh = blockIdx.x, l = blockIdx.y, kvh = qh % hkv;
    const size_t row_stride = (size_t)hkv * D;
    const float *kl = k_cache + (size_t)l * max_ctx * row_stride + (size_t)kvh * D;
    const float *vl = v_cache + (size_t)l * max_ctx * row_stride + (size_t)kvh * D;
    const uint32_t pos = n - 1;
    const float *kn = k_new ? k_new + (size_t)l * row_stride + (size_t)kvh * D : nullptr;
    const float *vn = v_new ? v_new + (size_t)l * row_stride + (size_t)kvh * D : nullptr;
    if (k_new && (qh < hkv)) {
        /* One writer per KV head: the block of query head == kv head. */
        for (uint32_t i = threadIdx.x; i < D; i += kThreads) {
            k_cache[((size_t)l * max_ctx + pos) * row_stride + (size_t)kvh * D + i] = kn[i];
            v_cache[((size_t)l * max_ctx + pos) * row_stride + (size_t)kvh * D + i] = vn[i];
        }
    }
    for (uint32_t i = threadIdx.x; i < D; i += kThreads) qs[i] = q[((size_t)l * hq + qh) * D + i];
    __syncthreads();
    const uint32_t groups = kThreads / D;            /* D <= 256 */
    const uint32_t g = threadIdx.x / D, di = threadIdx.x % D;
    float acc = 0.0f, m = -INFINITY, lsum = 0.0f;
    for (uint32_t t0 = 0; t0 < n; t0 += kThreads) {
        const uint32_t t = t0 + threadIdx.x;
        float s = -INFINITY;
        if (t < n) {
            const float *kr = (kn && t == pos) ? kn : kl + (size_t)t * row_stride;
            float dot = 0.0f;
            for (uint32_t i = 0; i < D; i++) dot = fmaf(qs[i], kr[i], dot);
            s = dot * scale;
        }
        const float tmax = block_max_f(s, red_f);
        const float m_new = fmaxf(m, tmax);
        const float p = t < n ? __expf(s - m_new) : 0.0f;
        ps[threadIdx.x] = p;
        if (threadIdx.x == 0) s_alpha = __expf(m - m_new);
        __syncthreads();
        const float alpha = s_alpha;
        lsum = lsum * alpha + ct_warp_sum(p);        /* per-warp partial, reduced at the end */
        m = m_new;
        acc *= alpha;
        if (g < groups) {
            const uint32_t tend = (n - t0) < (uint32_t)kThreads ? (n - t0) : (uint32_t)kThreads;
            for (uint32_t j = g; j < tend; j += groups) {
                const uint32_t tt = t0 + j;
                const float vv = (vn && tt == pos) ? vn[di] : vl[(size_t)tt * row_stride + di];
                acc = fmaf(ps[j], vv, acc);
            }
        }
        __syncthreads();
    }
    /* l: each warp holds the sum of its lanes' probabilities (same in all lanes). */
    if ((threadIdx.x & 31) == 0) red_f[threadIdx.x >> 5] = lsum;
    if (g < groups) part[g * D + di] = acc;
    __syncthreads();
    if (threadIdx.x < D) {
        float L = 0.0f;
        for (int w = 0; w < kThreads / 32; w++) L += red_f[w];
        float o = 0.0f;
        for (uint32_t gg = 0; gg < groups; gg++) o += part[gg * D + threadIdx.x];
        out[((size_t)l * hq + qh) * D + threadIdx.x] = L > 0.0f ? o / L : 0.0f;
    }
}

int launch_decode(const float *q, const float *k_new, const float *v_new, float *k_cache, float *v_cache,
                  uint32_t n_layers, uint32_t max_ctx, uint32_t hkv, uint32_t hq, uint32_t D, uint32_t n,
                  float scale, float *out, void *stream) {
    if (!q || !k_cache || !v_cache || !out || n == 0 || n > max_ctx || hkv == 0 || hq == 0 || D == 0 || D > 256)
        return CT_ERR_ARG;
    if (scale == 0.0f) scale = 1.0f / sqrtf((float)D);
    const uint32_t groups = kThreads / D;
    const size_t smem = (D + kThreads + (size_t)groups * D) * sizeof(float);
    k_decode_contig<<<dim3(hq, n_layers), kThreads, smem, (cudaStream_t)stream>>>(
        q, k_new, v_new, k_cache, v_cache, max_ctx, hkv, hq, D, n, scale, out);
    ct__count_launches(1);
    return ct__cuda_status(cudaGetLastError(), "decode_contig");
}

}  // namespace

extern "C" int ct__launch_attn_shared(const float *q, const float *k, const float *v, uint32_t n_tokens,
                                      uint32_t n_heads, uint32_t head_dim, float scale, float *out,
                                      float *scratch_scores, void *stream) {
    if (n_heads == 0) return CT_OK;
    const uint32_t nd = head_dim < (uint32_t)kThreads ? head_dim : (uint32_t)kThreads;
    const size_t smem = (size_t)(kThreads / nd) * head_dim * sizeof(double);
    if (smem > 200 * 1024) return CT_ERR_UNSUPPORTED;
    if (smem > 48 * 1024)
        cudaFuncSetAttribute(k_attn_shared, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_attn_shared<<<n_heads, kThreads, smem, (cudaStream_t)stream>>>(q, k, v, n_tokens, head_dim, scale, out,
                                                                    scratch_scores);
    ct__count_launches(1);
    return ct__cuda_status(cudaGetLastError(), "attn_shared");
}

extern "C" int ct__launch_softmax(float *x, uint32_t n, void *stream) {
    k_softmax<<<1, kThreads, 0, (cudaStream_t)stream>>>(x, n);
    ct__count_launches(1);
    return ct__cuda_status(cudaGetLastError(), "softmax");
}

extern "C" int ct_attn_decode_contig(const float *q, const float *k_cache, const float *v_cache,
                                     uint32_t n_layers, uint32_t max_ctx, uint32_t n_kv_heads,
                                     uint32_t n_q_heads, uint32_t head_dim, uint32_t n_tokens,
                                     float scale, float *out, void *stream) {
    return launch_decode(q, nullptr, nullptr, const_cast<float *>(k_cache), const_cast<float *>(v_cache),
                         n_layers, max_ctx, n_kv_heads, n_q_heads, head_dim, n_tokens, scale, out, stream);
}

extern "C" int ct_attn_decode_step_contig(const float *q, const float *k_new, const float *v_new,
                                          float *k_cache, float *v_cache, uint32_t n_layers,
                                          uint32_t max_ctx, uint32_t n_kv_heads, uint32_t n_q_heads,
                                          uint32_t head_dim, uint32_t pos, float scale, float *out,
                                          void *stream) {
    if (!k_new || !v_new) return CT_ERR_ARG;
    return launch_decode(q, k_new, v_new, k_cache, v_cache, n_layers, max_ctx, n_kv_heads, n_q_heads,
                         head_dim, pos + 1, scale, out, stream);
}
