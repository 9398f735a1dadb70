/*
 * attn_plain.cu -- single-query decode attention over contiguous K/V.
 *
 *  k_attn_shared     the reference's ct_attn_forward contract
 *                    (attention.c:23-53): every head reads one shared
 *                    [n][D] K and V; fp64 dot and PV, fp32 scores, expf,
 *                    double softmax sum, probabilities normalised before PV.
 *  k_softmax         ct_attn_softmax (attention.c:11-21).
 *  k_attn_part / k_attn_merge, k_softmax_max / _exp / _norm: the same two
 *                    contracts for long inputs, spread over many CTAs (a
 *                    single CTA per head reads at a few GB/s).
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

/* ---- long inputs ----------------------------------------------------------- */

__device__ __forceinline__ double warp_sum_d(double v) {
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

/* The reference's maximum: seeded with the first value, replaced only by a
 * larger one (a NaN is skipped unless it is the seed). */
__device__ __forceinline__ float ref_max(float m, float x) { return x > m ? x : m; }

/* ct_attn_forward for long contexts, part 1: a CTA per tile of `tile`
 * tokens, every head.  Scores as the reference forms them (fp64 dot, fp32
 * scale * dot), the tile's maximum m, e_t = expf(s_t - m), l = sum e_t and
 * o = sum e_t v_t in fp64, stored as part[(tile H + h)(D + 2) + {0, 1, 2..}]
 * = (m, l, o).  The K and V tiles and the queries are staged in shared
 * memory as fp64 (each value converted once: the products of two fp32
 * values are exact in fp64, as in the reference); a warp forms a score with
 * its lanes over the head dims, and the value sums split the tile's tokens
 * between thread groups. */
__global__ void __launch_bounds__(kThreads) k_attn_part(const float *q, const float *k, const float *v, uint32_t n,
                                                        uint32_t H, uint32_t D, float scale, uint32_t tile,
                                                        double *part) {
    extern __shared__ double sm_d[];
    double *ks = sm_d, *vs = ks + (size_t)tile * D, *qs = vs + (size_t)tile * D, *es = qs + (size_t)H * D;
    double *po = es + tile;                                    /* [kThreads] group sums */
    __shared__ double s_l;
    __shared__ float s_m;
    float *ss = reinterpret_cast<float *>(po + kThreads);     /* [tile] fp32 scores */
    const uint32_t t0 = blockIdx.x * tile, cnt = min(tile, n - t0);
    for (uint32_t i = threadIdx.x; i < cnt * D; i += kThreads) {
        ks[i] = (double)__ldg(k + (size_t)t0 * D + i);
        vs[i] = (double)__ldg(v + (size_t)t0 * D + i);
    }
    for (uint32_t i = threadIdx.x; i < H * D; i += kThreads) qs[i] = (double)__ldg(q + i);
    __syncthreads();
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t W = D < (uint32_t)kThreads ? D : (uint32_t)kThreads, G = (uint32_t)kThreads / W, g = threadIdx.x / W;
    for (uint32_t h = 0; h < H; h++) {
        const double *qh = qs + (size_t)h * D;
        for (uint32_t t = warp; t < cnt; t += kThreads / 32) {
            double dot = 0.0;
            for (uint32_t i = lane; i < D; i += 32) dot = fma(qh[i], ks[(size_t)t * D + i], dot);
            dot = warp_sum_d(dot);
            if (lane == 0) ss[t] = scale * (float)dot;
        }
        __syncthreads();
        if (warp == 0) {
            float m = ss[0];
            for (uint32_t t = lane; t < cnt; t += 32) m = ref_max(m, ss[t]);
            #pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = ref_max(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
            if (lane == 0) s_m = m;
        }
        __syncthreads();
        const float m = s_m;
        for (uint32_t t = threadIdx.x; t < cnt; t += kThreads) es[t] = (double)expf(ss[t] - m);
        __syncthreads();
        if (warp == 0) {
            double l = 0.0;
            for (uint32_t t = lane; t < cnt; t += 32) l += es[t];
            l = warp_sum_d(l);
            if (lane == 0) s_l = l;
        }
        double *ph = part + ((size_t)blockIdx.x * H + h) * (D + 2);
        for (uint32_t i0 = 0; i0 < D; i0 += W) {
            const uint32_t i = i0 + threadIdx.x % W;
            double acc = 0.0;
            if (g < G && i < D)
                for (uint32_t t = g; t < cnt; t += G) acc = fma(es[t], vs[(size_t)t * D + i], acc);
            po[threadIdx.x] = acc;
            __syncthreads();
            if (g == 0 && i < D) {
                double a = 0.0;
                for (uint32_t gg = 0; gg < G; gg++) a += po[gg * W + threadIdx.x];
                ph[2 + i] = a;
            }
            __syncthreads();
        }
        if (threadIdx.x == 0) {
            ph[0] = (double)m;
            ph[1] = s_l;
        }
    }
}

/* Part 2: merges items (m, l, o) of a head, in two levels.  CTA (h, s) takes
 * the items [s n / S, (s + 1) n / S): M = the reference maximum over their
 * m (seeded with the head's first item in CTA s = 0, as the reference seeds
 * its maximum with the first score; below every value elsewhere), f_b =
 * exp(m_b - M) (1 where m_b = M), L = sum f_b l_b, O = sum f_b o_b; with
 * `out` it writes O / L, else the record (M, L, O) at rec[(s H + h)(D + 2)].
 * Each f_b overwrites m_b, so the dims' pass reads it back. */
__global__ void __launch_bounds__(kThreads) k_attn_merge(double *part, uint32_t n_items, uint32_t H, uint32_t D,
                                                         double *rec, float *out) {
    __shared__ float red_m[kThreads / 32];
    __shared__ double red_l[kThreads / 32];
    __shared__ double red_o[kThreads];
    const uint32_t h = blockIdx.x, s = blockIdx.y, S = gridDim.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t b0 = (uint32_t)((uint64_t)n_items * s / S), b1 = (uint32_t)((uint64_t)n_items * (s + 1) / S);
    const size_t stride = (size_t)H * (D + 2);
    double *p0 = part + (size_t)h * (D + 2);
    float M = s == 0 ? (float)p0[0] : -INFINITY;
    for (uint32_t b = b0 + threadIdx.x; b < b1; b += kThreads) M = ref_max(M, (float)p0[b * stride]);
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = ref_max(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
    if (lane == 0) red_m[warp] = M;
    __syncthreads();
    M = red_m[0];
    for (int w = 1; w < kThreads / 32; w++) M = ref_max(M, red_m[w]);
    double L = 0.0;
    for (uint32_t b = b0 + threadIdx.x; b < b1; b += kThreads) {
        double *pb = p0 + b * stride;
        const float mb = (float)pb[0];
        const double f = mb == M ? 1.0 : exp((double)(mb - M));
        L += f * pb[1];
        pb[0] = f;
    }
    L = warp_sum_d(L);
    if (lane == 0) red_l[warp] = L;
    __syncthreads();                               /* also orders the f_b writes before their reads */
    L = 0.0;
    for (int w = 0; w < kThreads / 32; w++) L += red_l[w];
    /* the dims: kThreads / D groups of threads take every G-th item (D <
     * kThreads), eight items' loads in flight per thread; the groups' sums
     * are added in group order */
    const uint32_t W = D < (uint32_t)kThreads ? D : (uint32_t)kThreads;
    const uint32_t G = (uint32_t)kThreads / W, g = threadIdx.x / W;
    double *r = rec ? rec + ((size_t)s * H + h) * (D + 2) : nullptr;
    for (uint32_t i0 = 0; i0 < D; i0 += W) {
        const uint32_t i = i0 + threadIdx.x % W;
        double acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (g < G && i < D) {
            uint32_t b = b0 + g;
            for (; b + 7 * G < b1; b += 8 * G) {
                #pragma unroll
                for (int j = 0; j < 8; j++) {
                    const double *pb = p0 + (size_t)(b + j * G) * stride;
                    acc[j] += pb[0] * pb[2 + i];
                }
            }
            for (; b < b1; b += G) acc[0] += p0[(size_t)b * stride] * p0[(size_t)b * stride + 2 + i];
        }
        const double a = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
        __syncthreads();
        red_o[threadIdx.x] = a;
        __syncthreads();
        if (g == 0 && i < D) {
            double t = 0.0;
            for (uint32_t gg = 0; gg < G; gg++) t += red_o[gg * W + threadIdx.x];
            if (out) out[(size_t)h * D + i] = (float)(L > 0.0 ? t / L : t);
            else r[2 + i] = t;
        }
    }
    if (r && threadIdx.x == 0) {
        r[0] = (double)M;
        r[1] = L;
    }
}

/* ct_attn_softmax for long inputs: per-CTA maxima, then x = expf(x - M)
 * with per-CTA fp64 sums, then x = x / S; every CTA forms M and S from the
 * per-CTA values in the same order, so all use the same M and S. */
__global__ void __launch_bounds__(kThreads) k_softmax_max(const float *x, uint32_t n, uint32_t per, float *bmax) {
    __shared__ float red[kThreads / 32];
    const uint32_t a = blockIdx.x * per, e = min(n, a + per), warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    /* seeded as the reference's loop is: x[0] for the whole array, so other
     * CTAs start below every value (a NaN is then skipped everywhere else) */
    float m = blockIdx.x == 0 ? x[0] : -INFINITY;
    for (uint32_t i = a + threadIdx.x; i < e; i += kThreads) m = ref_max(m, x[i]);
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = ref_max(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float mm = red[0];
        for (int w = 1; w < kThreads / 32; w++) mm = ref_max(mm, red[w]);
        bmax[blockIdx.x] = mm;
    }
}

__global__ void __launch_bounds__(kThreads) k_softmax_exp(float *x, uint32_t n, uint32_t per, const float *bmax,
                                                          uint32_t nb, double *bsum) {
    __shared__ double red[kThreads / 32];
    __shared__ float red_m[kThreads / 32];
    const uint32_t a = blockIdx.x * per, e = min(n, a + per), warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    /* M: the seed bmax[0] (NaN when x[0] is), then the other CTAs' maxima,
     * none of them NaN, reduced in parallel */
    float mo = -INFINITY;
    for (uint32_t b = 1 + threadIdx.x; b < nb; b += kThreads) mo = fmaxf(mo, bmax[b]);
    mo = ct_warp_max(mo);
    if (lane == 0) red_m[warp] = mo;
    __syncthreads();
    for (int w = 0; w < kThreads / 32; w++) mo = fmaxf(mo, red_m[w]);
    const float M = ref_max(bmax[0], mo);
    /* a thread's values summed in fp32 with a compensation term (Kahan), its
     * total then in fp64: per-value fp64 work runs slowly on this part */
    float s32 = 0.0f, comp = 0.0f;
    auto add = [&](float y) {
        const float yy = __fsub_rn(y, comp), t = __fadd_rn(s32, yy);
        comp = __fsub_rn(__fsub_rn(t, s32), yy);
        s32 = t;
    };
    uint32_t i = a + threadIdx.x;
    for (; i + 7 * kThreads < e; i += 8 * kThreads) {      /* eight loads in flight before any store */
        float y[8];
        #pragma unroll
        for (int j = 0; j < 8; j++) y[j] = x[i + j * kThreads];
        #pragma unroll
        for (int j = 0; j < 8; j++) {
            y[j] = expf(y[j] - M);
            x[i + j * kThreads] = y[j];
            add(y[j]);
        }
    }
    for (; i < e; i += kThreads) {
        const float y = expf(x[i] - M);
        x[i] = y;
        add(y);
    }
    double s = (double)s32 - (double)comp;
    s = warp_sum_d(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < kThreads / 32; w++) t += red[w];
        bsum[blockIdx.x] = t;
    }
}

__global__ void __launch_bounds__(kThreads) k_softmax_norm(float *x, uint32_t n, uint32_t per, const double *bsum,
                                                           uint32_t nb) {
    __shared__ float s_r;
    __shared__ double red[kThreads / 32];
    /* S, the same in every CTA: thread t adds the sums t, t + kThreads, ...
     * in order, then the warps' and the block's totals in a fixed order */
    double part = 0.0;
    for (uint32_t b = threadIdx.x; b < nb; b += kThreads) part += bsum[b];
    part = warp_sum_d(part);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = part;
    __syncthreads();
    if (threadIdx.x == 0) {
        double S = 0.0;
        for (int w = 0; w < kThreads / 32; w++) S += red[w];
        s_r = S > 0.0 ? (float)(1.0 / S) : 0.0f;
    }
    __syncthreads();
    /* x / S as x * (1 / S) in fp32: within 1.5 ulp of the reference's fp64
     * quotient rounded to fp32 */
    const float r = s_r;
    if (!(r > 0.0f)) return;                        /* a zero or NaN sum: left as the reference leaves it */
    const uint32_t a = blockIdx.x * per, e = min(n, a + per);
    uint32_t i = a + threadIdx.x;
    for (; i + 7 * kThreads < e; i += 8 * kThreads) {      /* eight loads in flight before any store */
        float y[8];
        #pragma unroll
        for (int j = 0; j < 8; j++) y[j] = x[i + j * kThreads];
        #pragma unroll
        for (int j = 0; j < 8; j++) x[i + j * kThreads] = __fmul_rn(y[j], r);
    }
    for (; i < e; i += kThreads) x[i] = __fmul_rn(x[i], r);
}

constexpr uint32_t kAttnSplitTokens = 4096;      /* from this many tokens: the split form */
constexpr uint32_t kAttnMergeSplit = 64;         /* CTAs per head of the first merge level */
constexpr uint32_t kSoftmaxSplit = 1u << 16;
constexpr uint32_t kSoftmaxPer = 1u << 14;       /* values per CTA of the split softmax */

uint32_t attn_tile(uint32_t D) {
    uint32_t t = 4096u / (D ? D : 1);
    return t > 64 ? 64 : (t < 1 ? 1 : t);
}

/* shared memory of k_attn_part: K and V tiles and the queries in fp64, the
 * tile's exponentials, the group sums, the fp32 scores */
size_t attn_part_smem(uint32_t tile, uint32_t H, uint32_t D) {
    return ((2 * (size_t)tile * D + (size_t)H * D + tile + kThreads) * sizeof(double) + tile * sizeof(float) + 15) &
           ~(size_t)15;
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

extern "C" size_t ct__attn_scratch_bytes(uint32_t n_tokens, uint32_t n_heads, uint32_t head_dim) {
    const size_t scores = (size_t)n_heads * n_tokens * sizeof(float);
    if (n_tokens < kAttnSplitTokens) return scores;
    const size_t tiles = (n_tokens + attn_tile(head_dim) - 1) / attn_tile(head_dim);
    const size_t recs = tiles < kAttnMergeSplit ? tiles : kAttnMergeSplit;
    const size_t parts = (tiles + recs) * n_heads * ((size_t)head_dim + 2) * sizeof(double);
    return parts > scores ? parts : scores;
}

extern "C" size_t ct__softmax_scratch_bytes(uint32_t n) {
    if (n < kSoftmaxSplit) return 0;
    const size_t nb = (n + kSoftmaxPer - 1) / kSoftmaxPer;
    return nb * (sizeof(float) + sizeof(double)) + 16;
}

extern "C" int ct__launch_attn_shared(const float *q, const float *k, const float *v, uint32_t n_tokens,
                                      uint32_t n_heads, uint32_t head_dim, float scale, float *out,
                                      float *scratch, void *stream) {
    if (n_heads == 0) return CT_OK;
    cudaStream_t st = (cudaStream_t)stream;
    const uint32_t tile = attn_tile(head_dim);
    if (n_tokens >= kAttnSplitTokens && attn_part_smem(tile, n_heads, head_dim) <= 200 * 1024) {
        /* scratch holds ct__attn_scratch_bytes(n_tokens, n_heads, head_dim) */
        const uint32_t n_tiles = (n_tokens + tile - 1) / tile;
        const size_t smem = attn_part_smem(tile, n_heads, head_dim);
        static bool attr = false;
        if (!attr) {
            cudaFuncSetAttribute(k_attn_part, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
            attr = true;
        }
        double *part = reinterpret_cast<double *>(scratch);
        double *rec = part + (size_t)n_tiles * n_heads * (head_dim + 2);
        const uint32_t S = n_tiles < kAttnMergeSplit ? n_tiles : kAttnMergeSplit;
        k_attn_part<<<n_tiles, kThreads, smem, st>>>(q, k, v, n_tokens, n_heads, head_dim, scale, tile, part);
        k_attn_merge<<<dim3(n_heads, S), kThreads, 0, st>>>(part, n_tiles, n_heads, head_dim, rec, nullptr);
        k_attn_merge<<<dim3(n_heads, 1), kThreads, 0, st>>>(rec, S, n_heads, head_dim, nullptr, out);
        ct__count_launches(3);
        return ct__cuda_status(cudaGetLastError(), "attn_shared");
    }
    const uint32_t nd = head_dim < (uint32_t)kThreads ? head_dim : (uint32_t)kThreads;
    const size_t smem = (size_t)(kThreads / nd) * head_dim * sizeof(double);
    if (smem > 200 * 1024) return CT_ERR_UNSUPPORTED;
    if (smem > 48 * 1024)
        cudaFuncSetAttribute(k_attn_shared, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_attn_shared<<<n_heads, kThreads, smem, st>>>(q, k, v, n_tokens, head_dim, scale, out, scratch);
    ct__count_launches(1);
    return ct__cuda_status(cudaGetLastError(), "attn_shared");
}

extern "C" int ct__launch_softmax(float *x, uint32_t n, void *scratch, void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    if (n >= kSoftmaxSplit) {
        /* scratch holds ct__softmax_scratch_bytes(n) */
        const uint32_t nb = (n + kSoftmaxPer - 1) / kSoftmaxPer;
        double *bsum = reinterpret_cast<double *>(scratch);
        float *bmax = reinterpret_cast<float *>(bsum + nb);
        k_softmax_max<<<nb, kThreads, 0, st>>>(x, n, kSoftmaxPer, bmax);
        k_softmax_exp<<<nb, kThreads, 0, st>>>(x, n, kSoftmaxPer, bmax, nb, bsum);
        k_softmax_norm<<<nb, kThreads, 0, st>>>(x, n, kSoftmaxPer, bsum, nb);
        ct__count_launches(3);
        return ct__cuda_status(cudaGetLastError(), "softmax");
    }
    k_softmax<<<1, kThreads, 0, st>>>(x, n);
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
