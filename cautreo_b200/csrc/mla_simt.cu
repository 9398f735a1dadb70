/*
 * mla_simt.cu -- paged absorbed-MLA decode on CUDA cores (FMA), for shapes
 * the tensor-core kernel (mla_tc.cu) does not take: any head count, entry
 * dims up to 576, value dims up to 512, any page size, bf16 / fp32 / int8 /
 * e4m3 pools.  Plus the split-KV combine shared by both kernels.
 *
 * Math (per sequence s, head h, over entries e_t of mapped pages, t < len):
 *   s_t = scale * q_h . e_t          (all entry_dim values)
 *   o_h = sum_t softmax(s)_t * e_t[0:v_dim]
 * computed as a flash-decoding online softmax in the log2 domain (q is
 * pre-multiplied by scale*log2(e)); chunks of one sequence write partial
 * (o, m, l) that k_mla_combine merges with their log-sum-exp weights.
 *
 * Block = (chunk, group of 16 heads); 256 threads.  A sub-tile of 32 tokens
 * is dequantised to fp32 in shared memory (rows padded to 577 floats so the
 * 16 token rows a half-warp reads fall in distinct banks); each half-warp
 * scores one head against the 32 tokens; each thread accumulates 2 value
 * dims for all 16 heads.
 */
#include "../../include/attention.h"
#include "../../include/hal.h"
#include "../../include/kv_cache.h"
#include "ct_internal.h"

namespace {

constexpr int HG = 16;
constexpr int TT = 32;
constexpr int EMAX = 576;
constexpr int VMAX = 512;
constexpr int QSTR = EMAX + 1;
constexpr int KSTR = EMAX + 1;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

constexpr size_t kSmemBytes = sizeof(float) * ((size_t)HG * QSTR + (size_t)TT * KSTR + HG * TT + HG + 2 * HG);

template <int Dtype>
__device__ __forceinline__ void load_tile(float *kv_s, const void *pool, const float *scales, size_t slot0,
                                          uint32_t E, uint32_t nt) {
    /* 8 values (one 16-byte bf16 vector, or 8 codes) per step. */
    const uint32_t vec_per_tok = E / 8;
    for (uint32_t idx = threadIdx.x; idx < TT * vec_per_tok; idx += blockDim.x) {
        const uint32_t j = idx / vec_per_tok, c = idx % vec_per_tok;
        float v[8];
        if (j < nt) {
            const size_t slot = slot0 + j;
            if (Dtype == CT_KV_BF16) {
                uint4 w = __ldg(reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(pool) + slot * E) + c);
                const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
                #pragma unroll
                for (int i = 0; i < 4; i++) { v[2 * i] = __uint_as_float(ws[i] << 16); v[2 * i + 1] = __uint_as_float(ws[i] & 0xFFFF0000u); }
            } else if (Dtype == CT_KV_F32) {
                const float4 *p = reinterpret_cast<const float4 *>(static_cast<const float *>(pool) + slot * E) + 2 * c;
                float4 a = __ldg(p), b = __ldg(p + 1);
                v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
            } else {
                uint2 w = __ldg(reinterpret_cast<const uint2 *>(static_cast<const uint8_t *>(pool) + slot * E) + c);
                const float sc = __ldg(scales + slot);
                const uint32_t ws[2] = {w.x, w.y};
                #pragma unroll
                for (int i = 0; i < 8; i++) {
                    const uint8_t b = (uint8_t)(ws[i >> 2] >> (8 * (i & 3)));
                    v[i] = (Dtype == CT_KV_INT8 ? (float)(int8_t)b : ct_e4m3_to_f32(b)) * sc;
                }
            }
        } else {
            #pragma unroll
            for (int i = 0; i < 8; i++) v[i] = 0.0f;
        }
        float *dst = kv_s + (size_t)j * KSTR + c * 8;
        #pragma unroll
        for (int i = 0; i < 8; i++) dst[i] = v[i];
    }
}

template <int Dtype>
__global__ void __launch_bounds__(256) k_mla_simt(ct_mla_dims_t dims, const ct_mla_chunk_t *chunks,
                                                  const int32_t *counts, const uint16_t *q, const void *pool,
                                                  const float *scales, const int32_t *block_table,
                                                  const int32_t *seq_lens, uint16_t *out, float *lse, float *part_o,
                                                  float *part_ml) {
    if (counts && (int32_t)blockIdx.x >= counts[0]) return;       /* beyond the planned chunks */
    extern __shared__ float smem[];
    float *q_s = smem;                            /* [HG][QSTR] */
    float *kv_s = q_s + HG * QSTR;                /* [TT][KSTR] */
    float *p_s = kv_s + TT * KSTR;                /* [HG][TT] */
    float *alpha_s = p_s + HG * TT;               /* [HG] */
    float *ml_s = alpha_s + HG;                   /* [HG][2] */

    const ct_mla_chunk_t ch = chunks[blockIdx.x];
    const uint32_t H = dims.n_heads, E = dims.entry_dim, Dv = dims.v_dim, P = dims.page_tokens;
    const uint32_t h0 = blockIdx.y * HG;
    const float qscale = dims.scale * kLog2e;
    for (uint32_t idx = threadIdx.x; idx < HG * E; idx += blockDim.x) {
        const uint32_t h = idx / E, e = idx % E;
        q_s[h * QSTR + e] = (h0 + h < H) ? ct_bf16_to_f32(q[((size_t)ch.seq * H + h0 + h) * E + e]) * qscale : 0.0f;
    }
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t my_h = 2 * warp + (lane >> 4), jl = lane & 15;
    const uint32_t d0 = 2 * threadIdx.x;
    float m = -INFINITY, l = 0.0f;
    float acc[HG][2];
    #pragma unroll
    for (int h = 0; h < HG; h++) { acc[h][0] = 0.0f; acc[h][1] = 0.0f; }

    const int32_t len = seq_lens[ch.row];
    for (int32_t lp = ch.page_begin; lp < ch.page_end; lp++) {
        const int32_t pg = block_table[(size_t)ch.row * dims.max_pages_per_seq + lp];
        const int32_t ntok = min((int32_t)P, len - lp * (int32_t)P);
        if (pg < 0 || (uint32_t)pg >= dims.n_pages || ntok <= 0) continue;
        for (int32_t sub = 0; sub < ntok; sub += TT) {
            const uint32_t nt = (uint32_t)min(TT, ntok - sub);
            __syncthreads();
            load_tile<Dtype>(kv_s, pool, scales, (size_t)pg * P + sub, E, nt);
            __syncthreads();
            float s0 = -INFINITY, s1 = -INFINITY;
            {
                const float *qr = q_s + my_h * QSTR;
                const float *k0 = kv_s + jl * KSTR, *k1 = kv_s + (jl + 16) * KSTR;
                float a0 = 0.0f, a1 = 0.0f;
                for (uint32_t e = 0; e < E; e++) { const float qq = qr[e]; a0 = fmaf(qq, k0[e], a0); a1 = fmaf(qq, k1[e], a1); }
                if (jl < nt) s0 = a0;
                if (jl + 16 < nt) s1 = a1;
            }
            float tmax = fmaxf(s0, s1);
            #pragma unroll
            for (int o = 8; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xFFFFFFFFu, tmax, o));
            const float m_new = fmaxf(m, tmax);
            const float alpha = exp2f(m - m_new);
            const float p0 = exp2f(s0 - m_new), p1 = exp2f(s1 - m_new);
            float ps = p0 + p1;
            #pragma unroll
            for (int o = 8; o > 0; o >>= 1) ps += __shfl_xor_sync(0xFFFFFFFFu, ps, o);
            l = l * alpha + ps;
            m = m_new;
            p_s[my_h * TT + jl] = p0;
            p_s[my_h * TT + jl + 16] = p1;
            if (jl == 0) alpha_s[my_h] = alpha;
            __syncthreads();
            if (d0 < Dv) {
                #pragma unroll
                for (int h = 0; h < HG; h++) { const float a = alpha_s[h]; acc[h][0] *= a; acc[h][1] *= a; }
                for (uint32_t j = 0; j < nt; j += 4) {
                    float v0[4], v1[4];
                    #pragma unroll
                    for (int u = 0; u < 4; u++) { v0[u] = kv_s[(j + u) * KSTR + d0]; v1[u] = kv_s[(j + u) * KSTR + d0 + 1]; }
                    #pragma unroll
                    for (int h = 0; h < HG; h++) {
                        const float4 p = *reinterpret_cast<const float4 *>(p_s + h * TT + j);
                        acc[h][0] = fmaf(p.x, v0[0], fmaf(p.y, v0[1], fmaf(p.z, v0[2], fmaf(p.w, v0[3], acc[h][0]))));
                        acc[h][1] = fmaf(p.x, v1[0], fmaf(p.y, v1[1], fmaf(p.z, v1[2], fmaf(p.w, v1[3], acc[h][1]))));
                    }
                }
            }
        }
    }
    if (jl == 0) { ml_s[2 * my_h] = m; ml_s[2 * my_h + 1] = l; }
    __syncthreads();
    #pragma unroll
    for (int h = 0; h < HG; h++) {
        if (h0 + h >= H) break;
        const float mh = ml_s[2 * h], lh = ml_s[2 * h + 1];
        const size_t oh = (size_t)ch.seq * H + h0 + h;
        if (ch.part < 0) {
            const float inv = lh > 0.0f ? 1.0f / lh : 0.0f;
            if (d0 < Dv) {
                out[oh * Dv + d0] = ct_f32_to_bf16(acc[h][0] * inv);
                if (d0 + 1 < Dv) out[oh * Dv + d0 + 1] = ct_f32_to_bf16(acc[h][1] * inv);
            }
            if (lse && threadIdx.x == 0) lse[oh] = lh > 0.0f ? mh * kLn2 + logf(lh) : -INFINITY;
        } else {
            const size_t ph = (size_t)ch.part * H + h0 + h;
            if (d0 < Dv) {
                part_o[ph * Dv + d0] = acc[h][0];
                if (d0 + 1 < Dv) part_o[ph * Dv + d0 + 1] = acc[h][1];
            }
            if (threadIdx.x == 0) { part_ml[4 * ph] = mh; part_ml[4 * ph + 1] = lh; part_ml[4 * ph + 2] = lh; }
        }
    }
}

}  // namespace

/* Split-KV combine: partials (o_i unnormalised, m_i in log2 units, and the
 * row sums l_i of the value dims below and above v_dim / 2 -- the two SMs of
 * a tensor-core worker each normalise their half of the dims by their own
 * sum) merge as o = sum_i 2^(m_i - M) o_i / sum_i 2^(m_i - M) l_i.  Entries
 * of part_ml are (m, l_lo, l_hi, unused).  Block = one combine item x 4
 * heads, a warp per head: the lanes reduce M and L over the parts, then each
 * lane accumulates its value dims over the parts in part order (v_dim a
 * multiple of 128: four consecutive dims per 128, as 16-byte loads, all of a
 * part's loads issued before its FMAs). */
constexpr int kCombineHeads = 4;

__global__ void __launch_bounds__(32 * kCombineHeads) k_mla_combine(const ct_mla_combine_t *items,
                                                                   const int32_t *counts, uint32_t H, uint32_t Dv,
                                                                   const float *part_o, const float *part_ml,
                                                                   uint16_t *out, float *lse) {
    if (counts && (int32_t)blockIdx.x >= counts[1]) return;       /* beyond the planned combines */
    const ct_mla_combine_t it = items[blockIdx.x];
    const uint32_t lane = threadIdx.x & 31, h = blockIdx.y * kCombineHeads + (threadIdx.x >> 5);
    if (h >= H) return;
    float M = -INFINITY;
    for (int i = (int)lane; i < it.n_parts; i += 32) {
        const size_t ph = (size_t)(it.first_part + i) * H + h;
        if (part_ml[4 * ph + 1] > 0.0f) M = fmaxf(M, part_ml[4 * ph]);
    }
    #pragma unroll
    for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
    /* the row sums in part order, as one thread would add them */
    float L[2] = {0.0f, 0.0f};
    for (int i = 0; i < it.n_parts; i++) {
        const size_t ph = (size_t)(it.first_part + i) * H + h;
        const float4 ml = *reinterpret_cast<const float4 *>(part_ml + 4 * ph);
        if (ml.y > 0.0f) {
            const float w = exp2f(ml.x - M);
            L[0] += w * ml.y;
            L[1] += w * ml.z;
        }
    }
    const float inv[2] = {L[0] > 0.0f ? 1.0f / L[0] : 0.0f, L[1] > 0.0f ? 1.0f / L[1] : 0.0f};
    const size_t oh = (size_t)it.seq * H + h;
    if ((Dv & 127) == 0 && Dv <= 512) {
        const uint32_t slabs = Dv / 128;
        float4 acc[4];
        #pragma unroll
        for (int k = 0; k < 4; k++) acc[k] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int i = 0; i < it.n_parts; i++) {
            const size_t ph = (size_t)(it.first_part + i) * H + h;
            const float4 ml = *reinterpret_cast<const float4 *>(part_ml + 4 * ph);
            if (!(ml.y > 0.0f)) continue;
            const float w = exp2f(ml.x - M);
            const float4 *po = reinterpret_cast<const float4 *>(part_o + ph * Dv) + lane;
            float4 v[4];
            #pragma unroll
            for (int k = 0; k < 4; k++)
                if ((uint32_t)k < slabs) v[k] = __ldcs(po + 32 * k);
            #pragma unroll
            for (int k = 0; k < 4; k++) {
                if ((uint32_t)k >= slabs) continue;
                acc[k].x = fmaf(w, v[k].x, acc[k].x);
                acc[k].y = fmaf(w, v[k].y, acc[k].y);
                acc[k].z = fmaf(w, v[k].z, acc[k].z);
                acc[k].w = fmaf(w, v[k].w, acc[k].w);
            }
        }
        #pragma unroll
        for (int k = 0; k < 4; k++) {
            if ((uint32_t)k >= slabs) continue;
            const uint32_t d = 128 * k + 4 * lane;
            const float s = d >= Dv / 2 ? inv[1] : inv[0];          /* Dv / 2 is a multiple of 4 */
            uint2 pk;
            pk.x = (uint32_t)ct_f32_to_bf16(acc[k].x * s) | ((uint32_t)ct_f32_to_bf16(acc[k].y * s) << 16);
            pk.y = (uint32_t)ct_f32_to_bf16(acc[k].z * s) | ((uint32_t)ct_f32_to_bf16(acc[k].w * s) << 16);
            *reinterpret_cast<uint2 *>(out + oh * Dv + d) = pk;
        }
    } else {
        for (uint32_t d = lane; d < Dv; d += 32) {
            float o = 0.0f;
            for (int i = 0; i < it.n_parts; i++) {
                const size_t ph = (size_t)(it.first_part + i) * H + h;
                if (part_ml[4 * ph + 1] > 0.0f) o = fmaf(exp2f(part_ml[4 * ph] - M), part_o[ph * Dv + d], o);
            }
            out[oh * Dv + d] = ct_f32_to_bf16(o * (d >= Dv / 2 ? inv[1] : inv[0]));
        }
    }
    if (lse && lane == 0) lse[oh] = L[0] > 0.0f ? M * kLn2 + logf(L[0]) : -INFINITY;
}

/* Declared in mla_tc.cu: the tcgen05 kernel for H=128, E=576, Dv=512, P=64,
 * bf16 / int8 / e4m3 pools.  Returns CT_ERR_UNSUPPORTED when it does not take
 * the shape. */
extern "C" int ct__launch_mla_tc(const ct_mla_dims_t *dims, const ct_mla_chunk_t *chunks, uint32_t n_chunks,
                                 const int32_t *worker_begin, uint32_t n_workers, const void *q, const void *pool,
                                 const float *scales, const int32_t *block_table, const int32_t *seq_lens, void *out,
                                 float *lse, float *part_o, float *part_ml, void *stream);

extern "C" int ct__launch_mla_decode(const ct_mla_dims_t *dims, const ct_mla_chunk_t *chunks,
                                     uint32_t n_chunks, const int32_t *worker_begin, uint32_t n_workers,
                                     const ct_mla_combine_t *combines,
                                     uint32_t n_combines, const int32_t *counts, const void *q, const void *pool,
                                     const float *scales, const int32_t *block_table,
                                     const int32_t *seq_lens, void *out, float *lse, float *part_o,
                                     float *part_ml, void *stream, uint32_t *n_launches) {
    cudaStream_t st = (cudaStream_t)stream;
    uint32_t launches = 0;
    if (n_chunks > 0) {
        int rc = ct__launch_mla_tc(dims, chunks, n_chunks, worker_begin, n_workers, q, pool, scales, block_table,
                                   seq_lens, out, lse, part_o, part_ml, stream);
        if (rc == CT_ERR_UNSUPPORTED) {
            if (dims->entry_dim > EMAX || dims->v_dim > VMAX || dims->entry_dim % 8 != 0 || dims->page_tokens == 0)
                return CT_ERR_UNSUPPORTED;
            const dim3 grid(n_chunks, (dims->n_heads + HG - 1) / HG);
            switch (dims->kv_dtype) {
#define CT_SIMT(D)                                                                                        \
    cudaFuncSetAttribute(k_mla_simt<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes); \
    k_mla_simt<D><<<grid, 256, kSmemBytes, st>>>(*dims, chunks, counts, static_cast<const uint16_t *>(q), pool, \
                                                  scales, block_table, seq_lens,                         \
                                                  static_cast<uint16_t *>(out), lse, part_o, part_ml);   \
    break;
                case CT_KV_BF16: CT_SIMT(CT_KV_BF16)
                case CT_KV_F32: CT_SIMT(CT_KV_F32)
                case CT_KV_INT8: CT_SIMT(CT_KV_INT8)
                case CT_KV_E4M3: CT_SIMT(CT_KV_E4M3)
                default:
                    ct__set_error("MLA decode: block-quantised pools are gathered to bf16 before decoding");
                    return CT_ERR_UNSUPPORTED;
#undef CT_SIMT
            }
            rc = ct__cuda_status(cudaGetLastError(), "mla_simt");
        }
        if (rc != CT_OK) return rc;
        launches++;
    }
    if (n_combines > 0) {
        k_mla_combine<<<dim3(n_combines, (dims->n_heads + kCombineHeads - 1) / kCombineHeads), 32 * kCombineHeads, 0,
                        st>>>(
            combines, counts, dims->n_heads, dims->v_dim, part_o, part_ml, static_cast<uint16_t *>(out), lse);
        int rc = ct__cuda_status(cudaGetLastError(), "mla_combine");
        if (rc != CT_OK) return rc;
        launches++;
    }
    ct__count_launches(launches);
    if (n_launches) *n_launches = launches;
    return CT_OK;
}
