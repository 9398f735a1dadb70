/*
 * synth.cu -- device generator behind synth.h: counter-based SplitMix64
 * (Steele, Lea, Flood 2014) and the Box-Muller transform (1958), evaluated
 * in double precision so every element is independent of launch shape.
 */
#include "../../include/hal.h"
#include "../../include/kv_cache.h"
#include "../../include/synth.h"
#include "ct_internal.h"

namespace {

constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;

__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ uint64_t draw(uint64_t key, uint64_t i) { return mix64(key + (i + 1) * kGolden); }

__device__ __forceinline__ float value(uint64_t key, uint64_t okey, uint64_t i, uint32_t bp, float mul) {
    const double u1 = 1.0 - (double)(draw(key, 2 * i) >> 11) * (1.0 / 9007199254740992.0);
    const double u2 = (double)(draw(key, 2 * i + 1) >> 11) * (1.0 / 9007199254740992.0);
    float x = (float)(sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2));
    if (bp && (draw(okey, i) % 10000u) < bp) x *= mul;
    return x;
}

__global__ void k_fill(void *out, uint32_t dtype, uint64_t key, uint64_t okey, uint64_t start, uint64_t n,
                       uint32_t bp, float mul) {
    for (uint64_t j = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; j < n; j += (uint64_t)gridDim.x * blockDim.x) {
        const float x = value(key, okey, start + j, bp, mul);
        if (dtype == 0) static_cast<uint16_t *>(out)[j] = ct_f32_to_bf16(x);
        else static_cast<float *>(out)[j] = x;
    }
}

/* One warp per (sequence, token); lane l generates values l, l+32, ... */
__global__ void __launch_bounds__(256) k_fill_paged(void *pool, float *scales, uint32_t dtype, const int32_t *bt,
                                                    uint32_t max_pages, const uint32_t *rows, const int32_t *lens,
                                                    uint32_t n_seq, uint32_t max_len, uint32_t P, uint32_t E,
                                                    uint64_t key, uint64_t okey, uint32_t bp, float mul) {
    const uint64_t warp = blockIdx.x * 8ull + (threadIdx.x >> 5);
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t total = (uint64_t)n_seq * max_len;
    for (uint64_t w = warp; w < total; w += gridDim.x * 8ull) {
        const uint32_t i = (uint32_t)(w / max_len), t = (uint32_t)(w % max_len);
        if ((int32_t)t >= lens[i]) continue;
        const uint32_t row = rows ? rows[i] : i;
        const int32_t pg = bt[(size_t)row * max_pages + t / P];
        if (pg < 0) continue;
        const size_t slot = (size_t)pg * P + t % P;
        const uint64_t base = (((uint64_t)row << 24) | t) * E;
        if (dtype == CT_KV_BF16 || dtype == CT_KV_F32) {
            for (uint32_t e = lane; e < E; e += 32) {
                const float x = value(key, okey, base + e, bp, mul);
                if (dtype == CT_KV_BF16) static_cast<uint16_t *>(pool)[slot * E + e] = ct_f32_to_bf16(x);
                else static_cast<float *>(pool)[slot * E + e] = x;
            }
        } else {
            float amax = 0.0f;
            for (uint32_t e = lane; e < E; e += 32) amax = fmaxf(amax, fabsf(value(key, okey, base + e, bp, mul)));
            amax = ct_warp_max(amax);
            const float d = __fdiv_rn(amax, dtype == CT_KV_INT8 ? 127.0f : 448.0f);
            const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
            for (uint32_t e = lane; e < E; e += 32) {
                const float x = value(key, okey, base + e, bp, mul);
                static_cast<uint8_t *>(pool)[slot * E + e] =
                    dtype == CT_KV_INT8 ? (uint8_t)(int8_t)ct_q8_code(x, id) : ct_e4m3_code(x, id);
            }
            if (lane == 0) scales[slot] = d;
        }
    }
}

}  // namespace

extern "C" uint64_t ct_synth_key(uint64_t seed, uint64_t stream) {
    return mix64(seed * kGolden + mix64(stream + 0x632BE59BD9B4E019ull));
}

extern "C" int ct_synth_fill(void *out, uint32_t dtype, uint64_t key, uint64_t start, uint64_t n,
                             uint32_t outlier_bp, float outlier_mul, void *stream) {
    if (!out || dtype > 1) return CT_ERR_ARG;
    if (n == 0) return CT_OK;
    const int grid = ct__grid_for((size_t)n, 256, 148 * 16);
    k_fill<<<grid, 256, 0, (cudaStream_t)stream>>>(out, dtype, key, mix64(key ^ 0xA0761D6478BD642Full), start, n,
                                                   outlier_bp, outlier_mul);
    ct__count_launches(1);
    return ct__cuda_status(cudaGetLastError(), "synth_fill");
}

extern "C" int ct_synth_fill_paged(void *pool, float *scales, uint32_t pool_dtype, const int32_t *block_table,
                                   uint32_t max_pages_per_seq, const uint32_t *rows_dev, const int32_t *seq_lens_dev,
                                   uint32_t n_seq, uint32_t max_len, uint32_t page_tokens, uint32_t entry_dim,
                                   uint64_t key, uint32_t outlier_bp, float outlier_mul, void *stream) {
    if (!pool || !block_table || !seq_lens_dev || page_tokens == 0 || entry_dim == 0 || max_len >= (1u << 24))
        return CT_ERR_ARG;
    if ((pool_dtype == CT_KV_INT8 || pool_dtype == CT_KV_E4M3) && !scales) return CT_ERR_ARG;
    if (n_seq == 0 || max_len == 0) return CT_OK;
    const int grid = ct__grid_for((size_t)n_seq * max_len, 8, 148 * 32);
    k_fill_paged<<<grid, 256, 0, (cudaStream_t)stream>>>(pool, scales, pool_dtype, block_table, max_pages_per_seq,
                                                         rows_dev, seq_lens_dev, n_seq, max_len, page_tokens,
                                                         entry_dim, key, mix64(key ^ 0xA0761D6478BD642Full),
                                                         outlier_bp, outlier_mul);
    ct__count_launches(1);
    return ct__cuda_status(cudaGetLastError(), "synth_fill_paged");
}
