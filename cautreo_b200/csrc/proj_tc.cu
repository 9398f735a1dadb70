/*
 * proj_tc.cu -- the producer side of the latent cache on the tensor cores:
 * entry[t] = W . x[t] for a batch of new tokens (the latent projection of
 * ds4_forward.c:1548-1558, matvec_bf16 of ds4_forward.c:248-272, batched
 * over every sequence of a decode step), an optional RMS norm of the first
 * norm_dim values (rmsnorm_ip, ds4_forward.c:206-211), then the append into
 * the pool slots with the pool's codec (ct_kv_paged_write_slots).
 *
 * GEMM  D[128 tokens][NT outputs] = X[tokens][K] . W[outputs][K]^T on
 *       tcgen05 (kind::f16, bf16 operands, fp32 accumulation in TMEM), both
 *       operands K-major with the 128-byte swizzle, 64-value K blocks brought
 *       by TMA through a 4-stage ring.  The K range is split over CTAs
 *       (ksplit) so that a decode batch of ~1k tokens still fills the GPU;
 *       each CTA writes its fp32 partial tile to scratch [ksplit][n][dim].
 *       A batch with more 128-token tiles than SMs (a prefill chunk) gives
 *       each CTA two token tiles, two accumulators over the same W block, so
 *       the W bytes streamed from L2 per token halve (splitting K instead
 *       made such batches slower: their tiles' L2 traffic bounds them).
 * finish sums the ksplit partials in split order (the result does not
 *       depend on timing; one thread per 4 values), then, when asked, the
 *       norm (one warp per token), leaving the fp32 entry for the pool writer.
 *
 * Roles per CTA (192 threads): warp 0 TMA (one lane), warp 1 TMEM owner and
 * MMA issuer (one lane), warps 2-5 epilogue (one token row per thread, each
 * warp the TMEM lane quadrant it may access).  Every wait is bounded and
 * reports an error word; no load uses cluster multicast.
 */
#include "../../include/hal.h"
#include "../../include/kv_cache.h"
#include "ct_internal.h"
#include "tc_ptx.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

namespace {

using namespace ct_tc;

constexpr int kM = 128;                 /* tokens per tile */
constexpr int kKB = 64;                 /* K values per stage (one 128-byte swizzle row) */
constexpr int kStagesP = 4;
constexpr int kThreadsP = 192;
constexpr long long kWaitP = 4000000000LL;

__device__ int g_proj_error;

/* MT token tiles of 128 rows per CTA share each W block (MT = 2 halves the
 * W traffic per token for batches that fill the GPU without a K split). */
template <int NT, int MT>
struct Layout {
    static constexpr uint32_t kA = MT * kM * kKB * 2;     /* 16 KB per token tile */
    static constexpr uint32_t kB = NT * kKB * 2;
    static constexpr uint32_t kStage = kA + kB;
    static constexpr uint32_t kBars = kStagesP * kStage;  /* full[4], empty[4], acc */
    static constexpr uint32_t kTmemSlot = kBars + 9 * 8;
    static constexpr uint32_t kBytes = kTmemSlot + 16 + 1024;
    static constexpr uint32_t kCols1 = NT <= 32 ? 32 : NT <= 64 ? 64 : NT <= 128 ? 128 : 256;   /* one accumulator */
    static constexpr uint32_t kCols = MT * kCols1;
    static constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NT >> 3) << 17) |
                                       ((uint32_t)(kM >> 4) << 24);
};

__device__ bool wait_p(uint32_t bar, uint32_t parity, volatile int *abort, int code) {
    const long long t0 = clock64();
    for (;;) {
        if (mbar_try(bar, parity)) return true;
        if (*abort) return false;
        if (clock64() - t0 > kWaitP) {
            atomicCAS(&g_proj_error, 0, code);
            *abort = 1;
            return false;
        }
    }
}

template <int NT, int MT>
__global__ void __launch_bounds__(kThreadsP, 1)
    k_proj_tc(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap, float *scratch,
              uint32_t n, uint32_t dim, uint32_t kblocks, uint32_t per_split) {
    using Ly = Layout<NT, MT>;
    static_assert(Ly::kBytes <= 232448 && Ly::kCols <= 512, "shared memory / TMEM");
    extern __shared__ uint8_t smem_raw[];
    __shared__ int s_abort;
    const uint32_t raw = smem_addr(smem_raw);
    const uint32_t base = raw + ((1024u - (raw & 1023u)) & 1023u);
    uint8_t *sbase = smem_raw + (base - raw);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t m0 = blockIdx.x * (kM * MT), n0 = blockIdx.y * NT, split = blockIdx.z;
    const uint32_t kb0 = split * per_split, kb1 = min(kblocks, kb0 + per_split);
    const uint32_t nkb = kb1 > kb0 ? kb1 - kb0 : 0;
    auto full = [&](uint32_t s) { return base + Ly::kBars + 8 * s; };
    auto empty = [&](uint32_t s) { return base + Ly::kBars + 8 * (kStagesP + s); };
    const uint32_t acc = base + Ly::kBars + 8 * (2 * kStagesP);
    if (threadIdx.x == 0) {
        s_abort = 0;
        for (int s = 0; s < kStagesP; s++) { mbar_init(full(s), 1); mbar_init(empty(s), 1); }
        mbar_init(acc, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(base + Ly::kTmemSlot), "r"(Ly::kCols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(sbase + Ly::kTmemSlot);
    volatile int *abort = &s_abort;

    if (warp == 0 && lane == 0) {
        /* TMA: K block kb -> stage (i % 4) */
        uint32_t issued = 0;
        for (uint32_t i = 0; i < nkb; i++) {
            const uint32_t s = i % kStagesP;
            if (!wait_p(empty(s), ((i / kStagesP) & 1) ^ 1, abort, 1)) break;
            issued++;
            const uint32_t dst = base + s * Ly::kStage;
            mbar_expect_tx(full(s), Ly::kStage);
            const int kx = (int)((kb0 + i) * kKB);
            tma_load_2d(dst, &xmap, kx, (int)m0, full(s));
            tma_load_2d(dst + Ly::kA, &wmap, kx, (int)n0, full(s));
        }
        /* every issued load lands before the CTA may exit */
        for (uint32_t k = 0; k < (uint32_t)kStagesP && k < issued; k++) {
            const uint32_t last = issued - 1 - k;
            const long long t0 = clock64();
            while (!mbar_try(full(last % kStagesP), (last / kStagesP) & 1) && clock64() - t0 < kWaitP) {}
        }
    } else if (warp == 1 && lane == 0) {
        bool ok = true;
        for (uint32_t i = 0; i < nkb && ok; i++) {
            const uint32_t s = i % kStagesP;
            ok = wait_p(full(s), (i / kStagesP) & 1, abort, 2);
            if (!ok) break;
            tc_fence_after();
            const uint32_t a = base + s * Ly::kStage, b = a + Ly::kA;
            #pragma unroll
            for (int mt = 0; mt < MT; mt++) {
                #pragma unroll
                for (int k = 0; k < kKB / 16; k++)
                    mma_ss(tmem + mt * Ly::kCols1, sdesc(a + mt * (kM * 128) + k * 32, 1, 64, kSw128),
                           sdesc(b + k * 32, 1, 64, kSw128), Ly::kIdesc, (i > 0 || k > 0) ? 1u : 0u);
            }
            mma_commit(empty(s));
        }
        mma_commit(acc);                        /* also when nothing was issued: the epilogue waits on it */
        const long long t0 = clock64();
        while (!mbar_try(acc, 0) && clock64() - t0 < kWaitP) {}    /* drained before TMEM is freed */
    } else if (warp >= 2) {
        const uint32_t quad = warp & 3, row = quad * 32 + lane;
        if (__all_sync(0xFFFFFFFFu, wait_p(acc, 0, abort, 3))) {    /* warp-uniform: the TMEM loads are collective */
            tc_fence_after();
            #pragma unroll 1
            for (int mc = 0; mc < MT * NT; mc += 32) {
                const int mt = mc / NT, c = mc % NT;
                const uint32_t tok = m0 + mt * kM + row;
                float *dst = scratch + ((size_t)split * n + tok) * dim + n0;
                float v[32];
                if (nkb > 0) {
                    tmem_ld32(tmem + ((quad * 32) << 16) + mt * Ly::kCols1 + c, v);
                    tmem_wait_ld();
                } else {
                    #pragma unroll
                    for (int i = 0; i < 32; i++) v[i] = 0.0f;
                }
                if (tok < n) {
                    float4 *d4 = reinterpret_cast<float4 *>(dst + c);
                    #pragma unroll
                    for (int i = 0; i < 8; i++) d4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Ly::kCols) : "memory");
}

/* entry = sum of the ksplit partials, in split order (the result does not
 * depend on timing); one thread per 4 values, up to 16 partial loads in
 * flight per thread. */
__global__ void __launch_bounds__(256) k_proj_sum(const float4 *part, float4 *entry, size_t n4, uint32_t ksplit) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        float4 v[16];
        #pragma unroll
        for (uint32_t k = 0; k < 16; k++)
            if (k < ksplit) v[k] = __ldcs(part + k * n4 + i);
        float4 a = v[0];
        #pragma unroll
        for (uint32_t k = 1; k < 16; k++) {
            if (k < ksplit) { a.x += v[k].x; a.y += v[k].y; a.z += v[k].z; a.w += v[k].w; }
        }
        entry[i] = a;
    }
}

/* RMS norm of rmsnorm_ip over [0, norm_dim) of each entry, in place: one
 * warp per token, x * (1 / sqrt(mean(x^2) + eps)) * w, the mean in fp32 over
 * a warp-shuffle tree. */
__global__ void __launch_bounds__(256) k_proj_norm(float *entry, uint32_t n, uint32_t dim, const float *norm_w,
                                                   float eps, uint32_t norm_dim) {
    const uint32_t t = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (t >= n) return;
    float *e = entry + (size_t)t * dim;
    float ss = 0.0f;
    for (uint32_t i = lane; i < norm_dim; i += 32) ss += e[i] * e[i];
    ss = ct_warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)norm_dim + eps);
    for (uint32_t i = lane; i < norm_dim; i += 32) e[i] = e[i] * inv * norm_w[i];
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn_p() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void *p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        else
            cudaGetLastError();
    }
    return fn;
}

/* [rows][cols] bf16, box (64 x box_rows), 128-byte swizzle. */
bool map_bf16(CUtensorMap *m, const void *base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    auto fn = encode_fn_p();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    cuuint32_t box[2] = {(cuuint32_t)kKB, box_rows};
    cuuint32_t es[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NT, int MT>
int launch_proj(const CUtensorMap &xm, const CUtensorMap &wm, float *scratch, uint32_t n, uint32_t dim,
                uint32_t kblocks, uint32_t ksplit, uint32_t per_split, cudaStream_t st) {
    using Ly = Layout<NT, MT>;
    static int attr_set[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        if (cudaFuncSetAttribute(k_proj_tc<NT, MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Ly::kBytes) !=
            cudaSuccess)
            return ct__cuda_status(cudaGetLastError(), "proj smem");
        attr_set[dev] = 1;
    }
    const dim3 grid((n + kM * MT - 1) / (kM * MT), dim / NT, ksplit);
    k_proj_tc<NT, MT><<<grid, kThreadsP, Ly::kBytes, st>>>(xm, wm, scratch, n, dim, kblocks, per_split);
    return ct__cuda_status(cudaGetLastError(), "proj_tc");
}

}  // namespace

extern "C" int ct_kv_project_error(int clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_proj_error, sizeof v) != cudaSuccess) { cudaGetLastError(); return -1; }
    if (clear && v) {
        const int z = 0;
        cudaMemcpyToSymbol(g_proj_error, &z, sizeof z);
    }
    return v;
}

extern "C" int ct_kv_project_write_slots(const void *x, const void *w, const float *norm_w, float eps,
                                         uint32_t norm_dim, uint32_t n, uint32_t n_in, uint32_t dim, void *pool,
                                         float *scales, uint32_t pool_dtype, const int32_t *dest_slot,
                                         void *stream) {
    if (!x || !w || !pool || !dest_slot || n_in == 0 || n_in % kKB != 0 || dim == 0 || dim % 64 != 0) return CT_ERR_ARG;
    if (norm_w && (norm_dim == 0 || norm_dim > dim || norm_dim % 4 != 0)) return CT_ERR_ARG;
    if (((uintptr_t)x & 15) || ((uintptr_t)w & 15)) return CT_ERR_ARG;
    if (n == 0) return CT_OK;
    static int cc_major[64], sm_count[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return CT_ERR_ARG;
    if (!cc_major[dev]) {
        cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&cc_major[dev], cudaDevAttrComputeCapabilityMajor, dev);
    }
    const int major = cc_major[dev];
    if (major != 10) {
        ct__set_error("ct_kv_project_write_slots: needs an sm_100 GPU");
        return CT_ERR_UNSUPPORTED;
    }
    cudaStream_t st = (cudaStream_t)stream;
    /* output tile: the widest of 256 / 192 / 128 / 64 that divides dim */
    const uint32_t d64 = dim / 64;
    const uint32_t g = d64 % 4 == 0 ? 4 : d64 % 3 == 0 ? 3 : d64 % 2 == 0 ? 2 : 1;
    const uint32_t NT = 64 * g;
    /* K split: about one wave of CTAs, at least 4 K blocks each */
    const int n_sms = sm_count[dev] > 0 ? sm_count[dev] : 148;
    const uint32_t kblocks = n_in / kKB;
    uint32_t tiles = ((n + kM - 1) / kM) * (dim / NT);
    /* more 128-token tiles than SMs: two per CTA, sharing the W blocks */
    const uint32_t MT = (tiles > (uint32_t)n_sms && NT <= 192) ? 2 : 1;
    if (MT == 2) tiles = ((n + 2 * kM - 1) / (2 * kM)) * (dim / NT);
    uint32_t ksplit = (uint32_t)n_sms / (tiles ? tiles : 1);
    if (ksplit < 1) ksplit = 1;
    if (ksplit > kblocks / 4) ksplit = kblocks / 4 ? kblocks / 4 : 1;
    if (ksplit > 16) ksplit = 16;                     /* k_proj_sum keeps 16 partials in flight */
    const uint32_t per_split = (kblocks + ksplit - 1) / ksplit;
    ksplit = (kblocks + per_split - 1) / per_split;
    CUtensorMap xm, wm;
    if (!map_bf16(&xm, x, n, n_in, kM * MT) || !map_bf16(&wm, w, dim, n_in, NT)) {
        ct__set_error("ct_kv_project_write_slots: tensor map encoding failed");
        return CT_ERR_CUDA;
    }
    const size_t part_bytes = (size_t)ksplit * n * dim * sizeof(float);
    const size_t entry_bytes = (size_t)n * dim * sizeof(float);
    const bool direct = ksplit == 1 && !norm_w;       /* the partial is the entry */
    float *scratch = nullptr;
    int rc = ct__scratch_alloc((void **)&scratch, part_bytes + (direct ? 0 : entry_bytes), st);
    if (rc) return rc;
    switch (NT * 4 + MT) {
        case 256 * 4 + 1: rc = launch_proj<256, 1>(xm, wm, scratch, n, dim, kblocks, ksplit, per_split, st); break;
        case 192 * 4 + 1: rc = launch_proj<192, 1>(xm, wm, scratch, n, dim, kblocks, ksplit, per_split, st); break;
        case 192 * 4 + 2: rc = launch_proj<192, 2>(xm, wm, scratch, n, dim, kblocks, ksplit, per_split, st); break;
        case 128 * 4 + 1: rc = launch_proj<128, 1>(xm, wm, scratch, n, dim, kblocks, ksplit, per_split, st); break;
        case 128 * 4 + 2: rc = launch_proj<128, 2>(xm, wm, scratch, n, dim, kblocks, ksplit, per_split, st); break;
        case 64 * 4 + 2:  rc = launch_proj<64, 2>(xm, wm, scratch, n, dim, kblocks, ksplit, per_split, st); break;
        default:          rc = launch_proj<64, 1>(xm, wm, scratch, n, dim, kblocks, ksplit, per_split, st); break;
    }
    float *entry = direct ? scratch : scratch + (size_t)ksplit * n * dim;
    uint32_t launches = 1;
    if (!rc && !direct) {
        const size_t n4 = (size_t)n * dim / 4;
        const int grid = ct__grid_for(n4, 256, n_sms * 8);
        k_proj_sum<<<grid, 256, 0, st>>>(reinterpret_cast<const float4 *>(scratch), reinterpret_cast<float4 *>(entry),
                                         n4, ksplit);
        rc = ct__cuda_status(cudaGetLastError(), "proj_sum");
        launches++;
        if (!rc && norm_w) {
            k_proj_norm<<<(n + 7) / 8, 256, 0, st>>>(entry, n, dim, norm_w, eps, norm_dim);
            rc = ct__cuda_status(cudaGetLastError(), "proj_norm");
            launches++;
        }
    }
    ct__count_launches(launches);
    if (!rc) rc = ct_kv_paged_write_slots(pool, scales, pool_dtype, entry, CT_KV_F32, dest_slot, n, dim, stream);
    ct__scratch_free(scratch, st);
    return rc;
}
