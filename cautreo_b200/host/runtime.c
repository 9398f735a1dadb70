/*
 * runtime.c -- the CUDA backend of hal.h (Part 2) and the bookkeeping every
 * launcher shares: last-error text (per host thread) and a process-wide count
 * of kernel launches.
 */
#include "../../include/hal.h"
#include "../csrc/ct_internal.h"

#include <cuda_runtime_api.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdio.h>
#include <string.h>

static _Thread_local char g_last_error[256];
static _Atomic uint64_t g_launches;

int ct__cuda_status(int code, const char *where) {
    if (code == 0) return CT_OK;
    snprintf(g_last_error, sizeof g_last_error, "%s: %s (%d)", where ? where : "cuda",
             cudaGetErrorString((cudaError_t)code), code);
    return CT_ERR_CUDA;
}

void ct__set_error(const char *msg) {
    snprintf(g_last_error, sizeof g_last_error, "%s", msg ? msg : "");
}

void ct__count_launches(uint32_t n) { atomic_fetch_add(&g_launches, (uint64_t)n); }

/* One private pool per device, created on first use.  The default pool of a
 * device releases freed memory at every synchronisation (threshold 0), so a
 * per-step cudaMallocAsync of megabytes remaps memory each time; this pool
 * keeps up to 1 GiB and leaves the process's default pool as it is. */
#define CT_MAX_DEVICES 64
static cudaMemPool_t g_pools[CT_MAX_DEVICES];
static pthread_mutex_t g_pool_lock = PTHREAD_MUTEX_INITIALIZER;

static int scratch_pool(int dev, cudaMemPool_t *out) {
    if (dev < 0 || dev >= CT_MAX_DEVICES) return ct__cuda_status(cudaErrorInvalidDevice, "scratch pool");
    pthread_mutex_lock(&g_pool_lock);
    int rc = CT_OK;
    if (!g_pools[dev]) {
        struct cudaMemPoolProps props;
        memset(&props, 0, sizeof props);
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = dev;
        cudaMemPool_t pool = NULL;
        rc = ct__cuda_status(cudaMemPoolCreate(&pool, &props), "scratch pool");
        if (!rc) {
            uint64_t keep = 1ull << 30;
            rc = ct__cuda_status(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep), "scratch pool");
            if (rc) cudaMemPoolDestroy(pool);
            else g_pools[dev] = pool;
        }
    }
    *out = g_pools[dev];
    pthread_mutex_unlock(&g_pool_lock);
    return rc;
}

int ct__scratch_alloc(void **p, size_t bytes, void *stream) {
    int dev = 0;
    int rc = ct__cuda_status(cudaGetDevice(&dev), "scratch");
    cudaMemPool_t pool = NULL;
    if (!rc) rc = scratch_pool(dev, &pool);
    if (!rc) rc = ct__cuda_status(cudaMallocFromPoolAsync(p, bytes ? bytes : 16, pool, (cudaStream_t)stream),
                                  "scratch alloc");
    return rc;
}

void ct__scratch_free(void *p, void *stream) {
    if (p) cudaFreeAsync(p, (cudaStream_t)stream);
}

const char *ct_hal_cuda_last_error(void) { return g_last_error; }
uint64_t ct_hal_cuda_launch_count(void) { return atomic_load(&g_launches); }
const char *ct_hal_version(void) { return "cautreo_b200 0.1 (sm_100a)"; }

int ct_hal_cuda_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) { cudaGetLastError(); return 0; }
    return n;
}

int ct_hal_cuda_set_device(int device) { return ct__cuda_status(cudaSetDevice(device), "cudaSetDevice"); }

int ct_hal_cuda_device_info(int device, int *cc, int *n_sms, uint64_t *hbm_bytes) {
    struct cudaDeviceProp p;
    int rc = ct__cuda_status(cudaGetDeviceProperties(&p, device), "cudaGetDeviceProperties");
    if (rc) return rc;
    if (cc) *cc = p.major * 10 + p.minor;
    if (n_sms) *n_sms = p.multiProcessorCount;
    if (hbm_bytes) *hbm_bytes = (uint64_t)p.totalGlobalMem;
    return CT_OK;
}

void *ct_hal_cuda_alloc(size_t bytes) {
    void *p = NULL;
    if (ct__cuda_status(cudaMalloc(&p, bytes ? bytes : 16), "cudaMalloc")) return NULL;
    return p;
}

void ct_hal_cuda_free(void *p) { if (p) cudaFree(p); }

void *ct_hal_cuda_alloc_host(size_t bytes) {
    void *p = NULL;
    if (ct__cuda_status(cudaMallocHost(&p, bytes ? bytes : 16), "cudaMallocHost")) return NULL;
    return p;
}

void ct_hal_cuda_free_host(void *p) { if (p) cudaFreeHost(p); }

int ct_hal_cuda_memcpy(void *dst, const void *src, size_t bytes, int kind, void *stream) {
    if (!dst || !src) return CT_ERR_ARG;
    if (bytes == 0) return CT_OK;
    enum cudaMemcpyKind k = kind == 0 ? cudaMemcpyHostToDevice : kind == 1 ? cudaMemcpyDeviceToHost
                                                                           : cudaMemcpyDeviceToDevice;
    return ct__cuda_status(cudaMemcpyAsync(dst, src, bytes, k, (cudaStream_t)stream), "cudaMemcpyAsync");
}

int ct_hal_cuda_memset(void *dst, int value, size_t bytes, void *stream) {
    if (!dst) return CT_ERR_ARG;
    return ct__cuda_status(cudaMemsetAsync(dst, value, bytes, (cudaStream_t)stream), "cudaMemsetAsync");
}

void *ct_hal_cuda_stream_create(void) {
    cudaStream_t s = NULL;
    if (ct__cuda_status(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate")) return NULL;
    return (void *)s;
}

void ct_hal_cuda_stream_destroy(void *stream) { if (stream) cudaStreamDestroy((cudaStream_t)stream); }

int ct_hal_cuda_stream_sync(void *stream) {
    return ct__cuda_status(cudaStreamSynchronize((cudaStream_t)stream), "cudaStreamSynchronize");
}

int ct_hal_cuda_device_sync(void) { return ct__cuda_status(cudaDeviceSynchronize(), "cudaDeviceSynchronize"); }

void *ct_hal_cuda_event_create(void) {
    cudaEvent_t e = NULL;
    if (ct__cuda_status(cudaEventCreate(&e), "cudaEventCreate")) return NULL;
    return (void *)e;
}

void ct_hal_cuda_event_destroy(void *ev) { if (ev) cudaEventDestroy((cudaEvent_t)ev); }

int ct_hal_cuda_event_record(void *ev, void *stream) {
    return ct__cuda_status(cudaEventRecord((cudaEvent_t)ev, (cudaStream_t)stream), "cudaEventRecord");
}

float ct_hal_cuda_event_elapsed_ms(void *start, void *end) {
    float ms = -1.0f;
    if (ct__cuda_status(cudaEventSynchronize((cudaEvent_t)end), "cudaEventSynchronize")) return -1.0f;
    if (ct__cuda_status(cudaEventElapsedTime(&ms, (cudaEvent_t)start, (cudaEvent_t)end), "cudaEventElapsedTime"))
        return -1.0f;
    return ms;
}
