#ifndef CT_HAL_H
#define CT_HAL_H

/*
 * hal.h -- hardware abstraction: host scorecard + the CUDA backend.
 *
 * Part 1 keeps the reference interface of src/hal/hal.h:22-170 unchanged
 * (enums, ct_hardware_scorecard_t layout, ct_hal_* signatures).  On Linux the
 * reference fills fixed fallbacks (hal.c:43-47,110-115,276-280); here RAM
 * and CPU come from the OS and the GPU fields from the CUDA runtime.  The
 * strategy rule is the reference's (hal.c:285-305).
 *
 * Part 2 is the thin C-ABI CUDA backend every other module uses: devices,
 * memory, copies, streams, events, status codes.
 */

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ======================================================================== */
/* Part 1 -- reference interface (src/hal/hal.h:22-170)                     */
/* ======================================================================== */

typedef enum {
    CT_SSD_UNKNOWN = 0, CT_SSD_NVME, CT_SSD_SATA, CT_SSD_USB, CT_SSD_HDD, CT_SSD_RAMDISK,
} ct_ssd_type_t;

static inline const char *ct_ssd_type_name(ct_ssd_type_t t) {
    switch (t) {
        case CT_SSD_NVME:    return "NVMe";
        case CT_SSD_SATA:    return "SATA";
        case CT_SSD_USB:     return "USB";
        case CT_SSD_HDD:     return "HDD";
        case CT_SSD_RAMDISK: return "RAMDISK";
        default:             return "Unknown";
    }
}

typedef enum {
    CT_GPU_NONE = 0, CT_GPU_CUDA, CT_GPU_METAL, CT_GPU_ROCM, CT_GPU_VULKAN, CT_GPU_INTEL,
} ct_gpu_type_t;

static inline const char *ct_gpu_type_name(ct_gpu_type_t t) {
    switch (t) {
        case CT_GPU_CUDA:   return "CUDA";
        case CT_GPU_METAL:  return "Metal";
        case CT_GPU_ROCM:   return "ROCm";
        case CT_GPU_VULKAN: return "Vulkan";
        case CT_GPU_INTEL:  return "Intel";
        default:            return "None";
    }
}

typedef enum {
    CT_SIMD_NONE = 0, CT_SIMD_SSE2, CT_SIMD_AVX, CT_SIMD_AVX2, CT_SIMD_AVX512, CT_SIMD_NEON, CT_SIMD_SVE,
} ct_simd_t;

static inline const char *ct_simd_name(ct_simd_t s) {
    switch (s) {
        case CT_SIMD_AVX512: return "AVX-512";
        case CT_SIMD_AVX2:   return "AVX2";
        case CT_SIMD_AVX:    return "AVX";
        case CT_SIMD_SSE2:   return "SSE2";
        case CT_SIMD_NEON:   return "NEON";
        case CT_SIMD_SVE:    return "SVE";
        default:             return "None";
    }
}

typedef enum {
    CT_STRATEGY_RESIDENT = 0, CT_STRATEGY_STREAM, CT_STRATEGY_STREAM_NEN, CT_STRATEGY_OFFLOAD,
} ct_strategy_t;

static inline const char *ct_strategy_name(ct_strategy_t s) {
    switch (s) {
        case CT_STRATEGY_RESIDENT:   return "resident";
        case CT_STRATEGY_STREAM:     return "stream";
        case CT_STRATEGY_STREAM_NEN: return "stream+nén";
        case CT_STRATEGY_OFFLOAD:    return "offload";
        default:                     return "unknown";
    }
}

/* hal.h:116-145, same field order and types. */
typedef struct {
    uint64_t ram_total_bytes;
    uint64_t ram_avail_bytes;
    uint64_t ram_model_budget;
    uint32_t cpu_cores_physical;
    uint32_t cpu_cores_logical;
    ct_simd_t cpu_simd;
    double   cpu_ghz;
    bool     gpu_present;
    ct_gpu_type_t gpu_type;
    uint64_t gpu_vram_bytes;
    ct_ssd_type_t ssd_type;
    double   ssd_read_mbps;
    double   ssd_read_iops;
    ct_strategy_t suggested_strategy;
    uint64_t model_size_bytes;
    uint64_t model_n_params;
    bool     model_is_moe;
} ct_hardware_scorecard_t;

/* hal.h:153-170 */
const ct_hardware_scorecard_t *ct_hal_detect(void);
const ct_hardware_scorecard_t *ct_hal_redetect(void);
ct_strategy_t ct_hal_set_model(uint64_t model_bytes, uint64_t n_params, bool is_moe);
ct_strategy_t ct_hal_set_ram_budget(uint64_t ram_budget_bytes);
const ct_hardware_scorecard_t *ct_hal_get(void);
void ct_hal_print(const ct_hardware_scorecard_t *sc);

/* ======================================================================== */
/* Part 2 -- CUDA backend (new; replaces the Windows nvcuda.dll probe of    */
/* hal.c:126-157 and the CPU loops under kv_cache / attention / quant)      */
/* ======================================================================== */

/* Status codes returned by every device entry point of this library. */
typedef enum {
    CT_OK = 0,
    CT_ERR_ARG = -1,        /* NULL pointer, bad size, out of range */
    CT_ERR_CUDA = -2,       /* a CUDA call failed; see ct_hal_cuda_last_error() */
    CT_ERR_NOMEM = -3,      /* host or device allocation failed */
    CT_ERR_FULL = -4,       /* no page can be freed for an append */
    CT_ERR_UNMAPPED = -5,   /* a requested token lies in an evicted page */
    CT_ERR_UNSUPPORTED = -6,
    CT_ERR_IO = -7,
} ct_status_t;

int         ct_hal_cuda_device_count(void);
int         ct_hal_cuda_set_device(int device);
/* Compute capability (e.g. 100 for sm_100), SM count, total HBM bytes. */
int         ct_hal_cuda_device_info(int device, int *cc, int *n_sms, uint64_t *hbm_bytes);
void       *ct_hal_cuda_alloc(size_t bytes);                     /* device memory, NULL on failure */
void        ct_hal_cuda_free(void *p);
void       *ct_hal_cuda_alloc_host(size_t bytes);                /* pinned host memory */
void        ct_hal_cuda_free_host(void *p);
/* kind: 0 host->device, 1 device->host, 2 device->device (async on stream). */
int         ct_hal_cuda_memcpy(void *dst, const void *src, size_t bytes, int kind, void *stream);
int         ct_hal_cuda_memset(void *dst, int value, size_t bytes, void *stream);
void       *ct_hal_cuda_stream_create(void);
void        ct_hal_cuda_stream_destroy(void *stream);
int         ct_hal_cuda_stream_sync(void *stream);
int         ct_hal_cuda_device_sync(void);
void       *ct_hal_cuda_event_create(void);
void        ct_hal_cuda_event_destroy(void *ev);
int         ct_hal_cuda_event_record(void *ev, void *stream);
/* Milliseconds between two recorded events (synchronises on `end`). */
float       ct_hal_cuda_event_elapsed_ms(void *start, void *end);
/* Message of the last CUDA failure seen by this library ("" if none). */
const char *ct_hal_cuda_last_error(void);
/* Kernels this library has launched so far in this process. */
uint64_t    ct_hal_cuda_launch_count(void);
/* Library version string. */
const char *ct_hal_version(void);

#ifdef __cplusplus
}
#endif

#endif /* CT_HAL_H */
