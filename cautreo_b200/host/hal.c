/*
 * hal.c -- hardware scorecard (hal.h Part 1).
 *
 * Same public behaviour as the reference src/hal/hal.c: a static scorecard,
 * detect / redetect / set_model / set_ram_budget / get / print, the RAM
 * budget of 80 % (hal.c:319-321) and the strategy rule (hal.c:285-305).
 * Detection differs where the reference's Linux branch is a fixed fallback:
 * RAM from /proc/meminfo, CPU from sysconf and /proc/cpuinfo, GPU from the
 * CUDA runtime (first device).  The SSD fields keep the reference's Linux
 * values (hal.c:276-280); SSD streaming is outside this library.
 */
#include "../../include/hal.h"

#include <cuda_runtime_api.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

static ct_hardware_scorecard_t g_sc;
static bool g_detected = false;
static uint64_t g_user_ram_budget = 0;

static uint64_t meminfo_kb(const char *key) {
    FILE *f = fopen("/proc/meminfo", "r");
    if (!f) return 0;
    char line[256];
    uint64_t v = 0;
    size_t kl = strlen(key);
    while (fgets(line, sizeof line, f)) {
        if (strncmp(line, key, kl) == 0 && line[kl] == ':') { v = strtoull(line + kl + 1, NULL, 10); break; }
    }
    fclose(f);
    return v;
}

static void detect_ram(ct_hardware_scorecard_t *sc) {
    uint64_t tot = meminfo_kb("MemTotal"), av = meminfo_kb("MemAvailable");
    sc->ram_total_bytes = tot ? tot * 1024ull : 16ull << 30;
    sc->ram_avail_bytes = av ? av * 1024ull : 8ull << 30;
}

static void detect_cpu(ct_hardware_scorecard_t *sc) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    sc->cpu_cores_logical = n > 0 ? (uint32_t)n : 1;
    uint32_t cores_per_pkg = 0, pkgs = 0;
    int seen[64] = {0};
    double mhz = 0.0;
    FILE *f = fopen("/proc/cpuinfo", "r");
    if (f) {
        char line[512];
        while (fgets(line, sizeof line, f)) {
            if (!strncmp(line, "cpu cores", 9)) { const char *c = strchr(line, ':'); if (c) cores_per_pkg = (uint32_t)atoi(c + 1); }
            else if (!strncmp(line, "physical id", 11)) {
                const char *c = strchr(line, ':');
                int id = c ? atoi(c + 1) : 0;
                if (id >= 0 && id < 64 && !seen[id]) { seen[id] = 1; pkgs++; }
            } else if (!strncmp(line, "cpu MHz", 7) && mhz == 0.0) { const char *c = strchr(line, ':'); if (c) mhz = atof(c + 1); }
        }
        fclose(f);
    }
    sc->cpu_cores_physical = (cores_per_pkg && pkgs) ? cores_per_pkg * pkgs : (sc->cpu_cores_logical + 1) / 2;
    sc->cpu_ghz = mhz > 0.0 ? mhz / 1000.0 : 2.0;
#if defined(__x86_64__) || defined(__i386__)
    __builtin_cpu_init();
    if (__builtin_cpu_supports("avx512f")) sc->cpu_simd = CT_SIMD_AVX512;
    else if (__builtin_cpu_supports("avx2")) sc->cpu_simd = CT_SIMD_AVX2;
    else if (__builtin_cpu_supports("avx")) sc->cpu_simd = CT_SIMD_AVX;
    else if (__builtin_cpu_supports("sse2")) sc->cpu_simd = CT_SIMD_SSE2;
    else sc->cpu_simd = CT_SIMD_NONE;
#elif defined(__aarch64__)
    sc->cpu_simd = CT_SIMD_NEON;
#else
    sc->cpu_simd = CT_SIMD_NONE;
#endif
}

static void detect_gpu(ct_hardware_scorecard_t *sc) {
    sc->gpu_present = false;
    sc->gpu_type = CT_GPU_NONE;
    sc->gpu_vram_bytes = 0;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) { cudaGetLastError(); return; }
    struct cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, 0) != cudaSuccess) { cudaGetLastError(); return; }
    sc->gpu_present = true;
    sc->gpu_type = CT_GPU_CUDA;
    sc->gpu_vram_bytes = (uint64_t)p.totalGlobalMem;
}

static void detect_ssd(ct_hardware_scorecard_t *sc) {
    sc->ssd_type = CT_SSD_NVME;
    sc->ssd_read_mbps = 3000.0;
    sc->ssd_read_iops = 500000.0;
}

static ct_strategy_t compute_strategy(const ct_hardware_scorecard_t *sc) {
    if (sc->model_size_bytes == 0) return CT_STRATEGY_RESIDENT;
    uint64_t budget = g_user_ram_budget > 0 ? g_user_ram_budget : sc->ram_avail_bytes;
    if (sc->model_size_bytes <= budget * 0.8) return CT_STRATEGY_RESIDENT;
    if (sc->gpu_present && sc->gpu_vram_bytes >= sc->model_size_bytes * 0.5) return CT_STRATEGY_OFFLOAD;
    if (sc->ssd_read_mbps >= 500.0) return CT_STRATEGY_STREAM;
    return CT_STRATEGY_STREAM_NEN;
}

const ct_hardware_scorecard_t *ct_hal_detect(void) {
    ct_hardware_scorecard_t *sc = &g_sc;
    memset(sc, 0, sizeof *sc);
    detect_ram(sc);
    detect_cpu(sc);
    detect_gpu(sc);
    detect_ssd(sc);
    uint64_t budget = g_user_ram_budget > 0 ? g_user_ram_budget : sc->ram_avail_bytes;
    sc->ram_model_budget = (uint64_t)(budget * 0.8);
    sc->suggested_strategy = compute_strategy(sc);
    g_detected = true;
    return sc;
}

const ct_hardware_scorecard_t *ct_hal_redetect(void) {
    g_detected = false;
    return ct_hal_detect();
}

ct_strategy_t ct_hal_set_model(uint64_t model_bytes, uint64_t n_params, bool is_moe) {
    if (!g_detected) ct_hal_detect();
    g_sc.model_size_bytes = model_bytes;
    g_sc.model_n_params = n_params;
    g_sc.model_is_moe = is_moe;
    g_sc.suggested_strategy = compute_strategy(&g_sc);
    return g_sc.suggested_strategy;
}

ct_strategy_t ct_hal_set_ram_budget(uint64_t ram_budget_bytes) {
    g_user_ram_budget = ram_budget_bytes;
    if (g_detected) {
        g_sc.ram_model_budget = (uint64_t)(ram_budget_bytes * 0.8);
        g_sc.suggested_strategy = compute_strategy(&g_sc);
    }
    return g_detected ? g_sc.suggested_strategy : CT_STRATEGY_RESIDENT;
}

const ct_hardware_scorecard_t *ct_hal_get(void) {
    if (!g_detected) return ct_hal_detect();
    return &g_sc;
}

void ct_hal_print(const ct_hardware_scorecard_t *sc) {
    if (!sc) { printf("[hal] scorecard: NULL\n"); return; }
    printf("[hal] RAM total %.2f GB, avail %.2f GB, model budget %.2f GB\n",
           (double)sc->ram_total_bytes / (1 << 30), (double)sc->ram_avail_bytes / (1 << 30),
           (double)sc->ram_model_budget / (1 << 30));
    printf("[hal] CPU %u physical / %u logical cores, %s, %.2f GHz\n", sc->cpu_cores_physical,
           sc->cpu_cores_logical, ct_simd_name(sc->cpu_simd), sc->cpu_ghz);
    printf("[hal] GPU %s", sc->gpu_present ? ct_gpu_type_name(sc->gpu_type) : "none");
    if (sc->gpu_present) printf(", %.2f GB", (double)sc->gpu_vram_bytes / (1 << 30));
    printf("\n[hal] SSD %s, %.0f MB/s, %.0f IOPS\n", ct_ssd_type_name(sc->ssd_type), sc->ssd_read_mbps,
           sc->ssd_read_iops);
    if (sc->model_size_bytes > 0)
        printf("[hal] model %.2f GB (%llu params), MoE %s\n", (double)sc->model_size_bytes / (1 << 30),
               (unsigned long long)sc->model_n_params, sc->model_is_moe ? "yes" : "no");
    printf("[hal] strategy %s\n", ct_strategy_name(sc->suggested_strategy));
}
