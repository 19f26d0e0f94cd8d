/* xfer.c -- host<->device transfer helpers, environment parsing, the
 * reference's sampled weight fingerprint, and the allocation fault hook. */
#include <stdlib.h>
#include <string.h>

#include "bridge_internal.h"

static VB_THREAD_LOCAL VbXfer g_xfer;
static VB_THREAD_LOCAL int g_xfer_ready = 0;

/* Allocation fault injection (tests): -1 = off, otherwise the number of
 * device allocations that still succeed before one fails. */
static int g_fail_alloc_after = -1;

int vspec_b200_debug_fail_alloc_after(int n) {
    g_fail_alloc_after = n;
    return VSPEC_B200_OK;
}

int vb_alloc_should_fail(void) {
    if (g_fail_alloc_after < 0) return 0;
    if (g_fail_alloc_after == 0) {
        g_fail_alloc_after = -1;
        return 1;
    }
    g_fail_alloc_after -= 1;
    return 0;
}

VbXfer* vb_xfer(void) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return NULL;
    if (g_xfer_ready && g_xfer.device != dev) {
        /* buffers belong to another device: start over on this one */
        memset(&g_xfer, 0, sizeof(g_xfer));
        g_xfer_ready = 0;
    }
    if (!g_xfer_ready) {
        memset(&g_xfer, 0, sizeof(g_xfer));
        if (cudaStreamCreateWithFlags(&g_xfer.stream, cudaStreamNonBlocking) != cudaSuccess) return NULL;
        g_xfer.device = dev;
        g_xfer_ready = 1;
    }
    return &g_xfer;
}

int vb_ensure_device(void** p, size_t* cap, size_t bytes) {
    if (*cap >= bytes && *p) return 1;
    if (vb_alloc_should_fail()) return 0;
    if (*p) cudaFree(*p);
    *p = NULL;
    *cap = 0;
    size_t want = bytes < 4096 ? 4096 : bytes;
    if (cudaMalloc(p, want) != cudaSuccess) { *p = NULL; return 0; }
    *cap = want;
    return 1;
}

int vb_ensure_host(void** p, size_t* cap, size_t bytes) {
    if (*cap >= bytes && *p) return 1;
    if (*p) cudaFreeHost(*p);
    *p = NULL;
    *cap = 0;
    size_t want = bytes < 4096 ? 4096 : bytes;
    if (cudaMallocHost(p, want) != cudaSuccess) { *p = NULL; return 0; }
    *cap = want;
    return 1;
}

int vb_upload(VbXfer* x, void* d_dst, const void* h_src, size_t bytes) {
    if (bytes == 0) return 1;
    if (!vb_ensure_host((void**)&x->h_in, &x->h_in_cap, bytes)) return 0;
    memcpy(x->h_in, h_src, bytes);
    return cudaMemcpyAsync(d_dst, x->h_in, bytes, cudaMemcpyHostToDevice, x->stream) == cudaSuccess;
}

int vb_download(VbXfer* x, void* h_dst, const void* d_src, size_t bytes) {
    if (bytes == 0) return 1;
    if (!vb_ensure_host((void**)&x->h_out, &x->h_out_cap, bytes)) return 0;
    if (cudaMemcpyAsync(x->h_out, d_src, bytes, cudaMemcpyDeviceToHost, x->stream) != cudaSuccess) return 0;
    if (cudaStreamSynchronize(x->stream) != cudaSuccess) return 0;
    memcpy(h_dst, x->h_out, bytes);
    return 1;
}

uint64_t vb_hash_sample(const void* ptr, size_t bytes, size_t sample_count) {
    /* FNV-1a over every step-th byte, then the length (cuda_bridge.c:145-160). */
    if (!ptr || bytes == 0) return 0;
    const uint8_t* p = (const uint8_t*)ptr;
    const size_t samples = sample_count ? sample_count : 64;
    const size_t step = bytes / samples + 1;
    uint64_t h = 1469598103934665603ULL;
    for (size_t i = 0; i < bytes; i += step) {
        h ^= (uint64_t)p[i];
        h *= 1099511628211ULL;
    }
    h ^= (uint64_t)bytes;
    h *= 1099511628211ULL;
    return h;
}

int vb_env_flag(const char* name, int fallback) {
    const char* v = getenv(name);
    if (!v || !v[0]) return fallback;
    return (v[0] == '1' || v[0] == 'y' || v[0] == 'Y' || v[0] == 't' || v[0] == 'T') ? 1 : 0;
}

float vb_env_float(const char* name, float fallback) {
    const char* v = getenv(name);
    if (!v || !v[0]) return fallback;
    return (float)atof(v);
}

size_t vb_env_size(const char* name, size_t fallback) {
    const char* v = getenv(name);
    if (!v || !v[0]) return fallback;
    long long p = atoll(v);
    return p > 0 ? (size_t)p : fallback;
}
