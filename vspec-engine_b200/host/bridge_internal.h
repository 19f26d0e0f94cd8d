/* bridge_internal.h -- shared state helpers of the host-pointer C layer. */
#ifndef VSPEC_B200_BRIDGE_INTERNAL_H
#define VSPEC_B200_BRIDGE_INTERNAL_H

#include <stddef.h>
#include <stdint.h>

#include <cuda_runtime_api.h>

#include "vspec_b200.h"
#include "vspec_b200_compat.h"

#if defined(__GNUC__)
#define VB_THREAD_LOCAL __thread
#else
#define VB_THREAD_LOCAL _Thread_local
#endif

/* Per-host-thread transfer context: a non-blocking stream and grow-only
 * pinned staging + device buffers for activations and outputs. */
typedef struct VbXfer {
    cudaStream_t stream;
    int device;
    float* h_in;   size_t h_in_cap;
    float* h_out;  size_t h_out_cap;
    float* d_in;   size_t d_in_cap;
    float* d_out;  size_t d_out_cap;
    float* d_tmp;  size_t d_tmp_cap;
} VbXfer;

VbXfer* vb_xfer(void);
int vb_ensure_device(void** p, size_t* cap, size_t bytes);
int vb_ensure_host(void** p, size_t* cap, size_t bytes);
/* H2D of `bytes` from an arbitrary host array through the pinned buffer. */
int vb_upload(VbXfer* x, void* d_dst, const void* h_src, size_t bytes);
/* D2H into an arbitrary host array through the pinned buffer (synchronous). */
int vb_download(VbXfer* x, void* h_dst, const void* d_src, size_t bytes);

/* Sampled FNV-1a fingerprint of a host buffer, the reference's weight-cache
 * key (src/python/cuda_bridge.c:145-160). */
uint64_t vb_hash_sample(const void* ptr, size_t bytes, size_t sample_count);

/* Process-wide fault injection for host-side failure tests: when the counter
 * reaches zero the next device allocation of the C layer fails. */
int vb_alloc_should_fail(void);

/* Device copy of a host weight, cached per host thread by (pointers, sizes,
 * sampled fingerprints); refreshed in place when the fingerprint changes. */
typedef struct VbCacheEntry {
    const void* host_w;
    const float* host_s;
    const float* host_zp;
    int device;
    int bits;
    unsigned char* d_w;
    float* d_s;
    float* d_zp;
    size_t bytes_w, bytes_s, bytes_zp;
    uint64_t fp_w, fp_s, fp_zp;
    uint64_t last_used;
} VbCacheEntry;

VbCacheEntry* vb_weight_cache(int bits, const void* w, size_t bytes_w, const float* s, size_t bytes_s,
                              const float* zp, size_t bytes_zp, int want_zp, const char* cap_env);

/* Sets the thread-local message vspec_b200_last_error() returns. */
void vb_set_error(const char* fmt, ...);

int vb_env_flag(const char* name, int fallback);
float vb_env_float(const char* name, float fallback);
size_t vb_env_size(const char* name, size_t fallback);

#endif
