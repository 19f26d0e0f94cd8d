/* bridge.c -- the low-bit exports of src/python/cuda_bridge.c (host pointers,
 * return 1 = ok / 0 = fail so that callers fall back, per-thread state).
 *
 * Registered int4 weights live on the device for the life of the handle;
 * each call uploads only the activations and downloads the result, through
 * pinned staging buffers on a per-thread non-blocking stream.  The compute is
 * the sm_100a group-wise kernel of vspec_b200_lowbit_linear.
 */
#include <stdlib.h>
#include <string.h>

#include "bridge_internal.h"

/* ---------------------------------------------------------------- registry
 * Handle table with the reference's semantics (cuda_bridge.c:162-311,391-500):
 * handles 1..cap, dedupe on (host pointers, byte sizes, sampled fingerprints,
 * k, n, n_blocks), LRU eviction when full, capacity VSPEC_INT4_BRIDGE_CACHE_CAP
 * (default 256, at most 512). */
#define VB_REG_CAP_MAX 512u
#define VB_REG_CAP_DEFAULT 256u

typedef struct VbRegistered {
    int active;
    int handle;
    int device;
    const unsigned char* host_w;
    const float* host_s;
    const float* host_zp;
    unsigned char* d_w;
    float* d_s;
    float* d_zp;
    size_t bytes_w, bytes_s, bytes_zp;
    size_t n, k, n_blocks;
    uint64_t fp_w, fp_s, fp_zp;
    uint64_t last_used;
    /* The whole call (activation upload, the linear, result download) as one
     * CUDA graph for the last activation count, over this thread's staging
     * buffers: a call is then one graph launch instead of two copies and a
     * launch.  Rebuilt when m or a staging buffer changes. */
    cudaGraphExec_t gexec;
    size_t g_m;
    const void *g_d_in, *g_d_out, *g_h_in, *g_h_out;
    int g_failed;   /* capture did not succeed: stay on the direct path */
} VbRegistered;

static VB_THREAD_LOCAL VbRegistered g_reg[VB_REG_CAP_MAX];
static VB_THREAD_LOCAL uint64_t g_reg_clock = 0;
static VB_THREAD_LOCAL uint64_t g_stat_calls, g_stat_hits, g_stat_misses;
static VB_THREAD_LOCAL uint64_t g_stat_reg_calls, g_stat_reg_reuse, g_stat_reg_evict;

static size_t reg_cap(void) {
    size_t cap = vb_env_size("VSPEC_INT4_BRIDGE_CACHE_CAP", VB_REG_CAP_DEFAULT);
    if (cap == 0) cap = 1;
    if (cap > VB_REG_CAP_MAX) cap = VB_REG_CAP_MAX;
    return cap;
}

static void reg_release(VbRegistered* e) {
    if (e->gexec) cudaGraphExecDestroy(e->gexec);
    if (e->d_w) cudaFree(e->d_w);
    if (e->d_s) cudaFree(e->d_s);
    if (e->d_zp) cudaFree(e->d_zp);
    memset(e, 0, sizeof(*e));
}

static VbRegistered* reg_by_handle(int handle) {
    if (handle <= 0 || (size_t)(handle - 1) >= VB_REG_CAP_MAX) return NULL;
    VbRegistered* e = &g_reg[handle - 1];
    if (!e->active || e->handle != handle) return NULL;
    return e;
}

static int dev_alloc(void** p, size_t bytes) {
    if (vb_alloc_should_fail()) return 0;
    return cudaMalloc(p, bytes ? bytes : 1) == cudaSuccess;
}

int vspec_cuda_fused_linear_int4_register_weight_bridge(const unsigned char* packed_weight, const float* scales,
                                                        const float* zero_points, size_t k, size_t n,
                                                        size_t n_blocks) {
    g_stat_reg_calls += 1;
    if (!packed_weight || !scales || k == 0 || n == 0) return 0;
    if (n_blocks == 0) n_blocks = 1;
    const size_t bytes_w = n * ((k + 1) / 2);
    const size_t bytes_s = n * n_blocks * sizeof(float);
    const size_t bytes_zp = bytes_s;
    const uint64_t fp_w = vb_hash_sample(packed_weight, bytes_w, 128);
    const uint64_t fp_s = vb_hash_sample(scales, bytes_s, 64);
    const uint64_t fp_zp = zero_points ? vb_hash_sample(zero_points, bytes_zp, 64) : 0;
    int dev = 0;
    cudaGetDevice(&dev);

    const size_t cap = reg_cap();
    for (size_t i = 0; i < cap; ++i) {
        VbRegistered* e = &g_reg[i];
        if (e->active && e->host_w == packed_weight && e->host_s == scales && e->host_zp == zero_points &&
            e->bytes_w == bytes_w && e->bytes_s == bytes_s && e->bytes_zp == bytes_zp && e->fp_w == fp_w &&
            e->fp_s == fp_s && e->fp_zp == fp_zp && e->k == k && e->n == n && e->n_blocks == n_blocks &&
            e->device == dev) {
            e->last_used = ++g_reg_clock;
            g_stat_reg_reuse += 1;
            return e->handle;
        }
    }
    VbRegistered* slot = NULL;
    for (size_t i = 0; i < cap; ++i) {
        if (!g_reg[i].active) { slot = &g_reg[i]; break; }
    }
    if (!slot) {
        size_t lru = 0;
        for (size_t i = 1; i < cap; ++i)
            if (g_reg[i].last_used < g_reg[lru].last_used) lru = i;
        slot = &g_reg[lru];
        g_stat_reg_evict += 1;
    }
    if (slot->active) reg_release(slot);
    const int idx = (int)(slot - g_reg);
    memset(slot, 0, sizeof(*slot));
    slot->handle = idx + 1;
    slot->device = dev;
    slot->host_w = packed_weight;
    slot->host_s = scales;
    slot->host_zp = zero_points;
    slot->bytes_w = bytes_w;
    slot->bytes_s = bytes_s;
    slot->bytes_zp = bytes_zp;
    slot->n = n;
    slot->k = k;
    slot->n_blocks = n_blocks;
    slot->fp_w = fp_w;
    slot->fp_s = fp_s;
    slot->fp_zp = fp_zp;
    if (!dev_alloc((void**)&slot->d_w, bytes_w) || !dev_alloc((void**)&slot->d_s, bytes_s) ||
        !dev_alloc((void**)&slot->d_zp, bytes_zp)) {
        reg_release(slot);
        return 0;
    }
    if (cudaMemcpy(slot->d_w, packed_weight, bytes_w, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(slot->d_s, scales, bytes_s, cudaMemcpyHostToDevice) != cudaSuccess ||
        (zero_points ? cudaMemcpy(slot->d_zp, zero_points, bytes_zp, cudaMemcpyHostToDevice)
                     : cudaMemset(slot->d_zp, 0, bytes_zp)) != cudaSuccess) {
        reg_release(slot);
        return 0;
    }
    slot->active = 1;
    slot->last_used = ++g_reg_clock;
    return slot->handle;
}

/* Runs y = W x for a device-resident weight with host activations/outputs. */
static int run_int4_host(VbXfer* x, const float* input, size_t m, size_t k, const unsigned char* d_w,
                         const float* d_s, const float* d_zp, size_t n, size_t n_blocks, float* output) {
    const size_t bytes_in = m * k * sizeof(float);
    const size_t bytes_out = m * n * sizeof(float);
    if (!vb_ensure_device((void**)&x->d_in, &x->d_in_cap, bytes_in)) return 0;
    if (!vb_ensure_device((void**)&x->d_out, &x->d_out_cap, bytes_out)) return 0;
    if (!vb_upload(x, x->d_in, input, bytes_in)) return 0;
    VspecB200LinearArgs a;
    memset(&a, 0, sizeof(a));
    a.d_x = x->d_in;
    a.d_w = d_w;
    a.d_scales = d_s;
    a.d_zero_points = d_zp;
    a.d_y = x->d_out;
    a.m = m; a.n = n; a.k = k;
    a.n_groups = n_blocks;
    a.bits = 4;
    if (vspec_b200_lowbit_linear(&a, (void*)x->stream) != VSPEC_B200_OK) return 0;
    return vb_download(x, output, x->d_out, bytes_out);
}

/* Captures upload + linear + download of a registered weight at m activation
 * rows on this thread's stream (after a direct call sized every buffer and
 * workspace, so nothing is allocated inside the capture). */
static void capture_call(VbXfer* x, VbRegistered* e, size_t m, size_t k) {
    if (e->gexec) { cudaGraphExecDestroy(e->gexec); e->gexec = NULL; }
    if (!vb_env_flag("VSPEC_B200_BRIDGE_GRAPH", 1)) { e->g_failed = 1; return; }
    const size_t bytes_in = m * k * sizeof(float), bytes_out = m * e->n * sizeof(float);
    cudaGraph_t g = NULL;
    if (cudaStreamBeginCapture(x->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        cudaGetLastError();
        e->g_failed = 1;
        return;
    }
    VspecB200LinearArgs a;
    memset(&a, 0, sizeof(a));
    a.d_x = x->d_in;
    a.d_w = e->d_w;
    a.d_scales = e->d_s;
    a.d_zero_points = e->d_zp;
    a.d_y = x->d_out;
    a.m = m; a.n = e->n; a.k = k;
    a.n_groups = e->n_blocks;
    a.bits = 4;
    int ok = cudaMemcpyAsync(x->d_in, x->h_in, bytes_in, cudaMemcpyHostToDevice, x->stream) == cudaSuccess;
    ok = ok && vspec_b200_lowbit_linear(&a, (void*)x->stream) == VSPEC_B200_OK;
    ok = ok && cudaMemcpyAsync(x->h_out, x->d_out, bytes_out, cudaMemcpyDeviceToHost, x->stream) == cudaSuccess;
    const cudaError_t ec = cudaStreamEndCapture(x->stream, &g);
    if (ok && ec == cudaSuccess && g && cudaGraphInstantiate(&e->gexec, g, 0) == cudaSuccess) {
        e->g_m = m;
        e->g_d_in = x->d_in;
        e->g_d_out = x->d_out;
        e->g_h_in = x->h_in;
        e->g_h_out = x->h_out;
    } else {
        e->gexec = NULL;
        e->g_failed = 1;
    }
    if (g) cudaGraphDestroy(g);
    cudaGetLastError();
}

int vspec_cuda_fused_linear_int4_cached_bridge(const float* input, size_t m, size_t k, int weight_handle,
                                               size_t expected_n, float* output) {
    g_stat_calls += 1;
    if (!input || !output || m == 0 || k == 0 || expected_n == 0 || weight_handle <= 0) {
        g_stat_misses += 1;
        return 0;
    }
    VbRegistered* e = reg_by_handle(weight_handle);
    int dev = 0;
    cudaGetDevice(&dev);
    if (!e || e->k != k || e->n != expected_n || e->device != dev) {
        g_stat_misses += 1;
        return 0;
    }
    e->last_used = ++g_reg_clock;
    VbXfer* x = vb_xfer();
    if (!x) {
        g_stat_misses += 1;
        return 0;
    }
    if (e->gexec && e->g_m == m && e->g_d_in == x->d_in && e->g_d_out == x->d_out && e->g_h_in == x->h_in &&
        e->g_h_out == x->h_out) {
        memcpy(x->h_in, input, m * k * sizeof(float));
        if (cudaGraphLaunch(e->gexec, x->stream) == cudaSuccess && cudaStreamSynchronize(x->stream) == cudaSuccess) {
            memcpy(output, x->h_out, m * e->n * sizeof(float));
            g_stat_hits += 1;
            return 1;
        }
        g_stat_misses += 1;
        return 0;
    }
    if (!run_int4_host(x, input, m, k, e->d_w, e->d_s, e->d_zp, e->n, e->n_blocks, output)) {
        g_stat_misses += 1;
        return 0;
    }
    if (!e->g_failed) capture_call(x, e, m, k);
    g_stat_hits += 1;
    return 1;
}

int vspec_cuda_fused_linear_int4_cached_many_bridge(const float* input, size_t m, size_t k, const int* weight_handles,
                                                    const size_t* output_dims, size_t handle_count, float* output) {
    /* cuda_bridge.c:621-654: outputs concatenated as consecutive [m][n_i] blocks.
     * One activation upload serves every handle; one download returns all. */
    if (!input || !weight_handles || !output_dims || !output || m == 0 || k == 0 || handle_count == 0) return 0;
    size_t total_n = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    for (size_t i = 0; i < handle_count; ++i) {
        VbRegistered* e = reg_by_handle(weight_handles[i]);
        if (weight_handles[i] <= 0 || output_dims[i] == 0 || !e || e->n != output_dims[i] || e->k != k ||
            e->device != dev)
            return 0;
        total_n += output_dims[i];
    }
    VbXfer* x = vb_xfer();
    if (!x) return 0;
    const size_t bytes_in = m * k * sizeof(float);
    const size_t bytes_out = m * total_n * sizeof(float);
    if (!vb_ensure_device((void**)&x->d_in, &x->d_in_cap, bytes_in)) return 0;
    if (!vb_ensure_device((void**)&x->d_out, &x->d_out_cap, bytes_out)) return 0;
    if (!vb_upload(x, x->d_in, input, bytes_in)) return 0;
    size_t off = 0;
    for (size_t i = 0; i < handle_count; ++i) {
        VbRegistered* e = reg_by_handle(weight_handles[i]);
        g_stat_calls += 1;
        e->last_used = ++g_reg_clock;
        VspecB200LinearArgs a;
        memset(&a, 0, sizeof(a));
        a.d_x = x->d_in;
        a.d_w = e->d_w;
        a.d_scales = e->d_s;
        a.d_zero_points = e->d_zp;
        a.d_y = x->d_out + off;
        a.m = m; a.n = e->n; a.k = k;
        a.n_groups = e->n_blocks;
        a.bits = 4;
        if (vspec_b200_lowbit_linear(&a, (void*)x->stream) != VSPEC_B200_OK) { g_stat_misses += 1; return 0; }
        g_stat_hits += 1;
        off += m * e->n;
    }
    return vb_download(x, output, x->d_out, bytes_out);
}

int vspec_cuda_int4_cached_stats_bridge(uint64_t* calls, uint64_t* hits, uint64_t* misses, uint64_t* reg_calls,
                                        uint64_t* reg_reuse, uint64_t* reg_evict) {
    if (!calls || !hits || !misses || !reg_calls || !reg_reuse || !reg_evict) return 0;
    *calls = g_stat_calls;
    *hits = g_stat_hits;
    *misses = g_stat_misses;
    *reg_calls = g_stat_reg_calls;
    *reg_reuse = g_stat_reg_reuse;
    *reg_evict = g_stat_reg_evict;
    return 1;
}

/* ------------------------------------------------------ uncached bridges
 * Same contract as cuda_bridge.c:812-1158: weights are copied on first use
 * and cached by (host pointers, sizes, sampled fingerprint), stale entries
 * (same pointers, different fingerprint) are refreshed in place. */
#define VB_WCACHE_MAX 512u
static VB_THREAD_LOCAL VbCacheEntry g_wcache[VB_WCACHE_MAX];
static VB_THREAD_LOCAL size_t g_wcache_count = 0;
static VB_THREAD_LOCAL uint64_t g_wcache_clock = 0;

static void wcache_release(VbCacheEntry* e) {
    if (e->d_w) cudaFree(e->d_w);
    if (e->d_s) cudaFree(e->d_s);
    if (e->d_zp) cudaFree(e->d_zp);
    memset(e, 0, sizeof(*e));
}

/* Returns a device copy of (w, s, zp); zp may be NULL (device zp then zero-filled
 * when want_zp, else left NULL). */
VbCacheEntry* vb_weight_cache(int bits, const void* w, size_t bytes_w, const float* s, size_t bytes_s,
                              const float* zp, size_t bytes_zp, int want_zp, const char* cap_env) {
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t fp_w = vb_hash_sample(w, bytes_w, 128);
    const uint64_t fp_s = vb_hash_sample(s, bytes_s, 64);
    const uint64_t fp_zp = zp ? vb_hash_sample(zp, bytes_zp, 64) : 0;
    size_t cap = vb_env_size(cap_env, 256);
    if (cap == 0) cap = 1;
    if (cap > VB_WCACHE_MAX) cap = VB_WCACHE_MAX;
    VbCacheEntry* hit = NULL;
    VbCacheEntry* stale = NULL;
    for (size_t i = 0; i < g_wcache_count; ++i) {
        VbCacheEntry* e = &g_wcache[i];
        if (e->host_w == w && e->host_s == s && e->host_zp == zp && e->bytes_w == bytes_w && e->bytes_s == bytes_s &&
            e->bytes_zp == bytes_zp && e->bits == bits && e->device == dev) {
            if (e->fp_w == fp_w && e->fp_s == fp_s && e->fp_zp == fp_zp) { hit = e; break; }
            stale = e;
        }
    }
    if (!hit) {
        VbCacheEntry* e = stale;
        if (!e) {
            if (g_wcache_count < cap) {
                e = &g_wcache[g_wcache_count++];
            } else {
                size_t lru = 0;
                for (size_t i = 1; i < cap; ++i)
                    if (g_wcache[i].last_used < g_wcache[lru].last_used) lru = i;
                e = &g_wcache[lru];
            }
        }
        wcache_release(e);
        e->host_w = w;
        e->host_s = s;
        e->host_zp = zp;
        e->device = dev;
        e->bits = bits;
        e->bytes_w = bytes_w;
        e->bytes_s = bytes_s;
        e->bytes_zp = bytes_zp;
        e->fp_w = fp_w;
        e->fp_s = fp_s;
        e->fp_zp = fp_zp;
        if (!dev_alloc((void**)&e->d_w, bytes_w) || !dev_alloc((void**)&e->d_s, bytes_s) ||
            (want_zp && !dev_alloc((void**)&e->d_zp, bytes_zp))) {
            wcache_release(e);
            return NULL;
        }
        if (cudaMemcpy(e->d_w, w, bytes_w, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(e->d_s, s, bytes_s, cudaMemcpyHostToDevice) != cudaSuccess) {
            wcache_release(e);
            return NULL;
        }
        if (want_zp) {
            cudaError_t rc = zp ? cudaMemcpy(e->d_zp, zp, bytes_zp, cudaMemcpyHostToDevice)
                                : cudaMemset(e->d_zp, 0, bytes_zp);
            if (rc != cudaSuccess) { wcache_release(e); return NULL; }
        }
        hit = e;
    }
    hit->last_used = ++g_wcache_clock;
    return hit;
}

int vspec_cuda_fused_linear_int4_bridge(const float* input, const unsigned char* packed_weight, const float* scales,
                                        const float* zero_points, size_t m, size_t k, size_t n, size_t n_blocks,
                                        float* output) {
    if (!input || !packed_weight || !scales || !output || m == 0 || k == 0 || n == 0) return 0;
    if (n_blocks == 0) n_blocks = 1;
    const size_t bytes_w = n * ((k + 1) / 2);
    const size_t bytes_s = n * n_blocks * sizeof(float);
    VbCacheEntry* e = vb_weight_cache(4, packed_weight, bytes_w, scales, bytes_s, zero_points, bytes_s, 1,
                                      "VSPEC_INT4_BRIDGE_CACHE_CAP");
    if (!e) return 0;
    VbXfer* x = vb_xfer();
    if (!x) return 0;
    return run_int4_host(x, input, m, k, e->d_w, e->d_s, e->d_zp, n, n_blocks, output);
}

int vspec_cuda_fused_linear_int3_bridge(const float* input, const unsigned char* packed_weight, const float* scales,
                                        size_t m, size_t k, size_t n, float* output) {
    /* cuda_bridge.c:1039-1158: per-row scales; the reference launches its
     * int3 kernel with stochastic rounding on (line 1155). */
    if (!input || !packed_weight || !scales || !output || m == 0 || k == 0 || n == 0) return 0;
    const size_t bytes_w = n * ((k * 3 + 7) / 8);
    const size_t bytes_s = n * sizeof(float);
    VbCacheEntry* e = vb_weight_cache(3, packed_weight, bytes_w, scales, bytes_s, NULL, 0, 0,
                                      "VSPEC_INT3_BRIDGE_CACHE_CAP");
    if (!e) return 0;
    VbXfer* x = vb_xfer();
    if (!x) return 0;
    const size_t bytes_in = m * k * sizeof(float), bytes_out = m * n * sizeof(float);
    if (!vb_ensure_device((void**)&x->d_in, &x->d_in_cap, bytes_in)) return 0;
    if (!vb_ensure_device((void**)&x->d_out, &x->d_out_cap, bytes_out)) return 0;
    if (!vb_upload(x, x->d_in, input, bytes_in)) return 0;
    if (vspec_b200_int3_blocknorm_linear(x->d_in, e->d_w, e->d_s, x->d_out, m, n, k, 1, (void*)x->stream) !=
        VSPEC_B200_OK)
        return 0;
    return vb_download(x, output, x->d_out, bytes_out);
}

int vspec_cuda_gemm_dispatch_bridge(const float* input, const float* weight_f32, const unsigned char* packed_weight,
                                    const float* scales, const float* zero_points, size_t m, size_t k, size_t n,
                                    size_t n_blocks, int bits, int* inout_handle, float* output, int* out_path) {
    /* cuda_bridge.c:67-143: registered int4 (path 1) -> uncached int4 (2) ->
     * int3 (3) -> fp32 GEMM on weight_f32 (4). */
    if (!input || !output || m == 0 || k == 0 || n == 0) return 0;
    if (bits == 4 && packed_weight && scales) {
        int handle = inout_handle ? *inout_handle : 0;
        if (n_blocks == 0) n_blocks = 1;
        if (handle <= 0) {
            handle = vspec_cuda_fused_linear_int4_register_weight_bridge(packed_weight, scales, zero_points, k, n,
                                                                         n_blocks);
            if (inout_handle) *inout_handle = handle;
        }
        if (handle > 0 && vspec_cuda_fused_linear_int4_cached_bridge(input, m, k, handle, n, output)) {
            if (out_path) *out_path = 1;
            return 1;
        }
        if (vspec_cuda_fused_linear_int4_bridge(input, packed_weight, scales, zero_points, m, k, n, n_blocks,
                                                output)) {
            if (out_path) *out_path = 2;
            return 1;
        }
    } else if (bits == 3 && packed_weight && scales) {
        if (vspec_cuda_fused_linear_int3_bridge(input, packed_weight, scales, m, k, n, output)) {
            if (out_path) *out_path = 3;
            return 1;
        }
    }
    if (!weight_f32) return 0;
    vspec_cuda_gemm_f32(input, weight_f32, m, k, n, output);
    if (out_path) *out_path = 4;
    return 1;
}

int vspec_cuda_mem_info_bridge(size_t* free_bytes, size_t* total_bytes) {
    if (!free_bytes || !total_bytes) return 0;
    size_t f = 0, t = 0;
    if (cudaMemGetInfo(&f, &t) != cudaSuccess) return 0;
    *free_bytes = f;
    *total_bytes = t;
    return 1;
}

int vspec_cuda_device_capability_bridge(int* out_major, int* out_minor, int* out_multiprocessors) {
    if (!out_major || !out_minor || !out_multiprocessors) return 0;
    int sms = 0, maj = 0, min = 0;
    if (vspec_b200_device_info(&sms, &maj, &min, NULL) != VSPEC_B200_OK) return 0;
    *out_major = maj;
    *out_minor = min;
    *out_multiprocessors = sms;
    return 1;
}

int vspec_cuda_int4_tensorcore_available_bridge(void) {
    /* The int4 path runs on the tensor cores whenever the device is sm_100. */
    int maj = 0, min = 0, sms = 0;
    if (!vspec_cuda_device_capability_bridge(&maj, &min, &sms)) return 0;
    return maj >= 10 ? 1 : 0;
}

/* ---------------------------------------------------------------- ANF hybrid
 * vspec_cuda_fused_linear_hybrid_(profile_)bridge (cuda_bridge.c:1160-1683):
 * device copies of the int2 and int4 weights cached per host thread (pointers,
 * sizes, sampled fingerprints; the int4 zero-points zero-filled when NULL), the
 * activations and the hot list uploaded per call, int2 draft + int4 refine on
 * the device, the result downloaded.  With VSPEC_ENABLE_ANF, VSPEC_ANF_TCC_ENABLE
 * and VSPEC_ANF_MODE=active the temporal rule of cuda_bridge.c:1352-1404 picks
 * which hot columns are refined: after VSPEC_ANF_TCC_WARMUP calls (default 4),
 * only the columns absent from the previous call's list, when they are at most
 * VSPEC_ANF_TCC_MAX_CHANGED_RATIO (0.35, clamped to [0.01, 1]) of a list of at
 * least VSPEC_ANF_TCC_MIN_HOT (1) entries.  VSPEC_INT2_COMPUTE_MODE's TF32
 * cuBLAS draft (cuda_bridge.c:1585-1619) is served by the same fused draft. */
static VB_THREAD_LOCAL uint32_t* g_hot_prev = NULL;
static VB_THREAD_LOCAL uint32_t* g_hot_added = NULL;
static VB_THREAD_LOCAL size_t g_hot_prev_count = 0, g_hot_cap = 0, g_tcc_steps = 0;

static int anf_tcc_active(void) {
    const char* mode = getenv("VSPEC_ANF_MODE");
    return vb_env_flag("VSPEC_ENABLE_ANF", 0) && vb_env_flag("VSPEC_ANF_TCC_ENABLE", 0) && mode &&
           strcmp(mode, "active") == 0;
}

static float env_float_clamped(const char* name, float def, float lo, float hi) {
    float v = vb_env_float(name, def);
    return v < lo ? lo : (v > hi ? hi : v);
}

static size_t env_size_clamped(const char* name, size_t def, size_t lo, size_t hi) {
    size_t v = vb_env_size(name, def);
    return v < lo ? lo : (v > hi ? hi : v);
}

/* Returns 0 on allocation failure; otherwise sets *active / *active_count. */
static int anf_tcc_select(const uint32_t* hot, size_t hot_count, int have_int4, const uint32_t** active,
                          size_t* active_count) {
    *active = hot;
    *active_count = hot_count;
    if (!anf_tcc_active()) {
        g_hot_prev_count = 0;
        g_tcc_steps = 0;
        return 1;
    }
    if (hot_count == 0 || !hot || !have_int4) return 1;
    const float max_ratio = env_float_clamped("VSPEC_ANF_TCC_MAX_CHANGED_RATIO", 0.35f, 0.01f, 1.0f);
    const size_t warmup = env_size_clamped("VSPEC_ANF_TCC_WARMUP", 4, 0, 1024);
    const size_t min_hot = env_size_clamped("VSPEC_ANF_TCC_MIN_HOT", 1, 1, 65536);
    g_tcc_steps += 1;
    if (g_hot_cap < hot_count) {
        uint32_t* p = (uint32_t*)realloc(g_hot_prev, hot_count * sizeof(uint32_t));
        if (!p) return 0;
        g_hot_prev = p;
        p = (uint32_t*)realloc(g_hot_added, hot_count * sizeof(uint32_t));
        if (!p) return 0;
        g_hot_added = p;
        g_hot_cap = hot_count;
    }
    if (g_tcc_steps > warmup && g_hot_prev_count > 0 && hot_count >= min_hot) {
        size_t added = 0;
        for (size_t i = 0; i < hot_count; ++i) {
            int seen = 0;
            for (size_t j = 0; j < g_hot_prev_count; ++j)
                if (g_hot_prev[j] == hot[i]) { seen = 1; break; }
            if (!seen) g_hot_added[added++] = hot[i];
        }
        if ((float)added / (float)hot_count <= max_ratio) {
            *active = g_hot_added;
            *active_count = added;
        }
    }
    memcpy(g_hot_prev, hot, hot_count * sizeof(uint32_t));
    g_hot_prev_count = hot_count;
    return 1;
}

int vspec_b200_debug_anf_tcc_select(const uint32_t* hot, size_t hot_count, int have_int4, uint32_t* out,
                                    size_t* out_count) {
    if (!out_count || (hot_count && (!hot || !out))) return VSPEC_B200_ERR_ARG;
    const uint32_t* active = NULL;
    size_t n = 0;
    if (!anf_tcc_select(hot, hot_count, have_int4, &active, &n)) return VSPEC_B200_ERR_NOMEM;
    if (n) memcpy(out, active, n * sizeof(uint32_t));
    *out_count = n;
    return VSPEC_B200_OK;
}

int vspec_cuda_fused_linear_hybrid_profile_bridge(const float* input, const unsigned char* packed_weight_int2,
                                                  const float* scales_int2, const unsigned char* packed_weight_int4,
                                                  const float* scales_int4, const float* zero_points_int4, size_t m,
                                                  size_t k, size_t n, const uint32_t* hot_indices, size_t hot_count,
                                                  size_t n_blocks_int4, float* output, float* out_h2d_ms,
                                                  float* out_kernel_ms, float* out_d2h_ms, float* out_total_gpu_ms) {
    if (!input || !packed_weight_int2 || !scales_int2 || !output || m == 0 || k == 0 || n == 0) return 0;
    if (hot_count > 0 && !hot_indices) return 0;
    if (hot_count > 0 && (!packed_weight_int4 || !scales_int4)) return 0;
    if (n_blocks_int4 == 0) n_blocks_int4 = 1;
    const uint32_t* active = NULL;
    size_t active_count = 0;
    if (!anf_tcc_select(hot_indices, hot_count, packed_weight_int4 && scales_int4, &active, &active_count)) return 0;

    const size_t bytes_w2 = n * ((k + 3) / 4), bytes_s2 = n * sizeof(float);
    VbCacheEntry* e2 = vb_weight_cache(2, packed_weight_int2, bytes_w2, scales_int2, bytes_s2, NULL, 0, 0,
                                       "VSPEC_HYBRID_BRIDGE_CACHE_CAP");
    if (!e2) return 0;
    VbCacheEntry* e4 = NULL;
    if (hot_count > 0) {
        const size_t bytes_w4 = n * ((k + 1) / 2), bytes_s4 = n * n_blocks_int4 * sizeof(float);
        e4 = vb_weight_cache(4, packed_weight_int4, bytes_w4, scales_int4, bytes_s4, zero_points_int4, bytes_s4, 1,
                             "VSPEC_HYBRID_BRIDGE_CACHE_CAP");
        if (!e4) return 0;
    }
    VbXfer* x = vb_xfer();
    if (!x) return 0;
    const size_t bytes_in = m * k * sizeof(float), bytes_out = m * n * sizeof(float);
    const size_t hot_off = (bytes_in + 255) & ~(size_t)255;
    const size_t bytes_hot = active_count * sizeof(uint32_t);
    if (!vb_ensure_device((void**)&x->d_in, &x->d_in_cap, bytes_in)) return 0;
    if (!vb_ensure_device((void**)&x->d_out, &x->d_out_cap, bytes_out)) return 0;
    if (bytes_hot && !vb_ensure_device((void**)&x->d_tmp, &x->d_tmp_cap, bytes_hot)) return 0;
    /* one pinned staging buffer for the activations and the hot list */
    if (!vb_ensure_host((void**)&x->h_in, &x->h_in_cap, hot_off + bytes_hot)) return 0;
    memcpy(x->h_in, input, bytes_in);
    if (bytes_hot) memcpy((char*)x->h_in + hot_off, active, bytes_hot);

    cudaEvent_t ev[4] = {NULL, NULL, NULL, NULL};
    const int profile = out_h2d_ms || out_kernel_ms || out_d2h_ms || out_total_gpu_ms;
    int ok = 0;
    if (profile) {
        for (int i = 0; i < 4; ++i)
            if (cudaEventCreate(&ev[i]) != cudaSuccess) goto done;
        cudaEventRecord(ev[0], x->stream);
    }
    if (cudaMemcpyAsync(x->d_in, x->h_in, bytes_in, cudaMemcpyHostToDevice, x->stream) != cudaSuccess) goto done;
    if (bytes_hot && cudaMemcpyAsync(x->d_tmp, (char*)x->h_in + hot_off, bytes_hot, cudaMemcpyHostToDevice,
                                     x->stream) != cudaSuccess)
        goto done;
    if (profile) cudaEventRecord(ev[1], x->stream);
    if (vspec_b200_anf_hybrid_linear(x->d_in, e2->d_w, e2->d_s, e4 ? e4->d_w : NULL, e4 ? e4->d_s : NULL,
                                     e4 ? e4->d_zp : NULL, x->d_out, bytes_hot ? (const uint32_t*)x->d_tmp : NULL,
                                     active_count, m, n, k, n_blocks_int4, (void*)x->stream) != VSPEC_B200_OK)
        goto done;
    if (profile) cudaEventRecord(ev[2], x->stream);
    if (!vb_ensure_host((void**)&x->h_out, &x->h_out_cap, bytes_out)) goto done;
    if (cudaMemcpyAsync(x->h_out, x->d_out, bytes_out, cudaMemcpyDeviceToHost, x->stream) != cudaSuccess) goto done;
    if (profile) cudaEventRecord(ev[3], x->stream);
    if (cudaStreamSynchronize(x->stream) != cudaSuccess) goto done;
    memcpy(output, x->h_out, bytes_out);
    if (profile) {
        float h2d = 0.f, ker = 0.f, d2h = 0.f, tot = 0.f;
        cudaEventElapsedTime(&h2d, ev[0], ev[1]);
        cudaEventElapsedTime(&ker, ev[1], ev[2]);
        cudaEventElapsedTime(&d2h, ev[2], ev[3]);
        cudaEventElapsedTime(&tot, ev[0], ev[3]);
        if (out_h2d_ms) *out_h2d_ms = h2d;
        if (out_kernel_ms) *out_kernel_ms = ker;
        if (out_d2h_ms) *out_d2h_ms = d2h;
        if (out_total_gpu_ms) *out_total_gpu_ms = tot;
    }
    ok = 1;
done:
    for (int i = 0; i < 4; ++i)
        if (ev[i]) cudaEventDestroy(ev[i]);
    return ok;
}

int vspec_cuda_fused_linear_hybrid_bridge(const float* input, const unsigned char* packed_weight_int2,
                                          const float* scales_int2, const unsigned char* packed_weight_int4,
                                          const float* scales_int4, const float* zero_points_int4, size_t m,
                                          size_t k, size_t n, const uint32_t* hot_indices, size_t hot_count,
                                          size_t n_blocks_int4, float* output) {
    return vspec_cuda_fused_linear_hybrid_profile_bridge(input, packed_weight_int2, scales_int2, packed_weight_int4,
                                                         scales_int4, zero_points_int4, m, k, n, hot_indices,
                                                         hot_count, n_blocks_int4, output, NULL, NULL, NULL, NULL);
}
