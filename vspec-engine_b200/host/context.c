/* context.c -- VspecKernelContext launchers of include/vspec/kernel/cuda_fused.h
 * and the CUDA VspecBackend (src/kernel/cuda/cuda_backend_stub.c,
 * src/kernel/cuda/cuda_linear_int4.cu:72-114).
 *
 * Host pointers in, host pointers out, synchronous; invalid contexts are a
 * silent no-op, as in the reference.  Weights are cached on the device per
 * host thread by (pointer, size, sampled fingerprint).
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "bridge_internal.h"

/* Mean-code zero-points per cached int4 weight (the CPU backend's semantics,
 * src/kernel/cpu/cpu_backend.c:18-26 -> src/quant/int4.c:47-67). */
typedef struct VbZpEntry {
    const unsigned char* d_w;
    size_t n, k;
    float* d_zp;
} VbZpEntry;
#define VB_ZP_CACHE 64
static VB_THREAD_LOCAL VbZpEntry g_zp_cache[VB_ZP_CACHE];
static VB_THREAD_LOCAL int g_zp_next = 0;

static float* mean_code_zp(const unsigned char* d_w, size_t n, size_t k, cudaStream_t st) {
    for (int i = 0; i < VB_ZP_CACHE; ++i)
        if (g_zp_cache[i].d_w == d_w && g_zp_cache[i].n == n && g_zp_cache[i].k == k && g_zp_cache[i].d_zp)
            return g_zp_cache[i].d_zp;
    VbZpEntry* e = &g_zp_cache[g_zp_next];
    g_zp_next = (g_zp_next + 1) % VB_ZP_CACHE;
    if (e->d_zp) cudaFree(e->d_zp);
    memset(e, 0, sizeof(*e));
    if (cudaMalloc((void**)&e->d_zp, n * sizeof(float)) != cudaSuccess) { e->d_zp = NULL; return NULL; }
    if (vspec_b200_mean_code_zero_points(d_w, n, k, 4, e->d_zp, (void*)st) != VSPEC_B200_OK) {
        cudaFree(e->d_zp);
        e->d_zp = NULL;
        return NULL;
    }
    e->d_w = d_w;
    e->n = n;
    e->k = k;
    return e->d_zp;
}

/* y = W x for host x/y with an optional row clamp of x first. */
static void run_ctx_linear(VspecKernelContext* ctx, int bits, int zp_mode, float clamp_alpha) {
    /* zp_mode: 0 = none, 1 = per-row mean code */
    const size_t m = ctx->config.m, n = ctx->config.n, k = ctx->config.k;
    if (m == 0 || n == 0 || k == 0) return;
    const size_t bytes_w = n * ((k * (size_t)bits + 7) / 8);
    const size_t bytes_s = n * sizeof(float);
    VbCacheEntry* e = vb_weight_cache(bits, ctx->weight, bytes_w, ctx->qmeta.scales, bytes_s, NULL, 0, 0,
                                      bits == 4 ? "VSPEC_INT4_WEIGHT_CACHE_CAP" : "VSPEC_INT3_WEIGHT_CACHE_CAP");
    if (!e) return;
    VbXfer* x = vb_xfer();
    if (!x) return;
    const size_t bytes_in = m * k * sizeof(float), bytes_out = m * n * sizeof(float);
    if (!vb_ensure_device((void**)&x->d_in, &x->d_in_cap, bytes_in)) return;
    if (!vb_ensure_device((void**)&x->d_out, &x->d_out_cap, bytes_out)) return;
    if (!vb_upload(x, x->d_in, ctx->input, bytes_in)) return;
    const float* d_input = x->d_in;
    if (clamp_alpha > 0.0f) {
        if (!vb_ensure_device((void**)&x->d_tmp, &x->d_tmp_cap, bytes_in)) return;
        if (vspec_b200_clamp_rows_std(x->d_in, x->d_tmp, m, k, clamp_alpha, (void*)x->stream) != VSPEC_B200_OK) return;
        d_input = x->d_tmp;
    }
    VspecB200LinearArgs a;
    memset(&a, 0, sizeof(a));
    a.d_x = d_input;
    a.d_w = e->d_w;
    a.d_scales = e->d_s;
    a.d_y = x->d_out;
    a.m = m; a.n = n; a.k = k;
    a.n_groups = 1;
    a.bits = bits;
    if (zp_mode == 1) {
        a.d_zero_points = mean_code_zp(e->d_w, n, k, x->stream);
        if (!a.d_zero_points) return;
    }
    if (vspec_b200_lowbit_linear(&a, (void*)x->stream) != VSPEC_B200_OK) return;
    (void)vb_download(x, ctx->output, x->d_out, bytes_out);
}

void vspec_cuda_launch_fused_linear_int4(VspecKernelContext* ctx) {
    /* fused_linear_int4.cu:545-638: per-row scales, zp = NULL, optional
     * VSPEC_FUSED_INPUT_CLAMP_ENABLE row clamp (alpha VSPEC_FUSED_INPUT_CLAMP_ALPHA, 6). */
    if (!ctx || !ctx->input || !ctx->weight || !ctx->output) return;
    if (ctx->qmeta.type != VSPEC_QUANT_INT4 || !ctx->qmeta.scales) return;
    float alpha = 0.0f;
    if (vb_env_flag("VSPEC_FUSED_INPUT_CLAMP_ENABLE", 0)) alpha = vb_env_float("VSPEC_FUSED_INPUT_CLAMP_ALPHA", 6.0f);
    run_ctx_linear(ctx, 4, 0, alpha);
}

void vspec_cuda_launch_fused_linear_int3_storage(VspecKernelContext* ctx) {
    /* fused_linear_int4.cu:640-745: int3 codes expanded to int4 then the int4
     * kernel with per-row scales and zp = NULL -- the plain int3 contraction,
     * computed here without the expansion pass. */
    if (!ctx || !ctx->input || !ctx->weight || !ctx->output) return;
    if (ctx->qmeta.type != VSPEC_QUANT_INT3 || !ctx->qmeta.scales) return;
    float alpha = 0.0f;
    if (vb_env_flag("VSPEC_FUSED_INPUT_CLAMP_ENABLE", 0)) alpha = vb_env_float("VSPEC_FUSED_INPUT_CLAMP_ALPHA", 6.0f);
    run_ctx_linear(ctx, 3, 0, alpha);
}

void vspec_cuda_launch_fused_linear_int3(VspecKernelContext* ctx) {
    /* fused_linear_int3.cu:168-249: rows clamped to +-2.8 std, then the
     * block-normalized int3 kernel with stochastic rounding unless
     * VSPEC_3BIT_STOCHASTIC_ROUNDING starts with 0/n/N/f/F. */
    if (!ctx || !ctx->input || !ctx->weight || !ctx->output) return;
    if (ctx->qmeta.type != VSPEC_QUANT_INT3 || !ctx->qmeta.scales) return;
    const size_t m = ctx->config.m, n = ctx->config.n, k = ctx->config.k;
    if (m == 0 || n == 0 || k == 0) return;
    int sr = 1;
    const char* env = getenv("VSPEC_3BIT_STOCHASTIC_ROUNDING");
    if (env && env[0] && (env[0] == '0' || env[0] == 'n' || env[0] == 'N' || env[0] == 'f' || env[0] == 'F')) sr = 0;
    const size_t bytes_w = n * ((k * 3 + 7) / 8), bytes_s = n * sizeof(float);
    VbCacheEntry* e = vb_weight_cache(3, ctx->weight, bytes_w, ctx->qmeta.scales, bytes_s, NULL, 0, 0,
                                      "VSPEC_INT3_WEIGHT_CACHE_CAP");
    if (!e) return;
    VbXfer* x = vb_xfer();
    if (!x) return;
    const size_t bytes_in = m * k * sizeof(float), bytes_out = m * n * sizeof(float);
    if (!vb_ensure_device((void**)&x->d_in, &x->d_in_cap, bytes_in)) return;
    if (!vb_ensure_device((void**)&x->d_tmp, &x->d_tmp_cap, bytes_in)) return;
    if (!vb_ensure_device((void**)&x->d_out, &x->d_out_cap, bytes_out)) return;
    if (!vb_upload(x, x->d_in, ctx->input, bytes_in)) return;
    if (vspec_b200_clamp_rows_std(x->d_in, x->d_tmp, m, k, 2.8f, (void*)x->stream) != VSPEC_B200_OK) return;
    if (vspec_b200_int3_blocknorm_linear(x->d_tmp, e->d_w, e->d_s, x->d_out, m, n, k, sr, (void*)x->stream) !=
        VSPEC_B200_OK)
        return;
    (void)vb_download(x, ctx->output, x->d_out, bytes_out);
}

void vspec_cuda_launch_fused_linear_int2(VspecKernelContext* ctx) {
    /* fused_linear_int2.cu:153-212: unsigned codes, (q - 1.5) * s[row] */
    if (!ctx || !ctx->input || !ctx->weight || !ctx->output) return;
    if (ctx->qmeta.type != VSPEC_QUANT_INT2 || !ctx->qmeta.scales) return;
    const size_t m = ctx->config.m, n = ctx->config.n, k = ctx->config.k;
    if (m == 0 || n == 0 || k == 0) return;
    const size_t bytes_w = n * ((k + 3) / 4), bytes_s = n * sizeof(float);
    VbCacheEntry* e = vb_weight_cache(2, ctx->weight, bytes_w, ctx->qmeta.scales, bytes_s, NULL, 0, 0,
                                      "VSPEC_INT2_WEIGHT_CACHE_CAP");
    if (!e) return;
    VbXfer* x = vb_xfer();
    if (!x) return;
    const size_t bytes_in = m * k * sizeof(float), bytes_out = m * n * sizeof(float);
    if (!vb_ensure_device((void**)&x->d_in, &x->d_in_cap, bytes_in)) return;
    if (!vb_ensure_device((void**)&x->d_out, &x->d_out_cap, bytes_out)) return;
    if (!vb_upload(x, x->d_in, ctx->input, bytes_in)) return;
    VspecB200LinearArgs a;
    memset(&a, 0, sizeof(a));
    a.d_x = x->d_in;
    a.d_w = e->d_w;
    a.d_scales = e->d_s;
    a.zero_point_const = -0.5f;
    a.d_y = x->d_out;
    a.m = m; a.n = n; a.k = k;
    a.n_groups = 1;
    a.bits = 2;
    a.flags = VSPEC_B200_F_UNSIGNED;
    if (vspec_b200_lowbit_linear(&a, (void*)x->stream) != VSPEC_B200_OK) return;
    (void)vb_download(x, ctx->output, x->d_out, bytes_out);
}

/* ------------------------------------------------------------- backend */
int vspec_cuda_runtime_available(void) {
    int count = 0;
    return (cudaGetDeviceCount(&count) == cudaSuccess && count > 0) ? 1 : 0;
}

void vspec_cuda_launch_linear_impl(VspecKernelContext* ctx) {
    if (!ctx || !ctx->input || !ctx->weight || !ctx->output || !ctx->qmeta.scales) return;
    if (ctx->qmeta.type == VSPEC_QUANT_INT4) {
        /* the CPU backend's contract: mean-code zero-points per row */
        run_ctx_linear(ctx, 4, 1, 0.0f);
    } else if (ctx->qmeta.type == VSPEC_QUANT_INT3) {
        vspec_cuda_launch_fused_linear_int3_storage(ctx);
    }
}

void vspec_cuda_launch_attention_impl(VspecKernelContext* ctx) { vspec_cuda_launch_attention_fused(ctx); }

static void b200_launch_linear(VspecKernelContext* ctx) { vspec_cuda_launch_linear_impl(ctx); }
static void b200_launch_attention(VspecKernelContext* ctx) { vspec_cuda_launch_attention_impl(ctx); }

int vspec_cuda_backend_available(void) { return vspec_cuda_runtime_available(); }

VspecBackend vspec_make_cuda_backend(void) {
    VspecBackend b;
    b.name = "cuda-b200";
    b.launch_linear = b200_launch_linear;
    b.launch_attention = b200_launch_attention;
    return b;
}

/* The CPU backend (src/kernel/cpu/cpu_backend.c:9-48) with its arithmetic on the device:
 * INT4 linear with mean-code zero-points, attention with attention_ref.c's clamp. */
static void b200_launch_attention_ref(VspecKernelContext* ctx) { vspec_b200_launch_attention_ref(ctx); }

VspecBackend vspec_b200_make_cpu_semantics_backend(void) {
    VspecBackend b;
    b.name = "cpu-semantics-b200";
    b.launch_linear = b200_launch_linear;
    b.launch_attention = b200_launch_attention_ref;
    return b;
}
