// api_native.cu -- extern "C" entry points of include/vspec_b200.h (GEMV part,
// error state, device info).
#include "common.cuh"

#include <stdlib.h>
#include "lowbit_kernels.cuh"

#include <stdarg.h>
#include <stdio.h>
#include <string.h>

namespace vb200 {

static thread_local char g_last_error[512] = "ok";

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
}

}  // namespace vb200

// The same thread-local message for the C host layer (declared in
// host/bridge_internal.h; not part of the public headers).
extern "C" void vb_set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(vb200::g_last_error, sizeof(vb200::g_last_error), fmt, ap);
    va_end(ap);
}

namespace vb200 {

int cuda_status(cudaError_t e, const char* what) {
    set_error("%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
    return VSPEC_B200_ERR_CUDA;
}

struct DevInfo {
    int valid;
    int sms, major, minor;
    size_t smem_optin;
};
static DevInfo g_dev[64];

static const DevInfo* dev_info() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    DevInfo& d = g_dev[dev];
    if (!d.valid) {
        cudaDeviceProp prop;
        if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return nullptr;
        d.sms = prop.multiProcessorCount;
        d.major = prop.major;
        d.minor = prop.minor;
        d.smem_optin = prop.sharedMemPerBlockOptin;
        d.valid = 1;
    }
    return &d;
}

bool pdl_allowed() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("VSPEC_B200_PDL");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v == 1;
}

int device_sm_count() {
    const DevInfo* d = dev_info();
    return d ? d->sms : 148;
}

}  // namespace vb200

using namespace vb200;

extern "C" const char* vspec_b200_last_error(void) { return g_last_error; }

extern "C" const char* vspec_b200_version(void) { return "vspec_b200 0.1 (sm_100a)"; }

extern "C" int vspec_b200_device_info(int* sm_count, int* cc_major, int* cc_minor, size_t* smem_optin) {
    const DevInfo* d = dev_info();
    if (!d) { set_error("no CUDA device"); return VSPEC_B200_ERR_CUDA; }
    if (sm_count) *sm_count = d->sms;
    if (cc_major) *cc_major = d->major;
    if (cc_minor) *cc_minor = d->minor;
    if (smem_optin) *smem_optin = d->smem_optin;
    return VSPEC_B200_OK;
}

static int linear_common(const VspecB200LinearArgs* a, void* stream, int path) {
    if (!a) { set_error("args is NULL"); return VSPEC_B200_ERR_ARG; }
    if (!a->d_x || !a->d_w || !a->d_y) { set_error("NULL x/w/y"); return VSPEC_B200_ERR_ARG; }
    if (a->m == 0 || a->n == 0 || a->k == 0) { set_error("zero dimension"); return VSPEC_B200_ERR_ARG; }
    if (a->m > (1u << 24) || a->n > (1u << 30) || a->k > (1u << 30)) { set_error("dimension too large"); return VSPEC_B200_ERR_ARG; }
    if ((a->flags & VSPEC_B200_F_RESIDUAL) && !a->d_residual) { set_error("RESIDUAL without residual"); return VSPEC_B200_ERR_ARG; }
    if ((a->flags & VSPEC_B200_F_RMSNORM) && !a->d_norm_weight) { set_error("RMSNORM without weight"); return VSPEC_B200_ERR_ARG; }
    if ((a->flags & VSPEC_B200_F_SWIGLU) && (a->flags & VSPEC_B200_F_RESIDUAL)) {
        set_error("SWIGLU and RESIDUAL cannot be combined"); return VSPEC_B200_ERR_ARG;
    }
    size_t groups = a->n_groups ? a->n_groups : 1;
    if (groups > a->k) { set_error("n_groups (%zu) > k (%zu)", groups, a->k); return VSPEC_B200_ERR_ARG; }
    GemvParams p;
    memset(&p, 0, sizeof(p));
    p.x = a->d_x;
    p.w = a->d_w;
    p.s = a->d_scales;
    p.zp = a->d_zero_points;
    p.zp_const = a->zero_point_const;
    p.y = a->d_y;
    p.residual = a->d_residual;
    p.norm_w = a->d_norm_weight;
    p.eps = a->norm_eps;
    p.m = (int)a->m;
    p.n = (int)a->n;
    p.k = (int)a->k;
    p.n_groups = (int)groups;
    p.row_bytes = (int)row_bytes_for(a->k, a->bits);
    p.flags = a->flags;
    const int uns = (a->flags & VSPEC_B200_F_UNSIGNED) ? 1 : 0;
    cudaStream_t st = (cudaStream_t)stream;
    return lowbit_gemv_launch(p, a->bits, uns, st, path, a->d_workspace, a->workspace_bytes);
}

extern "C" int vspec_b200_lowbit_linear(const VspecB200LinearArgs* a, void* stream) {
    return linear_common(a, stream, kPathAuto);
}

extern "C" int vspec_b200_lowbit_linear_generic(const VspecB200LinearArgs* a, void* stream) {
    return linear_common(a, stream, kPathGeneric);
}

extern "C" int vspec_b200_lowbit_linear_path(const VspecB200LinearArgs* a, void* stream, int path) {
    if (path < kPathAuto || path > kPathRows) { set_error("unknown path %d", path); return VSPEC_B200_ERR_ARG; }
    return linear_common(a, stream, path);
}

extern "C" int vspec_b200_gemv_timeout_flag(int* out_flag) {
    if (!out_flag) { set_error("NULL out_flag"); return VSPEC_B200_ERR_ARG; }
    int a = 0, b = 0, c = 0, d = 0;
    int rc = gemv_tc_read_and_clear_timeout(&a);
    if (rc != VSPEC_B200_OK) return rc;
    rc = gemv_ring_read_and_clear_timeout(&b);
    if (rc != VSPEC_B200_OK) return rc;
    rc = gemm_tc_read_and_clear_timeout(&c);
    if (rc != VSPEC_B200_OK) return rc;
    rc = gemv_rows_read_and_clear_timeout(&d);
    if (rc != VSPEC_B200_OK) return rc;
    *out_flag = (a || b || c || d) ? 1 : 0;
    return VSPEC_B200_OK;
}

extern "C" size_t vspec_b200_lowbit_linear_workspace_bytes(size_t m, size_t n, size_t k, int flags) {
    return gemv_workspace_bytes((int)m, (int)n, (int)k, (flags & VSPEC_B200_F_SWIGLU) != 0);
}

extern "C" int vspec_b200_unpack_codes(const uint8_t* d_w, size_t n, size_t k, int bits, int unsigned_codes,
                                       int8_t* d_codes, int use_fast_decoder, void* stream) {
    if (!d_w || !d_codes || n == 0 || k == 0) { set_error("bad unpack arguments"); return VSPEC_B200_ERR_ARG; }
    if (bits < 2 || bits > 4) { set_error("bits must be 2..4"); return VSPEC_B200_ERR_ARG; }
    return unpack_codes_launch(d_w, (int)n, (int)k, bits, unsigned_codes, d_codes, (cudaStream_t)stream,
                               use_fast_decoder);
}
