// api_attention.cu -- extern "C" entry points for paged attention, the fp32
// helper ops, and the reference's host-pointer attention launchers.
#include "common.cuh"
#include "attention_kernels.cuh"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "vspec_b200_compat.h"

namespace vb200 {

// Library-managed scratch for the split merge: one grow-only buffer per device.
struct Scratch {
    void* ptr;
    size_t cap;
};
static thread_local Scratch g_attn_scratch[64];

static void* attn_scratch(size_t bytes) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    Scratch& s = g_attn_scratch[dev];
    if (s.cap < bytes) {
        if (s.ptr) cudaFree(s.ptr);
        s.ptr = nullptr;
        s.cap = 0;
        if (cudaMalloc(&s.ptr, bytes) != cudaSuccess) { s.ptr = nullptr; return nullptr; }
        s.cap = bytes;
    }
    return s.ptr;
}

// ---- fp32 helper kernels ----
__global__ void rmsnorm_rows_kernel(const float* x, const float* w, float eps, size_t rows, size_t dim, float* y) {
    const size_t row = blockIdx.x;
    if (row >= rows) return;
    __shared__ float red[32];
    const float* xr = x + row * dim;
    float ss = 0.f;
    for (size_t i = threadIdx.x; i < dim; i += blockDim.x) ss += xr[i] * xr[i];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        v = warp_sum(v);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float inv = 1.0f / sqrtf(red[0] / (float)dim + eps);
    for (size_t i = threadIdx.x; i < dim; i += blockDim.x) y[row * dim + i] = xr[i] * inv * (w ? w[i] : 1.0f);
}

__global__ void linear_f32_kernel(const float* x, const float* w, size_t m, size_t k, size_t n, float* y) {
    // one warp per output element, fixed-order warp tree
    const size_t wid = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (wid >= m * n) return;
    const size_t i = wid / n, j = wid % n;
    float acc = 0.f;
    for (size_t t = lane; t < k; t += 32) acc = fmaf(x[i * k + t], w[j * k + t], acc);
    acc = warp_sum(acc);
    if (lane == 0) y[i * n + j] = acc;
}

__global__ void silu_kernel(float* d, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float v = d[i];
        d[i] = v / (1.0f + expf(-v));
    }
}

__global__ void mul_kernel(float* d, const float* o, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        d[i] = d[i] * o[i];
}

// int3 KV rows -> fp32 (src/kernel/cuda/attention_fused.cu:23-45): q * s[block].
__global__ void dequant_int3_kv_kernel(const uint8_t* packed, const float* scales, float* out, size_t rows,
                                       size_t d, size_t packed_bytes, size_t blocks, size_t block_size) {
    const size_t total = rows * d;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t row = i / d, col = i % d;
        const int q = decode_code_generic(packed + row * packed_bytes, col, 3, 0);
        out[i] = (float)q * scales[row * blocks + col / block_size];
    }
}

static unsigned grid1d(size_t n) {
    size_t b = (n + 255) / 256;
    if (b > 4096) b = 4096;
    return (unsigned)(b ? b : 1);
}

}  // namespace vb200

using namespace vb200;

extern "C" size_t vspec_b200_paged_attention_workspace_bytes(size_t batch, size_t hq, size_t hkv, size_t d,
                                                             size_t max_ctx) {
    if (batch == 0 || hq == 0 || hkv == 0 || d == 0) return 0;
    // the finer of the plans of the fp16/fp32 and the int3 kernels
    const AttnPlanShape i3 = attn_plan_int3((int)hq, (int)hkv);
    const int s2 = attn_choose_split((int)batch, (int)hq, (int)hkv, (int)(max_ctx ? max_ctx : 1), 0, device_sm_count(),
                                     kAttnPlanF16.ctas_per_sm, kAttnPlanF16.max_staged_pages);
    const int s3 = attn_choose_split((int)batch, (int)hq, (int)hkv, (int)(max_ctx ? max_ctx : 1), 0, device_sm_count(),
                                     i3.ctas_per_sm, i3.max_staged_pages);
    const int split = s2 < s3 ? s2 : s3;
    const int max_splits = (int)((max_ctx + split - 1) / split);
    return attn_workspace_bytes((int)batch, (int)hq, (int)d, max_splits > 0 ? max_splits : 1);
}

extern "C" int vspec_b200_paged_attention(const VspecB200PagedAttnArgs* a, void* stream) {
    if (!a) { set_error("args is NULL"); return VSPEC_B200_ERR_ARG; }
    if (!a->d_q || !a->d_k_pages || !a->d_v_pages || !a->d_page_table || !a->d_ctx_len || !a->d_out) {
        set_error("NULL pointer argument"); return VSPEC_B200_ERR_ARG;
    }
    if (a->batch == 0 || a->num_q_heads == 0 || a->num_kv_heads == 0 || a->head_dim == 0 || a->page_tokens == 0 ||
        a->max_pages_per_seq == 0 || a->num_pages == 0) {
        set_error("zero dimension"); return VSPEC_B200_ERR_ARG;
    }
    if (a->num_q_heads % a->num_kv_heads != 0) { set_error("num_q_heads must be a multiple of num_kv_heads"); return VSPEC_B200_ERR_ARG; }
    if (a->head_dim > 256) { set_error("head_dim > 256 unsupported"); return VSPEC_B200_ERR_UNSUPPORTED; }
    if (a->kv_dtype != VSPEC_B200_KV_F16 && a->kv_dtype != VSPEC_B200_KV_F32) { set_error("bad kv_dtype"); return VSPEC_B200_ERR_ARG; }
    if (a->max_ctx > a->max_pages_per_seq * a->page_tokens) {
        set_error("max_ctx %zu exceeds the page table capacity %zu", a->max_ctx, a->max_pages_per_seq * a->page_tokens);
        return VSPEC_B200_ERR_ARG;
    }
    const size_t max_ctx = a->max_ctx ? a->max_ctx : a->max_pages_per_seq * a->page_tokens;
    AttnParams p;
    memset(&p, 0, sizeof(p));
    p.q = a->d_q;
    p.k_pages = a->d_k_pages;
    p.v_pages = a->d_v_pages;
    p.page_table = a->d_page_table;
    p.ctx_len = a->d_ctx_len;
    p.out = a->d_out;
    p.scale = a->scale;
    p.batch = (int)a->batch;
    p.hq = (int)a->num_q_heads;
    p.hkv = (int)a->num_kv_heads;
    p.d = (int)a->head_dim;
    p.page_tokens = (int)a->page_tokens;
    p.max_pages = (int)a->max_pages_per_seq;
    p.num_pages = (int)a->num_pages;
    p.split_tokens = attn_choose_split(p.batch, p.hq, p.hkv, (int)max_ctx, p.page_tokens, device_sm_count(),
                                       kAttnPlanF16.ctas_per_sm, kAttnPlanF16.max_staged_pages);
    p.max_splits = (int)((max_ctx + p.split_tokens - 1) / p.split_tokens);
    if (p.max_splits < 1) p.max_splits = 1;
    const size_t need = attn_workspace_bytes(p.batch, p.hq, p.d, p.max_splits);
    void* ws = a->d_workspace;
    if (ws) {
        if (a->workspace_bytes < need) { set_error("workspace too small (%zu < %zu)", a->workspace_bytes, need); return VSPEC_B200_ERR_ARG; }
    } else {
        ws = attn_scratch(need);
        if (!ws) { set_error("cannot allocate %zu bytes of attention scratch", need); return VSPEC_B200_ERR_NOMEM; }
    }
    p.part_o = reinterpret_cast<float*>(ws);
    p.part_ml = p.part_o + (size_t)p.batch * p.hq * p.max_splits * p.d;
    return paged_attention_launch(p, a->kv_dtype == VSPEC_B200_KV_F16 ? kKvF16 : kKvF32, (cudaStream_t)stream);
}

extern "C" int vspec_b200_kv_int3_quantize(const float* d_src, const int32_t* d_slots, size_t rows, size_t num_heads,
                                           size_t head_dim, size_t block_size, float percentile, uint8_t* d_codes,
                                           float* d_scales, void* stream) {
    if (!d_src || !d_codes || !d_scales) { set_error("NULL pointer argument"); return VSPEC_B200_ERR_ARG; }
    if (rows == 0 || num_heads == 0) return VSPEC_B200_OK;
    if (block_size != 16 && block_size != 32) { set_error("block_size must be 16 or 32"); return VSPEC_B200_ERR_ARG; }
    if (head_dim == 0 || head_dim > 256 || head_dim % block_size != 0 || head_dim % 8 != 0) {
        set_error("head_dim must be a multiple of block_size and of 8, at most 256"); return VSPEC_B200_ERR_ARG;
    }
    if (rows * num_heads > (size_t)1 << 30) { set_error("too many rows"); return VSPEC_B200_ERR_ARG; }
    return kv_int3_quantize_launch(d_src, d_slots, (int)rows, (int)num_heads, (int)head_dim, (int)block_size, percentile,
                                   d_codes, d_scales, (cudaStream_t)stream);
}

extern "C" int vspec_b200_paged_attention_int3(const VspecB200PagedAttnArgs* a, const float* d_k_scales,
                                               const float* d_v_scales, size_t block_size, void* stream) {
    if (!a) { set_error("args is NULL"); return VSPEC_B200_ERR_ARG; }
    if (!a->d_q || !a->d_k_pages || !a->d_v_pages || !a->d_page_table || !a->d_ctx_len || !a->d_out || !d_k_scales ||
        !d_v_scales) {
        set_error("NULL pointer argument"); return VSPEC_B200_ERR_ARG;
    }
    if (a->kv_dtype != VSPEC_B200_KV_INT3) { set_error("kv_dtype must be VSPEC_B200_KV_INT3"); return VSPEC_B200_ERR_ARG; }
    if (a->batch == 0 || a->num_q_heads == 0 || a->num_kv_heads == 0 || a->page_tokens == 0 ||
        a->max_pages_per_seq == 0 || a->num_pages == 0) {
        set_error("zero dimension"); return VSPEC_B200_ERR_ARG;
    }
    if (a->head_dim != 128) { set_error("int3 pages need head_dim 128"); return VSPEC_B200_ERR_UNSUPPORTED; }
    if (block_size != 16 && block_size != 32) { set_error("block_size must be 16 or 32"); return VSPEC_B200_ERR_ARG; }
    if (a->num_q_heads % a->num_kv_heads != 0 || a->num_q_heads / a->num_kv_heads > 8) {
        set_error("num_q_heads must be a multiple of num_kv_heads, at most 8 per KV head"); return VSPEC_B200_ERR_ARG;
    }
    const uintptr_t al = reinterpret_cast<uintptr_t>(a->d_k_pages) | reinterpret_cast<uintptr_t>(a->d_v_pages) |
                         reinterpret_cast<uintptr_t>(d_k_scales) | reinterpret_cast<uintptr_t>(d_v_scales);
    if (al % 16 != 0) { set_error("int3 page pools must be 16-byte aligned"); return VSPEC_B200_ERR_ARG; }
    if (a->max_ctx > a->max_pages_per_seq * a->page_tokens) {
        set_error("max_ctx %zu exceeds the page table capacity %zu", a->max_ctx, a->max_pages_per_seq * a->page_tokens);
        return VSPEC_B200_ERR_ARG;
    }
    const size_t max_ctx = a->max_ctx ? a->max_ctx : a->max_pages_per_seq * a->page_tokens;
    AttnParams p;
    memset(&p, 0, sizeof(p));
    p.q = a->d_q;
    p.k_pages = a->d_k_pages;
    p.v_pages = a->d_v_pages;
    p.k_scales = d_k_scales;
    p.v_scales = d_v_scales;
    p.kv_block = (int)block_size;
    p.page_table = a->d_page_table;
    p.ctx_len = a->d_ctx_len;
    p.out = a->d_out;
    p.scale = a->scale;
    p.batch = (int)a->batch;
    p.hq = (int)a->num_q_heads;
    p.hkv = (int)a->num_kv_heads;
    p.d = (int)a->head_dim;
    p.page_tokens = (int)a->page_tokens;
    p.max_pages = (int)a->max_pages_per_seq;
    p.num_pages = (int)a->num_pages;
    // the SIMT variant (VSPEC_B200_INT3_ATTN_SIMT=1) is planned like the fp16 kernel
    const char* simt = getenv("VSPEC_B200_INT3_ATTN_SIMT");
    const AttnPlanShape plan = (simt && simt[0] == '1') ? kAttnPlanF16 : attn_plan_int3(p.hq, p.hkv);
    p.split_tokens = attn_choose_split(p.batch, p.hq, p.hkv, (int)max_ctx, p.page_tokens, device_sm_count(),
                                       plan.ctas_per_sm, plan.max_staged_pages);
    p.max_splits = (int)((max_ctx + p.split_tokens - 1) / p.split_tokens);
    if (p.max_splits < 1) p.max_splits = 1;
    const size_t need = attn_workspace_bytes(p.batch, p.hq, p.d, p.max_splits);
    void* ws = a->d_workspace;
    if (ws) {
        if (a->workspace_bytes < need) { set_error("workspace too small (%zu < %zu)", a->workspace_bytes, need); return VSPEC_B200_ERR_ARG; }
    } else {
        ws = attn_scratch(need);
        if (!ws) { set_error("cannot allocate %zu bytes of attention scratch", need); return VSPEC_B200_ERR_NOMEM; }
    }
    p.part_o = reinterpret_cast<float*>(ws);
    p.part_ml = p.part_o + (size_t)p.batch * p.hq * p.max_splits * p.d;
    return paged_attention_launch(p, kKvInt3, (cudaStream_t)stream);
}

extern "C" int vspec_b200_paged_attention_page_fault(int* out_flag) {
    if (!out_flag) { set_error("NULL out_flag"); return VSPEC_B200_ERR_ARG; }
    return attn_read_and_clear_page_fault(out_flag);
}

extern "C" int vspec_b200_paged_gather(const void* kp, const void* vp, const int32_t* table, size_t ctx, size_t pt,
                                       size_t hkv, size_t d, int kv_dtype, void* kout, void* vout, void* stream) {
    if (!kp || !vp || !table || !kout || !vout || pt == 0 || hkv == 0 || d == 0) { set_error("bad gather arguments"); return VSPEC_B200_ERR_ARG; }
    if (ctx == 0) return VSPEC_B200_OK;
    return paged_gather_launch(kp, vp, table, (int)ctx, (int)pt, (int)hkv, (int)d,
                               kv_dtype == VSPEC_B200_KV_F16 ? kKvF16 : kKvF32, kout, vout, (cudaStream_t)stream);
}

extern "C" int vspec_b200_rmsnorm_f32(const float* x, const float* w, float eps, size_t rows, size_t dim, float* y,
                                      void* stream) {
    if (!x || !y || rows == 0 || dim == 0) { set_error("bad rmsnorm arguments"); return VSPEC_B200_ERR_ARG; }
    rmsnorm_rows_kernel<<<(unsigned)rows, 256, 0, (cudaStream_t)stream>>>(x, w, eps, rows, dim, y);
    VB_CHECK_CUDA(cudaGetLastError());
    return VSPEC_B200_OK;
}

extern "C" int vspec_b200_linear_f32(const float* x, const float* w, size_t m, size_t k, size_t n, float* y,
                                     void* stream) {
    if (!x || !w || !y || m == 0 || k == 0 || n == 0) { set_error("bad linear arguments"); return VSPEC_B200_ERR_ARG; }
    const size_t warps = m * n;
    linear_f32_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, (cudaStream_t)stream>>>(x, w, m, k, n, y);
    VB_CHECK_CUDA(cudaGetLastError());
    return VSPEC_B200_OK;
}

extern "C" int vspec_b200_silu_f32(float* d, size_t n, void* stream) {
    if (!d) { set_error("NULL data"); return VSPEC_B200_ERR_ARG; }
    if (n == 0) return VSPEC_B200_OK;
    silu_kernel<<<grid1d(n), 256, 0, (cudaStream_t)stream>>>(d, n);
    VB_CHECK_CUDA(cudaGetLastError());
    return VSPEC_B200_OK;
}

extern "C" int vspec_b200_mul_f32(float* d, const float* o, size_t n, void* stream) {
    if (!d || !o) { set_error("NULL data"); return VSPEC_B200_ERR_ARG; }
    if (n == 0) return VSPEC_B200_OK;
    mul_kernel<<<grid1d(n), 256, 0, (cudaStream_t)stream>>>(d, o, n);
    VB_CHECK_CUDA(cudaGetLastError());
    return VSPEC_B200_OK;
}

// ============================================================================
// Reference host-pointer attention entry points
// ============================================================================
namespace vb200 {

// Per host thread and device: grow-only device buffers and a stream for the
// host-array attention entry points (the reference keeps grow-only static
// buffers too, attention_fused.cu:160-195); allocating and freeing them on
// every call cost ~10 ms per call in synchronising cudaFree.
struct AttnHostState {
    float *q, *k, *v, *out;
    int32_t* meta;   // [0] page table = {0}, [1] context length
    size_t cap_q, cap_kv;
    cudaStream_t st;
};
static thread_local AttnHostState g_attn_host[64];

static bool grow(float** p, size_t* cap, size_t bytes) {
    if (*cap >= bytes) return true;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    if (cudaMalloc(p, bytes) != cudaSuccess) { *p = nullptr; return false; }
    *cap = bytes;
    return true;
}

static AttnHostState* attn_host_state(size_t qb, size_t kvb) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    AttnHostState& h = g_attn_host[dev];
    if (!h.st && cudaStreamCreateWithFlags(&h.st, cudaStreamNonBlocking) != cudaSuccess) { h.st = nullptr; return nullptr; }
    if (!h.meta && cudaMalloc(&h.meta, 2 * sizeof(int32_t)) != cudaSuccess) { h.meta = nullptr; return nullptr; }
    size_t cq = h.cap_q, ckv = h.cap_kv, cq2 = h.cap_q, ckv2 = h.cap_kv;
    if (!grow(&h.q, &cq, qb) || !grow(&h.out, &cq2, qb)) { h.cap_q = 0; return nullptr; }
    if (!grow(&h.k, &ckv, kvb) || !grow(&h.v, &ckv2, kvb)) { h.cap_kv = 0; return nullptr; }
    h.cap_q = cq < cq2 ? cq : cq2;
    h.cap_kv = ckv < ckv2 ? ckv : ckv2;
    return &h;
}

// Contiguous fp32 K/V [T][H][d] already on the device: a single page of T
// tokens; d_meta holds two ints of device scratch for the page table and the
// context length.
static int attention_contiguous_dev(const float* d_q, const float* d_k, const float* d_v, size_t T, size_t H, size_t d,
                                    float* d_out, int32_t* d_meta, cudaStream_t st) {
    const int32_t meta[2] = {0, (int32_t)T};
    cudaError_t e = cudaMemcpyAsync(d_meta, meta, sizeof(meta), cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return cuda_status(e, "attention metadata upload");
    VspecB200PagedAttnArgs a;
    memset(&a, 0, sizeof(a));
    a.d_q = d_q;
    a.d_k_pages = d_k;
    a.d_v_pages = d_v;
    a.d_page_table = d_meta;
    a.d_ctx_len = d_meta + 1;
    a.d_out = d_out;
    a.batch = 1;
    a.num_q_heads = H;
    a.num_kv_heads = H;
    a.head_dim = d;
    a.page_tokens = T;
    a.max_pages_per_seq = 1;
    a.num_pages = 1;
    a.max_ctx = T;
    a.scale = 1.0f / sqrtf((float)d);
    a.kv_dtype = VSPEC_B200_KV_F32;
    const int rc = vspec_b200_paged_attention(&a, st);
    e = cudaStreamSynchronize(st);   // `meta` lives on this stack frame
    if (rc == VSPEC_B200_OK && e != cudaSuccess) return cuda_status(e, "attention");
    return rc;
}

// Host arrays in, host array out (synchronous), like the reference launchers.
static void attention_host(const float* q, const float* k, const float* v, size_t T, size_t H, size_t d, float* out) {
    if (!q || !k || !v || !out || T == 0 || H == 0 || d == 0) return;
    const size_t kvb = T * H * d * sizeof(float), qb = H * d * sizeof(float);
    AttnHostState* h = attn_host_state(qb, kvb);
    if (!h) return;
    if (cudaMemcpyAsync(h->q, q, qb, cudaMemcpyHostToDevice, h->st) != cudaSuccess ||
        cudaMemcpyAsync(h->k, k, kvb, cudaMemcpyHostToDevice, h->st) != cudaSuccess ||
        cudaMemcpyAsync(h->v, v, kvb, cudaMemcpyHostToDevice, h->st) != cudaSuccess)
        return;
    if (attention_contiguous_dev(h->q, h->k, h->v, T, H, d, h->out, h->meta, h->st) == VSPEC_B200_OK) {
        if (cudaMemcpyAsync(out, h->out, qb, cudaMemcpyDeviceToHost, h->st) == cudaSuccess) cudaStreamSynchronize(h->st);
    }
}

}  // namespace vb200

extern "C" void vspec_cuda_attention_fused_single_f32(const float* query, const float* keys, const float* values,
                                                      size_t seq_len, size_t head_dim, float* output) {
    // src/kernel/cuda/attention_fused.cu:144-217
    attention_host(query, keys, values, seq_len, 1, head_dim, output);
}

extern "C" void vspec_cuda_attention_flash_single_f32(const float* query, const float* keys, const float* values,
                                                      size_t seq_len, size_t head_dim, size_t block_tokens,
                                                      float* output) {
    // src/kernel/cuda/attention_fused.cu:219-230: block_tokens is ignored
    (void)block_tokens;
    attention_host(query, keys, values, seq_len, 1, head_dim, output);
}

extern "C" void vspec_cuda_attention_single_f32(const float* query, const float* keys, const float* values,
                                                size_t seq_len, size_t head_dim, float* output) {
    // src/kernel/cuda/cuda_attention_f32.cu:73-127 (same math)
    attention_host(query, keys, values, seq_len, 1, head_dim, output);
}

extern "C" void vspec_cuda_launch_attention_fused(VspecKernelContext* ctx) {
    // src/kernel/cuda/attention_fused.cu:353-445: every head of a contiguous
    // VspecKVCache; int3-compressed caches are dequantized on the device first.
    if (!ctx || !ctx->input || !ctx->weight || !ctx->output) return;
    const VspecKVCache* cache = (const VspecKVCache*)ctx->weight;
    if (cache->current_tokens == 0 || cache->num_heads == 0 || cache->head_dim == 0) return;
    const size_t T = cache->current_tokens, H = cache->num_heads, d = cache->head_dim;
    if (!cache->int3_compressed) {
        attention_host((const float*)ctx->input, cache->key, cache->value, T, H, d, (float*)ctx->output);
        return;
    }
    if (!cache->key_int3 || !cache->value_int3 || !cache->key_scales || !cache->value_scales ||
        cache->packed_head_bytes == 0 || cache->blocks_per_head == 0 || cache->block_size == 0)
        return;
    const size_t rows = T * H;
    const size_t pb = rows * cache->packed_head_bytes, sb = rows * cache->blocks_per_head * sizeof(float);
    const size_t kvb = rows * d * sizeof(float), qb = H * d * sizeof(float);
    uint8_t *dkq = nullptr, *dvq = nullptr;
    float *dks = nullptr, *dvs = nullptr, *dk = nullptr, *dv = nullptr, *dq = nullptr, *dout = nullptr;
    bool ok = cudaMalloc(&dkq, pb) == cudaSuccess && cudaMalloc(&dvq, pb) == cudaSuccess &&
              cudaMalloc(&dks, sb) == cudaSuccess && cudaMalloc(&dvs, sb) == cudaSuccess &&
              cudaMalloc(&dk, kvb) == cudaSuccess && cudaMalloc(&dv, kvb) == cudaSuccess &&
              cudaMalloc(&dq, qb) == cudaSuccess && cudaMalloc(&dout, qb) == cudaSuccess;
    if (ok) {
        cudaMemcpy(dkq, cache->key_int3, pb, cudaMemcpyHostToDevice);
        cudaMemcpy(dvq, cache->value_int3, pb, cudaMemcpyHostToDevice);
        cudaMemcpy(dks, cache->key_scales, sb, cudaMemcpyHostToDevice);
        cudaMemcpy(dvs, cache->value_scales, sb, cudaMemcpyHostToDevice);
        cudaMemcpy(dq, ctx->input, qb, cudaMemcpyHostToDevice);
        dequant_int3_kv_kernel<<<grid1d(rows * d), 256>>>(dkq, dks, dk, rows, d, cache->packed_head_bytes,
                                                          cache->blocks_per_head, cache->block_size);
        dequant_int3_kv_kernel<<<grid1d(rows * d), 256>>>(dvq, dvs, dv, rows, d, cache->packed_head_bytes,
                                                          cache->blocks_per_head, cache->block_size);
        AttnHostState* h = attn_host_state(qb, 0);
        if (h && attention_contiguous_dev(dq, dk, dv, T, H, d, dout, h->meta, nullptr) == VSPEC_B200_OK)
            cudaMemcpy(ctx->output, dout, qb, cudaMemcpyDeviceToHost);
    }
    cudaFree(dkq); cudaFree(dvq); cudaFree(dks); cudaFree(dvs);
    cudaFree(dk); cudaFree(dv); cudaFree(dq); cudaFree(dout);
}

extern "C" void vspec_b200_launch_attention_ref(VspecKernelContext* ctx) {
    // The CPU backend's launch_attention (src/kernel/cpu/cpu_backend.c:29-46 ->
    // src/attention/attention_ref.c:7-88) on the device.  K/V rows come from the cache as
    // vspec_kv_cache_key_at/value_at read them (kv_cache.c:296-371): the fp32 arrays when the
    // cache keeps them, else the int3 codes dequantised on the device.
    if (!ctx || !ctx->input || !ctx->weight || !ctx->output) return;
    const VspecKVCache* cache = (const VspecKVCache*)ctx->weight;
    const size_t T = cache->current_tokens, H = cache->num_heads, d = cache->head_dim;
    if (T == 0 || H == 0 || d == 0) return;
    const size_t ws = vspec_b200_attention_ref_workspace_bytes(T, H, d);
    if (ws == 0) {
        set_error("vspec_b200_launch_attention_ref: unsupported cache sizes");
        return;
    }
    const size_t rows = T * H, kvb = rows * d * sizeof(float), qb = H * d * sizeof(float);
    AttnHostState* h = attn_host_state(qb, kvb);
    void* w = attn_scratch(ws);
    if (!h || !w) return;
    const bool fp32 = cache->key && cache->value;
    const bool int3 = cache->int3_compressed && cache->key_int3 && cache->value_int3 && cache->key_scales &&
                      cache->value_scales && cache->packed_head_bytes && cache->blocks_per_head && cache->block_size;
    if (fp32) {
        if (cudaMemcpyAsync(h->k, cache->key, kvb, cudaMemcpyHostToDevice, h->st) != cudaSuccess ||
            cudaMemcpyAsync(h->v, cache->value, kvb, cudaMemcpyHostToDevice, h->st) != cudaSuccess)
            return;
    } else if (int3) {
        const size_t pb = rows * cache->packed_head_bytes, sb = rows * cache->blocks_per_head * sizeof(float);
        uint8_t *dkq = nullptr, *dvq = nullptr;
        float *dks = nullptr, *dvs = nullptr;
        bool ok = cudaMalloc(&dkq, pb) == cudaSuccess && cudaMalloc(&dvq, pb) == cudaSuccess &&
                  cudaMalloc(&dks, sb) == cudaSuccess && cudaMalloc(&dvs, sb) == cudaSuccess;
        if (ok) {
            ok = cudaMemcpyAsync(dkq, cache->key_int3, pb, cudaMemcpyHostToDevice, h->st) == cudaSuccess &&
                 cudaMemcpyAsync(dvq, cache->value_int3, pb, cudaMemcpyHostToDevice, h->st) == cudaSuccess &&
                 cudaMemcpyAsync(dks, cache->key_scales, sb, cudaMemcpyHostToDevice, h->st) == cudaSuccess &&
                 cudaMemcpyAsync(dvs, cache->value_scales, sb, cudaMemcpyHostToDevice, h->st) == cudaSuccess;
            if (ok) {
                dequant_int3_kv_kernel<<<grid1d(rows * d), 256, 0, h->st>>>(
                    dkq, dks, h->k, rows, d, cache->packed_head_bytes, cache->blocks_per_head, cache->block_size);
                dequant_int3_kv_kernel<<<grid1d(rows * d), 256, 0, h->st>>>(
                    dvq, dvs, h->v, rows, d, cache->packed_head_bytes, cache->blocks_per_head, cache->block_size);
                ok = cudaStreamSynchronize(h->st) == cudaSuccess;
            }
        }
        cudaFree(dkq); cudaFree(dvq); cudaFree(dks); cudaFree(dvs);
        if (!ok) return;
    } else {
        return;
    }
    if (cudaMemcpyAsync(h->q, ctx->input, qb, cudaMemcpyHostToDevice, h->st) != cudaSuccess) return;
    if (vspec_b200_attention_ref_f32(h->q, h->k, h->v, T, H, d, -1, 0, w, ws, h->out, h->st) != VSPEC_B200_OK) return;
    if (cudaMemcpyAsync(ctx->output, h->out, qb, cudaMemcpyDeviceToHost, h->st) == cudaSuccess)
        cudaStreamSynchronize(h->st);
}

// ---- include/vspec/kernel/cuda_ops.h (host pointers, synchronous) ----
extern "C" void vspec_cuda_rmsnorm_f32(const float* input, const float* weight, float eps, size_t rows, size_t dim,
                                       float* output) {
    if (!input || !weight || !output || rows == 0 || dim == 0) return;
    float *dx = nullptr, *dw = nullptr, *dy = nullptr;
    const size_t xb = rows * dim * sizeof(float), wb = dim * sizeof(float);
    if (cudaMalloc(&dx, xb) == cudaSuccess && cudaMalloc(&dw, wb) == cudaSuccess && cudaMalloc(&dy, xb) == cudaSuccess) {
        cudaMemcpy(dx, input, xb, cudaMemcpyHostToDevice);
        cudaMemcpy(dw, weight, wb, cudaMemcpyHostToDevice);
        if (vspec_b200_rmsnorm_f32(dx, dw, eps, rows, dim, dy, nullptr) == VSPEC_B200_OK)
            cudaMemcpy(output, dy, xb, cudaMemcpyDeviceToHost);
    }
    cudaFree(dx); cudaFree(dw); cudaFree(dy);
}

static void linear_host(const float* input, const float* weight, size_t m, size_t k, size_t n, float* output) {
    if (!input || !weight || !output || m == 0 || k == 0 || n == 0) return;
    float *dx = nullptr, *dw = nullptr, *dy = nullptr;
    const size_t xb = m * k * sizeof(float), wb = n * k * sizeof(float), yb = m * n * sizeof(float);
    if (cudaMalloc(&dx, xb) == cudaSuccess && cudaMalloc(&dw, wb) == cudaSuccess && cudaMalloc(&dy, yb) == cudaSuccess) {
        cudaMemcpy(dx, input, xb, cudaMemcpyHostToDevice);
        cudaMemcpy(dw, weight, wb, cudaMemcpyHostToDevice);
        if (vspec_b200_linear_f32(dx, dw, m, k, n, dy, nullptr) == VSPEC_B200_OK)
            cudaMemcpy(output, dy, yb, cudaMemcpyDeviceToHost);
    }
    cudaFree(dx); cudaFree(dw); cudaFree(dy);
}

extern "C" void vspec_cuda_linear_f32(const float* input, const float* weight, size_t m, size_t k, size_t n,
                                      float* output) {
    linear_host(input, weight, m, k, n, output);  // weight [n][k] (cuda_linear_f32.cu:10-34)
}

extern "C" void vspec_cuda_gemm_f32(const float* input, const float* weight, size_t m, size_t k, size_t n,
                                    float* output) {
    linear_host(input, weight, m, k, n, output);  // same contraction (cuda_gemm_f32.cu:139-182)
}

extern "C" void vspec_cuda_silu_f32(float* data, size_t count) {
    if (!data || count == 0) return;
    float* d = nullptr;
    if (cudaMalloc(&d, count * sizeof(float)) == cudaSuccess) {
        cudaMemcpy(d, data, count * sizeof(float), cudaMemcpyHostToDevice);
        if (vspec_b200_silu_f32(d, count, nullptr) == VSPEC_B200_OK)
            cudaMemcpy(data, d, count * sizeof(float), cudaMemcpyDeviceToHost);
    }
    cudaFree(d);
}

extern "C" void vspec_cuda_mul_f32(float* data, const float* other, size_t count) {
    if (!data || !other || count == 0) return;
    float *d = nullptr, *o = nullptr;
    if (cudaMalloc(&d, count * sizeof(float)) == cudaSuccess && cudaMalloc(&o, count * sizeof(float)) == cudaSuccess) {
        cudaMemcpy(d, data, count * sizeof(float), cudaMemcpyHostToDevice);
        cudaMemcpy(o, other, count * sizeof(float), cudaMemcpyHostToDevice);
        if (vspec_b200_mul_f32(d, o, count, nullptr) == VSPEC_B200_OK)
            cudaMemcpy(data, d, count * sizeof(float), cudaMemcpyDeviceToHost);
    }
    cudaFree(d); cudaFree(o);
}

// ---- src/python/cuda_bridge.c f32 helpers ----
extern "C" void vspec_cuda_rmsnorm_f32_bridge(const float* input, const float* weight, float eps, size_t rows,
                                              size_t dim, float* output) {
    vspec_cuda_rmsnorm_f32(input, weight, eps, rows, dim, output);
}
extern "C" void vspec_cuda_linear_f32_bridge(const float* input, const float* weight, size_t m, size_t k, size_t n,
                                             float* output) {
    vspec_cuda_linear_f32(input, weight, m, k, n, output);
}
extern "C" void vspec_cuda_gemm_f32_bridge(const float* input, const float* weight, size_t m, size_t k, size_t n,
                                           float* output) {
    vspec_cuda_gemm_f32(input, weight, m, k, n, output);
}
extern "C" void vspec_cuda_attention_single_f32_bridge(const float* q, const float* k, const float* v, size_t seq_len,
                                                       size_t head_dim, float* out) {
    vspec_cuda_attention_single_f32(q, k, v, seq_len, head_dim, out);
}
extern "C" void vspec_cuda_attention_fused_single_f32_bridge(const float* q, const float* k, const float* v,
                                                             size_t seq_len, size_t head_dim, float* out) {
    vspec_cuda_attention_fused_single_f32(q, k, v, seq_len, head_dim, out);
}
extern "C" void vspec_attention_flash_single_f32_bridge(const float* q, const float* k, const float* v, size_t seq_len,
                                                        size_t head_dim, size_t block_tokens, float* out) {
    vspec_cuda_attention_flash_single_f32(q, k, v, seq_len, head_dim, block_tokens, out);
}
extern "C" void vspec_cuda_silu_f32_bridge(float* data, size_t count) { vspec_cuda_silu_f32(data, count); }
extern "C" void vspec_cuda_mul_f32_bridge(const float* a, const float* b, size_t count, float* output) {
    // cuda_bridge.c:748-756: output = a, then output *= b
    if (!output) return;
    for (size_t i = 0; i < count; ++i) output[i] = a[i];
    vspec_cuda_mul_f32(output, b, count);
}
