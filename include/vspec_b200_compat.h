/*
 * vspec_b200_compat.h -- the reference-named C ABI exported by libvspec_b200.so.
 *
 * libvspec_b200.so is a drop-in for the CUDA side of Vspec-Engine's kernel
 * boundary: the backend registry's CUDA backend (src/kernel/cuda/cuda_backend_stub.c),
 * the device launchers of include/vspec/kernel/cuda_fused.h, the host helpers of
 * include/vspec/kernel/cuda_ops.h and the Python-facing bridge exports of
 * src/python/cuda_bridge.c.  Every symbol below keeps the reference's name,
 * argument meaning, ownership and error behaviour (citations per entry).
 *
 * The structs are layout-identical restatements of the reference's public
 * structs (same member types in the same order), so a VspecKernelContext built
 * by the reference runtime can be passed straight in; tests/ compare
 * sizeof/offsetof against the reference headers.  When the reference headers
 * are included first (VSPEC_KERNEL_CONTEXT_H etc. defined) they are used instead.
 */
#ifndef VSPEC_B200_COMPAT_H
#define VSPEC_B200_COMPAT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- ABI structs (layouts of include/vspec/quant/quant.h:12-26,
 *      include/vspec/kernel/context.h:8-21, include/vspec/kernel/backend.h:6-10,
 *      include/vspec/attention/kv_cache.h:11-30) ---- */
#if !defined(VSPEC_QUANT_QUANT_H)
typedef enum VspecQuantType {
    VSPEC_QUANT_NONE = 0,
    VSPEC_QUANT_INT2 = 2,
    VSPEC_QUANT_INT3 = 3,
    VSPEC_QUANT_INT4 = 4
} VspecQuantType;

typedef struct VspecQuantMeta {
    unsigned int schema_version;
    VspecQuantType type;
    const float* scales;         /* per-output-row scales (scale_count of them) */
    size_t scale_count;
    int special_format;          /* VspecSpecialQuantFormat (an enum, int-sized) */
    const void* special_data;
} VspecQuantMeta;
#endif

#if !defined(VSPEC_KERNEL_CONTEXT_H)
typedef struct VspecExecConfig {
    size_t m;
    size_t n;
    size_t k;
    size_t flags;
} VspecExecConfig;

typedef struct VspecKernelContext {
    void* input;                 /* host pointer (borrowed for the call) */
    void* weight;                /* packed weight, or const VspecKVCache* for attention */
    void* output;                /* host pointer, written before return */
    VspecQuantMeta qmeta;
    VspecExecConfig config;
} VspecKernelContext;
#endif

#if !defined(VSPEC_KERNEL_BACKEND_H)
typedef struct VspecBackend {
    const char* name;
    void (*launch_linear)(VspecKernelContext* ctx);
    void (*launch_attention)(VspecKernelContext* ctx);
} VspecBackend;
#endif

#if !defined(VSPEC_ATTENTION_KV_CACHE_H)
typedef struct VspecKVCache {
    float* key;                  /* [max_tokens][num_heads][head_dim] */
    float* value;
    size_t max_tokens;
    size_t num_heads;
    size_t head_dim;
    size_t current_tokens;
    int int3_compressed;
    uint8_t* key_int3;           /* [tokens][heads][packed_head_bytes] */
    uint8_t* value_int3;
    float* key_scales;           /* [tokens][heads][blocks_per_head] */
    float* value_scales;
    size_t block_size;
    size_t blocks_per_head;
    size_t packed_head_bytes;
    float* scratch_key_head;
    float* scratch_value_head;
    int owns_int3_buffers;
} VspecKVCache;
#endif

/* Host paged KV cache (include/vspec/attention/kv_paged_cache.h:7-49), read by
 * vspec_b200_kv_paged_sync / _session_view in vspec_b200.h. */
#if !defined(VSPEC_ATTENTION_KV_PAGED_CACHE_H)
#define VSPEC_KV_PAGED_MAX_SESSIONS 128U
#define VSPEC_KV_PAGED_MAX_PAGES 4096U
#define VSPEC_KV_PAGED_MAX_PAGES_PER_SESSION 1024U

typedef struct VspecKVPagedStats {
    uint64_t page_alloc_count;
    uint64_t page_reuse_count;
    uint64_t evict_session_count;
    uint64_t append_token_count;
    size_t free_pages;
    size_t active_sessions;
} VspecKVPagedStats;

typedef struct VspecKVPagedCache {
    float* key_pages;            /* [max_pages][page_tokens][num_heads][head_dim] */
    float* value_pages;
    size_t page_tokens;
    size_t max_pages;
    size_t num_heads;
    size_t head_dim;
    VspecKVPagedStats stats;
    struct {
        uint8_t allocated;
        uint16_t owner_slot;
        uint16_t used_tokens;
        uint16_t ref_count;      /* > 1: a prefix page shared by several sessions */
        uint64_t last_touch_step;
    } page_meta[VSPEC_KV_PAGED_MAX_PAGES];
    struct {
        uint8_t active;
        uint64_t session_id;
        uint64_t last_touch_step;
        size_t total_tokens;
        size_t page_count;
        uint16_t pages[VSPEC_KV_PAGED_MAX_PAGES_PER_SESSION];   /* in token order */
    } sessions[VSPEC_KV_PAGED_MAX_SESSIONS];
    uint64_t clock_step;
} VspecKVPagedCache;
#endif

/* ---- CUDA backend (src/kernel/cuda/cuda_backend_stub.c:25-39,
 *      src/kernel/cuda/cuda_linear_int4.cu:72-114) ---- */
int vspec_cuda_backend_available(void);
VspecBackend vspec_make_cuda_backend(void);           /* name "cuda-b200" */
int vspec_cuda_runtime_available(void);
/* launch_linear: INT4 with the CPU backend's semantics (per-row scales,
 * mean-code zero-points, src/kernel/cpu/cpu_backend.c:9-27 ->
 * src/quant/int4.c:47-67); INT3 through the int3-storage path; others no-op. */
void vspec_cuda_launch_linear_impl(VspecKernelContext* ctx);
/* launch_attention: ctx->weight is a const VspecKVCache*, ctx->input q[H][d];
 * plain softmax attention per head (src/kernel/cuda/attention_fused.cu:353-445). */
void vspec_cuda_launch_attention_impl(VspecKernelContext* ctx);

/* ---- The CPU backend's semantics on the device (src/kernel/cpu/cpu_backend.c:9-48) ----
 * name "cpu-semantics-b200": launch_linear = vspec_cuda_launch_linear_impl (the CPU
 * backend's INT4 semantics), launch_attention = vspec_b200_launch_attention_ref:
 * vspec_attention_ref_single_query (src/attention/attention_ref.c:7-88) on a host
 * VspecKVCache, the 3-bit runtime module decided from the environment per call. */
VspecBackend vspec_b200_make_cpu_semantics_backend(void);
void vspec_b200_launch_attention_ref(VspecKernelContext* ctx);

/* ---- include/vspec/kernel/cuda_fused.h:10-122 ---- */
int vspec_cuda_fused_available(void);
/* Host-pointer context launchers (H2D, kernel, D2H, synchronous). */
void vspec_cuda_launch_fused_linear_int4(VspecKernelContext* ctx);          /* fused_linear_int4.cu:545-638, zp = NULL */
void vspec_cuda_launch_fused_linear_int3(VspecKernelContext* ctx);          /* fused_linear_int3.cu:168-249 */
void vspec_cuda_launch_fused_linear_int2(VspecKernelContext* ctx);          /* fused_linear_int2.cu:153-212 */
void vspec_cuda_launch_fused_linear_int3_storage(VspecKernelContext* ctx);  /* fused_linear_int4.cu:640-745 */
void vspec_cuda_launch_attention_fused(VspecKernelContext* ctx);            /* attention_fused.cu:353-445 */
/* Single-head attention on host arrays (attention_fused.cu:144-230). */
void vspec_cuda_attention_fused_single_f32(const float* query, const float* keys, const float* values,
                                           size_t seq_len, size_t head_dim, float* output);
void vspec_cuda_attention_flash_single_f32(const float* query, const float* keys, const float* values,
                                           size_t seq_len, size_t head_dim, size_t block_tokens, float* output);
/* Device-pointer launchers: asynchronous, default stream, invalid input is a no-op. */
void vspec_cuda_fused_linear_int4_device(const float* d_a, const unsigned char* d_b_packed, const float* d_scales,
                                         const float* d_zero_points, float* d_c, size_t m, size_t n, size_t k,
                                         size_t n_blocks);                  /* fused_linear_int4.cu:477-505 */
void vspec_cuda_dequant_int4_to_f32_device(const unsigned char* d_b_packed, const float* d_scales,
                                           const float* d_zero_points, float* d_w_f32, size_t n, size_t k,
                                           size_t n_blocks);                /* fused_linear_int4.cu:507-526 */
void vspec_cuda_fused_linear_int3_device(const float* d_a, const unsigned char* d_b_packed, const float* d_scales,
                                         float* d_c, size_t m, size_t n, size_t k,
                                         int stochastic_rounding);          /* fused_linear_int3.cu:149-166 */
void vspec_cuda_fused_linear_int2_device(const float* d_a, const unsigned char* d_b_packed, const float* d_scales,
                                         float* d_c, size_t m, size_t n, size_t k); /* fused_linear_int2.cu:78-95 */
void vspec_cuda_dequant_int2_to_f32_device(const unsigned char* d_b_packed, const float* d_scales, float* d_w_f32,
                                           size_t n, size_t k);             /* fused_linear_int2.cu:137-151 */
void vspec_cuda_expand_int3_to_int4_device(const unsigned char* d_b_int3, unsigned char* d_b_int4, size_t n,
                                           size_t k);                       /* fused_linear_int4.cu:528-543 */
void vspec_cuda_fused_linear_hybrid_device(const float* d_a, const unsigned char* d_b_int2_packed,
                                           const float* d_s_int2, const unsigned char* d_b_int4_packed,
                                           const float* d_s_int4, const float* d_zp_int4, float* d_c,
                                           const uint32_t* d_hot_indices, size_t hot_count, size_t m, size_t n,
                                           size_t k, size_t n_blocks_int4); /* fused_linear_hybrid.cu:70-113 */
void vspec_cuda_refine_hot_int4_device(const float* d_a, const unsigned char* d_b_int4_packed,
                                       const float* d_s_int4, const float* d_zp_int4, float* d_c,
                                       const uint32_t* d_hot_indices, size_t hot_count, size_t m, size_t n,
                                       size_t k, size_t n_blocks_int4);     /* fused_linear_hybrid.cu:115-153 */

/* ---- include/vspec/kernel/cuda_ops.h:10-15 (host pointers, synchronous) ---- */
void vspec_cuda_rmsnorm_f32(const float* input, const float* weight, float eps, size_t rows, size_t dim, float* output);
void vspec_cuda_linear_f32(const float* input, const float* weight, size_t m, size_t k, size_t n, float* output);
void vspec_cuda_gemm_f32(const float* input, const float* weight, size_t m, size_t k, size_t n, float* output);
void vspec_cuda_attention_single_f32(const float* query, const float* keys, const float* values, size_t seq_len,
                                     size_t head_dim, float* output);
void vspec_cuda_silu_f32(float* data, size_t count);
void vspec_cuda_mul_f32(float* data, const float* other, size_t count);

/* ---- src/python/cuda_bridge.c exports (host pointers; return 1 = ok, 0 = fail).
 * Weight state is per host thread, as in the reference (__thread registry). ---- */
int vspec_cuda_gemm_dispatch_bridge(const float* input, const float* weight_f32, const unsigned char* packed_weight,
                                    const float* scales, const float* zero_points, size_t m, size_t k, size_t n,
                                    size_t n_blocks, int bits, int* inout_handle, float* output,
                                    int* out_path);                         /* cuda_bridge.c:67-143 */
int vspec_cuda_fused_linear_int4_register_weight_bridge(const unsigned char* packed_weight, const float* scales,
                                                        const float* zero_points, size_t k, size_t n,
                                                        size_t n_blocks);   /* cuda_bridge.c:391-500 */
int vspec_cuda_fused_linear_int4_cached_bridge(const float* input, size_t m, size_t k, int weight_handle,
                                               size_t expected_n, float* output); /* cuda_bridge.c:502-619 */
int vspec_cuda_fused_linear_int4_cached_many_bridge(const float* input, size_t m, size_t k, const int* weight_handles,
                                                    const size_t* output_dims, size_t handle_count,
                                                    float* output);         /* cuda_bridge.c:621-654 */
int vspec_cuda_int4_cached_stats_bridge(uint64_t* out_dispatch_calls, uint64_t* out_dispatch_hits,
                                        uint64_t* out_dispatch_misses, uint64_t* out_register_calls,
                                        uint64_t* out_register_reuse,
                                        uint64_t* out_register_evictions);  /* cuda_bridge.c:656-675 */
int vspec_cuda_fused_linear_int4_bridge(const float* input, const unsigned char* packed_weight, const float* scales,
                                        const float* zero_points, size_t m, size_t k, size_t n, size_t n_blocks,
                                        float* output);                     /* cuda_bridge.c:812-1037 */
int vspec_cuda_fused_linear_int3_bridge(const float* input, const unsigned char* packed_weight, const float* scales,
                                        size_t m, size_t k, size_t n, float* output); /* cuda_bridge.c:1039-1158 */
int vspec_cuda_fused_linear_hybrid_profile_bridge(const float* input, const unsigned char* packed_weight_int2,
                                                  const float* scales_int2, const unsigned char* packed_weight_int4,
                                                  const float* scales_int4, const float* zero_points_int4, size_t m,
                                                  size_t k, size_t n, const uint32_t* hot_indices, size_t hot_count,
                                                  size_t n_blocks_int4, float* output, float* out_h2d_ms,
                                                  float* out_kernel_ms, float* out_d2h_ms,
                                                  float* out_total_gpu_ms); /* cuda_bridge.c:1216-1683 */
int vspec_cuda_fused_linear_hybrid_bridge(const float* input, const unsigned char* packed_weight_int2,
                                          const float* scales_int2, const unsigned char* packed_weight_int4,
                                          const float* scales_int4, const float* zero_points_int4, size_t m,
                                          size_t k, size_t n, const uint32_t* hot_indices, size_t hot_count,
                                          size_t n_blocks_int4, float* output); /* cuda_bridge.c:1180-1214 */
void vspec_cuda_rmsnorm_f32_bridge(const float* input, const float* weight, float eps, size_t rows, size_t dim,
                                   float* output);                          /* cuda_bridge.c:677-686 */
void vspec_cuda_linear_f32_bridge(const float* input, const float* weight, size_t m, size_t k, size_t n,
                                  float* output);                           /* cuda_bridge.c:688-697 */
void vspec_cuda_gemm_f32_bridge(const float* input, const float* weight, size_t m, size_t k, size_t n,
                                float* output);                             /* cuda_bridge.c:699-708 */
void vspec_cuda_attention_single_f32_bridge(const float* query, const float* keys, const float* values, size_t seq_len,
                                            size_t head_dim, float* output); /* cuda_bridge.c:710-719 */
void vspec_cuda_attention_fused_single_f32_bridge(const float* query, const float* keys, const float* values,
                                                  size_t seq_len, size_t head_dim,
                                                  float* output);           /* cuda_bridge.c:721-730 */
void vspec_attention_flash_single_f32_bridge(const float* query, const float* keys, const float* values,
                                             size_t seq_len, size_t head_dim, size_t block_tokens,
                                             float* output);                /* cuda_bridge.c:732-742 */
void vspec_cuda_silu_f32_bridge(float* data, size_t count);                 /* cuda_bridge.c:744-746 */
void vspec_cuda_mul_f32_bridge(const float* a, const float* b, size_t count, float* output); /* cuda_bridge.c:748-756 */
int vspec_cuda_mem_info_bridge(size_t* free_bytes, size_t* total_bytes);    /* cuda_bridge.c:758-771 */
int vspec_cuda_device_capability_bridge(int* out_major, int* out_minor,
                                        int* out_multiprocessors);          /* cuda_bridge.c:773-794 */
int vspec_cuda_int4_tensorcore_available_bridge(void);                      /* cuda_bridge.c:796-810 */

#ifdef __cplusplus
}
#endif

#endif /* VSPEC_B200_COMPAT_H */
