/*
 * vspec_b200.h -- native C ABI of libvspec_b200.so, the B200 (sm_100a)
 * implementation of Vspec-Engine's low-bit decode hot path.
 *
 * All pointers named d_* are device pointers; `stream` is a cudaStream_t
 * passed as void* (NULL = legacy default stream).  Every function returns a
 * VSPEC_B200_* status; on failure vspec_b200_last_error() describes why.
 * Launches are asynchronous unless stated otherwise.
 *
 * The reference-named entry points (include/vspec/kernel/cuda_fused.h,
 * src/python/cuda_bridge.c, include/vspec/kernel/backend.h) are declared in
 * vspec_b200_compat.h and are thin wrappers over these functions.
 */
#ifndef VSPEC_B200_H
#define VSPEC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status */
#define VSPEC_B200_OK 0
#define VSPEC_B200_ERR_ARG 1          /* invalid argument (checked on the host before launch) */
#define VSPEC_B200_ERR_CUDA 2         /* a CUDA runtime call failed */
#define VSPEC_B200_ERR_UNSUPPORTED 3  /* valid but not supported by this build */
#define VSPEC_B200_ERR_NOMEM 4        /* device or host allocation failed */
#define VSPEC_B200_ERR_TIMEOUT 5      /* a bounded device wait gave up */

/* Thread-local description of the last failure (never NULL). */
const char* vspec_b200_last_error(void);
/* Library version string. */
const char* vspec_b200_version(void);

/* ------------------------------------------------------ low-bit linear */
/* Flags of VspecB200LinearArgs.flags */
#define VSPEC_B200_F_SZ_F16 0x1     /* scales / zero-points are fp16 (default fp32) */
#define VSPEC_B200_F_UNSIGNED 0x2   /* codes are unsigned offsets u - 2^(bits-1) instead of two's complement */
#define VSPEC_B200_F_RESIDUAL 0x4   /* y = residual + W.x  (residual may alias y) */
#define VSPEC_B200_F_RMSNORM 0x8    /* x := x / sqrt(mean(x^2) + eps) * norm_weight before the product */
#define VSPEC_B200_F_SWIGLU 0x10    /* rows [0,n/2) are gate, [n/2,n) up; y[m][n/2] = silu(gate) * up */

/*
 * Group-wise dequant-matmul (GEMV for m <= 8, GEMM beyond):
 *   y[i][j] = sum_t x[i][t] * (code(j,t) - zp[j][g(t)]) * s[j][g(t)]
 *
 * Layouts are the reference's: w is [n][ceil(k*bits/8)] bytes, each row the
 * LSB-first bitstream of src/quant/pack.c:30-74 (bits 4: two codes per byte,
 * low nibble first, src/quant/int4.c:25-45); s / zp are row-major
 * [n][n_groups]; g(t) = min(G-1, t*G/k) (src/kernel/cuda/fused_linear_int4.cu:391-396).
 * zero_points == NULL uses zero_point_const for every group.
 *
 * Generalizes vspec_cuda_fused_linear_int4_device / _int3_device /
 * _int2_device (include/vspec/kernel/cuda_fused.h:34-75) with an explicit
 * stream, group-wise scales for every bit width, fp16 scale storage and the
 * fused RMSNorm-input / residual / SwiGLU epilogues of the Qwen decode step
 * (Vspec-chat/python/runtime_inference.py:1245-1499).
 */
typedef struct VspecB200LinearArgs {
    const float* d_x;            /* [m][k] fp32 */
    const uint8_t* d_w;          /* [n][ceil(k*bits/8)] */
    const void* d_scales;        /* [n][n_groups] fp32, or fp16 with VSPEC_B200_F_SZ_F16 */
    const void* d_zero_points;   /* same layout/dtype, or NULL */
    float zero_point_const;
    float* d_y;                  /* [m][n], or [m][n/2] with VSPEC_B200_F_SWIGLU */
    const float* d_residual;     /* [m][n] with VSPEC_B200_F_RESIDUAL */
    const float* d_norm_weight;  /* [k] with VSPEC_B200_F_RMSNORM */
    float norm_eps;
    size_t m, n, k, n_groups;
    int bits;                    /* 2, 3 or 4 */
    int flags;
    void* d_workspace;           /* NULL = library-managed device scratch; else
                                    >= vspec_b200_lowbit_linear_workspace_bytes()
                                    bytes, zero-filled before first use (every
                                    launch leaves it zero-filled again) */
    size_t workspace_bytes;
} VspecB200LinearArgs;

/* Device scratch of the split-K merge: a fixed 64 KiB region of per-tile
 * counters (zero between launches) followed by fp32 partials.  Calls sharing
 * one workspace must be stream-ordered; any sequence of shapes may share it.
 * The library-managed workspace (d_workspace == NULL) is allocated per device
 * and host thread on first use and grown when a larger shape arrives, so the
 * first call of each shape must precede any stream capture. */
size_t vspec_b200_lowbit_linear_workspace_bytes(size_t m, size_t n, size_t k, int flags);
int vspec_b200_lowbit_linear(const VspecB200LinearArgs* args, void* stream);

/* Reads and clears the flag a TMA-fed GEMV (ring or tcgen05 kernel) raises
 * when one of its bounded waits gave up (1 = seen since the last call; the
 * launch then left y incomplete and returned its resources). */
int vspec_b200_gemv_timeout_flag(int* out_flag);

/* Same contraction with scratch the library never allocates: a static 16 MiB
 * device array per device (no counterpart in the reference).  For callers that
 * cannot allow a device allocation inside the call: a runtime whose arena/pool
 * allocator owns the device memory, or a decode loop that must not stall on
 * the synchronising cudaFree/cudaMalloc of a growing library workspace.
 * args->d_workspace must be NULL and workspace_bytes 0; shapes whose
 * vspec_b200_lowbit_linear_workspace_bytes() exceeds 16 MiB return
 * VSPEC_B200_ERR_ARG.  The first call on a device (that device current) looks
 * up the array with cudaGetSymbolAddress; under CUDA's default lazy module
 * loading that lookup also reserves the 16 MiB on the device (at process start
 * with CUDA_MODULE_LOADING=EAGER).  Make that first call before the caller's
 * arena/pool allocator reserves the device's memory and before any stream
 * capture.  Every call clears the array's 64 KiB counter region with a
 * cudaMemsetAsync on `stream` before its launch, so a launch whose bounded wait
 * gave up (vspec_b200_gemv_timeout_flag) cannot poison later calls.  One array
 * per device: overlapping calls on a device (other streams, threads, concurrent
 * graph replays) race; order them on one stream. */
int vspec_b200_lowbit_linear_static(const VspecB200LinearArgs* args, void* stream);

/* ANF hybrid linear (src/kernel/cuda/fused_linear_hybrid.cu:70-113, the
 * device half of vspec_cuda_fused_linear_hybrid_bridge): y[m][n] = the int2
 * draft of every column, (q - 1.5) * s2[j] with unsigned 2-bit codes
 * (fused_linear_int2.cu:8-12), then each listed column j < n of d_hot
 * recomputed from int4: sum_t x[t] * ((q4 - 8) * s4[j][b] + zp4[j][b]),
 * b = min(t / ceil(k / n_blocks_int4), n_blocks_int4 - 1).  d_w4/d_s4/d_hot
 * may be NULL (or hot_count 0): draft only.  d_zp4 may be NULL (zero).
 * Both launches go on `stream`. */
int vspec_b200_anf_hybrid_linear(const float* d_x, const unsigned char* d_w2, const float* d_s2,
                                 const unsigned char* d_w4, const float* d_s4, const float* d_zp4, float* d_y,
                                 const uint32_t* d_hot, size_t hot_count, size_t m, size_t n, size_t k,
                                 size_t n_blocks_int4, void* stream);

/* The refine half alone (fused_linear_hybrid.cu:30-68,115-153): overwrites
 * y[r][j] for each listed column j < n with its int4 recompute. */
int vspec_b200_refine_hot_int4(const float* d_x, const unsigned char* d_w4, const float* d_s4, const float* d_zp4,
                               float* d_y, const uint32_t* d_hot, size_t hot_count, size_t m, size_t n, size_t k,
                               size_t n_blocks, void* stream);

/* Q4_K dequant-matmul (src/quant/formats/q4_k.c:41-134,
 * include/vspec/quant/formats/q4_k.h:7-16; the device counterpart of
 * vspec_q4k_matmul_ref_f32): y[m][n] = x[m][k] W^T for W stored as n rows of
 * k/256 VspecQ4KBlock (144 bytes: fp16 d, fp16 dmin, 12 bytes of sixteen 6-bit
 * sub-scales / sub-mins, 128 bytes of 4-bit codes), element =
 * d*(sc/63)*q - dmin*(mn/63).  k % 256 == 0; x and the blocks 16-byte aligned. */
int vspec_b200_q4k_linear(const float* d_x, const void* d_blocks, float* d_y, size_t m, size_t n, size_t k,
                          void* stream);

/* Same contraction through the any-shape path only (testing / odd shapes). */
int vspec_b200_lowbit_linear_generic(const VspecB200LinearArgs* args, void* stream);

/* Same contraction through an explicit kernel family:
 *   VSPEC_B200_PATH_AUTO    the dispatcher's choice (row-sliced where it is
 *                           faster, else ring, else warp-MMA, else generic)
 *   VSPEC_B200_PATH_GENERIC any shape, one warp per output row
 *   VSPEC_B200_PATH_WARPMMA persistent split-K warp-MMA kernel, weights
 *                           streamed through registers (m <= 8)
 *   VSPEC_B200_PATH_TCGEN05 TMA + TMEM + tcgen05.mma kernel (m <= 4)
 *   VSPEC_B200_PATH_RING    TMA shared-memory ring + warp-MMA decode, split-K
 *                           across CTAs (m <= 8)
 *   VSPEC_B200_PATH_ROWS    TMA ring + warp-MMA decode, each CTA a contiguous
 *                           row range over all of k, no workspace (m <= 8,
 *                           k % 1024 == 0, int4 k % 2048 == 0)
 * A fast path that does not support the shape returns VSPEC_B200_ERR_UNSUPPORTED. */
#define VSPEC_B200_PATH_AUTO 0
#define VSPEC_B200_PATH_GENERIC 1
#define VSPEC_B200_PATH_WARPMMA 2
#define VSPEC_B200_PATH_TCGEN05 3
#define VSPEC_B200_PATH_RING 4
#define VSPEC_B200_PATH_ROWS 5
int vspec_b200_lowbit_linear_path(const VspecB200LinearArgs* args, void* stream, int path);

/* Decode every code of a packed [n][k] matrix into int8 [n][k] (bit-exact
 * parity hook for vspec_quant_get_signed, src/quant/pack.c:53-74).
 * use_fast_decoder = 1 runs the register decoder of the GEMV fast path
 * (k % 32 == 0), 0 the generic per-field decoder. */
int vspec_b200_unpack_codes(const uint8_t* d_w, size_t n, size_t k, int bits, int unsigned_codes,
                            int8_t* d_codes, int use_fast_decoder, void* stream);

/* Dequantize a packed [n][k] matrix to fp32: (code - zp) * s, s == NULL -> 1,
 * zp == NULL -> zp_const (src/kernel/cuda/fused_linear_int4.cu:418-470,
 * src/kernel/cuda/fused_linear_int2.cu:97-135). */
int vspec_b200_dequant_f32(const uint8_t* d_w, const float* d_s, const float* d_zp, float zp_const, int bits,
                           int unsigned_codes, size_t n, size_t k, size_t n_groups, float* d_out, void* stream);

/* Clamp each row of an fp32 [rows][cols] matrix to +-alpha*std(row)
 * (src/kernel/cuda/fused_linear_int3.cu:20-53). */
int vspec_b200_clamp_rows_std(const float* d_in, float* d_out, size_t rows, size_t cols, float alpha, void* stream);

/* The reference int3 kernel's arithmetic: per-row scale, 32-wide block-abs
 * normalization, optional hash-seeded stochastic rounding to 1/16 steps
 * (src/kernel/cuda/fused_linear_int3.cu:68-147). */
int vspec_b200_int3_blocknorm_linear(const float* d_a, const uint8_t* d_w, const float* d_s, float* d_c, size_t m,
                                     size_t n, size_t k, int stochastic, void* stream);

/* Per-row mean code zero-points (src/quant/int4.c:69-89, src/quant/int3.c:28-48). */
int vspec_b200_mean_code_zero_points(const uint8_t* d_w, size_t n, size_t k, int bits, float* d_zp, void* stream);

/* ------------------------------------------------- paged decode attention */
#define VSPEC_B200_KV_F32 0
#define VSPEC_B200_KV_F16 1

/*
 * GQA decode attention of one query token per sequence over a paged K/V
 * cache (the fused paged attention the reference runs head by head on
 * contiguous host copies, src/kernel/cuda/attention_fused.cu:353-445,
 * Vspec-chat/python/runtime_inference.py:1413-1433):
 *   out[b][h] = softmax(q[b][h] . K_b^T * scale) V_b,  kv head = h / (Hq/Hkv)
 * Pages are [num_pages][page_tokens][num_kv_heads][head_dim] -- the layout of
 * VspecKVPagedCache pages (include/vspec/attention/kv_paged_cache.h:21-27) --
 * in fp16 or fp32; the page table row of a sequence is its session pages[]
 * widened to int32.  Token t is slot t % page_tokens of page
 * table[t / page_tokens] (all pages but the last are full).  ctx_len 0
 * yields zeros.  Page ids outside [0, num_pages) are redirected to page 0 and
 * reported by vspec_b200_paged_attention_page_fault().
 */
typedef struct VspecB200PagedAttnArgs {
    const float* d_q;             /* [batch][num_q_heads][head_dim] */
    const void* d_k_pages;
    const void* d_v_pages;
    const int32_t* d_page_table;  /* [batch][max_pages_per_seq] */
    const int32_t* d_ctx_len;     /* [batch] */
    float* d_out;                 /* [batch][num_q_heads][head_dim] */
    size_t batch, num_q_heads, num_kv_heads, head_dim;
    size_t page_tokens, max_pages_per_seq, num_pages;
    size_t max_ctx;               /* host-side upper bound of ctx_len (sizes the split grid) */
    float scale;
    int kv_dtype;                 /* VSPEC_B200_KV_F16 or VSPEC_B200_KV_F32 */
    void* d_workspace;            /* NULL = library-managed device scratch */
    size_t workspace_bytes;
} VspecB200PagedAttnArgs;

/* Scratch bytes the split-context merge needs for these sizes. */
size_t vspec_b200_paged_attention_workspace_bytes(size_t batch, size_t num_q_heads, size_t num_kv_heads,
                                                  size_t head_dim, size_t max_ctx);
int vspec_b200_paged_attention(const VspecB200PagedAttnArgs* args, void* stream);

/* The CPU backend's attention with its semantics (replaces the device side of
 * vspec_attention_ref_single_query, src/attention/attention_ref.c:7-88, reached
 * through the CPU backend's launch_attention, src/kernel/cpu/cpu_backend.c:29-46):
 * contiguous fp32 q [heads][head_dim] and K/V [tokens][heads][head_dim] (no GQA),
 * q and each k row clamped to +-max(1e-6, 4.5 * population std), softmax with a
 * double denominator, output summed in double.  three_bit_module: 1 = the 3-bit
 * runtime module's arithmetic (src/runtime/three_bit_runtime_modules.c:138-361:
 * noise reducer, block-normalised Kahan dot, qk-scale and logit clips, Kahan
 * output), 0 = without it, -1 = decided from VSPEC_FUSED_BITS /
 * VSPEC_3BIT_RUNTIME_MODULE at call time as the reference does.  block_size: the
 * module's dot block, 32 or 64; 0 = VSPEC_3BIT_BLOCK_SIZE (default 64).
 * head_dim <= 1024; d_workspace 256-byte aligned, at least
 * vspec_b200_attention_ref_workspace_bytes() (0 for unsupported sizes). */
size_t vspec_b200_attention_ref_workspace_bytes(size_t tokens, size_t heads, size_t head_dim);
int vspec_b200_attention_ref_f32(const float* d_q, const float* d_keys, const float* d_values, size_t tokens,
                                 size_t heads, size_t head_dim, int three_bit_module, size_t block_size,
                                 void* d_workspace, size_t workspace_bytes, float* d_out, void* stream);

/* int3 KV pages (VspecKVCache int3 compression, src/attention/kv_cache.c:64-126
 * and 160-226, dequantised in attention as src/kernel/cuda/attention_fused.cu:23-45
 * and 232-351 do, moved onto the paged layout):
 *   codes  [num_pages][page_tokens][num_kv_heads][head_dim*3/8] bytes, each
 *          head row the LSB-first 3-bit bitstream of src/quant/pack.c:30-51;
 *   scales [num_pages][page_tokens][num_kv_heads][head_dim/block_size] fp32.
 * vspec_b200_kv_int3_quantize compresses `rows` fp32 rows [num_heads][head_dim]
 * (one token each) into pool rows d_slots[r] (page * page_tokens + slot; r
 * when d_slots is NULL), bit for bit as vspec_kv_cache_append with int3
 * compression on: per block of block_size (16 or 32) dims the percentile
 * element of the sorted |x| (the reference uses 99.5), scale = that / 4,
 * codes lrintf(x / scale) clipped to [-4, 3].  head_dim % block_size == 0,
 * head_dim <= 256, head_dim % 8 == 0. */
#define VSPEC_B200_KV_INT3 2
int vspec_b200_kv_int3_quantize(const float* d_src, const int32_t* d_slots, size_t rows, size_t num_heads,
                                size_t head_dim, size_t block_size, float percentile, uint8_t* d_codes,
                                float* d_scales, void* stream);
/* Paged GQA decode attention over int3 pages: args->d_k_pages / d_v_pages are
 * the code pools, args->kv_dtype must be VSPEC_B200_KV_INT3, head_dim 128,
 * at most 8 query heads per KV head; pools and scale pools 16-byte aligned.
 * Same contract as vspec_b200_paged_attention otherwise. */
int vspec_b200_paged_attention_int3(const VspecB200PagedAttnArgs* args, const float* d_k_scales,
                                    const float* d_v_scales, size_t block_size, void* stream);
/* Reads and clears the out-of-range page id flag (1 = seen since last call). */
int vspec_b200_paged_attention_page_fault(int* out_flag);

/* ---- device view of the reference's host paged KV cache ----
 * `cache` is a VspecKVPagedCache* (include/vspec/attention/kv_paged_cache.h:7-49,
 * layout in vspec_b200_compat.h) filled by the reference's vspec_kv_paged_append
 * / reuse_prefix (src/attention/kv_paged_cache.c:185-310); the library only
 * reads it.  Device pools are [pages][page_tokens][num_heads][head_dim] in fp32
 * (VSPEC_B200_KV_F32) or fp16 (VSPEC_B200_KV_F16, rounded to nearest even), at
 * least cache->max_pages pages, plus any spare pages the session views use.
 *
 * vspec_b200_kv_paged_sync: copies every allocated page whose last write is
 * after clock step `since_step` (0: every allocated page) to the same page
 * index of the device pools; *out_step (optional) = the cache's clock, the
 * since_step of the next incremental call.  Returns after the copies landed. */
int vspec_b200_kv_paged_sync(const void* cache, int kv_dtype, void* d_k_pages, void* d_v_pages, uint64_t since_step,
                             uint64_t* out_step, void* stream);
/* vspec_b200_kv_paged_session_view: the session's page-table row
 * (d_page_table_row[0 .. max_pages_per_seq), unused entries 0) and context
 * length (*d_ctx_len = its token count) for vspec_b200_paged_attention, with
 * vspec_kv_paged_get_token_ptr's token order (kv_paged_cache.c:312-356).  While
 * every page of the session but the last is full the row is its pages[]
 * widened to int32.  A session that shares a partly filled prefix page and was
 * appended past it has a short page in the middle: its tokens from that page
 * on are gathered into the device pool pages spare_first .. spare_first +
 * spare_count - 1 (which must lie at or beyond cache->max_pages; the pools
 * must have room for them) and the row points there.  *out_ctx and
 * *out_spare_used (spare pages written) are optional.  Returns after the copies
 * landed.  An inactive session, a row too short for its tokens, or too few
 * spare pages return VSPEC_B200_ERR_ARG. */
int vspec_b200_kv_paged_session_view(const void* cache, uint64_t session_id, int kv_dtype, void* d_k_pages,
                                     void* d_v_pages, size_t spare_first, size_t spare_count,
                                     int32_t* d_page_table_row, size_t max_pages_per_seq, int32_t* d_ctx_len,
                                     size_t* out_ctx, size_t* out_spare_used, void* stream);

/* Bit-exact gather of one sequence's K and V rows in token order into
 * [ctx][num_kv_heads][head_dim] (parity hook for vspec_kv_paged_get_token_ptr,
 * src/attention/kv_paged_cache.c:312-356). */
int vspec_b200_paged_gather(const void* d_k_pages, const void* d_v_pages, const int32_t* d_page_table, size_t ctx,
                            size_t page_tokens, size_t num_kv_heads, size_t head_dim, int kv_dtype, void* d_k_out,
                            void* d_v_out, void* stream);

/* ------------------------------------------------------ fp32 helpers */
/* y = x / sqrt(mean(x^2) + eps) * w per row (src/kernel/cuda/cuda_rmsnorm_f32.cu:9-36). */
int vspec_b200_rmsnorm_f32(const float* d_x, const float* d_w, float eps, size_t rows, size_t dim, float* d_y,
                           void* stream);
/* y[m][n] = x[m][k] . W[n][k]^T in fp32 (src/kernel/cuda/cuda_linear_f32.cu:10-34). */
int vspec_b200_linear_f32(const float* d_x, const float* d_w, size_t m, size_t k, size_t n, float* d_y, void* stream);
/* data = silu(data) (src/kernel/cuda/cuda_elemwise_f32.cu:6-13) */
int vspec_b200_silu_f32(float* d_data, size_t count, void* stream);
/* data = data * other (src/kernel/cuda/cuda_elemwise_f32.cu:15-21) */
int vspec_b200_mul_f32(float* d_data, const float* d_other, size_t count, void* stream);

/* Test hook: the next `n` device allocations of the host C layer succeed and
 * the one after fails (n < 0 disables). */
int vspec_b200_debug_fail_alloc_after(int n);

/* Test hook: fills the split-K counter region of the current device's static
 * scratch (vspec_b200_lowbit_linear_static) with `byte`, the state a launch
 * whose bounded wait gave up can leave; the next static call must still be
 * correct.  A synchronous memset on the host's side, no kernel. */
int vspec_b200_debug_poison_static_scratch(int byte);

/* Test hook: one step of the hybrid bridge's temporal hot-column rule (the
 * selection vspec_cuda_fused_linear_hybrid_bridge makes before any device work,
 * with the same per-thread state and environment): writes the columns that
 * call would refine to out (capacity hot_count) and their number to *out_count.
 * No CUDA call is made. */
int vspec_b200_debug_anf_tcc_select(const uint32_t* hot, size_t hot_count, int have_int4, uint32_t* out,
                                    size_t* out_count);

/* Device properties used by the dispatch (filled on first use). */
int vspec_b200_device_info(int* sm_count, int* cc_major, int* cc_minor, size_t* smem_per_block_optin);

/* ------------------------------------------------------------------------
 * Decode-step kernels (no reference counterpart as kernels: the reference
 * runs this glue in numpy, Vspec-chat/python/runtime_inference.py:1297-1311,
 * 554-567).  Device pointers, async on `stream`.
 * ------------------------------------------------------------------------ */
/* x[b][:] = fp16 table[tok[b]][:] widened to fp32. */
int vspec_b200_decode_embed(const void* d_table_f16, const int32_t* d_tok, int batch, int hidden, float* d_x,
                            void* stream);
/* qkv [batch][(hq + 2 hkv) * head_dim] -> per-head RMSNorm of q and k (weights
 * [head_dim]), half-split rotary at position pos[b] (inv_freq = theta^(-i/(d/2))),
 * q to d_q_out [batch][hq][head_dim]; k and v appended as fp16 at slot
 * pos % page_tokens of page page_table[b][pos / page_tokens] ([P][page_tokens]
 * [hkv][head_dim] pools); ctx_len[b] = pos[b] + 1. */
int vspec_b200_decode_qk_rope_append(const float* d_qkv, const float* d_q_norm, const float* d_k_norm,
                                     const int32_t* d_pos, int batch, int hq, int hkv, int head_dim, float eps,
                                     float theta, float* d_q_out, void* d_k_pages, void* d_v_pages,
                                     const int32_t* d_page_table, int max_pages, int page_tokens, int32_t* d_ctx_len,
                                     void* stream);
/* Next token per sequence: the prompt's token at pos+1 while the prompt lasts,
 * else the argmax of the logits cleaned like _stabilize_logits (NaN -> 0,
 * clip to +-clip; ties -> lowest index); recorded at out_tokens[b][pos+1];
 * pos[b] += 1.  d_state: 12 bytes per sequence (8-byte aligned), zero before
 * the first call; every call leaves it zero. */
int vspec_b200_decode_next_token(const float* d_logits, int batch, int vocab, float clip, const int32_t* d_prompt,
                                 const int32_t* d_prompt_len, int max_prompt, int32_t* d_pos, int32_t* d_tok,
                                 int32_t* d_out_tokens, int max_steps, void* d_state, void* stream);
/* Seeded fill: kind 0 uniform bytes, 1 fp16 uniform in [lo, hi), 2 fp32 constant lo. */
int vspec_b200_random_fill(void* d_dst, size_t count, int kind, uint64_t seed, float lo, float hi, void* stream);
/* Same streams (kinds 0 and 1) for a rows x cols block of a [*][global_cols]
 * tensor starting at (row0, col0), stored with row stride dst_stride: a shard
 * receives exactly the values the whole tensor has there. */
int vspec_b200_random_fill_block(void* d_dst, size_t rows, size_t cols, size_t dst_stride, int kind, uint64_t seed,
                                 size_t global_cols, size_t row0, size_t col0, float lo, float hi, void* stream);

/* ------------------------------------------------------------------------
 * Load-time quantise + pack on the device, bit for bit the reference's
 * _quantize_weight_rowwise (Vspec-chat/python/runtime_inference.py:708-785)
 * on float32 weights.  d_w [n][k] fp32.  block_size: codes per scale group
 * along k, a multiple of 32 (the reference's int4 default path, block size
 * VSPEC_INT4_BLOCK_SIZE rounded up to 32), or 0 for whole rows (its int3 /
 * int2 path and int4 with VSPEC_INT4_BLOCKWISE_ENABLE off).  percentile as
 * VSPEC_QUANT_ROW_PERCENTILE (clamped to [0.95, 1]; >= 0.9999 uses min/max).
 * Outputs: d_packed [n][ceil(k*bits/8)] signed codes LSB first, d_scales and
 * d_zero_points [n][groups] fp32 (d_zero_points may be NULL: the reference
 * returns no zero-points for int2, though its codes carry them).  A group is
 * at most 46080 codes.
 * ------------------------------------------------------------------------ */
int vspec_b200_quantize_rowwise(const float* d_w, size_t n, size_t k, int bits, int block_size, double percentile,
                                uint8_t* d_packed, float* d_scales, float* d_zero_points, void* stream);

/* ------------------------------------------------------------------------
 * Qwen3-shape low-bit decode loop (36 or 64 layers, hidden 4096 / 5120), random-init weights.
 * Host C driving the kernels above, the low-bit linears (RMSNorm / SwiGLU /
 * residual fused) and the paged attention; one decode step = one CUDA graph.
 * Linear weights: packed `bits`-bit codes (unsigned reading, mid-range
 * zero-point), fp16 group scales (group 128) -- the engine's int4 layout.
 * ------------------------------------------------------------------------ */
typedef struct VspecB200QwenConfig {
    int num_layers, hidden, num_heads, num_kv_heads, head_dim, intermediate, vocab;
    int bits;          /* attention projections and lm_head: 4, 3 or 2 */
    int group;         /* codes per scale group along k (multiple of 128) */
    float rms_eps, rope_theta, logit_clip;
    int page_tokens;
    int bits_mlp;      /* gate/up and down projections; 0 = same as bits */
} VspecB200QwenConfig;

int vspec_b200_qwen_create(const VspecB200QwenConfig* cfg, uint64_t seed, int max_batch, int max_ctx,
                           void** out_model);
/* The 128-byte NCCL unique id a tensor-parallel group shares: rank 0 makes it
 * and hands the same bytes to every rank. */
int vspec_b200_nccl_unique_id(void* out_id128);
/* Tensor-parallel shard (rank tp_rank of tp_size, one GPU each, the device
 * current when called; every rank calls it, it returns once all joined).
 * Column-parallel q/k/v heads and gate/up rows, row-parallel o-proj and down
 * projections followed by an NCCL all-reduce over NVLink; embedding and
 * lm_head replicated, so every rank produces the same tokens.  Each rank holds
 * exactly its slice of the same random-init weights as the unsharded model.
 * Requires num_heads, num_kv_heads and intermediate divisible by tp_size, and
 * the row-parallel slices (num_heads*head_dim/tp, intermediate/tp) to be whole
 * scale groups. */
int vspec_b200_qwen_create_tp(const VspecB200QwenConfig* cfg, uint64_t seed, int max_batch, int max_ctx, int tp_size,
                              int tp_rank, const void* nccl_id128, void** out_model);
void vspec_b200_qwen_destroy(void* model);
/* Prompt prefill (one decode step per prompt token) and greedy generation for
 * `batch` sequences.  h_prompts [batch][prompt_len]; h_tokens_out
 * [batch][prompt_len + gen_tokens] receives the prompt followed by the
 * generated tokens.  *out_gen_ms (optional) = device time of the steps that
 * produced the gen_tokens tokens.  h_logits_out (optional) receives the
 * logits of every step, [steps][batch][vocab] with steps = prompt_len +
 * gen_tokens - 1. */
int vspec_b200_qwen_generate(void* model, int batch, const int32_t* h_prompts, int prompt_len, int gen_tokens,
                             int32_t* h_tokens_out, float* out_gen_ms, float* h_logits_out);
/* Device tensors of the model (this rank's shard), for checking against a host oracle:
 * kind 0 embedding fp16 [vocab][hidden]; per layer 1/2 qkv codes/scales,
 * 3/4 o-proj, 5/6 gate+up (gate rows first), 7/8 down; 9/10 lm_head
 * codes/scales.  Norm weights are all ones.  Returns the byte size, copies
 * it to h_dst when h_dst is not NULL (0 on error). */
size_t vspec_b200_qwen_tensor(void* model, int kind, int layer, void* h_dst);

#ifdef __cplusplus
}
#endif

#endif /* VSPEC_B200_H */
