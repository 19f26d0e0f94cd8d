// attention_kernels.cuh -- internal interface of the paged attention kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

namespace vb200 {

constexpr int kKvF32 = 0;
constexpr int kKvF16 = 1;
constexpr int kKvInt3 = 2;

struct AttnParams {
    const float* q;             // [batch][hq][d]
    const void* k_pages;        // [pages][page_tokens][hkv][d]
    const void* v_pages;
    const int32_t* page_table;  // [batch][max_pages]
    const int32_t* ctx_len;     // [batch]
    float* out;                 // [batch][hq][d]
    float* part_o;              // [batch][hq][max_splits][d]
    float* part_ml;             // [batch][hq][max_splits][2]
    float scale;
    int batch, hq, hkv, d, page_tokens, max_pages;
    int split_tokens, max_splits, head_groups;
    int num_pages;              // valid page ids are [0, num_pages)
    // int3 pages (kv_dtype kKvInt3): k_pages / v_pages hold the codes
    // [pages][page_tokens][hkv][3*d/8], these the per-block fp32 scales
    // [pages][page_tokens][hkv][d/kv_block]
    const float* k_scales;
    const float* v_scales;
    int kv_block;
};

int attn_read_and_clear_page_fault(int* out);

int attn_choose_split(int batch, int hq, int hkv, int max_ctx, int page_tokens, int sms, int ctas_per_sm,
                      int max_staged_pages);
// What the planner assumes per kernel: resident CTAs per SM and staged page ids per CTA.
struct AttnPlanShape {
    int ctas_per_sm, max_staged_pages;
};
// fp16/fp32 kernels, and the SIMT int3 kernel
constexpr AttnPlanShape kAttnPlanF16 = {2, 512};
// int3 tensor-core kernel: four CTAs per SM with one column tile (query groups up to 4), else three
inline AttnPlanShape attn_plan_int3(int hq, int hkv) {
    const int group = hkv > 0 ? hq / hkv : 1;
    return AttnPlanShape{group <= 4 ? 4 : 3, 256};
}
size_t attn_workspace_bytes(int batch, int hq, int d, int max_splits);
int paged_attention_launch(AttnParams p, int kv_dtype, cudaStream_t st);
// int3 KV compression of rows [rows][heads][d] fp32 into pool rows slots[r]
// (rows r when slots is NULL): codes [.][heads][3*d/8], scales [.][heads][d/block].
int kv_int3_quantize_launch(const float* src, const int32_t* slots, int rows, int heads, int d, int block,
                            float percentile, uint8_t* codes, float* scales, cudaStream_t st);
int paged_gather_launch(const void* kp, const void* vp, const int32_t* table, int ctx, int pt, int hkv, int d,
                        int kv_dtype, void* kout, void* vout, cudaStream_t st);

}  // namespace vb200
