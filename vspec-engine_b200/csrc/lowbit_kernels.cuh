// lowbit_kernels.cuh -- internal interface between the kernels and the C-ABI layer.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

namespace vb200 {

struct GemvParams {
    const float* x;          // [m][k] fp32 activations
    const uint8_t* w;        // [n][row_bytes] packed codes
    const void* s;           // [n][n_groups] fp32 or fp16
    const void* zp;          // [n][n_groups] same dtype or nullptr
    float zp_const;          // zero-point used when zp == nullptr
    float* y;                // [m][n] (or [m][n/2] with SwiGLU)
    const float* residual;   // [m][n] added when VSPEC_B200_F_RESIDUAL
    const float* norm_w;     // [k] RMSNorm weight when VSPEC_B200_F_RMSNORM
    float eps;
    int m, n, k, n_groups;
    int row_bytes;
    int kb_total;            // k / 128 (fast path)
    int kb_per_group;        // (k / n_groups) / 128 (fast path)
    int kb_per_group_shift;  // log2(kb_per_group), or -1 if not a power of two
    int flags;
    // persistent split-K plan (fast path)
    int tiles;               // 16-row tiles
    int total_warps;         // warps sharing the (tile, k-block) units
    int max_slots;           // partial slots per counter
    float* scratch;          // [counters][max_slots][16*m] fp32 partials
    int* counters;           // [counters], zero between launches
    int stages;              // tcgen05 path: weight ring depth
    int tile_parts;          // ring path: 0 = contiguous unit runs, P = each tile's k-blocks split over P CTAs
    int cluster_merge;       // ring path: the P parts of a tile are one cluster, merged through DSMEM
};

constexpr int kEpiPlain = 0;
constexpr int kEpiSwiGLU = 1;
constexpr int kGemvMaxM = 8;
constexpr size_t kGemvMaxSmem = 200 * 1024;

#define EPI_HAS_RMSNORM(flags) (((flags) & VSPEC_B200_F_RMSNORM) != 0)

constexpr int kPathAuto = 0;
constexpr int kPathGeneric = 1;
constexpr int kPathWarpMma = 2;
constexpr int kPathTensorCore = 3;
constexpr int kPathRing = 4;
constexpr int kPathRows = 5;
int lowbit_gemv_launch(GemvParams p, int bits, int unsigned_codes, cudaStream_t st, int path,
                       void* workspace, size_t workspace_bytes);
size_t gemv_workspace_bytes(int m, int n, int k, bool swiglu);
// tcgen05 / TMA path (lowbit_gemv_tc.cu)
bool gemv_tc_supported(const GemvParams& p, int bits, size_t counter_slots);
int gemv_tc_launch(GemvParams p, int bits, int unsigned_codes, cudaStream_t st, bool pdl);
size_t gemv_tc_scratch_floats(int m, int n, int k, bool swiglu);
int gemv_tc_read_and_clear_timeout(int* out);
// TMA ring + warp-MMA path (lowbit_gemv_ring.cu)
bool gemv_ring_supported(const GemvParams& p, int bits, size_t counter_slots);
int gemv_ring_launch(GemvParams p, int bits, int unsigned_codes, cudaStream_t st, bool pdl);
size_t gemv_ring_scratch_floats(int m, int n, int k, bool swiglu);
int gemv_ring_read_and_clear_timeout(int* out);
// row-sliced TMA GEMV, no workspace (lowbit_gemv_rows.cu)
bool gemv_rows_supported(const GemvParams& p, int bits);
bool gemv_rows_preferred(const GemvParams& p, int bits);
int gemv_rows_launch(GemvParams p, int bits, int unsigned_codes, cudaStream_t st, bool pdl);
int gemv_rows_read_and_clear_timeout(int* out);
// tcgen05 GEMM for m > kGemvMaxM (lowbit_gemm_tc.cu)
bool gemm_tc_supported(const GemvParams& p, int bits, size_t counter_slots);
size_t gemm_tc_workspace_bytes(int m, int n, int k, bool swiglu);
int gemm_tc_launch(const GemvParams& p, int bits, int unsigned_codes, cudaStream_t st, void* work);
int gemm_tc_read_and_clear_timeout(int* out);
int unpack_codes_launch(const uint8_t* w, int n, int k, int bits, int unsigned_codes, int8_t* out, cudaStream_t st,
                        int use_fast_decoder);

}  // namespace vb200
