// hybrid.cu -- the ANF hybrid linear: an int2 draft of every
// output column, then the "hot" columns recomputed from int4 weights
// (src/kernel/cuda/fused_linear_hybrid.cu:7-153).
//
// Draft: the int2 device GEMV, (q - 1.5) * s[col] with one fp32 scale per
// column (fused_linear_int2.cu:8-12), on the library's low-bit GEMV.
// Refine: for each listed column j < n and every activation row,
//   y[r][j] = sum_t x[r][t] * ((q4(j,t) - 8) * s4[j][b] + zp4[j][b]),
//   b = min(t / ceil(k / n_blocks), n_blocks - 1)   (b = 0 when n_blocks == 1),
// with unsigned nibbles (element 2i in the low nibble of byte i) and the
// zero-point ADDED (fused_linear_hybrid.cu:7-27).  The refine runs after the
// draft on the same stream and overwrites the draft values of those columns.
#include <string.h>

#include "common.cuh"
#include "lowbit_kernels.cuh"

namespace vb200 {

constexpr int kRefineThreads = 256;
constexpr int kRefineRows = 8;   // activation rows per pass over a column
constexpr int kRefineChunk = 16; // elements per thread and step (8 bytes of codes)

// One CTA per listed column; thread i takes the 16-element chunks i, i+256, ...
// of the row (a k = 4096 row is one round of loads: 8 bytes of codes and four
// float4 of x per activation row).  Per chunk the 16 weights are dequantised
// once into registers (the block index advanced at block boundaries inside the
// chunk) and reused for up to 8 activation rows; warp sums, then the 8 warps'
// partials through shared memory.
template <bool VEC>
__global__ void __launch_bounds__(kRefineThreads)
refine_hot_int4_kernel(const float* __restrict__ x, const uint8_t* __restrict__ w4, const float* __restrict__ s4,
                       const float* __restrict__ zp4, float* __restrict__ y, const uint32_t* __restrict__ hot,
                       int m, int n, int k, int nblk, int bs) {
    __shared__ float red[kRefineThreads / 32][kRefineRows];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t col = __ldg(hot + blockIdx.x);
    if (col >= (uint32_t)n) return;   // fused_linear_hybrid.cu:50-52 (uniform over the CTA)
    const size_t rb = ((size_t)k + 1) / 2;
    const uint8_t* wr = w4 + (size_t)col * rb;
    const float* sr = s4 + (size_t)col * nblk;
    const float* zr = zp4 ? zp4 + (size_t)col * nblk : nullptr;
    for (int r0 = 0; r0 < m; r0 += kRefineRows) {
        float acc[kRefineRows];
#pragma unroll
        for (int r = 0; r < kRefineRows; ++r) acc[r] = 0.f;
        for (int t0 = tid * kRefineChunk; t0 < k; t0 += kRefineThreads * kRefineChunk) {
            uint32_t cw[2];
            if (VEC) {
                const uint2 v = __ldg(reinterpret_cast<const uint2*>(wr + t0 / 2));
                cw[0] = v.x; cw[1] = v.y;
            } else {
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    uint32_t word = 0;
#pragma unroll
                    for (int bte = 0; bte < 4; ++bte) {
                        const size_t off = (size_t)t0 / 2 + 4 * i + bte;
                        if (off < rb) word |= (uint32_t)__ldg(wr + off) << (8 * bte);
                    }
                    cw[i] = word;
                }
            }
            int b = nblk > 1 ? min(t0 / bs, nblk - 1) : 0;
            int next = (b + 1) * bs;
            float s = __ldg(sr + b), z = zr ? __ldg(zr + b) : 0.f;
            float wv[kRefineChunk];
#pragma unroll
            for (int e = 0; e < kRefineChunk; ++e) {
                if (nblk > 1 && t0 + e >= next && b < nblk - 1) {
                    ++b;
                    next += bs;
                    s = __ldg(sr + b);
                    z = zr ? __ldg(zr + b) : 0.f;
                }
                const float q = (float)((cw[e >> 3] >> (4 * (e & 7))) & 0xFu);
                wv[e] = (t0 + e < k) ? fmaf(q - 8.0f, s, z) : 0.f;
            }
#pragma unroll
            for (int r = 0; r < kRefineRows; ++r) {
                if (r0 + r < m) {
                    const float* xr = x + (size_t)(r0 + r) * k + t0;
                    float a = acc[r];
                    if (VEC) {
#pragma unroll
                        for (int i = 0; i < kRefineChunk / 4; ++i) {
                            const float4 xv = __ldg(reinterpret_cast<const float4*>(xr) + i);
                            a = fmaf(xv.x, wv[4 * i], a);
                            a = fmaf(xv.y, wv[4 * i + 1], a);
                            a = fmaf(xv.z, wv[4 * i + 2], a);
                            a = fmaf(xv.w, wv[4 * i + 3], a);
                        }
                    } else {
#pragma unroll
                        for (int e = 0; e < kRefineChunk; ++e)
                            if (t0 + e < k) a = fmaf(__ldg(xr + e), wv[e], a);
                    }
                    acc[r] = a;
                }
            }
        }
#pragma unroll
        for (int r = 0; r < kRefineRows; ++r) {
            const float v = warp_sum(acc[r]);
            if (lane == 0) red[warp][r] = v;
        }
        __syncthreads();
        if (tid < kRefineRows && r0 + tid < m) {
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < kRefineThreads / 32; ++w) v += red[w][tid];
            y[(size_t)(r0 + tid) * n + col] = v;
        }
        __syncthreads();
    }
}

}  // namespace vb200

using namespace vb200;

extern "C" int vspec_b200_refine_hot_int4(const float* d_x, const unsigned char* d_w4, const float* d_s4,
                                          const float* d_zp4, float* d_y, const uint32_t* d_hot, size_t hot_count,
                                          size_t m, size_t n, size_t k, size_t n_blocks, void* stream) {
    if (hot_count == 0 || m == 0 || n == 0) return VSPEC_B200_OK;
    if (!d_x || !d_w4 || !d_s4 || !d_y || !d_hot) { set_error("NULL pointer argument"); return VSPEC_B200_ERR_ARG; }
    if (k == 0) { set_error("refine_hot_int4: k must be positive"); return VSPEC_B200_ERR_ARG; }
    if (n_blocks == 0) n_blocks = 1;   // fused_linear_hybrid.cu:132-134
    if (hot_count > (size_t)INT32_MAX || n_blocks > (size_t)INT32_MAX || m > (size_t)INT32_MAX ||
        n > (size_t)UINT32_MAX || k > (size_t)INT32_MAX - 1024) {
        set_error("refine_hot_int4: shape too large");
        return VSPEC_B200_ERR_ARG;
    }
    const int bs = n_blocks > 1 ? (int)((k + n_blocks - 1) / n_blocks) : (int)k;
    const bool vec = k % kRefineChunk == 0 && reinterpret_cast<uintptr_t>(d_w4) % 8 == 0 &&
                     reinterpret_cast<uintptr_t>(d_x) % 16 == 0;
    const unsigned grid = (unsigned)hot_count;
    cudaStream_t st = (cudaStream_t)stream;
    if (vec)
        refine_hot_int4_kernel<true><<<grid, kRefineThreads, 0, st>>>(d_x, d_w4, d_s4, d_zp4, d_y, d_hot, (int)m,
                                                                      (int)n, (int)k, (int)n_blocks, bs);
    else
        refine_hot_int4_kernel<false><<<grid, kRefineThreads, 0, st>>>(d_x, d_w4, d_s4, d_zp4, d_y, d_hot, (int)m,
                                                                       (int)n, (int)k, (int)n_blocks, bs);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e, "refine_hot_int4_kernel launch");
    return VSPEC_B200_OK;
}

extern "C" int vspec_b200_anf_hybrid_linear(const float* d_x, const unsigned char* d_w2, const float* d_s2,
                                            const unsigned char* d_w4, const float* d_s4, const float* d_zp4,
                                            float* d_y, const uint32_t* d_hot, size_t hot_count, size_t m, size_t n,
                                            size_t k, size_t n_blocks_int4, void* stream) {
    if (!d_x || !d_w2 || !d_s2 || !d_y) { set_error("NULL pointer argument"); return VSPEC_B200_ERR_ARG; }
    if (m == 0 || n == 0 || k == 0) return VSPEC_B200_OK;
    // draft: unsigned 2-bit codes, (u - 2) - (-0.5) = u - 1.5, one scale per column
    VspecB200LinearArgs a;
    memset(&a, 0, sizeof(a));
    a.d_x = d_x;
    a.d_w = d_w2;
    a.d_scales = d_s2;
    a.zero_point_const = -0.5f;
    a.d_y = d_y;
    a.m = m; a.n = n; a.k = k;
    a.n_groups = 1;
    a.bits = 2;
    a.flags = VSPEC_B200_F_UNSIGNED;
    int rc = vspec_b200_lowbit_linear(&a, stream);
    if (rc != VSPEC_B200_OK) return rc;
    if (hot_count == 0 || !d_hot || !d_w4 || !d_s4) return VSPEC_B200_OK;   // fused_linear_hybrid.cu:127-131
    return vspec_b200_refine_hot_int4(d_x, d_w4, d_s4, d_zp4, d_y, d_hot, hot_count, m, n, k, n_blocks_int4, stream);
}

// ---- include/vspec/kernel/cuda_fused.h:85-115 (default stream, no status) ----

extern "C" void vspec_cuda_refine_hot_int4_device(const float* d_a, const unsigned char* d_b_int4_packed,
                                                  const float* d_s_int4, const float* d_zp_int4, float* d_c,
                                                  const uint32_t* d_hot_indices, size_t hot_count, size_t m,
                                                  size_t n, size_t k, size_t n_blocks_int4) {
    // fused_linear_hybrid.cu:115-153: returns without work on NULL / empty arguments
    if (!d_a || !d_b_int4_packed || !d_s_int4 || !d_c || !d_hot_indices || hot_count == 0 || m == 0 || n == 0 ||
        k == 0)
        return;
    (void)vspec_b200_refine_hot_int4(d_a, d_b_int4_packed, d_s_int4, d_zp_int4, d_c, d_hot_indices, hot_count, m, n,
                                     k, n_blocks_int4, nullptr);
}

extern "C" void vspec_cuda_fused_linear_hybrid_device(const float* d_a, const unsigned char* d_b_int2_packed,
                                                      const float* d_s_int2, const unsigned char* d_b_int4_packed,
                                                      const float* d_s_int4, const float* d_zp_int4, float* d_c,
                                                      const uint32_t* d_hot_indices, size_t hot_count, size_t m,
                                                      size_t n, size_t k, size_t n_blocks_int4) {
    // fused_linear_hybrid.cu:70-113
    if (!d_a || !d_b_int2_packed || !d_s_int2 || !d_c || m == 0 || n == 0 || k == 0) return;
    (void)vspec_b200_anf_hybrid_linear(d_a, d_b_int2_packed, d_s_int2, d_b_int4_packed, d_s_int4, d_zp_int4, d_c,
                                       d_hot_indices, hot_count, m, n, k, n_blocks_int4, nullptr);
}
