// q4k.cu -- Q4_K dequant-matmul on the GPU: the reference's
// 256-element super-block format (src/quant/formats/q4_k.c:41-134,
// include/vspec/quant/formats/q4_k.h:7-16) behind a decode GEMV.
//
// A row of W is k/256 blocks of 144 bytes: fp16 d, fp16 dmin, 12 bytes of
// sixteen 6-bit values packed LSB first (sub-scales 0..7, sub-mins 8..15),
// 128 bytes of 4-bit codes (element 2i in the low nibble of byte i).  Element
// t of sub-block sb is d*(sc[sb]/63) * q - dmin*(mn[sb]/63); y = x W^T.
//
// x is staged once per CTA in shared memory; each warp streams 4 output rows
// for all activation rows of the launch (m <= 8, as many as the staging
// budget holds); lane l takes the 32-element sub-blocks l, l+32, ... of a
// row: one 16-byte load of the block header (shared by the 8 lanes of a
// block) and one of its 32 codes.  Per sub-block the partial is
// sub_scale * sum(x*q) - sub_min * sum(x) in fp32; warp sums give y.
#include "common.cuh"

namespace vb200 {

constexpr int kQ4kWarps = 8;
constexpr int kQ4kMaxM = 8;
constexpr int kQ4kRowsPerWarp = 4;
constexpr int kQ4kSubPad = 36;   // floats per staged 32-element sub-block (+16 B: conflict-free float4 reads)
constexpr size_t kQ4kStageMax = 96 * 1024;
constexpr size_t kQ4kSumMax = kQ4kMaxM * (8192 / 32) * sizeof(float);   // per-sub-block sums of x

__device__ __forceinline__ uint32_t q4k_field6(uint32_t w0, uint32_t w1, uint32_t w2, int idx) {
    const int bit = 6 * idx, word = bit >> 5, off = bit & 31;
    const uint32_t lo = word == 0 ? w0 : (word == 1 ? w1 : w2);
    const uint32_t hi = word == 0 ? w1 : (word == 1 ? w2 : 0u);
    return __funnelshift_r(lo, hi, (uint32_t)off) & 0x3Fu;
}

// The low nibble of w as a float, exactly: 2^23 + q has q in its mantissa's
// low bits, and subtracting 2^23 leaves q (a logic op and an add instead of an
// integer-to-float conversion).
__device__ __forceinline__ float q4k_code(uint32_t w) {
    return __uint_as_float(0x4B000000u | (w & 0xFu)) - 8388608.0f;
}

// x is staged once per CTA in shared memory, [m][k/32][36] floats (every
// 32-element sub-block padded by 16 bytes, so the 8 lanes of a load phase,
// which read 8 different sub-blocks, hit different banks).  Warp w then takes
// rows CTA*32 + 4w .. +3, RPS of them at a time; lane l the sub-blocks l,
// l+32, ... of each, with all header and code loads of those RPS rows issued
// before the math (SPL sub-blocks per lane and row; m = 1 with k <= 4096 runs
// RPS 2 and SPL 4, the rest RPS 1 and SPL 8; a
// double-buffered variant, 4 sub-blocks per lane and chunk with the next
// chunk's loads issued before the current chunk's math, measured 31.9 us
// against 28.7 us for this kernel with per-code conversions at K=4096
// N=12288 M=1).
template <int MM, int RPS, int SPL>
__global__ void __launch_bounds__(kQ4kWarps * 32)
q4k_gemv_kernel(const float* __restrict__ x, const uint8_t* __restrict__ w, float* __restrict__ y, int m, int n,
                int k) {
    extern __shared__ __align__(16) float xs_sm[];
    __shared__ float div63[64];   // v / 63 for the 6-bit fields, the same IEEE quotient as q4_k.c:94-95
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nb = k / 256, nsub = nb * 8;
    if (tid < 64) div63[tid] = __fdiv_rn((float)tid, 63.0f);
    // stage x (float4 granules)
    const int nq = m * k / 4;
    for (int i = tid; i < nq; i += kQ4kWarps * 32) {
        const int r = (4 * i) / k, t = 4 * i - r * k;
        const float4 v = __ldg(reinterpret_cast<const float4*>(x + (size_t)r * k + t));
        *reinterpret_cast<float4*>(xs_sm + ((size_t)r * nsub + (t >> 5)) * kQ4kSubPad + (t & 31)) = v;
    }
    __syncthreads();
    // sum(x) of every staged sub-block, once per CTA (the sub-min term needs only that)
    float* xsum_sm = xs_sm + (size_t)m * nsub * kQ4kSubPad;
    for (int i = tid; i < m * nsub; i += kQ4kWarps * 32) {
        const float4* xp = reinterpret_cast<const float4*>(xs_sm + (size_t)i * kQ4kSubPad);
        float sum = 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float4 v = xp[q];
            sum += (v.x + v.y) + (v.z + v.w);
        }
        xsum_sm[i] = sum;
    }
    __syncthreads();
    // RPS rows of a warp are streamed together: every header and code load of
    // those rows is issued before the math, so a warp waits RPS times fewer
    // memory round trips (SPL sub-blocks per lane and row cover k <= 32*SPL*32)
    for (int rr = 0; rr < kQ4kRowsPerWarp; rr += RPS) {
        int js[RPS];
        bool vj[RPS];
#pragma unroll
        for (int q = 0; q < RPS; ++q) {
            js[q] = (blockIdx.x * kQ4kWarps + warp) * kQ4kRowsPerWarp + rr + q;
            vj[q] = js[q] < n;
        }
        if (!vj[0]) break;
        float acc[RPS][MM];
#pragma unroll
        for (int q = 0; q < RPS; ++q)
#pragma unroll
            for (int r = 0; r < MM; ++r) acc[q][r] = 0.f;
        for (int s0 = lane; s0 < nsub; s0 += 32 * SPL) {
            uint4 hdr[RPS][SPL], qv[RPS][SPL];
#pragma unroll
            for (int q = 0; q < RPS; ++q) {
                const uint8_t* row = w + (size_t)js[q] * nb * 144;
#pragma unroll
                for (int u = 0; u < SPL; ++u) {
                    const int s = s0 + 32 * u;
                    if (vj[q] && s < nsub) {
                        const uint8_t* blk = row + (size_t)(s >> 3) * 144;
                        hdr[q][u] = __ldg(reinterpret_cast<const uint4*>(blk));
                        qv[q][u] = __ldg(reinterpret_cast<const uint4*>(blk + 16 + (s & 7) * 16));
                    }
                }
            }
#pragma unroll
            for (int q = 0; q < RPS; ++q) {
#pragma unroll
                for (int u = 0; u < SPL; ++u) {
                    const int s = s0 + 32 * u;
                    if (vj[q] && s < nsub) {
                        const int sb = s & 7;
                        const float d = __half2float(__ushort_as_half((unsigned short)(hdr[q][u].x & 0xFFFFu)));
                        const float dmin = __half2float(__ushort_as_half((unsigned short)(hdr[q][u].x >> 16)));
                        const uint32_t sc = q4k_field6(hdr[q][u].y, hdr[q][u].z, hdr[q][u].w, sb);
                        const uint32_t mn = q4k_field6(hdr[q][u].y, hdr[q][u].z, hdr[q][u].w, 8 + sb);
                        const float sub_scale = d * div63[sc];   // q4_k.c:94-95
                        const float sub_min = dmin * div63[mn];
                        const uint32_t qw[4] = {qv[q][u].x, qv[q][u].y, qv[q][u].z, qv[q][u].w};
#pragma unroll
                        for (int r = 0; r < MM; ++r) {
                            if (r < m) {
                                const float4* xp = reinterpret_cast<const float4*>(xs_sm + ((size_t)r * nsub + s) * kQ4kSubPad);
                                float xq = 0.f;
#pragma unroll
                                for (int i = 0; i < 8; ++i) {
                                    const float4 v = xp[i];
                                    const uint32_t wd = qw[i >> 1] >> (16 * (i & 1));   // 4 codes, low nibble first
                                    xq = fmaf(v.x, q4k_code(wd), xq);
                                    xq = fmaf(v.y, q4k_code(wd >> 4), xq);
                                    xq = fmaf(v.z, q4k_code(wd >> 8), xq);
                                    xq = fmaf(v.w, q4k_code(wd >> 12), xq);
                                }
                                const float xsum = xsum_sm[(size_t)r * nsub + s];
                                acc[q][r] = fmaf(sub_scale, xq, fmaf(-sub_min, xsum, acc[q][r]));
                            }
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int q = 0; q < RPS; ++q) {
#pragma unroll
            for (int r = 0; r < MM; ++r) {
                if (r < m) {
                    const float v = warp_sum(acc[q][r]);
                    if (lane == 0 && vj[q]) y[(size_t)r * n + js[q]] = v;
                }
            }
        }
    }
}

}  // namespace vb200

using namespace vb200;

extern "C" int vspec_b200_q4k_linear(const float* d_x, const void* d_blocks, float* d_y, size_t m, size_t n, size_t k,
                                     void* stream) {
    if (!d_x || !d_blocks || !d_y) { set_error("NULL pointer argument"); return VSPEC_B200_ERR_ARG; }
    if (m == 0 || n == 0) return VSPEC_B200_OK;
    if (k == 0 || k % 256 != 0) { set_error("q4k_linear: k must be a positive multiple of 256"); return VSPEC_B200_ERR_UNSUPPORTED; }
    if (n > (size_t)INT32_MAX / (kQ4kWarps * kQ4kRowsPerWarp) || k > (size_t)INT32_MAX) { set_error("q4k_linear: shape too large"); return VSPEC_B200_ERR_ARG; }
    if (reinterpret_cast<uintptr_t>(d_blocks) % 16 != 0 || reinterpret_cast<uintptr_t>(d_x) % 16 != 0) {
        set_error("q4k_linear: x and the blocks must be 16-byte aligned");
        return VSPEC_B200_ERR_ARG;
    }
    if (k > 8192) { set_error("q4k_linear: k above 8192 unsupported"); return VSPEC_B200_ERR_UNSUPPORTED; }
    cudaStream_t st = (cudaStream_t)stream;
    const size_t rows_per_cta = (size_t)kQ4kWarps * kQ4kRowsPerWarp;
    const unsigned grid = (unsigned)((n + rows_per_cta - 1) / rows_per_cta);
    // activation rows per launch: as many as fit the staged-x budget (at most 8)
    const size_t per_row = (k / 32) * kQ4kSubPad * sizeof(float);
    size_t mmax = kQ4kStageMax / per_row;
    if (mmax > (size_t)kQ4kMaxM) mmax = kQ4kMaxM;
    // m = 1 and k <= 4096: two rows in flight per warp with 4 sub-blocks per
    // lane each (K=4096 N=12288: 20.7 us against 23.1 us for one row); larger k
    // and m > 1 keep one row with 8 sub-blocks per lane (two rows measured
    // slower there: the staged-x reads, not the weight loads, bound them)
    const bool two_rows = m == 1 && k <= 4096;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        const int smax = (int)(kQ4kStageMax + kQ4kSumMax);
        cudaError_t e = cudaFuncSetAttribute(q4k_gemv_kernel<1, 1, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, smax);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(q4k_gemv_kernel<kQ4kMaxM, 1, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, smax);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(q4k_gemv_kernel<1, 2, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, smax);
        if (e != cudaSuccess) return cuda_status(e, "q4k_gemv_kernel smem attribute");
        configured[dev] = 1;
    }
    for (size_t i0 = 0; i0 < m; i0 += mmax) {
        const int mm = (int)((m - i0) < mmax ? (m - i0) : mmax);
        const float* xb = d_x + i0 * k;
        float* yb = d_y + i0 * n;
        const uint8_t* wb = (const uint8_t*)d_blocks;
        const size_t smem = (size_t)mm * (per_row + (k / 32) * sizeof(float));
        const unsigned th = kQ4kWarps * 32;
        if (two_rows) q4k_gemv_kernel<1, 2, 4><<<grid, th, smem, st>>>(xb, wb, yb, mm, (int)n, (int)k);
        else if (mm == 1) q4k_gemv_kernel<1, 1, 8><<<grid, th, smem, st>>>(xb, wb, yb, mm, (int)n, (int)k);
        else q4k_gemv_kernel<kQ4kMaxM, 1, 8><<<grid, th, smem, st>>>(xb, wb, yb, mm, (int)n, (int)k);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return cuda_status(e, "q4k_gemv_kernel launch");
    }
    return VSPEC_B200_OK;
}
