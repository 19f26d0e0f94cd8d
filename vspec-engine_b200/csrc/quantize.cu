// quantize.cu -- load-time quantise + pack on the GPU, bit for bit the
// reference's float-to-low-bit weight quantiser, _quantize_weight_rowwise
// (Vspec-chat/python/runtime_inference.py:708-785), as numpy runs it on
// float32 weights:
//   * per group (a block of block_size codes along k -- the int4 default --
//     or a whole row): lo / hi = the group's (1 - p) and p quantiles by
//     numpy's 'linear' method (q in float32, virtual index (n-1)*q, gamma its
//     fractional part, a + (b-a)*g below 0.5 and b - (b-a)*(1-g) from 0.5),
//     or min / max when p >= 0.9999;
//   * scale = max(hi - lo, 1e-8) / levels, zp = clip(round(min_q - lo/scale)),
//     code = clip(round(w/scale + zp)), float32 with round-half-to-even;
//   * codes packed LSB first per row (src/quant/pack.c:30-51, one row at a
//     time as runtime_inference.py:679-705 does).
// One CTA per group keeps the group's values in shared memory; the needed
// order statistics come from a radix select over order-preserving keys
// (4 passes of 8 bits).  The float steps use the _rn intrinsics, which the
// compiler never fuses, so every rounding is the one numpy performs.
#include "common.cuh"

#include <math.h>

namespace vb200 {

constexpr int kQThreads = 256;
constexpr size_t kQMaxGroup = 45 * 1024;   // values of one group held in shared memory (5 bytes each)

__device__ __forceinline__ uint32_t q_key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float q_unkey(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// The kth smallest (0-based) of vals[0, n) (shared memory), by all threads.
__device__ float q_select(const float* vals, int n, int kth, unsigned* hist, unsigned* sel) {
    uint32_t prefix = 0, mask = 0;
    unsigned k = (unsigned)kth;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0u;
        __syncthreads();
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const uint32_t key = q_key(vals[i]);
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            // warp 0: bins 8l .. 8l+7 per lane, inclusive scan over lanes
            const int lane = threadIdx.x;
            unsigned local[8], sum = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) { local[j] = hist[8 * lane + j]; sum += local[j]; }
            unsigned incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            const unsigned excl = incl - sum;
            if (excl <= k && k < incl) {
                unsigned acc = excl;
                int d = 0;
                for (; d < 7; ++d) {
                    if (acc + local[d] > k) break;
                    acc += local[d];
                }
                sel[0] = (unsigned)(8 * lane + d);
                sel[1] = acc;
            }
        }
        __syncthreads();
        const uint32_t digit = sel[0];
        k -= sel[1];
        prefix |= digit << shift;
        mask |= 255u << shift;
        __syncthreads();
    }
    return q_unkey(prefix);
}

// numpy's linear quantile of the group (same steps as np.quantile on float32).
__device__ float q_quantile(const float* vals, int n, float q32, unsigned* hist, unsigned* sel) {
    const float vi = __fmul_rn((float)(n - 1), q32);
    if (!(vi > 0.0f)) return q_select(vals, n, 0, hist, sel);
    if (vi >= (float)(n - 1)) return q_select(vals, n, n - 1, hist, sel);
    const float prev = floorf(vi);
    const int lo = (int)prev;
    const float g = __fsub_rn(vi, prev);
    const float a = q_select(vals, n, lo, hist, sel);
    const float b = q_select(vals, n, lo + 1, hist, sel);
    const float d = __fsub_rn(b, a);
    if (g >= 0.5f) return __fsub_rn(b, __fmul_rn(d, __fsub_rn(1.0f, g)));
    return __fadd_rn(a, __fmul_rn(d, g));
}

struct QuantParams {
    const float* w;
    uint8_t* packed;
    float* scales;
    float* zero_points;   // may be null
    int n, k, bits, group;   // group: codes per scale group along k (k for whole rows)
    int n_groups;            // groups per row
    int minmax;              // percentile >= 0.9999: min / max
    float q_lo, q_hi;        // (1 - p) and p as float32
    size_t row_bytes;
};

__global__ void __launch_bounds__(kQThreads) quantize_rowwise_kernel(const QuantParams p) {
    extern __shared__ __align__(16) unsigned char q_smem[];
    __shared__ unsigned hist[256];
    __shared__ unsigned sel[2];
    __shared__ float sz[2];
    const int r = blockIdx.x, gb = blockIdx.y;
    const int s0 = gb * p.group;
    const int s1 = min(p.k, s0 + p.group);
    const int len = s1 - s0;
    float* vals = reinterpret_cast<float*>(q_smem);
    int8_t* codes = reinterpret_cast<int8_t*>(vals + p.group);
    const float* wr = p.w + (size_t)r * p.k;
    for (int i = threadIdx.x; i < len; i += blockDim.x) vals[i] = wr[s0 + i];
    __syncthreads();
    float lo, hi;
    if (p.minmax) {
        lo = q_select(vals, len, 0, hist, sel);
        hi = q_select(vals, len, len - 1, hist, sel);
    } else {
        lo = q_quantile(vals, len, p.q_lo, hist, sel);
        hi = q_quantile(vals, len, p.q_hi, hist, sel);
    }
    const float max_q = (float)((1 << (p.bits - 1)) - 1);
    const float min_q = (float)(-(1 << (p.bits - 1)));
    if (threadIdx.x == 0) {
        const float levels = fmaxf(1.0f, __fsub_rn(max_q, min_q));
        float span = __fsub_rn(hi, lo);
        if (span < 1e-8f) span = 1e-8f;
        const float scale = __fdiv_rn(span, levels);
        float zp = rintf(__fsub_rn(min_q, __fdiv_rn(lo, scale)));
        zp = fminf(fmaxf(zp, min_q), max_q);
        sz[0] = scale;
        sz[1] = zp;
        p.scales[(size_t)r * p.n_groups + gb] = scale;
        if (p.zero_points) p.zero_points[(size_t)r * p.n_groups + gb] = zp;
    }
    __syncthreads();
    const float scale = sz[0], zp = sz[1];
    for (int i = threadIdx.x; i < len; i += blockDim.x) {
        float q = rintf(__fadd_rn(__fdiv_rn(vals[i], scale), zp));
        q = fminf(fmaxf(q, min_q), max_q);
        codes[i] = (int8_t)q;
    }
    __syncthreads();
    // pack the group's bytes: [s0*bits/8, ceil(s1*bits/8)) -- groups start on
    // a byte (multiples of 32 codes, or the row start); pad bits stay zero
    const int bits = p.bits;
    const unsigned mask = (1u << bits) - 1u;
    const int b0 = (s0 * bits) >> 3;
    const int b1 = (s1 * bits + 7) >> 3;
    uint8_t* out = p.packed + (size_t)r * p.row_bytes;
    for (int j = b0 + threadIdx.x; j < b1; j += blockDim.x) {
        unsigned v = 0u;
        const int c_first = (8 * j) / bits, c_last = (8 * j + 7) / bits;
        for (int c = c_first; c <= c_last; ++c) {
            if (c < s0 || c >= s1) continue;
            const unsigned u = (unsigned)(int)codes[c - s0] & mask;
            const int pos = c * bits - 8 * j;
            v |= pos >= 0 ? (u << pos) : (u >> (-pos));
        }
        out[j] = (uint8_t)(v & 0xFFu);
    }
}

}  // namespace vb200

using namespace vb200;

extern "C" int vspec_b200_quantize_rowwise(const float* d_w, size_t n, size_t k, int bits, int block_size,
                                           double percentile, uint8_t* d_packed, float* d_scales,
                                           float* d_zero_points, void* stream) {
    if (!d_w || !d_packed || !d_scales || n == 0 || k == 0 || bits < 2 || bits > 4 || block_size < 0 ||
        (block_size > 0 && block_size % 32 != 0) || n > (size_t)INT32_MAX || k > (size_t)INT32_MAX) {
        set_error("bad quantize_rowwise arguments");
        return VSPEC_B200_ERR_ARG;
    }
    const size_t group = block_size > 0 ? (size_t)block_size : k;
    const size_t g_eff = group < k ? group : k;
    if (g_eff > kQMaxGroup) {
        set_error("quantize_rowwise: group of %zu codes exceeds %zu", g_eff, kQMaxGroup);
        return VSPEC_B200_ERR_UNSUPPORTED;
    }
    double pc = percentile;
    if (!(pc >= 0.95)) pc = 0.95;
    if (pc > 1.0) pc = 1.0;
    QuantParams p;
    p.w = d_w;
    p.packed = d_packed;
    p.scales = d_scales;
    p.zero_points = d_zero_points;
    p.n = (int)n;
    p.k = (int)k;
    p.bits = bits;
    p.group = (int)g_eff;
    p.n_groups = (int)((k + g_eff - 1) / g_eff);
    p.minmax = pc >= 0.9999 ? 1 : 0;
    p.q_lo = (float)(1.0 - pc);
    p.q_hi = (float)pc;
    p.row_bytes = (k * (size_t)bits + 7) / 8;
    const size_t smem = g_eff * sizeof(float) + g_eff;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(quantize_rowwise_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)(kQMaxGroup * sizeof(float) + kQMaxGroup));
        if (e != cudaSuccess) return cuda_status(e, "quantize_rowwise smem attribute");
        configured[dev] = 1;
    }
    if (p.n_groups > 65535) {
        set_error("quantize_rowwise: %d groups per row exceed the grid", p.n_groups);
        return VSPEC_B200_ERR_UNSUPPORTED;
    }
    quantize_rowwise_kernel<<<dim3((unsigned)n, (unsigned)p.n_groups), kQThreads, smem, (cudaStream_t)stream>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? VSPEC_B200_OK : cuda_status(e, "quantize_rowwise_kernel launch");
}
