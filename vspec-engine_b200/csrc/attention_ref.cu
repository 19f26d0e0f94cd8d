// attention_ref.cu -- the reference CPU backend's attention (vspec_attention_ref_single_query,
// src/attention/attention_ref.c:7-88; the CPU backend's launch_attention, cpu_backend.c:29-46)
// on the GPU, for callers that need its semantics rather than the plain softmax attention of
// the CUDA backend.  Per head h of a contiguous [tokens][heads][head_dim] fp32 cache (Hq = Hkv):
//   * q_h and every k row clamped to +-max(1e-6, 4.5 * population std), std computed in double
//     (three_bit_runtime_modules.c:175-203);
//   * score = dot(q_c, k_c) * (1 / sqrtf(d)), softmax with a double denominator (:205-250),
//     output = double sum over tokens of p_t * v_t[x] (:260-289);
//   * with the 3-bit runtime module on (VSPEC_FUSED_BITS=3 or VSPEC_3BIT_RUNTIME_MODULE, decided
//     as three_bit_runtime_modules.c:60-66 does): the noise reducer (clip +-16, consecutive-delta
//     limit 32; :138-173), a dot over blocks of 32 or 64 normalised by the block's largest
//     magnitude with Kahan sums (:291-342), the qk scale clipped to [1e-4, 32] (:344-361), logits
//     clipped to +-24 before the softmax, and Kahan output sums with the 1e7 limit (:260-282).
//
// Four launches, sized to fill the SMs rather than one CTA per head:
//   ref_scores_kernel  (tokens/TS x heads)   a CTA stages TS key rows of one head in shared memory
//                                            with coalesced loads; thread t conditions row t and
//                                            runs its dot in the reference's element order;
//   ref_softmax_kernel (heads)               max, double denominator, probabilities in place;
//   ref_output_kernel  (chunks x heads)      per dimension, a double (or Kahan) sum over the
//                                            chunk's tokens in order, coalesced over dimensions;
//   ref_combine_kernel (heads)               chunk partials added in chunk order.
// Per-token dots and per-row statistics use IEEE operations without contraction
// (__fmul_rn/__fadd_rn/__dmul_rn/__dadd_rn), so they round as the reference's SSE code does; the
// softmax denominator is a tree sum and the output sum is chunked, which moves only double
// roundings (a few 1e-16 relative) before the final rounding to float; expf is CUDA's (within
// 2 ulp) where the reference calls the C library's.
#include "common.cuh"

#include <float.h>
#include <stdint.h>
#include <stdlib.h>

#include "vspec_b200.h"

namespace vb200 {

constexpr int kRefMaxHeadDim = 1024;
constexpr int kRefOutThreads = 128;
constexpr size_t kRefStageBytes = 200u << 10;   // key-tile budget of one scores CTA

struct RefAttnParams {
    const float* q;       // [heads][d]
    const float* k;       // [tokens][heads][d]
    const float* v;
    float* out;           // [heads][d]
    float* probs;         // [heads][tokens] (workspace)
    double* part;         // [chunks][heads][d][2] (workspace): sum, compensation
    int tokens, heads, d;
    int module;           // 3-bit runtime module on
    int block;            // module dot block: 32 or 64
    int ts;               // tokens per scores CTA (= its threads)
    int tc;               // tokens per output chunk
    int chunks;
};

// The reference's clip: comparisons, so a NaN passes through unchanged.
__device__ __forceinline__ float ref_clip(float x, float lo, float hi) { return x < lo ? lo : (x > hi ? hi : x); }

// One step of the noise reducer on an already std-clamped value; prev is the previous output.
__device__ __forceinline__ float ref_denoise(float v, int i, float prev) {
    v = ref_clip(v, -16.f, 16.f);
    if (i > 0) {
        const float delta = __fsub_rn(v, prev);
        if (fabsf(delta) > 32.f) v = __fadd_rn(prev, delta > 0.f ? 32.f : -32.f);
    }
    return v;
}

// Kahan step of the reference's accumulator (double state, compensation limit 1e7).
__device__ __forceinline__ void ref_kahan(double& sum, double& comp, double value) {
    const double y = __dsub_rn(value, comp);
    const double t = __dadd_rn(sum, y);
    comp = __dsub_rn(__dsub_rn(t, sum), y);
    sum = t;
    if (fabs(sum) > 1e7) {
        sum = (double)ref_clip((float)sum, -1e7f, 1e7f);
        comp = 0.0;
    }
}

__device__ __forceinline__ float threshold_from_var(double var) {
    const float sd = (float)sqrt(var);
    return fmaxf(1e-6f, __fmul_rn(4.5f, sd));
}

// Scores of TS tokens of one head.  Warp 0 conditions q_h (statistics in the reference's order,
// by lane 0) while the other warps stage the key rows; shared rows use an odd stride, so the
// column-wise reads of the per-token loops are free of bank conflicts.
__global__ void __launch_bounds__(128) ref_scores_kernel(const RefAttnParams p) {
    extern __shared__ float ref_smem[];
    const int d = p.d, ld = d | 1, h = blockIdx.y;
    const int t0 = blockIdx.x * p.ts;
    const int nt = min(p.ts, p.tokens - t0);
    float* qc = ref_smem;
    float* ks = ref_smem + d;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const int lw = nw > 1 ? nw - 1 : 1, w0 = nw > 1 ? 1 : 0;   // loader warps
    if (warp >= w0) {
        for (int r = warp - w0; r < nt; r += lw) {
            const float* src = p.k + ((size_t)(t0 + r) * p.heads + h) * d;
            for (int i = lane; i < d; i += 32) ks[r * ld + i] = __ldg(src + i);
        }
    }
    if (warp == 0 && lane == 0) {
        const float* qh = p.q + (size_t)h * d;
        double mean = 0.0, var = 0.0;
        for (int i = 0; i < d; ++i) mean = __dadd_rn(mean, (double)qh[i]);
        mean = __ddiv_rn(mean, (double)d);
        for (int i = 0; i < d; ++i) {
            const double dd = __dsub_rn((double)qh[i], mean);
            var = __dadd_rn(var, __dmul_rn(dd, dd));
        }
        const float th = threshold_from_var(__ddiv_rn(var, (double)d));
        float prev = 0.f;
        for (int i = 0; i < d; ++i) {
            float v = ref_clip(qh[i], -th, th);
            if (p.module) v = ref_denoise(v, i, prev);
            prev = v;
            qc[i] = v;
        }
    }
    __syncthreads();
    if (tid >= nt) return;
    const float* row = ks + tid * ld;
    double mean = 0.0, var = 0.0;
    for (int i = 0; i < d; ++i) mean = __dadd_rn(mean, (double)row[i]);
    mean = __ddiv_rn(mean, (double)d);
    for (int i = 0; i < d; ++i) {
        const double dd = __dsub_rn((double)row[i], mean);
        var = __dadd_rn(var, __dmul_rn(dd, dd));
    }
    const float th = threshold_from_var(__ddiv_rn(var, (double)d));
    const float inv_sqrt_d = __fdiv_rn(1.0f, __fsqrt_rn((float)d));
    float dot;
    if (!p.module) {
        dot = 0.f;
        for (int i = 0; i < d; ++i) dot = __fadd_rn(dot, __fmul_rn(qc[i], ref_clip(row[i], -th, th)));
    } else {
        double tot = 0.0, tcomp = 0.0;
        float prev = 0.f;
        for (int base = 0; base < d; base += p.block) {
            const int end = min(base + p.block, d);
            // pass 1: the block's largest magnitude; pass 2 replays the reducer from the same state
            const float prev0 = prev;
            float babs = 0.f;
            for (int i = base; i < end; ++i) {
                const float kv = ref_denoise(ref_clip(row[i], -th, th), i, prev);
                prev = kv;
                babs = fmaxf(babs, fmaxf(fabsf(qc[i]), fabsf(kv)));
            }
            const float bs = fmaxf(babs, 1e-6f);
            double lsum = 0.0, lcomp = 0.0;
            prev = prev0;
            for (int i = base; i < end; ++i) {
                const float kv = ref_denoise(ref_clip(row[i], -th, th), i, prev);
                prev = kv;
                ref_kahan(lsum, lcomp, (double)__fmul_rn(__fdiv_rn(qc[i], bs), __fdiv_rn(kv, bs)));
            }
            ref_kahan(tot, tcomp, (double)__fmul_rn(__fmul_rn((float)lsum, bs), bs));
        }
        dot = (float)tot;
    }
    float s;
    if (p.module) s = ref_clip(__fmul_rn(dot, ref_clip(inv_sqrt_d, 1e-4f, 32.f)), -24.f, 24.f);
    else s = __fmul_rn(dot, inv_sqrt_d);
    p.probs[(size_t)h * p.tokens + t0 + tid] = s;
}

// Softmax of one head's scores in place: max, exp, double denominator, probabilities.
__global__ void __launch_bounds__(1024) ref_softmax_kernel(const RefAttnParams p) {
    __shared__ float s_max[32];
    __shared__ double s_den[32];
    const int T = p.tokens, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    float* sc = p.probs + (size_t)blockIdx.x * T;
    float mx = -FLT_MAX;
    for (int t = tid; t < T; t += blockDim.x) mx = fmaxf(mx, sc[t]);
    mx = warp_max(mx);
    if (lane == 0) s_max[warp] = mx;
    __syncthreads();
    mx = s_max[0];
    for (int w = 1; w < nw; ++w) mx = fmaxf(mx, s_max[w]);
    double den = 0.0;
    for (int t = tid; t < T; t += blockDim.x) {
        const float ex = expf(__fsub_rn(sc[t], mx));
        sc[t] = ex;
        den = __dadd_rn(den, (double)ex);
    }
    for (int off = 16; off > 0; off >>= 1) den = __dadd_rn(den, __shfl_xor_sync(0xffffffffu, den, off));
    if (lane == 0) s_den[warp] = den;
    __syncthreads();
    den = 0.0;
    for (int w = 0; w < nw; ++w) den = __dadd_rn(den, s_den[w]);
    if (den < (double)1e-12f) {
        const float uni = __fdiv_rn(1.0f, (float)T);
        for (int t = tid; t < T; t += blockDim.x) sc[t] = uni;
    } else {
        const float inv = __fdiv_rn(1.0f, (float)den);
        for (int t = tid; t < T; t += blockDim.x) sc[t] = __fmul_rn(sc[t], inv);
    }
}

// Partial output sums of one token chunk of one head, one dimension per thread.
__global__ void __launch_bounds__(kRefOutThreads) ref_output_kernel(const RefAttnParams p) {
    extern __shared__ float ref_probs[];
    const int h = blockIdx.y, c = blockIdx.x, d = p.d;
    const int t0 = c * p.tc, nt = min(p.tc, p.tokens - t0);
    const float* pr = p.probs + (size_t)h * p.tokens + t0;
    for (int t = threadIdx.x; t < nt; t += blockDim.x) ref_probs[t] = pr[t];
    __syncthreads();
    const size_t vstride = (size_t)p.heads * d;
    for (int x = threadIdx.x; x < d; x += blockDim.x) {
        const float* vp = p.v + ((size_t)t0 * p.heads + h) * d + x;
        double sum = 0.0, comp = 0.0;
        for (int t = 0; t < nt; ++t) {
            const double val = (double)__fmul_rn(ref_probs[t], __ldg(vp + (size_t)t * vstride));
            if (p.module) ref_kahan(sum, comp, val);
            else sum = __dadd_rn(sum, val);
        }
        double* dst = p.part + (((size_t)c * p.heads + h) * d + x) * 2;
        dst[0] = sum;
        dst[1] = comp;
    }
}

// Chunk partials added in chunk order; a Kahan partial stands for sum - compensation.
__global__ void __launch_bounds__(kRefOutThreads) ref_combine_kernel(const RefAttnParams p) {
    const int h = blockIdx.x, d = p.d;
    for (int x = threadIdx.x; x < d; x += blockDim.x) {
        double sum = 0.0, comp = 0.0;
        for (int c = 0; c < p.chunks; ++c) {
            const double* src = p.part + (((size_t)c * p.heads + h) * d + x) * 2;
            if (p.module) {
                ref_kahan(sum, comp, src[0]);
                ref_kahan(sum, comp, -src[1]);
            } else {
                sum = __dadd_rn(sum, src[0]);
            }
        }
        p.out[(size_t)h * d + x] = (float)sum;
    }
}

// ---- host side ----
struct RefAttnPlan {
    int ts, tc, chunks;
    size_t probs_bytes, part_bytes, smem_scores, smem_output;
};

static size_t round256(size_t b) { return (b + 255u) & ~(size_t)255u; }

static RefAttnPlan ref_plan(size_t tokens, size_t heads, size_t d) {
    RefAttnPlan pl;
    const size_t ld = d | 1u;
    pl.ts = 128;
    while (pl.ts > 32 && (d + (size_t)pl.ts * ld) * sizeof(float) > kRefStageBytes) pl.ts >>= 1;
    // output chunks: about two CTAs per SM over all heads, chunks a multiple of 32 tokens
    const size_t want = (296 + heads - 1) / heads;
    size_t chunks = (tokens + 31) / 32;
    if (chunks > want) chunks = want;
    if (chunks < 1) chunks = 1;
    size_t tc = (tokens + chunks - 1) / chunks;
    tc = (tc + 31) & ~(size_t)31;
    if (tc > 8192) tc = 8192;
    pl.tc = (int)tc;
    pl.chunks = (int)((tokens + tc - 1) / tc);
    pl.probs_bytes = round256(heads * tokens * sizeof(float));
    pl.part_bytes = round256((size_t)pl.chunks * heads * d * 2 * sizeof(double));
    pl.smem_scores = (d + (size_t)pl.ts * ld) * sizeof(float);
    pl.smem_output = tc * sizeof(float);
    return pl;
}

// The reference's switch (three_bit_runtime_modules.c:18-24, 60-66), read per call like it.
static int three_bit_module_from_env() {
    const char* fb = getenv("VSPEC_FUSED_BITS");
    if (fb && fb[0] == '3' && fb[1] == '\0') return 1;
    const char* m = getenv("VSPEC_3BIT_RUNTIME_MODULE");
    if (!m || !m[0]) return 0;
    return (m[0] == '1' || m[0] == 'y' || m[0] == 'Y' || m[0] == 't' || m[0] == 'T') ? 1 : 0;
}

// VSPEC_3BIT_BLOCK_SIZE: 32 or 64, anything else 64 (three_bit_runtime_modules.c:41-58, 105).
static int three_bit_block_from_env() {
    const char* b = getenv("VSPEC_3BIT_BLOCK_SIZE");
    if (!b || !b[0]) return 64;
    const int v = atoi(b);
    return v == 32 ? 32 : 64;
}

static bool ref_args_ok(size_t tokens, size_t heads, size_t d) {
    return tokens > 0 && heads > 0 && d > 0 && d <= (size_t)kRefMaxHeadDim && heads <= 65535 &&
           tokens * heads <= (size_t)INT32_MAX;
}

}  // namespace vb200

using namespace vb200;

extern "C" size_t vspec_b200_attention_ref_workspace_bytes(size_t tokens, size_t heads, size_t head_dim) {
    if (!ref_args_ok(tokens, heads, head_dim)) return 0;
    const RefAttnPlan pl = ref_plan(tokens, heads, head_dim);
    return pl.probs_bytes + pl.part_bytes;
}

extern "C" int vspec_b200_attention_ref_f32(const float* d_q, const float* d_keys, const float* d_values,
                                            size_t tokens, size_t heads, size_t head_dim, int three_bit_module,
                                            size_t block_size, void* d_workspace, size_t workspace_bytes,
                                            float* d_out, void* stream) {
    if (!d_q || !d_keys || !d_values || !d_out || !d_workspace || !ref_args_ok(tokens, heads, head_dim) ||
        (block_size != 0 && block_size != 32 && block_size != 64) || ((uintptr_t)d_workspace & 255u)) {
        set_error("vspec_b200_attention_ref_f32: bad arguments (head_dim <= %d, block 0/32/64, workspace "
                  "256-byte aligned)", kRefMaxHeadDim);
        return VSPEC_B200_ERR_ARG;
    }
    const RefAttnPlan pl = ref_plan(tokens, heads, head_dim);
    if (workspace_bytes < pl.probs_bytes + pl.part_bytes) {
        set_error("vspec_b200_attention_ref_f32: workspace %zu bytes < %zu", workspace_bytes,
                  pl.probs_bytes + pl.part_bytes);
        return VSPEC_B200_ERR_ARG;
    }
    static int smem_set[64];
    int dev = 0;
    VB_CHECK_CUDA(cudaGetDevice(&dev));
    if (dev >= 0 && dev < 64 && !smem_set[dev]) {
        VB_CHECK_CUDA(cudaFuncSetAttribute(ref_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)kRefStageBytes));
        VB_CHECK_CUDA(cudaFuncSetAttribute(ref_output_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)(8192 * sizeof(float))));
        smem_set[dev] = 1;
    }
    RefAttnParams p;
    p.q = d_q;
    p.k = d_keys;
    p.v = d_values;
    p.out = d_out;
    p.probs = (float*)d_workspace;
    p.part = (double*)((char*)d_workspace + pl.probs_bytes);
    p.tokens = (int)tokens;
    p.heads = (int)heads;
    p.d = (int)head_dim;
    p.module = three_bit_module < 0 ? three_bit_module_from_env() : (three_bit_module ? 1 : 0);
    p.block = block_size ? (int)block_size : three_bit_block_from_env();
    p.ts = pl.ts;
    p.tc = pl.tc;
    p.chunks = pl.chunks;
    cudaStream_t st = (cudaStream_t)stream;
    ref_scores_kernel<<<dim3((unsigned)((tokens + pl.ts - 1) / pl.ts), (unsigned)heads), pl.ts, pl.smem_scores, st>>>(p);
    ref_softmax_kernel<<<(unsigned)heads, 1024, 0, st>>>(p);
    ref_output_kernel<<<dim3((unsigned)pl.chunks, (unsigned)heads), kRefOutThreads, pl.smem_output, st>>>(p);
    ref_combine_kernel<<<(unsigned)heads, kRefOutThreads, 0, st>>>(p);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? VSPEC_B200_OK : cuda_status(e, "attention_ref launch");
}
