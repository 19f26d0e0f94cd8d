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
// Two launches after a counter reset, sized to fill the SMs rather than one CTA per head:
//   ref_scores_kernel (tokens/TS x heads)  a CTA stages TS key rows of one head in shared memory
//                                          (cp.async, 16-byte chunks XOR-swizzled by row); thread t
//                                          conditions row t and runs its dot in the reference's
//                                          element order; the last CTA of a head turns the head's
//                                          scores into probabilities (max, exp, double denominator);
//   ref_output_kernel (chunks x heads)     a CTA stages a token chunk of V (cp.async), one thread per
//                                          dimension sums p_t * v_t[x] in token order in double (or
//                                          Kahan); the last CTA of a head adds the chunk partials in
//                                          chunk order.
// Heads whose head_dim is not a multiple of 32, or unaligned buffers, take plain loads instead of
// the staged copies.  Arithmetic uses IEEE operations without contraction (__fmul_rn/__fadd_rn/
// __dmul_rn/__dadd_rn), and each per-token dot runs in the reference's element order, so it
// rounds as the reference's SSE code does.  Sums the reference keeps in double run as parallel
// partials here (row statistics in four interleaved partials, the softmax denominator as a tree,
// the output over token chunks and four interleaved partials), which moves only double roundings
// (a few 1e-16 relative) before the rounding to float; expf is CUDA's (within 2 ulp) where the
// reference calls the C library's.
#include "common.cuh"

#include <float.h>
#include <stdint.h>
#include <stdlib.h>

#include "vspec_b200.h"

namespace vb200 {

constexpr int kRefMaxHeadDim = 1024;
constexpr int kRefOutThreads = 128;
constexpr size_t kRefStageBytes = 200u << 10;   // key tile of one scores CTA
constexpr size_t kRefVTileBytes = 96u << 10;    // value tile of one output CTA

struct RefAttnParams {
    const float* q;       // [heads][d]
    const float* k;       // [tokens][heads][d]
    const float* v;
    float* out;           // [heads][d]
    float* probs;         // [heads][tokens] (workspace): scores, then probabilities
    double* part;         // [chunks][heads][d][2] (workspace): sum, compensation
    unsigned* counters;   // [2][heads] (workspace, zeroed per call): CTAs done per head
    int tokens, heads, d;
    int module;           // 3-bit runtime module on
    int block;            // module dot block: 32 or 64
    int vec;              // d % 32 == 0 and q, k, v 16-byte aligned: staged 16-byte copies
    int ts;               // tokens per scores CTA (= its threads)
    int tc;               // tokens per output chunk
    int chunks;
};

__device__ __forceinline__ void ar_cp16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void ar_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void ar_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }
__device__ __forceinline__ uint32_t ar_smem(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

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

// Population statistics of a row as the clamp threshold: mean and variance summed in double, in
// four interleaved partials (element i into partial i % 4, combined as (p0 + p1) + (p2 + p3)), so
// four addition chains run side by side; the reference sums in one chain, which moves only double
// roundings, far below the float rounding of the threshold.
template <bool EXACT4, class Get4>
__device__ __forceinline__ float row_threshold(int d, Get4 get4) {
    const int nc = (d + 3) >> 2;
    double m[4] = {0.0, 0.0, 0.0, 0.0};
    for (int c = 0; c < nc; ++c) {
        const float4 x = get4(c);
        const float e[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (EXACT4 || 4 * c + u < d) m[u] = __dadd_rn(m[u], (double)e[u]);
    }
    const double mean = __ddiv_rn(__dadd_rn(__dadd_rn(m[0], m[1]), __dadd_rn(m[2], m[3])), (double)d);
    double v[4] = {0.0, 0.0, 0.0, 0.0};
    for (int c = 0; c < nc; ++c) {
        const float4 x = get4(c);
        const float e[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            if (EXACT4 || 4 * c + u < d) {
                const double dd = __dsub_rn((double)e[u], mean);
                v[u] = __dadd_rn(v[u], __dmul_rn(dd, dd));
            }
        }
    }
    return threshold_from_var(__ddiv_rn(__dadd_rn(__dadd_rn(v[0], v[1]), __dadd_rn(v[2], v[3])), (double)d));
}

// Sum over the warp in a fixed order (down the lanes), lane 0's value given to every lane.
__device__ __forceinline__ double warp_sum_bcast(double v) {
    for (int off = 16; off > 0; off >>= 1) v = __dadd_rn(v, __shfl_down_sync(0xffffffffu, v, off));
    return __shfl_sync(0xffffffffu, v, 0);
}

// q_h conditioned in shared memory by one warp: statistics as warp sums in double, the clamp per
// element, then (module) the noise reducer, which is sequential, by lane 0.
__device__ void condition_q_warp(float* qc, int d, int module) {
    const int lane = threadIdx.x & 31;
    double m = 0.0;
    for (int i = lane; i < d; i += 32) m = __dadd_rn(m, (double)qc[i]);
    const double mean = __ddiv_rn(warp_sum_bcast(m), (double)d);
    double v = 0.0;
    for (int i = lane; i < d; i += 32) {
        const double dd = __dsub_rn((double)qc[i], mean);
        v = __dadd_rn(v, __dmul_rn(dd, dd));
    }
    const float th = threshold_from_var(__ddiv_rn(warp_sum_bcast(v), (double)d));
    for (int i = lane; i < d; i += 32) qc[i] = ref_clip(qc[i], -th, th);
    __syncwarp();
    if (module && lane == 0) {
        float prev = 0.f;
        for (int i = 0; i < d; ++i) {
            const float x = ref_denoise(qc[i], i, prev);
            prev = x;
            qc[i] = x;
        }
    }
}

// Score of one key row read as 4-element chunks (get4(c) = elements 4c .. 4c+3; past d unused):
// clamp threshold, then the dot in the reference's element order (plain, or the module's
// block-normalised Kahan dot), scale.
template <bool EXACT4, class Get4>
__device__ __forceinline__ float row_score(const RefAttnParams& p, const float* qc, Get4 get4) {
    const int d = p.d, nc = (d + 3) >> 2;
    const float th = row_threshold<EXACT4>(d, get4);
    const float inv_sqrt_d = __fdiv_rn(1.0f, __fsqrt_rn((float)d));
    if (!p.module) {
        float dot = 0.f;
        for (int c = 0; c < nc; ++c) {
            const float4 x = get4(c);
            const float e[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (EXACT4 || 4 * c + u < d) dot = __fadd_rn(dot, __fmul_rn(qc[4 * c + u], ref_clip(e[u], -th, th)));
        }
        return __fmul_rn(dot, inv_sqrt_d);
    }
    double tot = 0.0, tcomp = 0.0;
    float prev = 0.f;
    for (int base = 0; base < d; base += p.block) {   // block of 32 or 64: whole chunks
        const int end = min(base + p.block, d);
        // pass 1: the block's largest magnitude; pass 2 replays the reducer from the same state
        const float prev0 = prev;
        float babs = 0.f;
        for (int c = base >> 2; 4 * c < end; ++c) {
            const float4 x = get4(c);
            const float e[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = 4 * c + u;
                if (i < end) {
                    const float kv = ref_denoise(ref_clip(e[u], -th, th), i, prev);
                    prev = kv;
                    babs = fmaxf(babs, fmaxf(fabsf(qc[i]), fabsf(kv)));
                }
            }
        }
        const float bs = fmaxf(babs, 1e-6f);
        double lsum = 0.0, lcomp = 0.0;
        prev = prev0;
        for (int c = base >> 2; 4 * c < end; ++c) {
            const float4 x = get4(c);
            const float e[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = 4 * c + u;
                if (i < end) {
                    const float kv = ref_denoise(ref_clip(e[u], -th, th), i, prev);
                    prev = kv;
                    ref_kahan(lsum, lcomp, (double)__fmul_rn(__fdiv_rn(qc[i], bs), __fdiv_rn(kv, bs)));
                }
            }
        }
        ref_kahan(tot, tcomp, (double)__fmul_rn(__fmul_rn((float)lsum, bs), bs));
    }
    return ref_clip(__fmul_rn((float)tot, ref_clip(inv_sqrt_d, 1e-4f, 32.f)), -24.f, 24.f);
}

// One head's scores -> probabilities in place, by the CTA that finished the head last: max, exp,
// double denominator (uniform below 1e-12, as the reference), probabilities.  The scores are
// first copied into `buf` (cap floats of this CTA's idle key tile) in one round of 16-byte
// copies, or read with eight loads in flight when they do not fit or are not 16-byte aligned.
__device__ void head_softmax(const RefAttnParams& p, int h, float* buf, int cap, float* s_red, double* s_dred) {
    const int T = p.tokens, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const int nth = blockDim.x;
    float* sc = p.probs + (size_t)h * T;
    const bool staged = T <= cap && ((T & 3) == 0);   // row h starts 16-byte aligned when T % 4 == 0
    if (staged) {
        for (int c = tid; c < (T >> 2); c += nth) ar_cp16(ar_smem(buf + 4 * c), sc + 4 * c);
        ar_commit();
        ar_wait<0>();
        __syncthreads();
    }
    auto ld = [&](int t) { return staged ? buf[t] : __ldcg(sc + t); };
    float mx = -FLT_MAX;
    for (int tb = tid; tb < T; tb += 8 * nth) {
        float r[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) r[u] = tb + u * nth < T ? ld(tb + u * nth) : -FLT_MAX;
#pragma unroll
        for (int u = 0; u < 8; ++u) mx = fmaxf(mx, r[u]);
    }
    mx = warp_max(mx);
    if (lane == 0) s_red[warp] = mx;
    __syncthreads();
    mx = s_red[0];
    for (int w = 1; w < nw; ++w) mx = fmaxf(mx, s_red[w]);
    double den = 0.0;
    for (int tb = tid; tb < T; tb += 8 * nth) {
        float r[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) r[u] = tb + u * nth < T ? ld(tb + u * nth) : 0.f;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int t = tb + u * nth;
            if (t < T) {
                const float ex = expf(__fsub_rn(r[u], mx));
                if (staged) buf[t] = ex;
                else sc[t] = ex;
                den = __dadd_rn(den, (double)ex);
            }
        }
    }
    for (int off = 16; off > 0; off >>= 1) den = __dadd_rn(den, __shfl_xor_sync(0xffffffffu, den, off));
    if (lane == 0) s_dred[warp] = den;
    __syncthreads();
    den = 0.0;
    for (int w = 0; w < nw; ++w) den = __dadd_rn(den, s_dred[w]);
    const bool uniform = den < (double)1e-12f;
    const float uni = __fdiv_rn(1.0f, (float)T);
    const float inv = uniform ? 0.f : __fdiv_rn(1.0f, (float)den);
    // each thread rescales the elements it wrote itself
    for (int t = tid; t < T; t += nth) sc[t] = uniform ? uni : __fmul_rn(staged ? buf[t] : sc[t], inv);
}

// True in every thread of the CTA that is the last of `total` CTAs to reach this point for
// counter `ctr`; everything the CTA wrote before is visible to that one.
__device__ __forceinline__ bool last_cta(unsigned* ctr, unsigned total) {
    __shared__ int s_last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(ctr, 1u) == total - 1u;
    __syncthreads();
    const bool last = s_last != 0;
    if (last) __threadfence();
    return last;
}

// Scores of TS tokens of one head.  VEC: q_h and the key rows arrive by cp.async (the rows in
// 16-byte chunks placed at chunk c ^ (row & 7), so the float4 reads of eight consecutive rows hit
// distinct bank groups); warp 0 conditions q_h while the key tile is in flight.  Otherwise
// plain loads into rows of odd stride.
template <bool VEC>
__global__ void __launch_bounds__(128) ref_scores_kernel(const RefAttnParams p) {
    extern __shared__ __align__(16) float ref_smem[];
    __shared__ float s_red[32];
    __shared__ double s_dred[32];
    const int d = p.d, h = blockIdx.y, t0 = blockIdx.x * p.ts;
    const int nt = min(p.ts, p.tokens - t0);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    float* qc = ref_smem;
    float* ks = ref_smem + ((d + 3) & ~3);
    const float* qh = p.q + (size_t)h * d;
    const float* kh = p.k + ((size_t)t0 * p.heads + h) * d;
    const size_t kstride = (size_t)p.heads * d;
    if (VEC) {
        const int dq = d >> 2;
        if (warp == 0)
            for (int c = lane; c < dq; c += 32) ar_cp16(ar_smem(qc + 4 * c), qh + 4 * c);
        ar_commit();
        for (int r = warp; r < nt; r += nw)   // a warp per row, lanes over its 16-byte chunks
            for (int c = lane; c < dq; c += 32)
                ar_cp16(ar_smem(ks + r * d + 4 * (c ^ (r & 7))), kh + (size_t)r * kstride + 4 * c);
        ar_commit();
        if (warp == 0) {
            ar_wait<1>();
            __syncwarp();
            condition_q_warp(qc, d, p.module);
        }
        ar_wait<0>();
    } else {
        const int ld = d | 1;
        if (warp == 0) {
            for (int i = lane; i < d; i += 32) qc[i] = __ldg(qh + i);
            __syncwarp();
            condition_q_warp(qc, d, p.module);
        }
        if (warp >= (nw > 1 ? 1 : 0)) {   // loader warps: eight loads in flight per thread
            const int w0 = nw > 1 ? 1 : 0, nl = (nw - w0) * 32, me = tid - w0 * 32, total = nt * d;
            for (int base = me; base < total; base += 8 * nl) {
                float r[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int e = base + u * nl, row = e / d;
                    r[u] = e < total ? __ldg(kh + (size_t)row * kstride + (e - row * d)) : 0.f;
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int e = base + u * nl, row = e / d;
                    if (e < total) ks[row * ld + (e - row * d)] = r[u];
                }
            }
        }
    }
    __syncthreads();
    if (tid < nt) {
        float s;
        if (VEC) {
            const float4* row = reinterpret_cast<const float4*>(ks + tid * d);
            const int sw = tid & 7;
            s = row_score<true>(p, qc, [&](int c) { return row[c ^ sw]; });
        } else {
            const float* row = ks + tid * (d | 1);
            s = row_score<false>(p, qc, [&](int c) {
                const int i = 4 * c;
                return make_float4(row[i], i + 1 < d ? row[i + 1] : 0.f, i + 2 < d ? row[i + 2] : 0.f,
                                   i + 3 < d ? row[i + 3] : 0.f);
            });
        }
        p.probs[(size_t)h * p.tokens + t0 + tid] = s;
    }
    if (last_cta(&p.counters[h], gridDim.x)) {
        __syncthreads();   // the key tile is free: it holds the head's scores
        const int cap = p.ts * (d | 1) & ~3;
        head_softmax(p, h, ks, cap, s_red, s_dred);
    }
}

// Partial output sums of one token chunk of one head, one dimension per thread, tokens in order;
// the CTA that finishes the head last adds the chunk partials in chunk order (a Kahan partial
// stands for sum - compensation).
template <bool VEC>
__global__ void __launch_bounds__(kRefOutThreads) ref_output_kernel(const RefAttnParams p) {
    extern __shared__ __align__(16) float ref_osmem[];
    const int h = blockIdx.y, c = blockIdx.x, d = p.d;
    const int t0 = c * p.tc, nt = min(p.tc, p.tokens - t0);
    float* pr = ref_osmem;                          // [tc] probabilities
    float* vt = ref_osmem + ((p.tc + 3) & ~3);      // [tc][d] values (VEC)
    const float* vh = p.v + ((size_t)t0 * p.heads + h) * d;
    const size_t vstride = (size_t)p.heads * d;
    if (VEC) {
        const int dq = d >> 2;
        const int lane = threadIdx.x & 31, nw = blockDim.x >> 5;
        for (int r = threadIdx.x >> 5; r < nt; r += nw)   // a warp per row, lanes over its chunks
            for (int cc = lane; cc < dq; cc += 32)
                ar_cp16(ar_smem(vt + r * d + 4 * cc), vh + (size_t)r * vstride + 4 * cc);
        ar_commit();
    }
    for (int t = threadIdx.x; t < nt; t += blockDim.x) pr[t] = __ldcg(p.probs + (size_t)h * p.tokens + t0 + t);
    if (VEC) ar_wait<0>();
    __syncthreads();
    for (int x = threadIdx.x; x < d; x += blockDim.x) {
        double sum = 0.0, comp = 0.0;
        if (VEC) {   // four interleaved partials (token t into t % 4), added in order at the end
            double ps[4] = {0.0, 0.0, 0.0, 0.0}, pc[4] = {0.0, 0.0, 0.0, 0.0};
            int t = 0;
            for (; t + 4 <= nt; t += 4) {
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const double val = (double)__fmul_rn(pr[t + u], vt[(t + u) * d + x]);
                    if (p.module) ref_kahan(ps[u], pc[u], val);
                    else ps[u] = __dadd_rn(ps[u], val);
                }
            }
#pragma unroll
            for (int u = 0; u < 3; ++u) {
                if (t + u < nt) {
                    const double val = (double)__fmul_rn(pr[t + u], vt[(t + u) * d + x]);
                    if (p.module) ref_kahan(ps[u], pc[u], val);
                    else ps[u] = __dadd_rn(ps[u], val);
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (p.module) {
                    ref_kahan(sum, comp, ps[u]);
                    ref_kahan(sum, comp, -pc[u]);
                } else {
                    sum = __dadd_rn(sum, ps[u]);
                }
            }
        } else {
            const float* vp = vh + x;
            for (int tb = 0; tb < nt; tb += 16) {   // sixteen loads in flight, then the sums in order
                float r[16];
#pragma unroll
                for (int u = 0; u < 16; ++u) r[u] = tb + u < nt ? __ldg(vp + (size_t)(tb + u) * vstride) : 0.f;
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    if (tb + u >= nt) break;
                    const double val = (double)__fmul_rn(pr[tb + u], r[u]);
                    if (p.module) ref_kahan(sum, comp, val);
                    else sum = __dadd_rn(sum, val);
                }
            }
        }
        reinterpret_cast<double2*>(p.part)[((size_t)c * p.heads + h) * d + x] = make_double2(sum, comp);
    }
    if (!last_cta(&p.counters[p.heads + h], gridDim.x)) return;
    const size_t cstride = (size_t)p.heads * d;
    for (int x = threadIdx.x; x < d; x += blockDim.x) {
        double sum = 0.0, comp = 0.0;
        const double2* src = reinterpret_cast<const double2*>(p.part) + (size_t)h * d + x;
        for (int cb = 0; cb < p.chunks; cb += 8) {   // eight partials in flight, added in chunk order
            double2 r[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                r[u] = cb + u < p.chunks ? __ldcg(src + (size_t)(cb + u) * cstride) : make_double2(0.0, 0.0);
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                if (cb + u >= p.chunks) break;
                if (p.module) {
                    ref_kahan(sum, comp, r[u].x);
                    ref_kahan(sum, comp, -r[u].y);
                } else {
                    sum = __dadd_rn(sum, r[u].x);
                }
            }
        }
        p.out[(size_t)h * d + x] = (float)sum;
    }
}

// ---- host side ----
struct RefAttnPlan {
    int ts, tc, chunks;
    size_t probs_bytes, part_bytes, counter_bytes, smem_scores, smem_output;
};

static size_t round256(size_t b) { return (b + 255u) & ~(size_t)255u; }

static RefAttnPlan ref_plan(size_t tokens, size_t heads, size_t d) {
    RefAttnPlan pl;
    const size_t qpad = (d + 3) & ~(size_t)3;
    // scores CTA: TS key rows (the plain-load layout, stride d | 1, is the larger one)
    pl.ts = 128;
    while (pl.ts > 32 && (qpad + (size_t)pl.ts * (d | 1u)) * sizeof(float) > kRefStageBytes) pl.ts >>= 1;
    // output chunks: about two CTAs per SM over all heads, a multiple of 8 tokens, the value tile
    // within its budget
    size_t cap = (kRefVTileBytes / sizeof(float)) / (d + 1);
    cap = cap < 8 ? 8 : (cap > 8192 ? 8192 : cap & ~(size_t)7);
    const size_t want = (296 + heads - 1) / heads;
    size_t chunks = (tokens + 7) / 8;
    if (chunks > want) chunks = want;
    if (chunks < 1) chunks = 1;
    size_t tc = (tokens + chunks - 1) / chunks;
    tc = (tc + 7) & ~(size_t)7;
    if (tc > cap) tc = cap;
    pl.tc = (int)tc;
    pl.chunks = (int)((tokens + tc - 1) / tc);
    pl.probs_bytes = round256(heads * tokens * sizeof(float));
    pl.part_bytes = round256((size_t)pl.chunks * heads * d * 2 * sizeof(double));
    pl.counter_bytes = round256(2 * heads * sizeof(unsigned));
    pl.smem_scores = (qpad + (size_t)pl.ts * (d | 1u)) * sizeof(float);
    pl.smem_output = (((tc + 3) & ~(size_t)3) + tc * d) * sizeof(float);
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
    return pl.probs_bytes + pl.part_bytes + pl.counter_bytes;
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
    const size_t need = pl.probs_bytes + pl.part_bytes + pl.counter_bytes;
    if (workspace_bytes < need) {
        set_error("vspec_b200_attention_ref_f32: workspace %zu bytes < %zu", workspace_bytes, need);
        return VSPEC_B200_ERR_ARG;
    }
    static int smem_set[64];
    int dev = 0;
    VB_CHECK_CUDA(cudaGetDevice(&dev));
    if (dev >= 0 && dev < 64 && !smem_set[dev]) {
        VB_CHECK_CUDA(cudaFuncSetAttribute(ref_scores_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)kRefStageBytes));
        VB_CHECK_CUDA(cudaFuncSetAttribute(ref_scores_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)kRefStageBytes));
        VB_CHECK_CUDA(cudaFuncSetAttribute(ref_output_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)(kRefVTileBytes + 64 * 1024)));
        VB_CHECK_CUDA(cudaFuncSetAttribute(ref_output_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)(kRefVTileBytes + 64 * 1024)));
        smem_set[dev] = 1;
    }
    RefAttnParams p;
    p.q = d_q;
    p.k = d_keys;
    p.v = d_values;
    p.out = d_out;
    p.probs = (float*)d_workspace;
    p.part = (double*)((char*)d_workspace + pl.probs_bytes);
    p.counters = (unsigned*)((char*)d_workspace + pl.probs_bytes + pl.part_bytes);
    p.tokens = (int)tokens;
    p.heads = (int)heads;
    p.d = (int)head_dim;
    p.module = three_bit_module < 0 ? three_bit_module_from_env() : (three_bit_module ? 1 : 0);
    p.block = block_size ? (int)block_size : three_bit_block_from_env();
    p.vec = (head_dim % 32 == 0) && !(((uintptr_t)d_q | (uintptr_t)d_keys | (uintptr_t)d_values) & 15u);
    p.ts = pl.ts;
    p.tc = pl.tc;
    p.chunks = pl.chunks;
    cudaStream_t st = (cudaStream_t)stream;
    VB_CHECK_CUDA(cudaMemsetAsync(p.counters, 0, 2 * heads * sizeof(unsigned), st));
    const dim3 gs((unsigned)((tokens + pl.ts - 1) / pl.ts), (unsigned)heads), go((unsigned)pl.chunks, (unsigned)heads);
    if (p.vec) {
        ref_scores_kernel<true><<<gs, pl.ts, pl.smem_scores, st>>>(p);
        ref_output_kernel<true><<<go, kRefOutThreads, pl.smem_output, st>>>(p);
    } else {
        ref_scores_kernel<false><<<gs, pl.ts, pl.smem_scores, st>>>(p);
        ref_output_kernel<false><<<go, kRefOutThreads, pl.smem_output, st>>>(p);
    }
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? VSPEC_B200_OK : cuda_status(e, "attention_ref launch");
}
