// attention.cu -- GQA split-K paged decode attention on sm_100a.
//
// One query token per sequence attends over its paged K/V cache:
//   pages   [P][page_tokens][Hkv][d]   (layout of src/attention/kv_paged_cache.c:292-298)
//   table   [B][max_pages]             (a session's pages[] widened to int32)
//   kv_h    = h / (Hq/Hkv)             (Vspec-chat/python/runtime_inference.py:151)
//   out_h   = softmax(q_h . K^T * scale) V   (src/attention/flash_stub.c:7-55)
// Token t of a sequence is slot t % page_tokens of page table[t / page_tokens]:
// every page but the last one is full.
//
// fp16 pages, d = 128 (the decode product path): warp-level tensor-core MMA.
//   QK^T: A = 16 tokens x 16 dims of K straight from the page rows (thread
//         (g,c) streams 64 contiguous bytes per token row), B = 8 columns =
//         4 query heads x {hi, lo} fp16 parts of q -> fp32-accurate scores.
//   PV:   A = V^T (pairs of token rows merged with PRMT), B = p as {hi, lo}
//         fp16 parts (p pre-scaled by 2^14 so no part underflows).
//   Online softmax per warp in fp32; warps merge in shared memory; splits of
//   the context merge in a second kernel (fixed order: deterministic).
// fp32 pages or other head sizes: a plain fp32 SIMT kernel with the same
// split/merge structure.
#include "common.cuh"
#include "attention_kernels.cuh"

#include <math.h>
#include <string.h>

namespace vb200 {

constexpr int kAttnWarps = 4;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kNegBig = -1.0e30f;
constexpr float kPScale = 16384.0f;  // 2^14: keeps p's fp16 hi/lo parts normal

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm volatile("prmt.b32 %0, %1, %2, %3;\n" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    return (uint32_t)__half_as_ushort(__float2half_rn(lo)) | ((uint32_t)__half_as_ushort(__float2half_rn(hi)) << 16);
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

__device__ __forceinline__ uint32_t u4_word(const uint4& v, int w) {
    return w == 0 ? v.x : (w == 1 ? v.y : (w == 2 ? v.z : v.w));
}

// Set when a page table entry lies outside [0, num_pages): the access is
// redirected to page 0 and the host reads the flag back
// (vspec_b200_paged_attention_page_fault).
__device__ int g_attn_page_fault = 0;

// Address of token t's row for kv head kvh (element offset into the pool).
__device__ __forceinline__ size_t token_row(const int32_t* table, int t, int pt, int hkv, int d, int kvh,
                                            int num_pages) {
    int page = __ldg(table + t / pt);
    if (page < 0 || page >= num_pages) {
        atomicOr(&g_attn_page_fault, 1);
        page = 0;
    }
    return ((size_t)page * pt + (size_t)(t % pt)) * (size_t)hkv * d + (size_t)kvh * d;
}

// ---------------------------------------------------------------------------
// Tensor-core kernel: fp16 pages, d = 128, up to 4 query heads per CTA.
// grid = (splits, Hkv * head_groups, B)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kAttnThreads)
paged_attn_f16_mma_kernel(const AttnParams p) {
    pdl_wait();
    pdl_trigger();
    constexpr int D = 128;
    const int split = blockIdx.x;
    const int kvh = blockIdx.y / p.head_groups;
    const int hg = blockIdx.y % p.head_groups;
    const int b = blockIdx.z;
    const int group = p.hq / p.hkv;
    const int ctx = p.ctx_len[b];
    const int t_begin = split * p.split_tokens;
    if (t_begin >= ctx) return;
    const int t_end = min(ctx, t_begin + p.split_tokens);
    const int nsplit = (ctx + p.split_tokens - 1) / p.split_tokens;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, c = lane & 3;
    const int32_t* table = p.page_table + (size_t)b * p.max_pages;
    const __half* kp = reinterpret_cast<const __half*>(p.k_pages);
    const __half* vp = reinterpret_cast<const __half*>(p.v_pages);

    __shared__ float sm_q[4][D];                  // the CTA's (up to) 4 query heads, fp32
    __shared__ float sm_qmax[4];
    __shared__ float sm_p[kAttnWarps][16][4];     // p exchange, per warp
    __shared__ float sm_ml[kAttnWarps][4][2];     // per-warp (m, l) per head
    __shared__ float sm_o[kAttnWarps][4][D];      // per-warp unnormalized O per head

    // ---- q: load, per-head power-of-two rescale, hi/lo B fragments ----
    for (int i = tid; i < 4 * D; i += kAttnThreads) {
        const int hl = i / D, dd = i % D;
        const int h = hg * 4 + hl;
        sm_q[hl][dd] = (hl < 4 && h < group) ? p.q[((size_t)b * p.hq + (size_t)kvh * group + h) * D + dd] : 0.f;
    }
    __syncthreads();
    if (warp == 0) {
        for (int hl = 0; hl < 4; ++hl) {
            float mx = 0.f;
            for (int dd = lane; dd < D; dd += 32) mx = fmaxf(mx, fabsf(sm_q[hl][dd]));
            mx = warp_max(mx);
            if (lane == 0) {
                int ex = 0;
                if (mx > 0.f && isfinite(mx)) { (void)frexpf(mx, &ex); ex -= 14; }
                sm_qmax[hl] = (float)ex;   // exponent of the rescale
            }
        }
    }
    __syncthreads();
    // B fragment for k-step j: column g (head g/2, part g%2), k-slots of thread c
    // map to dims 8c + 32(j/2) + 4(j%2) + {0,1,2,3}.
    uint32_t qf[8][2];
    {
        const int hl = g >> 1;
        const bool lo = (g & 1) != 0;
        const float sc = ldexpf(1.0f, -(int)sm_qmax[hl]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int base = 8 * c + 32 * (j >> 1) + 4 * (j & 1);
            float v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                float x = sm_q[hl][base + u] * sc;
                if (lo) x = x - __half2float(__float2half_rn(x));
                v[u] = x;
            }
            qf[j][0] = pack_half2(v[0], v[1]);
            qf[j][1] = pack_half2(v[2], v[3]);
        }
    }
    // per-head score multiplier: 2^e * scale * log2(e) (exp2-domain scores)
    const float score_mul = ldexpf(p.scale * kLog2e, (int)sm_qmax[c]);

    float m_run = kNegBig, l_run = 0.f;     // head c of this thread
    float oacc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) oacc[i][0] = oacc[i][1] = oacc[i][2] = oacc[i][3] = 0.f;

    const int ntiles = (t_end - t_begin + 15) / 16;
    for (int tile = warp; tile < ntiles; tile += kAttnWarps) {
        const int t0 = t_begin + tile * 16;
        // ---- K rows g and g+8: 4 x 16 bytes each at dims 8c + 32i ----
        uint4 kr[2][4];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int t = t0 + g + 8 * r;
            if (t < t_end) {
                const __half* row = kp + token_row(table, t, p.page_tokens, p.hkv, D, kvh, p.num_pages);
#pragma unroll
                for (int i = 0; i < 4; ++i) kr[r][i] = ldg_nc_v4(row + 8 * c + 32 * i);
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) kr[r][i] = make_uint4(0u, 0u, 0u, 0u);
            }
        }
        // ---- V rows 4c..4c+3: dims [16g, 16g+16) ----
        uint4 vr[4][2];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int t = t0 + 4 * c + r;
            if (t < t_end) {
                const __half* row = vp + token_row(table, t, p.page_tokens, p.hkv, D, kvh, p.num_pages);
                vr[r][0] = ldg_nc_v4(row + 16 * g);
                vr[r][1] = ldg_nc_v4(row + 16 * g + 8);
            } else {
                vr[r][0] = vr[r][1] = make_uint4(0u, 0u, 0u, 0u);
            }
        }
        // ---- S = K Q^T over 8 k-steps of 16 dims ----
        float s[4] = {0.f, 0.f, 0.f, 0.f};
        const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = j >> 1, sub = j & 1;
            const uint32_t a[4] = {u4_word(kr[0][i], 2 * sub), u4_word(kr[1][i], 2 * sub),
                                   u4_word(kr[0][i], 2 * sub + 1), u4_word(kr[1][i], 2 * sub + 1)};
            mma_16816_f16(s, a, qf[j][0], qf[j][1], j == 0 ? zero4 : s);
        }
        // scores of tokens g and g+8 for head c (hi + lo columns), exp2 domain
        const bool v0 = (t0 + g) < t_end, v1 = (t0 + g + 8) < t_end;
        float sc0 = v0 ? (s[0] + s[1]) * score_mul : kNegBig;
        float sc1 = v1 ? (s[2] + s[3]) * score_mul : kNegBig;
        float tmax = fmaxf(sc0, sc1);
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 4));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 8));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 16));
        const float m_new = fmaxf(m_run, tmax);
        const float alpha = exp2f(m_run - m_new);
        const float p0 = v0 ? exp2f(sc0 - m_new) : 0.f;
        const float p1 = v1 ? exp2f(sc1 - m_new) : 0.f;
        l_run = l_run * alpha + (p0 + p1);
        m_run = m_new;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            oacc[i][0] *= alpha; oacc[i][1] *= alpha; oacc[i][2] *= alpha; oacc[i][3] *= alpha;
        }
        // ---- p exchange: thread (g,c) -> P^T B fragment of thread (g', c') ----
        sm_p[warp][g][c] = p0 * kPScale;
        sm_p[warp][g + 8][c] = p1 * kPScale;
        __syncwarp();
        uint32_t pb0, pb1;
        {
            const int hl = g >> 1;
            const bool lo = (g & 1) != 0;
            float pv[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                float x = sm_p[warp][4 * c + r][hl];
                if (lo) x = x - __half2float(__float2half_rn(x));
                pv[r] = x;
            }
            pb0 = pack_half2(pv[0], pv[1]);
            pb1 = pack_half2(pv[2], pv[3]);
        }
        __syncwarp();
        // ---- O^T += V^T P^T over 8 dim blocks ----
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int u = i >> 2, w = i & 3;
            const uint32_t w0 = u4_word(vr[0][u], w), w1 = u4_word(vr[1][u], w);
            const uint32_t w2 = u4_word(vr[2][u], w), w3 = u4_word(vr[3][u], w);
            const uint32_t a[4] = {prmt(w0, w1, 0x5410), prmt(w0, w1, 0x7632), prmt(w2, w3, 0x5410),
                                   prmt(w2, w3, 0x7632)};
            mma_16816_f16(oacc[i], a, pb0, pb1, oacc[i]);
        }
    }

    // ---- merge the warps ----
    // l: sum of the per-thread partials over the 8 lanes of head c
    float l_tot = l_run;
    l_tot += __shfl_xor_sync(0xffffffffu, l_tot, 4);
    l_tot += __shfl_xor_sync(0xffffffffu, l_tot, 8);
    l_tot += __shfl_xor_sync(0xffffffffu, l_tot, 16);
    if (g == 0) {
        sm_ml[warp][c][0] = m_run;
        sm_ml[warp][c][1] = l_tot;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        sm_o[warp][c][16 * g + 2 * i] = (oacc[i][0] + oacc[i][1]) * (1.0f / kPScale);
        sm_o[warp][c][16 * g + 2 * i + 1] = (oacc[i][2] + oacc[i][3]) * (1.0f / kPScale);
    }
    __syncthreads();
    for (int z = tid; z < 4 * D; z += kAttnThreads) {
        const int hl = z / D, dd = z % D;
        const int h_in_group = hg * 4 + hl;
        if (h_in_group >= group) continue;
        float M = kNegBig;
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, sm_ml[w][hl][0]);
        float L = 0.f, O = 0.f;
        for (int w = 0; w < kAttnWarps; ++w) {
            const float f = exp2f(sm_ml[w][hl][0] - M);
            L += sm_ml[w][hl][1] * f;
            O += sm_o[w][hl][dd] * f;
        }
        const int h = kvh * group + h_in_group;
        const size_t bh = (size_t)b * p.hq + h;
        if (nsplit == 1) {
            p.out[bh * D + dd] = O / fmaxf(L, 1e-12f);
        } else {
            p.part_o[(bh * p.max_splits + split) * D + dd] = O;
            if (dd == 0) {
                p.part_ml[(bh * p.max_splits + split) * 2 + 0] = M;
                p.part_ml[(bh * p.max_splits + split) * 2 + 1] = L;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// SIMT fp32 kernel: fp32 or fp16 pages, any d <= 256, one query head per CTA.
// grid = (splits, Hq, B); scores in the natural-exp domain like the reference.
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

template <typename T>
__global__ void __launch_bounds__(kAttnThreads)
paged_attn_simt_kernel(const AttnParams p) {
    pdl_wait();
    pdl_trigger();
    const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int D = p.d;
    const int group = p.hq / p.hkv;
    const int kvh = min(p.hkv - 1, h / (group > 0 ? group : 1));
    const int ctx = p.ctx_len[b];
    const int t_begin = split * p.split_tokens;
    if (t_begin >= ctx) return;
    const int t_end = min(ctx, t_begin + p.split_tokens);
    const int nsplit = (ctx + p.split_tokens - 1) / p.split_tokens;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int32_t* table = p.page_table + (size_t)b * p.max_pages;
    const T* kp = reinterpret_cast<const T*>(p.k_pages);
    const T* vp = reinterpret_cast<const T*>(p.v_pages);
    const float* q = p.q + ((size_t)b * p.hq + h) * D;

    __shared__ float sm_m[kAttnWarps], sm_l[kAttnWarps];
    __shared__ float sm_o[kAttnWarps][256];

    float qr[8], o[8];
    int nd = 0;
    for (int dd = lane; dd < D; dd += 32) { qr[nd] = q[dd]; o[nd] = 0.f; ++nd; }
    float m_run = kNegBig, l_run = 0.f;
    for (int t = t_begin + warp; t < t_end; t += kAttnWarps) {
        const size_t off = token_row(table, t, p.page_tokens, p.hkv, D, kvh, p.num_pages);
        float part = 0.f;
        int i = 0;
        for (int dd = lane; dd < D; dd += 32, ++i) part = fmaf(qr[i], to_f<T>(kp[off + dd]), part);
        const float sc = warp_sum(part) * p.scale;
        const float m_new = fmaxf(m_run, sc);
        const float alpha = expf(m_run - m_new);
        const float pw = expf(sc - m_new);
        l_run = l_run * alpha + pw;
        m_run = m_new;
        i = 0;
        for (int dd = lane; dd < D; dd += 32, ++i) o[i] = fmaf(pw, to_f<T>(vp[off + dd]), o[i] * alpha);
    }
    if (lane == 0) { sm_m[warp] = m_run; sm_l[warp] = l_run; }
    {
        int i = 0;
        for (int dd = lane; dd < D; dd += 32, ++i) sm_o[warp][dd] = o[i];
    }
    __syncthreads();
    for (int dd = tid; dd < D; dd += kAttnThreads) {
        float M = kNegBig;
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, sm_m[w]);
        float L = 0.f, O = 0.f;
        for (int w = 0; w < kAttnWarps; ++w) {
            const float f = expf(sm_m[w] - M);
            L += sm_l[w] * f;
            O += sm_o[w][dd] * f;
        }
        const size_t bh = (size_t)b * p.hq + h;
        if (nsplit == 1) {
            p.out[bh * D + dd] = O / fmaxf(L, 1e-12f);
        } else {
            p.part_o[(bh * p.max_splits + split) * D + dd] = O;
            if (dd == 0) {
                // the combine works in the exp2 domain: store m * log2(e)
                p.part_ml[(bh * p.max_splits + split) * 2 + 0] = M * kLog2e;
                p.part_ml[(bh * p.max_splits + split) * 2 + 1] = L;
            }
        }
    }
}

// Merge of the context splits (exp2 domain), fixed order over splits.
__global__ void paged_attn_combine_kernel(const AttnParams p) {
    pdl_wait();
    pdl_trigger();
    const int h = blockIdx.x, b = blockIdx.y;
    const int ctx = p.ctx_len[b];
    const int nsplit = (ctx + p.split_tokens - 1) / p.split_tokens;
    const size_t bh = (size_t)b * p.hq + h;
    if (ctx <= 0) {
        for (int dd = threadIdx.x; dd < p.d; dd += blockDim.x) p.out[bh * p.d + dd] = 0.f;
        return;
    }
    if (nsplit <= 1) return;
    float M = kNegBig;
    for (int s = 0; s < nsplit; ++s) M = fmaxf(M, p.part_ml[(bh * p.max_splits + s) * 2]);
    float L = 0.f;
    for (int s = 0; s < nsplit; ++s)
        L += p.part_ml[(bh * p.max_splits + s) * 2 + 1] * exp2f(p.part_ml[(bh * p.max_splits + s) * 2] - M);
    const float inv = 1.0f / fmaxf(L, 1e-12f);
    for (int dd = threadIdx.x; dd < p.d; dd += blockDim.x) {
        float O = 0.f;
        for (int s = 0; s < nsplit; ++s)
            O += p.part_o[(bh * p.max_splits + s) * p.d + dd] * exp2f(p.part_ml[(bh * p.max_splits + s) * 2] - M);
        p.out[bh * p.d + dd] = O * inv;
    }
}

// Bit-exact gather of one sequence's K/V rows (parity hook for
// vspec_kv_paged_get_token_ptr, src/attention/kv_paged_cache.c:312-356).
template <typename T>
__global__ void paged_gather_kernel(const T* kp, const T* vp, const int32_t* table, int ctx, int pt, int hkv, int d,
                                    T* kout, T* vout) {
    const size_t stride = (size_t)hkv * d;
    const size_t total = (size_t)ctx * stride;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / stride);
        const size_t within = i % stride;
        const size_t src = ((size_t)table[t / pt] * pt + (size_t)(t % pt)) * stride + within;
        kout[i] = kp[src];
        vout[i] = vp[src];
    }
}

int attn_read_and_clear_page_fault(int* out) {
    int v = 0, zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_attn_page_fault, sizeof(int));
    if (e != cudaSuccess) return cuda_status(e, "read page-fault flag");
    e = cudaMemcpyToSymbol(g_attn_page_fault, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_status(e, "clear page-fault flag");
    *out = v;
    return VSPEC_B200_OK;
}

int attn_choose_split(int batch, int hkv, int max_ctx, int sms) {
    long long want = (long long)batch * hkv * (long long)max_ctx / (4LL * sms);
    int s = (int)((want + 63) / 64) * 64;
    if (s < 64) s = 64;
    if (s > 512) s = 512;
    return s;
}

size_t attn_workspace_bytes(int batch, int hq, int d, int max_splits) {
    const size_t rows = (size_t)batch * hq * max_splits;
    return rows * d * sizeof(float) + rows * 2 * sizeof(float);
}

int paged_attention_launch(AttnParams p, int kv_dtype, cudaStream_t st) {
    const int group = p.hq / p.hkv;
    const bool mma = kv_dtype == kKvF16 && p.d == 128 && p.page_tokens > 0;
    const dim3 block(kAttnThreads);
    p.head_groups = mma ? (group + 3) / 4 : 1;
    const dim3 grid(p.max_splits, p.hkv * p.head_groups, p.batch);
    cudaError_t e;
    if (mma) {
        e = launch_pdl(paged_attn_f16_mma_kernel, grid, block, 0, st, p);
    } else {
        p.head_groups = 1;
        const dim3 sgrid(p.max_splits, p.hq, p.batch);
        if (kv_dtype == kKvF16) e = launch_pdl(paged_attn_simt_kernel<__half>, sgrid, block, 0, st, p);
        else e = launch_pdl(paged_attn_simt_kernel<float>, sgrid, block, 0, st, p);
    }
    if (e != cudaSuccess) return cuda_status(e, "paged attention launch");
    e = launch_pdl(paged_attn_combine_kernel, dim3(p.hq, p.batch), dim3(128), 0, st, p);
    if (e != cudaSuccess) return cuda_status(e, "paged attention combine launch");
    return VSPEC_B200_OK;
}

int paged_gather_launch(const void* kp, const void* vp, const int32_t* table, int ctx, int pt, int hkv, int d,
                        int kv_dtype, void* kout, void* vout, cudaStream_t st) {
    const size_t total = (size_t)ctx * hkv * d;
    unsigned blocks = (unsigned)((total + 255) / 256);
    if (blocks > 4096) blocks = 4096;
    if (blocks == 0) blocks = 1;
    if (kv_dtype == kKvF16)
        paged_gather_kernel<__half><<<blocks, 256, 0, st>>>((const __half*)kp, (const __half*)vp, table, ctx, pt, hkv,
                                                            d, (__half*)kout, (__half*)vout);
    else
        paged_gather_kernel<float><<<blocks, 256, 0, st>>>((const float*)kp, (const float*)vp, table, ctx, pt, hkv, d,
                                                           (float*)kout, (float*)vout);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e, "paged gather launch");
    return VSPEC_B200_OK;
}

}  // namespace vb200
