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
//   K and V page rows stream through a per-warp cp.async shared-memory ring.
//   QK^T: A = 16 tokens x 16 dims of K (ldmatrix), B = one or two 8-column
//         tiles of 4 query heads x {hi, lo} fp16 parts of q -> fp32-accurate
//         scores; a CTA serves up to 8 heads of one KV head.
//   PV:   A = V^T (ldmatrix.trans), B = p as {hi, lo} fp16 parts (p
//         pre-scaled by 2^14 so no part underflows).
//   Online softmax per warp in fp32; warps merge in shared memory; splits of
//   the context merge in a second kernel (fixed order: deterministic).
// fp32 pages or other head sizes: a plain fp32 SIMT kernel with the same
// split/merge structure.
#include "common.cuh"
#include "attention_kernels.cuh"
#include "tc_primitives.cuh"

#include <math.h>
#include <stdlib.h>
#include <string.h>

namespace vb200 {

constexpr int kAttnWarps = 4;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kNegBig = -1.0e30f;
constexpr float kPScale = 16384.0f;  // 2^14: keeps p's fp16 hi/lo parts normal

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    return (uint32_t)__half_as_ushort(__float2half_rn(lo)) | ((uint32_t)__half_as_ushort(__float2half_rn(hi)) << 16);
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

// Page ids of a CTA's context piece, staged once in shared memory (checked
// and redirected like token_row), so the K/V loads of a tile do not wait on a
// page-table load first.
constexpr int kAttnMaxStagedPages = 512;
constexpr int kAttnInt3MaxStagedPages = 256;   // int3 tensor-core kernel (four CTAs per SM)

__device__ __forceinline__ size_t staged_row(const int* sm_pages, int t, int first_page, int pt, int hkv, int d,
                                             int kvh) {
    const int page = sm_pages[t / pt - first_page];
    return ((size_t)page * pt + (size_t)(t % pt)) * (size_t)hkv * d + (size_t)kvh * d;
}

// ---------------------------------------------------------------------------
// Tensor-core kernel: fp16 pages, d = 128, up to 4*NT query heads per CTA
// (NT column tiles of 4 heads x {hi, lo}); every K/V row a CTA streams serves
// all its heads, so a GQA group of up to 8 reads each page row once.
// Each warp owns the 16-token tiles warp, warp + 4, ... of the CTA's context
// piece and streams their K and V rows with cp.async into a 3-stage shared
// memory ring (rows past the context are zero-filled), so several tiles are
// in flight per warp; fragments come out with ldmatrix (.trans for V^T) from
// an XOR-swizzled layout (16-byte chunk c of row r at chunk c ^ (r & 7)).
// grid = (splits, Hkv * head_groups, B), dynamic shared memory kAttnPipeSmem.
// ---------------------------------------------------------------------------
constexpr int kAttnStages = 3;
constexpr uint32_t kAttnTileBytes = 16u * 256u;                 // 16 token rows x 128 fp16 (one KV head)
constexpr uint32_t kAttnStageBytes = 2u * kAttnTileBytes;       // K + V
constexpr uint32_t kAttnPipeSmem = (uint32_t)kAttnWarps * kAttnStages * kAttnStageBytes;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr) : "memory");
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr) : "memory");
}

template <int NT>
__global__ void __launch_bounds__(kAttnThreads, 2)
paged_attn_f16_mma_kernel(const AttnParams p) {
    pdl_wait();
    pdl_trigger();
    constexpr int D = 128;
    constexpr int HPC = 4 * NT;                   // query heads per CTA
    constexpr int S = kAttnStages;
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

    extern __shared__ __align__(128) unsigned char attn_smem[];   // K/V rings; O partials after the loop
    __shared__ float sm_q[HPC][D];                // the CTA's query heads, fp32
    __shared__ float sm_qmax[HPC];
    __shared__ float sm_p[kAttnWarps][16][HPC];   // p exchange, per warp
    __shared__ float sm_ml[kAttnWarps][HPC][2];   // per-warp (m, l) per head
    __shared__ int sm_pages[kAttnMaxStagedPages];  // page ids of [t_begin, t_end)

    const int first_page = t_begin / p.page_tokens;
    const int n_pages = (t_end - 1) / p.page_tokens - first_page + 1;   // <= staged capacity (host)
    for (int i = tid; i < n_pages; i += kAttnThreads) {
        int page = __ldg(table + first_page + i);
        if (page < 0 || page >= p.num_pages) {
            atomicOr(&g_attn_page_fault, 1);
            page = 0;
        }
        sm_pages[i] = page;
    }
    // ---- q: load, per-head power-of-two rescale ----
    for (int i = tid; i < HPC * D; i += kAttnThreads) {
        const int hl = i / D, dd = i % D;
        const int h = hg * HPC + hl;
        sm_q[hl][dd] = h < group ? p.q[((size_t)b * p.hq + (size_t)kvh * group + h) * D + dd] : 0.f;
    }
    __syncthreads();

    // ---- this warp's tiles: start streaming K/V before anything else ----
    const int ntiles = (t_end - t_begin + 15) / 16;
    const int my_tiles = ntiles > warp ? (ntiles - warp + kAttnWarps - 1) / kAttnWarps : 0;
    const uint32_t wbase = smem_u32(attn_smem) + (uint32_t)warp * S * kAttnStageBytes;
    auto issue = [&](int it) {   // it-th tile of this warp -> stage it % S
        const int t0 = t_begin + (warp + it * kAttnWarps) * 16;
        const uint32_t st = wbase + (uint32_t)(it % S) * kAttnStageBytes;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int idx = i * 32 + lane;
            const int row = idx >> 4, ch = idx & 15;
            const int t = t0 + row;
            const bool valid = t < t_end;
            const size_t ro = staged_row(sm_pages, valid ? t : t_end - 1, first_page, p.page_tokens, p.hkv, D, kvh) +
                              (size_t)ch * 8;
            const uint32_t off = (uint32_t)row * 256u + ((uint32_t)(ch ^ (row & 7)) << 4);
            cp_async16(st + off, kp + ro, valid ? 16u : 0u);
            cp_async16(st + kAttnTileBytes + off, vp + ro, valid ? 16u : 0u);
        }
    };
#pragma unroll
    for (int it = 0; it < S - 1; ++it) {
        if (it < my_tiles) issue(it);
        cp_async_commit();
    }

    if (warp == 0) {
        for (int hl = 0; hl < HPC; ++hl) {
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
    // B fragment of column tile nt, k-step j: column g (head 4nt + g/2, part
    // g%2), k rows 2c, 2c+1 and 2c+8, 2c+9 = dims 16j + {2c, 2c+1, 2c+8, 2c+9}
    uint32_t qf[NT][8][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int hl = 4 * nt + (g >> 1);
        const bool lo = (g & 1) != 0;
        const float sc = ldexpf(1.0f, -(int)sm_qmax[hl]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int dims[4] = {16 * j + 2 * c, 16 * j + 2 * c + 1, 16 * j + 2 * c + 8, 16 * j + 2 * c + 9};
            float v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                float x = sm_q[hl][dims[u]] * sc;
                if (lo) x = x - __half2float(__float2half_rn(x));
                v[u] = x;
            }
            qf[nt][j][0] = pack_half2(v[0], v[1]);
            qf[nt][j][1] = pack_half2(v[2], v[3]);
        }
    }
    // this thread's heads are 4nt + c; score multiplier 2^e * scale * log2(e)
    float score_mul[NT], m_run[NT], l_run[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        score_mul[nt] = ldexpf(p.scale * kLog2e, (int)sm_qmax[4 * nt + c]);
        m_run[nt] = kNegBig;
        l_run[nt] = 0.f;
    }
    float oacc[NT][8][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 8; ++i) oacc[nt][i][0] = oacc[nt][i][1] = oacc[nt][i][2] = oacc[nt][i][3] = 0.f;

    // ldmatrix row addresses of this lane: K (tokens x dims) and V^T (.trans)
    const int k_row = (lane & 7) + 8 * ((lane >> 3) & 1), k_chi = lane >> 4;
    const int v_row = (lane & 7) + 8 * (lane >> 4), v_chi = (lane >> 3) & 1;
    for (int it = 0; it < my_tiles; ++it) {
        cp_async_wait<S - 2>();
        __syncwarp();   // tile it has landed; every lane is done with tile it-1 and sm_p
        // refill the stage of tile it-1 before computing tile it
        if (it + S - 1 < my_tiles) issue(it + S - 1);
        cp_async_commit();
        const int t0 = t_begin + (warp + it * kAttnWarps) * 16;
        const uint32_t st = wbase + (uint32_t)(it % S) * kAttnStageBytes;
        // ---- S = K Q^T over 8 k-steps of 16 dims, per column tile ----
        float s[NT][4];
        const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            uint32_t a[4];
            const int ch = 2 * j + k_chi;
            ldsm_x4(st + (uint32_t)k_row * 256u + ((uint32_t)(ch ^ (k_row & 7)) << 4), a);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) mma_16816_f16(s[nt], a, qf[nt][j][0], qf[nt][j][1], j == 0 ? zero4 : s[nt]);
        }
        // scores of tokens g and g+8 for heads 4nt + c (hi + lo columns), exp2 domain
        const bool v0 = (t0 + g) < t_end, v1 = (t0 + g + 8) < t_end;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const float sc0 = v0 ? (s[nt][0] + s[nt][1]) * score_mul[nt] : kNegBig;
            const float sc1 = v1 ? (s[nt][2] + s[nt][3]) * score_mul[nt] : kNegBig;
            float tmax = fmaxf(sc0, sc1);
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 4));
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 8));
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 16));
            const float m_new = fmaxf(m_run[nt], tmax);
            const float alpha = exp2f(m_run[nt] - m_new);
            const float p0 = v0 ? exp2f(sc0 - m_new) : 0.f;
            const float p1 = v1 ? exp2f(sc1 - m_new) : 0.f;
            l_run[nt] = l_run[nt] * alpha + (p0 + p1);
            m_run[nt] = m_new;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                oacc[nt][i][0] *= alpha; oacc[nt][i][1] *= alpha; oacc[nt][i][2] *= alpha; oacc[nt][i][3] *= alpha;
            }
            sm_p[warp][g][4 * nt + c] = p0 * kPScale;
            sm_p[warp][g + 8][4 * nt + c] = p1 * kPScale;
        }
        __syncwarp();
        // P^T B fragments: column g (head 4nt + g/2, part g%2), tokens 2c, 2c+1 and 2c+8, 2c+9
        uint32_t pb[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int hl = 4 * nt + (g >> 1);
            const bool lo = (g & 1) != 0;
            const int toks[4] = {2 * c, 2 * c + 1, 2 * c + 8, 2 * c + 9};
            float pv[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                float x = sm_p[warp][toks[r]][hl];
                if (lo) x = x - __half2float(__float2half_rn(x));
                pv[r] = x;
            }
            pb[nt][0] = pack_half2(pv[0], pv[1]);
            pb[nt][1] = pack_half2(pv[2], pv[3]);
        }
        // ---- O^T += V^T P^T over 8 blocks of 16 dims ----
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            uint32_t a[4];
            const int ch = 2 * i + v_chi;
            ldsm_x4_t(st + kAttnTileBytes + (uint32_t)v_row * 256u + ((uint32_t)(ch ^ (v_row & 7)) << 4), a);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) mma_16816_f16(oacc[nt][i], a, pb[nt][0], pb[nt][1], oacc[nt][i]);
        }
    }
    cp_async_wait<0>();

    // ---- merge the warps (O partials reuse the ring) ----
    __syncthreads();
    float* sm_o = reinterpret_cast<float*>(attn_smem);   // [kAttnWarps][HPC][D]
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        // l: sum of the per-thread partials over the 8 lanes of head 4nt + c
        float l_tot = l_run[nt];
        l_tot += __shfl_xor_sync(0xffffffffu, l_tot, 4);
        l_tot += __shfl_xor_sync(0xffffffffu, l_tot, 8);
        l_tot += __shfl_xor_sync(0xffffffffu, l_tot, 16);
        if (g == 0) {
            sm_ml[warp][4 * nt + c][0] = m_run[nt];
            sm_ml[warp][4 * nt + c][1] = l_tot;
        }
        float* o = sm_o + ((size_t)warp * HPC + 4 * nt + c) * D;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            o[16 * i + g] = (oacc[nt][i][0] + oacc[nt][i][1]) * (1.0f / kPScale);
            o[16 * i + g + 8] = (oacc[nt][i][2] + oacc[nt][i][3]) * (1.0f / kPScale);
        }
    }
    __syncthreads();
    for (int z = tid; z < HPC * D; z += kAttnThreads) {
        const int hl = z / D, dd = z % D;
        const int h_in_group = hg * HPC + hl;
        if (h_in_group >= group) continue;
        float M = kNegBig;
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, sm_ml[w][hl][0]);
        float L = 0.f, O = 0.f;
        for (int w = 0; w < kAttnWarps; ++w) {
            const float f = exp2f(sm_ml[w][hl][0] - M);
            L += sm_ml[w][hl][1] * f;
            O += sm_o[((size_t)w * HPC + hl) * D + dd] * f;
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

// ---------------------------------------------------------------------------
// int3 KV pages: per-(token, head) codes of 3 bits packed
// LSB-first (src/quant/pack.c:30-51) with fp32 scales per block of 16 or 32
// dims, as vspec_kv_cache_append stores them with int3 compression on
// (src/attention/kv_cache.c:64-126,160-226).  d = 128: 48 bytes of codes and
// 16 or 32 bytes of scales per token and head instead of 256 bytes of fp16.
// ---------------------------------------------------------------------------

// Quantisation on append: one warp per (row, head).  Per block: the
// percentile element of the sorted |x| by rank selection across the lanes
// (position idx = (size_t)((n-1) * percentile/100), computed on the host in
// double like kv_cache.c:35-58), scale = rep/4 (1 for rep 0, >= 1e-6), then
// q = lrintf(x/scale) truncated to int8 and clipped to [-4, 3]
// (kv_cache.c:86-101); IEEE division and round-to-nearest-even as the C code.
constexpr int kKvQuantWarps = 4;

__global__ void __launch_bounds__(kKvQuantWarps * 32)
kv_int3_quantize_kernel(const float* __restrict__ src, const int32_t* __restrict__ slots, int rows, int heads, int d,
                        int block, int idx, uint8_t* __restrict__ codes, float* __restrict__ scales) {
    __shared__ uint8_t sm_codes[kKvQuantWarps][256];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long item = (long long)blockIdx.x * kKvQuantWarps + warp;
    if (item >= (long long)rows * heads) return;
    const int r = (int)(item / heads), h = (int)(item - (long long)r * heads);
    const float* x = src + ((size_t)r * heads + h) * d;
    const int pb = d * 3 / 8, nb = d / block;
    const size_t orow = (size_t)(slots ? slots[r] : r) * heads + h;
    uint8_t* cw = sm_codes[warp];
    const bool in_block = lane < block;
    for (int b = 0; b < nb; ++b) {
        const float v = in_block ? x[b * block + lane] : 0.f;
        const float a = fabsf(v);
        int less = 0, le = 0;
        for (int j = 0; j < block; ++j) {
            const float aj = __shfl_sync(0xffffffffu, a, j);
            less += aj < a ? 1 : 0;
            le += aj <= a ? 1 : 0;
        }
        const unsigned hit = __ballot_sync(0xffffffffu, in_block && less <= idx && idx < le);
        const float rep = __shfl_sync(0xffffffffu, a, hit ? __ffs(hit) - 1 : 0);
        float scale = rep > 0.0f ? rep * 0.25f : 1.0f;   // rep / 4, exact
        if (scale < 1e-6f) scale = 1e-6f;
        if (in_block) {
            const long long qi = __float2ll_rn(__fdiv_rn(v, scale));
            int q = (int)(signed char)(qi & 0xFF);          // the int8 cast before the clip
            q = q < -4 ? -4 : (q > 3 ? 3 : q);
            cw[b * block + lane] = (uint8_t)(q & 7);
        }
        if (lane == 0) scales[orow * nb + b] = scale;
    }
    __syncwarp();
    uint8_t* crow = codes + orow * pb;
    for (int j = lane; j < pb; j += 32) {
        unsigned val = 0;
        for (int i = (8 * j) / 3; i <= (8 * j + 7) / 3 && i < d; ++i) {
            const int sh = 3 * i - 8 * j;
            const unsigned c = cw[i];
            val |= sh >= 0 ? (c << sh) : (c >> -sh);
        }
        crow[j] = (uint8_t)(val & 0xFFu);
    }
}

// Paged GQA decode attention over int3 pages, d = 128, up to 8 query heads
// per KV head.  grid = (splits, Hkv, B), 4 warps; each warp takes 32-token
// chunks of the CTA's piece.  QK: lane = token, the 128 codes of its K row
// decoded in registers against q (shared memory broadcast), block scales
// applied per block.  Softmax online in the exp2 domain per query head.  PV:
// the chunk's V rows staged in shared memory, lane = 4 dims, p from shared
// memory.  Warps merge in shared memory; splits merge in
// paged_attn_combine_kernel.  The math is the reference's dequantise-then-
// attend (src/kernel/cuda/attention_fused.cu:23-45,232-351).
constexpr int kInt3MaxGroup = 8;

template <int NBLK, int GM>
__global__ void __launch_bounds__(kAttnThreads, 4)
paged_attn_int3_kernel(const AttnParams p) {
    pdl_wait();
    pdl_trigger();
    constexpr int D = 128, PB = 48;
    constexpr int BS = D / NBLK;   // dims per scale block
    const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int G = p.hq / p.hkv;
    const int ctx = p.ctx_len[b];
    const int t_begin = split * p.split_tokens;
    if (t_begin >= ctx) return;
    const int t_end = min(ctx, t_begin + p.split_tokens);
    const int nsplit = (ctx + p.split_tokens - 1) / p.split_tokens;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int32_t* table = p.page_table + (size_t)b * p.max_pages;
    const uint8_t* kc = reinterpret_cast<const uint8_t*>(p.k_pages);
    const uint8_t* vc = reinterpret_cast<const uint8_t*>(p.v_pages);

    __shared__ __align__(16) float sm_q[kInt3MaxGroup][D];
    __shared__ __align__(16) uint32_t sm_v[kAttnWarps][32][PB / 4];
    __shared__ __align__(16) float sm_vs[kAttnWarps][32][NBLK];
    __shared__ float sm_p[kAttnWarps][kInt3MaxGroup][32];
    __shared__ float sm_ml[kAttnWarps][kInt3MaxGroup][2];
    __shared__ float sm_o[kAttnWarps][kInt3MaxGroup][D];

    const float qmul = p.scale * kLog2e;
    for (int i = tid; i < G * D; i += kAttnThreads) {
        const int g = i / D, dd = i - g * D;
        sm_q[g][dd] = p.q[((size_t)b * p.hq + h * G + g) * D + dd] * qmul;
    }
    __syncthreads();

    float m_run[GM], l_run[GM], o[GM][4];
#pragma unroll
    for (int g = 0; g < GM; ++g) {
        m_run[g] = kNegBig;
        l_run[g] = 0.f;
        o[g][0] = o[g][1] = o[g][2] = o[g][3] = 0.f;
    }
    const int nchunks = (t_end - t_begin + 31) / 32;
    for (int ch = warp; ch < nchunks; ch += kAttnWarps) {
        const int t = t_begin + ch * 32 + lane;
        const bool valid = t < t_end;
        size_t row = 0;
        if (valid) {
            int page = __ldg(table + t / p.page_tokens);
            if (page < 0 || page >= p.num_pages) {
                atomicOr(&g_attn_page_fault, 1);
                page = 0;
            }
            row = ((size_t)page * p.page_tokens + (size_t)(t % p.page_tokens)) * p.hkv + h;
        }
        // ---- QK: this lane's token ----
        uint32_t w[12];
        float ks[NBLK];
        if (valid) {
            const uint4* kr = reinterpret_cast<const uint4*>(kc + row * PB);
#pragma unroll
            for (int i = 0; i < 3; ++i) {
                const uint4 v4 = __ldg(kr + i);
                w[4 * i] = v4.x; w[4 * i + 1] = v4.y; w[4 * i + 2] = v4.z; w[4 * i + 3] = v4.w;
            }
            const float4* sr = reinterpret_cast<const float4*>(p.k_scales + row * NBLK);
#pragma unroll
            for (int i = 0; i < NBLK / 4; ++i) {
                const float4 f = __ldg(sr + i);
                ks[4 * i] = f.x; ks[4 * i + 1] = f.y; ks[4 * i + 2] = f.z; ks[4 * i + 3] = f.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 12; ++i) w[i] = 0u;
#pragma unroll
            for (int i = 0; i < NBLK; ++i) ks[i] = 0.f;
        }
        float sc[GM];
#pragma unroll
        for (int g = 0; g < GM; ++g) sc[g] = 0.f;
#pragma unroll
        for (int blk = 0; blk < NBLK; ++blk) {
            float part[GM];
#pragma unroll
            for (int g = 0; g < GM; ++g) part[g] = 0.f;
#pragma unroll
            for (int i4 = 0; i4 < BS / 4; ++i4) {
                float kv[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int i = blk * BS + 4 * i4 + e;   // dim, compile-time
                    const int bit = 3 * i, wi = bit >> 5, off = bit & 31;
                    uint32_t c = w[wi] >> off;
                    if (off > 29) c |= w[wi + 1] << (32 - off);
                    // 2^23 + (code + 4) from the bits, minus 2^23 + 4: exact, no int-to-float conversion
                    kv[e] = __int_as_float(0x4B000000 | (int)((c & 7u) ^ 4u)) - 8388612.0f;
                }
#pragma unroll
                for (int g = 0; g < GM; ++g) {
                    if (GM == 8 ? g < G : true) {
                        const float4 qv = *reinterpret_cast<const float4*>(&sm_q[g][blk * BS + 4 * i4]);
                        part[g] = fmaf(qv.x, kv[0], fmaf(qv.y, kv[1], fmaf(qv.z, kv[2], fmaf(qv.w, kv[3], part[g]))));
                    }
                }
            }
#pragma unroll
            for (int g = 0; g < GM; ++g) sc[g] = fmaf(part[g], ks[blk], sc[g]);
        }
        // ---- V rows of the chunk into shared memory ----
        if (valid) {
            const uint4* vr = reinterpret_cast<const uint4*>(vc + row * PB);
            uint4* dst = reinterpret_cast<uint4*>(&sm_v[warp][lane][0]);
#pragma unroll
            for (int i = 0; i < 3; ++i) dst[i] = __ldg(vr + i);
            const float4* sr = reinterpret_cast<const float4*>(p.v_scales + row * NBLK);
            float4* sd = reinterpret_cast<float4*>(&sm_vs[warp][lane][0]);
#pragma unroll
            for (int i = 0; i < NBLK / 4; ++i) sd[i] = __ldg(sr + i);
        }
        // ---- online softmax per query head ----
#pragma unroll
        for (int g = 0; g < GM; ++g) {
            if (GM == 8 ? g < G : true) {
                const float s = valid ? sc[g] : kNegBig;
                const float cmax = warp_max(s);
                const float m_new = fmaxf(m_run[g], cmax);
                const float alpha = exp2f(m_run[g] - m_new);
                const float pw = valid ? exp2f(s - m_new) : 0.f;
                l_run[g] = l_run[g] * alpha + warp_sum(pw);
                m_run[g] = m_new;
                o[g][0] *= alpha; o[g][1] *= alpha; o[g][2] *= alpha; o[g][3] *= alpha;
                sm_p[warp][g][lane] = pw;
            }
        }
        __syncwarp();
        // ---- PV: lane owns dims 4*lane .. 4*lane+3 (bits 12*lane .. +11) ----
        const int nvalid = min(32, t_end - (t_begin + ch * 32));
        const int bit0 = 12 * lane, w0 = bit0 >> 5, off0 = bit0 & 31;
        const int vblk = (4 * lane) / BS;
        for (int j = 0; j < nvalid; ++j) {
            uint32_t c = sm_v[warp][j][w0] >> off0;
            if (off0 > 20) c |= sm_v[warp][j][w0 + 1] << (32 - off0);
            const float vs = sm_vs[warp][j][vblk];
            float vv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
                vv[e] = (__int_as_float(0x4B000000 | (int)(((c >> (3 * e)) & 7u) ^ 4u)) - 8388612.0f) * vs;
#pragma unroll
            for (int g = 0; g < GM; ++g) {
                if (GM == 8 ? g < G : true) {
                    const float pj = sm_p[warp][g][j];
                    o[g][0] = fmaf(pj, vv[0], o[g][0]);
                    o[g][1] = fmaf(pj, vv[1], o[g][1]);
                    o[g][2] = fmaf(pj, vv[2], o[g][2]);
                    o[g][3] = fmaf(pj, vv[3], o[g][3]);
                }
            }
        }
        __syncwarp();
    }
    // ---- merge the warps ----
#pragma unroll
    for (int g = 0; g < GM; ++g) {
        if (GM == 8 ? g < G : true) {
            if (lane == 0) { sm_ml[warp][g][0] = m_run[g]; sm_ml[warp][g][1] = l_run[g]; }
#pragma unroll
            for (int e = 0; e < 4; ++e) sm_o[warp][g][4 * lane + e] = o[g][e];
        }
    }
    __syncthreads();
    for (int i = tid; i < G * D; i += kAttnThreads) {
        const int g = i / D, dd = i - g * D;
        float M = kNegBig;
        for (int wv = 0; wv < kAttnWarps; ++wv) M = fmaxf(M, sm_ml[wv][g][0]);
        float L = 0.f, O = 0.f;
        for (int wv = 0; wv < kAttnWarps; ++wv) {
            const float f = exp2f(sm_ml[wv][g][0] - M);
            L += sm_ml[wv][g][1] * f;
            O += sm_o[wv][g][dd] * f;
        }
        const size_t bh = (size_t)b * p.hq + h * G + g;
        if (nsplit == 1) {
            p.out[bh * D + dd] = O / fmaxf(L, 1e-12f);
        } else {
            p.part_o[(bh * p.max_splits + split) * D + dd] = O;
            if (dd == 0) {
                p.part_ml[(bh * p.max_splits + split) * 2 + 0] = M;   // exp2 domain already
                p.part_ml[(bh * p.max_splits + split) * 2 + 1] = L;
            }
        }
    }
}

// Tensor-core kernel over int3 pages (d = 128): the fp16 kernel's pipeline
// with a decode step.  Per warp and 16-token tile, cp.async stages the K and V
// code rows (48 B per token) and their block scales; after they land the warp
// turns the codes into fp16 small integers (exact) in the fp16 kernel's
// swizzled tile layout, one tile per warp (the K codes for QK^T, then the V
// codes for PV), so QK^T and PV run as in paged_attn_f16_mma_kernel.
// The scales stay out of the fp16 operands: QK^T accumulates per scale block
// and multiplies each token's block partial by its K scale in fp32, and PV
// folds each token's V scale into p (split into fp16 hi + lo parts) per block
// of dims.  Math as the reference's dequantise-then-attend
// (src/kernel/cuda/attention_fused.cu:23-45,232-351).
constexpr uint32_t kI3Codes = 16u * 48u;   // 16 token rows of one head's K (or V) codes
template <int NBLK>
struct I3Smem {
    static constexpr uint32_t kScales = 16u * NBLK * 4u;                   // 16 rows of fp32 block scales
    static constexpr uint32_t kStage = 2u * kI3Codes + 2u * kScales;      // K codes, V codes, K scales, V scales
    static constexpr uint32_t kWarp = kAttnTileBytes + kAttnStages * kStage;   // one decoded tile, the ring
    static constexpr uint32_t kTotal = kAttnWarps * kWarp;
};

// 64 codes (bits [0, 192) of w) -> 8 chunks of 8 fp16 values (code as a small integer).
// Each chunk is one 24-bit group of 8 codes: one XOR turns every code into
// its offset u = code + 4 (flip bit 2 of each field), then a pair of codes
// becomes two fp16 1024 + u with one shift-select and one mask-or, and one
// half2 subtraction of 1028 leaves the codes, exactly.
__device__ __forceinline__ void i3_decode64(const uint32_t (&w)[6], uint4 (&out)[8]) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int bit = 24 * k, wi = bit >> 5, off = bit & 31;
        uint32_t grp = w[wi] >> off;
        if (off > 8) grp |= w[wi + 1] << (32 - off);
        grp ^= 0x00924924u;   // bit 2 of each of the 8 three-bit fields
        uint32_t h2[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint32_t lo = grp >> (6 * q);          // codes 2q (bits 0-2) and 2q+1 (bits 3-5)
            const uint32_t t = (lo & 0xFFFFu) | ((lo << 13) & 0xFFFF0000u);   // code 2q+1 to bits 16-18
            h2[q] = hsub2_bits((t & 0x00070007u) | 0x64006400u, 0x64046404u);
        }
        out[k] = make_uint4(h2[0], h2[1], h2[2], h2[3]);
    }
}

template <int NT, int NBLK>
__global__ void __launch_bounds__(kAttnThreads, NT == 1 ? 4 : 3)   // 4 CTAs per SM for one column tile, 3 for two
paged_attn_int3_mma_kernel(const AttnParams p) {
    pdl_wait();
    pdl_trigger();
    constexpr int D = 128;
    constexpr int HPC = 4 * NT;
    constexpr int S = kAttnStages;
    constexpr int KS = 8 / NBLK;                 // 16-dim k-steps per scale block
    using SM = I3Smem<NBLK>;
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
    const uint8_t* kc = reinterpret_cast<const uint8_t*>(p.k_pages);
    const uint8_t* vc = reinterpret_cast<const uint8_t*>(p.v_pages);

    extern __shared__ __align__(128) unsigned char attn_smem[];
    // the query heads (fp32) live in warp 0's decoded-K tile until the fragments are built
    float (*sm_q)[D] = reinterpret_cast<float (*)[D]>(attn_smem);
    static_assert(HPC * D * sizeof(float) <= kAttnTileBytes, "query heads exceed one decoded tile");
    __shared__ float sm_qmax[HPC];
    __shared__ float sm_p[kAttnWarps][16][HPC];
    __shared__ float sm_ml[kAttnWarps][HPC][2];
    __shared__ int sm_pages[kAttnInt3MaxStagedPages];

    const int first_page = t_begin / p.page_tokens;
    const int n_pages = (t_end - 1) / p.page_tokens - first_page + 1;
    for (int i = tid; i < n_pages; i += kAttnThreads) {
        int page = __ldg(table + first_page + i);
        if (page < 0 || page >= p.num_pages) {
            atomicOr(&g_attn_page_fault, 1);
            page = 0;
        }
        sm_pages[i] = page;
    }
    for (int i = tid; i < HPC * D; i += kAttnThreads) {
        const int hl = i / D, dd = i % D;
        const int h = hg * HPC + hl;
        sm_q[hl][dd] = h < group ? p.q[((size_t)b * p.hq + (size_t)kvh * group + h) * D + dd] : 0.f;
    }
    __syncthreads();

    const int ntiles = (t_end - t_begin + 15) / 16;
    const int my_tiles = ntiles > warp ? (ntiles - warp + kAttnWarps - 1) / kAttnWarps : 0;
    unsigned char* wptr = attn_smem + (size_t)warp * SM::kWarp;
    const uint32_t wbase = smem_u32(wptr);
    // one decoded tile per warp: K for QK^T, then V for PV
    const uint32_t tile_k = wbase, tile_v = wbase;
    const uint32_t stage0 = wbase + kAttnTileBytes;
    // issue: lane -> one token row of the tile, K (lanes 0-15) or V (lanes 16-31): its 48 code bytes
    // (three 16-byte chunks) and its NBLK block scales
    const int i_row = lane & 15, i_kv = lane >> 4;
    const bool pt_pow2 = (p.page_tokens & (p.page_tokens - 1)) == 0;
    const int pt_shift = __ffs(p.page_tokens) - 1;
    const uint8_t* i_codes = i_kv ? vc : kc;
    const float* i_scales = i_kv ? p.v_scales : p.k_scales;
    auto issue = [&](int it) {   // codes and scales of this warp's it-th tile -> stage it % S
        const int t0 = t_begin + (warp + it * kAttnWarps) * 16;
        const uint32_t st = stage0 + (uint32_t)(it % S) * SM::kStage;
        const int t = t0 + i_row;
        const bool valid = t < t_end;
        const int tt = valid ? t : t_end - 1;
        const int pg = pt_pow2 ? (tt >> pt_shift) : tt / p.page_tokens;
        const int slot = pt_pow2 ? (tt & (p.page_tokens - 1)) : tt - pg * p.page_tokens;
        const size_t ri = ((size_t)sm_pages[pg - first_page] * p.page_tokens + (size_t)slot) * (size_t)p.hkv + kvh;
        const uint32_t nb = valid ? 16u : 0u;
        const uint32_t cdst = st + (uint32_t)i_kv * kI3Codes + (uint32_t)i_row * 48u;
        const uint8_t* csrc = i_codes + ri * 48;
        cp_async16(cdst, csrc, nb);
        cp_async16(cdst + 16u, csrc + 16, nb);
        cp_async16(cdst + 32u, csrc + 32, nb);
        const uint32_t sdst = st + 2u * kI3Codes + (uint32_t)i_kv * SM::kScales + (uint32_t)i_row * (NBLK * 4u);
#pragma unroll
        for (int k = 0; k < NBLK / 4; ++k) cp_async16(sdst + 16u * k, i_scales + ri * NBLK + 4 * k, nb);
    };
#pragma unroll
    for (int it = 0; it < S - 1; ++it) {
        if (it < my_tiles) issue(it);
        cp_async_commit();
    }

    if (warp == 0) {
        for (int hl = 0; hl < HPC; ++hl) {
            float mx = 0.f;
            for (int dd = lane; dd < D; dd += 32) mx = fmaxf(mx, fabsf(sm_q[hl][dd]));
            mx = warp_max(mx);
            if (lane == 0) {
                int ex = 0;
                if (mx > 0.f && isfinite(mx)) { (void)frexpf(mx, &ex); ex -= 14; }
                sm_qmax[hl] = (float)ex;
            }
        }
    }
    __syncthreads();
    uint32_t qf[NT][8][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int hl = 4 * nt + (g >> 1);
        const bool lo = (g & 1) != 0;
        const float sc = ldexpf(1.0f, -(int)sm_qmax[hl]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int dims[4] = {16 * j + 2 * c, 16 * j + 2 * c + 1, 16 * j + 2 * c + 8, 16 * j + 2 * c + 9};
            float v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                float x = sm_q[hl][dims[u]] * sc;
                if (lo) x = x - __half2float(__float2half_rn(x));
                v[u] = x;
            }
            qf[nt][j][0] = pack_half2(v[0], v[1]);
            qf[nt][j][1] = pack_half2(v[2], v[3]);
        }
    }
    float score_mul[NT], m_run[NT], l_run[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        score_mul[nt] = ldexpf(p.scale * kLog2e, (int)sm_qmax[4 * nt + c]);
        m_run[nt] = kNegBig;
        l_run[nt] = 0.f;
    }
    float oacc[NT][8][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 8; ++i) oacc[nt][i][0] = oacc[nt][i][1] = oacc[nt][i][2] = oacc[nt][i][3] = 0.f;

    const int k_row = (lane & 7) + 8 * ((lane >> 3) & 1), k_chi = lane >> 4;
    const int v_row = (lane & 7) + 8 * (lane >> 4), v_chi = (lane >> 3) & 1;
    const int dr = lane & 15, dh = lane >> 4;     // decode: token row and half of the dims (8 lanes of a
                                                  // 16-byte store phase write 8 distinct bank groups)
    __syncthreads();   // every warp has its q fragments: warp 0's tile may now be overwritten
    for (int it = 0; it < my_tiles; ++it) {
        cp_async_wait<S - 2>();
        __syncwarp();   // tile it has landed; every lane is done with tile it-1 (decoded tiles, sm_p)
        const int t0 = t_begin + (warp + it * kAttnWarps) * 16;
        const uint32_t st = stage0 + (uint32_t)(it % S) * SM::kStage;
        const unsigned char* stp = wptr + kAttnTileBytes + (size_t)(it % S) * SM::kStage;
        // codes of K (kv 0) or V (kv 1) -> the warp's fp16 tile (row dr, dims 64*dh ..)
        auto decode_tile = [&](int kv) {
            const uint32_t* src = reinterpret_cast<const uint32_t*>(stp + kv * kI3Codes + dr * 48 + dh * 24);
            uint32_t w[6];
#pragma unroll
            for (int i = 0; i < 6; ++i) w[i] = src[i];
            uint4 outc[8];
            i3_decode64(w, outc);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int ch = 8 * dh + k;
                *reinterpret_cast<uint4*>(wptr + dr * 256 + ((ch ^ (dr & 7)) << 4)) = outc[k];
            }
        };
        decode_tile(0);
        __syncwarp();
        // refill the stage of tile it-1 (its codes were decoded in the previous step)
        if (it + S - 1 < my_tiles) issue(it + S - 1);
        cp_async_commit();
        const float* ks = reinterpret_cast<const float*>(stp + 2u * kI3Codes);
        const float* vs = reinterpret_cast<const float*>(stp + 2u * kI3Codes + SM::kScales);
        // ---- S = K Q^T per scale block, scaled per token in fp32 ----
        float s[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
        const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
        float ksg[NBLK], ksg8[NBLK];   // K scales of token rows g and g + 8
#pragma unroll
        for (int k4 = 0; k4 < NBLK / 4; ++k4) {
            const float4 a = *reinterpret_cast<const float4*>(ks + g * NBLK + 4 * k4);
            const float4 b = *reinterpret_cast<const float4*>(ks + (g + 8) * NBLK + 4 * k4);
            ksg[4 * k4] = a.x; ksg[4 * k4 + 1] = a.y; ksg[4 * k4 + 2] = a.z; ksg[4 * k4 + 3] = a.w;
            ksg8[4 * k4] = b.x; ksg8[4 * k4 + 1] = b.y; ksg8[4 * k4 + 2] = b.z; ksg8[4 * k4 + 3] = b.w;
        }
#pragma unroll
        for (int bl = 0; bl < NBLK; ++bl) {
            float sb[NT][4];
#pragma unroll
            for (int jj = 0; jj < KS; ++jj) {
                const int j = bl * KS + jj;
                uint32_t a[4];
                const int ch = 2 * j + k_chi;
                ldsm_x4(tile_k + (uint32_t)k_row * 256u + ((uint32_t)(ch ^ (k_row & 7)) << 4), a);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
                    mma_16816_f16(sb[nt], a, qf[nt][j][0], qf[nt][j][1], jj == 0 ? zero4 : sb[nt]);
            }
            const float k0 = ksg[bl], k1 = ksg8[bl];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                s[nt][0] = fmaf(sb[nt][0], k0, s[nt][0]);
                s[nt][1] = fmaf(sb[nt][1], k0, s[nt][1]);
                s[nt][2] = fmaf(sb[nt][2], k1, s[nt][2]);
                s[nt][3] = fmaf(sb[nt][3], k1, s[nt][3]);
            }
        }
        const bool v0 = (t0 + g) < t_end, v1 = (t0 + g + 8) < t_end;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const float sc0 = v0 ? (s[nt][0] + s[nt][1]) * score_mul[nt] : kNegBig;
            const float sc1 = v1 ? (s[nt][2] + s[nt][3]) * score_mul[nt] : kNegBig;
            float tmax = fmaxf(sc0, sc1);
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 4));
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 8));
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 16));
            const float m_new = fmaxf(m_run[nt], tmax);
            const float alpha = exp2f(m_run[nt] - m_new);
            const float p0 = v0 ? exp2f(sc0 - m_new) : 0.f;
            const float p1 = v1 ? exp2f(sc1 - m_new) : 0.f;
            l_run[nt] = l_run[nt] * alpha + (p0 + p1);
            m_run[nt] = m_new;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                oacc[nt][i][0] *= alpha; oacc[nt][i][1] *= alpha; oacc[nt][i][2] *= alpha; oacc[nt][i][3] *= alpha;
            }
            sm_p[warp][g][4 * nt + c] = p0 * kPScale;
            sm_p[warp][g + 8][4 * nt + c] = p1 * kPScale;
        }
        __syncwarp();   // every lane's ldmatrix reads of the K tile are done: V may overwrite it
        decode_tile(1);
        __syncwarp();
        // ---- O^T += V^T (P s_v)^T, per scale block of dims ----
        const int toks[4] = {2 * c, 2 * c + 1, 2 * c + 8, 2 * c + 9};
        float pt4[NT][4], vs4[4][NBLK];   // p of this lane's 4 tokens; their V scales
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int r = 0; r < 4; ++r) pt4[nt][r] = sm_p[warp][toks[r]][4 * nt + (g >> 1)];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int k4 = 0; k4 < NBLK / 4; ++k4) {
                const float4 a = *reinterpret_cast<const float4*>(vs + toks[r] * NBLK + 4 * k4);
                vs4[r][4 * k4] = a.x; vs4[r][4 * k4 + 1] = a.y; vs4[r][4 * k4 + 2] = a.z; vs4[r][4 * k4 + 3] = a.w;
            }
#pragma unroll
        for (int bl = 0; bl < NBLK; ++bl) {
            uint32_t pb[NT][2];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const bool lo = (g & 1) != 0;
                float pv[4];
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    float x = pt4[nt][r] * vs4[r][bl];
                    if (lo) x = x - __half2float(__float2half_rn(x));
                    pv[r] = x;
                }
                pb[nt][0] = pack_half2(pv[0], pv[1]);
                pb[nt][1] = pack_half2(pv[2], pv[3]);
            }
#pragma unroll
            for (int ii = 0; ii < KS; ++ii) {
                const int i = bl * KS + ii;
                uint32_t a[4];
                const int ch = 2 * i + v_chi;
                ldsm_x4_t(tile_v + (uint32_t)v_row * 256u + ((uint32_t)(ch ^ (v_row & 7)) << 4), a);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) mma_16816_f16(oacc[nt][i], a, pb[nt][0], pb[nt][1], oacc[nt][i]);
            }
        }
    }
    cp_async_wait<0>();

    // ---- merge the warps (O partials reuse the staging area) ----
    __syncthreads();
    float* sm_o = reinterpret_cast<float*>(attn_smem);   // [kAttnWarps][HPC][D]
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        float l_tot = l_run[nt];
        l_tot += __shfl_xor_sync(0xffffffffu, l_tot, 4);
        l_tot += __shfl_xor_sync(0xffffffffu, l_tot, 8);
        l_tot += __shfl_xor_sync(0xffffffffu, l_tot, 16);
        if (g == 0) {
            sm_ml[warp][4 * nt + c][0] = m_run[nt];
            sm_ml[warp][4 * nt + c][1] = l_tot;
        }
        float* o = sm_o + ((size_t)warp * HPC + 4 * nt + c) * D;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            o[16 * i + g] = (oacc[nt][i][0] + oacc[nt][i][1]) * (1.0f / kPScale);
            o[16 * i + g + 8] = (oacc[nt][i][2] + oacc[nt][i][3]) * (1.0f / kPScale);
        }
    }
    __syncthreads();
    for (int z = tid; z < HPC * D; z += kAttnThreads) {
        const int hl = z / D, dd = z % D;
        const int h_in_group = hg * HPC + hl;
        if (h_in_group >= group) continue;
        float M = kNegBig;
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, sm_ml[w][hl][0]);
        float L = 0.f, O = 0.f;
        for (int w = 0; w < kAttnWarps; ++w) {
            const float f = exp2f(sm_ml[w][hl][0] - M);
            L += sm_ml[w][hl][1] * f;
            O += sm_o[((size_t)w * HPC + hl) * D + dd] * f;
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

// Context piece per CTA: enough pieces for about four CTAs per resident slot
// (ctas_per_sm per SM: the kernel's residency), no split at all when the
// (sequence, KV head group) pairs alone fill the slots, pieces under 512
// tokens only as far as one CTA per slot needs them, and at most the kernel's
// staged page capacity (page_tokens <= 0: the capacity for one-token pages,
// the most conservative).
int attn_choose_split(int batch, int hq, int hkv, int max_ctx, int page_tokens, int sms, int ctas_per_sm,
                      int max_staged_pages) {
    const int group = hkv > 0 ? hq / hkv : 1;
    const int hpc = group <= 4 ? 4 : 8;
    const long long pairs = (long long)batch * hkv * ((group + hpc - 1) / hpc);
    const long long slots = (long long)ctas_per_sm * sms;
    const int pt = page_tokens > 0 ? page_tokens : 1;
    int cap = (max_staged_pages - 1) * pt / 64 * 64;
    if (cap < 64) cap = 64;
    const long long np = pairs > 0 ? pairs : 1;
    long long pieces = pairs >= slots ? 1 : (4 * slots + np - 1) / np;
    long long s = ((max_ctx + pieces - 1) / pieces + 63) / 64 * 64;
    if (s < 512) {
        // pieces shorter than 512 tokens only as far as needed for one CTA
        // per slot: a piece pays a fixed prologue (page ids, q fragments)
        const long long p1 = (slots + np - 1) / np;
        const long long s1 = ((max_ctx + p1 - 1) / p1 + 63) / 64 * 64;
        const long long floor_s = s1 < 512 ? s1 : 512;
        if (s < floor_s) s = floor_s;
    }
    // at least 128 tokens a piece: a piece pays its prologue and the combine a slot, and at batch 1
    // (8 KV heads, ctx 512 / 768 / 2048) 128-token pieces measured 8.8 / 9.5 / 11.8 us per call
    // against 9.2 / 10.4 / 15.3 with 64
    if (s < 128) s = 128;
    if (s > cap) s = cap;
    return (int)s;
}

size_t attn_workspace_bytes(int batch, int hq, int d, int max_splits) {
    const size_t rows = (size_t)batch * hq * max_splits;
    return rows * d * sizeof(float) + rows * 2 * sizeof(float);
}

int kv_int3_quantize_launch(const float* src, const int32_t* slots, int rows, int heads, int d, int block,
                            float percentile, uint8_t* codes, float* scales, cudaStream_t st) {
    if (percentile < 50.0f) percentile = 50.0f;   // kv_cache.c:38-43
    if (percentile > 100.0f) percentile = 100.0f;
    size_t idx = (size_t)((double)(block - 1) * ((double)percentile / 100.0));
    if (idx >= (size_t)block) idx = (size_t)block - 1;
    const long long items = (long long)rows * heads;
    const unsigned grid = (unsigned)((items + kKvQuantWarps - 1) / kKvQuantWarps);
    kv_int3_quantize_kernel<<<grid, kKvQuantWarps * 32, 0, st>>>(src, slots, rows, heads, d, block, (int)idx, codes,
                                                                 scales);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e, "kv_int3_quantize_kernel launch");
    return VSPEC_B200_OK;
}

// VSPEC_B200_INT3_ATTN_SIMT=1 runs int3 pages through the SIMT kernel (A/B timing).
static bool int3_mma_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("VSPEC_B200_INT3_ATTN_SIMT");
        v = (e && e[0] == '1') ? 0 : 1;
    }
    return v == 1;
}

int paged_attention_launch(AttnParams p, int kv_dtype, cudaStream_t st) {
    const int group = p.hq / p.hkv;
    if (kv_dtype == kKvInt3 && int3_mma_enabled()) {
        const int hpc = group <= 4 ? 4 : 8;
        p.head_groups = (group + hpc - 1) / hpc;
        const dim3 grid(p.max_splits, p.hkv * p.head_groups, p.batch);
        static int configured[64] = {0};
        int dev = 0;
        cudaGetDevice(&dev);
        cudaError_t e = cudaSuccess;
        if (dev >= 0 && dev < 64 && !configured[dev]) {
            e = cudaFuncSetAttribute(paged_attn_int3_mma_kernel<1, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)I3Smem<4>::kTotal);
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(paged_attn_int3_mma_kernel<2, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)I3Smem<4>::kTotal);
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(paged_attn_int3_mma_kernel<1, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)I3Smem<8>::kTotal);
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(paged_attn_int3_mma_kernel<2, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)I3Smem<8>::kTotal);
            // the whole unified memory as shared memory, so four CTAs of one column tile fit per SM
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(paged_attn_int3_mma_kernel<1, 4>,
                                         cudaFuncAttributePreferredSharedMemoryCarveout, 100);
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(paged_attn_int3_mma_kernel<1, 8>,
                                         cudaFuncAttributePreferredSharedMemoryCarveout, 100);
            if (e != cudaSuccess) return cuda_status(e, "paged int3 attention smem attribute");
            configured[dev] = 1;
        }
        const dim3 blk(kAttnThreads);
        if (p.kv_block == 16)
            e = hpc == 4 ? launch_pdl(paged_attn_int3_mma_kernel<1, 8>, grid, blk, I3Smem<8>::kTotal, st, p)
                         : launch_pdl(paged_attn_int3_mma_kernel<2, 8>, grid, blk, I3Smem<8>::kTotal, st, p);
        else
            e = hpc == 4 ? launch_pdl(paged_attn_int3_mma_kernel<1, 4>, grid, blk, I3Smem<4>::kTotal, st, p)
                         : launch_pdl(paged_attn_int3_mma_kernel<2, 4>, grid, blk, I3Smem<4>::kTotal, st, p);
        if (e != cudaSuccess) return cuda_status(e, "paged int3 attention launch");
        e = launch_pdl(paged_attn_combine_kernel, dim3(p.hq, p.batch), dim3(128), 0, st, p);
        if (e != cudaSuccess) return cuda_status(e, "paged attention combine launch");
        return VSPEC_B200_OK;
    }
    if (kv_dtype == kKvInt3) {
        p.head_groups = 1;
        const dim3 grid(p.max_splits, p.hkv, p.batch);
        // query heads per KV head: exact kernels for 1, 2 and 4, predicated up to 8 otherwise
        const int gm = group == 1 ? 1 : (group == 2 ? 2 : (group == 4 ? 4 : 8));
        auto pick = [&](auto k1, auto k2, auto k4, auto k8) {
            return gm == 1 ? launch_pdl(k1, grid, dim3(kAttnThreads), 0, st, p)
                 : gm == 2 ? launch_pdl(k2, grid, dim3(kAttnThreads), 0, st, p)
                 : gm == 4 ? launch_pdl(k4, grid, dim3(kAttnThreads), 0, st, p)
                           : launch_pdl(k8, grid, dim3(kAttnThreads), 0, st, p);
        };
        cudaError_t e = p.kv_block == 16
            ? pick(paged_attn_int3_kernel<8, 1>, paged_attn_int3_kernel<8, 2>, paged_attn_int3_kernel<8, 4>,
                   paged_attn_int3_kernel<8, 8>)
            : pick(paged_attn_int3_kernel<4, 1>, paged_attn_int3_kernel<4, 2>, paged_attn_int3_kernel<4, 4>,
                   paged_attn_int3_kernel<4, 8>);
        if (e != cudaSuccess) return cuda_status(e, "paged int3 attention launch");
        e = launch_pdl(paged_attn_combine_kernel, dim3(p.hq, p.batch), dim3(128), 0, st, p);
        if (e != cudaSuccess) return cuda_status(e, "paged attention combine launch");
        return VSPEC_B200_OK;
    }
    const bool mma = kv_dtype == kKvF16 && p.d == 128 && p.page_tokens > 0;
    const dim3 block(kAttnThreads);
    // 4 query heads per CTA for groups up to 4, else 8 (two column tiles)
    const int hpc = group <= 4 ? 4 : 8;
    p.head_groups = mma ? (group + hpc - 1) / hpc : 1;
    const dim3 grid(p.max_splits, p.hkv * p.head_groups, p.batch);
    cudaError_t e;
    if (mma) {
        static int configured[64] = {0};
        int dev = 0;
        cudaGetDevice(&dev);
        if (dev >= 0 && dev < 64 && !configured[dev]) {
            e = cudaFuncSetAttribute(paged_attn_f16_mma_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kAttnPipeSmem);
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(paged_attn_f16_mma_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kAttnPipeSmem);
            if (e != cudaSuccess) return cuda_status(e, "paged attention smem attribute");
            configured[dev] = 1;
        }
        e = hpc == 4 ? launch_pdl(paged_attn_f16_mma_kernel<1>, grid, block, kAttnPipeSmem, st, p)
                     : launch_pdl(paged_attn_f16_mma_kernel<2>, grid, block, kAttnPipeSmem, st, p);
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
