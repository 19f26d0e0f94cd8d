// lowbit_gemv_tc.cu -- tcgen05 / TMEM / TMA low-bit GEMV for decode (M <= 4).
//
// Same contraction and numerics contract as lowbit_gemv.cu (group-wise
// dequant, fp32 activations split into fp16 hi + lo, fp32 accumulation), laid
// out for Blackwell:
//   * one persistent CTA per SM owns a contiguous run of (128-row tile,
//     128-code k-block) units (split-K across CTAs, deterministic merge);
//   * warp 4 (one thread) streams weight tiles with 2-D TMA into a 16-24
//     stage shared-memory ring (~96-128 KB in flight per SM);
//   * warps 0-3 decode one weight row per thread straight from shared memory
//     into tensor memory (the MMA's A operand, 64 fp16 pairs per k-block);
//   * warp 5 owns TMEM and issues tcgen05.mma (M=128, N=16, K=16) with A in
//     TMEM and the activation fragments (B) in shared memory; the fp32
//     accumulator lives in TMEM and is read back per k-block for the
//     group-scale / zero-point epilogue.
// Every wait is bounded; a timeout raises a device flag, drains in-flight
// copies and MMAs, frees TMEM and returns.
#include "common.cuh"
#include "lowbit_decode.cuh"
#include "lowbit_kernels.cuh"
#include "tc_primitives.cuh"

#include <cudaTypedefs.h>
#include <string.h>

namespace vb200 {

constexpr int kTcRows = 128;
constexpr int kTcConsumerThreads = 128;
constexpr int kTcThreads = 6 * 32;
constexpr int kTcAStages = 4;
constexpr uint32_t kTcTmemCols = 512;
constexpr uint32_t kTcWaitLimit = 1u << 24;
constexpr int kTcMaxM = 4;

template <int BITS> struct TcCfg;
template <> struct TcCfg<4> { static constexpr int kStages = 16; static constexpr int kRowBytes = 64; };
template <> struct TcCfg<3> { static constexpr int kStages = 16; static constexpr int kRowBytes = 48; };
template <> struct TcCfg<2> { static constexpr int kStages = 24; static constexpr int kRowBytes = 32; };

// Set when a bounded wait of the tensor-core GEMV gave up.
__device__ int g_tc_timeout = 0;

// Byte offset of 16-byte chunk c of row r inside a TMA stage, matching the
// swizzle the tensor map was encoded with (64B for int4, 32B for int2, none
// for int3 whose 48-byte rows are already bank-conflict free).
template <int BITS>
__device__ __forceinline__ uint32_t stage_chunk_offset(int r, int c) {
    if constexpr (BITS == 4) return (uint32_t)(r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
    else if constexpr (BITS == 2) return (uint32_t)(r * 32 + ((c ^ ((r >> 2) & 1)) << 4));
    else return (uint32_t)(r * 48 + (c << 4));
}

struct TcSmem {
    uint32_t w_ring;      // offsets from the 1024-aligned base
    uint32_t bfrag;
    uint32_t xs, cs, misc;
    uint32_t total;
};

template <int BITS>
__host__ __device__ inline TcSmem tc_smem_plan(int m, int kbt) {
    TcSmem s;
    const uint32_t stage = kTcRows * TcCfg<BITS>::kRowBytes;
    s.w_ring = 0;
    s.bfrag = TcCfg<BITS>::kStages * stage;
    const uint32_t lbo = 32u * (uint32_t)m;
    const uint32_t bbytes = (uint32_t)kbt * 16u * lbo + 128u;
    s.xs = (s.bfrag + bbytes + 15u) & ~15u;
    s.cs = s.xs + (uint32_t)(kbt * m) * 4u;
    s.misc = (s.cs + (uint32_t)(kbt * m) * 4u + 15u) & ~15u;
    s.total = s.misc + 1024u;   // barriers, flags, reduction scratch
    return s;
}

template <int BITS, bool UNSIGNED, int EPI>
__global__ void __launch_bounds__(kTcThreads, 1)
lowbit_gemv_tc_kernel(const __grid_constant__ CUtensorMap wmap, const GemvParams p) {
    constexpr int NS = TcCfg<BITS>::kStages;
    constexpr int RB = TcCfg<BITS>::kRowBytes;
    constexpr uint32_t STAGE_BYTES = kTcRows * RB;
    constexpr int NA = kTcAStages;

    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    unsigned char* base = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    const int m = p.m;
    const int kbt = p.kb_total;
    const TcSmem plan = tc_smem_plan<BITS>(m, kbt);
    const uint32_t lbo = 32u * (uint32_t)m;   // activation fragment K-chunk stride (2m rows of 16 B)

    unsigned char* wring = base + plan.w_ring;
    unsigned char* bfr = base + plan.bfrag;
    float* xs = reinterpret_cast<float*>(base + plan.xs);
    float* cs = reinterpret_cast<float*>(base + plan.cs);
    unsigned char* misc = base + plan.misc;
    uint64_t* full = reinterpret_cast<uint64_t*>(misc);
    uint64_t* empty = full + NS;
    uint64_t* a_ready = empty + NS;
    uint64_t* d_ready = a_ready + NA;
    uint64_t* fl_bar = d_ready + NA;          // [2] flush rendezvous
    uint64_t* drain_bar = fl_bar + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* merge_flag = abort_flag + 1;
    float* maxbuf = reinterpret_cast<float*>(tmem_slot + 4);   // [6][4]
    float* row_scale = maxbuf + 24;                            // [4]
    float* row_norm = row_scale + 4;                           // [4]

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;

    const long long U = (long long)p.tiles * kbt;
    const long long C = gridDim.x;
    const int u0 = (int)(((long long)blockIdx.x * U) / C);
    const int u1 = (int)(((long long)(blockIdx.x + 1) * U) / C);
    const int n_units = u1 - u0;

    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kTcConsumerThreads);
        }
        for (int a = 0; a < NA; ++a) {
            mbar_init(&a_ready[a], kTcConsumerThreads);
            mbar_init(&d_ready[a], 1);
        }
        mbar_init(&fl_bar[0], kTcConsumerThreads);
        mbar_init(&fl_bar[1], 1);
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 5) {
        tmem_alloc(tmem_slot, kTcTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    // ---- producer: first ring fill (weights only: no dependency on x) ----
    int p_issued = 0;
    int p_tile = u0 / (kbt > 0 ? kbt : 1), p_kb = u0 - p_tile * kbt;
    if (warp == 4 && lane == 0) {
        tma_prefetch_desc(&wmap);
        for (; p_issued < n_units && p_issued < NS; ++p_issued) {
            mbar_arrive_expect_tx(&full[p_issued], STAGE_BYTES);
            tma_load_2d(wring + p_issued * STAGE_BYTES, &wmap, p_kb * RB, p_tile * kTcRows, &full[p_issued]);
            if (++p_kb == kbt) { p_kb = 0; ++p_tile; }
        }
    }

    // ---- activation prologue (x may come from the previous kernel) ----
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    const int K = p.k;
    const bool rms = EPI_HAS_RMSNORM(p.flags);
    if (rms) {
        for (int r = warp; r < m; r += 6) {
            const float4* xr = reinterpret_cast<const float4*>(p.x + (size_t)r * K);
            float ss = 0.f;
            for (int t = lane; t < K / 4; t += 32) {
                const float4 v = xr[t];
                ss += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
            }
            ss = warp_sum(ss);
            if (lane == 0) row_norm[r] = 1.0f / sqrtf(ss / (float)K + p.eps);
        }
        __syncthreads();
    }
    auto xval = [&](int r, int t) -> float {
        float v = p.x[(size_t)r * K + t];
        if (rms) v = v * row_norm[r] * p.norm_w[t];
        return v;
    };
    // (a) X = sum x, W = sum x/mult per (k-block, row); per-row max |x|
    {
        float mx[kTcMaxM] = {0.f, 0.f, 0.f, 0.f};
        float mlt[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) mlt[e] = 1.0f / code_mult<BITS>((lane * 4 + e) & 31);
        for (int pr = warp; pr < kbt * m; pr += 6) {
            const int r = pr % m, kb = pr / m;
            const int t = kb * 128 + lane * 4;
            float4 v = *reinterpret_cast<const float4*>(p.x + (size_t)r * K + t);
            if (rms) {
                const float nr = row_norm[r];
                const float4 wn = *reinterpret_cast<const float4*>(p.norm_w + t);
                v.x *= nr * wn.x; v.y *= nr * wn.y; v.z *= nr * wn.z; v.w *= nr * wn.w;
            }
            const float sx = warp_sum((v.x + v.y) + (v.z + v.w));
            const float sw = warp_sum((v.x * mlt[0] + v.y * mlt[1]) + (v.z * mlt[2] + v.w * mlt[3]));
            const float a = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
            for (int rr = 0; rr < kTcMaxM; ++rr)
                if (rr == r) mx[rr] = fmaxf(mx[rr], a);
            if (lane == 0) {
                xs[kb * m + r] = sx;
                cs[kb * m + r] = sw;
            }
        }
#pragma unroll
        for (int r = 0; r < kTcMaxM; ++r) {
            const float v = warp_max(mx[r]);
            if (lane == 0) maxbuf[warp * 4 + r] = v;
        }
        __syncthreads();
        if (tid < m) {
            float v = 0.f;
            for (int w = 0; w < 6; ++w) v = fmaxf(v, maxbuf[w * 4 + tid]);
            int ex = 0;   // exact power-of-two rescale: max |x| in [2^13, 2^14)
            if (v > 0.f && isfinite(v)) { (void)frexpf(v, &ex); ex -= 14; }
            row_scale[tid] = ldexpf(1.0f, -ex);
        }
        __syncthreads();
    }
    // (b) activation fragments: K-chunk kc of k-block kb is a core matrix whose
    // row n = 2r + {0: hi, 1: lo} holds the 8 fp16 values matching A columns
    // 4kc..4kc+3 (pairs (lo_code(q), hi_code(q)) of 32-code chunk col/16),
    // divided by their decode multiplier.  Rows are 16 B apart and K-chunks
    // 2m rows apart; the core matrix's unused rows alias later chunks.
    {
        const int items = kbt * 16 * 2 * m;
        for (int it = tid; it < items; it += kTcThreads) {
            const int n = it % (2 * m);
            const int kc = (it / (2 * m)) % 16;
            const int kb = it / (32 * m);
            const int r = n >> 1;
            const bool lo_part = (n & 1) != 0;
            const float sc = row_scale[r];
            uint32_t w4[4];
#pragma unroll
            for (int e2 = 0; e2 < 4; ++e2) {
                const int col = 4 * kc + e2;
                const int c32 = col >> 4, q = col & 15;
                const int j0 = lo_code<BITS>(q), j1 = hi_code<BITS>(q);
                float v0 = xval(r, kb * 128 + 32 * c32 + j0) * sc / code_mult<BITS>(j0);
                float v1 = xval(r, kb * 128 + 32 * c32 + j1) * sc / code_mult<BITS>(j1);
                __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
                if (lo_part) {
                    h0 = __float2half_rn(v0 - __half2float(h0));
                    h1 = __float2half_rn(v1 - __half2float(h1));
                }
                w4[e2] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
            }
            *reinterpret_cast<uint4*>(bfr + (size_t)(kb * 16 + kc) * lbo + 16 * n) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
        if (tid < 32) *reinterpret_cast<uint4*>(bfr + (size_t)kbt * 16 * lbo + 16 * (tid & 7)) = make_uint4(0, 0, 0, 0);
        constexpr float kOff = (float)(1 << (BITS - 1));
        for (int i = tid; i < kbt * m; i += kTcThreads) {
            const float sc = row_scale[i % m];
            const float X = xs[i] * sc;
            xs[i] = X;
            cs[i] = fmaf(1024.0f, cs[i] * sc, kOff * X);
        }
    }
    // make the generic-proxy smem writes (B fragments) visible to the tensor core
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    __syncthreads();
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");

    const int half_tiles = p.tiles >> 1;
    if (warp < 4) {
        // ======================= decode warps (one weight row per thread) ====
        const int row = warp * 32 + lane;
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        float acc[kTcMaxM] = {0.f, 0.f, 0.f, 0.f};
        uint32_t e_s[NA], e_z[NA];
        const bool sz16 = (p.flags & VSPEC_B200_F_SZ_F16) != 0;
        const uint32_t one_bits = sz16 ? 0x3C00u : 0x3F800000u;
        const uint32_t zc_bits = sz16 ? (uint32_t)__half_as_ushort(__float2half_rn(p.zp_const)) : __float_as_uint(p.zp_const);
        int e_kb[NA], e_tile[NA], e_last[NA];
        int c_tile = u0 / kbt, c_kb = u0 - c_tile * kbt;
        int flushes = 0;
        bool ok = true;

        auto flush = [&](int tile) {
            const int fw = (int)((((long long)tile * kbt + 1) * C - 1) / U);
            const int lw = (int)((((long long)(tile + 1) * kbt) * C - 1) / U);
            int L = tile, slot = (int)blockIdx.x - fw, total = lw - fw + 1, n_gate = total;
            if (EPI == kEpiSwiGLU) {
                const bool up = tile >= half_tiles;
                L = up ? tile - half_tiles : tile;
                const int gt = L, ut = L + half_tiles;
                const int g_fw = (int)((((long long)gt * kbt + 1) * C - 1) / U);
                const int g_n = (int)((((long long)(gt + 1) * kbt) * C - 1) / U) - g_fw + 1;
                const int u_fw = (int)((((long long)ut * kbt + 1) * C - 1) / U);
                const int u_n = (int)((((long long)(ut + 1) * kbt) * C - 1) / U) - u_fw + 1;
                n_gate = g_n;
                total = g_n + u_n;
                slot = up ? g_n + ((int)blockIdx.x - u_fw) : ((int)blockIdx.x - g_fw);
            }
            float* part = p.scratch + ((size_t)L * p.max_slots + slot) * (size_t)(kTcRows * m);
            for (int r = 0; r < m; ++r) part[r * kTcRows + row] = acc[r];
            __threadfence();
            const uint32_t ph = (uint32_t)(flushes & 1);
            mbar_arrive(&fl_bar[0]);
            if (tid == 0) {
                if (mbar_wait(&fl_bar[0], ph, abort_flag, kTcWaitLimit)) {
                    const int old = atomicAdd(p.counters + L, 1);
                    *merge_flag = (old == total - 1) ? 1 : 0;
                } else {
                    *merge_flag = 0;
                }
                __threadfence_block();
                mbar_arrive(&fl_bar[1]);
            }
            if (!mbar_wait(&fl_bar[1], ph, abort_flag, kTcWaitLimit)) { ok = false; return; }
            ++flushes;
            if (*merge_flag) {
                __threadfence();
                const float* basep = p.scratch + (size_t)L * p.max_slots * (size_t)(kTcRows * m);
                const int orow = L * kTcRows + row;
                for (int r = 0; r < m; ++r) {
                    const float inv = 1.0f / row_scale[r];
                    if (EPI == kEpiSwiGLU) {
                        float gs = 0.f, us = 0.f;
                        for (int s = 0; s < n_gate; ++s) gs += __ldcg(basep + ((size_t)s * m + r) * kTcRows + row);
                        for (int s = n_gate; s < total; ++s) us += __ldcg(basep + ((size_t)s * m + r) * kTcRows + row);
                        gs *= inv;
                        us *= inv;
                        if (orow < (p.n >> 1)) p.y[(size_t)r * (p.n >> 1) + orow] = gs / (1.0f + expf(-gs)) * us;
                    } else {
                        float sum = 0.f;
                        for (int s = 0; s < total; ++s) sum += __ldcg(basep + ((size_t)s * m + r) * kTcRows + row);
                        sum *= inv;
                        if (orow < p.n) {
                            const size_t o = (size_t)r * p.n + orow;
                            if (p.flags & VSPEC_B200_F_RESIDUAL) sum += p.residual[o];
                            p.y[o] = sum;
                        }
                    }
                }
                if (tid == 0) p.counters[L] = 0;
            }
#pragma unroll
            for (int r = 0; r < kTcMaxM; ++r) acc[r] = 0.f;
        };

        for (int b0 = 0; ok && b0 < n_units + NA; b0 += NA) {
#pragma unroll
            for (int a = 0; a < NA; ++a) {
                const int i = b0 + a;
                // (A) epilogue of unit i - NA (TMEM stage a)
                if (ok && i >= NA && i - NA < n_units) {
                    if (!mbar_wait(&d_ready[a], (uint32_t)(((i - NA) / NA) & 1), abort_flag, kTcWaitLimit)) {
                        ok = false;
                    } else {
                        tc_fence_after();
                        float d[8];
                        tmem_ld_x8(tmem_base + lane_off + (uint32_t)(256 + 16 * a), d);
                        tmem_wait_ld();
                        const int kb = e_kb[a];
                        const float sv = sz_to_float(p.s ? e_s[a] : one_bits, sz16);
                        const float zv = p.zp ? sz_to_float(e_z[a], sz16) : p.zp_const;
                        (void)zc_bits;
#pragma unroll
                        for (int r = 0; r < kTcMaxM; ++r) {
                            if (r < m) {
                                const float dd = d[2 * r] + d[2 * r + 1];
                                acc[r] = fmaf(sv, dd - fmaf(zv, xs[kb * m + r], cs[kb * m + r]), acc[r]);
                            }
                        }
                        if (e_last[a]) flush(e_tile[a]);
                    }
                }
                // (B) decode unit i into TMEM stage a
                if (ok && i < n_units) {
                    const int s = i % NS;
                    if (!mbar_wait(&full[s], (uint32_t)((i / NS) & 1), abort_flag, kTcWaitLimit)) {
                        ok = false;
                    } else {
                        const unsigned char* st = wring + (size_t)s * STAGE_BYTES;
                        uint32_t words[4 * BITS];
#pragma unroll
                        for (int c16 = 0; c16 < BITS; ++c16) {
                            const uint4 v = *reinterpret_cast<const uint4*>(st + stage_chunk_offset<BITS>(row, c16));
                            words[4 * c16 + 0] = v.x;
                            words[4 * c16 + 1] = v.y;
                            words[4 * c16 + 2] = v.z;
                            words[4 * c16 + 3] = v.w;
                        }
                        mbar_arrive(&empty[s]);
                        // scale / zero-point of this row and k-block's group
                        int grow = c_tile * kTcRows + row;
                        grow = grow < p.n ? grow : p.n - 1;
                        const int grp = p.kb_per_group_shift >= 0 ? (c_kb >> p.kb_per_group_shift) : c_kb / p.kb_per_group;
                        // raw bits only: the loads complete while later units decode
                        const size_t sidx = (size_t)grow * p.n_groups + grp;
                        e_s[a] = load_sz_raw(p.s, sidx, sz16);
                        e_z[a] = load_sz_raw(p.zp, sidx, sz16);
                        e_kb[a] = c_kb;
                        e_tile[a] = c_tile;
                        e_last[a] = (c_kb == kbt - 1) || (i == n_units - 1);
                        // decode 4 chunks of 32 codes -> 64 fp16 pairs -> TMEM columns
                        uint32_t hv[32];
#pragma unroll
                        for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
                            for (int cc = 0; cc < 2; ++cc) {
                                Chunk<BITS> ch;
#pragma unroll
                                for (int w = 0; w < BITS; ++w) ch.w[w] = words[BITS * (2 * hh + cc) + w];
#pragma unroll
                                for (int mm = 0; mm < 8; ++mm)
                                    unpack_mm<BITS, UNSIGNED>(ch, mm, hv[16 * cc + 2 * mm], hv[16 * cc + 2 * mm + 1]);
                            }
                            tmem_st_x32(tmem_base + lane_off + (uint32_t)(64 * a + 32 * hh), hv);
                        }
                        tmem_wait_st();
                        tc_fence_before();
                        mbar_arrive(&a_ready[a]);
                        if (++c_kb == kbt) { c_kb = 0; ++c_tile; }
                    }
                }
            }
        }
        if (!ok) {
            *abort_flag = 1;
            atomicOr(&g_tc_timeout, 1);
        }
    } else if (warp == 4) {
        // ======================= TMA producer =================================
        if (lane == 0) {
            for (; p_issued < n_units; ++p_issued) {
                const int s = p_issued % NS;
                if (!mbar_wait(&empty[s], (uint32_t)(((p_issued / NS) - 1) & 1), abort_flag, kTcWaitLimit)) {
                    *abort_flag = 1;
                    atomicOr(&g_tc_timeout, 1);
                    break;
                }
                mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
                tma_load_2d(wring + (size_t)s * STAGE_BYTES, &wmap, p_kb * RB, p_tile * kTcRows, &full[s]);
                if (++p_kb == kbt) { p_kb = 0; ++p_tile; }
            }
            // drain: every issued copy must land before the CTA's smem goes away
            const int first = p_issued > NS ? p_issued - NS : 0;
            for (int i = first; i < p_issued; ++i)
                (void)mbar_wait(&full[i % NS], (uint32_t)((i / NS) & 1), abort_flag, kTcWaitLimit);
        }
    } else {
        // ======================= MMA issuer (warp 5) ===========================
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(128, 16);
            const uint32_t bfr_addr = smem_u32(bfr);
            int k_tile = u0 / kbt, k_kb = u0 - k_tile * kbt;
            (void)k_tile;
            for (int i = 0; i < n_units; ++i) {
                const int a = i % NA;
                if (!mbar_wait(&a_ready[a], (uint32_t)((i / NA) & 1), abort_flag, kTcWaitLimit)) {
                    *abort_flag = 1;
                    atomicOr(&g_tc_timeout, 1);
                    break;
                }
                tc_fence_after();
                const uint32_t b0 = bfr_addr + (uint32_t)k_kb * 16u * lbo;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint64_t bdesc = umma_desc_noswizzle(b0 + 2u * (uint32_t)j * lbo, lbo, 0u);
                    umma_f16_tmemA(tmem_base + (uint32_t)(256 + 16 * a), tmem_base + (uint32_t)(64 * a + 8 * j), bdesc,
                                   idesc, j > 0 ? 1u : 0u);
                }
                umma_commit(&d_ready[a]);
                if (++k_kb == kbt) { k_kb = 0; ++k_tile; }
            }
            // drain: all issued MMAs complete before TMEM is released
            umma_commit(drain_bar);
            volatile int never = 0;
            (void)mbar_wait(drain_bar, 0u, &never, kTcWaitLimit);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTcTmemCols);
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

template <int BITS>
static int make_weight_map(CUtensorMap* map, const uint8_t* w, int n, int row_bytes) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) { set_error("cuTensorMapEncodeTiled unavailable"); return VSPEC_B200_ERR_CUDA; }
    cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)n};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {(cuuint32_t)TcCfg<BITS>::kRowBytes, (cuuint32_t)kTcRows};
    cuuint32_t estr[2] = {1, 1};
    const CUtensorMapSwizzle swz = BITS == 4 ? CU_TENSOR_MAP_SWIZZLE_64B
                                 : (BITS == 2 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_NONE);
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(w), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) { set_error("cuTensorMapEncodeTiled failed (%d)", (int)r); return VSPEC_B200_ERR_CUDA; }
    return VSPEC_B200_OK;
}

bool gemv_tc_supported(const GemvParams& p, int bits) {
    if (p.m < 1 || p.m > kTcMaxM) return false;
    if (p.k % 128 != 0 || p.n_groups < 1 || p.k % p.n_groups != 0 || (p.k / p.n_groups) % 128 != 0) return false;
    if (reinterpret_cast<uintptr_t>(p.w) % 16 != 0 || reinterpret_cast<uintptr_t>(p.x) % 16 != 0) return false;
    if ((p.flags & VSPEC_B200_F_RMSNORM) && reinterpret_cast<uintptr_t>(p.norm_w) % 16 != 0) return false;
    if ((p.flags & VSPEC_B200_F_SWIGLU) && ((p.n / 2) % kTcRows != 0)) return false;
    const int kbt = p.k / 128;
    size_t total = 0;
    if (bits == 4) total = tc_smem_plan<4>(p.m, kbt).total;
    else if (bits == 3) total = tc_smem_plan<3>(p.m, kbt).total;
    else total = tc_smem_plan<2>(p.m, kbt).total;
    return total + 1024 <= 227 * 1024;
}

int gemv_tc_read_and_clear_timeout(int* out) {
    int v = 0, zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_tc_timeout, sizeof(int));
    if (e != cudaSuccess) return cuda_status(e, "read tensor-core timeout flag");
    e = cudaMemcpyToSymbol(g_tc_timeout, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_status(e, "clear tensor-core timeout flag");
    *out = v;
    return VSPEC_B200_OK;
}

template <int BITS, bool UNS, int EPI>
static cudaError_t launch_tc_t(const CUtensorMap& map, const GemvParams& p, int grid, size_t smem, cudaStream_t st,
                               bool pdl) {
    auto kern = lowbit_gemv_tc_kernel<BITS, UNS, EPI>;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        configured[dev] = 1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, map, p);
}

template <int BITS>
static cudaError_t launch_tc_bits(const CUtensorMap& map, const GemvParams& p, bool uns, bool swiglu, int grid,
                                  size_t smem, cudaStream_t st, bool pdl) {
    if (uns) return swiglu ? launch_tc_t<BITS, true, kEpiSwiGLU>(map, p, grid, smem, st, pdl)
                           : launch_tc_t<BITS, true, kEpiPlain>(map, p, grid, smem, st, pdl);
    return swiglu ? launch_tc_t<BITS, false, kEpiSwiGLU>(map, p, grid, smem, st, pdl)
                  : launch_tc_t<BITS, false, kEpiPlain>(map, p, grid, smem, st, pdl);
}

// p must already carry kb_total / kb_per_group(_shift) and the workspace.
int gemv_tc_launch(GemvParams p, int bits, int unsigned_codes, cudaStream_t st, bool pdl) {
    const bool swiglu = (p.flags & VSPEC_B200_F_SWIGLU) != 0;
    CUtensorMap map;
    int rc;
    if (bits == 4) rc = make_weight_map<4>(&map, p.w, p.n, p.row_bytes);
    else if (bits == 3) rc = make_weight_map<3>(&map, p.w, p.n, p.row_bytes);
    else rc = make_weight_map<2>(&map, p.w, p.n, p.row_bytes);
    if (rc != VSPEC_B200_OK) return rc;
    const int kbt = p.kb_total;
    p.tiles = (p.n + kTcRows - 1) / kTcRows;
    const long long U = (long long)p.tiles * kbt;
    const int sms = device_sm_count();
    const int grid = (int)(U < sms ? U : sms);
    const long long per = U / grid;
    int per_tile = (int)((kbt + per - 1) / per) + 1;
    if (per_tile > grid) per_tile = grid;
    p.max_slots = swiglu ? 2 * per_tile : per_tile;
    p.total_warps = grid;
    size_t smem = 0;
    if (bits == 4) smem = tc_smem_plan<4>(p.m, kbt).total;
    else if (bits == 3) smem = tc_smem_plan<3>(p.m, kbt).total;
    else smem = tc_smem_plan<2>(p.m, kbt).total;
    smem += 1024;   // manual 1024-byte alignment of the dynamic base
    // one CTA per SM: it owns all 512 TMEM columns
    if (smem < 120 * 1024) smem = 120 * 1024;
    cudaError_t e;
    if (bits == 4) e = launch_tc_bits<4>(map, p, unsigned_codes != 0, swiglu, grid, smem, st, pdl);
    else if (bits == 3) e = launch_tc_bits<3>(map, p, unsigned_codes != 0, swiglu, grid, smem, st, pdl);
    else e = launch_tc_bits<2>(map, p, unsigned_codes != 0, swiglu, grid, smem, st, pdl);
    if (e != cudaSuccess) return cuda_status(e, "lowbit_gemv_tc_kernel launch");
    return VSPEC_B200_OK;
}

// Scratch needed by the tcgen05 path (fp32 partials after the counter region).
size_t gemv_tc_scratch_floats(int m, int n, int k, bool swiglu) {
    const int kbt = k / 128;
    const int tiles = (n + kTcRows - 1) / kTcRows;
    const long long U = (long long)tiles * kbt;
    const int sms = device_sm_count();
    const int grid = (int)(U < sms ? U : sms);
    if (grid <= 0) return 0;
    const long long per = U / grid;
    int per_tile = (int)((kbt + per - 1) / per) + 1;
    if (per_tile > grid) per_tile = grid;
    const int slots = swiglu ? 2 * per_tile : per_tile;
    const int logical = swiglu ? tiles / 2 : tiles;
    return (size_t)logical * slots * kTcRows * m;
}

}  // namespace vb200
