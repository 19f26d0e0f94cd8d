// lowbit_gemv_tc.cu -- tcgen05 / TMEM / TMA low-bit GEMV for decode (M <= 4).
//
// Same contraction and numerics contract as lowbit_gemv.cu (group-wise
// dequant, fp32 activations split into fp16 hi + lo, fp32 accumulation), laid
// out for Blackwell:
//   * one persistent CTA per SM owns a contiguous run of (128-row tile,
//     128-code k-block) units (split-K across CTAs, deterministic merge);
//   * warp 8 (one thread) streams weight tiles with 2-D TMA into a shared
//     memory ring (~60-95 KB in flight per CTA);
//   * warps 0-7 decode straight from shared memory into tensor memory (the
//     MMA's A operand): warp w serves TMEM lane quarter w%4 (one weight row per
//     thread) and half w/4 of the k-block's 64 fp16 pairs;
//   * warp 9 owns TMEM and issues tcgen05.mma (M=128, N=16, K=16) with A in
//     TMEM and the activation fragments (B) in shared memory; the fp32
//     accumulator lives in TMEM and is read back per k-block for the
//     group-scale / zero-point epilogue, which the two decode halves take in
//     turns.
// A CTA holds 256 TMEM columns and at most ~113 KB of shared memory when the
// shape allows, so the next launch in the stream (programmatic dependent
// launch) can become resident beside it and prefetch its own weights.
//
// Activation scaling: every (k-block, row) gets its own exact power-of-two
// scale (max |x| of the block lands in [2^13, 2^14)), so the prologue needs
// no reduction across k-blocks and a CTA only prepares the k-blocks it uses.
// RMSNorm's row factor is applied once, at the merge.
//
// Every wait is bounded; a timeout raises a device flag, drains in-flight
// copies and MMAs, frees TMEM and returns.
#include "common.cuh"
#include "lowbit_decode.cuh"
#include "lowbit_kernels.cuh"
#include "tc_primitives.cuh"
#include "tma_map.cuh"

#include <cudaTypedefs.h>
#include <string.h>

namespace vb200 {

constexpr int kTcRows = 128;
constexpr int kTcDecodeWarps = 8;
constexpr int kTcDecodeThreads = kTcDecodeWarps * 32;
constexpr int kTcProducerWarp = 8;
constexpr int kTcMmaWarp = 9;
constexpr int kTcThreads = 10 * 32;
constexpr int kTcAStages = 3;
constexpr uint32_t kTcTmemCols = 256;
constexpr uint32_t kTcDCol = 64u * kTcAStages;   // first accumulator column
constexpr uint32_t kTcWaitLimit = 1u << 24;
constexpr int kTcMaxM = 4;
constexpr uint32_t kTcSmemShared = 113u * 1024u;  // two CTAs per SM
constexpr uint32_t kTcSmemMax = 227u * 1024u;

template <int BITS> struct TcCfg;
template <> struct TcCfg<4> { static constexpr int kRowBytes = 64; static constexpr int kMaxStages = 24; };
template <> struct TcCfg<3> { static constexpr int kRowBytes = 48; static constexpr int kMaxStages = 32; };
template <> struct TcCfg<2> { static constexpr int kRowBytes = 32; static constexpr int kMaxStages = 48; };

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
    uint32_t xs, cs, is;  // per (k-block, row): scaled sum, decode offset, inverse scale
    uint32_t red;         // [2][kTcMaxM][128] half-1 partials handed over at a flush
    uint32_t misc;
    uint32_t total;
};

template <int BITS>
__host__ __device__ inline TcSmem tc_smem_plan(int m, int kbt, int stages) {
    TcSmem s;
    const uint32_t stage = kTcRows * TcCfg<BITS>::kRowBytes;
    s.w_ring = 0;
    s.bfrag = (uint32_t)stages * stage;
    const uint32_t lbo = 32u * (uint32_t)m;
    const uint32_t bbytes = (uint32_t)kbt * 16u * lbo + 128u;
    s.xs = (s.bfrag + bbytes + 15u) & ~15u;
    s.cs = s.xs + (uint32_t)(kbt * m) * 4u;
    s.is = s.cs + (uint32_t)(kbt * m) * 4u;
    s.red = (s.is + (uint32_t)(kbt * m) * 4u + 15u) & ~15u;
    s.misc = s.red + 2u * kTcMaxM * kTcRows * 4u;
    // barriers: full/empty per ring stage, a_ready/d_ready per TMEM stage,
    // 3 flush barriers, 1 drain barrier; then slot, flags, row norms
    s.total = s.misc + 8u * (2u * (uint32_t)stages + 2u * kTcAStages + 4u) + 64u;
    return s;
}

// Flush of one finished tile part (all 256 decode threads, same order).
// Half 1 handed its partial over in red[parity]; half 0 adds its own, writes
// the CTA's slot, and the CTA that completes the tile's contributor count
// merges all slots in slot order.  Returns false when a bounded wait gave up.
template <int EPI>
__device__ __noinline__ bool tc_flush(const GemvParams& p, int tile, int row, int half, float a0, float a1, float a2,
                                      float a3, const float* red, uint64_t* fl_bar, uint32_t ph,
                                      volatile int* abort_flag, volatile int* merge_flag, const float* row_norm) {
    const int m = p.m;
    const int kbt = p.kb_total;
    const long long U = (long long)p.tiles * kbt;
    const long long C = gridDim.x;
    mbar_arrive(&fl_bar[0]);
    if (!mbar_wait(&fl_bar[0], ph, abort_flag, kTcWaitLimit)) return false;
    if (half != 0) return true;
    const int tid = threadIdx.x;
    auto first_cta = [&](long long u) { return (int)(((u + 1) * C - 1) / U); };
    int L = tile;
    int slot = (int)blockIdx.x - first_cta((long long)tile * kbt);
    int total = first_cta((long long)(tile + 1) * kbt - 1) - first_cta((long long)tile * kbt) + 1;
    int n_gate = total;
    if (EPI == kEpiSwiGLU) {
        const int half_tiles = p.tiles >> 1;
        const bool up = tile >= half_tiles;
        L = up ? tile - half_tiles : tile;
        const int gt = L, ut = L + half_tiles;
        const int g_fw = first_cta((long long)gt * kbt);
        const int g_n = first_cta((long long)(gt + 1) * kbt - 1) - g_fw + 1;
        const int u_fw = first_cta((long long)ut * kbt);
        const int u_n = first_cta((long long)(ut + 1) * kbt - 1) - u_fw + 1;
        n_gate = g_n;
        total = g_n + u_n;
        slot = up ? g_n + ((int)blockIdx.x - u_fw) : ((int)blockIdx.x - g_fw);
    }
    const float mine[kTcMaxM] = {a0, a1, a2, a3};
    float* part = p.scratch + ((size_t)L * p.max_slots + slot) * (size_t)(kTcRows * m);
    for (int r = 0; r < m; ++r) part[r * kTcRows + row] = mine[r] + red[r * kTcRows + row];
    __threadfence();
    mbar_arrive(&fl_bar[1]);
    if (tid == 0) {
        if (mbar_wait(&fl_bar[1], ph, abort_flag, kTcWaitLimit)) {
            const int old = atomicAdd(p.counters + L, 1);
            *merge_flag = (old == total - 1) ? 1 : 0;
        } else {
            *merge_flag = 0;
        }
        __threadfence_block();
        mbar_arrive(&fl_bar[2]);
    }
    if (!mbar_wait(&fl_bar[2], ph, abort_flag, kTcWaitLimit)) return false;
    if (*merge_flag) {
        __threadfence();
        const float* basep = p.scratch + (size_t)L * p.max_slots * (size_t)(kTcRows * m);
        const int orow = L * kTcRows + row;
        const bool rms = EPI_HAS_RMSNORM(p.flags);
        for (int r = 0; r < m; ++r) {
            const float nr = rms ? row_norm[r] : 1.0f;
            if (EPI == kEpiSwiGLU) {
                float gs = 0.f, us = 0.f;
                for (int s = 0; s < n_gate; ++s) gs += __ldcg(basep + ((size_t)s * m + r) * kTcRows + row);
                for (int s = n_gate; s < total; ++s) us += __ldcg(basep + ((size_t)s * m + r) * kTcRows + row);
                gs *= nr;
                us *= nr;
                if (orow < (p.n >> 1)) p.y[(size_t)r * (p.n >> 1) + orow] = gs / (1.0f + expf(-gs)) * us;
            } else {
                float sum = 0.f;
                for (int s = 0; s < total; ++s) sum += __ldcg(basep + ((size_t)s * m + r) * kTcRows + row);
                sum *= nr;
                if (orow < p.n) {
                    const size_t o = (size_t)r * p.n + orow;
                    if (p.flags & VSPEC_B200_F_RESIDUAL) sum += p.residual[o];
                    p.y[o] = sum;
                }
            }
        }
        if (tid == 0) p.counters[L] = 0;
    }
    return true;
}

template <int BITS, bool UNSIGNED, int EPI>
__global__ void __launch_bounds__(kTcThreads, 2)
lowbit_gemv_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ GemvParams p) {
    constexpr int RB = TcCfg<BITS>::kRowBytes;
    constexpr uint32_t STAGE_BYTES = kTcRows * RB;
    constexpr int NA = kTcAStages;
    const int NS = p.stages;

    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    unsigned char* base = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    const int m = p.m;
    const int kbt = p.kb_total;
    const TcSmem plan = tc_smem_plan<BITS>(m, kbt, NS);
    const uint32_t lbo = 32u * (uint32_t)m;   // activation fragment K-chunk stride (2m rows of 16 B)

    unsigned char* wring = base + plan.w_ring;
    unsigned char* bfr = base + plan.bfrag;
    float* xs = reinterpret_cast<float*>(base + plan.xs);
    float* cs = reinterpret_cast<float*>(base + plan.cs);
    float* isc = reinterpret_cast<float*>(base + plan.is);
    float* red = reinterpret_cast<float*>(base + plan.red);
    uint64_t* full = reinterpret_cast<uint64_t*>(base + plan.misc);
    uint64_t* empty = full + NS;
    uint64_t* a_ready = empty + NS;
    uint64_t* d_ready = a_ready + NA;
    uint64_t* fl_bar = d_ready + NA;          // [3] flush rendezvous
    uint64_t* drain_bar = fl_bar + 3;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* merge_flag = abort_flag + 1;
    float* row_norm = reinterpret_cast<float*>(tmem_slot + 4);   // [4]

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
            mbar_init(&empty[s], kTcDecodeThreads);
        }
        for (int a = 0; a < NA; ++a) {
            mbar_init(&a_ready[a], kTcDecodeThreads);
            mbar_init(&d_ready[a], 1);
        }
        mbar_init(&fl_bar[0], kTcDecodeThreads);
        mbar_init(&fl_bar[1], kTcDecodeThreads / 2);
        mbar_init(&fl_bar[2], 1);
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == kTcMmaWarp) {
        tmem_alloc(tmem_slot, kTcTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // the next launch in the stream may become resident and stage its weights
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");

    // ---- producer: first ring fill (weights only: no dependency on x) ----
    int p_issued = 0;
    int p_tile = u0 / (kbt > 0 ? kbt : 1), p_kb = u0 - p_tile * kbt;
    if (warp == kTcProducerWarp && lane == 0) {
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
        for (int r = warp; r < m; r += kTcThreads / 32) {
            const float4* xr = reinterpret_cast<const float4*>(p.x + (size_t)r * K);
            float ss = 0.f;
            for (int t = lane; t < K / 4; t += 32) {
                const float4 v = xr[t];
                ss += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
            }
            ss = warp_sum(ss);
            if (lane == 0) row_norm[r] = 1.0f / sqrtf(ss / (float)K + p.eps);
        }
    }
    {
        // k-blocks this CTA's units touch: all, or a (wrapping) run
        const int kb_first = n_units >= kbt ? 0 : u0 % kbt;
        const int kb_count = n_units >= kbt ? kbt : n_units;
        constexpr float kOff = (float)(1 << (BITS - 1));
        float imul[4];
        int boff[4];   // byte offset of code 4*lane+e inside a k-block's fragments
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int t = 4 * lane + e;
            const int j = t & 31;
            imul[e] = code_inv_mult<BITS>(j);
            int q, hh;
            code_slot<BITS>(j, q, hh);
            const int col = 16 * (t >> 5) + q;
            boff[e] = (col >> 2) * (int)lbo + 2 * ((2 * col + hh) & 7);
        }
        for (int pr = warp; pr < kb_count * m; pr += kTcThreads / 32) {
            const int r = pr % m;
            int kb = kb_first + pr / m;
            if (kb >= kbt) kb -= kbt;
            const int t = kb * 128 + lane * 4;
            float4 v = *reinterpret_cast<const float4*>(p.x + (size_t)r * K + t);
            if (rms) {
                const float4 wn = *reinterpret_cast<const float4*>(p.norm_w + t);
                v.x *= wn.x; v.y *= wn.y; v.z *= wn.z; v.w *= wn.w;
            }
            const float amax = warp_max(fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
            // sc = 2^(13 - floor(log2 amax)), built from the exponent bits
            int sbits = 127;
            if (amax > 0.f && isfinite(amax)) {
                const int e = (int)((__float_as_uint(amax) >> 23) & 0xFFu);
                sbits = 267 - e;
                sbits = sbits < 1 ? 1 : (sbits > 253 ? 253 : sbits);
            }
            const float sc = __uint_as_float((uint32_t)sbits << 23);
            const float inv_sc = __uint_as_float((uint32_t)(254 - sbits) << 23);
            const float vv[4] = {v.x * sc, v.y * sc, v.z * sc, v.w * sc};
            const float sx = warp_sum((vv[0] + vv[1]) + (vv[2] + vv[3]));
            const float sw = warp_sum((vv[0] * imul[0] + vv[1] * imul[1]) + (vv[2] * imul[2] + vv[3] * imul[3]));
            if (lane == 0) {
                xs[kb * m + r] = sx;
                cs[kb * m + r] = fmaf(1024.0f, sw, kOff * sx);
                isc[kb * m + r] = inv_sc;
            }
            unsigned char* fb = bfr + (size_t)kb * 16 * lbo + 32 * r;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float val = vv[e] * imul[e];
                const __half hv = __float2half_rn(val);
                const __half lv = __float2half_rn(val - __half2float(hv));
                *reinterpret_cast<__half*>(fb + boff[e]) = hv;
                *reinterpret_cast<__half*>(fb + boff[e] + 16) = lv;
            }
        }
        if (tid < 8) *reinterpret_cast<uint4*>(bfr + (size_t)kbt * 16 * lbo + 16 * tid) = make_uint4(0, 0, 0, 0);
    }
    // make the generic-proxy smem writes (B fragments) visible to the tensor core
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    __syncthreads();

    if (warp < kTcDecodeWarps) {
        // ======================= decode warps =================================
        const int quarter = warp & 3;
        const int half = warp >> 2;
        const int row = quarter * 32 + lane;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        const bool sz16 = (p.flags & VSPEC_B200_F_SZ_F16) != 0;
        const bool has_s = p.s != nullptr, has_zp = p.zp != nullptr;
        float acc[kTcMaxM] = {0.f, 0.f, 0.f, 0.f};
        uint32_t e_s[NA], e_z[NA];
        int e_kb[NA], e_tile[NA];
        bool e_last[NA];
        int c_tile = u0 / kbt, c_kb = u0 - c_tile * kbt;
        int ring = 0;
        uint32_t ring_ph = 0;
        uint32_t blk_ph = 0;   // parity of (b0 / NA)
        uint32_t flushes = 0;
        bool ok = true;

        for (int b0 = 0; ok && b0 < n_units + NA - 1; b0 += NA, blk_ph ^= 1u) {
#pragma unroll
            for (int a = 0; a < NA; ++a) {
                const int i = b0 + a;
                // (A) decode unit i into TMEM stage a
                if (ok && i < n_units) {
                    if (!mbar_wait(&full[ring], ring_ph, abort_flag, kTcWaitLimit)) {
                        ok = false;
                    } else {
                        const unsigned char* st = wring + (size_t)ring * STAGE_BYTES;
                        uint32_t words[2 * BITS];
                        if constexpr (BITS == 4) {
#pragma unroll
                            for (int c16 = 0; c16 < 2; ++c16) {
                                const uint4 v = *reinterpret_cast<const uint4*>(st + stage_chunk_offset<4>(row, 2 * half + c16));
                                words[4 * c16 + 0] = v.x; words[4 * c16 + 1] = v.y;
                                words[4 * c16 + 2] = v.z; words[4 * c16 + 3] = v.w;
                            }
                        } else if constexpr (BITS == 2) {
                            const uint4 v = *reinterpret_cast<const uint4*>(st + stage_chunk_offset<2>(row, half));
                            words[0] = v.x; words[1] = v.y; words[2] = v.z; words[3] = v.w;
                        } else {
#pragma unroll
                            for (int c8 = 0; c8 < 3; ++c8) {
                                const uint2 v = *reinterpret_cast<const uint2*>(st + row * 48 + 24 * half + 8 * c8);
                                words[2 * c8] = v.x; words[2 * c8 + 1] = v.y;
                            }
                        }
                        // released after the TMEM store below has consumed the
                        // words (a release right after the loads let the refill
                        // land before the loads had read the stage)
                        const int stage_used = ring;
                        if (++ring == NS) { ring = 0; ring_ph ^= 1u; }
                        if ((i & 1) == half) {
                            // scale / zero-point of this row and k-block's group, as
                            // raw bits: the loads complete while later units decode
                            int grow = c_tile * kTcRows + row;
                            grow = grow < p.n ? grow : p.n - 1;
                            const int grp = p.kb_per_group_shift >= 0 ? (c_kb >> p.kb_per_group_shift) : c_kb / p.kb_per_group;
                            const size_t sidx = (size_t)grow * p.n_groups + grp;
                            e_s[a] = has_s ? load_sz_raw(p.s, sidx, sz16) : 0u;
                            e_z[a] = has_zp ? load_sz_raw(p.zp, sidx, sz16) : 0u;
                        }
                        e_kb[a] = c_kb;
                        e_tile[a] = c_tile;
                        e_last[a] = (c_kb == kbt - 1) || (i == n_units - 1);
                        uint32_t hv[32];
#pragma unroll
                        for (int cc = 0; cc < 2; ++cc) {
                            Chunk<BITS> ch;
#pragma unroll
                            for (int w = 0; w < BITS; ++w) ch.w[w] = words[BITS * cc + w];
#pragma unroll
                            for (int mm = 0; mm < 8; ++mm)
                                unpack_mm<BITS, UNSIGNED>(ch, mm, hv[16 * cc + 2 * mm], hv[16 * cc + 2 * mm + 1]);
                        }
                        tmem_st_x32(tmem_base + lane_off + (uint32_t)(64 * a + 32 * half), hv);
                        mbar_arrive(&empty[stage_used]);
                        if (++c_kb == kbt) { c_kb = 0; ++c_tile; }
                    }
                }
                // (B) epilogue of unit j = i + 1 - NA (TMEM stage (a + 1) % NA)
                const int aj = (a + 1) % NA;   // a constant after unrolling
                const int j = i + 1 - NA;
                if (ok && j >= 0 && j < n_units) {
                    const uint32_t par = (a + 1 < NA) ? (blk_ph ^ 1u) : blk_ph;
                    if (!mbar_wait(&d_ready[aj], par, abort_flag, kTcWaitLimit)) {
                        ok = false;
                    } else {
                        tc_fence_after();
                        if ((j & 1) == half) {
                            float d[8];
                            tmem_ld_x8(tmem_base + lane_off + kTcDCol + (uint32_t)(16 * aj), d);
                            tmem_wait_ld();
                            const int kb = e_kb[aj];
                            const float sv = has_s ? sz_to_float(e_s[aj], sz16) : 1.0f;
                            const float zv = has_zp ? sz_to_float(e_z[aj], sz16) : p.zp_const;
#pragma unroll
                            for (int r = 0; r < kTcMaxM; ++r) {
                                if (r < m) {
                                    const float dd = d[2 * r] + d[2 * r + 1];
                                    acc[r] = fmaf(sv * isc[kb * m + r], dd - fmaf(zv, xs[kb * m + r], cs[kb * m + r]),
                                                  acc[r]);
                                }
                            }
                        }
                        if (e_last[aj]) {
                            float* rb = red + (flushes & 1u) * (kTcMaxM * kTcRows);
                            if (half) {
#pragma unroll
                                for (int r = 0; r < kTcMaxM; ++r)
                                    if (r < m) rb[r * kTcRows + row] = acc[r];
                            }
                            ok = tc_flush<EPI>(p, e_tile[aj], row, half, acc[0], acc[1], acc[2], acc[3], rb, fl_bar,
                                               flushes & 1u, abort_flag, merge_flag, row_norm);
                            ++flushes;
#pragma unroll
                            for (int r = 0; r < kTcMaxM; ++r) acc[r] = 0.f;
                        }
                    }
                }
                // (C) unit i's A operand is in TMEM: hand it to the MMA warp
                if (ok && i < n_units) {
                    tmem_wait_st();
                    tc_fence_before();
                    mbar_arrive(&a_ready[a]);
                }
            }
        }
        if (!ok) {
            *abort_flag = 1;
            atomicOr(&g_tc_timeout, 1);
        }
    } else if (warp == kTcProducerWarp) {
        // ======================= TMA producer =================================
        if (lane == 0) {
            int s = p_issued % (NS > 0 ? NS : 1);
            uint32_t ph = (uint32_t)((p_issued / NS) & 1);
            for (; p_issued < n_units; ++p_issued) {
                // stage s was last filled by copy p_issued - NS (phase ph ^ 1)
                if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, kTcWaitLimit)) {
                    *abort_flag = 1;
                    atomicOr(&g_tc_timeout, 1);
                    break;
                }
                mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
                tma_load_2d(wring + (size_t)s * STAGE_BYTES, &wmap, p_kb * RB, p_tile * kTcRows, &full[s]);
                if (++p_kb == kbt) { p_kb = 0; ++p_tile; }
                if (++s == NS) { s = 0; ph ^= 1u; }
            }
            // drain: every issued copy must land before the CTA's smem goes away
            const int first = p_issued > NS ? p_issued - NS : 0;
            for (int i = first; i < p_issued; ++i)
                (void)mbar_wait_drain(&full[i % NS], (uint32_t)((i / NS) & 1), 1u << 16);
        }
    } else {
        // ======================= MMA issuer (warp 9) ==========================
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(128, 16);
            const uint32_t bfr_addr = smem_u32(bfr);
            int k_kb = u0 % (kbt > 0 ? kbt : 1);
            int a = 0;
            uint32_t ph = 0;
            for (int i = 0; i < n_units; ++i) {
                if (!mbar_wait(&a_ready[a], ph, abort_flag, kTcWaitLimit)) {
                    *abort_flag = 1;
                    atomicOr(&g_tc_timeout, 1);
                    break;
                }
                tc_fence_after();
                const uint32_t b0 = bfr_addr + (uint32_t)k_kb * 16u * lbo;
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) {
                    const uint64_t bdesc = umma_desc_noswizzle(b0 + 2u * (uint32_t)jj * lbo, lbo, 0u);
                    umma_f16_tmemA(tmem_base + kTcDCol + (uint32_t)(16 * a), tmem_base + (uint32_t)(64 * a + 8 * jj),
                                   bdesc, idesc, jj > 0 ? 1u : 0u);
                }
                umma_commit(&d_ready[a]);
                if (++k_kb == kbt) k_kb = 0;
                if (++a == NA) { a = 0; ph ^= 1u; }
            }
            // drain: all issued MMAs complete before TMEM is released
            umma_commit(drain_bar);
            volatile int never = 0;
            (void)mbar_wait(drain_bar, 0u, &never, kTcWaitLimit);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kTcMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTcTmemCols);
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
template <int BITS>
static int make_weight_map(CUtensorMap* map, const uint8_t* w, int n, int row_bytes) {
    const CUtensorMapSwizzle swz = BITS == 4 ? CU_TENSOR_MAP_SWIZZLE_64B
                                 : (BITS == 2 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_NONE);
    return make_row_tile_map(map, w, n, row_bytes, TcCfg<BITS>::kRowBytes, kTcRows, swz);
}

// Ring depth and dynamic shared memory for a shape: the deepest ring that
// still lets two CTAs share an SM (so the next launch can overlap), or, when
// the activation fragments are too large for that, the deepest ring one CTA
// can hold.  Returns 0 when not even 4 stages fit.
template <int BITS>
static int tc_pick_stages(int m, int kbt, size_t* smem_bytes) {
    const uint32_t stage = kTcRows * TcCfg<BITS>::kRowBytes + 16u;   // ring bytes + 2 barriers
    const uint32_t fixed = tc_smem_plan<BITS>(m, kbt, 0).total + 1024u;   // + base alignment
    int ns = fixed < kTcSmemShared ? (int)((kTcSmemShared - fixed) / stage) : 0;
    if (ns > TcCfg<BITS>::kMaxStages) ns = TcCfg<BITS>::kMaxStages;
    if (ns < 8) {
        ns = fixed < kTcSmemMax ? (int)((kTcSmemMax - fixed) / stage) : 0;
        if (ns > TcCfg<BITS>::kMaxStages) ns = TcCfg<BITS>::kMaxStages;
    }
    if (ns < 4) return 0;
    *smem_bytes = tc_smem_plan<BITS>(m, kbt, ns).total + 1024u;
    return ns;
}

static int tc_stages_for(int bits, int m, int kbt, size_t* smem_bytes) {
    if (bits == 4) return tc_pick_stages<4>(m, kbt, smem_bytes);
    if (bits == 3) return tc_pick_stages<3>(m, kbt, smem_bytes);
    return tc_pick_stages<2>(m, kbt, smem_bytes);
}

bool gemv_tc_supported(const GemvParams& p, int bits, size_t counter_slots) {
    if (p.m < 1 || p.m > kTcMaxM) return false;
    const int tiles = (p.n + kTcRows - 1) / kTcRows;
    const int logical = (p.flags & VSPEC_B200_F_SWIGLU) ? tiles / 2 : tiles;
    if ((size_t)logical > counter_slots) return false;
    if (p.k % 128 != 0 || p.n_groups < 1 || p.k % p.n_groups != 0 || (p.k / p.n_groups) % 128 != 0) return false;
    if (reinterpret_cast<uintptr_t>(p.w) % 16 != 0 || reinterpret_cast<uintptr_t>(p.x) % 16 != 0) return false;
    if ((p.flags & VSPEC_B200_F_RMSNORM) && reinterpret_cast<uintptr_t>(p.norm_w) % 16 != 0) return false;
    if ((p.flags & VSPEC_B200_F_SWIGLU) && ((p.n / 2) % kTcRows != 0)) return false;
    size_t smem = 0;
    return tc_stages_for(bits, p.m, p.k / 128, &smem) > 0;
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
        // the largest carveout, so two CTAs (this launch and the next) can share an SM
        e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
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
    p.stages = tc_stages_for(bits, p.m, kbt, &smem);
    if (p.stages <= 0) { set_error("shape too large for the tcgen05 GEMV"); return VSPEC_B200_ERR_UNSUPPORTED; }
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
