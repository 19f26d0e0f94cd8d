// lowbit_gemm_tc.cu -- tcgen05 / TMEM / TMA low-bit GEMM for prefill and large
// batch (M > 8): Y[M][N] = X[M][K] . dequant(W)[N][K]^T.
//
// Same contraction as the GEMV (src/quant/int4.c:107-132 with the group
// indexing of src/kernel/cuda/fused_linear_int4.cu:391-396, bitstream of
// src/quant/pack.c:53-74), computed on the 5th-generation tensor cores with
// dequantisation fused into the operand load:
//   * a pre-pass converts X to fp16 with an exact per-row power-of-two scale
//     (max |x| in [2^14, 2^15)), applies the RMSNorm input epilogue, and stores
//     each 128-code block in the order the weight decoder produces pairs, so
//     no shuffle is needed on either operand;
//   * output tiles are 128 weight rows x BN tokens (BN <= 256; SwiGLU pairs a
//     gate and an up tile, BN <= 128); persistent CTAs (one per SM) take work
//     items = (tile, K range) round-robin, the K range being the whole of K or,
//     when tiles are too few for the SMs, an equal share of it;
//   * warp 4 (one thread) streams weight tiles (2-D TMA, 64B/32B swizzle) and
//     activation tiles (2-D TMA, 128-byte swizzle, the MMA's K-major B
//     layout) through shared-memory rings;
//   * warps 0-3 decode one weight row per thread into fp16 (code - zp) * s --
//     magic-number LOP3, then two f16x2 FMAs -- and store the MMA's A operand
//     into tensor memory (tcgen05.st, two stages);
//   * warp 5 issues tcgen05.mma.cta_group::1.kind::f16 (M=128, N=BN, K=16,
//     A from TMEM, B from shared memory), accumulating the whole K range in
//     TMEM; tcgen05.commit recycles the A and B stages;
//   * warps 0-3 then read the accumulator (tcgen05.ld), undo the activation
//     scale and apply residual / SwiGLU; a tile split along K is published as
//     fp32 partials that gemm_merge_kernel, launched right after over the
//     whole GPU, sums in K order (deterministic).
// Numerics: fp16 operands (dequantised weight rounded once to fp16, x to
// fp16 after the exact row scale), fp32 accumulation: the tensor-core
// tolerance 2e-2 applies, observed errors are ~1e-3.
// Every wait is bounded; a timeout raises a device flag and returns.
#include "common.cuh"
#include "lowbit_decode.cuh"
#include "lowbit_kernels.cuh"
#include "tc_primitives.cuh"
#include "tma_map.cuh"

#include <stdlib.h>
#include <string.h>

namespace vb200 {

constexpr int kGmRows = 128;                   // weight rows per tile (MMA M)
constexpr int kGmThreads = 6 * 32;             // 4 decode/epilogue warps, TMA warp, MMA warp
constexpr int kGmProducerWarp = 4;
constexpr int kGmMmaWarp = 5;
constexpr uint32_t kGmTmemCols = 512;
constexpr uint32_t kGmWaitLimit = 1u << 16;    // checks of up to kGmSleepNs each
constexpr uint32_t kGmSleepNs = 20000;
constexpr uint32_t kGmSmemMax = 227u * 1024u;
constexpr int kGmScalePipe = 4;                // k-blocks of scale loads in flight per decode thread

// Set when a bounded wait of the GEMM gave up.
__device__ int g_gemm_timeout = 0;

struct GemmParams {
    const uint8_t* w;
    const void* s;
    const void* zp;
    float zp_const;
    float* y;
    const float* residual;
    const float* xinv;       // [m] inverse row scales of the fp16 activations
    float* scratch;          // [tiles][splits] fp32 partials of tiles split along K
    int m, n, k, n_groups;
    int row_bytes, kb_total, kb_per_group, kb_per_group_shift;
    int flags;
    int bn, wtiles, ttiles, splits, kb_per_split, items;
    int nsw, nsb;            // ring depths (weights, activations)
    int half_n;              // SwiGLU: offset of the up rows
};

template <int BITS> struct GmCfg;
template <> struct GmCfg<4> { static constexpr int kRowBytes = 64; };
template <> struct GmCfg<3> { static constexpr int kRowBytes = 48; };
template <> struct GmCfg<2> { static constexpr int kRowBytes = 32; };

// Byte offset of 16-byte chunk c of weight row r inside a TMA stage (the
// swizzle of the weight tensor map).
template <int BITS>
__device__ __forceinline__ uint32_t gm_chunk_offset(int r, int c) {
    if constexpr (BITS == 4) return (uint32_t)(r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
    else if constexpr (BITS == 2) return (uint32_t)(r * 32 + ((c ^ ((r >> 2) & 1)) << 4));
    else return (uint32_t)(r * 48 + (c << 4));
}

// fp16 pair constants of decoded pair q: the halves carry 1024 + mult*u, so
// code = (h - 1024)/mult - 2^(bits-1) = h * im + c with im = 1/mult exact.
template <int BITS, int Q> struct GmPairConst {
    static constexpr uint32_t im = f16x2_bits(1.0 / code_mult<BITS>(lo_code<BITS>(Q)),
                                              1.0 / code_mult<BITS>(hi_code<BITS>(Q)));
    static constexpr uint32_t c = f16x2_bits(-1024.0 / code_mult<BITS>(lo_code<BITS>(Q)) - (1 << (BITS - 1)),
                                             -1024.0 / code_mult<BITS>(hi_code<BITS>(Q)) - (1 << (BITS - 1)));
};
template <int BITS>
__device__ __forceinline__ void gm_pair_const(int q, uint32_t& im, uint32_t& c) {
    switch (q) {   // q is a constant after unrolling
#define VB_GM_Q(Q) case Q: im = GmPairConst<BITS, Q>::im; c = GmPairConst<BITS, Q>::c; break;
        VB_GM_Q(0) VB_GM_Q(1) VB_GM_Q(2) VB_GM_Q(3) VB_GM_Q(4) VB_GM_Q(5) VB_GM_Q(6) VB_GM_Q(7)
        VB_GM_Q(8) VB_GM_Q(9) VB_GM_Q(10) VB_GM_Q(11) VB_GM_Q(12) VB_GM_Q(13) VB_GM_Q(14)
        default: im = GmPairConst<BITS, 15>::im; c = GmPairConst<BITS, 15>::c; break;
#undef VB_GM_Q
    }
}

// Position p (0..127) of a 128-code block in the activation order: pair
// column col = p/2 of the decoder holds codes (lo_code, hi_code) of pair
// q = col%16 of 32-code chunk col/16.
template <int BITS>
__host__ __device__ __forceinline__ int gm_src_code(int p) {
    const int col = p >> 1, c32 = col >> 4, q = col & 15;
    return 32 * c32 + ((p & 1) ? hi_code<BITS>(q) : lo_code<BITS>(q));
}

// ---------------------------------------------------------------------------
// Pre-pass: x (fp32, optional RMSNorm) -> fp16 rows in decoder order.
// ---------------------------------------------------------------------------
constexpr int kGmPrepThreads = 512;

template <int BITS>
__global__ void __launch_bounds__(kGmPrepThreads)
gemm_prep_x_kernel(const float* __restrict__ x, const float* __restrict__ norm_w, float eps, int rms, int k,
                   __half* __restrict__ xh, float* __restrict__ xinv) {
    __shared__ float red[2][kGmPrepThreads / 32];
    pdl_wait();
    // the GEMM may start its set-up and weight prefetch now (it waits for
    // this grid to complete before it reads the rows)
    pdl_trigger();
    const int row = blockIdx.x;
    const float* xr = x + (size_t)row * k;
    const float4* xr4 = reinterpret_cast<const float4*>(xr);
    const float4* nw4 = reinterpret_cast<const float4*>(norm_w);
    const int k4 = k / 4;
    constexpr int NWARP = kGmPrepThreads / 32;
    // pass 1: sum of squares (RMSNorm) and max |x * norm_w| (the latter is
    // rescaled by the row factor afterwards: both are positive scalings)
    float ss = 0.f, mx = 0.f;
    for (int t = threadIdx.x; t < k4; t += kGmPrepThreads) {
        const float4 v = xr4[t];
        ss += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
        float4 u = v;
        if (rms) {
            const float4 w = nw4[t];
            u.x *= w.x; u.y *= w.y; u.z *= w.z; u.w *= w.w;
        }
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(u.x), fabsf(u.y)), fmaxf(fabsf(u.z), fabsf(u.w))));
    }
    ss = warp_sum(ss);
    mx = warp_max(mx);
    if ((threadIdx.x & 31) == 0) { red[0][threadIdx.x >> 5] = ss; red[1][threadIdx.x >> 5] = mx; }
    __syncthreads();
    ss = 0.f;
    mx = 0.f;
#pragma unroll
    for (int w = 0; w < NWARP; ++w) { ss += red[0][w]; mx = fmaxf(mx, red[1][w]); }
    const float nr = rms ? 1.0f / sqrtf(ss / (float)k + eps) : 1.0f;
    mx *= nr;
    // sc = 2^(14 - floor(log2 max)): max lands in [2^14, 2^15), below fp16 max
    int sbits = 127;
    if (mx > 0.f && isfinite(mx)) {
        sbits = 268 - (int)((__float_as_uint(mx) >> 23) & 0xFFu);
        sbits = sbits < 1 ? 1 : (sbits > 253 ? 253 : sbits);
    }
    const float sc = __uint_as_float((uint32_t)sbits << 23);
    const float f = rms ? nr * sc : sc;
    if (threadIdx.x == 0) xinv[row] = __uint_as_float((uint32_t)(254 - sbits) << 23);
    // pass 2: eight consecutive output positions per thread (one 16-byte
    // store), gathered from the same 128-code block of x
    uint4* out = reinterpret_cast<uint4*>(xh + (size_t)row * k);
    for (int i = threadIdx.x; i < k / 8; i += kGmPrepThreads) {
        const int p0 = 8 * i;
        const int blk = p0 & ~127;
        uint32_t h2[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int ta = blk + gm_src_code<BITS>((p0 + 2 * e) & 127);
            const int tb = blk + gm_src_code<BITS>((p0 + 2 * e + 1) & 127);
            float va = xr[ta] * f, vb = xr[tb] * f;
            if (rms) { va *= norm_w[ta]; vb *= norm_w[tb]; }
            const __half2 hp = __floats2half2_rn(va, vb);
            h2[e] = *reinterpret_cast<const uint32_t*>(&hp);
        }
        out[i] = make_uint4(h2[0], h2[1], h2[2], h2[3]);
    }
}

// ---------------------------------------------------------------------------
// GEMM kernel
// ---------------------------------------------------------------------------
struct GmSmem {
    uint32_t b_ring, w_ring, misc, xsc, total;
};

template <int BITS>
__host__ __device__ inline GmSmem gm_smem_plan(int bn, int nw, int nsw, int nsb) {
    GmSmem s;
    s.b_ring = 0;                                                   // 1024-aligned stages
    s.w_ring = (uint32_t)nsb * (uint32_t)bn * 256u;
    s.misc = s.w_ring + (uint32_t)nsw * kGmRows * GmCfg<BITS>::kRowBytes * (uint32_t)nw;
    s.misc = (s.misc + 15u) & ~15u;
    // barriers: w full/empty, b full/empty, a full/empty (<= 4 groups), d full/empty, drain; slot + flags
    s.xsc = s.misc + ((8u * (2u * nsw + 2u * nsb + 8u + 2u + 1u) + 64u + 15u) & ~15u);
    s.total = s.xsc + 256u * 4u;   // + one tile's inverse activation scales (BN <= 256)
    return s;
}

template <int BITS, bool UNSIGNED, bool SWIGLU>
__global__ void __launch_bounds__(kGmThreads, 1)
lowbit_gemm_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                      const __grid_constant__ GemmParams p) {
    constexpr int RB = GmCfg<BITS>::kRowBytes;
    constexpr int NW = SWIGLU ? 2 : 1;                  // weight tiles per output tile
    constexpr int AS = SWIGLU ? 2 : 4;                  // TMEM A stage groups
    constexpr uint32_t W_TILE = kGmRows * RB;
    const int BN = p.bn;
    const uint32_t B_STAGE = (uint32_t)BN * 256u;
    const int NSW = p.nsw, NSB = p.nsb;

    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    unsigned char* base = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    const GmSmem plan = gm_smem_plan<BITS>(BN, NW, NSW, NSB);
    unsigned char* bring = base + plan.b_ring;
    unsigned char* wring = base + plan.w_ring;
    uint64_t* w_full = reinterpret_cast<uint64_t*>(base + plan.misc);
    uint64_t* w_empty = w_full + NSW;
    uint64_t* b_full = w_empty + NSW;
    uint64_t* b_empty = b_full + NSB;
    uint64_t* a_full = b_empty + NSB;     // [AS]
    uint64_t* a_empty = a_full + AS;      // [AS]
    uint64_t* d_full = a_empty + AS;
    uint64_t* d_empty = d_full + 1;
    uint64_t* drain_bar = d_empty + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* xsc_smem = reinterpret_cast<float*>(base + plan.xsc);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int G = gridDim.x;
    // The launch may start while the activation pre-pass still runs
    // (programmatic dependent launch): set-up, weight tiles, scales and
    // decoded A stages are model data; only the producer's activation loads
    // and the epilogue's reads and writes wait for the pre-pass (and, through
    // it, for everything before it in the stream).
    pdl_trigger();

    if (tid == 0) {
        for (int i = 0; i < NSW; ++i) { mbar_init(&w_full[i], 1); mbar_init(&w_empty[i], 128); }
        for (int i = 0; i < NSB; ++i) { mbar_init(&b_full[i], 1); mbar_init(&b_empty[i], 1); }
        for (int i = 0; i < AS; ++i) { mbar_init(&a_full[i], 128); mbar_init(&a_empty[i], 1); }
        mbar_init(d_full, 1);
        mbar_init(d_empty, 128);
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == kGmMmaWarp) {
        tmem_alloc(tmem_slot, kGmTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // TMEM columns: A stage group g (0..AS-1) for weight tile h at 64*(g*NW + h);
    // accumulator of weight tile h at 64*AS*NW + h*BN (at most 512 columns).
    const uint32_t d_col0 = 64u * AS * NW;

    // Work items it = (tile, ks), tile-major: tile = it / splits, K range
    // [ks, ks + 1) * kb_per_split; CTA b takes items b, b + G, ...
    int it_cur = blockIdx.x;
    auto next_item = [&](int& cur, int& tile, int& kb0, int& kb1, int& ks) -> bool {
        if (cur >= p.items) return false;
        tile = cur / p.splits;
        ks = cur - tile * p.splits;
        kb0 = ks * p.kb_per_split;
        kb1 = kb0 + p.kb_per_split;
        cur += G;
        return true;
    };
    // x (and the activations) depend on the previous kernel only through the
    // pre-pass launched just before this one on the same stream.
    if (warp == kGmProducerWarp) {
        // ======================= TMA producer =================================
        if (lane == 0) {
            tma_prefetch_desc(&wmap);
            tma_prefetch_desc(&xmap);
            int sw = 0, sb = 0;
            uint32_t pw = 0, pb = 0;
            long long u = 0;
            bool ok = true;
            int cur = it_cur;
            int tile, kb0, kb1, ks;
            while (ok && next_item(cur, tile, kb0, kb1, ks)) {
                const int wt = tile % p.wtiles, tt = tile / p.wtiles;
                for (int kb = kb0; kb < kb1; ++kb, ++u) {
                    if (u >= NSW && !mbar_wait_sleep(&w_empty[sw], pw ^ 1u, abort_flag, kGmWaitLimit, kGmSleepNs)) { ok = false; break; }
                    mbar_arrive_expect_tx(&w_full[sw], W_TILE * NW);
                    unsigned char* wdst = wring + (size_t)sw * W_TILE * NW;
                    tma_load_2d(wdst, &wmap, kb * RB, wt * kGmRows, &w_full[sw]);
                    if (SWIGLU) tma_load_2d(wdst + W_TILE, &wmap, kb * RB, p.half_n + wt * kGmRows, &w_full[sw]);
                    if (++sw == NSW) { sw = 0; pw ^= 1u; }
                    if (u >= NSB && !mbar_wait_sleep(&b_empty[sb], pb ^ 1u, abort_flag, kGmWaitLimit, kGmSleepNs)) { ok = false; break; }
                    if (u == 0) pdl_wait();   // activations come from the pre-pass
                    mbar_arrive_expect_tx(&b_full[sb], B_STAGE);
                    unsigned char* bdst = bring + (size_t)sb * B_STAGE;
                    // the activation map is over bytes: k-block kb spans bytes [256 kb, 256 kb + 256)
                    tma_load_2d(bdst, &xmap, kb * 256, tt * BN, &b_full[sb]);
                    tma_load_2d(bdst + (size_t)BN * 128, &xmap, kb * 256 + 128, tt * BN, &b_full[sb]);
                    if (++sb == NSB) { sb = 0; pb ^= 1u; }
                }
            }
            if (!ok) { *abort_flag = 1; atomicOr(&g_gemm_timeout, 1); }
            // every issued copy lands before the CTA's shared memory goes away
            const long long issued = u;
            for (long long i = (issued > NSW ? issued - NSW : 0); i < issued; ++i)
                (void)mbar_wait_drain(&w_full[i % NSW], (uint32_t)((i / NSW) & 1), kGmWaitLimit);
            for (long long i = (issued > NSB ? issued - NSB : 0); i < issued; ++i)
                (void)mbar_wait_drain(&b_full[i % NSB], (uint32_t)((i / NSB) & 1), kGmWaitLimit);
        }
    } else if (warp == kGmMmaWarp) {
        // ======================= MMA issuer ===================================
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(128, BN);
            const uint32_t bring_addr = smem_u32(bring);
            int sb = 0;
            uint32_t pb = 0;
            long long u = 0;
            int n_items = 0;
            bool ok = true;
            int cur = it_cur;
            int tile, kb0, kb1, ks;
            for (; ok && next_item(cur, tile, kb0, kb1, ks); ++n_items) {
                // the accumulator is free once the previous item's epilogue read it
                if (n_items > 0 && !mbar_wait_sleep(d_empty, (uint32_t)((n_items - 1) & 1), abort_flag, kGmWaitLimit, kGmSleepNs)) { ok = false; break; }
                tc_fence_after();
                for (int j = 0; j < kb1 - kb0; ++j, ++u) {
                    const int g = (int)(u % AS);
                    if (!mbar_wait_sleep(&b_full[sb], pb, abort_flag, kGmWaitLimit, kGmSleepNs) ||
                        !mbar_wait_sleep(&a_full[g], (uint32_t)((u / AS) & 1), abort_flag, kGmWaitLimit, kGmSleepNs)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t bst = bring_addr + (uint32_t)sb * B_STAGE;
#pragma unroll
                    for (int h = 0; h < NW; ++h) {
#pragma unroll
                        for (int kk = 0; kk < 8; ++kk) {
                            const uint32_t baddr = bst + (uint32_t)(kk >> 2) * (uint32_t)BN * 128u + (uint32_t)(kk & 3) * 32u;
                            umma_f16_tmemA(tmem_base + d_col0 + (uint32_t)(h * BN),
                                           tmem_base + (uint32_t)(64 * (g * NW + h) + 8 * kk), umma_desc_sw128(baddr),
                                           idesc, (j > 0 || kk > 0) ? 1u : 0u);
                        }
                    }
                    umma_commit(&a_empty[g]);
                    umma_commit(&b_empty[sb]);
                    if (++sb == NSB) { sb = 0; pb ^= 1u; }
                }
                if (ok) umma_commit(d_full);
            }
            if (!ok) { *abort_flag = 1; atomicOr(&g_gemm_timeout, 1); }
            // drain: every issued MMA completes before TMEM is released
            umma_commit(drain_bar);
            volatile int never = 0;
            (void)mbar_wait_sleep(drain_bar, 0u, &never, kGmWaitLimit, kGmSleepNs);
        }
    } else {
        // ======================= decode + epilogue warps (0-3) ================
        const int row = warp * 32 + lane;            // weight row inside a tile / TMEM lane
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        const bool sz16 = (p.flags & VSPEC_B200_F_SZ_F16) != 0;
        const bool has_s = p.s != nullptr, has_zp = p.zp != nullptr;
        int sw = 0;
        uint32_t pw = 0;
        long long u = 0;
        int n_items = 0;
        bool ok = true;
        // Group scale / zero-point of this thread's row (and its up row) as raw
        // bits, kGmScalePipe k-blocks ahead along this CTA's item sequence, so
        // no decode waits on their load latency.
        auto ld_raw = [&](const void* b, size_t idx) -> uint32_t {
            return sz16 ? (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(b) + idx)
                        : __ldg(reinterpret_cast<const unsigned int*>(b) + idx);
        };
        auto raw_to_f = [&](uint32_t v) -> float {
            return sz16 ? __half2float(__ushort_as_half((unsigned short)v)) : __uint_as_float(v);
        };
        uint32_t szq[kGmScalePipe][NW][2];
        int pf_cur = it_cur, pf_tile = 0, pf_kb = 0, pf_kb1 = 0, pf_ks = 0;
        auto pf_issue = [&](uint32_t (&d)[NW][2]) {
            if (pf_kb >= pf_kb1 && !next_item(pf_cur, pf_tile, pf_kb, pf_kb1, pf_ks)) return;
            const int pwt = pf_tile % p.wtiles, pkb = pf_kb++;
            const int grp = p.kb_per_group_shift >= 0 ? (pkb >> p.kb_per_group_shift) : pkb / p.kb_per_group;
#pragma unroll
            for (int h = 0; h < NW; ++h) {
                int grow = (h ? p.half_n : 0) + pwt * kGmRows + row;
                grow = grow < p.n ? grow : p.n - 1;
                const size_t idx = (size_t)grow * p.n_groups + grp;
                d[h][0] = has_s ? ld_raw(p.s, idx) : 0u;
                d[h][1] = has_zp ? ld_raw(p.zp, idx) : 0u;
            }
        };
#pragma unroll
        for (int i = 0; i < kGmScalePipe; ++i) pf_issue(szq[i]);
        int cur = it_cur;
        int tile, kb0, kb1, ks;
        for (; ok && next_item(cur, tile, kb0, kb1, ks); ++n_items) {
            const int wt = tile % p.wtiles, tt = tile / p.wtiles;
            for (int kb = kb0; kb < kb1; ++kb, ++u) {
                const int g = (int)(u % AS);
                // this k-block's scale / zero-point as fp16 pairs; then shift the
                // queue and request the one kGmScalePipe k-blocks ahead
                uint32_t s2[NW], nz2[NW];
#pragma unroll
                for (int h = 0; h < NW; ++h) {
                    const float sv = has_s ? raw_to_f(szq[0][h][0]) : 1.0f;
                    const float zv = has_zp ? raw_to_f(szq[0][h][1]) : p.zp_const;
                    const __half2 sh = __float2half2_rn(sv);
                    const __half2 nzh = __float2half2_rn(-zv * sv);
                    s2[h] = *reinterpret_cast<const uint32_t*>(&sh);
                    nz2[h] = *reinterpret_cast<const uint32_t*>(&nzh);
                }
#pragma unroll
                for (int i = 0; i + 1 < kGmScalePipe; ++i)
#pragma unroll
                    for (int h = 0; h < NW; ++h) { szq[i][h][0] = szq[i + 1][h][0]; szq[i][h][1] = szq[i + 1][h][1]; }
                pf_issue(szq[kGmScalePipe - 1]);
                if (!mbar_wait_sleep(&w_full[sw], pw, abort_flag, kGmWaitLimit, kGmSleepNs)) { ok = false; break; }
                uint32_t words[NW][4 * BITS];
                const unsigned char* wst = wring + (size_t)sw * W_TILE * NW;
#pragma unroll
                for (int h = 0; h < NW; ++h)
#pragma unroll
                    for (int c16 = 0; c16 < BITS; ++c16) {
                        const uint4 v = *reinterpret_cast<const uint4*>(wst + h * W_TILE + gm_chunk_offset<BITS>(row, c16));
                        words[h][4 * c16 + 0] = v.x; words[h][4 * c16 + 1] = v.y;
                        words[h][4 * c16 + 2] = v.z; words[h][4 * c16 + 3] = v.w;
                    }
                // the weight stage is released after the TMEM stores below have
                // consumed these words (a release right after the loads let the
                // refill land before the loads had read the stage)
                const int sw_used = sw;
                if (++sw == NSW) { sw = 0; pw ^= 1u; }
                // A stage group g was last read by the MMAs of unit u - AS
                if (u >= AS && !mbar_wait_sleep(&a_empty[g], (uint32_t)((u / AS - 1) & 1), abort_flag, kGmWaitLimit, kGmSleepNs)) { ok = false; break; }
                tc_fence_after();
#pragma unroll
                for (int h = 0; h < NW; ++h) {
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
                        uint32_t hv[32];
#pragma unroll
                        for (int cc = 0; cc < 2; ++cc) {
                            Chunk<BITS> ch;
#pragma unroll
                            for (int w = 0; w < BITS; ++w) ch.w[w] = words[h][BITS * (2 * hh + cc) + w];
#pragma unroll
                            for (int mm = 0; mm < 8; ++mm) {
                                uint32_t r0, r1;
                                unpack_mm<BITS, UNSIGNED>(ch, mm, r0, r1);
                                uint32_t im0, c0, im1, c1;
                                gm_pair_const<BITS>(2 * mm, im0, c0);
                                gm_pair_const<BITS>(2 * mm + 1, im1, c1);
                                const uint32_t code0 = hfma2_bits(r0, im0, c0);   // exact small integers
                                const uint32_t code1 = hfma2_bits(r1, im1, c1);
                                hv[16 * cc + 2 * mm] = hfma2_bits(code0, s2[h], nz2[h]);
                                hv[16 * cc + 2 * mm + 1] = hfma2_bits(code1, s2[h], nz2[h]);
                            }
                        }
                        tmem_st_x32(tmem_base + lane_off + (uint32_t)(64 * (g * NW + h) + 32 * hh), hv);
                    }
                }
                mbar_arrive(&w_empty[sw_used]);
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(&a_full[g]);
            }
            if (!ok) break;
            // ---- epilogue of the item ----
            if (!mbar_wait_sleep(d_full, (uint32_t)(n_items & 1), abort_flag, kGmWaitLimit, kGmSleepNs)) { ok = false; break; }
            if (n_items == 0) pdl_wait();   // x scales, residual, y and the partials follow the pre-pass
            tc_fence_after();
            const int out_n = SWIGLU ? p.half_n : p.n;
            const int col = wt * kGmRows + row;           // output column of this thread
            if (p.splits == 1) {
                // the whole tile: finish it directly.  The tile's inverse
                // activation scales are staged once in shared memory and the
                // residuals of the next 16 tokens are requested while these are
                // stored, so no chunk waits a full load round trip.
                for (int t = row; t < BN; t += kGmRows) {
                    const int tok = tt * BN + t;
                    xsc_smem[t] = tok < p.m ? p.xinv[tok] : 0.f;
                }
                named_bar_sync(1, kGmRows);
                const bool add_res = !SWIGLU && (p.flags & VSPEC_B200_F_RESIDUAL) && col < out_n;
                float rv[16];
                auto load_res = [&](int j0) {
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) {
                        const int tok = tt * BN + j0 + jj;
                        rv[jj] = (add_res && tok < p.m) ? p.residual[(size_t)tok * out_n + col] : 0.f;
                    }
                };
                load_res(0);
                for (int j0 = 0; j0 < BN; j0 += 16) {
                    float dv[NW][16];
#pragma unroll
                    for (int h = 0; h < NW; ++h) tmem_ld_x16(tmem_base + lane_off + d_col0 + (uint32_t)(h * BN + j0), dv[h]);
                    float rc[16];
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) rc[jj] = rv[jj];
                    if (j0 + 16 < BN) load_res(j0 + 16);
                    tmem_wait_ld();
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) {
                        const int tok = tt * BN + j0 + jj;
                        if (tok < p.m && col < out_n) {
                            const float xi = xsc_smem[j0 + jj];
                            float v = dv[0][jj] * xi;
                            if (SWIGLU) {
                                const float up = dv[NW - 1][jj] * xi;
                                v = v / (1.0f + expf(-v)) * up;
                            }
                            if (add_res) v += rc[jj];
                            p.y[(size_t)tok * out_n + col] = v;
                        }
                    }
                }
                named_bar_sync(1, kGmRows);   // the staged scales are reused by the next item
                tc_fence_before();
                mbar_arrive(d_empty);
            } else {
                // split along K: publish this item's fp32 partial in slot ks,
                // [tile][split][h][token quad][row] float4s (coalesced: a warp
                // writes 32 consecutive rows); gemm_merge_kernel sums the
                // slots in K order and finishes the tile
                float4* part4 = reinterpret_cast<float4*>(p.scratch) +
                                ((size_t)tile * p.splits + ks) * (size_t)NW * (size_t)(BN / 4) * kGmRows;
                for (int j0 = 0; j0 < BN; j0 += 16) {
                    float dv[NW][16];
#pragma unroll
                    for (int h = 0; h < NW; ++h) tmem_ld_x16(tmem_base + lane_off + d_col0 + (uint32_t)(h * BN + j0), dv[h]);
                    tmem_wait_ld();
#pragma unroll
                    for (int h = 0; h < NW; ++h)
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            part4[((size_t)h * (BN / 4) + (j0 >> 2) + q) * kGmRows + row] =
                                make_float4(dv[h][4 * q], dv[h][4 * q + 1], dv[h][4 * q + 2], dv[h][4 * q + 3]);
                }
                tc_fence_before();
                mbar_arrive(d_empty);
            }
        }
        if (!ok) { *abort_flag = 1; atomicOr(&g_gemm_timeout, 1); }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kGmMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kGmTmemCols);
    }
}

// ---------------------------------------------------------------------------
// Split-K merge: one thread per (tile, token quad, weight row) sums the K
// slots' fp32 partials in slot order (deterministic), undoes the activation
// row scale and applies SwiGLU / residual.  Runs over the whole GPU right
// after the GEMM (programmatic dependent launch), so no CTA of the GEMM sums
// a tile alone.
// ---------------------------------------------------------------------------
template <bool SWIGLU>
__global__ void __launch_bounds__(256) gemm_merge_kernel(const GemmParams p) {
    pdl_wait();
    pdl_trigger();
    constexpr int NW = SWIGLU ? 2 : 1;
    const int q4 = p.bn / 4;
    const long long per_tile = (long long)q4 * kGmRows;   // float4 slots of one (split, h)
    const long long total = (long long)p.wtiles * p.ttiles * per_tile;
    const int out_n = SWIGLU ? p.half_n : p.n;
    const float4* part = reinterpret_cast<const float4*>(p.scratch);
    for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (long long)gridDim.x * blockDim.x) {
        const int tile = (int)(idx / per_tile);
        const int rem = (int)(idx - (long long)tile * per_tile);
        const int jq = rem / kGmRows, row = rem - jq * kGmRows;
        const int wt = tile % p.wtiles, tt = tile / p.wtiles;
        const float4* src = part + (size_t)tile * p.splits * NW * per_tile + (size_t)jq * kGmRows + row;
        float4 acc[NW];
#pragma unroll
        for (int h = 0; h < NW; ++h) acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s0 = 0; s0 < p.splits; s0 += 4) {
            float4 v[4][NW];
#pragma unroll
            for (int sl = 0; sl < 4; ++sl)
#pragma unroll
                for (int h = 0; h < NW; ++h)
                    v[sl][h] = s0 + sl < p.splits ? __ldcg(src + ((size_t)(s0 + sl) * NW + h) * per_tile)
                                                  : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int sl = 0; sl < 4; ++sl)
                if (s0 + sl < p.splits)
#pragma unroll
                    for (int h = 0; h < NW; ++h) {
                        acc[h].x += v[sl][h].x; acc[h].y += v[sl][h].y;
                        acc[h].z += v[sl][h].z; acc[h].w += v[sl][h].w;
                    }
        }
        const int col = wt * kGmRows + row;
        if (col >= out_n) continue;
        const float g4[4] = {acc[0].x, acc[0].y, acc[0].z, acc[0].w};
        const float u4[4] = {acc[NW - 1].x, acc[NW - 1].y, acc[NW - 1].z, acc[NW - 1].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int tok = tt * p.bn + 4 * jq + e;
            if (tok >= p.m) break;
            const float xi = p.xinv[tok];
            float v = g4[e] * xi;
            if (SWIGLU) {
                const float up = u4[e] * xi;
                v = v / (1.0f + expf(-v)) * up;
            }
            const size_t o = (size_t)tok * out_n + col;
            if (!SWIGLU && (p.flags & VSPEC_B200_F_RESIDUAL)) v += p.residual[o];
            p.y[o] = v;
        }
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
struct GemmPlan {
    int bn, wtiles, ttiles, splits, kb_per_split, items, grid, nsw, nsb;
    size_t smem;
    size_t xh_bytes, xinv_bytes, part_bytes;
};

static int gm_row_bytes(int bits) { return bits == 4 ? 64 : (bits == 3 ? 48 : 32); }

static size_t gm_smem_total(int bits, int bn, int nw, int nsw, int nsb) {
    if (bits == 4) return gm_smem_plan<4>(bn, nw, nsw, nsb).total + 1024u;
    if (bits == 3) return gm_smem_plan<3>(bn, nw, nsw, nsb).total + 1024u;
    return gm_smem_plan<2>(bn, nw, nsw, nsb).total + 1024u;
}

static bool gemm_plan(int m, int n, int k, int bits, bool swiglu, GemmPlan* gp) {
    memset(gp, 0, sizeof(*gp));
    const int nw = swiglu ? 2 : 1;
    const int out_n = swiglu ? n / 2 : n;
    const int bn_max = swiglu ? 128 : 256;
    const int tt = (m + bn_max - 1) / bn_max;
    int bn = (m + tt - 1) / tt;
    bn = (bn + 15) & ~15;
    if (bn < 16) bn = 16;
    gp->bn = bn;
    gp->ttiles = (m + bn - 1) / bn;
    gp->wtiles = (out_n + kGmRows - 1) / kGmRows;
    const int kbt = k / 128;
    const int tiles = gp->wtiles * gp->ttiles;
    const int sms = device_sm_count();
    // K split with the shortest makespan, in k-block times: rounds of items per
    // CTA x (k-blocks of an item + ~3 for its epilogue, which drains the TMEM
    // accumulator before the next item's MMAs start), plus the merge kernel: ~3 k-blocks of launch and latency and the partial
    // bytes (items x NW x BN x 128 fp32, mostly L2-resident), ~20000 such
    // per-token columns per k-block time (calibrated on B200 at M = 64 and 256)
    // An unsplit item on a GPU with idle SMs (fewer tiles than SMs) and a token tile above 128 costs
    // more than the model's 3: measured at M = 256, N = 5120, K = 1024 (40 tiles of 256 tokens, 8
    // k-blocks): 26.8 us unsplit against 14.7 us in two splits with the merge.
    const double epi1 = (bn > 128 && tiles < sms) ? 3.0 + (bn - 128) / 16.0 : 3.0;
    int splits = 1;
    double best = -1.0;
    for (int d = 1; d <= kbt; ++d) {
        if (kbt % d != 0 || (d > 1 && kbt / d < 2)) continue;
        const long long items = (long long)tiles * d;
        const long long rounds = (items + sms - 1) / sms;
        double cost = (double)rounds * (kbt / d + (d == 1 ? epi1 : 3.0));
        if (d > 1) cost += 3.0 + (double)items * nw * bn / 20000.0;
        if (best < 0.0 || cost < best) { best = cost; splits = d; }
    }
    // tuning override: VSPEC_B200_GEMM_SPLITS=d (a divisor of the k-blocks)
    if (const char* e = getenv("VSPEC_B200_GEMM_SPLITS")) {
        const int d = atoi(e);
        if (d >= 1 && d <= kbt && kbt % d == 0) splits = d;
    }
    gp->splits = splits;
    gp->kb_per_split = kbt / splits;
    gp->items = tiles * splits;
    gp->grid = gp->items < sms ? gp->items : sms;
    // rings: as many activation stages (<= 4) and weight stages (<= 8) as fit
    gp->nsb = 0;
    for (int nsb = 4; nsb >= 2 && !gp->nsb; --nsb)
        for (int nsw = 8; nsw >= 2; --nsw)
            if (gm_smem_total(bits, bn, nw, nsw, nsb) <= kGmSmemMax) { gp->nsb = nsb; gp->nsw = nsw; break; }
    if (!gp->nsb) return false;
    gp->smem = gm_smem_total(bits, bn, nw, gp->nsw, gp->nsb);
    gp->xh_bytes = ((size_t)m * k * 2 + 255) & ~(size_t)255;
    gp->xinv_bytes = ((size_t)m * 4 + 255) & ~(size_t)255;
    gp->part_bytes = splits > 1 ? (size_t)tiles * splits * nw * bn * kGmRows * sizeof(float) : 0;
    return true;
}

bool gemm_tc_supported(const GemvParams& p, int bits, size_t counter_slots) {
    if (p.m <= kGemvMaxM) return false;
    if (p.k % 128 != 0 || p.n_groups < 1 || p.k % p.n_groups != 0 || (p.k / p.n_groups) % 128 != 0) return false;
    if (reinterpret_cast<uintptr_t>(p.w) % 16 != 0 || (size_t)p.row_bytes % 16 != 0) return false;
    if (reinterpret_cast<uintptr_t>(p.x) % 16 != 0) return false;   // vectorised pre-pass
    if ((p.flags & VSPEC_B200_F_RMSNORM) && reinterpret_cast<uintptr_t>(p.norm_w) % 16 != 0) return false;
    const bool swiglu = (p.flags & VSPEC_B200_F_SWIGLU) != 0;
    if (swiglu && (p.n % 2 != 0 || (p.n / 2) % kGmRows != 0)) return false;
    GemmPlan gp;
    if (!gemm_plan(p.m, p.n, p.k, bits, swiglu, &gp)) return false;
    (void)counter_slots;   // split tiles merge in gemm_merge_kernel: no counters
    return true;
}

size_t gemm_tc_workspace_bytes(int m, int n, int k, bool swiglu) {
    if (m <= kGemvMaxM || k < 128) return 0;
    size_t most = 0;
    for (int bits = 2; bits <= 4; ++bits) {
        GemmPlan gp;
        if (!gemm_plan(m, n, k, bits, swiglu, &gp)) continue;
        const size_t b = gp.xh_bytes + gp.xinv_bytes + gp.part_bytes;
        if (b > most) most = b;
    }
    return most;
}

int gemm_tc_read_and_clear_timeout(int* out) {
    int v = 0, zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_gemm_timeout, sizeof(int));
    if (e != cudaSuccess) return cuda_status(e, "read GEMM timeout flag");
    e = cudaMemcpyToSymbol(g_gemm_timeout, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_status(e, "clear GEMM timeout flag");
    *out = v;
    return VSPEC_B200_OK;
}

template <int BITS, bool UNS, bool SWIGLU>
static cudaError_t launch_gemm_t(const CUtensorMap& wm, const CUtensorMap& xm, const GemmParams& gp, int grid,
                                 size_t smem, cudaStream_t st) {
    auto kern = lowbit_gemm_tc_kernel<BITS, UNS, SWIGLU>;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGmSmemMax);
        if (e != cudaSuccess) return e;
        configured[dev] = 1;
    }
    return launch_pdl(kern, dim3(grid), dim3(kGmThreads), smem, st, wm, xm, gp);
}

template <int BITS>
static cudaError_t launch_gemm_bits(const CUtensorMap& wm, const CUtensorMap& xm, const GemmParams& gp, bool uns,
                                    bool swiglu, int grid, size_t smem, cudaStream_t st) {
    if (uns) return swiglu ? launch_gemm_t<BITS, true, true>(wm, xm, gp, grid, smem, st)
                           : launch_gemm_t<BITS, true, false>(wm, xm, gp, grid, smem, st);
    return swiglu ? launch_gemm_t<BITS, false, true>(wm, xm, gp, grid, smem, st)
                  : launch_gemm_t<BITS, false, false>(wm, xm, gp, grid, smem, st);
}

// p: the GEMV parameter block (x, w, s, zp, y, residual, norm, dims, flags,
// kb bookkeeping, counters); work: device scratch of at least
// gemm_tc_workspace_bytes() bytes.
int gemm_tc_launch(const GemvParams& p, int bits, int unsigned_codes, cudaStream_t st, void* work) {
    const bool swiglu = (p.flags & VSPEC_B200_F_SWIGLU) != 0;
    GemmPlan plan;
    if (!gemm_plan(p.m, p.n, p.k, bits, swiglu, &plan)) {
        set_error("shape not supported by the tcgen05 GEMM");
        return VSPEC_B200_ERR_UNSUPPORTED;
    }
    unsigned char* wb = reinterpret_cast<unsigned char*>(work);
    __half* xh = reinterpret_cast<__half*>(wb);
    float* xinv = reinterpret_cast<float*>(wb + plan.xh_bytes);
    float* part = reinterpret_cast<float*>(wb + plan.xh_bytes + plan.xinv_bytes);
    const int rms = (p.flags & VSPEC_B200_F_RMSNORM) ? 1 : 0;
    cudaError_t e;
    if (bits == 4) e = launch_pdl(gemm_prep_x_kernel<4>, dim3(p.m), dim3(kGmPrepThreads), 0, st, p.x, p.norm_w, p.eps, rms, p.k, xh, xinv);
    else if (bits == 3) e = launch_pdl(gemm_prep_x_kernel<3>, dim3(p.m), dim3(kGmPrepThreads), 0, st, p.x, p.norm_w, p.eps, rms, p.k, xh, xinv);
    else e = launch_pdl(gemm_prep_x_kernel<2>, dim3(p.m), dim3(kGmPrepThreads), 0, st, p.x, p.norm_w, p.eps, rms, p.k, xh, xinv);
    if (e != cudaSuccess) return cuda_status(e, "gemm_prep_x_kernel launch");

    CUtensorMap wm, xm;
    const CUtensorMapSwizzle wswz = bits == 4 ? CU_TENSOR_MAP_SWIZZLE_64B
                                  : (bits == 2 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_NONE);
    int rc = make_row_tile_map(&wm, p.w, p.n, p.row_bytes, gm_row_bytes(bits), kGmRows, wswz);
    if (rc != VSPEC_B200_OK) return rc;
    // activations: [m][k] fp16 viewed as bytes, tiles of bn rows x 128 bytes (64 values)
    rc = make_row_tile_map(&xm, reinterpret_cast<const uint8_t*>(xh), p.m, p.k * 2, 128, plan.bn,
                           CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != VSPEC_B200_OK) return rc;

    GemmParams gp;
    memset(&gp, 0, sizeof(gp));
    gp.w = p.w; gp.s = p.s; gp.zp = p.zp; gp.zp_const = p.zp_const;
    gp.y = p.y; gp.residual = p.residual; gp.xinv = xinv; gp.scratch = part;
    gp.m = p.m; gp.n = p.n; gp.k = p.k; gp.n_groups = p.n_groups;
    gp.row_bytes = p.row_bytes; gp.kb_total = p.kb_total; gp.kb_per_group = p.kb_per_group;
    gp.kb_per_group_shift = p.kb_per_group_shift; gp.flags = p.flags;
    gp.bn = plan.bn; gp.wtiles = plan.wtiles; gp.ttiles = plan.ttiles; gp.splits = plan.splits;
    gp.kb_per_split = plan.kb_per_split; gp.items = plan.items; gp.nsw = plan.nsw; gp.nsb = plan.nsb;
    gp.half_n = swiglu ? p.n / 2 : 0;
    const bool uns = unsigned_codes != 0;
    if (bits == 4) e = launch_gemm_bits<4>(wm, xm, gp, uns, swiglu, plan.grid, plan.smem, st);
    else if (bits == 3) e = launch_gemm_bits<3>(wm, xm, gp, uns, swiglu, plan.grid, plan.smem, st);
    else e = launch_gemm_bits<2>(wm, xm, gp, uns, swiglu, plan.grid, plan.smem, st);
    if (e != cudaSuccess) return cuda_status(e, "lowbit_gemm_tc_kernel launch");
    if (plan.splits > 1) {
        const long long work = (long long)plan.wtiles * plan.ttiles * (plan.bn / 4) * kGmRows;
        long long blocks = (work + 255) / 256;
        const long long cap = (long long)device_sm_count() * 8;
        if (blocks > cap) blocks = cap;
        e = swiglu ? launch_pdl(gemm_merge_kernel<true>, dim3((unsigned)blocks), dim3(256), 0, st, gp)
                   : launch_pdl(gemm_merge_kernel<false>, dim3((unsigned)blocks), dim3(256), 0, st, gp);
        if (e != cudaSuccess) return cuda_status(e, "gemm_merge_kernel launch");
    }
    return VSPEC_B200_OK;
}

}  // namespace vb200
