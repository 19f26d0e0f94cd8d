// lowbit_gemv_ring.cu -- TMA-fed low-bit GEMV for decode (M <= 8), the default
// fast path on sm_100a.
//
// Same contraction and numerics contract as lowbit_gemv.cu (reference
// semantics: src/quant/int4.c:107-132 with the group indexing of
// src/kernel/cuda/fused_linear_int4.cu:391-396; bitstream of
// src/quant/pack.c:53-74):
//     y[i][j] = sum_t x[i][t] * (code(j,t) - zp[j][g(t)]) * s[j][g(t)]
//
// Layout of the work:
//   * unit = (tile of W, 128-code k-block), a tile being 256 rows for m <= 4
//     and 128 rows for m <= 8; persistent CTAs (two per SM when the shared
//     memory plan allows) own contiguous runs of units in tile-major order
//     (split-K across CTAs), or, when the tiles are fewer than the CTA
//     slots, each tile's k-blocks are split evenly over P CTAs so that no
//     CTA crosses a tile boundary;
//   * warp 8 (one thread) streams the units' weight tiles with 2-D TMA into a
//     deep shared-memory ring (8-48 stages, 60-190 KB in flight per SM), so
//     HBM sees many outstanding bulk requests without register staging;
//   * warps 0-7 each own a 32-row (m <= 4) or 16-row slice of every tile,
//     i.e. one or two blocks of 16 rows.  A thread (g, c) reads its 32-code
//     chunk c of rows g and g+8 of each block from the ring and decodes it in
//     registers into MMA A fragments, multiplied with activation fragments
//     staged once in shared memory.  Default (IMMA): one mask per register
//     gives offset codes as bytes for mma.sync m16n8k32 u8 x s8, against x
//     quantised per k-block to 14-bit integers split into int8 hi/lo columns,
//     so block dot products are exact int32.  Otherwise: fp16 pairs from a
//     magic-number LOP3 for m16n8k16 against x split into fp16 hi + lo (see
//     lowbit_decode.cuh).  Warp-level MMA sustains ~128 codes/cycle/SM here, well
//     above what HBM delivers; small-N tcgen05.mma does not (it costs ~95
//     cycles per 128x16 A tile whatever N is), so the tensor-memory path is
//     kept for large M only;
//   * each k-block's fp32 partial is scaled on the fly:
//         acc += s * inv_scale * (dot - (zp * X + C)),
//     X and C being the block's scaled activation sums (decode offsets);
//   * at the end of a tile part a warp publishes its slice's partial and bumps
//     the slice's counter; the warp that completes the count sums the slots in
//     CTA order (deterministic), applies the epilogue (residual, SwiGLU,
//     RMSNorm row factor) and resets the counter.  No warp waits on another.
//     When the P parts of a tile can run as one thread-block cluster (all
//     clusters resident in one wave), the partials stay in shared memory and
//     the cluster sums them through distributed shared memory after a
//     cluster barrier instead, in part order.
// Every CTA triggers programmatic dependent launch at its start, so the next
// launch in the stream becomes resident as soon as resources free up and
// stages its weights before it waits for this one.  Every wait is bounded.
#include "common.cuh"
#include "lowbit_decode.cuh"
#include "lowbit_kernels.cuh"
#include "tc_primitives.cuh"
#include "tma_map.cuh"

#include <stdlib.h>
#include <string.h>

namespace vb200 {

constexpr int kRingConsumerWarps = 8;
constexpr int kRingThreads = (kRingConsumerWarps + 1) * 32;
constexpr int kRingProducerWarp = kRingConsumerWarps;
constexpr int kRingScalePipe = 4;          // units of scale loads in flight per warp
constexpr uint32_t kRingWaitLimit = 1u << 16;   // checks of up to kRingSleepNs each
constexpr uint32_t kRingSleepNs = 20000;
constexpr uint32_t kRingSmemShared = 113u * 1024u;
constexpr uint32_t kRingSmemMax = 227u * 1024u;
constexpr uint32_t kRingMinSharedRing = 64u * 1024u;   // ring worth sharing an SM for
constexpr uint32_t kRingMaxRing = 192u * 1024u;

template <int BITS> struct RingCfg;
template <> struct RingCfg<4> { static constexpr int kRowBytes = 64; };
template <> struct RingCfg<3> { static constexpr int kRowBytes = 48; };
template <> struct RingCfg<2> { static constexpr int kRowBytes = 32; };

// Set when a bounded wait of the ring GEMV gave up.
__device__ int g_ring_timeout = 0;

__host__ __device__ __forceinline__ int ring_nt(int m) { return (2 * m + 7) / 8; }
__host__ __device__ __forceinline__ int ring_lanes(int m) { return 4 * (2 * m < 8 ? 2 * m : 8); }
// 16-row blocks per consumer warp: two when one n-tile of activations (m <= 4)
// leaves the registers for it, so per-unit costs are shared by 32 rows.
__host__ __device__ constexpr int ring_row_blocks(int nt) { return nt == 1 ? 2 : 1; }
__host__ __device__ inline int ring_tile_rows(int m) { return 16 * ring_row_blocks(ring_nt(m)) * kRingConsumerWarps; }

struct RingSmem {
    uint32_t frag;        // offsets from the 1024-aligned base; the ring starts at 0
    uint32_t xs, cs, is;  // per (k-block, row): scaled sum, decode offset, inverse scale
    uint32_t cpart;       // this CTA's tile partial for the cluster merge
    uint32_t misc;
    uint32_t total;
};

// Activation fragments per k-block: fp16 path 4 MMA steps x NT x lanes x 16 B;
// integer path NT x lanes x 32 B (four k32 MMAs x two registers).
template <int BITS>
__host__ __device__ inline RingSmem ring_smem_plan(int m, int kbt, int stages, bool imma) {
    RingSmem s;
    const uint32_t stage = (uint32_t)ring_tile_rows(m) * RingCfg<BITS>::kRowBytes;
    s.frag = (uint32_t)stages * stage;
    const uint32_t fbytes = (uint32_t)kbt * (uint32_t)ring_nt(m) * (uint32_t)ring_lanes(m) * (imma ? 32u : 64u);
    s.xs = s.frag + fbytes;
    s.cs = s.xs + (uint32_t)(kbt * m) * 4u;
    s.is = s.cs + (uint32_t)(kbt * m) * 4u;
    s.cpart = (s.is + (uint32_t)(kbt * m) * 4u + 15u) & ~15u;   // cluster merge: [warp][row][slice row] fp32
    s.misc = s.cpart + (uint32_t)ring_tile_rows(m) * (uint32_t)m * 4u;
    s.total = s.misc + 8u * 2u * (uint32_t)stages + 64u;   // full/empty barriers, abort flag, row norms
    return s;
}

// Byte offset of 32-code chunk c of row r inside a ring stage (the swizzle the
// tensor map was encoded with: 64B for int4, 32B for int2, none for int3).
template <int BITS>
__device__ __forceinline__ uint32_t ring_chunk_offset(int r, int c) {
    if constexpr (BITS == 4) return (uint32_t)(r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
    else if constexpr (BITS == 2) return (uint32_t)(r * 32 + (((c >> 1) ^ ((r >> 2) & 1)) << 4) + 8 * (c & 1));
    else return (uint32_t)(r * 48 + 12 * c);
}

template <int BITS>
__device__ __forceinline__ void lds_chunk(Chunk<BITS>& ch, const unsigned char* p) {
    if constexpr (BITS == 4) {
        const uint4 v = *reinterpret_cast<const uint4*>(p);
        ch.w[0] = v.x; ch.w[1] = v.y; ch.w[2] = v.z; ch.w[3] = v.w;
    } else if constexpr (BITS == 2) {
        const uint2 v = *reinterpret_cast<const uint2*>(p);
        ch.w[0] = v.x; ch.w[1] = v.y;
    } else {
        const uint32_t* q = reinterpret_cast<const uint32_t*>(p);
        ch.w[0] = q[0]; ch.w[1] = q[1]; ch.w[2] = q[2];
    }
}

template <int BITS, int NT, bool UNSIGNED, int EPI, bool SZ16, bool IMMA>
__global__ void __launch_bounds__(kRingThreads, 2)
lowbit_gemv_ring_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ GemvParams p) {
    constexpr int RB = RingCfg<BITS>::kRowBytes;
    constexpr int RBW = ring_row_blocks(NT);          // 16-row blocks per consumer warp
    constexpr int TROWS = 16 * RBW * kRingConsumerWarps;
    constexpr uint32_t STAGE_BYTES = TROWS * RB;
    constexpr int PD = kRingScalePipe / RBW;
    const int NS = p.stages;

    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    unsigned char* base = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    const int m = p.m;
    const int kbt = p.kb_total;
    const int lanes = ring_lanes(m);
    const RingSmem plan = ring_smem_plan<BITS>(m, kbt, NS, IMMA);
    unsigned char* wring = base;
    const uint4* frag = reinterpret_cast<const uint4*>(base + plan.frag);
    float* xs = reinterpret_cast<float*>(base + plan.xs);
    float* cs = reinterpret_cast<float*>(base + plan.cs);
    float* isc = reinterpret_cast<float*>(base + plan.is);
    float* cpart = reinterpret_cast<float*>(base + plan.cpart);
    uint64_t* full = reinterpret_cast<uint64_t*>(base + plan.misc);
    uint64_t* empty = full + NS;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + NS);
    float* row_norm = reinterpret_cast<float*>(empty + NS) + 4;   // [8]

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const long long U = (long long)p.tiles * kbt;
    const long long C = gridDim.x;
    // units [u0, u1) of this CTA: a contiguous run in tile-major order, or
    // (tile_parts P > 0) part blockIdx % P of tile blockIdx / P
    const int TP = p.tile_parts;
    const int tp_tile = TP > 0 ? (int)blockIdx.x / TP : 0;
    const int tp_part = TP > 0 ? (int)blockIdx.x - tp_tile * TP : 0;
    const int u0 = TP > 0 ? tp_tile * kbt + (tp_part * kbt) / TP : (int)(((long long)blockIdx.x * U) / C);
    const int u1 = TP > 0 ? tp_tile * kbt + ((tp_part + 1) * kbt) / TP : (int)(((long long)(blockIdx.x + 1) * U) / C);
    const int n_units = u1 - u0;

    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kRingConsumerWarps);
        }
        *abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();
    // the next launch in the stream may become resident and stage its weights
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");

    // ---- producer: first ring fill (weights only: no dependency on x) ----
    int p_issued = 0;
    int p_tile = u0 / kbt, p_kb = u0 - p_tile * kbt;
    if (warp == kRingProducerWarp && lane == 0) {
        tma_prefetch_desc(&wmap);
        for (; p_issued < n_units && p_issued < NS; ++p_issued) {
            mbar_arrive_expect_tx(&full[p_issued], STAGE_BYTES);
            tma_load_2d(wring + p_issued * STAGE_BYTES, &wmap, p_kb * RB, p_tile * TROWS, &full[p_issued]);
            if (++p_kb == kbt) { p_kb = 0; ++p_tile; }
        }
    }

    // ---- consumer state and the first scale / zero-point loads: model
    // data like the weights, so they are requested before the dependency
    // wait and arrive while the activation prologue runs ----
    // Warp w owns rows [w*16*RBW, (w+1)*16*RBW) of every tile: RBW blocks
    // of 16 rows, thread (g, c) rows g and g+8 of each block, chunk c.
    const int g = lane >> 2;
    const int c = lane & 3;
    const int wrow = warp * 16 * RBW;
    const bool lane_has_b = lane < lanes;
    const bool has_s = p.s != nullptr, has_zp = p.zp != nullptr;
    constexpr int SZB = SZ16 ? 2 : 4;   // bytes per scale / zero-point element
    const int half_tiles = p.tiles >> 1;
    // scale / zero-point prefetch, PD units ahead, as raw bits.  Byte
    // offsets of this thread's rows in the current tile are kept and only
    // re-derived at tile boundaries.
    uint32_t sz[PD][RBW][4];
    int s_tile = u0 / kbt, s_kb = u0 - s_tile * kbt;
    const unsigned char* sb = reinterpret_cast<const unsigned char*>(p.s);
    const unsigned char* zb = reinterpret_cast<const unsigned char*>(p.zp);
    size_t srow[RBW][2];
    auto set_srows = [&]() {
#pragma unroll
        for (int j = 0; j < RBW; ++j)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                int r = s_tile * TROWS + wrow + 16 * j + g + 8 * h;
                r = r < p.n ? r : p.n - 1;
                srow[j][h] = (size_t)r * p.n_groups * SZB;
            }
    };
    set_srows();
    auto ld_sz = [&](const unsigned char* b, size_t off) -> uint32_t {
        if constexpr (SZ16) return (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(b + off));
        else return __ldg(reinterpret_cast<const unsigned int*>(b + off));
    };
    auto issue_sz = [&](uint32_t (&d)[RBW][4]) {
        const int grp = p.kb_per_group_shift >= 0 ? (s_kb >> p.kb_per_group_shift) : s_kb / p.kb_per_group;
        const uint32_t go = (uint32_t)grp * SZB;
#pragma unroll
        for (int j = 0; j < RBW; ++j) {
            if (has_s) {
                d[j][0] = ld_sz(sb, srow[j][0] + go);
                d[j][2] = ld_sz(sb, srow[j][1] + go);
            }
            if (has_zp) {
                d[j][1] = ld_sz(zb, srow[j][0] + go);
                d[j][3] = ld_sz(zb, srow[j][1] + go);
            }
        }
        if (++s_kb == kbt) {
            s_kb = 0;
            ++s_tile;
            set_srows();
        }
    };
    if (warp < kRingConsumerWarps) {
#pragma unroll
        for (int st = 0; st < PD; ++st)
            if (st < n_units) issue_sz(sz[st]);
    }

    // ---- activation prologue (x may be the previous kernel's output) ----
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    const int K = p.k;
    const bool rms = EPI_HAS_RMSNORM(p.flags);
    if (rms) {
        for (int r = warp; r < m; r += kRingThreads / 32) {
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
    if constexpr (IMMA) {
        // Per (k-block, row) of the k-blocks this CTA touches: an exact
        // power-of-two scale sc (block max |x| * sc in [2^13, 2^14)), the
        // integer activations q = rint(x * sc) in [-2^14, 2^14] split as
        // q = 256 * xh + xl (xh in [-64, 64], xl in [-128, 127]) into the int8
        // B columns 2r (xh) and 2r + 1 (xl), and X = sum q.  Integer MMAs
        // then give sum q * v exactly; the epilogue removes the offset
        // (2^(bits-1) + zp) * X and multiplies by s / sc.
        const int kb_first = n_units >= kbt ? 0 : u0 % kbt;
        const int kb_count = n_units >= kbt ? kbt : n_units;
        constexpr float kOff = (float)(1 << (BITS - 1));
        int boff[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int t = 4 * lane + e;   // code of the k-block this lane holds
            int q, r, i;
            i8_code_place<BITS>(t & 31, q, r, i);
            boff[e] = (t >> 5) * 32 + q * 8 + r * 4 + i;   // + B lane 4n' of the column, x 32
        }
        unsigned char* fbase = base + plan.frag;
        constexpr int NW = kRingThreads / 32;
        constexpr int QB = 4;
        const int npairs = kb_count * m;
        for (int pr0 = warp; pr0 < npairs; pr0 += QB * NW) {
            float4 v[QB];
            int kbq[QB], rq[QB];
#pragma unroll
            for (int q = 0; q < QB; ++q) {
                const int pr = pr0 + q * NW;
                rq[q] = pr % m;
                int kb = kb_first + pr / m;
                kbq[q] = kb >= kbt ? kb - kbt : kb;
                v[q] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (pr < npairs) {
                    const int t = kbq[q] * 128 + lane * 4;
                    v[q] = *reinterpret_cast<const float4*>(p.x + (size_t)rq[q] * K + t);
                    if (rms) {
                        const float4 wn = *reinterpret_cast<const float4*>(p.norm_w + t);
                        v[q].x *= wn.x; v[q].y *= wn.y; v[q].z *= wn.z; v[q].w *= wn.w;
                    }
                }
            }
            float amax[QB];
#pragma unroll
            for (int q = 0; q < QB; ++q)
                amax[q] = fmaxf(fmaxf(fabsf(v[q].x), fabsf(v[q].y)), fmaxf(fabsf(v[q].z), fabsf(v[q].w)));
            // |x| bit patterns order like the values: one warp max each
#pragma unroll
            for (int q = 0; q < QB; ++q)
                amax[q] = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(amax[q])));
            int qv[QB][4], xsum[QB];
            float sc[QB];
#pragma unroll
            for (int q = 0; q < QB; ++q) {
                int sbits = 127;   // sc = 2^(13 - floor(log2 amax)) from the exponent bits
                if (amax[q] > 0.f && isfinite(amax[q])) {
                    sbits = 267 - (int)((__float_as_uint(amax[q]) >> 23) & 0xFFu);
                    sbits = sbits < 1 ? 1 : (sbits > 253 ? 253 : sbits);
                }
                sc[q] = __uint_as_float((uint32_t)sbits << 23);
                qv[q][0] = __float2int_rn(v[q].x * sc[q]);
                qv[q][1] = __float2int_rn(v[q].y * sc[q]);
                qv[q][2] = __float2int_rn(v[q].z * sc[q]);
                qv[q][3] = __float2int_rn(v[q].w * sc[q]);
                xsum[q] = (qv[q][0] + qv[q][1]) + (qv[q][2] + qv[q][3]);
            }
#pragma unroll
            for (int q = 0; q < QB; ++q) xsum[q] = __reduce_add_sync(0xffffffffu, xsum[q]);
#pragma unroll
            for (int q = 0; q < QB; ++q) {
                if (pr0 + q * NW < npairs) {
                    const int kb = kbq[q], r = rq[q];
                    if (lane == 0) {
                        const float X = (float)xsum[q];
                        xs[kb * m + r] = X;
                        cs[kb * m + r] = kOff * X;
                        isc[kb * m + r] = 1.0f / sc[q];   // power of two: exact
                    }
                    const int n = 2 * r;   // xh column; xl is n + 1, four B lanes on
                    unsigned char* fb = fbase + ((size_t)(kb * NT + (n >> 3)) * lanes + 4 * (n & 7)) * 32;
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int xh = (qv[q][e] + 128) >> 8;
                        const int xl = qv[q][e] - (xh << 8);
                        fb[boff[e]] = (unsigned char)(signed char)xh;
                        fb[boff[e] + 128] = (unsigned char)(signed char)xl;
                    }
                }
            }
        }
    } else {
        // Per (k-block, row) of the k-blocks this CTA touches: an exact
        // power-of-two scale (block max |x| lands in [2^13, 2^14)), the scaled
        // sums and the B fragments.  Lane l holds codes 4l..4l+3 of the block;
        // B fragment (k-block, mp, n-tile, lane' = 4*col + chunk) word qq holds
        // the activations of codes (lo_code(4mp+qq), hi_code(4mp+qq)) of that
        // chunk, divided by their decode multipliers, as fp16 (hi part in
        // column 2r, lo part in column 2r+1).
        const int kb_first = n_units >= kbt ? 0 : u0 % kbt;
        const int kb_count = n_units >= kbt ? kbt : n_units;
        constexpr float kOff = (float)(1 << (BITS - 1));
        float imul[4];
        int boff[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int j = (4 * lane + e) & 31;
            imul[e] = code_inv_mult<BITS>(j);
            int q, hh;
            code_slot<BITS>(j, q, hh);
            // (mp * NT) * lanes * 16 + chunk * 16 + qq * 4 + half * 2; the row
            // dependent part is added below
            boff[e] = (q >> 2) * NT * lanes * 16 + (lane >> 3) * 16 + (q & 3) * 4 + hh * 2;
        }
        unsigned char* fbase = base + plan.frag;
        constexpr int NW = kRingThreads / 32;
        constexpr int QB = 4;   // (k-block, row) pairs per warp and batch: loads and reductions overlap
        const int npairs = kb_count * m;
        for (int pr0 = warp; pr0 < npairs; pr0 += QB * NW) {
            float4 v[QB];
            int kbq[QB], rq[QB];
#pragma unroll
            for (int q = 0; q < QB; ++q) {
                const int pr = pr0 + q * NW;
                rq[q] = pr % m;
                int kb = kb_first + pr / m;
                kbq[q] = kb >= kbt ? kb - kbt : kb;
                v[q] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (pr < npairs) {
                    const int t = kbq[q] * 128 + lane * 4;
                    v[q] = *reinterpret_cast<const float4*>(p.x + (size_t)rq[q] * K + t);
                    if (rms) {
                        const float4 wn = *reinterpret_cast<const float4*>(p.norm_w + t);
                        v[q].x *= wn.x; v[q].y *= wn.y; v[q].z *= wn.z; v[q].w *= wn.w;
                    }
                }
            }
            // max |x|, sum x and sum x/mult of every pair, reduced together.
            // Scaling by a power of two commutes exactly with the sums, so
            // they need not wait for the scale.
            float amax[QB], s1[QB], s2[QB];
#pragma unroll
            for (int q = 0; q < QB; ++q) {
                amax[q] = fmaxf(fmaxf(fabsf(v[q].x), fabsf(v[q].y)), fmaxf(fabsf(v[q].z), fabsf(v[q].w)));
                s1[q] = (v[q].x + v[q].y) + (v[q].z + v[q].w);
                s2[q] = (v[q].x * imul[0] + v[q].y * imul[1]) + (v[q].z * imul[2] + v[q].w * imul[3]);
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
                for (int q = 0; q < QB; ++q) {
                    amax[q] = fmaxf(amax[q], __shfl_xor_sync(0xffffffffu, amax[q], off));
                    s1[q] += __shfl_xor_sync(0xffffffffu, s1[q], off);
                    s2[q] += __shfl_xor_sync(0xffffffffu, s2[q], off);
                }
            }
#pragma unroll
            for (int q = 0; q < QB; ++q) {
                if (pr0 + q * NW < npairs) {
                    const int kb = kbq[q], r = rq[q];
                    int sbits = 127;   // sc = 2^(13 - floor(log2 amax)) from the exponent bits
                    if (amax[q] > 0.f && isfinite(amax[q])) {
                        sbits = 267 - (int)((__float_as_uint(amax[q]) >> 23) & 0xFFu);
                        sbits = sbits < 1 ? 1 : (sbits > 253 ? 253 : sbits);
                    }
                    const float sc = __uint_as_float((uint32_t)sbits << 23);
                    if (lane == 0) {
                        const float sx = s1[q] * sc;
                        xs[kb * m + r] = sx;
                        cs[kb * m + r] = fmaf(1024.0f, s2[q] * sc, kOff * sx);
                        isc[kb * m + r] = __uint_as_float((uint32_t)(254 - sbits) << 23);
                    }
                    const float vv[4] = {v[q].x * sc, v[q].y * sc, v[q].z * sc, v[q].w * sc};
                    const int col = 2 * r;
                    unsigned char* fb =
                        fbase + (size_t)kb * 4 * NT * lanes * 16 + ((col >> 3) * lanes + 4 * (col & 7)) * 16;
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float val = vv[e] * imul[e];
                        const __half hv = __float2half_rn(val);
                        const __half lv = __float2half_rn(val - __half2float(hv));
                        *reinterpret_cast<__half*>(fb + boff[e]) = hv;
                        *reinterpret_cast<__half*>(fb + boff[e] + 64) = lv;   // column 2r+1: 4 lanes on
                    }
                }
            }
        }
    }
    __syncthreads();

    if (warp < kRingConsumerWarps) {
        // ======================= consumer warps ===============================
        // Warp w owns rows [w*16*RBW, (w+1)*16*RBW) of every tile: RBW blocks
        // of 16 rows, thread (g, c) rows g and g+8 of each block, chunk c.
        float acc[RBW][NT][2];
#pragma unroll
        for (int j = 0; j < RBW; ++j)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) acc[j][nt][0] = acc[j][nt][1] = 0.f;


        int c_tile = u0 / kbt, c_kb = u0 - c_tile * kbt;
        int ring = 0;
        uint32_t ring_ph = 0;
        bool ok = true;

        auto flush = [&](int tile) {
            constexpr int WR = 16 * RBW;   // rows of this warp's slice
            if (p.cluster_merge) {
                // the tile's parts are one cluster: keep the partial in shared
                // memory; the cluster reduces it after the barrier below
                float* cp = cpart + warp * (WR * m);
#pragma unroll
                for (int j = 0; j < RBW; ++j)
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        const int r = 4 * nt + c;
                        if (r < m) {
                            cp[r * WR + 16 * j + g] = acc[j][nt][0];
                            cp[r * WR + 16 * j + g + 8] = acc[j][nt][1];
                        }
                    }
#pragma unroll
                for (int j = 0; j < RBW; ++j)
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) acc[j][nt][0] = acc[j][nt][1] = 0.f;
                return;
            }
            auto first_cta = [&](long long u) { return (int)(((u + 1) * C - 1) / U); };
            int L = tile;
            int slot, total, n_gate;
            if (TP > 0) {
                // one tile per CTA: slot = part; SwiGLU gate parts first, then up parts
                slot = tp_part;
                total = n_gate = TP;
                if (EPI == kEpiSwiGLU) {
                    const bool up = tile >= half_tiles;
                    L = up ? tile - half_tiles : tile;
                    slot += up ? TP : 0;
                    total = 2 * TP;
                }
            } else {
            slot = (int)blockIdx.x - first_cta((long long)tile * kbt);
            total = first_cta((long long)(tile + 1) * kbt - 1) - first_cta((long long)tile * kbt) + 1;
            n_gate = total;
            if (EPI == kEpiSwiGLU) {
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
            }
            const int ci = L * kRingConsumerWarps + warp;   // counter of this warp's slice
            float* part = p.scratch + ((size_t)ci * p.max_slots + slot) * (WR * m);
#pragma unroll
            for (int j = 0; j < RBW; ++j)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    const int r = 4 * nt + c;
                    if (r < m) {
                        part[r * WR + 16 * j + g] = acc[j][nt][0];
                        part[r * WR + 16 * j + g + 8] = acc[j][nt][1];
                    }
                }
            // message passing: every lane fences its own partial stores at GPU
            // scope before the warp barrier, lane 0 bumps the counter, and every
            // lane of the warp that completes the count fences again before it
            // reads the other slots.  (A fence by lane 0 alone orders only its
            // own stores: other lanes' partials were then sometimes still in
            // flight when the merging warp of another CTA read them, which left
            // a few stale rows in about one launch in eight at k = 6144 or 5120.)
            asm volatile("fence.acq_rel.gpu;\n" ::: "memory");
            __syncwarp();
            int old = 0;
            if (lane == 0) old = atomicAdd(p.counters + ci, 1);
            old = __shfl_sync(0xffffffffu, old, 0);
            if (old == total - 1) {
                asm volatile("fence.acq_rel.gpu;\n" ::: "memory");
                __syncwarp();
                const float* sbase = p.scratch + (size_t)ci * p.max_slots * (WR * m);
                // Sum of slots [s0, s1) in slot order; the loads of a batch of
                // eight are issued together, so the merge costs one L2 round
                // trip per eight partials instead of one per partial.
                auto slot_sum = [&](int s0, int s1, int z) {
                    float sum = 0.f;
                    for (int sb0 = s0; sb0 < s1; sb0 += 8) {
                        float v[8];
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            v[q] = sb0 + q < s1 ? __ldcg(sbase + (size_t)(sb0 + q) * WR * m + z) : 0.f;
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            if (sb0 + q < s1) sum += v[q];
                    }
                    return sum;
                };
                for (int z = lane; z < WR * m; z += 32) {
                    const int r = z / WR, i = z - r * WR;
                    const float nr = rms ? row_norm[r] : 1.0f;
                    const int orow = L * TROWS + wrow + i;
                    if (EPI == kEpiSwiGLU) {
                        float gs = slot_sum(0, n_gate, z), us = slot_sum(n_gate, total, z);
                        gs *= nr;
                        us *= nr;
                        if (orow < (p.n >> 1)) p.y[(size_t)r * (p.n >> 1) + orow] = gs / (1.0f + expf(-gs)) * us;
                    } else {
                        float sum = slot_sum(0, total, z);
                        sum *= nr;
                        if (orow < p.n) {
                            const size_t o = (size_t)r * p.n + orow;
                            if (p.flags & VSPEC_B200_F_RESIDUAL) sum += p.residual[o];
                            p.y[o] = sum;
                        }
                    }
                }
                if (lane == 0) p.counters[ci] = 0;
            }
#pragma unroll
            for (int j = 0; j < RBW; ++j)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) acc[j][nt][0] = acc[j][nt][1] = 0.f;
        };

        for (int b0 = 0; ok && b0 < n_units; b0 += PD) {
#pragma unroll
            for (int st = 0; st < PD; ++st) {
                const int i = b0 + st;
                if (ok && i < n_units) {
                    if (!mbar_wait_sleep(&full[ring], ring_ph, abort_flag, kRingWaitLimit, kRingSleepNs)) {
                        ok = false;
                    } else {
                        const unsigned char* stg = wring + (size_t)ring * STAGE_BYTES;
                        Chunk<BITS> ch[RBW][2];
#pragma unroll
                        for (int j = 0; j < RBW; ++j) {
                            lds_chunk<BITS>(ch[j][0], stg + ring_chunk_offset<BITS>(wrow + 16 * j + g, c));
                            lds_chunk<BITS>(ch[j][1], stg + ring_chunk_offset<BITS>(wrow + 16 * j + g + 8, c));
                        }
                        // the stage is released only after the MMAs that consume
                        // these words (below): releasing it right after the loads let
                        // the refill land before the last loads had read the stage
                        const int stage_used = ring;
                        if (++ring == NS) { ring = 0; ring_ph ^= 1u; }

                        const int kb = c_kb;
                        // e[j][nt][h]: the block's dot product for rows g (h=0) and g+8
                        // of row block j, activation row 4*nt + c, before scaling
                        float e[RBW][NT][2];
                        if constexpr (IMMA) {
                            constexpr int NC = I8Cfg<BITS>::kClasses;
                            const uint4* fb = frag + (size_t)kb * NT * lanes * 2;
                            uint4 bb[NT][2];
#pragma unroll
                            for (int nt = 0; nt < NT; ++nt) {
                                bb[nt][0] = bb[nt][1] = make_uint4(0u, 0u, 0u, 0u);
                                if (lane_has_b) {
                                    bb[nt][0] = fb[(nt * lanes + lane) * 2];
                                    bb[nt][1] = fb[(nt * lanes + lane) * 2 + 1];
                                }
                            }
                            I8Words<BITS> wv[RBW][2];
#pragma unroll
                            for (int j = 0; j < RBW; ++j) {
                                i8_prepare<BITS, UNSIGNED>(ch[j][0], wv[j][0]);
                                i8_prepare<BITS, UNSIGNED>(ch[j][1], wv[j][1]);
                            }
                            int D[RBW][NC][NT][4];
#pragma unroll
                            for (int j = 0; j < RBW; ++j)
#pragma unroll
                                for (int cl = 0; cl < NC; ++cl)
#pragma unroll
                                    for (int nt = 0; nt < NT; ++nt)
                                        D[j][cl][nt][0] = D[j][cl][nt][1] = D[j][cl][nt][2] = D[j][cl][nt][3] = 0;
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
#pragma unroll
                                for (int j = 0; j < RBW; ++j) {
                                    const uint32_t a[4] = {i8_reg<BITS>(wv[j][0], q, 0), i8_reg<BITS>(wv[j][1], q, 0),
                                                           i8_reg<BITS>(wv[j][0], q, 1), i8_reg<BITS>(wv[j][1], q, 1)};
#pragma unroll
                                    for (int nt = 0; nt < NT; ++nt) {
                                        const uint4& b = bb[nt][q >> 1];
                                        imma_16832_u8s8(D[j][i8_class<BITS>(q)][nt], a, (q & 1) ? b.z : b.x,
                                                        (q & 1) ? b.w : b.y);
                                    }
                                }
                            }
#pragma unroll
                            for (int j = 0; j < RBW; ++j)
#pragma unroll
                                for (int nt = 0; nt < NT; ++nt) {
                                    int cmb[4];
#pragma unroll
                                    for (int k4 = 0; k4 < 4; ++k4) {
                                        int v = D[j][0][nt][k4];
#pragma unroll
                                        for (int cl = 1; cl < NC; ++cl) v += D[j][cl][nt][k4] >> i8_class_shift<BITS>(cl);
                                        cmb[k4] = v;
                                    }
                                    e[j][nt][0] = (float)(cmb[0] * 256 + cmb[1]);   // xh * 256 + xl parts
                                    e[j][nt][1] = (float)(cmb[2] * 256 + cmb[3]);
                                }
                        } else {
                        const uint4* fb = frag + (size_t)kb * 4 * NT * lanes;
                        // per row block, even / odd MMAs accumulate apart (shorter chains)
                        float d[RBW][2][NT][4];
#pragma unroll
                        for (int mp = 0; mp < 4; ++mp) {
                            uint4 bb[NT];
#pragma unroll
                            for (int nt = 0; nt < NT; ++nt) {
                                bb[nt] = make_uint4(0u, 0u, 0u, 0u);
                                if (lane_has_b) bb[nt] = fb[(mp * NT + nt) * lanes + lane];
                            }
#pragma unroll
                            for (int hf = 0; hf < 2; ++hf) {
                                const int mm = 2 * mp + hf;
#pragma unroll
                                for (int j = 0; j < RBW; ++j) {
                                    uint32_t a[4];
                                    unpack_mm<BITS, UNSIGNED>(ch[j][0], mm, a[0], a[2]);
                                    unpack_mm<BITS, UNSIGNED>(ch[j][1], mm, a[1], a[3]);
#pragma unroll
                                    for (int nt = 0; nt < NT; ++nt) {
                                        const uint32_t b0r = hf ? bb[nt].z : bb[nt].x;
                                        const uint32_t b1r = hf ? bb[nt].w : bb[nt].y;
                                        if (mp == 0) {
                                            const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
                                            mma_16816_f16(d[j][hf][nt], a, b0r, b1r, zero4);
                                        } else {
                                            mma_16816_f16_acc(d[j][hf][nt], a, b0r, b1r);
                                        }
                                    }
                                }
                            }
                        }
#pragma unroll
                        for (int j = 0; j < RBW; ++j)
#pragma unroll
                            for (int nt = 0; nt < NT; ++nt) {
                                e[j][nt][0] = (d[j][0][nt][0] + d[j][1][nt][0]) + (d[j][0][nt][1] + d[j][1][nt][1]);
                                e[j][nt][1] = (d[j][0][nt][2] + d[j][1][nt][2]) + (d[j][0][nt][3] + d[j][1][nt][3]);
                            }
                        }
                        // every MMA reading this stage's words has issued (volatile
                        // asm keeps them ahead of the arrive; the hardware issues an
                        // MMA only once its registers, i.e. the loads, are complete)
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&empty[stage_used]);
                        float sv[RBW][2], zv[RBW][2];
#pragma unroll
                        for (int j = 0; j < RBW; ++j) {
                            sv[j][0] = has_s ? sz_to_float(sz[st][j][0], SZ16) : 1.0f;
                            sv[j][1] = has_s ? sz_to_float(sz[st][j][2], SZ16) : 1.0f;
                            zv[j][0] = has_zp ? sz_to_float(sz[st][j][1], SZ16) : p.zp_const;
                            zv[j][1] = has_zp ? sz_to_float(sz[st][j][3], SZ16) : p.zp_const;
                        }
                        if (i + PD < n_units) issue_sz(sz[st]);
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt) {
                            const int r = 4 * nt + c;
                            if (r < m) {
                                const float xsum = xs[kb * m + r];
                                const float coff = cs[kb * m + r];
                                const float inv = isc[kb * m + r];
#pragma unroll
                                for (int j = 0; j < RBW; ++j) {
                                    acc[j][nt][0] = fmaf(sv[j][0] * inv, e[j][nt][0] - fmaf(zv[j][0], xsum, coff), acc[j][nt][0]);
                                    acc[j][nt][1] = fmaf(sv[j][1] * inv, e[j][nt][1] - fmaf(zv[j][1], xsum, coff), acc[j][nt][1]);
                                }
                            }
                        }
                        if (++c_kb == kbt || i + 1 == n_units) {
                            flush(c_tile);
                            ++c_tile;
                            c_kb = 0;
                        }
                    }
                }
            }
        }
        if (!ok) {
            *abort_flag = 1;
            atomicOr(&g_ring_timeout, 1);
        }
    } else if (lane == 0) {
        // ======================= TMA producer =================================
        int s = p_issued < NS ? p_issued : 0;
        uint32_t ph = 0;
        if (p_issued == NS) { s = 0; ph = 1; }
        // after the first fill, stage s is next; its previous copy has phase ph ^ 1
        for (; p_issued < n_units; ++p_issued) {
            if (!mbar_wait_sleep(&empty[s], ph ^ 1u, abort_flag, kRingWaitLimit, kRingSleepNs)) {
                *abort_flag = 1;
                atomicOr(&g_ring_timeout, 1);
                break;
            }
            mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
            tma_load_2d(wring + (size_t)s * STAGE_BYTES, &wmap, p_kb * RB, p_tile * TROWS, &full[s]);
            if (++p_kb == kbt) { p_kb = 0; ++p_tile; }
            if (++s == NS) { s = 0; ph ^= 1u; }
        }
        // every issued copy lands before the CTA's shared memory goes away
        const int first = p_issued > NS ? p_issued - NS : 0;
        for (int i = first; i < p_issued; ++i)
            (void)mbar_wait_drain(&full[i % NS], (uint32_t)((i / NS) & 1), kRingWaitLimit);
    }

    if (p.cluster_merge) {
        // Cluster merge (plain epilogue, one tile per cluster of TP CTAs): after
        // the barrier every CTA sums a share of the tile's outputs over the
        // parts' shared-memory partials in part order (deterministic), applies
        // the epilogue and writes y; the second barrier keeps every CTA's
        // shared memory alive until all reads are done.
        constexpr int WR = 16 * RBW;
        __syncwarp();
        cluster_sync_all();
        const int rank = (int)cluster_cta_rank();
        const int outs = TROWS * m;
        const uint32_t cp_addr = smem_u32(cpart);
        for (int o = rank * kRingThreads + tid; o < outs; o += TP * kRingThreads) {
            const int r = o / TROWS, i = o - r * TROWS;
            const uint32_t off = (uint32_t)(((i / WR) * m + r) * WR + (i % WR)) * 4u;
            float sum = 0.f;
            for (int j = 0; j < TP; ++j) sum += ld_dsmem_f32(cp_addr + off, (uint32_t)j);
            const int orow = tp_tile * TROWS + i;
            if (rms) sum *= row_norm[r];
            if (orow < p.n) {
                const size_t o2 = (size_t)r * p.n + orow;
                if (p.flags & VSPEC_B200_F_RESIDUAL) sum += p.residual[o2];
                p.y[o2] = sum;
            }
        }
        cluster_sync_all();
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

// Ring depth and dynamic shared memory: the deepest ring that still lets two
// CTAs share an SM, or, when the activation fragments are too large for that,
// the deepest ring one CTA can hold.  0 when not even 4 stages fit.
template <int BITS>
static int ring_pick_stages(int m, int kbt, size_t* smem_bytes, bool imma) {
    const uint32_t sbytes = (uint32_t)ring_tile_rows(m) * RingCfg<BITS>::kRowBytes;
    const uint32_t stage = sbytes + 16u;   // ring bytes + 2 barriers
    const uint32_t fixed = ring_smem_plan<BITS>(m, kbt, 0, imma).total + 1024u;   // + base alignment
    const int max_ns = (int)(kRingMaxRing / sbytes);
    int ns = fixed < kRingSmemShared ? (int)((kRingSmemShared - fixed) / stage) : 0;
    if (ns > max_ns) ns = max_ns;
    if ((uint32_t)ns * sbytes < kRingMinSharedRing) {
        ns = fixed < kRingSmemMax ? (int)((kRingSmemMax - fixed) / stage) : 0;
        if (ns > max_ns) ns = max_ns;
    }
    if (ns < 3) return 0;
    *smem_bytes = ring_smem_plan<BITS>(m, kbt, ns, imma).total + 1024u;
    return ns;
}

static int ring_stages_for(int bits, int m, int kbt, size_t* smem, bool imma) {
    if (bits == 4) return ring_pick_stages<4>(m, kbt, smem, imma);
    if (bits == 3) return ring_pick_stages<3>(m, kbt, smem, imma);
    return ring_pick_stages<2>(m, kbt, smem, imma);
}

// Integer-MMA decode (VSPEC_B200_GEMV_IMMA, default on; "0" selects the
// fp16-pair decode with hi/lo fp16 activations).
static bool ring_imma() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("VSPEC_B200_GEMV_IMMA");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v != 0;
}

// Persistent CTAs per SM (VSPEC_B200_RING_CTAS_PER_SM, 1 or 2; default 2:
// sixteen decode warps per SM hide the decode/MMA latency chains better than
// leaving room for the next launch).
static int ring_ctas_per_sm() {
    static int v = 0;
    if (v == 0) {
        const char* e = getenv("VSPEC_B200_RING_CTAS_PER_SM");
        v = (e && e[0] == '1') ? 1 : 2;
    }
    return v;
}

struct RingPlan {
    int tiles, grid, max_slots, stages, tile_parts, cluster;
    size_t smem;
    size_t scratch_floats;
};

static RingPlan ring_plan(int m, int n, int k, int bits, bool swiglu, bool imma) {
    RingPlan rp;
    memset(&rp, 0, sizeof(rp));
    const int kbt = k / 128;
    const int trows = ring_tile_rows(m);
    rp.tiles = (n + trows - 1) / trows;
    const long long U = (long long)rp.tiles * kbt;
    rp.stages = ring_stages_for(bits, m, kbt, &rp.smem, imma);
    // two CTAs per SM only when the shared-memory plan lets them co-reside
    const int per_sm = rp.smem <= kRingSmemShared ? ring_ctas_per_sm() : 1;
    const int ctas = device_sm_count() * per_sm;
    rp.grid = (int)(U < ctas ? U : ctas);
    if (rp.grid < 1) return rp;
    const long long per = U / rp.grid;
    int per_tile = (int)((kbt + per - 1) / per) + 1;
    if (per_tile > rp.grid) per_tile = rp.grid;
    // Fewer tiles than CTA slots: split every tile's k-blocks over P CTAs
    // instead, when that costs no more units on the busiest CTA.  No CTA then
    // crosses a tile boundary, so none pays a mid-run merge.
    if (rp.tiles <= ctas) {
        int P = ctas / rp.tiles;
        if (P > kbt) P = kbt;
        const long long tp_max = (kbt + P - 1) / P;
        const long long ct_max = (U + ctas - 1) / ctas;
        if (tp_max <= ct_max) {
            rp.tile_parts = P;
            rp.grid = rp.tiles * P;
            per_tile = P;
        }
    }
    rp.max_slots = swiglu ? 2 * per_tile : per_tile;
    const int logical = swiglu ? rp.tiles / 2 : rp.tiles;
    rp.scratch_floats = (size_t)logical * kRingConsumerWarps * rp.max_slots * (trows / kRingConsumerWarps) * m;
    return rp;
}

bool gemv_ring_supported(const GemvParams& p, int bits, size_t counter_slots) {
    if (p.m < 1 || p.m > kGemvMaxM) return false;
    if (p.k % 128 != 0 || p.n_groups < 1 || p.k % p.n_groups != 0 || (p.k / p.n_groups) % 128 != 0) return false;
    if (reinterpret_cast<uintptr_t>(p.w) % 16 != 0 || reinterpret_cast<uintptr_t>(p.x) % 16 != 0) return false;
    if ((size_t)p.row_bytes % 16 != 0) return false;   // TMA global stride
    if ((p.flags & VSPEC_B200_F_RMSNORM) && reinterpret_cast<uintptr_t>(p.norm_w) % 16 != 0) return false;
    const bool swiglu = (p.flags & VSPEC_B200_F_SWIGLU) != 0;
    const int trows = ring_tile_rows(p.m);
    if (swiglu && ((p.n / 2) % trows != 0)) return false;
    const int tiles = (p.n + trows - 1) / trows;
    const int logical = swiglu ? tiles / 2 : tiles;
    if ((size_t)logical * kRingConsumerWarps > counter_slots) return false;
    size_t smem = 0;
    return ring_stages_for(bits, p.m, p.k / 128, &smem, ring_imma()) > 0;
}

size_t gemv_ring_scratch_floats(int m, int n, int k, bool swiglu) {
    if (k < 128) return 0;
    size_t most = 0;
    for (int bits = 2; bits <= 4; ++bits) {
        for (int im = 0; im < 2; ++im) {
            const size_t f = ring_plan(m, n, k, bits, swiglu, im != 0).scratch_floats;
            if (f > most) most = f;
        }
    }
    return most;
}

int gemv_ring_read_and_clear_timeout(int* out) {
    int v = 0, zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_ring_timeout, sizeof(int));
    if (e != cudaSuccess) return cuda_status(e, "read ring GEMV timeout flag");
    e = cudaMemcpyToSymbol(g_ring_timeout, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_status(e, "clear ring GEMV timeout flag");
    *out = v;
    return VSPEC_B200_OK;
}

// Cluster merge (VSPEC_B200_RING_CLUSTER, default on; "0" keeps the
// global-memory merge for every shape).
static bool ring_cluster_allowed() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("VSPEC_B200_RING_CLUSTER");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v != 0;
}

template <int BITS, int NT, bool UNS, int EPI, bool SZ16, bool IMMA>
static cudaError_t launch_ring_k(const CUtensorMap& map, GemvParams p, int grid, size_t smem, cudaStream_t st,
                                 bool pdl) {
    auto kern = lowbit_gemv_ring_kernel<BITS, NT, UNS, EPI, SZ16, IMMA>;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kRingSmemMax);
        if (e != cudaSuccess) return e;
        // the largest carveout, so two CTAs (this launch and the next) can share an SM
        e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        if (e != cudaSuccess) return e;
        configured[dev] = 1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kRingThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (p.cluster_merge) {
        // every cluster of the grid must be resident at once (one wave): the
        // largest cluster size P' <= P (and <= 8) whose clusters all fit
        // takes the tile's parts; otherwise the global-memory merge.  The
        // occupancy answer is cached per (device, cluster size, smem) and
        // taken before any capture by the first, eager launch of a shape.
        struct Ent { int dev, P, smem, active; };
        static Ent cache[64];
        static int n_cache = 0;
        int dev = 0;
        cudaGetDevice(&dev);
        const int tiles = grid / p.tile_parts;
        // a smaller cluster puts more units on the busiest CTA: accept none
        // for m = 1, at most one more for larger m (whose merge moves more)
        const int kbt_ = p.kb_total;
        const int units0 = (kbt_ + p.tile_parts - 1) / p.tile_parts;
        const int extra_ok = p.m >= 2 ? 1 : 0;
        int chosen = 0;
        for (int P = p.tile_parts < 8 ? p.tile_parts : 8; P >= 2 && !chosen; --P) {
            if ((kbt_ + P - 1) / P - units0 > extra_ok) break;
            int active = -1;
            for (int i = 0; i < n_cache; ++i)
                if (cache[i].dev == dev && cache[i].P == P && cache[i].smem == (int)smem) active = cache[i].active;
            if (active < 0) {
                cudaLaunchAttribute ca;
                ca.id = cudaLaunchAttributeClusterDimension;
                ca.val.clusterDim.x = (unsigned)P;
                ca.val.clusterDim.y = 1;
                ca.val.clusterDim.z = 1;
                cfg.gridDim = dim3(tiles * P);
                cfg.attrs = &ca;
                cfg.numAttrs = 1;
                int nclusters = 0;
                if (cudaOccupancyMaxActiveClusters(&nclusters, kern, &cfg) != cudaSuccess) {
                    (void)cudaGetLastError();
                    nclusters = 0;
                }
                active = nclusters;
                if (n_cache < 64) cache[n_cache++] = Ent{dev, P, (int)smem, active};
            }
            if (active >= tiles) chosen = P;
        }
        if (chosen) {
            p.tile_parts = chosen;
            grid = tiles * chosen;
            cfg.gridDim = dim3(grid);
        } else {
            p.cluster_merge = 0;
        }
    }
    if (p.cluster_merge) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = (unsigned)p.tile_parts;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, kern, map, p);
}

template <int BITS, int NT, bool UNS, int EPI>
static cudaError_t launch_ring_t(const CUtensorMap& map, const GemvParams& p, int grid, size_t smem, cudaStream_t st,
                                 bool pdl) {
    const bool sz16 = (p.flags & VSPEC_B200_F_SZ_F16) != 0;
    if (ring_imma()) {
        if (sz16) return launch_ring_k<BITS, NT, UNS, EPI, true, true>(map, p, grid, smem, st, pdl);
        return launch_ring_k<BITS, NT, UNS, EPI, false, true>(map, p, grid, smem, st, pdl);
    }
    if (sz16) return launch_ring_k<BITS, NT, UNS, EPI, true, false>(map, p, grid, smem, st, pdl);
    return launch_ring_k<BITS, NT, UNS, EPI, false, false>(map, p, grid, smem, st, pdl);
}

template <int BITS, int NT>
static cudaError_t launch_ring_nt(const CUtensorMap& map, const GemvParams& p, bool uns, bool swiglu, int grid,
                                  size_t smem, cudaStream_t st, bool pdl) {
    if (uns) return swiglu ? launch_ring_t<BITS, NT, true, kEpiSwiGLU>(map, p, grid, smem, st, pdl)
                           : launch_ring_t<BITS, NT, true, kEpiPlain>(map, p, grid, smem, st, pdl);
    return swiglu ? launch_ring_t<BITS, NT, false, kEpiSwiGLU>(map, p, grid, smem, st, pdl)
                  : launch_ring_t<BITS, NT, false, kEpiPlain>(map, p, grid, smem, st, pdl);
}

template <int BITS>
static cudaError_t launch_ring_bits(const CUtensorMap& map, const GemvParams& p, bool uns, bool swiglu, int grid,
                                    size_t smem, cudaStream_t st, bool pdl) {
    if (ring_nt(p.m) == 1) return launch_ring_nt<BITS, 1>(map, p, uns, swiglu, grid, smem, st, pdl);
    return launch_ring_nt<BITS, 2>(map, p, uns, swiglu, grid, smem, st, pdl);
}

// p must carry kb_total / kb_per_group(_shift), counters and scratch.
int gemv_ring_launch(GemvParams p, int bits, int unsigned_codes, cudaStream_t st, bool pdl) {
    const bool swiglu = (p.flags & VSPEC_B200_F_SWIGLU) != 0;
    const RingPlan rp = ring_plan(p.m, p.n, p.k, bits, swiglu, ring_imma());
    if (rp.stages <= 0 || rp.grid <= 0) { set_error("shape too large for the ring GEMV"); return VSPEC_B200_ERR_UNSUPPORTED; }
    CUtensorMap map;
    const CUtensorMapSwizzle swz = bits == 4 ? CU_TENSOR_MAP_SWIZZLE_64B
                                 : (bits == 2 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_NONE);
    const int box = bits == 4 ? RingCfg<4>::kRowBytes : (bits == 3 ? RingCfg<3>::kRowBytes : RingCfg<2>::kRowBytes);
    const int rc = make_row_tile_map(&map, p.w, p.n, p.row_bytes, box, ring_tile_rows(p.m), swz);
    if (rc != VSPEC_B200_OK) return rc;
    p.tiles = rp.tiles;
    p.max_slots = rp.max_slots;
    p.total_warps = rp.grid;
    p.stages = rp.stages;
    p.tile_parts = rp.tile_parts;
    p.cluster_merge = (rp.tile_parts >= 2 && rp.tile_parts <= 8 && !swiglu && ring_cluster_allowed()) ? 1 : 0;
    cudaError_t e;
    const bool uns = unsigned_codes != 0;
    if (bits == 4) e = launch_ring_bits<4>(map, p, uns, swiglu, rp.grid, rp.smem, st, pdl);
    else if (bits == 3) e = launch_ring_bits<3>(map, p, uns, swiglu, rp.grid, rp.smem, st, pdl);
    else e = launch_ring_bits<2>(map, p, uns, swiglu, rp.grid, rp.smem, st, pdl);
    if (e != cudaSuccess) return cuda_status(e, "lowbit_gemv_ring_kernel launch");
    return VSPEC_B200_OK;
}

}  // namespace vb200
