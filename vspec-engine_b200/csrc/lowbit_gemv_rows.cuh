// lowbit_gemv_rows.cuh -- row-sliced TMA GEMV for decode (M <= 8): each CTA a
// contiguous range of output rows over all of k, no workspace.
//
// Same contraction and numerics contract as lowbit_gemv_ring.cu (reference
// semantics: src/quant/int4.c:107-132 with the group indexing of
// src/kernel/cuda/fused_linear_int4.cu:391-396; bitstream of
// src/quant/pack.c:53-74):
//     y[i][j] = sum_t x[i][t] * (code(j,t) - zp[j][g(t)]) * s[j][g(t)]
//
// Layout of the work:
//   * CTA c owns the output rows [c*n_out/P, (c+1)*n_out/P) over ALL of k.  No
//     partial sum leaves the CTA, so there is no workspace, no cross-CTA
//     merge and no merge tail, and every CTA streams the same bytes to within
//     one row.
//   * The rows are cut into row groups of BR = 16 * NB rows (NB <= 6, a
//     compile-time constant, so a warp keeps its partial sums of the group's
//     rows in registers; with SwiGLU a gate group is followed by the matching
//     up group).  One
//     unit = (row group, 128-code k-block) = one TMA box [BR rows][row slice]
//     with the ring kernel's swizzle, streamed by one producer thread into a
//     shared-memory ring.  Rows of a box past the CTA's range belong to the
//     next CTA (or lie past the matrix and read as zero): the duplicate lines
//     are served by L2, not HBM.
//   * The 8 consumer warps split k: warp w owns the k-blocks w, w+8, w+16, ...
//     of every group, so the producer streams a group's units in k order
//     (memory order along the rows) and every warp has units in flight from
//     the first ring fill on.
//   * A warp decodes each 16-row block of its unit into mma.sync m16n8k32
//     u8 x s8 fragments against the per-k-block 14-bit integer activation
//     parts (the ring kernel's integer decode: exact int32 block dots), scales
//     the block dot products,
//         part += s * inv_scale * (dot - (zp * X + C)),
//     into its register accumulators.
//   * The group scales (and zero-points) of a row group arrive as one TMA box
//     [BR rows][n_groups] into a double buffer.
//   * At the end of a group each warp stores its partial rows to shared
//     memory, the consumer warps meet at a named barrier, sum the
//     eight warp partials in warp order (deterministic), apply the RMSNorm row
//     factor / residual / SwiGLU and write y.
// Every CTA triggers programmatic dependent launch at its start and requests
// its weights and scales before it waits for the previous kernel; only the
// activation prologue waits.  Every mbarrier wait is bounded.
#pragma once

#include "common.cuh"
#include "lowbit_decode.cuh"
#include "lowbit_kernels.cuh"
#include "tc_primitives.cuh"
#include "tma_map.cuh"

namespace vb200 {

constexpr int kRowsWarps = 8;                        // consumer warps
constexpr int kRowsThreads = (kRowsWarps + 1) * 32;  // + one TMA producer warp
constexpr int kRowsProducerWarp = kRowsWarps;
constexpr uint32_t kRowsWaitLimit = 1u << 16;        // checks of up to kRowsSleepNs each
constexpr uint32_t kRowsSleepNs = 20000;
constexpr uint32_t kRowsSmemShared = 113u * 1024u;   // two CTAs per SM
constexpr uint32_t kRowsSmemMax = 227u * 1024u;
constexpr int kRowsMaxStages = 512;
constexpr int kRowsMaxNB = 6;                      // row groups of up to 96 rows

// Set when a bounded wait of the row-sliced GEMV gave up.  The kernels are
// instantiated per bit width in lowbit_gemv_rows_b{2,3,4}.cu (no relocatable
// device code), so each of those translation units has its own flag.
static __device__ int g_rows_timeout = 0;

__host__ __device__ constexpr int rows_row_bytes(int bits) { return bits == 4 ? 64 : (bits == 3 ? 48 : 32); }
// k-blocks per unit (TMA box): int4 boxes of row groups up to 64 rows carry two
// 128-code k-blocks per row (128 B, 128-byte swizzle), halving the boxes a CTA
// issues; larger row groups keep one k-block per row (64 B, 64-byte swizzle)
// so that a ring of at least kRowsWarps stages fits in half an SM.
__host__ __device__ constexpr int rows_kpu(int bits, int br) { return (bits == 4 && br <= 64) ? 2 : 1; }
__host__ __device__ constexpr int rows_unit_bytes(int bits, int br) { return rows_row_bytes(bits) * rows_kpu(bits, br); }
__host__ __device__ inline int rows_nt(int m) { return (2 * m + 7) / 8; }
__host__ __device__ inline int rows_lanes(int m) { return 4 * (2 * m < 8 ? 2 * m : 8); }
__host__ __device__ inline uint32_t rows_align(uint32_t v, uint32_t a) { return (v + a - 1u) & ~(a - 1u); }

struct RowsGeom {
    int ctas;        // P: CTAs sharing the output rows
    int n_out;       // output rows (n, or n/2 with SwiGLU)
    int br;          // rows per row group (multiple of 16)
    int stages;      // ring depth
    int srow_bytes;  // bytes of one scale row (n_groups * element size)
    int has_s, has_zp;
    int prefetch_delay_ns;   // producer holds its first copies back this long unless the dependency resolved
    int box_rows;            // rows of a weight box and ring stage (a CTA's rows rounded up to 8, <= br)
};

struct RowsSmem {
    uint32_t sbuf, zbuf, frag, xs, cs, is, red, gbuf, bars, misc, total;
};

// Offsets from the 1024-aligned base; the ring starts at 0.
// The ring holds ns stages of box_rows rows; the scale boxes hold br rows.
__host__ __device__ inline RowsSmem rows_smem_plan(int bits, int m, int kbt, int br, int ns, int srow_bytes,
                                                   bool has_s, bool has_zp, bool swiglu, int box_rows) {
    RowsSmem s;
    uint32_t o = (uint32_t)ns * (uint32_t)box_rows * (uint32_t)rows_unit_bytes(bits, br);
    o = rows_align(o, 128u);
    // a CTA holds one row group, so without SwiGLU (gate, up: two physical
    // groups) the scale boxes and warp partials need no second buffer
    const uint32_t nbuf = swiglu ? 2u : 1u;
    s.sbuf = o;
    if (has_s) o += nbuf * (uint32_t)br * (uint32_t)srow_bytes;
    o = rows_align(o, 128u);
    s.zbuf = o;
    if (has_zp) o += nbuf * (uint32_t)br * (uint32_t)srow_bytes;
    o = rows_align(o, 16u);
    s.frag = o;
    o += (uint32_t)kbt * (uint32_t)rows_nt(m) * (uint32_t)rows_lanes(m) * 32u;
    s.xs = o;
    o += (uint32_t)(kbt * m) * 4u;
    s.cs = o;
    o += (uint32_t)(kbt * m) * 4u;
    s.is = o;
    o += (uint32_t)(kbt * m) * 4u;
    s.red = o;                      // [nbuf][warps][m][br] fp32 warp partials
    o += nbuf * kRowsWarps * (uint32_t)m * (uint32_t)br * 4u;
    s.gbuf = o;                     // [m][br] SwiGLU gate sums
    if (swiglu) o += (uint32_t)m * (uint32_t)br * 4u;
    o = rows_align(o, 8u);
    s.bars = o;                     // full[ns], empty[ns], sfull[2], sempty[2]
    o += (2u * (uint32_t)ns + 4u) * 8u;
    s.misc = o;                     // abort flag, row norms [8], units issued
    o += 64u;
    s.total = o;
    return s;
}

// Byte offset of 32-code chunk c of row r inside a ring stage: the swizzle the
// weight tensor map is encoded with (64B for int4, 32B for int2, none for int3).
template <int BITS>
__device__ __forceinline__ uint32_t rows_chunk_offset(int r, int c) {
    if constexpr (BITS == 4) return (uint32_t)(r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
    else if constexpr (BITS == 2) return (uint32_t)(r * 32 + (((c >> 1) ^ ((r >> 2) & 1)) << 4) + 8 * (c & 1));
    else return (uint32_t)(r * 48 + 12 * c);
}

template <int BITS>
__device__ __forceinline__ void rows_lds_chunk(Chunk<BITS>& ch, const unsigned char* p) {
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

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait until the producer thread has issued at least `want` units
// (a volatile shared-memory counter it raises after every copy).
__device__ __forceinline__ bool wait_issued(volatile int* issued, int want, volatile int* abort) {
    if (*issued >= want) return true;
    for (uint32_t i = 0; i < kRowsWaitLimit * 64u; ++i) {
        __nanosleep(64);
        if (*issued >= want) return true;
        if (*abort) return false;
    }
    return false;
}

// NB = 16-row blocks per row group (BR = 16 * NB): a warp's partial sums of
// its rows live in registers for the whole group.
template <int BITS, int NT, bool UNSIGNED, int EPI, bool SZ16, int NB>
__global__ void __launch_bounds__(kRowsThreads, 2)
lowbit_gemv_rows_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap smap,
                        const __grid_constant__ CUtensorMap zmap, const __grid_constant__ GemvParams p,
                        const RowsGeom geo) {
    constexpr int RB = rows_row_bytes(BITS);
    constexpr int KPU = rows_kpu(BITS, 16 * NB);
    constexpr int UB = rows_unit_bytes(BITS, 16 * NB);
    constexpr bool SWIGLU = EPI == kEpiSwiGLU;
    constexpr int S = SWIGLU ? 2 : 1;   // physical groups per row group (gate, up)
    constexpr int SZB = SZ16 ? 2 : 4;
    const int NS = geo.stages;
    constexpr int BR = 16 * NB;
    // A stage holds geo.box_rows <= BR rows.  The 16-row MMA blocks still read
    // BR rows: rows past the box belong to the next stage (or, for the last
    // stage, to the buffers after the ring) and only feed output rows past the
    // CTA's range, which are never stored.
    const uint32_t STAGE_BYTES = (uint32_t)geo.box_rows * UB;

    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    unsigned char* base = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    const int m = p.m;
    const int kbt = p.kb_total;
    const int lanes = rows_lanes(m);
    const bool has_s = geo.has_s != 0, has_zp = geo.has_zp != 0;
    const RowsSmem plan = rows_smem_plan(BITS, m, kbt, BR, NS, geo.srow_bytes, has_s, has_zp, SWIGLU, geo.box_rows);
    unsigned char* wring = base;
    unsigned char* sbuf = base + plan.sbuf;
    unsigned char* zbuf = base + plan.zbuf;
    const uint4* frag = reinterpret_cast<const uint4*>(base + plan.frag);
    float* xs = reinterpret_cast<float*>(base + plan.xs);
    float* cs = reinterpret_cast<float*>(base + plan.cs);
    float* isc = reinterpret_cast<float*>(base + plan.is);
    float* red = reinterpret_cast<float*>(base + plan.red);
    float* gbuf = reinterpret_cast<float*>(base + plan.gbuf);
    uint64_t* full = reinterpret_cast<uint64_t*>(base + plan.bars);
    uint64_t* empty = full + NS;
    uint64_t* sfull = empty + NS;
    uint64_t* sempty = sfull + 2;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(base + plan.misc);
    float* row_norm = reinterpret_cast<float*>(base + plan.misc) + 4;   // [8]
    volatile int* issued = reinterpret_cast<volatile int*>(base + plan.misc) + 12;   // units the producer issued
    volatile int* dep_done = reinterpret_cast<volatile int*>(base + plan.misc) + 13;  // consumers passed the dependency wait

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    // this CTA's output rows and row groups
    const int r0 = (int)(((long long)blockIdx.x * geo.n_out) / geo.ctas);
    const int r1 = (int)(((long long)(blockIdx.x + 1) * geo.n_out) / geo.ctas);
    const int n_grp = (r1 - r0 + BR - 1) / BR;
    const int n_phys = n_grp * S;
    const int kut = kbt / KPU;                   // units per physical group
    const int total_units = n_phys * kut;
    const int q_per_warp = kut / kRowsWarps;     // kut % 8 == 0 (host check)
    const int half_n = p.n >> 1;
    const uint32_t sbytes = (uint32_t)BR * (uint32_t)geo.srow_bytes;
    const uint32_t sz_tx = (has_s ? sbytes : 0u) + (has_zp ? sbytes : 0u);

    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&sfull[b], 1);
            mbar_init(&sempty[b], kRowsWarps);
        }
        *abort_flag = 0;
        *issued = 0;
        *dep_done = 0;
        mbar_fence_init();
    }
    __syncthreads();
    // the next launch in the stream may become resident and stage its weights
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");

    if (warp == kRowsProducerWarp) {
        // ======================= TMA producer =================================
        // One thread streams the units in order, unit u = pg * kbt + kb
        // (k-block kb of physical group pg, consumed by warp kb % 8), with
        // incremental ring counters (no divisions on the issue path).  It
        // never joins the activation prologue or the consumers' barriers, so
        // the ring fills while they wait for the previous kernel.
        if (lane == 0) {
            tma_prefetch_desc(&wmap);
            if (has_s) tma_prefetch_desc(&smap);
            if (has_zp) tma_prefetch_desc(&zmap);
            // While the previous kernel still runs, its activation prologue and
            // refills share this SM's memory path with this CTA's first copies;
            // hold them back a bounded time unless the dependency has resolved
            if (geo.prefetch_delay_ns > 0) {
                const unsigned long long t0 = globaltimer_ns();
                while (!*dep_done && globaltimer_ns() - t0 < (unsigned long long)geo.prefetch_delay_ns)
                    __nanosleep(32);
            }
            bool ok = true;
            int pg = 0, kb = 0, stage = 0, use = 0, sz_issued = 0;
            int row = r0;
            for (int u = 0; u < total_units && ok; ++u) {
                if (kb == 0) {
                    const int b = pg & 1;
                    if (pg >= 2 && !mbar_wait_sleep(&sempty[b], (uint32_t)(((pg >> 1) - 1) & 1), abort_flag,
                                                    kRowsWaitLimit, kRowsSleepNs)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&sfull[b], sz_tx);
                    if (has_s) tma_load_2d(sbuf + (size_t)b * sbytes, &smap, 0, row, &sfull[b]);
                    if (has_zp) tma_load_2d(zbuf + (size_t)b * sbytes, &zmap, 0, row, &sfull[b]);
                    ++sz_issued;
                }
                if (use > 0 && !mbar_wait_sleep(&empty[stage], (uint32_t)((use - 1) & 1), abort_flag, kRowsWaitLimit,
                                                kRowsSleepNs)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
                tma_load_2d(wring + (size_t)stage * STAGE_BYTES, &wmap, kb * UB, row, &full[stage]);
                *issued = u + 1;
                if (++stage == NS) { stage = 0; ++use; }
                if (++kb == kut) {
                    kb = 0;
                    ++pg;
                    row = r0 + (pg / S) * BR + ((SWIGLU && (pg & 1)) ? half_n : 0);
                }
            }
            if (!ok) {
                *abort_flag = 1;
                atomicOr(&g_rows_timeout, 1);
            }
            // every issued copy lands before the CTA's shared memory goes away
            // (bounded, and not cut short by the abort flag)
            const int issued = pg * kut + kb;
            int i = issued > NS ? issued - NS : 0;
            int ds = i % NS;
            uint32_t dph = (uint32_t)((i / NS) & 1);
            for (; i < issued; ++i) {
                (void)mbar_wait_drain(&full[ds], dph, kRowsWaitLimit);
                if (++ds == NS) { ds = 0; dph ^= 1u; }
            }
            for (int q = sz_issued - 2 < 0 ? 0 : sz_issued - 2; q < sz_issued; ++q)
                (void)mbar_wait_drain(&sfull[q & 1], (uint32_t)((q >> 1) & 1), kRowsWaitLimit);
        }
        return;
    }

    // ---- activation prologue (x may be the previous kernel's output) ----
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    if (tid == 0) *dep_done = 1;
    const int K = p.k;
    const bool rms = EPI_HAS_RMSNORM(p.flags);
    if (rms) {
        for (int r = warp; r < m; r += kRowsWarps) {
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
        // Per (k-block, activation row): an exact power-of-two scale sc (block
        // max |x| * sc in [2^13, 2^14)), q = rint(x * sc) in [-2^14, 2^14]
        // split as q = 256 * xh + xl (xh in [-64, 64], xl in [-128, 127]) into
        // the int8 B columns 2r (xh) and 2r + 1 (xl), and X = sum q.  The
        // integer MMAs give sum q * v exactly; the unit epilogue removes the
        // offset (2^(bits-1) + zp) * X and multiplies by s / sc.
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
        constexpr int NW = kRowsWarps;
        constexpr int QB = 4;
        // Each warp quantises the (k-block, row) pairs of exactly the k-blocks
        // its consumer units use (units w, w+8, ... of KPU k-blocks each), so no
        // other warp reads what it writes and a warp-level sync ends the
        // prologue: every warp starts its first unit as soon as its own parts
        // are ready.  kut % 8 == 0 gives every warp the same number of pairs.
        const int per_warp = kbt * m / NW;
        for (int i0 = 0; i0 < per_warp; i0 += QB) {
            float4 v[QB];
            int kbq[QB], rq[QB];
#pragma unroll
            for (int q = 0; q < QB; ++q) {
                const int i = i0 + q;
                const int j = i / m;
                rq[q] = i - j * m;
                kbq[q] = (warp + NW * (j / KPU)) * KPU + (j % KPU);
                v[q] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (i < per_warp) {
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
                if (i0 + q < per_warp) {
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
    }
    __syncwarp();

    {
        // ======================= consumer warps ===============================
        const int g = lane >> 2;
        const int c = lane & 3;
        const bool lane_has_b = lane < lanes;
        constexpr int NC = I8Cfg<BITS>::kClasses;
        bool ok = true;
        // unit positions advance by 8 per unit of a warp: incremental ring slot
        int stage = warp % NS, use = warp / NS;
        for (int pg = 0; pg < n_phys; ++pg) {
            const int par = pg & 1;
            const int grp = pg / S;
            const bool up = SWIGLU && (pg & 1);
            const int orow0 = r0 + grp * BR;
            const int rows_valid = (r1 - orow0) < BR ? (r1 - orow0) : BR;
            float acc[NB][NT][2];
#pragma unroll
            for (int j = 0; j < NB; ++j)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) acc[j][nt][0] = acc[j][nt][1] = 0.f;
            if (ok && !mbar_wait_sleep(&sfull[par], (uint32_t)((pg >> 1) & 1), abort_flag, kRowsWaitLimit,
                                       kRowsSleepNs))
                ok = false;
            const unsigned char* sg = sbuf + (size_t)par * sbytes;
            const unsigned char* zg = zbuf + (size_t)par * sbytes;
            // One unit's contribution to a set of accumulators: every 16-row
            // block of the unit's stage against the k-block's activation parts.
            // One unit's contribution to a set of accumulators: every 16-row
            // block of the unit's stage against its k-blocks' activation parts.
            auto unit_math = [&](const unsigned char* stg, int ku, float (&ac)[NB][NT][2]) {
                uint4 bb[KPU][NT][2];
                float xsum[KPU][NT], coff[KPU][NT], inv[KPU][NT];
                const unsigned char* sgc[KPU];
                const unsigned char* zgc[KPU];
#pragma unroll
                for (int h = 0; h < KPU; ++h) {
                    const int kb = ku * KPU + h;
                    const uint4* fb = frag + (size_t)kb * NT * lanes * 2;
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        bb[h][nt][0] = bb[h][nt][1] = make_uint4(0u, 0u, 0u, 0u);
                        if (lane_has_b) {
                            bb[h][nt][0] = fb[(nt * lanes + lane) * 2];
                            bb[h][nt][1] = fb[(nt * lanes + lane) * 2 + 1];
                        }
                        const int r = 4 * nt + c;
                        const int ri = r < m ? r : 0;
                        xsum[h][nt] = xs[kb * m + ri];
                        coff[h][nt] = cs[kb * m + ri];
                        inv[h][nt] = isc[kb * m + ri];
                    }
                    const int col = p.kb_per_group_shift >= 0 ? (kb >> p.kb_per_group_shift) : kb / p.kb_per_group;
                    sgc[h] = sg + (uint32_t)col * SZB;
                    zgc[h] = zg + (uint32_t)col * SZB;
                }
                // Every 16-row block of the box, also past rows_valid (NB = BR / 16, so
                // those rows are inside the staged box: the next CTA's rows or the
                // zero fill past n; their sums are never stored).  Without a branch per
                // block the blocks form one straight-line region the compiler overlaps.
#pragma unroll
                for (int j = 0; j < NB; ++j) {
                    {
                        const int ra = 16 * j + g, rb2 = ra + 8;
                        Chunk<BITS> ch0[KPU], ch1[KPU];   // rows g and g+8, per k-block of the unit
                        if constexpr (KPU == 2) {
                            // 128-byte swizzle: chunk q of row r at (q ^ (r & 7)) * 16.  Odd rows read
                            // the second k-block first, so each quarter-warp's two rows fall in
                            // opposite bank halves (conflict-free).
                            const int par = g & 1;
                            const int qa = 4 * par + c, qb = 4 * (1 - par) + c;
                            Chunk<BITS> a0, b0, a1, b1;
                            rows_lds_chunk<BITS>(a0, stg + ra * UB + ((qa ^ (ra & 7)) << 4));
                            rows_lds_chunk<BITS>(b0, stg + ra * UB + ((qb ^ (ra & 7)) << 4));
                            rows_lds_chunk<BITS>(a1, stg + rb2 * UB + ((qa ^ (rb2 & 7)) << 4));
                            rows_lds_chunk<BITS>(b1, stg + rb2 * UB + ((qb ^ (rb2 & 7)) << 4));
#pragma unroll
                            for (int wd = 0; wd < BITS; ++wd) {
                                ch0[0].w[wd] = par ? b0.w[wd] : a0.w[wd];
                                ch0[1].w[wd] = par ? a0.w[wd] : b0.w[wd];
                                ch1[0].w[wd] = par ? b1.w[wd] : a1.w[wd];
                                ch1[1].w[wd] = par ? a1.w[wd] : b1.w[wd];
                            }
                        } else {
                            rows_lds_chunk<BITS>(ch0[0], stg + rows_chunk_offset<BITS>(ra, c));
                            rows_lds_chunk<BITS>(ch1[0], stg + rows_chunk_offset<BITS>(rb2, c));
                        }
#pragma unroll
                        for (int h = 0; h < KPU; ++h) {
                            float sv0 = 1.0f, sv1 = 1.0f, zv0 = p.zp_const, zv1 = p.zp_const;
                            if (has_s) {
                                if constexpr (SZ16) {
                                    sv0 = __half2float(*reinterpret_cast<const __half*>(sgc[h] + ra * geo.srow_bytes));
                                    sv1 = __half2float(*reinterpret_cast<const __half*>(sgc[h] + rb2 * geo.srow_bytes));
                                } else {
                                    sv0 = *reinterpret_cast<const float*>(sgc[h] + ra * geo.srow_bytes);
                                    sv1 = *reinterpret_cast<const float*>(sgc[h] + rb2 * geo.srow_bytes);
                                }
                            }
                            if (has_zp) {
                                if constexpr (SZ16) {
                                    zv0 = __half2float(*reinterpret_cast<const __half*>(zgc[h] + ra * geo.srow_bytes));
                                    zv1 = __half2float(*reinterpret_cast<const __half*>(zgc[h] + rb2 * geo.srow_bytes));
                                } else {
                                    zv0 = *reinterpret_cast<const float*>(zgc[h] + ra * geo.srow_bytes);
                                    zv1 = *reinterpret_cast<const float*>(zgc[h] + rb2 * geo.srow_bytes);
                                }
                            }
                            I8Words<BITS> w0, w1;
                            i8_prepare<BITS, UNSIGNED>(ch0[h], w0);
                            i8_prepare<BITS, UNSIGNED>(ch1[h], w1);
                            int D[NC][NT][4];
#pragma unroll
                            for (int cl = 0; cl < NC; ++cl)
#pragma unroll
                                for (int nt = 0; nt < NT; ++nt) D[cl][nt][0] = D[cl][nt][1] = D[cl][nt][2] = D[cl][nt][3] = 0;
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                const uint32_t a[4] = {i8_reg<BITS>(w0, q, 0), i8_reg<BITS>(w1, q, 0),
                                                       i8_reg<BITS>(w0, q, 1), i8_reg<BITS>(w1, q, 1)};
#pragma unroll
                                for (int nt = 0; nt < NT; ++nt) {
                                    const uint4& b = bb[h][nt][q >> 1];
                                    imma_16832_u8s8(D[i8_class<BITS>(q)][nt], a, (q & 1) ? b.z : b.x,
                                                    (q & 1) ? b.w : b.y);
                                }
                            }
#pragma unroll
                            for (int nt = 0; nt < NT; ++nt) {
                                int cmb[4];
#pragma unroll
                                for (int k4 = 0; k4 < 4; ++k4) {
                                    int v = D[0][nt][k4];
#pragma unroll
                                    for (int cl = 1; cl < NC; ++cl) v += D[cl][nt][k4] >> i8_class_shift<BITS>(cl);
                                    cmb[k4] = v;
                                }
                                const float e0 = (float)(cmb[0] * 256 + cmb[1]);   // xh * 256 + xl parts
                                const float e1 = (float)(cmb[2] * 256 + cmb[3]);
                                ac[j][nt][0] = fmaf(sv0 * inv[h][nt], e0 - fmaf(zv0, xsum[h][nt], coff[h][nt]),
                                                    ac[j][nt][0]);
                                ac[j][nt][1] = fmaf(sv1 * inv[h][nt], e1 - fmaf(zv1, xsum[h][nt], coff[h][nt]),
                                                    ac[j][nt][1]);
                            }
                        }
                    }
                }
            };
            // One unit per step, in order: units are issued in order and each
            // warp consumes its own in order, so the oldest unconsumed unit is
            // always issued and the ring cannot stall.  Before the parity wait
            // on a unit's stage a warp checks that the producer has issued the
            // unit: the producer issues unit u only after the stage's previous
            // occupant, unit u - NS, was consumed (so it had landed), hence the
            // stage's full barrier is then at most one phase behind the phase
            // awaited.  Without that check, a stage whose previous occupant
            // belongs to another warp and is still in flight (TMA copies land
            // out of order) passes the parity test one phase early.
            for (int t = 0; t < q_per_warp; ++t) {
                const int ku = kRowsWarps * t + warp;   // unit (k-blocks ku*KPU ...)
                const int cur = stage;
                const uint32_t cur_ph = (uint32_t)(use & 1);
                stage += kRowsWarps;
                while (stage >= NS) { stage -= NS; ++use; }
                // the unit must have been issued before its stage's parity is
                // tested (see above); usually it long has been
                if (ok && !wait_issued(issued, pg * kut + ku + 1, abort_flag)) ok = false;
                if (ok && !mbar_wait_sleep(&full[cur], cur_ph, abort_flag, kRowsWaitLimit, kRowsSleepNs)) ok = false;
                if (!ok) continue;
                unit_math(wring + (size_t)cur * STAGE_BYTES, ku, acc);
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[cur]);
            }
            // this warp is done with the group's scale buffer
            __syncwarp();
            if (lane == 0) mbar_arrive(&sempty[par]);
            // the warp's partial rows into shared memory, [warp][m][BR]
            float* redw = red + (size_t)((par * kRowsWarps + warp) * m) * BR;
#pragma unroll
            for (int j = 0; j < NB; ++j)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    const int r = 4 * nt + c;
                    if (r < m) {
                        redw[r * BR + 16 * j + g] = acc[j][nt][0];
                        redw[r * BR + 16 * j + g + 8] = acc[j][nt][1];
                    }
                }
            // every warp's partial of the group is in shared memory
            named_bar_sync(1, kRowsWarps * 32);
            const int outs = rows_valid * m;
            for (int o = tid; o < outs; o += kRowsWarps * 32) {
                const int r = o / rows_valid, i = o - r * rows_valid;
                const float* rp = red + (size_t)(par * kRowsWarps * m + r) * BR + i;
                float sum = 0.f;
#pragma unroll
                for (int w = 0; w < kRowsWarps; ++w) sum += rp[(size_t)w * m * BR];
                if (rms) sum *= row_norm[r];
                const int orow = orow0 + i;
                if constexpr (SWIGLU) {
                    if (!up) {
                        gbuf[r * BR + i] = sum;
                    } else {
                        const float gs = gbuf[r * BR + i];
                        p.y[(size_t)r * half_n + orow] = gs / (1.0f + expf(-gs)) * sum;
                    }
                } else {
                    const size_t o2 = (size_t)r * p.n + orow;
                    if (p.flags & VSPEC_B200_F_RESIDUAL) sum += p.residual[o2];
                    p.y[o2] = sum;
                }
            }
        }
        if (!ok) {
            *abort_flag = 1;
            atomicOr(&g_rows_timeout, 1);
        }
    }
}

// Launch of the kernel for one bit width (instantiated in lowbit_gemv_rows_b*.cu).
template <int BITS>
cudaError_t rows_launch_bits(const CUtensorMap& wm, const CUtensorMap& sm, const CUtensorMap& zm,
                             const GemvParams& p, const RowsGeom& geo, size_t smem, bool uns, bool swiglu,
                             cudaStream_t st, bool pdl);
// Reads and clears the timeout flag of that translation unit.
template <int BITS>
int rows_timeout_bits(int* out);

}  // namespace vb200
