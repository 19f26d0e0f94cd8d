// lowbit_gemv.cu -- packed int2/int3/int4 dequant-GEMV for decode (M <= 8) on sm_100a.
//
// Contraction (reference semantics, src/quant/int4.c:107-132 with the group
// indexing of src/kernel/cuda/fused_linear_int4.cu:391-396):
//     y[i][j] = sum_t x[i][t] * (code(j,t) - zp[j][g(t)]) * s[j][g(t)]
// with code() the signed LSB-first b-bit field of the reference bitstream
// (src/quant/pack.c:53-74), or the unsigned-offset reading u - 2^(b-1) used by
// the reference int2 kernel (src/kernel/cuda/fused_linear_int2.cu:8-12).
//
// Fast path (K % 128 == 0 and every group a multiple of 128 codes):
//   * Each warp owns a 16-row tile of W and a strided subset of the 128-code
//     k-blocks.  A thread (g = lane/4, c = lane%4) streams one 32-code chunk of
//     rows g and g+8 per k-block with 128/96/64-bit read-only loads, software
//     pipelined PIPE k-blocks deep.
//   * Codes are decoded in registers straight into fp16 pairs (magic-number
//     LOP3 + one f16x2 FMA per pair; exact small integers), which are the A
//     fragments of mma.m16n8k16 -- no shared memory traffic for weights.
//   * The fp32 activation is split into fp16 hi + lo parts (after an exact
//     per-row power-of-two rescale), so the tensor-core product keeps ~22
//     significant bits: each x row occupies two B columns.  The B fragments
//     are staged once per CTA in shared memory, already in fragment order.
//   * Each k-block's fp32 partial is scaled on the fly:
//         acc += s * (dot(x, code) - zp * sum(x over the block)).
//   * Warps reduce through shared memory in a fixed order: deterministic.
#include "common.cuh"
#include "lowbit_decode.cuh"
#include "lowbit_kernels.cuh"

#include <stdio.h>
#include <stdlib.h>

namespace vb200 {

// -------------------------------------------------------------------------
// Persistent split-K GEMV.
//
// Work unit = (16-row tile, 128-code k-block).  Units are numbered tile-major
// and every warp of the (persistent) grid owns a contiguous run of them,
// balanced to +-1 unit, so all SMs stream weights from the first to the last
// cycle of the launch.  A warp keeps PIPE units of loads in flight across
// tile boundaries.  When a warp finishes its part of a tile it publishes the
// fp32 partial to scratch and bumps the tile's counter; the warp that brings
// the counter to the tile's contributor count sums the partials in slot
// (= k) order, applies the epilogue, writes y and resets the counter to zero,
// so the next launch finds it clean.  No warp ever waits on another.
// -------------------------------------------------------------------------
constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * 32;

__host__ __device__ __forceinline__ int gemv_nt(int m) { return (2 * m + 7) / 8; }
__host__ __device__ __forceinline__ int gemv_lanes(int m) { return 4 * (2 * m < 8 ? 2 * m : 8); }

static size_t gemv_smem_bytes(int m, int kbt) {
    const int nt = gemv_nt(m);
    return (size_t)kbt * 4 * nt * gemv_lanes(m) * 16   // B fragments
           + 2 * (size_t)kbt * m * sizeof(float)         // per-(k-block,row) sums X and C
           + (size_t)kGemvWarps * 16 * sizeof(float)     // max-reduction area
           + 32 * sizeof(float);                         // row scale + row norm
}

// warp that owns unit u when U units are split over W warps as
// [floor(w*U/W), floor((w+1)*U/W))
__device__ __forceinline__ int owner_of(long long u, long long U, long long W) {
    return (int)(((u + 1) * W - 1) / U);
}

template <int BITS, int NT, bool UNSIGNED, int EPI>
__global__ void __launch_bounds__(kGemvThreads, 2)
lowbit_gemv_split_kernel(const GemvParams p) {
    constexpr int PIPE = (NT == 1) ? 4 : 3;      // units in flight per warp
    constexpr int CHUNK_BYTES = 4 * BITS;        // 32 codes
    constexpr int KBLOCK_BYTES = 16 * BITS;      // 128 codes

    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int m = p.m;
    const int kbt = p.kb_total;
    const int lanes = gemv_lanes(m);
    uint4* frag = reinterpret_cast<uint4*>(smem_raw);
    float* xs = reinterpret_cast<float*>(smem_raw + (size_t)kbt * 4 * NT * lanes * 16);
    float* cs = xs + (size_t)kbt * m;              // [kbt][m] decode-offset sums
    float* maxbuf = cs + (size_t)kbt * m;          // [kGemvWarps][<=16]
    float* row_scale = maxbuf + kGemvWarps * 16;   // [16]
    float* row_norm = row_scale + 16;              // [16]

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int g = lane >> 2;
    const int c = lane & 3;
    const long long U = (long long)p.tiles * kbt;
    const long long W = p.total_warps;
    const int gw = blockIdx.x * kGemvWarps + warp;
    const bool active = gw < W;
    const long long u0 = active ? ((long long)gw * U) / W : 0;
    const long long u1 = active ? ((long long)(gw + 1) * U) / W : 0;

    // ---- weight stream: issue the first PIPE units before the prologue ----
    // Units are walked with incremental (tile, k-block) cursors: no integer
    // division on the streaming path.
    Chunk<BITS> buf[PIPE][2];
    uint32_t sz[PIPE][4];   // raw bits of s(g), zp(g), s(g+8), zp(g+8)
    const bool sz16 = (p.flags & VSPEC_B200_F_SZ_F16) != 0;
    int itile = (int)(u0 / kbt);
    int ikb = (int)(u0 - (long long)itile * kbt);
    const int grp_shift = p.kb_per_group_shift;   // -1: kb_per_group not a power of two

    auto issue_next = [&](Chunk<BITS> (&b)[2], uint32_t (&s)[4]) {
        const int grp = grp_shift >= 0 ? (ikb >> grp_shift) : ikb / p.kb_per_group;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            int row = itile * 16 + g + 8 * h;
            row = row < p.n ? row : p.n - 1;
            load_chunk<BITS>(b[h], p.w + (size_t)row * p.row_bytes + (size_t)ikb * KBLOCK_BYTES + c * CHUNK_BYTES);
            const size_t sidx = (size_t)row * p.n_groups + grp;
            s[2 * h] = load_sz_raw(p.s, sidx, sz16);       // converted at use
            s[2 * h + 1] = load_sz_raw(p.zp, sidx, sz16);
        }
        if (++ikb == kbt) {
            ikb = 0;
            ++itile;
        }
    };
    const int n_units = (int)(u1 - u0);
#pragma unroll
    for (int st = 0; st < PIPE; ++st)
        if (st < n_units) issue_next(buf[st], sz[st]);

    // ---- activation prologue (once per CTA) ----
    // Everything above touched only immutable weights; x may be the output of
    // the previous kernel in the stream (programmatic dependent launch).
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    const int K = p.k;
    const bool rms = EPI_HAS_RMSNORM(p.flags);
    if (rms) {
        for (int r = warp; r < m; r += kGemvWarps) {
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
    auto xval4 = [&](int r, int t) -> float4 {   // x (or RMSNorm(x)) at t..t+3 of row r
        float4 v = *reinterpret_cast<const float4*>(p.x + (size_t)r * K + t);
        if (rms) {
            const float nr = row_norm[r];
            const float4 wn = *reinterpret_cast<const float4*>(p.norm_w + t);
            v.x = v.x * nr * wn.x; v.y = v.y * nr * wn.y; v.z = v.z * nr * wn.z; v.w = v.w * nr * wn.w;
        }
        return v;
    };
    // (a) per-(k-block, row) sums X = sum x and W = sum x/mult(t), and per-row max |x|
    {
        float mx[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) mx[r] = 0.f;
        const int pairs = kbt * m;
        float mlt[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) mlt[e] = 1.0f / code_mult<BITS>((lane * 4 + e) & 31);
        for (int pr0 = warp; pr0 < pairs; pr0 += 4 * kGemvWarps) {
            float4 v[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {   // four independent loads in flight
                const int pr = pr0 + q * kGemvWarps;
                v[q] = pr < pairs ? xval4(pr % m, (pr / m) * 128 + lane * 4) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int pr = pr0 + q * kGemvWarps;
                if (pr < pairs) {
                    const int r = pr % m, kb = pr / m;
                    const float4 x4 = v[q];
                    const float sx = warp_sum((x4.x + x4.y) + (x4.z + x4.w));
                    const float sw = warp_sum((x4.x * mlt[0] + x4.y * mlt[1]) + (x4.z * mlt[2] + x4.w * mlt[3]));
                    const float a = fmaxf(fmaxf(fabsf(x4.x), fabsf(x4.y)), fmaxf(fabsf(x4.z), fabsf(x4.w)));
#pragma unroll
                    for (int rr = 0; rr < 8; ++rr)
                        if (rr == r) mx[rr] = fmaxf(mx[rr], a);
                    if (lane == 0) {
                        xs[kb * m + r] = sx;
                        cs[kb * m + r] = sw;
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            if (r < m) {
                const float v = warp_max(mx[r]);
                if (lane == 0) maxbuf[warp * 16 + r] = v;
            }
        }
        __syncthreads();
        if (tid < m) {
            float v = 0.f;
            for (int w = 0; w < kGemvWarps; ++w) v = fmaxf(v, maxbuf[w * 16 + tid]);
            // exact power-of-two rescale: max |x| lands in [2^13, 2^14), so the
            // fp16 hi part never overflows and the lo part stays normal
            int ex = 0;
            if (v > 0.f && isfinite(v)) { (void)frexpf(v, &ex); ex -= 14; }
            row_scale[tid] = ldexpf(1.0f, -ex);
        }
        __syncthreads();
    }
    // (b) B fragments: for every (row, k-block, mp, c') the 4 fp16 pairs of MMA
    // slot (kb, mp, lane) as hi and lo parts, in fragment order.
    {
        const int rows_pad = 4 * NT;
        const int items = rows_pad * kbt * 16;
        for (int it = tid; it < items; it += kGemvThreads) {
            const int cc = it & 3;
            const int mp = (it >> 2) & 3;
            const int kb = (it >> 4) % kbt;
            const int r = (it >> 4) / kbt;
            uint4 hi = make_uint4(0u, 0u, 0u, 0u), lo = hi;
            if (r < m) {
                // pair qq of this slot holds codes (lo_code(4mp)+qq, hi_code(4mp)+qq)
                const int t = kb * 128 + 32 * cc;
                const float sc = row_scale[r];
                const int jl = lo_code<BITS>(4 * mp), jh = hi_code<BITS>(4 * mp);
                const float4 a = xval4(r, t + jl), b = xval4(r, t + jh);
                // activation divided by the code's decode multiplier (exact: powers of two)
                const float va[4] = {a.x * sc / code_mult<BITS>(jl), a.y * sc / code_mult<BITS>(jl + 1),
                                     a.z * sc / code_mult<BITS>(jl + 2), a.w * sc / code_mult<BITS>(jl + 3)};
                const float vb[4] = {b.x * sc / code_mult<BITS>(jh), b.y * sc / code_mult<BITS>(jh + 1),
                                     b.z * sc / code_mult<BITS>(jh + 2), b.w * sc / code_mult<BITS>(jh + 3)};
                uint32_t wh[4], wl[4];
#pragma unroll
                for (int qq = 0; qq < 4; ++qq) {
                    const __half h0 = __float2half_rn(va[qq]), h1 = __float2half_rn(vb[qq]);
                    const __half l0 = __float2half_rn(va[qq] - __half2float(h0));
                    const __half l1 = __float2half_rn(vb[qq] - __half2float(h1));
                    wh[qq] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
                    wl[qq] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
                }
                hi = make_uint4(wh[0], wh[1], wh[2], wh[3]);
                lo = make_uint4(wl[0], wl[1], wl[2], wl[3]);
            }
            {
                // columns 2r (hi) and 2r+1 (lo) of n-tile (2r)/8
                const int col = 2 * r;
                const int nt = col >> 3;
                const int gh = col & 7;
                const size_t base = ((size_t)(kb * 4 + mp) * NT + nt) * lanes;
                if (4 * gh + cc < lanes) frag[base + 4 * gh + cc] = hi;
                if (4 * (gh + 1) + cc < lanes) frag[base + 4 * (gh + 1) + cc] = lo;
            }
        }
        // scaled sums: X and the decode offset C = 1024 * W + 2^(bits-1) * X
        constexpr float kOff = (float)(1 << (BITS - 1));
        for (int i = tid; i < kbt * m; i += kGemvThreads) {
            const float sc = row_scale[i % m];
            const float X = xs[i] * sc;
            xs[i] = X;
            cs[i] = fmaf(1024.0f, cs[i] * sc, kOff * X);
        }
    }
    __syncthreads();
    // the next kernel in the stream may start staging its weights now
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    if (!active) return;

    // ---- main stream ----
    const bool lane_has_b = lane < lanes;
    const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
    float acc[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = 0.f;
    int cur_tile = (int)(u0 / kbt);
    const int half_tiles = p.tiles >> 1;

    auto flush = [&](int tile) {
        // contributors of this physical tile and this warp's slot
        const int fw = owner_of((long long)tile * kbt, U, W);
        const int lw = owner_of((long long)(tile + 1) * kbt - 1, U, W);
        int L = tile, slot = gw - fw, total = lw - fw + 1, n_gate = total;
        if (EPI == kEpiSwiGLU) {
            const bool up = tile >= half_tiles;
            L = up ? tile - half_tiles : tile;
            const int gt = L, ut = L + half_tiles;
            const int g_fw = owner_of((long long)gt * kbt, U, W);
            const int g_n = owner_of((long long)(gt + 1) * kbt - 1, U, W) - g_fw + 1;
            const int u_fw = owner_of((long long)ut * kbt, U, W);
            const int u_n = owner_of((long long)(ut + 1) * kbt - 1, U, W) - u_fw + 1;
            n_gate = g_n;
            total = g_n + u_n;
            slot = up ? g_n + (gw - u_fw) : (gw - g_fw);
        }
        float* part = p.scratch + ((size_t)L * p.max_slots + slot) * (16 * m);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int r = 4 * nt + c;
            if (r < m) {
                part[r * 16 + g] = acc[nt][0];
                part[r * 16 + g + 8] = acc[nt][1];
            }
        }
        __threadfence();
        __syncwarp();
        int old = 0;
        if (lane == 0) old = atomicAdd(p.counters + L, 1);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old == total - 1) {
            __threadfence();
            const float* base = p.scratch + (size_t)L * p.max_slots * (16 * m);
            for (int z = lane; z < 16 * m; z += 32) {
                const int r = z >> 4, i = z & 15;
                const float inv = 1.0f / row_scale[r];
                if (EPI == kEpiSwiGLU) {
                    float gs = 0.f, us = 0.f;
                    for (int s = 0; s < n_gate; ++s) gs += __ldcg(base + (size_t)s * 16 * m + z);
                    for (int s = n_gate; s < total; ++s) us += __ldcg(base + (size_t)s * 16 * m + z);
                    gs *= inv;
                    us *= inv;
                    const int orow = L * 16 + i;
                    if (orow < (p.n >> 1)) p.y[(size_t)r * (p.n >> 1) + orow] = gs / (1.0f + expf(-gs)) * us;
                } else {
                    float sum = 0.f;
                    for (int s = 0; s < total; ++s) sum += __ldcg(base + (size_t)s * 16 * m + z);
                    sum *= inv;
                    const int orow = L * 16 + i;
                    if (orow < p.n) {
                        const size_t o = (size_t)r * p.n + orow;
                        if (p.flags & VSPEC_B200_F_RESIDUAL) sum += p.residual[o];
                        p.y[o] = sum;
                    }
                }
            }
            if (lane == 0) p.counters[L] = 0;
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = 0.f;
    };

    int ckb = (int)(u0 - (long long)cur_tile * kbt);
    for (int base_i = 0; base_i < n_units; base_i += PIPE) {
#pragma unroll
        for (int st = 0; st < PIPE; ++st) {
            const int i = base_i + st;
            if (i < n_units) {
                const int kb = ckb;
                float d[NT][4];
                const uint4* fb = frag + (size_t)kb * 4 * NT * lanes;
#pragma unroll
                for (int mp = 0; mp < 4; ++mp) {
                    uint4 bb[NT];
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        bb[nt] = make_uint4(0u, 0u, 0u, 0u);
                        if (lane_has_b) bb[nt] = fb[(mp * NT + nt) * lanes + lane];
                    }
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        const int mm = 2 * mp + half;
                        // A fragment: rows g / g+8, k-slots {2c,2c+1} and {2c+8,2c+9}
                        uint32_t a[4];
                        unpack_mm<BITS, UNSIGNED>(buf[st][0], mm, a[0], a[2]);
                        unpack_mm<BITS, UNSIGNED>(buf[st][1], mm, a[1], a[3]);
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt) {
                            const uint32_t b0 = half ? bb[nt].z : bb[nt].x;
                            const uint32_t b1 = half ? bb[nt].w : bb[nt].y;
                            mma_16816_f16(d[nt], a, b0, b1, mm == 0 ? zero4 : d[nt]);
                        }
                    }
                }
                const float s0 = p.s ? sz_to_float(sz[st][0], sz16) : 1.0f;
                const float s1 = p.s ? sz_to_float(sz[st][2], sz16) : 1.0f;
                const float z0 = p.zp ? sz_to_float(sz[st][1], sz16) : p.zp_const;
                const float z1 = p.zp ? sz_to_float(sz[st][3], sz16) : p.zp_const;
                // refill this stage while the tensor cores drain
                if (i + PIPE < n_units) issue_next(buf[st], sz[st]);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    const int r = 4 * nt + c;
                    if (r < m) {
                        const float xsum = xs[kb * m + r];
                        const float coff = cs[kb * m + r];
                        acc[nt][0] = fmaf(s0, (d[nt][0] + d[nt][1]) - fmaf(z0, xsum, coff), acc[nt][0]);
                        acc[nt][1] = fmaf(s1, (d[nt][2] + d[nt][3]) - fmaf(z1, xsum, coff), acc[nt][1]);
                    }
                }
                // advance the consume cursor; publish a finished tile part
                if (++ckb == kbt || i + 1 == n_units) {
                    flush(cur_tile);
                    ++cur_tile;
                    ckb = 0;
                }
            }
        }
    }
}

// -------------------------------------------------------------------------
// Generic path: any k, any group count, any alignment.  One warp per output
// row; lanes stride the reduction; fp32 FMA; fixed-order warp reduction.
// -------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
lowbit_gemv_generic_kernel(const GemvParams p, int bits, int unsigned_codes, int n_rows_total) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= n_rows_total) return;
    const int j = warp;  // weight row
    const size_t K = (size_t)p.k;
    const uint8_t* wrow = p.w + (size_t)j * p.row_bytes;
    for (int i = 0; i < p.m; ++i) {
        const float* xr = p.x + (size_t)i * K;
        float nr = 1.0f;
        if (EPI_HAS_RMSNORM(p.flags)) {
            float ss = 0.f;
            for (size_t t = lane; t < K; t += 32) ss += xr[t] * xr[t];
            ss = warp_sum(ss);
            nr = 1.0f / sqrtf(ss / (float)K + p.eps);
        }
        float acc = 0.f;
        for (size_t t = lane; t < K; t += 32) {
            const size_t idx = (size_t)j * p.n_groups + group_of(t, K, (size_t)p.n_groups);
            float sv, zv;
            if (p.flags & VSPEC_B200_F_SZ_F16) {
                sv = p.s ? __half2float(reinterpret_cast<const __half*>(p.s)[idx]) : 1.0f;
                zv = p.zp ? __half2float(reinterpret_cast<const __half*>(p.zp)[idx]) : p.zp_const;
            } else {
                sv = p.s ? reinterpret_cast<const float*>(p.s)[idx] : 1.0f;
                zv = p.zp ? reinterpret_cast<const float*>(p.zp)[idx] : p.zp_const;
            }
            float xv = xr[t];
            if (EPI_HAS_RMSNORM(p.flags)) xv = xv * nr * p.norm_w[t];
            const float q = (float)decode_code_generic(wrow, t, bits, unsigned_codes);
            acc = fmaf(xv, (q - zv) * sv, acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) {
            const size_t o = (size_t)i * p.n + j;
            if (p.flags & VSPEC_B200_F_RESIDUAL) acc += p.residual[o];
            p.y[o] = acc;
        }
    }
}

// SwiGLU combine for the generic path: y_act[i][j] = silu(y[i][j]) * y[i][n/2 + j].
__global__ void swiglu_combine_kernel(const float* y_full, float* y_act, int m, int half_n) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= m * half_n) return;
    const int i = idx / half_n, j = idx % half_n;
    const float gt = y_full[(size_t)i * 2 * half_n + j];
    const float up = y_full[(size_t)i * 2 * half_n + half_n + j];
    y_act[idx] = gt / (1.0f + expf(-gt)) * up;
}

// -------------------------------------------------------------------------
// Debug/parity kernel: decode every code of a packed matrix with the exact
// device routine the fast GEMV uses (fast layout) or the generic decoder.
// -------------------------------------------------------------------------
template <int BITS, bool UNSIGNED>
__global__ void unpack_codes_fast_kernel(const uint8_t* w, int n, int k, int row_bytes, int8_t* out) {
    const size_t chunk = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t chunks_per_row = (size_t)k / 32;
    if (chunk >= (size_t)n * chunks_per_row) return;
    const size_t row = chunk / chunks_per_row, ci = chunk % chunks_per_row;
    Chunk<BITS> cbuf;
    const uint8_t* src = w + row * row_bytes + ci * (4 * BITS);
    uint8_t tmp[4 * BITS];   // byte-wise gather: no alignment assumption
    for (int i = 0; i < 4 * BITS; ++i) tmp[i] = src[i];
    for (int i = 0; i < BITS; ++i)
        cbuf.w[i] = (uint32_t)tmp[4 * i] | ((uint32_t)tmp[4 * i + 1] << 8) | ((uint32_t)tmp[4 * i + 2] << 16) |
                    ((uint32_t)tmp[4 * i + 3] << 24);
    int8_t* o = out + row * (size_t)k + ci * 32;
#pragma unroll
    for (int mm = 0; mm < 8; ++mm) {
        uint32_t h[2];
        unpack_mm<BITS, UNSIGNED>(cbuf, mm, h[0], h[1]);
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int q = 2 * mm + e;
            const __half2 v = *reinterpret_cast<const __half2*>(&h[e]);
            const int jl = lo_code<BITS>(q), jh = hi_code<BITS>(q);
            // decoded value = 1024 + mult * u, code = u - 2^(bits-1)
            o[jl] = (int8_t)((int)((__half2float(__low2half(v)) - 1024.0f) / code_mult<BITS>(jl)) - (1 << (BITS - 1)));
            o[jh] = (int8_t)((int)((__half2float(__high2half(v)) - 1024.0f) / code_mult<BITS>(jh)) - (1 << (BITS - 1)));
        }
    }
}

__global__ void unpack_codes_generic_kernel(const uint8_t* w, int n, int k, int row_bytes, int bits, int unsigned_codes,
                                            int8_t* out) {
    const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (size_t)n * k) return;
    const size_t row = idx / k, t = idx % k;
    out[idx] = (int8_t)decode_code_generic(w + row * row_bytes, t, bits, unsigned_codes);
}

// -------------------------------------------------------------------------
// Host-side dispatch
// -------------------------------------------------------------------------
// -------------------------------------------------------------------------
// Host-side dispatch
// -------------------------------------------------------------------------
static bool fast_path_ok(const GemvParams& p, int bits) {
    if (p.m < 1 || p.m > kGemvMaxM) return false;
    if (p.k % 128 != 0) return false;
    if (p.n_groups < 1 || p.k % p.n_groups != 0) return false;
    const int gsize = p.k / p.n_groups;
    if (gsize % 128 != 0) return false;
    if ((size_t)p.row_bytes != row_bytes_for((size_t)p.k, bits)) return false;
    const uintptr_t a = reinterpret_cast<uintptr_t>(p.w);
    const int need = bits == 4 ? 16 : (bits == 2 ? 8 : 4);
    if (a % need != 0) return false;
    if (reinterpret_cast<uintptr_t>(p.x) % 16 != 0) return false;
    if ((p.flags & VSPEC_B200_F_RMSNORM) && reinterpret_cast<uintptr_t>(p.norm_w) % 16 != 0) return false;
    if (gemv_smem_bytes(p.m, p.k / 128) > kGemvMaxSmem) return false;
    if ((size_t)(p.n + 15) / 16 > 16384) return false;   // counter region of the workspace
    return true;
}

// Warps of the persistent grid and partial slots per tile for a launch.
struct SplitPlan {
    int tiles;          // physical 16-row tiles
    int logical_tiles;  // tiles owning a counter (SwiGLU pairs gate+up tiles)
    long long units;
    int total_warps;
    int max_slots;
    int grid;
    size_t scratch_floats;
};

static SplitPlan split_plan(int m, int n, int k, bool swiglu) {
    SplitPlan sp;
    sp.tiles = (n + 15) / 16;
    sp.logical_tiles = swiglu ? sp.tiles / 2 : sp.tiles;
    const int kbt = k / 128;
    sp.units = (long long)sp.tiles * kbt;
    const long long target = (long long)device_sm_count() * 2 * kGemvWarps;
    sp.total_warps = (int)(sp.units < target ? sp.units : target);
    const long long per = sp.units / sp.total_warps;  // >= 1
    int per_tile = (int)((kbt + per - 1) / per) + 1;  // contributors of one physical tile
    if (per_tile > sp.total_warps) per_tile = sp.total_warps;
    sp.max_slots = swiglu ? 2 * per_tile : per_tile;
    sp.grid = (sp.total_warps + kGemvWarps - 1) / kGemvWarps;
    sp.scratch_floats = (size_t)sp.logical_tiles * sp.max_slots * 16 * m;
    return sp;
}

// Workspace layout: a fixed region of kGemvCounterSlots int counters (zero
// between launches: every merge resets the counter it used) followed by the
// fp32 partials.  The counter region does not depend on the shape, so one
// workspace serves any sequence of stream-ordered launches of any shape.
constexpr size_t kGemvCounterSlots = 16384;
constexpr size_t kGemvCounterBytes = kGemvCounterSlots * sizeof(int);

size_t gemv_workspace_bytes(int m, int n, int k, bool swiglu) {
    if (m < 1 || n < 1 || k < 128) return 0;
    const int mm = m > kGemvMaxM ? kGemvMaxM : m;
    SplitPlan sp = split_plan(mm, n, k, swiglu);
    size_t floats = sp.scratch_floats;
    const size_t tc = gemv_tc_scratch_floats(mm, n, k, swiglu);
    if (tc > floats) floats = tc;
    const size_t ring = gemv_ring_scratch_floats(mm, n, k, swiglu);
    if (ring > floats) floats = ring;
    size_t bytes = kGemvCounterBytes + floats * sizeof(float);
    if (m > kGemvMaxM) {
        const size_t gemm = kGemvCounterBytes + gemm_tc_workspace_bytes(m, n, k, swiglu);
        if (gemm > bytes) bytes = gemm;
    }
    return bytes;
}

// VSPEC_B200_GEMM=0 makes the dispatcher run m > 8 as row blocks of the GEMV.
static bool gemm_path_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("VSPEC_B200_GEMM");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v == 1;
}

// VSPEC_B200_GEMV_RING=0 makes the dispatcher skip the ring kernel (A/B timing).
static bool ring_path_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("VSPEC_B200_GEMV_RING");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v == 1;
}

// Row-sliced kernel in the automatic dispatch (VSPEC_B200_GEMV_ROWS): unset =
// the shapes where it measured faster (2), "1" = every shape it supports (1),
// "0" = never (0, A/B timing).
static int rows_path_mode() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("VSPEC_B200_GEMV_ROWS");
        v = (e && e[0] == '1') ? 1 : ((e && e[0] == '0') ? 0 : 2);
    }
    return v;
}

// Library-managed workspace: one grow-only, zero-initialized buffer per device
// and host thread (each host thread is expected to use one stream).
struct GemvWs {
    void* ptr;
    size_t cap;
};
static thread_local GemvWs g_gemv_ws[64];

static void* gemv_managed_ws(size_t bytes) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    GemvWs& w = g_gemv_ws[dev];
    if (w.cap < bytes) {
        if (w.ptr) {
            cudaDeviceSynchronize();
            cudaFree(w.ptr);
        }
        w.ptr = nullptr;
        w.cap = 0;
        size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
        if (cudaMalloc(&w.ptr, want) != cudaSuccess) { w.ptr = nullptr; return nullptr; }
        if (cudaMemset(w.ptr, 0, want) != cudaSuccess) { cudaFree(w.ptr); w.ptr = nullptr; return nullptr; }
        if (cudaDeviceSynchronize() != cudaSuccess) { cudaFree(w.ptr); w.ptr = nullptr; return nullptr; }
        w.cap = want;
    }
    return w.ptr;
}

// VSPEC_B200_PDL=0 disables programmatic dependent launch (A/B timing).
static bool pdl_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("VSPEC_B200_PDL");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v == 1;
}

template <int BITS, int NT, bool UNS, int EPI>
static cudaError_t launch_split_t(const GemvParams& p, int grid, size_t smem, cudaStream_t st) {
    auto kern = lowbit_gemv_split_kernel<BITS, NT, UNS, EPI>;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && (size_t)configured[dev] < smem) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemvMaxSmem);
        if (e != cudaSuccess) return e;
        configured[dev] = (int)kGemvMaxSmem;
    }
    // Programmatic dependent launch: the kernel prefetches weights before
    // griddepcontrol.wait, overlapping the previous kernel's tail.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int BITS, bool UNS>
static cudaError_t launch_split_bits(const GemvParams& p, int epi, int grid, size_t smem, cudaStream_t st) {
    const int nt = gemv_nt(p.m);
    if (epi == kEpiSwiGLU) {
        return nt == 1 ? launch_split_t<BITS, 1, UNS, kEpiSwiGLU>(p, grid, smem, st)
                       : launch_split_t<BITS, 2, UNS, kEpiSwiGLU>(p, grid, smem, st);
    }
    return nt == 1 ? launch_split_t<BITS, 1, UNS, kEpiPlain>(p, grid, smem, st)
                   : launch_split_t<BITS, 2, UNS, kEpiPlain>(p, grid, smem, st);
}

int lowbit_gemv_launch(GemvParams p, int bits, int unsigned_codes, cudaStream_t st, int path,
                       void* workspace, size_t workspace_bytes) {
    const int force_generic = path == kPathGeneric;
    if (bits < 2 || bits > 4) { set_error("bits must be 2, 3 or 4 (got %d)", bits); return VSPEC_B200_ERR_ARG; }
    const bool swiglu = (p.flags & VSPEC_B200_F_SWIGLU) != 0;
    if (swiglu && (p.n % 2 != 0)) { set_error("SwiGLU needs an even row count (n=%d)", p.n); return VSPEC_B200_ERR_ARG; }
    p.kb_total = p.k / 128;
    p.kb_per_group = (p.n_groups > 0 && p.k % p.n_groups == 0) ? (p.k / p.n_groups) / 128 : 1;
    if (p.kb_per_group < 1) p.kb_per_group = 1;
    p.kb_per_group_shift = -1;
    for (int sh = 0; sh < 31; ++sh)
        if ((1 << sh) == p.kb_per_group) p.kb_per_group_shift = sh;

    if (p.m > kGemvMaxM) {
        // large m: the tcgen05 GEMM where it applies, else row blocks of the GEMV
        if (!force_generic && (path == kPathTensorCore || (path == kPathAuto && gemm_path_enabled())) &&
            gemm_tc_supported(p, bits, kGemvCounterSlots)) {
            const size_t need = kGemvCounterBytes + gemm_tc_workspace_bytes(p.m, p.n, p.k, swiglu);
            void* ws = workspace;
            if (ws) {
                if (workspace_bytes < need) {
                    set_error("GEMM workspace too small (%zu < %zu)", workspace_bytes, need);
                    return VSPEC_B200_ERR_ARG;
                }
            } else {
                ws = gemv_managed_ws(need);
                if (!ws) { set_error("cannot allocate %zu bytes of GEMM workspace", need); return VSPEC_B200_ERR_NOMEM; }
            }
            p.counters = reinterpret_cast<int*>(ws);
            return gemm_tc_launch(p, bits, unsigned_codes, st, reinterpret_cast<char*>(ws) + kGemvCounterBytes);
        }
        if (path == kPathTensorCore) {
            set_error("shape not supported by the tcgen05 GEMM (k %% 128 == 0, groups of 128*i, n/2 %% 128 == 0 "
                      "with SwiGLU)");
            return VSPEC_B200_ERR_UNSUPPORTED;
        }
        const size_t out_cols = swiglu ? (size_t)p.n / 2 : (size_t)p.n;
        for (int i0 = 0; i0 < p.m; i0 += kGemvMaxM) {
            GemvParams q = p;
            q.m = (p.m - i0) < kGemvMaxM ? (p.m - i0) : kGemvMaxM;
            q.x = p.x + (size_t)i0 * p.k;
            q.y = p.y + (size_t)i0 * out_cols;
            if (p.residual) q.residual = p.residual + (size_t)i0 * p.n;
            const int rc = lowbit_gemv_launch(q, bits, unsigned_codes, st, path, workspace, workspace_bytes);
            if (rc != VSPEC_B200_OK) return rc;
        }
        return VSPEC_B200_OK;
    }

    const bool fast = !force_generic && fast_path_ok(p, bits) && (!swiglu || (p.n / 2) % 16 == 0);
    // The fast kernels hold every k-block of the m activation rows in shared
    // memory, so deep k at m up to 8 (e.g. k = 12288, m = 8) can exceed it
    // while half the rows fit.  Automatic dispatch then runs the rows in two
    // halves instead of the one-warp-per-row generic kernel (at m = 8, n = 4096,
    // k = 12288 that is ~35 us against ~1.5 ms).
    // Two halves also for m > 4 on large weights: past four activation rows
    // the fast kernels run two MMA column tiles, and from n * k = 12288 * 4096
    // on that costs 2.1-2.3x the one-tile time, more than reading the weights
    // twice (measured, W4 k = 4096, m = 6 / 8: n = 12288 23.6 / 26.1 us against
    // 20.9 / 21.6 in halves; SwiGLU n = 24576 43.0 / 47.1 against 35.9 / 39.4;
    // n = 151936 168 / 173 against 138 / 145).  Below it one call is faster
    // (n = 6144, m = 8: 15.4 against 21.5 us).
    const bool big_halves = fast && path == kPathAuto && p.m > 4 && (long long)p.n * p.k >= 12288LL * 4096LL;
    if ((!fast || big_halves) && path == kPathAuto && p.m > 1) {
        GemvParams h = p;
        h.m = (p.m + 1) / 2;
        if (fast_path_ok(h, bits) && (!swiglu || (p.n / 2) % 16 == 0)) {
            const size_t out_cols = swiglu ? (size_t)p.n / 2 : (size_t)p.n;
            for (int i0 = 0; i0 < p.m; i0 += h.m) {
                GemvParams q = p;
                q.m = (p.m - i0) < h.m ? (p.m - i0) : h.m;
                q.x = p.x + (size_t)i0 * p.k;
                q.y = p.y + (size_t)i0 * out_cols;
                if (p.residual) q.residual = p.residual + (size_t)i0 * p.n;
                const int rc = lowbit_gemv_launch(q, bits, unsigned_codes, st, path, workspace, workspace_bytes);
                if (rc != VSPEC_B200_OK) return rc;
            }
            return VSPEC_B200_OK;
        }
    }
    // The row-sliced kernel needs no workspace: it runs before any is taken (a
    // caller workspace is still checked against the documented size).
    const int rows_mode = rows_path_mode();
    const bool rows_auto = path == kPathAuto && (rows_mode == 1 ? gemv_rows_supported(p, bits)
                                                 : (rows_mode == 2 && gemv_rows_preferred(p, bits)));
    if (!force_generic && (path == kPathRows || rows_auto)) {
        if (gemv_rows_supported(p, bits)) {
            if (fast && workspace && workspace_bytes < gemv_workspace_bytes(p.m, p.n, p.k, swiglu)) {
                set_error("GEMV workspace too small (%zu < %zu)", workspace_bytes,
                          gemv_workspace_bytes(p.m, p.n, p.k, swiglu));
                return VSPEC_B200_ERR_ARG;
            }
            return gemv_rows_launch(p, bits, unsigned_codes, st, pdl_enabled());
        }
        if (path == kPathRows) {
            set_error("shape not supported by the row-sliced GEMV (m <= 8, k %% 1024 == 0 (int4: k %% 2048 == 0), "
                      "groups of 128*i, 16-byte aligned rows / scale rows, smem)");
            return VSPEC_B200_ERR_UNSUPPORTED;
        }
    }
    if (!fast && (path == kPathWarpMma || path == kPathTensorCore || path == kPathRing)) {
        set_error("shape not supported by the requested fast path");
        return VSPEC_B200_ERR_UNSUPPORTED;
    }
    if (fast) {
        SplitPlan sp = split_plan(p.m, p.n, p.k, swiglu);
        const size_t need = gemv_workspace_bytes(p.m, p.n, p.k, swiglu);
        void* ws = workspace;
        if (ws) {
            if (workspace_bytes < need) {
                set_error("GEMV workspace too small (%zu < %zu)", workspace_bytes, need);
                return VSPEC_B200_ERR_ARG;
            }
        } else {
            ws = gemv_managed_ws(need);
            if (!ws) { set_error("cannot allocate %zu bytes of GEMV workspace", need); return VSPEC_B200_ERR_NOMEM; }
        }
        p.counters = reinterpret_cast<int*>(ws);
        p.scratch = reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + kGemvCounterBytes);
        if (path == kPathTensorCore) {
            if (!gemv_tc_supported(p, bits, kGemvCounterSlots)) {
                set_error("shape not supported by the tcgen05 GEMV (m <= 4, groups of 128*i, smem)");
                return VSPEC_B200_ERR_UNSUPPORTED;
            }
            return gemv_tc_launch(p, bits, unsigned_codes, st, pdl_enabled());
        }
        if (path == kPathRing || path == kPathAuto) {
            const bool ring_ok = gemv_ring_supported(p, bits, kGemvCounterSlots);
            if (path == kPathRing && !ring_ok) {
                set_error("shape not supported by the ring GEMV (m <= 8, groups of 128*i, smem, n)");
                return VSPEC_B200_ERR_UNSUPPORTED;
            }
            if (ring_ok && (path == kPathRing || ring_path_enabled()))
                return gemv_ring_launch(p, bits, unsigned_codes, st, pdl_enabled());
        }
        p.tiles = sp.tiles;
        p.total_warps = sp.total_warps;
        p.max_slots = sp.max_slots;
        const size_t smem = gemv_smem_bytes(p.m, p.kb_total);
        const int epi = swiglu ? kEpiSwiGLU : kEpiPlain;
        cudaError_t e;
        if (unsigned_codes) {
            if (bits == 4) e = launch_split_bits<4, true>(p, epi, sp.grid, smem, st);
            else if (bits == 3) e = launch_split_bits<3, true>(p, epi, sp.grid, smem, st);
            else e = launch_split_bits<2, true>(p, epi, sp.grid, smem, st);
        } else {
            if (bits == 4) e = launch_split_bits<4, false>(p, epi, sp.grid, smem, st);
            else if (bits == 3) e = launch_split_bits<3, false>(p, epi, sp.grid, smem, st);
            else e = launch_split_bits<2, false>(p, epi, sp.grid, smem, st);
        }
        if (e != cudaSuccess) return cuda_status(e, "lowbit_gemv_split_kernel launch");
        return VSPEC_B200_OK;
    }
    // generic path
    if (swiglu) {
        set_error("SwiGLU epilogue requires the fast path shape (k %% 128 == 0, groups of 128*i, n/2 %% 16 == 0, m <= %d)",
                  kGemvMaxM);
        return VSPEC_B200_ERR_UNSUPPORTED;
    }
    const int rows = p.n;
    const int threads = 256;
    const int blocks = (rows * 32 + threads - 1) / threads;
    lowbit_gemv_generic_kernel<<<blocks, threads, 0, st>>>(p, bits, unsigned_codes, rows);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e, "lowbit_gemv_generic_kernel launch");
    return VSPEC_B200_OK;
}

int unpack_codes_launch(const uint8_t* w, int n, int k, int bits, int unsigned_codes, int8_t* out, cudaStream_t st,
                        int use_fast_decoder) {
    const int rb = (int)row_bytes_for((size_t)k, bits);
    if (use_fast_decoder) {
        if (k % 32 != 0) { set_error("fast decoder needs k %% 32 == 0"); return VSPEC_B200_ERR_ARG; }
        const size_t chunks = (size_t)n * (k / 32);
        const int threads = 256;
        const unsigned blocks = (unsigned)((chunks + threads - 1) / threads);
        if (bits == 4) unsigned_codes ? unpack_codes_fast_kernel<4, true><<<blocks, threads, 0, st>>>(w, n, k, rb, out)
                                      : unpack_codes_fast_kernel<4, false><<<blocks, threads, 0, st>>>(w, n, k, rb, out);
        else if (bits == 3) unsigned_codes ? unpack_codes_fast_kernel<3, true><<<blocks, threads, 0, st>>>(w, n, k, rb, out)
                                           : unpack_codes_fast_kernel<3, false><<<blocks, threads, 0, st>>>(w, n, k, rb, out);
        else unsigned_codes ? unpack_codes_fast_kernel<2, true><<<blocks, threads, 0, st>>>(w, n, k, rb, out)
                            : unpack_codes_fast_kernel<2, false><<<blocks, threads, 0, st>>>(w, n, k, rb, out);
    } else {
        const size_t total = (size_t)n * k;
        const int threads = 256;
        unpack_codes_generic_kernel<<<(unsigned)((total + threads - 1) / threads), threads, 0, st>>>(
            w, n, k, rb, bits, unsigned_codes, out);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e, "unpack_codes launch");
    return VSPEC_B200_OK;
}

}  // namespace vb200
