// lowbit_gemv_rows.cu -- host side of the row-sliced TMA GEMV (kernel in
// lowbit_gemv_rows.cuh, instantiated per bit width in lowbit_gemv_rows_b*.cu):
// geometry planner, tensor maps, dispatch.
#include "lowbit_gemv_rows.cuh"

#include <stdlib.h>
#include <string.h>

namespace vb200 {

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

// A [rows][n_groups] fp16 / fp32 scale (or zero-point) matrix as a TMA map of
// boxes [box_rows rows][n_groups]; rows past the end read as zero.
static int make_scale_map(CUtensorMap* map, const void* base, int rows, int n_groups, int elem_bytes, int box_rows) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) { set_error("cuTensorMapEncodeTiled unavailable"); return VSPEC_B200_ERR_CUDA; }
    cuuint64_t dims[2] = {(cuuint64_t)n_groups, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)n_groups * (cuuint64_t)elem_bytes};
    cuuint32_t box[2] = {(cuuint32_t)n_groups, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT32;
    CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) { set_error("cuTensorMapEncodeTiled (scales) failed (%d)", (int)r); return VSPEC_B200_ERR_CUDA; }
    return VSPEC_B200_OK;
}

// One CTA per SM per launch, each in at most half an SM
// (VSPEC_B200_GEMV_ROWS_PAIR: default on, "0" off): the CTAs of the next
// launch in the stream then fit beside this launch's and start streaming their
// weights as soon as programmatic dependent launch lets them in, instead of
// after this launch's CTAs exit.
static bool rows_pair_mode() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("VSPEC_B200_GEMV_ROWS_PAIR");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v == 1;
}

// Pair mode: how long a CTA's producer holds its first copies back while the
// previous kernel still runs.  A CTA of the next launch becomes resident while
// this launch's activation prologue reads x; its first copies then compete
// with those reads on the SM's memory path.  600 ns measured best where the
// prologue reads at least 16 KB of x (W4 K=4096 N=12288 8.81 -> 8.41 us, W3
// 9.48 -> 8.90, N=8192 7.27 -> 6.85); shorter launches (K=2048: 4.44 -> 4.54)
// keep no delay.  VSPEC_B200_ROWS_PREFETCH_DELAY_NS overrides it (0: off).
static int rows_prefetch_delay_ns(int m, int k) {
    static int v = -2;
    if (v == -2) {
        const char* e = getenv("VSPEC_B200_ROWS_PREFETCH_DELAY_NS");
        if (e && e[0]) {
            const int d = atoi(e);
            v = d < 0 ? 0 : (d > 20000 ? 20000 : d);
        } else {
            v = -1;
        }
    }
    if (v >= 0) return v;
    return (long long)m * k >= 4096 ? 600 : 0;
}

// Row-group size, ring depth and CTA count.  Candidate geometries, first fit
// wins: (pair mode) one CTA per SM in half an SM, row groups up to 96 rows;
// two CTAs per SM in half an SM each; one CTA per SM in a whole SM; the last
// two with row groups up to 64 rows.  The row group holds all of a CTA's rows.
// The ring holds every unit of the busiest CTA, or wraps with at least one
// stage per consumer warp and 24 KB in flight.
static bool rows_plan(const GemvParams& p, int bits, bool swiglu, RowsGeom* geo, size_t* smem) {
    const int m = p.m, kbt = p.k / 128;
    const int n_out = swiglu ? p.n / 2 : p.n;
    const int S = swiglu ? 2 : 1;
    const int szb = (p.flags & VSPEC_B200_F_SZ_F16) ? 2 : 4;
    const int srow = p.n_groups * szb;
    const bool has_s = p.s != nullptr, has_zp = p.zp != nullptr;
    struct Cand { int per_sm; uint32_t budget; int brmax; };
    Cand cands[3];
    int nc = 0;
    // (SwiGLU gate/up pairs measured slower in it: n = 24576, k = 4096 went 15.5 -> 17.4 us)
    if (rows_pair_mode() && !swiglu) cands[nc++] = Cand{1, kRowsSmemShared, 16 * kRowsMaxNB};
    cands[nc++] = Cand{2, kRowsSmemShared, 64};
    cands[nc++] = Cand{1, kRowsSmemMax, 64};
    for (int ci = 0; ci < nc; ++ci) {
        const Cand& cd = cands[ci];
        const int slots = device_sm_count() * cd.per_sm;
        const int min_rows = 8;
        int P = (n_out + min_rows - 1) / min_rows;
        if (P > slots) P = slots;
        if (P < 1) P = 1;
        const int rmax = (n_out + P - 1) / P;
        for (int ngrp = (rmax + cd.brmax - 1) / cd.brmax; ngrp <= 64; ++ngrp) {
            const int per = (rmax + ngrp - 1) / ngrp;
            const int br = 16 * ((per + 15) / 16);
            if (br > cd.brmax) continue;
            // a box (ring stage) covers the CTA's rows rounded up to 8 (the
            // swizzle period), not the whole 16-row-block group
            const int box = ((rmax + 7) / 8) * 8 < br ? ((rmax + 7) / 8) * 8 : br;
            const uint32_t stage = (uint32_t)box * (uint32_t)rows_unit_bytes(bits, br);
            const int kut = kbt / rows_kpu(bits, br);
            const uint32_t fixed = rows_smem_plan(bits, m, kbt, br, 0, srow, has_s, has_zp, swiglu, box).total + 1024u;
            if (fixed + 4u * (stage + 16u) > cd.budget) {
                if (br == 16) break;
                continue;
            }
            // one row group per CTA (a CTA's rows fit one box); shapes that
            // would need several groups per CTA take the split-K ring kernel
            if (rmax > br) break;
            int ns = (int)((cd.budget - fixed) / (stage + 16u));
            const int most = ((rmax + br - 1) / br) * S * kut;   // the busiest CTA's units
            if (ns > most) ns = most;
            if (ns > kRowsMaxStages) ns = kRowsMaxStages;
            // a ring that wraps keeps a stage per consumer warp and >= 24 KB in
            // flight per CTA (or everything); else smaller row groups (or the
            // next candidate)
            const uint64_t want = (uint64_t)most * stage < 24576u ? (uint64_t)most * stage : 24576u;
            if ((ns < most && ns < kRowsWarps) || (uint64_t)ns * stage < want) {
                if (br == 16) break;
                continue;
            }
            geo->ctas = P;
            geo->n_out = n_out;
            geo->br = br;
            geo->stages = ns;
            geo->srow_bytes = srow;
            geo->has_s = has_s ? 1 : 0;
            geo->has_zp = has_zp ? 1 : 0;
            geo->prefetch_delay_ns = (cd.per_sm == 1 && cd.budget == kRowsSmemShared) ? rows_prefetch_delay_ns(m, p.k) : 0;
            // the last stage's MMA blocks read (br - box) rows past the ring:
            // the buffers after it must cover them
            const RowsSmem pl = rows_smem_plan(bits, m, kbt, br, ns, srow, has_s, has_zp, swiglu, box);
            const uint32_t ring_end = (uint32_t)ns * stage;
            if (pl.total - ring_end < (uint32_t)(br - box) * (uint32_t)rows_unit_bytes(bits, br)) {
                if (br == 16) break;
                continue;
            }
            geo->box_rows = box;
            *smem = pl.total + 1024u;
            return true;
        }
    }
    return false;
}

bool gemv_rows_supported(const GemvParams& p, int bits) {
    if (p.m < 1 || p.m > kGemvMaxM) return false;
    if (p.k % (1024 * rows_kpu(bits, 16)) != 0 || p.n_groups < 1 || p.k % p.n_groups != 0 || (p.k / p.n_groups) % 128 != 0) return false;
    if (reinterpret_cast<uintptr_t>(p.w) % 16 != 0 || reinterpret_cast<uintptr_t>(p.x) % 16 != 0) return false;
    if ((size_t)p.row_bytes != row_bytes_for((size_t)p.k, bits)) return false;
    if ((size_t)p.row_bytes % 16 != 0) return false;   // TMA global stride
    if ((p.flags & VSPEC_B200_F_RMSNORM) && reinterpret_cast<uintptr_t>(p.norm_w) % 16 != 0) return false;
    const int szb = (p.flags & VSPEC_B200_F_SZ_F16) ? 2 : 4;
    // scale rows as TMA boxes: 16-byte multiples, at most 256 elements
    if (p.n_groups > 256 || (p.n_groups * szb) % 16 != 0) return false;
    if (p.s && reinterpret_cast<uintptr_t>(p.s) % 16 != 0) return false;
    if (p.zp && reinterpret_cast<uintptr_t>(p.zp) % 16 != 0) return false;
    const bool swiglu = (p.flags & VSPEC_B200_F_SWIGLU) != 0;
    if (swiglu && (p.n % 2 != 0)) return false;
    RowsGeom geo;
    size_t smem = 0;
    return rows_plan(p, bits, swiglu, &geo, &smem);
}

// Where the row-sliced kernel beats the split-K ring kernel (measured on B200,
// back-to-back launches in a CUDA graph over weights larger than L2, us per
// launch, ring -> rows with one CTA per SM per launch): one activation row,
// k <= 4096, e.g. int4 k = 4096 with n = 4096: 7.23 -> 5.44, n = 6144:
// 8.69 -> 5.89, n = 12288: 10.6 -> 9.18; int3 n = 12288: 12.2 -> 9.93; int2
// n = 12288: 9.71 -> 7.50.  Deeper rows (k = 12288: 12.3 -> 14.4) and several
// activation rows (m = 4: 11.6 -> 15.0) stay on the ring kernel, as do shapes
// with more than one row group per CTA.
bool gemv_rows_preferred(const GemvParams& p, int bits) {
    if (p.k > 4096 || p.m < 1) return false;
    if (p.m > 1) {
        // 2-4 activation rows, int4, no SwiGLU: faster than the ring kernel while m * n <= 24576
        // for m <= 3 and m * n <= 16384 for m = 4 (measured, k = 4096, rows / ring us: n = 4096 at
        // m = 2 / 3 / 4: 6.71 / - / 9.96 against 8.56 / 10.18 / 11.66; n = 6144 at m = 3: 9.28
        // against 9.88; n = 12288 at m = 2: 10.08 against 10.67; the ring kernel wins at m = 4 for
        // n = 6144 (10.98 against 11.19) and n = 12288 (11.44 against 13.77))
        if (p.m > 4 || bits != 4 || (p.flags & VSPEC_B200_F_SWIGLU)) return false;
        if ((long long)p.m * p.n > (p.m <= 3 ? 24576 : 16384)) return false;
        return gemv_rows_supported(p, bits);
    }
    if (bits == 2 && !rows_pair_mode()) return false;   // int2 gains only with one CTA per SM
    return gemv_rows_supported(p, bits);
}

int gemv_rows_read_and_clear_timeout(int* out) {
    int a = 0, b = 0, c = 0;
    int rc = rows_timeout_bits<2>(&a);
    if (rc != VSPEC_B200_OK) return rc;
    rc = rows_timeout_bits<3>(&b);
    if (rc != VSPEC_B200_OK) return rc;
    rc = rows_timeout_bits<4>(&c);
    if (rc != VSPEC_B200_OK) return rc;
    *out = (a || b || c) ? 1 : 0;
    return VSPEC_B200_OK;
}

// p must carry kb_total / kb_per_group(_shift).  Uses no workspace.
int gemv_rows_launch(GemvParams p, int bits, int unsigned_codes, cudaStream_t st, bool pdl) {
    const bool swiglu = (p.flags & VSPEC_B200_F_SWIGLU) != 0;
    RowsGeom geo;
    size_t smem = 0;
    if (!rows_plan(p, bits, swiglu, &geo, &smem)) {
        set_error("shape too large for the row-sliced GEMV");
        return VSPEC_B200_ERR_UNSUPPORTED;
    }
    CUtensorMap wmap, smap, zmap;
    memset(&smap, 0, sizeof(smap));
    memset(&zmap, 0, sizeof(zmap));
    // the swizzle the kernel's shared-memory reads assume: 128 B for two-k-block
    // int4 boxes, 64 B for one-k-block int4 boxes, 32 B for int2, none for int3
    const CUtensorMapSwizzle swz = bits == 4 ? (rows_kpu(bits, geo.br) == 2 ? CU_TENSOR_MAP_SWIZZLE_128B
                                                                              : CU_TENSOR_MAP_SWIZZLE_64B)
                                 : (bits == 2 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_NONE);
    int rc = make_row_tile_map(&wmap, p.w, p.n, p.row_bytes, rows_unit_bytes(bits, geo.br), geo.box_rows, swz);
    if (rc != VSPEC_B200_OK) return rc;
    const int szb = (p.flags & VSPEC_B200_F_SZ_F16) ? 2 : 4;
    if (p.s) {
        rc = make_scale_map(&smap, p.s, p.n, p.n_groups, szb, geo.br);
        if (rc != VSPEC_B200_OK) return rc;
    }
    if (p.zp) {
        rc = make_scale_map(&zmap, p.zp, p.n, p.n_groups, szb, geo.br);
        if (rc != VSPEC_B200_OK) return rc;
    }
    p.stages = geo.stages;
    const bool uns = unsigned_codes != 0;
    cudaError_t e;
    if (bits == 4) e = rows_launch_bits<4>(wmap, smap, zmap, p, geo, smem, uns, swiglu, st, pdl);
    else if (bits == 3) e = rows_launch_bits<3>(wmap, smap, zmap, p, geo, smem, uns, swiglu, st, pdl);
    else e = rows_launch_bits<2>(wmap, smap, zmap, p, geo, smem, uns, swiglu, st, pdl);
    if (e != cudaSuccess) return cuda_status(e, "lowbit_gemv_rows_kernel launch");
    return VSPEC_B200_OK;
}

}  // namespace vb200
