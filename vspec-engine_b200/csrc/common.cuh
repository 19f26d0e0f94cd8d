// common.cuh -- shared device/host helpers for the sm_100a kernels of libvspec_b200.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stddef.h>

#include "vspec_b200.h"

namespace vb200 {

// ---------------------------------------------------------------------------
// Error reporting: every extern "C" entry point of the library returns a
// VSPEC_B200_* status and leaves a message retrievable with
// vspec_b200_last_error() (thread-local, like the reference bridge's state).
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);
int cuda_status(cudaError_t e, const char* what);

#define VB_CHECK_CUDA(expr)                                                   \
    do {                                                                      \
        cudaError_t _e = (expr);                                              \
        if (_e != cudaSuccess) return ::vb200::cuda_status(_e, #expr);        \
    } while (0)

// ---------------------------------------------------------------------------
// fp16 bit patterns of exactly representable constants (compile time).
// ---------------------------------------------------------------------------
__host__ __device__ constexpr uint16_t f16_bits(double v) {
    // Exact encoder for normal binary16 values that have <= 11 significant bits.
    uint16_t sign = v < 0 ? 0x8000 : 0;
    double a = v < 0 ? -v : v;
    if (a == 0.0) return sign;
    int e = 0;
    while (a >= 2.0) { a /= 2.0; ++e; }
    while (a < 1.0) { a *= 2.0; --e; }
    uint16_t frac = (uint16_t)((a - 1.0) * 1024.0);
    return (uint16_t)(sign | (uint16_t)((e + 15) << 10) | frac);
}
__host__ __device__ constexpr uint32_t f16x2_bits(double lo, double hi) {
    return (uint32_t)f16_bits(lo) | ((uint32_t)f16_bits(hi) << 16);
}
static_assert(f16_bits(1024.0) == 0x6400, "f16 encoder");
static_assert(f16_bits(-1032.0) == 0xE408, "f16 encoder");
static_assert(f16_bits(-72.0) == 0xD480, "f16 encoder");
static_assert(f16_bits(0.0625) == 0x2C00, "f16 encoder");

// ---------------------------------------------------------------------------
// Inline PTX helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t magic) {
    uint32_t r;
    // (a & mask) | magic
    asm volatile("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(r) : "r"(a), "r"(mask), "r"(magic));
    return r;
}

__device__ __forceinline__ uint32_t hfma2_bits(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm volatile("fma.rn.f16x2 %0, %1, %2, %3;\n" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

__device__ __forceinline__ uint32_t hsub2_bits(uint32_t a, uint32_t b) {
    uint32_t r;
    asm volatile("sub.rn.f16x2 %0, %1, %2;\n" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

__device__ __forceinline__ uint32_t funnel_r(uint32_t lo, uint32_t hi, uint32_t sh) {
    uint32_t r;
    asm volatile("shf.r.clamp.b32 %0, %1, %2, %3;\n" : "=r"(r) : "r"(lo), "r"(hi), "r"(sh));
    return r;
}

// Streaming 128-bit load of packed weights: read-only path, no L1 allocation.
__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
__device__ __forceinline__ uint2 ldg_stream_v2(const void* p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];\n"
                 : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}
__device__ __forceinline__ uint32_t ldg_stream_u32(const void* p) {
    uint32_t r;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];\n" : "=r"(r) : "l"(p));
    return r;
}

// D = A(16x16 f16, row) * B(16x8 f16, col) + C, fp32 accumulate (warp-level MMA).
__device__ __forceinline__ void mma_16816_f16(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1,
                                              const float c[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1),
          "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}
// D += A * B with D in place.
__device__ __forceinline__ void mma_16816_f16_acc(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// D (+)= A * B, 16x8x32, A unsigned 8-bit (row major), B signed 8-bit
// (column major), exact int32 accumulation.
__device__ __forceinline__ void imma_16832_u8s8(int d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Signed b-bit code t of an LSB-first packed row (the reference bitstream,
// src/quant/pack.c:53-74).  Used by the generic (any-shape) kernels.
__device__ __forceinline__ int decode_code_generic(const uint8_t* row, size_t t, int bits, int unsigned_codes) {
    const size_t bit = t * (size_t)bits;
    const size_t byte = bit >> 3;
    const unsigned shift = (unsigned)(bit & 7u);
    unsigned v = (unsigned)row[byte] >> shift;
    if (8u - shift < (unsigned)bits) v |= (unsigned)row[byte + 1] << (8u - shift);
    v &= (1u << bits) - 1u;
    if (unsigned_codes) return (int)v - (1 << (bits - 1));
    return (v & (1u << (bits - 1))) ? (int)v - (1 << bits) : (int)v;
}

__host__ __device__ __forceinline__ size_t row_bytes_for(size_t k, int bits) {
    return (k * (size_t)bits + 7u) / 8u;
}

// Group of reduction index t (src/kernel/cuda/fused_linear_int4.cu:391-392).
__host__ __device__ __forceinline__ size_t group_of(size_t t, size_t k, size_t n_groups) {
    if (n_groups <= 1) return 0;
    size_t g = (t * n_groups) / k;
    return g < n_groups ? g : n_groups - 1;
}

int device_sm_count();

// Programmatic dependent launch (VSPEC_B200_PDL=0 turns it off).  A kernel
// launched with launch_pdl() may start while its predecessor in the stream is
// still running, so it must call pdl_wait() before it reads or writes any
// global memory the predecessors touch; pdl_trigger() lets the next launch
// in the stream start early in turn.
bool pdl_allowed();
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_allowed() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

}  // namespace vb200
