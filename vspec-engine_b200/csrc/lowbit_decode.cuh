// lowbit_decode.cuh -- register decoder for packed int2/int3/int4 codes
// (the reference's LSB-first bitstream, src/quant/pack.c:30-74), shared by the
// warp-MMA and the tcgen05 GEMV kernels.
#pragma once

#include "common.cuh"

namespace vb200 {

// -------------------------------------------------------------------------
// Code-order tables: fp16 pair q (0..15) of a decoded 32-code chunk holds
// codes (lo_code(q), hi_code(q)).
// -------------------------------------------------------------------------
template <int BITS>
__host__ __device__ constexpr int lo_code(int q) {
    if (BITS == 4) return 8 * (q >> 2) + (q & 3);
    if (BITS == 2) return 16 * (q >> 3) + (q & 7);
    // BITS == 3: window w = q/2 starts at code j(w) in {0,2,8,10,16,18,24,26}
    const int w = q >> 1;
    const int j = 8 * (w >> 1) + 2 * (w & 1);
    return j + (q & 1);
}
template <int BITS>
__host__ __device__ constexpr int hi_code(int q) {
    if (BITS == 4) return lo_code<4>(q) + 4;
    if (BITS == 2) return lo_code<2>(q) + 8;
    return lo_code<3>(q) + 4;
}

template <int BITS> struct Chunk { uint32_t w[BITS]; };  // 32 codes = 4*BITS bytes

template <int BITS>
__device__ __forceinline__ void load_chunk(Chunk<BITS>& c, const uint8_t* p) {
    if constexpr (BITS == 4) {
        uint4 v = ldg_stream_v4(p);
        c.w[0] = v.x; c.w[1] = v.y; c.w[2] = v.z; c.w[3] = v.w;
    } else if constexpr (BITS == 2) {
        uint2 v = ldg_stream_v2(p);
        c.w[0] = v.x; c.w[1] = v.y;
    } else {
        c.w[0] = ldg_stream_u32(p);
        c.w[1] = ldg_stream_u32(p + 4);
        c.w[2] = ldg_stream_u32(p + 8);
    }
}

constexpr uint32_t kMagic = 0x64006400u;  // fp16 1024.0 in both halves

// Decoded fp16 pairs carry 1024 + mult * u, where u is the offset-encoded code
// (u = code + 2^(bits-1), exact in fp16) and mult a power of two that depends
// only on the code's position j inside its 32-code chunk.  The GEMV divides
// the matching activation by mult and removes sum(x * (1024/mult + 2^(bits-1)))
// per k-block, so no fp16 arithmetic is spent on decoding.
template <int BITS>
__host__ __device__ constexpr float code_mult(int j) {
    if (BITS == 4) return (j & 1) ? 16.0f : 1.0f;
    if (BITS == 2) return (float)(1 << (2 * (j & 3)));
    const int t = j & 7;   // BITS == 3
    return t < 4 ? ((t & 1) ? 128.0f : 16.0f) : ((t & 1) ? 8.0f : 1.0f);
}

// Exact reciprocal of code_mult (powers of two), without a division.
template <int BITS>
__host__ __device__ __forceinline__ float code_inv_mult(int j) {
    if (BITS == 4) return (j & 1) ? 0.0625f : 1.0f;
    if (BITS == 2) {
        const int e = j & 3;
        return e == 0 ? 1.0f : (e == 1 ? 0.25f : (e == 2 ? 0.0625f : 0.015625f));
    }
    const int t = j & 7;   // BITS == 3
    return t < 4 ? ((t & 1) ? 0.0078125f : 0.0625f) : ((t & 1) ? 0.125f : 1.0f);
}

// Inverse of (lo_code, hi_code): fp16 pair q (0..15) and half (0: low fp16,
// 1: high fp16) that carry code j (0..31) of a 32-code chunk.
template <int BITS>
__host__ __device__ __forceinline__ void code_slot(int j, int& q, int& half) {
    if (BITS == 4) {
        half = (j >> 2) & 1;
        q = 4 * (j >> 3) + (j & 3);
    } else if (BITS == 2) {
        half = (j >> 3) & 1;
        q = 8 * (j >> 4) + (j & 7);
    } else {
        half = (j >> 2) & 1;
        const int b = j - 4 * half;
        q = 2 * (2 * (b >> 3) + ((b >> 1) & 1)) + (b & 1);
    }
}

// Pairs 2*mm and 2*mm+1 of a chunk (the A registers of MMA number mm) as raw
// magic halves.  Two's-complement codes become offset codes by flipping every
// field's top bit.  mm is a constant after loop unrolling.
template <int BITS, bool UNSIGNED>
__device__ __forceinline__ void unpack_mm(const Chunk<BITS>& c, const int mm, uint32_t& h0, uint32_t& h1) {
    if constexpr (BITS == 4) {
        uint32_t q = UNSIGNED ? c.w[mm >> 1] : (c.w[mm >> 1] ^ 0x88888888u);
        if (mm & 1) q >>= 8;
        h0 = lop3_and_or(q, 0x000F000Fu, kMagic);    // nibbles 2(mm&1) and +4: mult 1
        h1 = lop3_and_or(q, 0x00F000F0u, kMagic);    // nibbles 2(mm&1)+1 and +5: mult 16
    } else if constexpr (BITS == 2) {
        uint32_t q = UNSIGNED ? c.w[mm >> 2] : (c.w[mm >> 2] ^ 0xAAAAAAAAu);
        const int p0 = 2 * (mm & 3);  // pair index inside the word: 0, 2, 4, 6
        if (p0 >= 4) q >>= 8;
        const int j = p0 & 3;         // 0 or 2: field positions j and j+1
        h0 = lop3_and_or(q, 0x00030003u << (2 * j), kMagic);
        h1 = lop3_and_or(q, 0x00030003u << (2 * j + 2), kMagic);
    } else {
        // 32 three-bit codes in 96 bits, code j at bits [3j, 3j+3).  Window
        // R = bits [3J-4, 3J+28) puts codes J, J+1 at bits 4, 7 and codes
        // J+4, J+5 at bits 16, 19, for J = 0,2,8,10,16,18,24,26.
        uint32_t w0 = c.w[0], w1 = c.w[1], w2 = c.w[2];
        if (!UNSIGNED) {
            w0 ^= 0x24924924u;
            w1 ^= 0x49249249u;
            w2 ^= 0x92492492u;
        }
        uint32_t R;
        switch (mm) {
            case 0: R = w0 << 4; break;
            case 1: R = w0 >> 2; break;
            case 2: R = funnel_r(w0, w1, 20); break;
            case 3: R = funnel_r(w0, w1, 26); break;
            case 4: R = funnel_r(w1, w2, 12); break;
            case 5: R = funnel_r(w1, w2, 18); break;
            case 6: R = w2 >> 4; break;
            default: R = w2 >> 10; break;
        }
        h0 = lop3_and_or(R, 0x00070070u, kMagic);    // codes J (mult 16), J+4 (mult 1)
        h1 = lop3_and_or(R, 0x00380380u, kMagic);    // codes J+1 (mult 128), J+5 (mult 8)
    }
}

// -------------------------------------------------------------------------
// Integer-MMA decode (mma.sync m16n8k32, A unsigned 8-bit, B signed 8-bit).
// A 32-code chunk of one row feeds four k32 MMAs; MMA q takes two registers
// of four byte lanes each (register r = 0 goes to a0/a1, r = 1 to a2/a3).  A
// byte carries an offset code v in [0, 2^bits) times a power of two 2^shift
// that depends only on the MMA's class, so a register is one mask of the
// packed word (one LOP3, no shifts for int4 and int2).  MMAs of one class
// accumulate into their own int32 registers, which are shifted back exactly.
// -------------------------------------------------------------------------
template <int BITS> struct I8Cfg;
// int4: byte i of word j holds codes 8j+2i (low nibble, class 0) and 8j+2i+1
// (high nibble x16, class 1); MMA q = 2*class + pair, pair p -> words 2p, 2p+1.
template <> struct I8Cfg<4> { static constexpr int kClasses = 2; };
// int2: byte i of word j holds codes 16j+4i+s at bits 2s (class s, x4^s);
// MMA q = s, register r = word j.
template <> struct I8Cfg<2> { static constexpr int kClasses = 4; };
// int3: each 24-bit group k (codes 8k..8k+7) is spread so byte i holds code
// 8k+2i at bits 0-2 (class 0) and 8k+2i+1 at bits 3-5 (class 1, x8); MMA
// q = 2*class + pair, pair p -> groups 2p, 2p+1.
template <> struct I8Cfg<3> { static constexpr int kClasses = 2; };

template <int BITS>
__host__ __device__ constexpr int i8_class(int q) { return BITS == 2 ? q : (q >> 1); }
template <int BITS>
__host__ __device__ constexpr int i8_class_shift(int cls) { return BITS == 4 ? 4 * cls : (BITS == 3 ? 3 * cls : 2 * cls); }

// Code t (0..31) of a chunk -> MMA q, register r, byte i.
template <int BITS>
__host__ __device__ inline void i8_code_place(int t, int& q, int& r, int& i) {
    if (BITS == 2) {
        q = t & 3;
        r = t >> 4;
        i = (t & 15) >> 2;
    } else {
        const int j = t >> 3;
        i = (t & 7) >> 1;
        q = 2 * (t & 1) + (j >> 1);
        r = j & 1;
    }
}

// A chunk prepared for masking: offset codes (two's-complement fields with
// their top bit flipped, or the raw fields in the unsigned reading), and for
// int3 the four spread 24-bit groups.
template <int BITS> struct I8Words { uint32_t v[BITS == 2 ? 2 : 4]; };

template <int BITS, bool UNSIGNED>
__device__ __forceinline__ void i8_prepare(const Chunk<BITS>& c, I8Words<BITS>& o) {
    if constexpr (BITS == 4) {
#pragma unroll
        for (int j = 0; j < 4; ++j) o.v[j] = UNSIGNED ? c.w[j] : (c.w[j] ^ 0x88888888u);
    } else if constexpr (BITS == 2) {
#pragma unroll
        for (int j = 0; j < 2; ++j) o.v[j] = UNSIGNED ? c.w[j] : (c.w[j] ^ 0xAAAAAAAAu);
    } else {
        uint32_t w0 = c.w[0], w1 = c.w[1], w2 = c.w[2];
        if (!UNSIGNED) {
            w0 ^= 0x24924924u;
            w1 ^= 0x49249249u;
            w2 ^= 0x92492492u;
        }
        const uint32_t g[4] = {w0, funnel_r(w0, w1, 24), funnel_r(w1, w2, 16), w2 >> 8};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            // codes 4..7 of the group move up 4 bits (to 16..27), then codes
            // 2, 3 and 6, 7 up 2 more: code 2i at byte i bits 0-2, 2i+1 at 3-5
            const uint32_t a = (g[k] & 0x0000FFFFu) | ((g[k] << 4) & 0xFFFF0000u);
            o.v[k] = (a & 0x00FF00FFu) | ((a << 2) & 0xFF00FF00u);
        }
    }
}

// Register r of MMA q.
template <int BITS>
__device__ __forceinline__ uint32_t i8_reg(const I8Words<BITS>& o, int q, int r) {
    if constexpr (BITS == 4) return o.v[2 * (q & 1) + r] & ((q >> 1) ? 0xF0F0F0F0u : 0x0F0F0F0Fu);
    else if constexpr (BITS == 2) return o.v[r] & (0x03030303u << (2 * q));
    else return o.v[2 * (q & 1) + r] & ((q >> 1) ? 0x38383838u : 0x07070707u);
}

// Scale / zero-point element as raw bits (fp16 or fp32 storage), read through
// the read-only path.  Converting only where the value is used keeps the load
// latency off the critical path.
__device__ __forceinline__ uint32_t load_sz_raw(const void* base, size_t idx, bool f16) {
    if (!base) return 0u;
    if (f16) return (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(base) + idx);
    return __ldg(reinterpret_cast<const unsigned int*>(base) + idx);
}
__device__ __forceinline__ float sz_to_float(uint32_t raw, bool f16) {
    return f16 ? __half2float(__ushort_as_half((unsigned short)raw)) : __uint_as_float(raw);
}

}  // namespace vb200
