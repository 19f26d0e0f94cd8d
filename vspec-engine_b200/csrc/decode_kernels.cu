// decode_kernels.cu -- the small per-token kernels of a Qwen3-shape decode step
// (everything between the low-bit linears and the paged attention):
//   * token embedding lookup;
//   * per-head q/k RMSNorm + half-split rotary embedding + append of k and v
//     (fp16) into the paged KV pools, and the context length update
//     (Vspec-chat/python/runtime_inference.py:1297-1311: q/k RMSNorm, then
//      q1*cos - q2*sin, q1*sin + q2*cos on the two halves, inv_freq =
//      theta^(-i/(d/2)), runtime_inference.py:4227);
//   * greedy next token: logits cleaned like _stabilize_logits
//     (runtime_inference.py:554-567: NaN -> 0, +-inf -> +-clip, clip to
//     +-clip; the entropy/margin steps never change the argmax), argmax with
//     the lowest index on ties, or the next prompt token while the prompt lasts;
//   * seeded random initialisation of packed weights, scales and fp16
//     tensors (random-init model of the benchmark; no checkpoint exists).
// Positions live in device memory so a captured decode step replays as is.
#include "common.cuh"

#include <stdint.h>

#include "vspec_b200.h"

namespace vb200 {

__global__ void embed_kernel(const __half* __restrict__ table, const int32_t* __restrict__ tok, int hidden,
                             float* __restrict__ x) {
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.y;
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t < hidden) x[(size_t)b * hidden + t] = __half2float(table[(size_t)tok[b] * hidden + t]);
}

// One warp per (head, sequence), eight heads per block: heads [0, hq) are
// query heads, [hq, hq+hkv) key heads, [hq+hkv, hq+2hkv) value heads.  Lane l
// holds elements l + 32k (k < E = head_dim / 32), so both elements of every
// rotary pair (i, i + head_dim/2) sit in the same lane.
template <int E>
__global__ void __launch_bounds__(256)
qk_norm_rope_append_kernel(const float* __restrict__ qkv, const float* __restrict__ q_norm,
                           const float* __restrict__ k_norm, const int32_t* __restrict__ pos, int hq, int hkv,
                           float eps, float theta, float* __restrict__ q_out, __half* __restrict__ k_pages,
                           __half* __restrict__ v_pages, const int32_t* __restrict__ page_table, int max_pages,
                           int page_tokens, int32_t* __restrict__ ctx_len) {
    pdl_wait();
    pdl_trigger();
    constexpr int d = 32 * E;
    constexpr int HE = E / 2;   // elements per lane in each half
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nh = hq + 2 * hkv;
    const int h = blockIdx.x * 8 + warp;
    const int b = blockIdx.y;
    if (h >= nh) return;
    const float* src = qkv + (size_t)b * nh * d + (size_t)h * d;
    float v[E];
#pragma unroll
    for (int k = 0; k < E; ++k) v[k] = src[lane + 32 * k];
    const int p = pos[b];
    const int page = page_table[(size_t)b * max_pages + p / page_tokens];
    const int slot = p % page_tokens;
    if (h >= hq + hkv) {
        // value head: straight into the page
        __half* dst = v_pages + (((size_t)page * page_tokens + slot) * hkv + (h - hq - hkv)) * d;
#pragma unroll
        for (int k = 0; k < E; ++k) dst[lane + 32 * k] = __float2half_rn(v[k]);
        return;
    }
    // RMSNorm over the head
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < E; ++k) ss += v[k] * v[k];
    ss = warp_sum(ss);
    const bool is_q = h < hq;
    const float* nw = is_q ? q_norm : k_norm;
    const float inv = 1.0f / sqrtf(ss / (float)d + eps);
    float y[E];
#pragma unroll
    for (int k = 0; k < E; ++k) y[k] = v[k] * inv * nw[lane + 32 * k];
    // rotary, half split: element i < d/2 pairs with i + d/2
    float r[E];
#pragma unroll
    for (int k = 0; k < HE; ++k) {
        const int i = lane + 32 * k;
        // The reference's float32 arithmetic (runtime_inference.py:4227,1187-1191):
        // inv_freq = fl32(1 / fl32(theta ** fl32(i / half))), angle = fl32(pos *
        // inv_freq), cos / sin of that float angle as float32.  The power and the
        // sin / cos are evaluated in double and rounded once, which gives the
        // correctly rounded float32 values numpy's float32 path aims at.
        const float e = (float)i / (float)(d / 2);
        const float pw = (float)pow((double)theta, (double)e);
        const float inv_freq = 1.0f / pw;
        const float ang = (float)p * inv_freq;
        double snd, csd;
        sincos((double)ang, &snd, &csd);
        const float sn = (float)snd, cs = (float)csd;
        r[k] = y[k] * cs - y[k + HE] * sn;
        r[k + HE] = y[k] * sn + y[k + HE] * cs;
    }
    if (is_q) {
        float* dst = q_out + ((size_t)b * hq + h) * d;
#pragma unroll
        for (int k = 0; k < E; ++k) dst[lane + 32 * k] = r[k];
    } else {
        const int kvh = h - hq;
        __half* dst = k_pages + (((size_t)page * page_tokens + slot) * hkv + kvh) * d;
#pragma unroll
        for (int k = 0; k < E; ++k) dst[lane + 32 * k] = __float2half_rn(r[k]);
        if (kvh == 0 && lane == 0) ctx_len[b] = p + 1;
    }
}

// Next token (prompt or greedy argmax), position + 1.  Grid (blocks, batch):
// every block folds its share of the vocabulary into one 64-bit key per
// sequence -- cleaned value in the high word (order-preserving bits), lowest
// index winning ties in the low word -- with atomicMax; the last block of a
// sequence to finish reads and resets the key and its counter and moves the
// sequence on.  state: [batch] keys then [batch] counters, zero between calls.
__device__ __forceinline__ uint32_t ordered_bits(float v) {
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void __launch_bounds__(256) next_token_kernel(const float* __restrict__ logits, int vocab, float clip,
                                                         const int32_t* __restrict__ prompt, const int32_t* __restrict__ prompt_len,
                                                         int max_prompt, int32_t* __restrict__ pos, int32_t* __restrict__ tok,
                                                         int32_t* __restrict__ out_tokens, int max_steps,
                                                         unsigned long long* __restrict__ keys, unsigned int* __restrict__ counts) {
    __shared__ unsigned long long red[8];
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.y;
    const float* lg = logits + (size_t)b * vocab;
    const int chunk = (vocab + gridDim.x - 1) / gridDim.x;
    const int j0 = blockIdx.x * chunk;
    const int j1 = min(vocab, j0 + chunk);
    unsigned long long best = 0ull;
    for (int j = j0 + threadIdx.x; j < j1; j += blockDim.x) {
        float v = lg[j];
        if (isnan(v)) v = 0.f;
        v = fminf(fmaxf(v, -clip), clip) + 0.0f;   // -0 -> +0: equal values tie on the index
        const unsigned long long key = ((unsigned long long)ordered_bits(v) << 32) | (0xFFFFFFFFu - (uint32_t)j);
        best = key > best ? key : best;
    }
    for (int off = 16; off > 0; off >>= 1) {
        const unsigned long long o = __shfl_xor_sync(0xffffffffu, best, off);
        best = o > best ? o : best;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = red[w] > best ? red[w] : best;
        atomicMax(&keys[b], best);
        __threadfence();
        if (atomicAdd(&counts[b], 1u) == gridDim.x - 1) {
            __threadfence();
            const unsigned long long key = atomicExch(&keys[b], 0ull);
            counts[b] = 0u;
            const int arg = (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
            const int p = pos[b];
            const int nxt = (p + 1 < prompt_len[b]) ? prompt[(size_t)b * max_prompt + p + 1] : arg;
            tok[b] = nxt;
            if (p + 1 < max_steps) out_tokens[(size_t)b * max_steps + p + 1] = nxt;
            pos[b] = p + 1;
        }
    }
}

// splitmix64 of (seed, index): the random-init stream of every tensor.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void rand_bytes_kernel(uint8_t* __restrict__ out, size_t n, uint64_t seed) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = (uint8_t)(mix64(seed ^ mix64(i)) >> 32);
}

// uniform in [lo, hi)
__global__ void rand_half_kernel(__half* __restrict__ out, size_t n, uint64_t seed, float lo, float hi) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float u = (float)(mix64(seed ^ mix64(i)) >> 40) * (1.0f / 16777216.0f);
        out[i] = __float2half_rn(lo + (hi - lo) * u);
    }
}

// Rows x cols block of a larger tensor: element (j, t) of the block is element
// (row0 + j, col0 + t) of a [*][global_cols] tensor, whose random stream it
// takes, so a shard of a tensor holds exactly the values of the whole.
__global__ void rand_block_kernel(void* __restrict__ out, int kind, size_t rows, size_t cols, size_t dst_stride,
                                  uint64_t seed, size_t global_cols, size_t row0, size_t col0, float lo, float hi) {
    const size_t n = rows * cols;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t j = i / cols, t = i - j * cols;
        const uint64_t h = mix64(seed ^ mix64((row0 + j) * global_cols + col0 + t));
        if (kind == 0) {
            reinterpret_cast<uint8_t*>(out)[j * dst_stride + t] = (uint8_t)(h >> 32);
        } else {
            const float u = (float)(h >> 40) * (1.0f / 16777216.0f);
            reinterpret_cast<__half*>(out)[j * dst_stride + t] = __float2half_rn(lo + (hi - lo) * u);
        }
    }
}

__global__ void fill_f32_kernel(float* __restrict__ out, size_t n, float v) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = v;
}

static int grid_for(size_t n) {
    size_t g = (n + 255) / 256;
    return (int)(g < 65535 ? (g > 0 ? g : 1) : 65535);
}

}  // namespace vb200

using namespace vb200;

extern "C" int vspec_b200_decode_embed(const void* d_table_f16, const int32_t* d_tok, int batch, int hidden,
                                       float* d_x, void* stream) {
    if (!d_table_f16 || !d_tok || !d_x || batch <= 0 || hidden <= 0) { set_error("bad embed arguments"); return VSPEC_B200_ERR_ARG; }
    const cudaError_t e = launch_pdl(embed_kernel, dim3((hidden + 255) / 256, batch), dim3(256), 0,
                                     (cudaStream_t)stream, reinterpret_cast<const __half*>(d_table_f16), d_tok, hidden,
                                     d_x);
    return e == cudaSuccess ? VSPEC_B200_OK : cuda_status(e, "embed_kernel launch");
}

extern "C" int vspec_b200_decode_qk_rope_append(const float* d_qkv, const float* d_q_norm, const float* d_k_norm,
                                                const int32_t* d_pos, int batch, int hq, int hkv, int head_dim,
                                                float eps, float theta, float* d_q_out, void* d_k_pages,
                                                void* d_v_pages, const int32_t* d_page_table, int max_pages,
                                                int page_tokens, int32_t* d_ctx_len, void* stream) {
    if (!d_qkv || !d_q_norm || !d_k_norm || !d_pos || !d_q_out || !d_k_pages || !d_v_pages || !d_page_table ||
        !d_ctx_len || batch <= 0 || hq <= 0 || hkv <= 0 || hq % hkv != 0 || head_dim <= 0 || head_dim > 256 ||
        head_dim % 64 != 0 || page_tokens <= 0 || max_pages <= 0) {
        set_error("bad qk/rope/append arguments");
        return VSPEC_B200_ERR_ARG;
    }
    const dim3 grid((hq + 2 * hkv + 7) / 8, batch);
    __half* kpg = reinterpret_cast<__half*>(d_k_pages);
    __half* vpg = reinterpret_cast<__half*>(d_v_pages);
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e;
    switch (head_dim / 32) {
        case 2: e = launch_pdl(qk_norm_rope_append_kernel<2>, grid, dim3(256), 0, st, d_qkv, d_q_norm, d_k_norm, d_pos,
                               hq, hkv, eps, theta, d_q_out, kpg, vpg, d_page_table, max_pages, page_tokens, d_ctx_len);
                break;
        case 4: e = launch_pdl(qk_norm_rope_append_kernel<4>, grid, dim3(256), 0, st, d_qkv, d_q_norm, d_k_norm, d_pos,
                               hq, hkv, eps, theta, d_q_out, kpg, vpg, d_page_table, max_pages, page_tokens, d_ctx_len);
                break;
        case 6: e = launch_pdl(qk_norm_rope_append_kernel<6>, grid, dim3(256), 0, st, d_qkv, d_q_norm, d_k_norm, d_pos,
                               hq, hkv, eps, theta, d_q_out, kpg, vpg, d_page_table, max_pages, page_tokens, d_ctx_len);
                break;
        default: e = launch_pdl(qk_norm_rope_append_kernel<8>, grid, dim3(256), 0, st, d_qkv, d_q_norm, d_k_norm, d_pos,
                                hq, hkv, eps, theta, d_q_out, kpg, vpg, d_page_table, max_pages, page_tokens, d_ctx_len);
                 break;
    }
    return e == cudaSuccess ? VSPEC_B200_OK : cuda_status(e, "qk_norm_rope_append_kernel launch");
}

extern "C" int vspec_b200_decode_next_token(const float* d_logits, int batch, int vocab, float clip,
                                            const int32_t* d_prompt, const int32_t* d_prompt_len, int max_prompt,
                                            int32_t* d_pos, int32_t* d_tok, int32_t* d_out_tokens, int max_steps,
                                            void* d_state, void* stream) {
    if (!d_logits || !d_prompt || !d_prompt_len || !d_pos || !d_tok || !d_out_tokens || !d_state || batch <= 0 ||
        vocab <= 0) {
        set_error("bad next-token arguments");
        return VSPEC_B200_ERR_ARG;
    }
    if (reinterpret_cast<uintptr_t>(d_state) % 8 != 0) { set_error("next-token state must be 8-byte aligned"); return VSPEC_B200_ERR_ARG; }
    unsigned long long* keys = reinterpret_cast<unsigned long long*>(d_state);
    unsigned int* counts = reinterpret_cast<unsigned int*>(keys + batch);
    int blocks = (vocab + 2047) / 2048;   // ~8 values per thread
    blocks = blocks < 1 ? 1 : (blocks > 256 ? 256 : blocks);
    const cudaError_t e = launch_pdl(next_token_kernel, dim3(blocks, batch), dim3(256), 0, (cudaStream_t)stream,
                                     d_logits, vocab, clip, d_prompt, d_prompt_len, max_prompt, d_pos, d_tok,
                                     d_out_tokens, max_steps, keys, counts);
    return e == cudaSuccess ? VSPEC_B200_OK : cuda_status(e, "next_token_kernel launch");
}

extern "C" int vspec_b200_random_fill(void* d_dst, size_t count, int kind, uint64_t seed, float lo, float hi,
                                      void* stream) {
    if (!d_dst || count == 0) { set_error("bad random_fill arguments"); return VSPEC_B200_ERR_ARG; }
    cudaStream_t st = (cudaStream_t)stream;
    if (kind == 0) rand_bytes_kernel<<<grid_for(count), 256, 0, st>>>(reinterpret_cast<uint8_t*>(d_dst), count, seed);
    else if (kind == 1) rand_half_kernel<<<grid_for(count), 256, 0, st>>>(reinterpret_cast<__half*>(d_dst), count, seed, lo, hi);
    else if (kind == 2) fill_f32_kernel<<<grid_for(count), 256, 0, st>>>(reinterpret_cast<float*>(d_dst), count, lo);
    else { set_error("unknown random_fill kind %d", kind); return VSPEC_B200_ERR_ARG; }
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? VSPEC_B200_OK : cuda_status(e, "random_fill launch");
}

extern "C" int vspec_b200_random_fill_block(void* d_dst, size_t rows, size_t cols, size_t dst_stride, int kind,
                                            uint64_t seed, size_t global_cols, size_t row0, size_t col0, float lo,
                                            float hi, void* stream) {
    if (!d_dst || rows == 0 || cols == 0 || dst_stride < cols || (kind != 0 && kind != 1) || col0 + cols > global_cols) {
        set_error("bad random_fill_block arguments");
        return VSPEC_B200_ERR_ARG;
    }
    rand_block_kernel<<<grid_for(rows * cols), 256, 0, (cudaStream_t)stream>>>(d_dst, kind, rows, cols, dst_stride,
                                                                               seed, global_cols, row0, col0, lo, hi);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? VSPEC_B200_OK : cuda_status(e, "random_fill_block launch");
}
