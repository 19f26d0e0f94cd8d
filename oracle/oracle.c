/*
 * oracle.c -- CPU restatement of Vspec-Engine's low-bit dequant-matmul and
 * paged GQA decode attention.  TEST INFRASTRUCTURE ONLY (see oracle.h):
 * the shipped library never links or calls it.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

size_t oracle_row_bytes(size_t k, int bits) {
    /* src/quant/pack.c:11-16 */
    return (k * (size_t)bits + 7U) / 8U;
}

int8_t oracle_get_code(const uint8_t* row, size_t t, int bits) {
    /* src/quant/pack.c:53-74: LSB-first field of `bits` bits at bit t*bits,
     * possibly spanning two bytes, read as two's complement. */
    const size_t bit = t * (size_t)bits;
    const size_t byte = bit >> 3;
    const unsigned shift = (unsigned)(bit & 7U);
    unsigned v = (unsigned)row[byte] >> shift;
    if (8U - shift < (unsigned)bits) {
        v |= (unsigned)row[byte + 1U] << (8U - shift);
    }
    v &= (1U << bits) - 1U;
    if (v & (1U << (bits - 1))) {
        return (int8_t)((int)v - (1 << bits));
    }
    return (int8_t)v;
}

void oracle_pack_rows(const int8_t* codes, size_t n, size_t k, int bits, uint8_t* out) {
    /* src/quant/pack.c:30-51, applied per row so rows stay byte aligned
     * (Vspec-chat/python/runtime_inference.py:679-705 packs row by row). */
    const size_t rb = oracle_row_bytes(k, bits);
    const int lo = -(1 << (bits - 1));
    const int hi = (1 << (bits - 1)) - 1;
    const unsigned mask = (1U << bits) - 1U;
    memset(out, 0, n * rb);
    for (size_t j = 0; j < n; ++j) {
        uint8_t* row = out + j * rb;
        for (size_t t = 0; t < k; ++t) {
            int v = codes[j * k + t];
            if (v < lo) v = lo;
            if (v > hi) v = hi;
            const unsigned u = (unsigned)v & mask;
            const size_t bit = t * (size_t)bits;
            const size_t byte = bit >> 3;
            const unsigned shift = (unsigned)(bit & 7U);
            row[byte] |= (uint8_t)(u << shift);
            if (8U - shift < (unsigned)bits) {
                row[byte + 1U] |= (uint8_t)(u >> (8U - shift));
            }
        }
    }
}

void oracle_unpack_rows(const uint8_t* packed, size_t n, size_t k, int bits, int8_t* out) {
    const size_t rb = oracle_row_bytes(k, bits);
    for (size_t j = 0; j < n; ++j) {
        for (size_t t = 0; t < k; ++t) {
            out[j * k + t] = oracle_get_code(packed + j * rb, t, bits);
        }
    }
}

size_t oracle_group_of(size_t t, size_t k, size_t n_groups) {
    /* src/kernel/cuda/fused_linear_int4.cu:391-392 */
    if (n_groups <= 1U) return 0U;
    size_t g = (t * n_groups) / k;
    return g < n_groups ? g : n_groups - 1U;
}

void oracle_lowbit_matmul_f32(const float* a, size_t m, size_t k,
                              const uint8_t* w, size_t n, int bits,
                              const float* s, const float* zp, size_t n_groups,
                              float* c) {
    /* src/quant/int4.c:107-132 with the group indexing of
     * src/kernel/cuda/fused_linear_int4.cu:391-396: one fp32 accumulator per
     * output, terms added in t order, each term a[t] * ((q - zp) * s). */
    if (n_groups == 0U) n_groups = 1U;
    const size_t rb = oracle_row_bytes(k, bits);
    for (size_t i = 0; i < m; ++i) {
        const float* arow = a + i * k;
        for (size_t j = 0; j < n; ++j) {
            const uint8_t* wrow = w + j * rb;
            float acc = 0.0f;
            for (size_t t = 0; t < k; ++t) {
                const size_t idx = j * n_groups + oracle_group_of(t, k, n_groups);
                const float scale = s[idx];
                const float z = zp ? zp[idx] : 0.0f;
                const float q = (float)oracle_get_code(wrow, t, bits);
                acc += arow[t] * ((q - z) * scale);
            }
            c[i * n + j] = acc;
        }
    }
}

float oracle_half_to_float(uint16_t h) {
    /* IEEE 754 binary16: 1 sign, 5 exponent (bias 15), 10 fraction bits. */
    const int sign = (h >> 15) & 1;
    const int exp = (h >> 10) & 0x1F;
    const int frac = h & 0x3FF;
    float v;
    if (exp == 0) {
        v = ldexpf((float)frac, -24);              /* subnormal: frac * 2^-24 */
    } else if (exp == 31) {
        v = frac ? NAN : INFINITY;
    } else {
        v = ldexpf((float)(frac | 0x400), exp - 25); /* (1.frac) * 2^(exp-15) */
    }
    return sign ? -v : v;
}

void oracle_lowbit_matmul_f16sz(const float* a, size_t m, size_t k,
                                const uint8_t* w, size_t n, int bits,
                                const uint16_t* s16, const uint16_t* zp16, size_t n_groups,
                                float* c) {
    if (n_groups == 0U) n_groups = 1U;
    const size_t cnt = n * n_groups;
    float* s = (float*)malloc(cnt * sizeof(float));
    float* z = zp16 ? (float*)malloc(cnt * sizeof(float)) : NULL;
    for (size_t i = 0; i < cnt; ++i) {
        s[i] = oracle_half_to_float(s16[i]);
        if (z) z[i] = oracle_half_to_float(zp16[i]);
    }
    oracle_lowbit_matmul_f32(a, m, k, w, n, bits, s, z, n_groups, c);
    free(s);
    free(z);
}

void oracle_lowbit_matmul_f64acc(const float* a, size_t m, size_t k,
                                 const uint8_t* w, size_t n, int bits,
                                 const float* s, const float* zp, size_t n_groups,
                                 double* c) {
    if (n_groups == 0U) n_groups = 1U;
    const size_t rb = oracle_row_bytes(k, bits);
    for (size_t i = 0; i < m; ++i) {
        const float* arow = a + i * k;
        for (size_t j = 0; j < n; ++j) {
            const uint8_t* wrow = w + j * rb;
            double acc = 0.0;
            for (size_t t = 0; t < k; ++t) {
                const size_t idx = j * n_groups + oracle_group_of(t, k, n_groups);
                const double z = zp ? (double)zp[idx] : 0.0;
                const double q = (double)oracle_get_code(wrow, t, bits);
                acc += (double)arow[t] * ((q - z) * (double)s[idx]);
            }
            c[i * n + j] = acc;
        }
    }
}

void oracle_paged_gather_f32(const float* k_pages, const float* v_pages,
                             const int32_t* page_table, size_t ctx,
                             size_t page_tokens, size_t num_kv_heads, size_t head_dim,
                             float* k_out, float* v_out) {
    /* Token t lives in page page_table[t / page_tokens] at slot t % page_tokens
     * (kv_paged_cache.c:332-354 walks full pages in order). */
    const size_t stride = num_kv_heads * head_dim;      /* kv_paged_cache.c:5-7 */
    const size_t span = page_tokens * stride;           /* kv_paged_cache.c:9-11 */
    for (size_t t = 0; t < ctx; ++t) {
        const size_t page = (size_t)page_table[t / page_tokens];
        const size_t off = page * span + (t % page_tokens) * stride;
        memcpy(k_out + t * stride, k_pages + off, stride * sizeof(float));
        memcpy(v_out + t * stride, v_pages + off, stride * sizeof(float));
    }
}

static const float* token_row(const float* pages, const int32_t* table, size_t t,
                              size_t page_tokens, size_t num_kv_heads, size_t head_dim,
                              size_t kv_h) {
    const size_t stride = num_kv_heads * head_dim;
    const size_t page = (size_t)table[t / page_tokens];
    return pages + page * page_tokens * stride + (t % page_tokens) * stride + kv_h * head_dim;
}

void oracle_paged_gqa_attention_f32(const float* q, const float* k_pages, const float* v_pages,
                                    const int32_t* page_table, size_t max_pages_per_seq,
                                    const int32_t* ctx_len, size_t batch,
                                    size_t num_q_heads, size_t num_kv_heads, size_t head_dim,
                                    size_t page_tokens, float scale, float* out) {
    const size_t group = num_q_heads / num_kv_heads;
    for (size_t b = 0; b < batch; ++b) {
        const size_t ctx = (size_t)ctx_len[b];
        const int32_t* table = page_table + b * max_pages_per_seq;
        float* scores = (float*)malloc((ctx ? ctx : 1) * sizeof(float));
        for (size_t h = 0; h < num_q_heads; ++h) {
            /* runtime_inference.py:151 */
            size_t kv_h = h / (group ? group : 1);
            if (kv_h > num_kv_heads - 1) kv_h = num_kv_heads - 1;
            const float* qh = q + (b * num_q_heads + h) * head_dim;
            float* oh = out + (b * num_q_heads + h) * head_dim;
            for (size_t d = 0; d < head_dim; ++d) oh[d] = 0.0f;
            if (ctx == 0) continue;
            /* flash_stub.c:21-32 */
            float max_score = -1.0e30f;
            for (size_t t = 0; t < ctx; ++t) {
                const float* kt = token_row(k_pages, table, t, page_tokens, num_kv_heads, head_dim, kv_h);
                float acc = 0.0f;
                for (size_t d = 0; d < head_dim; ++d) acc += qh[d] * kt[d];
                scores[t] = acc * scale;
                if (scores[t] > max_score) max_score = scores[t];
            }
            /* flash_stub.c:34-41 */
            float sum = 0.0f;
            for (size_t t = 0; t < ctx; ++t) {
                scores[t] = expf(scores[t] - max_score);
                sum += scores[t];
            }
            if (sum < 1e-12f) sum = 1e-12f;
            /* flash_stub.c:43-52 */
            for (size_t t = 0; t < ctx; ++t) {
                const float p = scores[t] / sum;
                const float* vt = token_row(v_pages, table, t, page_tokens, num_kv_heads, head_dim, kv_h);
                for (size_t d = 0; d < head_dim; ++d) oh[d] += p * vt[d];
            }
        }
        free(scores);
    }
}

void oracle_paged_gqa_attention_f64(const float* q, const float* k_pages, const float* v_pages,
                                    const int32_t* page_table, size_t max_pages_per_seq,
                                    const int32_t* ctx_len, size_t batch,
                                    size_t num_q_heads, size_t num_kv_heads, size_t head_dim,
                                    size_t page_tokens, float scale, double* out) {
    const size_t group = num_q_heads / num_kv_heads;
    for (size_t b = 0; b < batch; ++b) {
        const size_t ctx = (size_t)ctx_len[b];
        const int32_t* table = page_table + b * max_pages_per_seq;
        double* scores = (double*)malloc((ctx ? ctx : 1) * sizeof(double));
        for (size_t h = 0; h < num_q_heads; ++h) {
            size_t kv_h = h / (group ? group : 1);
            if (kv_h > num_kv_heads - 1) kv_h = num_kv_heads - 1;
            const float* qh = q + (b * num_q_heads + h) * head_dim;
            double* oh = out + (b * num_q_heads + h) * head_dim;
            for (size_t d = 0; d < head_dim; ++d) oh[d] = 0.0;
            if (ctx == 0) continue;
            double max_score = -1.0e300;
            for (size_t t = 0; t < ctx; ++t) {
                const float* kt = token_row(k_pages, table, t, page_tokens, num_kv_heads, head_dim, kv_h);
                double acc = 0.0;
                for (size_t d = 0; d < head_dim; ++d) acc += (double)qh[d] * (double)kt[d];
                scores[t] = acc * (double)scale;
                if (scores[t] > max_score) max_score = scores[t];
            }
            double sum = 0.0;
            for (size_t t = 0; t < ctx; ++t) {
                scores[t] = exp(scores[t] - max_score);
                sum += scores[t];
            }
            for (size_t t = 0; t < ctx; ++t) {
                const double p = scores[t] / sum;
                const float* vt = token_row(v_pages, table, t, page_tokens, num_kv_heads, head_dim, kv_h);
                for (size_t d = 0; d < head_dim; ++d) oh[d] += p * (double)vt[d];
            }
        }
        free(scores);
    }
}

/* Row clamp to +-alpha*std, fp32 mean/variance accumulated in order
 * (src/kernel/cuda/fused_linear_int3.cu:20-53). */
void oracle_clamp_rows_std(const float* in, size_t rows, size_t cols, float alpha, float* out) {
    for (size_t r = 0; r < rows; ++r) {
        const float* x = in + r * cols;
        float mean = 0.0f;
        for (size_t i = 0; i < cols; ++i) mean += x[i];
        mean /= (float)cols;
        float var = 0.0f;
        for (size_t i = 0; i < cols; ++i) {
            const float d = x[i] - mean;
            var += d * d;
        }
        var /= (float)cols;
        const float sd = sqrtf(var > 0.0f ? var : 0.0f);
        float th = fabsf(alpha) * sd;
        if (th < 1e-6f) th = 1e-6f;
        for (size_t i = 0; i < cols; ++i) {
            float v = x[i];
            if (v < -th) v = -th;
            if (v > th) v = th;
            out[r * cols + i] = v;
        }
    }
}

/* ---- the CPU backend's attention (src/attention/attention_ref.c:7-88) ----
 * Per head of a contiguous [tokens][heads][d] fp32 cache: q and each k row clamped
 * to +-max(1e-6, 4.5 * population std, std in double; three_bit_runtime_modules.c:
 * 175-203), score = dot * (1/sqrtf(d)), softmax with a double denominator (:205-250),
 * output = double sum of p_t * v_t[x] (:260-282).  module != 0 is the 3-bit runtime
 * module: noise reducer (clip +-16, consecutive-delta limit 32; :138-173), dot over
 * blocks of `block` (32 or 64) normalised by the block's max |value| with Kahan
 * sums (:291-342), qk scale clipped to [1e-4, 32] (:344-361), logits clipped to
 * +-24, Kahan output sums with the 1e7 limit (:260-282). */
static float ar_clip(float x, float lo, float hi) { return x < lo ? lo : (x > hi ? hi : x); }

static void ar_condition(const float* x, size_t n, int module, float* out) {
    double mean = 0.0, var = 0.0;
    for (size_t i = 0; i < n; ++i) mean += (double)x[i];
    mean /= (double)n;
    for (size_t i = 0; i < n; ++i) var += ((double)x[i] - mean) * ((double)x[i] - mean);
    var /= (double)n;
    const float sd = (float)sqrt(var);
    const float th = fmaxf(1e-6f, 4.5f * sd);
    float prev = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        float v = ar_clip(x[i], -th, th);
        if (module) {
            v = ar_clip(v, -16.0f, 16.0f);
            if (i > 0) {
                const float delta = v - prev;
                if (fabsf(delta) > 32.0f) v = prev + (delta > 0.0f ? 32.0f : -32.0f);
            }
            prev = v;
        }
        out[i] = v;
    }
}

typedef struct { double sum, comp; } ArAcc;

static void ar_add(ArAcc* a, float value, int module) {
    if (!module) {
        a->sum += (double)value;
        return;
    }
    const double y = (double)value - a->comp;
    const double t = a->sum + y;
    a->comp = (t - a->sum) - y;
    a->sum = t;
    if (fabs(a->sum) > 1e7) {
        a->sum = (double)ar_clip((float)a->sum, -1e7f, 1e7f);
        a->comp = 0.0;
    }
}

static float ar_dot(const float* a, const float* b, size_t n, int module, size_t block) {
    if (!module) {
        float s = 0.0f;
        for (size_t i = 0; i < n; ++i) s += a[i] * b[i];
        return s;
    }
    ArAcc total = {0.0, 0.0};
    for (size_t base = 0; base < n; base += block) {
        const size_t end = base + block < n ? base + block : n;
        float babs = 0.0f;
        for (size_t i = base; i < end; ++i) {
            if (fabsf(a[i]) > babs) babs = fabsf(a[i]);
            if (fabsf(b[i]) > babs) babs = fabsf(b[i]);
        }
        const float bs = fmaxf(babs, 1e-6f);
        ArAcc local = {0.0, 0.0};
        for (size_t i = base; i < end; ++i) ar_add(&local, (a[i] / bs) * (b[i] / bs), 1);
        ar_add(&total, (float)local.sum * bs * bs, 1);
    }
    return (float)total.sum;
}

void oracle_attention_ref_f32(const float* q, const float* keys, const float* values, size_t tokens, size_t heads,
                              size_t d, int module, size_t block, float* out) {
    if (block != 32) block = 64;
    float* qc = (float*)malloc(d * sizeof(float));
    float* kc = (float*)malloc(d * sizeof(float));
    float* sc = (float*)malloc(tokens * sizeof(float));
    ArAcc* acc = (ArAcc*)malloc(d * sizeof(ArAcc));
    const float inv_sqrt_d = 1.0f / sqrtf((float)d);
    const float scale = module ? ar_clip(inv_sqrt_d, 1e-4f, 32.0f) : inv_sqrt_d;
    for (size_t h = 0; h < heads; ++h) {
        ar_condition(q + h * d, d, module, qc);
        float mx = -3.402823466e38f;
        for (size_t t = 0; t < tokens; ++t) {
            ar_condition(keys + (t * heads + h) * d, d, module, kc);
            float s = ar_dot(qc, kc, d, module, block) * scale;
            if (module) s = ar_clip(s, -24.0f, 24.0f);
            sc[t] = s;
            if (s > mx) mx = s;
        }
        double den = 0.0;
        for (size_t t = 0; t < tokens; ++t) {
            sc[t] = expf(sc[t] - mx);
            den += (double)sc[t];
        }
        if (den < (double)1e-12f) {
            for (size_t t = 0; t < tokens; ++t) sc[t] = 1.0f / (float)tokens;
        } else {
            const float inv = 1.0f / (float)den;
            for (size_t t = 0; t < tokens; ++t) sc[t] *= inv;
        }
        for (size_t x = 0; x < d; ++x) acc[x].sum = acc[x].comp = 0.0;
        for (size_t t = 0; t < tokens; ++t) {
            const float* vr = values + (t * heads + h) * d;
            for (size_t x = 0; x < d; ++x) ar_add(&acc[x], sc[t] * vr[x], module);
        }
        for (size_t x = 0; x < d; ++x) out[h * d + x] = (float)acc[x].sum;
    }
    free(qc);
    free(kc);
    free(sc);
    free(acc);
}

static float sr_uniform01(uint32_t state) {
    /* xorshift32 -> 24-bit uniform (src/kernel/cuda/fused_linear_int3.cu:68-73) */
    state ^= state << 13;
    state ^= state >> 17;
    state ^= state << 5;
    return (float)(state & 0x00FFFFFFu) / 16777216.0f;
}

/* The reference int3 CUDA kernel's arithmetic (src/kernel/cuda/fused_linear_int3.cu:82-147):
 * per-row scale, 32-wide blocks normalized by max(|a|, |w|), optional stochastic rounding of
 * the normalized weight to 1/16 steps seeded by (i, j, t), block sums rescaled by bs^2. */
void oracle_int3_blocknorm_f32(const float* a, size_t m, size_t k, const uint8_t* w, size_t n,
                               const float* s, int stochastic, float* c) {
    const size_t rb = oracle_row_bytes(k, 3);
    for (size_t i = 0; i < m; ++i) {
        for (size_t j = 0; j < n; ++j) {
            const uint8_t* row = w + j * rb;
            const float scale = s[j];
            float acc = 0.0f;
            for (size_t base = 0; base < k; base += 32) {
                const size_t end = base + 32 < k ? base + 32 : k;
                float babs = 0.0f;
                for (size_t t = base; t < end; ++t) {
                    const float av = fabsf(a[i * k + t]);
                    const float wv = fabsf((float)oracle_get_code(row, t, 3) * scale);
                    if (av > babs) babs = av;
                    if (wv > babs) babs = wv;
                }
                const float bs = babs > 1e-6f ? babs : 1e-6f;
                float bacc = 0.0f;
                for (size_t t = base; t < end; ++t) {
                    const float an = a[i * k + t] / bs;
                    float wn = ((float)oracle_get_code(row, t, 3) * scale) / bs;
                    if (stochastic) {
                        const uint32_t seed = (uint32_t)((uint32_t)(i * 2654435761u) ^ (uint32_t)(j * 2246822519u) ^
                                                         (uint32_t)(t * 3266489917u) ^ 0x9E3779B9u);
                        const float steps = wn * 16.0f;
                        const float lo = floorf(steps);
                        wn = ((sr_uniform01(seed) < steps - lo) ? (lo + 1.0f) : lo) / 16.0f;
                    }
                    bacc += an * wn;
                }
                acc += bacc * bs * bs;
            }
            c[i * n + j] = acc;
        }
    }
}

/* ------------------------------------------------------------------------
 * fp16 rounding (round to nearest, ties to even; subnormals and overflow to
 * infinity handled), used where the engine stores fp16.
 * ------------------------------------------------------------------------ */
uint16_t oracle_float_to_half(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t absx = x & 0x7FFFFFFFu;
    if (absx >= 0x7F800000u) return (uint16_t)(sign | (absx > 0x7F800000u ? 0x7E00u : 0x7C00u));
    const int e = (int)(absx >> 23) - 127;
    if (e > 15) return (uint16_t)(sign | 0x7C00u);
    if (e >= -14) {
        /* normal: keep 10 mantissa bits, round the 13 dropped bits */
        uint32_t mant = absx & 0x7FFFFFu;
        uint32_t h = ((uint32_t)(e + 15) << 10) | (mant >> 13);
        const uint32_t rem = mant & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u;   /* may carry into the exponent: fine */
        return (uint16_t)(sign | h);
    }
    if (e < -25) return sign;
    /* subnormal: value = mant_full * 2^(e-23), in units of 2^-24 */
    const uint32_t mant_full = (absx & 0x7FFFFFu) | 0x800000u;
    const int shift = -e - 14 + 13;   /* 14..24 */
    uint32_t h = mant_full >> shift;
    const uint32_t rem = mant_full & ((1u << shift) - 1u);
    const uint32_t halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (h & 1u))) h += 1u;
    return (uint16_t)(sign | h);
}

/* ------------------------------------------------------------------------
 * Qwen3-shape decode (test oracle; see oracle.h for the reference lines).
 * ------------------------------------------------------------------------ */
static void oq_rmsnorm(const float* x, int n, float eps, float* out) {
    double ss = 0.0;
    for (int i = 0; i < n; ++i) ss += (double)x[i] * (double)x[i];
    const float inv = (float)(1.0 / sqrt(ss / (double)n + (double)eps));
    for (int i = 0; i < n; ++i) out[i] = x[i] * inv;   /* weight = 1 */
}

/* Unsigned b-bit fields of one packed row (the LSB-first bitstream of
 * src/quant/pack.c:53-74 read without sign), minus 2^(bits-1): the same values
 * as (oracle_get_code + 2^bits) mod 2^bits - 2^(bits-1), a row at a time. */
static void oq_unpack_row_centered(const uint8_t* row, int k, int bits, double* out) {
    const int off = 1 << (bits - 1);
    if (bits == 4) {
        for (int t = 0; t + 1 < k; t += 2) {
            const uint8_t b = row[t >> 1];
            out[t] = (double)((b & 0xF) - off);
            out[t + 1] = (double)((b >> 4) - off);
        }
        if (k & 1) out[k - 1] = (double)((row[(k - 1) >> 1] & 0xF) - off);
        return;
    }
    int t0 = 0;
    if (bits == 3) {
        /* eight fields per 24-bit little-endian word */
        for (; t0 + 8 <= k; t0 += 8) {
            const uint8_t* p = row + (t0 / 8) * 3;
            const uint32_t wv = (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16);
            for (int e = 0; e < 8; ++e) out[t0 + e] = (double)((int)((wv >> (3 * e)) & 7u) - off);
        }
    } else if (bits == 2) {
        for (; t0 + 4 <= k; t0 += 4) {
            const uint8_t b = row[t0 / 4];
            for (int e = 0; e < 4; ++e) out[t0 + e] = (double)((int)((b >> (2 * e)) & 3u) - off);
        }
    }
    for (int t = t0; t < k; ++t) {
        const int code = oracle_get_code(row, (size_t)t, bits);
        out[t] = (double)(((code + (1 << bits)) & ((1 << bits) - 1)) - off);
    }
}

/* y[n] = sum_t x[t] * (u(n,t) - 2^(bits-1)) * s[n][t / group], double accumulate */
static void oq_linear(const float* x, int k, const uint8_t* w, const uint16_t* s, int n, int bits, int group, float* y) {
    const size_t rb = oracle_row_bytes((size_t)k, bits);
    const int groups = k / group;
    double* xd = (double*)malloc(sizeof(double) * (size_t)k);
    double* cd = (double*)malloc(sizeof(double) * (size_t)k);
    if (!xd || !cd) { free(xd); free(cd); for (int j = 0; j < n; ++j) y[j] = NAN; return; }
    for (int t = 0; t < k; ++t) xd[t] = (double)x[t];
    for (int j = 0; j < n; ++j) {
        oq_unpack_row_centered(w + (size_t)j * rb, k, bits, cd);
        double acc = 0.0;
        for (int g = 0; g < groups; ++g) {
            const double sc = (double)oracle_half_to_float(s[(size_t)j * groups + g]);
            double part = 0.0;
            for (int t = g * group; t < (g + 1) * group; ++t) part += xd[t] * cd[t];
            acc += part * sc;
        }
        y[j] = (float)acc;
    }
    free(xd);
    free(cd);
}

int oracle_qwen_generate(const OracleQwen* q, const int32_t* prompt, int prompt_len, int gen, int32_t* tokens_out,
                         float* logits_out) {
    const int H = q->hidden, hq = q->heads, hkv = q->kv_heads, d = q->head_dim, I = q->inter, V = q->vocab;
    const int qdim = hq * d, qkvn = qdim + 2 * hkv * d;
    const int bm = q->bits_mlp ? q->bits_mlp : q->bits;
    const int total = prompt_len + gen;
    const int steps = total - 1;
    float* x = (float*)malloc(sizeof(float) * H);
    float* xn = (float*)malloc(sizeof(float) * (H > I ? H : I));
    float* qkv = (float*)malloc(sizeof(float) * qkvn);
    float* att = (float*)malloc(sizeof(float) * qdim);
    float* tmp = (float*)malloc(sizeof(float) * (H > 2 * I ? H : 2 * I));
    float* hbuf = (float*)malloc(sizeof(float) * I);
    float* logits = (float*)malloc(sizeof(float) * V);
    float* scores = (float*)malloc(sizeof(float) * total);
    /* fp16 K/V cache [layers][total][hkv][d] */
    uint16_t* kc = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)q->layers * total * hkv * d);
    uint16_t* vc = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)q->layers * total * hkv * d);
    if (!x || !xn || !qkv || !att || !tmp || !hbuf || !logits || !scores || !kc || !vc) return -1;
    for (int i = 0; i < prompt_len; ++i) tokens_out[i] = prompt[i];
    int tok = prompt[0];
    const int half = d / 2;
    for (int pos = 0; pos < steps; ++pos) {
        for (int i = 0; i < H; ++i) x[i] = oracle_half_to_float(q->emb[(size_t)tok * H + i]);
        for (int l = 0; l < q->layers; ++l) {
            const uint8_t* const* W = q->w + (size_t)l * 4;
            const uint16_t* const* S = q->s + (size_t)l * 4;
            oq_rmsnorm(x, H, q->eps, xn);
            oq_linear(xn, H, W[0], S[0], qkvn, q->bits, q->group, qkv);
            /* per-head RMSNorm of q and k, rotary, cache k and v as fp16 */
            for (int h = 0; h < hq + hkv; ++h) {
                float* v = qkv + (size_t)h * d;
                float nv[256];
                oq_rmsnorm(v, d, q->eps, nv);
                for (int t = 0; t < d; ++t) {
                    const int i = t < half ? t : t - half;
                    /* runtime_inference.py:4227,1187-1191 in float32: inv_freq =
                     * fl32(1 / fl32(theta ** fl32(i / half))), angle = fl32(pos * inv_freq),
                     * cos / sin of the float angle; power and sin / cos correctly rounded
                     * (evaluated in double, rounded once) */
                    const float pw = (float)pow((double)q->theta, (double)((float)i / (float)half));
                    const float inv_freq = 1.0f / pw;
                    const float ang = (float)pos * inv_freq;
                    const float cs = (float)cos((double)ang), sn = (float)sin((double)ang);
                    v[t] = t < half ? nv[t] * cs - nv[t + half] * sn : nv[t - half] * sn + nv[t] * cs;
                }
                if (h >= hq) {
                    uint16_t* dst = kc + (((size_t)l * total + pos) * hkv + (h - hq)) * d;
                    for (int t = 0; t < d; ++t) dst[t] = oracle_float_to_half(v[t]);
                }
            }
            for (int h = 0; h < hkv; ++h) {
                const float* v = qkv + (size_t)(hq + hkv + h) * d;
                uint16_t* dst = vc + (((size_t)l * total + pos) * hkv + h) * d;
                for (int t = 0; t < d; ++t) dst[t] = oracle_float_to_half(v[t]);
            }
            /* GQA attention over positions 0..pos (flash_stub math) */
            const int group = hq / hkv;
            const float scale = 1.0f / sqrtf((float)d);
            for (int h = 0; h < hq; ++h) {
                const int kh = h / group;
                const float* qh = qkv + (size_t)h * d;
                float mx = -INFINITY;
                for (int t = 0; t <= pos; ++t) {
                    const uint16_t* kr = kc + (((size_t)l * total + t) * hkv + kh) * d;
                    double dot = 0.0;
                    for (int e = 0; e < d; ++e) dot += (double)qh[e] * (double)oracle_half_to_float(kr[e]);
                    scores[t] = (float)dot * scale;
                    if (scores[t] > mx) mx = scores[t];
                }
                double sum = 0.0;
                for (int t = 0; t <= pos; ++t) { scores[t] = expf(scores[t] - mx); sum += scores[t]; }
                for (int e = 0; e < d; ++e) {
                    double o = 0.0;
                    for (int t = 0; t <= pos; ++t)
                        o += (double)scores[t] * (double)oracle_half_to_float(vc[(((size_t)l * total + t) * hkv + kh) * d + e]);
                    att[(size_t)h * d + e] = (float)(o / sum);
                }
            }
            oq_linear(att, qdim, W[1], S[1], H, q->bits, q->group, tmp);
            for (int i = 0; i < H; ++i) x[i] += tmp[i];
            oq_rmsnorm(x, H, q->eps, xn);
            oq_linear(xn, H, W[2], S[2], 2 * I, bm, q->group, tmp);
            for (int i = 0; i < I; ++i) {
                const float g = tmp[i], u = tmp[I + i];
                hbuf[i] = g / (1.0f + expf(-g)) * u;
            }
            oq_linear(hbuf, I, W[3], S[3], H, bm, q->group, tmp);
            for (int i = 0; i < H; ++i) x[i] += tmp[i];
        }
        oq_rmsnorm(x, H, q->eps, xn);
        oq_linear(xn, H, q->w_lm, q->s_lm, V, q->bits, q->group, logits);
        if (logits_out) memcpy(logits_out + (size_t)pos * V, logits, sizeof(float) * V);
        int best = 0;
        float bv = -INFINITY;
        for (int j = 0; j < V; ++j) {
            float v = logits[j];
            if (v != v) v = 0.f;
            v = v > q->clip ? q->clip : (v < -q->clip ? -q->clip : v);
            if (v > bv) { bv = v; best = j; }
        }
        const int nxt = (pos + 1 < prompt_len) ? prompt[pos + 1] : best;
        tokens_out[pos + 1] = nxt;
        tok = nxt;
    }
    free(x); free(xn); free(qkv); free(att); free(tmp); free(hbuf); free(logits); free(scores); free(kc); free(vc);
    return 0;
}

/* ---------------------------------------------------------------------------
 * Load-time quantizer: Vspec-chat/python/runtime_inference.py:708-785
 * (_quantize_weight_rowwise) restated with numpy's float32 semantics:
 *   - quantiles by numpy's default 'linear' method on float32 data
 *     (numpy/lib/_function_base_impl.py _quantile/_lerp): q cast to float32,
 *     virtual index (n-1)*q in float32, gamma its fractional part, and
 *     a + (b-a)*g for g < 0.5, b - (b-a)*(1-g) otherwise;
 *   - np.min / np.max when the percentile is >= 0.9999 (:722-724);
 *   - span = max(hi - lo, 1e-8), scale = span / levels, zp = clip(round(
 *     min_q - lo/scale)), q = clip(round(w/scale + zp)), all float32 with
 *     round-half-to-even (np.round), blocks along k (:734-764) or whole rows
 *     (:766-773);
 * and the codes packed per row (oracle_pack_rows).  block_size 0 = per row;
 * zero_points may be NULL (the reference returns None for int2, :775-777,
 * but the codes still carry the zero-point).  The arithmetic is kept in
 * separate float operations (this file is built without FMA contraction).
 * ------------------------------------------------------------------------- */
static int cmp_f32(const void* a, const void* b) {
    const float x = *(const float*)a, y = *(const float*)b;
    return (x > y) - (x < y);
}

static float np_quantile_sorted_f32(const float* sorted, int n, double q) {
    const float q32 = (float)q;
    const float vi = (float)(n - 1) * q32;
    if (!(vi > 0.0f)) return sorted[0];
    if (vi >= (float)(n - 1)) return sorted[n - 1];
    const float prev = floorf(vi);
    const int lo = (int)prev;
    const int hi = lo + 1 < n ? lo + 1 : n - 1;
    const float g = vi - prev;
    const float a = sorted[lo], b = sorted[hi];
    const float d = b - a;
    if (g >= 0.5f) {
        const float t = 1.0f - g;
        const float dt = d * t;
        return b - dt;
    }
    const float dg = d * g;
    return a + dg;
}

int oracle_quantize_rowwise(const float* w, size_t n, size_t k, int bits, int block_size, double percentile,
                            uint8_t* packed, float* scales, float* zero_points) {
    if (!w || !packed || !scales || n == 0 || k == 0 || bits < 2 || bits > 4 || block_size < 0) return -1;
    double pc = percentile;
    if (pc < 0.95) pc = 0.95;
    if (pc > 1.0) pc = 1.0;
    const double lo_q = 1.0 - pc;
    const float max_q = (float)((1 << (bits - 1)) - 1);
    const float min_q = (float)(-(1 << (bits - 1)));
    const float levels = (max_q - min_q) > 1.0f ? (max_q - min_q) : 1.0f;
    const size_t bs = block_size > 0 ? (size_t)block_size : k;
    const size_t nb = (k + bs - 1) / bs;
    float* buf = (float*)malloc(sizeof(float) * bs);
    int8_t* codes = (int8_t*)malloc(k);
    if (!buf || !codes) { free(buf); free(codes); return -1; }
    const size_t rb = oracle_row_bytes(k, bits);
    for (size_t r = 0; r < n; ++r) {
        const float* wr = w + r * k;
        for (size_t b = 0; b < nb; ++b) {
            const size_t s0 = b * bs, s1 = s0 + bs < k ? s0 + bs : k;
            const int len = (int)(s1 - s0);
            memcpy(buf, wr + s0, sizeof(float) * (size_t)len);
            qsort(buf, (size_t)len, sizeof(float), cmp_f32);
            float bmin, bmax;
            if (pc >= 0.9999) {
                bmin = buf[0];
                bmax = buf[len - 1];
            } else {
                bmin = np_quantile_sorted_f32(buf, len, lo_q);
                bmax = np_quantile_sorted_f32(buf, len, pc);
            }
            float span = bmax - bmin;
            const float floor_span = 1e-8f;
            if (span < floor_span) span = floor_span;
            const float scale = span / levels;
            const float ratio = bmin / scale;
            float zp = rintf(min_q - ratio);
            zp = zp < min_q ? min_q : (zp > max_q ? max_q : zp);
            for (size_t t = s0; t < s1; ++t) {
                const float v = wr[t] / scale;
                float qv = rintf(v + zp);
                qv = qv < min_q ? min_q : (qv > max_q ? max_q : qv);
                codes[t] = (int8_t)qv;
            }
            scales[r * nb + b] = scale;
            if (zero_points) zero_points[r * nb + b] = zp;
        }
        oracle_pack_rows(codes, 1, k, bits, packed + r * rb);
    }
    free(buf);
    free(codes);
    return 0;
}

/* ---- int3 KV-cache compression (src/attention/kv_cache.c:32-126, 160-226) ---- */
static int cmp_float_asc(const void* a, const void* b) {
    const float x = *(const float*)a, y = *(const float*)b;
    return x < y ? -1 : (x > y ? 1 : 0);
}

void oracle_kv_int3_quantize(const float* src, size_t rows, size_t heads, size_t head_dim, size_t block_size,
                             float percentile, uint8_t* codes, float* scales) {
    const size_t pb = oracle_row_bytes(head_dim, 3);
    const size_t nb = (head_dim + block_size - 1) / block_size;
    if (percentile < 50.0f) percentile = 50.0f;       /* kv_cache.c:38-43 */
    if (percentile > 100.0f) percentile = 100.0f;
    int8_t* q = (int8_t*)malloc(head_dim);
    float tmp[32];
    for (size_t r = 0; r < rows; ++r) {
        for (size_t h = 0; h < heads; ++h) {
            const float* x = src + (r * heads + h) * head_dim;
            float* sc = scales + (r * heads + h) * nb;
            for (size_t b = 0; b < nb; ++b) {
                const size_t base = b * block_size;
                size_t len = block_size;
                if (base + len > head_dim) len = head_dim - base;
                size_t n = len > 32 ? 32 : len;
                for (size_t i = 0; i < n; ++i) tmp[i] = fabsf(x[base + i]);
                qsort(tmp, n, sizeof(float), cmp_float_asc);
                size_t idx = (size_t)((double)(n - 1) * ((double)percentile / 100.0));
                if (idx >= n) idx = n - 1;
                const float rep = n ? tmp[idx] : 0.0f;
                float scale = rep > 0.0f ? rep / 4.0f : 1.0f;   /* qmax = 4 */
                if (scale < 1e-6f) scale = 1e-6f;
                sc[b] = scale;
                for (size_t i = 0; i < len; ++i) {
                    const long qi = lrintf(x[base + i] / scale);
                    int v = (int8_t)qi;                          /* the int8 cast before the clip */
                    if (v < -4) v = -4;
                    if (v > 3) v = 3;
                    q[base + i] = (int8_t)v;
                }
            }
            oracle_pack_rows(q, 1, head_dim, 3, codes + (r * heads + h) * pb);
        }
    }
    free(q);
}

void oracle_paged_int3_attention_f64(const float* q, const uint8_t* k_codes, const uint8_t* v_codes,
                                     const float* k_scales, const float* v_scales, const int32_t* page_table,
                                     size_t max_pages_per_seq, const int32_t* ctx_len, size_t batch,
                                     size_t num_q_heads, size_t num_kv_heads, size_t head_dim, size_t page_tokens,
                                     size_t block_size, float scale, double* out) {
    const size_t group = num_q_heads / num_kv_heads;
    const size_t pb = oracle_row_bytes(head_dim, 3);
    const size_t nb = (head_dim + block_size - 1) / block_size;
    float* kd = (float*)malloc(head_dim * sizeof(float));
    float* vd = (float*)malloc(head_dim * sizeof(float));
    for (size_t b = 0; b < batch; ++b) {
        const size_t ctx = (size_t)ctx_len[b];
        const int32_t* table = page_table + b * max_pages_per_seq;
        double* scores = (double*)malloc((ctx ? ctx : 1) * sizeof(double));
        for (size_t h = 0; h < num_q_heads; ++h) {
            size_t kv_h = h / (group ? group : 1);
            if (kv_h > num_kv_heads - 1) kv_h = num_kv_heads - 1;
            const float* qh = q + (b * num_q_heads + h) * head_dim;
            double* oh = out + (b * num_q_heads + h) * head_dim;
            for (size_t d = 0; d < head_dim; ++d) oh[d] = 0.0;
            if (ctx == 0) continue;
            double max_score = -1.0e300;
            for (size_t t = 0; t < ctx; ++t) {
                const size_t row = ((size_t)table[t / page_tokens] * page_tokens + t % page_tokens) * num_kv_heads + kv_h;
                for (size_t d = 0; d < head_dim; ++d)   /* attention_fused.cu:23-45: q * s[block] */
                    kd[d] = (float)oracle_get_code(k_codes + row * pb, d, 3) * k_scales[row * nb + d / block_size];
                double acc = 0.0;
                for (size_t d = 0; d < head_dim; ++d) acc += (double)qh[d] * (double)kd[d];
                scores[t] = acc * (double)scale;
                if (scores[t] > max_score) max_score = scores[t];
            }
            double sum = 0.0;
            for (size_t t = 0; t < ctx; ++t) {
                scores[t] = exp(scores[t] - max_score);
                sum += scores[t];
            }
            for (size_t t = 0; t < ctx; ++t) {
                const size_t row = ((size_t)table[t / page_tokens] * page_tokens + t % page_tokens) * num_kv_heads + kv_h;
                for (size_t d = 0; d < head_dim; ++d)
                    vd[d] = (float)oracle_get_code(v_codes + row * pb, d, 3) * v_scales[row * nb + d / block_size];
                const double pr = scores[t] / sum;
                for (size_t d = 0; d < head_dim; ++d) oh[d] += pr * (double)vd[d];
            }
        }
        free(scores);
    }
    free(kd);
    free(vd);
}

/* ---- Q4_K (src/quant/formats/q4_k.c:41-134) ---- */
static float q4k_half(uint16_t h) {   /* fp16 -> fp32 by the IEEE definition */
    const int e = (h >> 10) & 0x1F, f = h & 0x3FF;
    float v;
    if (e == 0) v = ldexpf((float)f, -24);
    else if (e == 31) v = f ? NAN : INFINITY;
    else v = ldexpf((float)(f | 0x400), e - 25);
    return (h & 0x8000) ? -v : v;
}

void oracle_q4k_matmul_f32(const float* a, size_t m, size_t k, const uint8_t* blocks, size_t n, float* c) {
    const size_t nb = k / 256;
    float* row = (float*)malloc(k * sizeof(float));
    for (size_t j = 0; j < n; ++j) {
        for (size_t b = 0; b < nb; ++b) {
            const uint8_t* blk = blocks + (j * nb + b) * 144;
            const float d = q4k_half((uint16_t)(blk[0] | (blk[1] << 8)));
            const float dmin = q4k_half((uint16_t)(blk[2] | (blk[3] << 8)));
            uint8_t sm[16];
            for (int i = 0; i < 16; ++i) {   /* 6-bit fields, LSB first */
                const int bit = 6 * i;
                const unsigned v = (unsigned)blk[4 + bit / 8] | ((bit / 8 + 1 < 12) ? (unsigned)blk[4 + bit / 8 + 1] << 8 : 0u);
                sm[i] = (uint8_t)((v >> (bit % 8)) & 0x3F);
            }
            for (int sb = 0; sb < 8; ++sb) {
                const float sub_scale = d * ((float)sm[sb] / 63.0f);
                const float sub_min = dmin * ((float)sm[8 + sb] / 63.0f);
                for (int t = 0; t < 32; ++t) {
                    const int local = sb * 32 + t;
                    const uint8_t byte = blk[16 + local / 2];
                    const float q = (float)((local & 1) ? (byte >> 4) : (byte & 0x0F));
                    row[b * 256 + local] = (sub_scale * q) - sub_min;
                }
            }
        }
        for (size_t i = 0; i < m; ++i) {
            float acc = 0.0f;
            for (size_t t = 0; t < k; ++t) acc += a[i * k + t] * row[t];
            c[i * n + j] = acc;
        }
    }
    free(row);
}

/* ---- ANF hybrid linear (src/kernel/cuda/fused_linear_hybrid.cu:7-153,
 *      src/kernel/cuda/fused_linear_int2.cu:8-12,14-76) ---- */
void oracle_anf_hybrid_f32(const float* a, size_t m, size_t k, const uint8_t* w2, const float* s2,
                           const uint8_t* w4, const float* s4, const float* zp4, size_t n_blocks,
                           const uint32_t* hot, size_t hot_count, size_t n, float* c) {
    const size_t pk2 = (k + 3) / 4, pk4 = (k + 1) / 2;
    for (size_t i = 0; i < m; ++i)
        for (size_t j = 0; j < n; ++j) {
            const float s = s2 ? s2[j] : 1.0f;
            float acc = 0.0f;
            for (size_t t = 0; t < k; ++t) {
                const unsigned q = (w2[j * pk2 + (t >> 2)] >> ((t & 3) * 2)) & 3u;
                acc += a[i * k + t] * (((float)q - 1.5f) * s);
            }
            c[i * n + j] = acc;
        }
    if (!hot || hot_count == 0 || !w4 || !s4) return;
    if (n_blocks == 0) n_blocks = 1;
    const size_t bs = n_blocks > 1 ? (k + n_blocks - 1) / n_blocks : k;
    for (size_t h = 0; h < hot_count; ++h) {
        const size_t j = hot[h];
        if (j >= n) continue;
        for (size_t i = 0; i < m; ++i) {
            float acc = 0.0f;
            for (size_t t = 0; t < k; ++t) {
                const uint8_t byte = w4[j * pk4 + (t >> 1)];
                const unsigned q = (t & 1) ? (byte >> 4) & 0xFu : byte & 0xFu;
                size_t b = 0;
                if (n_blocks > 1) {
                    b = t / bs;
                    if (b >= n_blocks) b = n_blocks - 1;
                }
                const float zp = zp4 ? zp4[j * n_blocks + b] : 0.0f;
                acc += a[i * k + t] * (((float)q - 8.0f) * s4[j * n_blocks + b] + zp);
            }
            c[i * n + j] = acc;
        }
    }
}
