/*
 * ref_shim.c -- small helpers, compiled together with Vspec-Engine's own CPU
 * sources into oracle/_ref/libvspec_ref.so, so that tests can drive the
 * reference's structs (VspecKernelContext, VspecKVCache, VspecKVPagedCache)
 * through ctypes.  TEST INFRASTRUCTURE ONLY.
 *
 * This file is this project's own code; it only includes the reference's
 * public headers (include/vspec/...).
 */
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "vspec/attention/attention.h"
#include "vspec/attention/flash_stub.h"
#include "vspec/attention/kv_cache.h"
#include "vspec/attention/kv_paged_cache.h"
#include "vspec/kernel/backend.h"
#include "vspec/kernel/context.h"
#include "vspec/quant/quant.h"

/* ---- ABI layout facts of the reference headers (checked against the B200 library) ---- */
size_t ref_sizeof_kernel_context(void) { return sizeof(VspecKernelContext); }
size_t ref_sizeof_quant_meta(void) { return sizeof(VspecQuantMeta); }
size_t ref_sizeof_exec_config(void) { return sizeof(VspecExecConfig); }
size_t ref_sizeof_kv_cache(void) { return sizeof(VspecKVCache); }
size_t ref_sizeof_kv_paged_cache(void) { return sizeof(VspecKVPagedCache); }
size_t ref_sizeof_backend(void) { return sizeof(VspecBackend); }
size_t ref_offsetof_ctx_qmeta(void) { return offsetof(VspecKernelContext, qmeta); }
size_t ref_offsetof_ctx_config(void) { return offsetof(VspecKernelContext, config); }
size_t ref_offsetof_qmeta_scales(void) { return offsetof(VspecQuantMeta, scales); }
size_t ref_offsetof_qmeta_scale_count(void) { return offsetof(VspecQuantMeta, scale_count); }
size_t ref_offsetof_kv_current_tokens(void) { return offsetof(VspecKVCache, current_tokens); }
size_t ref_offsetof_kv_int3(void) { return offsetof(VspecKVCache, int3_compressed); }
size_t ref_offsetof_paged_sessions(void) { return offsetof(VspecKVPagedCache, sessions); }
size_t ref_offsetof_paged_page_meta(void) { return offsetof(VspecKVPagedCache, page_meta); }

/* ---- CPU backend (src/kernel/cpu/cpu_backend.c) driven through its context ABI ---- */
void ref_cpu_backend_linear_int4(const float* a, size_t m, size_t k, const uint8_t* w, size_t n,
                                 const float* scales, float* out) {
    VspecKernelContext ctx;
    memset(&ctx, 0, sizeof(ctx));
    vspec_quant_meta_init(&ctx.qmeta);
    ctx.input = (void*)a;
    ctx.weight = (void*)w;
    ctx.output = (void*)out;
    ctx.qmeta.type = VSPEC_QUANT_INT4;
    ctx.qmeta.scales = scales;
    ctx.qmeta.scale_count = n;
    ctx.config.m = m;
    ctx.config.n = n;
    ctx.config.k = k;
    VspecBackend be = vspec_make_cpu_backend();
    be.launch_linear(&ctx);
}

/* Contiguous fp32 cache [tokens][heads][d] through vspec_kv_cache_init/append, then the
 * CPU backend's launch_attention (vspec_attention_ref_single_query). */
int ref_cpu_backend_attention(const float* q, const float* keys, const float* values,
                              size_t tokens, size_t heads, size_t d, float* out) {
    float* kb = (float*)calloc(tokens * heads * d, sizeof(float));
    float* vb = (float*)calloc(tokens * heads * d, sizeof(float));
    if (!kb || !vb) { free(kb); free(vb); return 0; }
    VspecKVCache cache;
    memset(&cache, 0, sizeof(cache));
    if (!vspec_kv_cache_init(&cache, kb, vb, tokens, heads, d)) { free(kb); free(vb); return 0; }
    for (size_t t = 0; t < tokens; ++t) {
        if (!vspec_kv_cache_append(&cache, keys + t * heads * d, values + t * heads * d)) {
            free(kb); free(vb); return 0;
        }
    }
    VspecKernelContext ctx;
    memset(&ctx, 0, sizeof(ctx));
    ctx.input = (void*)q;
    ctx.weight = (void*)&cache;
    ctx.output = (void*)out;
    VspecBackend be = vspec_make_cpu_backend();
    be.launch_attention(&ctx);
    free(kb);
    free(vb);
    return 1;
}

/* ---- Paged cache helpers ---- */
VspecKVPagedCache* ref_paged_create(size_t page_tokens, size_t max_pages, size_t heads, size_t d) {
    VspecKVPagedCache* c = (VspecKVPagedCache*)calloc(1, sizeof(VspecKVPagedCache));
    float* kp = (float*)calloc(page_tokens * max_pages * heads * d, sizeof(float));
    float* vp = (float*)calloc(page_tokens * max_pages * heads * d, sizeof(float));
    if (!c || !kp || !vp || !vspec_kv_paged_cache_init(c, kp, vp, page_tokens, max_pages, heads, d)) {
        free(c); free(kp); free(vp);
        return NULL;
    }
    return c;
}

void ref_paged_destroy(VspecKVPagedCache* c) {
    if (!c) return;
    free(c->key_pages);
    free(c->value_pages);
    free(c);
}

const float* ref_paged_key_pool(const VspecKVPagedCache* c) { return c->key_pages; }
const float* ref_paged_value_pool(const VspecKVPagedCache* c) { return c->value_pages; }

/* Copies the session's page list (uint16 pool ids, in order) and returns its length. */
size_t ref_paged_session_pages(const VspecKVPagedCache* c, uint64_t session, uint16_t* out, size_t cap) {
    for (size_t i = 0; i < VSPEC_KV_PAGED_MAX_SESSIONS; ++i) {
        if (c->sessions[i].active && c->sessions[i].session_id == session) {
            size_t n = c->sessions[i].page_count;
            if (out) {
                for (size_t p = 0; p < n && p < cap; ++p) out[p] = c->sessions[i].pages[p];
            }
            return n;
        }
    }
    return 0;
}

size_t ref_paged_page_used(const VspecKVPagedCache* c, size_t page) {
    return page < c->max_pages ? c->page_meta[page].used_tokens : 0;
}

/* Gathers every token of a session for every head through vspec_kv_paged_get_token_ptr
 * (src/attention/kv_paged_cache.c:312-356).  Output [tokens][heads][d]. */
int ref_paged_gather(const VspecKVPagedCache* c, uint64_t session, float* k_out, float* v_out) {
    const size_t tokens = vspec_kv_paged_session_tokens(c, session);
    for (size_t t = 0; t < tokens; ++t) {
        for (size_t h = 0; h < c->num_heads; ++h) {
            const float* kp = NULL;
            const float* vp = NULL;
            if (!vspec_kv_paged_get_token_ptr(c, session, t, h, &kp, &vp)) return 0;
            memcpy(k_out + (t * c->num_heads + h) * c->head_dim, kp, c->head_dim * sizeof(float));
            memcpy(v_out + (t * c->num_heads + h) * c->head_dim, vp, c->head_dim * sizeof(float));
        }
    }
    return 1;
}

/* ---- int3 KV compression through the reference cache (src/attention/kv_cache.c) ----
 * Appends `rows` tokens of [heads][head_dim] fp32 to a cache with int3
 * compression on (block 16 or 32) and copies out the key codes and scales. */
int ref_kv_int3_quantize(const float* src, size_t rows, size_t heads, size_t head_dim, size_t block_size,
                         uint8_t* codes_out, float* scales_out) {
    VspecKVCache c;
    memset(&c, 0, sizeof(c));
    const size_t n = rows * heads * head_dim;
    float* kb = (float*)calloc(n ? n : 1, sizeof(float));
    float* vb = (float*)calloc(n ? n : 1, sizeof(float));
    int ok = kb && vb && vspec_kv_cache_init(&c, kb, vb, rows, heads, head_dim) &&
             vspec_kv_cache_enable_int3_compression(&c, block_size);
    for (size_t r = 0; ok && r < rows; ++r)
        ok = vspec_kv_cache_append(&c, src + r * heads * head_dim, src + r * heads * head_dim);
    if (ok) {
        memcpy(codes_out, c.key_int3, rows * heads * c.packed_head_bytes);
        memcpy(scales_out, c.key_scales, rows * heads * c.blocks_per_head * sizeof(float));
    }
    vspec_kv_cache_disable_int3_compression(&c);
    free(kb);
    free(vb);
    return ok ? 0 : 1;
}
