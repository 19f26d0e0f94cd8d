/* kv_adapter.c -- device view of the reference's host paged KV cache.
 *
 * Vspec keeps decode K/V in a VspecKVPagedCache (include/vspec/attention/
 * kv_paged_cache.h:7-49): fp32 pools [max_pages][page_tokens][heads][head_dim]
 * on the host, sessions holding their pages in token order, pages filled by
 * vspec_kv_paged_append (src/attention/kv_paged_cache.c:243-310) and shared
 * between sessions by vspec_kv_paged_reuse_prefix (:185-241).  The paged
 * attention of this library reads the same page layout from device pools with
 * an int32 page table per sequence.  The two functions here connect them:
 *
 *   vspec_b200_kv_paged_sync          copies the pages written since a given
 *                                     clock step to the device pools, at the
 *                                     same page index, as fp32 or fp16;
 *   vspec_b200_kv_paged_session_view  writes one session's page-table row and
 *                                     context length on the device.
 *
 * The attention finds token t at slot t % page_tokens of page row[t /
 * page_tokens], i.e. every page but the last is full.  A session made by
 * reuse_prefix from a source whose last page was partly filled continues on a
 * fresh page after that short page (an append never writes into a page with
 * ref_count > 1, :273-277), so its token order walks a short page in the
 * middle (vspec_kv_paged_get_token_ptr subtracts each page's used_tokens,
 * :332-348).  For such a session the view gathers the tokens from the short
 * page on, in that order, into spare device pages beyond cache->max_pages and
 * points the row at them; the pages before it map through unchanged.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "bridge_internal.h"

/* IEEE binary16 of a float, round to nearest even (the engine's fp16 pages). */
static uint16_t vb_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t a = x & 0x7FFFFFFFu;
    if (a >= 0x7F800000u) return (uint16_t)(sign | (a > 0x7F800000u ? 0x7E00u : 0x7C00u));
    const int e = (int)(a >> 23) - 127;
    if (e > 15) return (uint16_t)(sign | 0x7C00u);
    if (e >= -14) {
        uint32_t h = ((uint32_t)(e + 15) << 10) | ((a & 0x7FFFFFu) >> 13);
        const uint32_t rem = a & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u;
        return (uint16_t)(sign | h);
    }
    if (e < -25) return sign;
    const uint32_t m = (a & 0x7FFFFFu) | 0x800000u;
    const int sh = -e - 1;   /* 14..24: value = m * 2^(e - 23) in units of 2^-24 */
    uint32_t h = m >> sh;
    const uint32_t rem = m & ((1u << sh) - 1u);
    const uint32_t half = 1u << (sh - 1);
    if (rem > half || (rem == half && (h & 1u))) h += 1u;
    return (uint16_t)(sign | h);
}

static int vb_cuda_err(cudaError_t e, const char* what) {
    vb_set_error("%s: %s", what, cudaGetErrorString(e));
    return VSPEC_B200_ERR_CUDA;
}

/* Copies `tokens` token rows (stride floats each) from src to the device pool
 * at element offset dst_off, converting to fp16 when asked; synchronous. */
static int vb_put_rows(const float* src, size_t tokens, size_t stride, int kv_dtype, void* d_pool, size_t dst_off,
                       cudaStream_t st, void** scratch, size_t* scratch_cap) {
    const size_t n = tokens * stride;
    if (n == 0) return VSPEC_B200_OK;
    cudaError_t e;
    if (kv_dtype == VSPEC_B200_KV_F32) {
        e = cudaMemcpyAsync((float*)d_pool + dst_off, src, n * sizeof(float), cudaMemcpyHostToDevice, st);
    } else {
        if (*scratch_cap < n * 2) {
            void* p = realloc(*scratch, n * 2);
            if (!p) { vb_set_error("out of host memory (%zu bytes)", n * 2); return VSPEC_B200_ERR_NOMEM; }
            *scratch = p;
            *scratch_cap = n * 2;
        }
        uint16_t* h = (uint16_t*)*scratch;
        for (size_t i = 0; i < n; ++i) h[i] = vb_f32_to_f16(src[i]);
        e = cudaMemcpyAsync((uint16_t*)d_pool + dst_off, h, n * 2, cudaMemcpyHostToDevice, st);
    }
    if (e != cudaSuccess) return vb_cuda_err(e, "cudaMemcpyAsync (paged KV upload)");
    e = cudaStreamSynchronize(st);   /* the conversion buffer is reused by the next run */
    if (e != cudaSuccess) return vb_cuda_err(e, "cudaStreamSynchronize (paged KV upload)");
    return VSPEC_B200_OK;
}

int vspec_b200_kv_paged_sync(const void* cache_ptr, int kv_dtype, void* d_k_pages, void* d_v_pages,
                             uint64_t since_step, uint64_t* out_step, void* stream) {
    const VspecKVPagedCache* c = (const VspecKVPagedCache*)cache_ptr;
    if (!c || !d_k_pages || !d_v_pages || !c->key_pages || !c->value_pages ||
        (kv_dtype != VSPEC_B200_KV_F32 && kv_dtype != VSPEC_B200_KV_F16) || c->max_pages > VSPEC_KV_PAGED_MAX_PAGES) {
        vb_set_error("bad vspec_b200_kv_paged_sync arguments");
        return VSPEC_B200_ERR_ARG;
    }
    cudaStream_t st = (cudaStream_t)stream;
    const size_t stride = c->num_heads * c->head_dim;
    const size_t span = c->page_tokens * stride;
    void* scratch = NULL;
    size_t cap = 0;
    int rc = VSPEC_B200_OK;
    /* runs of consecutive allocated pages touched after since_step, one copy per run and pool */
    size_t p = 0;
    while (p < c->max_pages && rc == VSPEC_B200_OK) {
        if (!(c->page_meta[p].allocated && c->page_meta[p].last_touch_step > since_step)) { ++p; continue; }
        size_t q = p + 1;
        while (q < c->max_pages && c->page_meta[q].allocated && c->page_meta[q].last_touch_step > since_step) ++q;
        rc = vb_put_rows(c->key_pages + p * span, (q - p) * c->page_tokens, stride, kv_dtype, d_k_pages, p * span,
                         st, &scratch, &cap);
        if (rc == VSPEC_B200_OK)
            rc = vb_put_rows(c->value_pages + p * span, (q - p) * c->page_tokens, stride, kv_dtype, d_v_pages,
                             p * span, st, &scratch, &cap);
        p = q;
    }
    free(scratch);
    if (rc == VSPEC_B200_OK && out_step) *out_step = c->clock_step;
    return rc;
}

int vspec_b200_kv_paged_session_view(const void* cache_ptr, uint64_t session_id, int kv_dtype, void* d_k_pages,
                                     void* d_v_pages, size_t spare_first, size_t spare_count,
                                     int32_t* d_page_table_row, size_t max_pages_per_seq, int32_t* d_ctx_len,
                                     size_t* out_ctx, size_t* out_spare_used, void* stream) {
    const VspecKVPagedCache* c = (const VspecKVPagedCache*)cache_ptr;
    if (!c || !d_page_table_row || !d_ctx_len || max_pages_per_seq == 0 || c->page_tokens == 0 ||
        (kv_dtype != VSPEC_B200_KV_F32 && kv_dtype != VSPEC_B200_KV_F16) || c->max_pages > VSPEC_KV_PAGED_MAX_PAGES) {
        vb_set_error("bad vspec_b200_kv_paged_session_view arguments");
        return VSPEC_B200_ERR_ARG;
    }
    /* the session, found as vspec_find_session_slot does (kv_paged_cache.c:13-24) */
    int slot = -1;
    for (size_t i = 0; session_id != 0 && i < VSPEC_KV_PAGED_MAX_SESSIONS; ++i)
        if (c->sessions[i].active && c->sessions[i].session_id == session_id) { slot = (int)i; break; }
    if (slot < 0) {
        vb_set_error("session %llu is not active in the paged cache", (unsigned long long)session_id);
        return VSPEC_B200_ERR_ARG;
    }
    const size_t pt = c->page_tokens;
    const size_t npg = c->sessions[slot].page_count;
    const uint16_t* pages = c->sessions[slot].pages;
    size_t tokens = 0;
    for (size_t i = 0; i < npg; ++i) {
        if (pages[i] >= c->max_pages) {
            vb_set_error("session %llu lists page %u beyond max_pages %zu", (unsigned long long)session_id,
                         (unsigned)pages[i], c->max_pages);
            return VSPEC_B200_ERR_ARG;
        }
        tokens += c->page_meta[pages[i]].used_tokens;
    }
    /* pages before the first short one (not the last) map through */
    size_t direct = 0;
    while (direct + 1 < npg && c->page_meta[pages[direct]].used_tokens == pt) ++direct;
    if (direct + 1 == npg || npg == 0) direct = npg;
    /* spare pages for the tokens from the first short page on */
    const size_t need = direct == npg ? 0 : (tokens - direct * pt + pt - 1) / pt;
    if ((tokens + pt - 1) / pt > max_pages_per_seq || direct + need > max_pages_per_seq) {
        vb_set_error("session %llu holds %zu tokens: more than max_pages_per_seq %zu pages", (unsigned long long)session_id,
                     tokens, max_pages_per_seq);
        return VSPEC_B200_ERR_ARG;
    }
    if (need > spare_count || (need > 0 && (spare_first < c->max_pages || !d_k_pages || !d_v_pages))) {
        vb_set_error("session %llu needs %zu spare device pages beyond max_pages (got %zu at %zu)",
                     (unsigned long long)session_id, need, spare_count, spare_first);
        return VSPEC_B200_ERR_ARG;
    }
    cudaStream_t st = (cudaStream_t)stream;
    int32_t* row = (int32_t*)calloc(max_pages_per_seq, sizeof(int32_t));
    if (!row) { vb_set_error("out of host memory"); return VSPEC_B200_ERR_NOMEM; }
    for (size_t i = 0; i < direct; ++i) row[i] = (int32_t)pages[i];
    int rc = VSPEC_B200_OK;
    if (need > 0) {
        /* the remaining tokens in get_token_ptr order, packed page by page */
        const size_t stride = c->num_heads * c->head_dim;
        const size_t span = pt * stride;
        float* kbuf = (float*)malloc(need * span * sizeof(float));
        float* vbuf = (float*)malloc(need * span * sizeof(float));
        void* scratch = NULL;
        size_t cap = 0;
        if (!kbuf || !vbuf) {
            vb_set_error("out of host memory");
            rc = VSPEC_B200_ERR_NOMEM;
        } else {
            memset(kbuf, 0, need * span * sizeof(float));
            memset(vbuf, 0, need * span * sizeof(float));
            size_t t = 0;
            for (size_t i = direct; i < npg; ++i) {
                const size_t used = c->page_meta[pages[i]].used_tokens;
                memcpy(kbuf + t * stride, c->key_pages + (size_t)pages[i] * span, used * stride * sizeof(float));
                memcpy(vbuf + t * stride, c->value_pages + (size_t)pages[i] * span, used * stride * sizeof(float));
                t += used;
            }
            for (size_t j = 0; j < need; ++j) row[direct + j] = (int32_t)(spare_first + j);
            rc = vb_put_rows(kbuf, need * pt, stride, kv_dtype, d_k_pages, spare_first * span, st, &scratch, &cap);
            if (rc == VSPEC_B200_OK)
                rc = vb_put_rows(vbuf, need * pt, stride, kv_dtype, d_v_pages, spare_first * span, st, &scratch, &cap);
        }
        free(kbuf);
        free(vbuf);
        free(scratch);
    }
    if (rc == VSPEC_B200_OK) {
        const int32_t ctx = (int32_t)tokens;
        cudaError_t e = cudaMemcpyAsync(d_page_table_row, row, max_pages_per_seq * sizeof(int32_t),
                                        cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = cudaMemcpyAsync(d_ctx_len, &ctx, sizeof(int32_t), cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);   /* row and ctx live on this stack frame */
        if (e != cudaSuccess) rc = vb_cuda_err(e, "page-table upload");
    }
    free(row);
    if (rc == VSPEC_B200_OK) {
        if (out_ctx) *out_ctx = tokens;
        if (out_spare_used) *out_spare_used = need;
    }
    return rc;
}
