/* qwen_decode.c -- Qwen3-shape low-bit decode loop on the B200 kernels
 * (Qwen3-8B and Qwen3-32B layer shapes; the reference's GenericTransformerRuntime
 * ._forward_token, Vspec-chat/python/runtime_inference.py:1245-1500, Qwen
 * profile).
 *
 * One decode step for a batch of sequences, all on one stream:
 *   x = embed(tok)
 *   per layer:  qkv = Wqkv . RMSNorm(x)                   (fused RMSNorm)
 *               q, k = per-head RMSNorm + rotary(pos); k, v -> paged KV
 *               a = paged GQA attention(q, KV[0..pos])
 *               x = x + Wo . a                             (fused residual)
 *               h = SwiGLU(Wgate_up . RMSNorm(x))         (fused RMSNorm, SwiGLU)
 *               x = x + Wdown . h                          (fused residual)
 *   logits = Wlm . RMSNorm(x); tok = prompt token or greedy argmax; pos += 1
 * Positions, context lengths and tokens stay on the device, so the step is
 * captured once as a CUDA graph and replayed for every position (prompt
 * prefill and generation alike); the host only waits at the end.
 * The residual stabilisation of the reference is the identity for this
 * profile (residual_clamp_alpha = 0, runtime_inference.py:162-171).
 *
 * Tensor parallelism (tp > 1, one GPU per rank): each rank keeps its slice of
 * the query/key/value heads and of the gate/up rows (column parallel) and the
 * matching input columns of the o-proj and down projections (row parallel);
 * the partial products of those two are summed by an in-place NCCL
 * all-reduce, rank 0 alone adding the residual.  Embedding and lm_head are
 * replicated, so every rank computes the same logits and tokens.
 * NCCL is resolved at run time, when the first tensor-parallel model is made
 * (an NCCL already loaded into the process is reused, VSPEC_B200_NCCL_LIB
 * names another), so single-GPU users never load it. */
#include <dlfcn.h>
#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>
#include <nccl.h>

#include "vspec_b200.h"

typedef struct QwenLayer {
    uint8_t *w_qkv, *w_o, *w_gu, *w_down;
    void *s_qkv, *s_o, *s_gu, *s_down;
    void *k_pages, *v_pages;
} QwenLayer;

typedef struct QwenModel {
    VspecB200QwenConfig cfg;
    int bits_attn, bits_mlp;
    int tp, rank;
    ncclComm_t comm;
    int max_batch, max_ctx, pages_per_seq, num_pages;
    int hq, hkv, q_dim, qkv_n, inter;   /* this rank's heads, q width, qkv rows, intermediate slice */
    void* emb;              /* fp16 [vocab][hidden] */
    QwenLayer* layers;
    uint8_t* w_lm;
    void* s_lm;
    float* ones;            /* norm weights (all ones), max(hidden, intermediate slice, head_dim) */
    float *x, *qkv, *q, *attn, *h, *logits;
    int32_t *tok, *pos, *ctx_len, *page_table, *prompt, *prompt_len, *out_tokens;
    void* nt_state;         /* next-token reduction state, zero between steps */
    int max_prompt, max_steps;
    cudaStream_t stream;
    cudaGraphExec_t exec;
    int graph_batch;
} QwenModel;

static size_t row_bytes(int k, int bits) { return ((size_t)k * (size_t)bits + 7) / 8; }

/* The NCCL entry points the decode loop uses. */
typedef struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*);
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int);
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*comm_destroy)(ncclComm_t);
} NcclApi;

static NcclApi g_nccl;
static int g_nccl_ok;
static pthread_once_t g_nccl_once = PTHREAD_ONCE_INIT;

static void nccl_load(void) {
    const char* name = getenv("VSPEC_B200_NCCL_LIB");
    void* h = NULL;
    if (name && *name) {
        h = dlopen(name, RTLD_NOW | RTLD_GLOBAL);
    } else {
        h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    }
    if (!h) return;
    *(void**)&g_nccl.get_unique_id = dlsym(h, "ncclGetUniqueId");
    *(void**)&g_nccl.comm_init_rank = dlsym(h, "ncclCommInitRank");
    *(void**)&g_nccl.all_reduce = dlsym(h, "ncclAllReduce");
    *(void**)&g_nccl.comm_destroy = dlsym(h, "ncclCommDestroy");
    g_nccl_ok = g_nccl.get_unique_id && g_nccl.comm_init_rank && g_nccl.all_reduce && g_nccl.comm_destroy;
}

static const NcclApi* nccl_api(void) {
    pthread_once(&g_nccl_once, nccl_load);
    return g_nccl_ok ? &g_nccl : NULL;
}

static int cuda_ok(cudaError_t e) { return e == cudaSuccess; }

static int alloc_dev(void** p, size_t bytes) {
    *p = NULL;
    if (bytes == 0) return 1;
    return cuda_ok(cudaMalloc(p, bytes));
}

static int alloc_linear(QwenModel* m, uint8_t** w, void** s, int n, int k, int bits) {
    return alloc_dev((void**)w, (size_t)n * row_bytes(k, bits)) &&
           alloc_dev(s, (size_t)n * (size_t)(k / m->cfg.group) * 2);
}

/* Random-init linear: codes uniform, fp16 scales ~U(0.003, 0.006), which with
 * the mid-range zero-point gives weights of std ~0.02.  Writes rows
 * [row0, row0 + rows) of the whole [*][k_global] tensor, restricted to input
 * columns [k0, k0 + k_local), at local row `lrow` of a [*][k_local] shard.
 * Every element takes the random stream of its place in the whole tensor
 * (byte index row * row_bytes(k_global) + byte, scale index row * groups +
 * group), so shards hold exactly the unsharded model's values.  k0 is a whole
 * number of scale groups, so the sliced LSB-first bitstream starts on a byte. */
static int fill_rows(QwenModel* m, uint8_t* w, void* s, int bits, int lrow, int rows, int row0, int k_local,
                     int k_global, int k0, uint64_t seed) {
    const int g = m->cfg.group;
    const size_t lrb = row_bytes(k_local, bits), grb = row_bytes(k_global, bits);
    const size_t lg = (size_t)(k_local / g), gg = (size_t)(k_global / g);
    if (vspec_b200_random_fill_block(w + (size_t)lrow * lrb, (size_t)rows, lrb, lrb, 0, seed, grb, (size_t)row0,
                                     row_bytes(k0, bits), 0.f, 0.f, m->stream) != VSPEC_B200_OK)
        return 0;
    return vspec_b200_random_fill_block((uint8_t*)s + (size_t)lrow * lg * 2, (size_t)rows, lg, lg, 1,
                                        seed ^ 0x5ca1eull, gg, (size_t)row0, (size_t)(k0 / g), 0.003f, 0.006f,
                                        m->stream) == VSPEC_B200_OK;
}

static int linear(QwenModel* m, const float* x, const uint8_t* w, const void* s, float* y, int batch, int n, int k,
                  int bits, int flags, const float* residual, const float* norm_w) {
    VspecB200LinearArgs a;
    memset(&a, 0, sizeof(a));
    a.d_x = x;
    a.d_w = w;
    a.d_scales = s;
    a.d_zero_points = NULL;
    a.zero_point_const = 0.0f;   /* unsigned reading: code = u - 2^(bits-1), i.e. mid-range zero-point */
    a.d_y = y;
    a.d_residual = residual;
    a.d_norm_weight = norm_w;
    a.norm_eps = m->cfg.rms_eps;
    a.m = (size_t)batch;
    a.n = (size_t)n;
    a.k = (size_t)k;
    a.n_groups = (size_t)(k / m->cfg.group);
    a.bits = bits;
    a.flags = flags | VSPEC_B200_F_SZ_F16 | VSPEC_B200_F_UNSIGNED;
    return vspec_b200_lowbit_linear(&a, m->stream);
}

/* x = sum over the ranks of the row-parallel partials, in place. */
static int allreduce_x(QwenModel* m, int batch) {
    if (m->tp == 1) return VSPEC_B200_OK;
    if (nccl_api()->all_reduce(m->x, m->x, (size_t)batch * (size_t)m->cfg.hidden, ncclFloat, ncclSum, m->comm,
                               m->stream) != ncclSuccess)
        return VSPEC_B200_ERR_CUDA;
    return VSPEC_B200_OK;
}

/* One decode step (enqueue only). */
static int enqueue_step(QwenModel* m, int batch) {
    const VspecB200QwenConfig* c = &m->cfg;
    /* rank 0 adds the residual to its row-parallel partial, the others write theirs */
    const int res_flag = m->rank == 0 ? VSPEC_B200_F_RESIDUAL : 0;
    const float* res = m->rank == 0 ? m->x : NULL;
    int rc = vspec_b200_decode_embed(m->emb, m->tok, batch, c->hidden, m->x, m->stream);
    if (rc != VSPEC_B200_OK) return rc;
    for (int l = 0; l < c->num_layers; ++l) {
        QwenLayer* L = &m->layers[l];
        rc = linear(m, m->x, L->w_qkv, L->s_qkv, m->qkv, batch, m->qkv_n, c->hidden, m->bits_attn,
                    VSPEC_B200_F_RMSNORM, NULL, m->ones);
        if (rc != VSPEC_B200_OK) return rc;
        rc = vspec_b200_decode_qk_rope_append(m->qkv, m->ones, m->ones, m->pos, batch, m->hq, m->hkv, c->head_dim,
                                              c->rms_eps, c->rope_theta, m->q, L->k_pages, L->v_pages, m->page_table,
                                              m->pages_per_seq, c->page_tokens, m->ctx_len, m->stream);
        if (rc != VSPEC_B200_OK) return rc;
        VspecB200PagedAttnArgs pa;
        memset(&pa, 0, sizeof(pa));
        pa.d_q = m->q;
        pa.d_k_pages = L->k_pages;
        pa.d_v_pages = L->v_pages;
        pa.d_page_table = m->page_table;
        pa.d_ctx_len = m->ctx_len;
        pa.d_out = m->attn;
        pa.batch = (size_t)batch;
        pa.num_q_heads = (size_t)m->hq;
        pa.num_kv_heads = (size_t)m->hkv;
        pa.head_dim = (size_t)c->head_dim;
        pa.page_tokens = (size_t)c->page_tokens;
        pa.max_pages_per_seq = (size_t)m->pages_per_seq;
        pa.num_pages = (size_t)m->num_pages;
        pa.max_ctx = (size_t)m->max_ctx;
        pa.scale = 1.0f / sqrtf((float)c->head_dim);
        pa.kv_dtype = VSPEC_B200_KV_F16;
        rc = vspec_b200_paged_attention(&pa, m->stream);
        if (rc != VSPEC_B200_OK) return rc;
        rc = linear(m, m->attn, L->w_o, L->s_o, m->x, batch, c->hidden, m->q_dim, m->bits_attn, res_flag, res, NULL);
        if (rc == VSPEC_B200_OK) rc = allreduce_x(m, batch);
        if (rc != VSPEC_B200_OK) return rc;
        rc = linear(m, m->x, L->w_gu, L->s_gu, m->h, batch, 2 * m->inter, c->hidden, m->bits_mlp,
                    VSPEC_B200_F_RMSNORM | VSPEC_B200_F_SWIGLU, NULL, m->ones);
        if (rc != VSPEC_B200_OK) return rc;
        rc = linear(m, m->h, L->w_down, L->s_down, m->x, batch, c->hidden, m->inter, m->bits_mlp, res_flag, res, NULL);
        if (rc == VSPEC_B200_OK) rc = allreduce_x(m, batch);
        if (rc != VSPEC_B200_OK) return rc;
    }
    rc = linear(m, m->x, m->w_lm, m->s_lm, m->logits, batch, c->vocab, c->hidden, m->bits_attn, VSPEC_B200_F_RMSNORM,
                NULL, m->ones);
    if (rc != VSPEC_B200_OK) return rc;
    return vspec_b200_decode_next_token(m->logits, batch, c->vocab, c->logit_clip, m->prompt, m->prompt_len,
                                        m->max_prompt, m->pos, m->tok, m->out_tokens, m->max_steps, m->nt_state,
                                        m->stream);
}

void vspec_b200_qwen_destroy(void* model) {
    QwenModel* m = (QwenModel*)model;
    if (!m) return;
    if (m->stream) cudaStreamSynchronize(m->stream);
    /* the captured step holds NCCL calls: release it before the communicator */
    if (m->exec) cudaGraphExecDestroy(m->exec);
    if (m->comm) nccl_api()->comm_destroy(m->comm);
    if (m->layers) {
        for (int l = 0; l < m->cfg.num_layers; ++l) {
            QwenLayer* L = &m->layers[l];
            cudaFree(L->w_qkv); cudaFree(L->w_o); cudaFree(L->w_gu); cudaFree(L->w_down);
            cudaFree(L->s_qkv); cudaFree(L->s_o); cudaFree(L->s_gu); cudaFree(L->s_down);
            cudaFree(L->k_pages); cudaFree(L->v_pages);
        }
        free(m->layers);
    }
    cudaFree(m->emb); cudaFree(m->w_lm); cudaFree(m->s_lm); cudaFree(m->ones);
    cudaFree(m->x); cudaFree(m->qkv); cudaFree(m->q); cudaFree(m->attn); cudaFree(m->h); cudaFree(m->logits);
    cudaFree(m->tok); cudaFree(m->pos); cudaFree(m->ctx_len); cudaFree(m->page_table);
    cudaFree(m->prompt); cudaFree(m->prompt_len); cudaFree(m->out_tokens); cudaFree(m->nt_state);
    if (m->stream) cudaStreamDestroy(m->stream);
    free(m);
}

int vspec_b200_nccl_unique_id(void* out_id128) {
    if (!out_id128) return VSPEC_B200_ERR_ARG;
    const NcclApi* nc = nccl_api();
    if (!nc) return VSPEC_B200_ERR_UNSUPPORTED;
    ncclUniqueId id;
    if (nc->get_unique_id(&id) != ncclSuccess) return VSPEC_B200_ERR_CUDA;
    memset(out_id128, 0, 128);
    memcpy(out_id128, &id, sizeof(id) < 128 ? sizeof(id) : 128);
    return VSPEC_B200_OK;
}

int vspec_b200_qwen_create_tp(const VspecB200QwenConfig* cfg, uint64_t seed, int max_batch, int max_ctx, int tp_size,
                              int tp_rank, const void* nccl_id128, void** out_model) {
    if (!cfg || !out_model || max_batch <= 0 || max_ctx <= 0 || tp_size <= 0 || tp_rank < 0 || tp_rank >= tp_size ||
        (tp_size > 1 && !nccl_id128))
        return VSPEC_B200_ERR_ARG;
    *out_model = NULL;
    const VspecB200QwenConfig* c = cfg;
    const int T = tp_size, r = tp_rank;
    const int bits_mlp = c->bits_mlp ? c->bits_mlp : c->bits;
    if (c->num_layers <= 0 || c->hidden <= 0 || c->num_heads <= 0 || c->num_kv_heads <= 0 ||
        c->num_heads % c->num_kv_heads != 0 || c->head_dim <= 0 || c->head_dim % 64 != 0 || c->head_dim > 256 ||
        c->intermediate <= 0 || c->vocab <= 0 || c->group <= 0 || c->group % 128 != 0 || c->hidden % c->group != 0 ||
        (c->bits != 2 && c->bits != 3 && c->bits != 4) || (bits_mlp != 2 && bits_mlp != 3 && bits_mlp != 4) ||
        c->page_tokens <= 0 || c->num_heads % T != 0 || c->num_kv_heads % T != 0 || c->intermediate % T != 0 ||
        ((c->num_heads / T) * c->head_dim) % c->group != 0 || (c->intermediate / T) % c->group != 0)
        return VSPEC_B200_ERR_ARG;
    if (T > 1 && !nccl_api()) return VSPEC_B200_ERR_UNSUPPORTED;
    QwenModel* m = (QwenModel*)calloc(1, sizeof(QwenModel));
    if (!m) return VSPEC_B200_ERR_NOMEM;
    m->cfg = *cfg;
    m->bits_attn = c->bits;
    m->bits_mlp = bits_mlp;
    m->tp = T;
    m->rank = r;
    m->max_batch = max_batch;
    m->max_ctx = max_ctx;
    m->pages_per_seq = (max_ctx + c->page_tokens - 1) / c->page_tokens;
    m->num_pages = m->pages_per_seq * max_batch;
    m->hq = c->num_heads / T;
    m->hkv = c->num_kv_heads / T;
    m->q_dim = m->hq * c->head_dim;
    m->qkv_n = m->q_dim + 2 * m->hkv * c->head_dim;
    m->inter = c->intermediate / T;
    m->max_prompt = max_ctx;
    m->max_steps = max_ctx;
    int ok = cuda_ok(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
    if (ok && T > 1) {
        const NcclApi* nc = nccl_api();
        ncclUniqueId id;
        memcpy(&id, nccl_id128, sizeof(id) < 128 ? sizeof(id) : 128);
        ok = nc != NULL && nc->comm_init_rank(&m->comm, T, id, r) == ncclSuccess;
        if (!ok) m->comm = NULL;
    }
    m->layers = (QwenLayer*)calloc((size_t)c->num_layers, sizeof(QwenLayer));
    ok = ok && m->layers != NULL;
    const int gq = c->num_heads * c->head_dim, gkv = c->num_kv_heads * c->head_dim;   /* unsharded widths */
    const int lkv = m->hkv * c->head_dim;
    const int ba = m->bits_attn, bm = m->bits_mlp;
    const size_t page_elems = (size_t)m->num_pages * c->page_tokens * m->hkv * c->head_dim;
    for (int l = 0; ok && l < c->num_layers; ++l) {
        QwenLayer* L = &m->layers[l];
        const uint64_t ls = seed * 1000003ull + (uint64_t)l * 16ull;
        /* qkv: this rank's q, k and v head rows of the whole [q | k | v] */
        ok = alloc_linear(m, &L->w_qkv, &L->s_qkv, m->qkv_n, c->hidden, ba) &&
             fill_rows(m, L->w_qkv, L->s_qkv, ba, 0, m->q_dim, r * m->q_dim, c->hidden, c->hidden, 0, ls + 1) &&
             fill_rows(m, L->w_qkv, L->s_qkv, ba, m->q_dim, lkv, gq + r * lkv, c->hidden, c->hidden, 0, ls + 1) &&
             fill_rows(m, L->w_qkv, L->s_qkv, ba, m->q_dim + lkv, lkv, gq + gkv + r * lkv, c->hidden, c->hidden, 0,
                       ls + 1) &&
             /* o-proj: every row, this rank's input columns */
             alloc_linear(m, &L->w_o, &L->s_o, c->hidden, m->q_dim, ba) &&
             fill_rows(m, L->w_o, L->s_o, ba, 0, c->hidden, 0, m->q_dim, gq, r * m->q_dim, ls + 2) &&
             /* gate rows then up rows of this rank's intermediate slice */
             alloc_linear(m, &L->w_gu, &L->s_gu, 2 * m->inter, c->hidden, bm) &&
             fill_rows(m, L->w_gu, L->s_gu, bm, 0, m->inter, r * m->inter, c->hidden, c->hidden, 0, ls + 3) &&
             fill_rows(m, L->w_gu, L->s_gu, bm, m->inter, m->inter, c->intermediate + r * m->inter, c->hidden,
                       c->hidden, 0, ls + 3) &&
             /* down: every row, this rank's input columns */
             alloc_linear(m, &L->w_down, &L->s_down, c->hidden, m->inter, bm) &&
             fill_rows(m, L->w_down, L->s_down, bm, 0, c->hidden, 0, m->inter, c->intermediate, r * m->inter,
                       ls + 4) &&
             alloc_dev(&L->k_pages, page_elems * 2) && alloc_dev(&L->v_pages, page_elems * 2) &&
             cuda_ok(cudaMemsetAsync(L->k_pages, 0, page_elems * 2, m->stream)) &&
             cuda_ok(cudaMemsetAsync(L->v_pages, 0, page_elems * 2, m->stream));
    }
    const size_t emb_elems = (size_t)c->vocab * c->hidden;
    ok = ok && alloc_dev(&m->emb, emb_elems * 2) &&
         vspec_b200_random_fill(m->emb, emb_elems, 1, seed * 7919ull + 11ull, -0.05f, 0.05f, m->stream) == VSPEC_B200_OK;
    ok = ok && alloc_linear(m, &m->w_lm, &m->s_lm, c->vocab, c->hidden, ba) &&
         fill_rows(m, m->w_lm, m->s_lm, ba, 0, c->vocab, 0, c->hidden, c->hidden, 0, seed * 7919ull + 13ull);
    int ones_n = c->hidden > m->inter ? c->hidden : m->inter;
    if (c->head_dim > ones_n) ones_n = c->head_dim;
    ok = ok && alloc_dev((void**)&m->ones, (size_t)ones_n * 4) &&
         vspec_b200_random_fill(m->ones, (size_t)ones_n, 2, 0, 1.0f, 0.f, m->stream) == VSPEC_B200_OK;
    const size_t B = (size_t)max_batch;
    ok = ok && alloc_dev((void**)&m->x, B * c->hidden * 4) && alloc_dev((void**)&m->qkv, B * m->qkv_n * 4) &&
         alloc_dev((void**)&m->q, B * m->q_dim * 4) && alloc_dev((void**)&m->attn, B * m->q_dim * 4) &&
         alloc_dev((void**)&m->h, B * m->inter * 4) && alloc_dev((void**)&m->logits, B * c->vocab * 4) &&
         alloc_dev((void**)&m->tok, B * 4) && alloc_dev((void**)&m->pos, B * 4) && alloc_dev((void**)&m->ctx_len, B * 4) &&
         alloc_dev((void**)&m->page_table, B * m->pages_per_seq * 4) &&
         alloc_dev((void**)&m->prompt, B * m->max_prompt * 4) && alloc_dev((void**)&m->prompt_len, B * 4) &&
         alloc_dev((void**)&m->out_tokens, B * m->max_steps * 4) && alloc_dev(&m->nt_state, B * 16) &&
         cuda_ok(cudaMemsetAsync(m->nt_state, 0, B * 16, m->stream));
    if (ok) {
        /* page table: a seeded permutation of the pool (pages of one sequence
         * scattered over the pool, as a paged cache hands them out) */
        int32_t* perm = (int32_t*)malloc((size_t)m->num_pages * 4);
        ok = perm != NULL;
        if (ok) {
            for (int i = 0; i < m->num_pages; ++i) perm[i] = i;
            uint64_t st = seed ^ 0x9E3779B97F4A7C15ull;
            for (int i = m->num_pages - 1; i > 0; --i) {
                st = st * 6364136223846793005ull + 1442695040888963407ull;
                const int j = (int)((st >> 33) % (uint64_t)(i + 1));
                const int32_t t = perm[i]; perm[i] = perm[j]; perm[j] = t;
            }
            ok = cuda_ok(cudaMemcpyAsync(m->page_table, perm, (size_t)m->num_pages * 4, cudaMemcpyHostToDevice, m->stream)) &&
                 cuda_ok(cudaStreamSynchronize(m->stream));
            free(perm);
        }
    }
    ok = ok && cuda_ok(cudaStreamSynchronize(m->stream));
    if (!ok) {
        vspec_b200_qwen_destroy(m);
        return VSPEC_B200_ERR_CUDA;
    }
    *out_model = m;
    return VSPEC_B200_OK;
}

int vspec_b200_qwen_create(const VspecB200QwenConfig* cfg, uint64_t seed, int max_batch, int max_ctx,
                           void** out_model) {
    return vspec_b200_qwen_create_tp(cfg, seed, max_batch, max_ctx, 1, 0, NULL, out_model);
}

int vspec_b200_qwen_generate(void* model, int batch, const int32_t* h_prompts, int prompt_len, int gen_tokens,
                             int32_t* h_tokens_out, float* out_gen_ms, float* h_logits_out) {
    QwenModel* m = (QwenModel*)model;
    if (!m || !h_prompts || !h_tokens_out || batch <= 0 || batch > m->max_batch || prompt_len <= 0 || gen_tokens <= 0 ||
        prompt_len + gen_tokens > m->max_ctx)
        return VSPEC_B200_ERR_ARG;
    const int total = prompt_len + gen_tokens;
    const int steps = total - 1;
    const VspecB200QwenConfig* c = &m->cfg;
    int rc = VSPEC_B200_OK;
    /* state: prompts, positions 0, first token, context 0, recorded tokens */
    int32_t* hp = (int32_t*)calloc((size_t)batch * m->max_prompt, 4);
    int32_t* hl = (int32_t*)malloc((size_t)batch * 4);
    int32_t* first = (int32_t*)malloc((size_t)batch * 4);
    int32_t* outs = (int32_t*)calloc((size_t)batch * m->max_steps, 4);
    if (!hp || !hl || !first || !outs) { free(hp); free(hl); free(first); free(outs); return VSPEC_B200_ERR_NOMEM; }
    for (int b = 0; b < batch; ++b) {
        memcpy(hp + (size_t)b * m->max_prompt, h_prompts + (size_t)b * prompt_len, (size_t)prompt_len * 4);
        hl[b] = prompt_len;
        first[b] = h_prompts[(size_t)b * prompt_len];
        outs[(size_t)b * m->max_steps] = first[b];
    }
    int ok = cuda_ok(cudaMemcpyAsync(m->prompt, hp, (size_t)batch * m->max_prompt * 4, cudaMemcpyHostToDevice, m->stream)) &&
             cuda_ok(cudaMemcpyAsync(m->prompt_len, hl, (size_t)batch * 4, cudaMemcpyHostToDevice, m->stream)) &&
             cuda_ok(cudaMemcpyAsync(m->tok, first, (size_t)batch * 4, cudaMemcpyHostToDevice, m->stream)) &&
             cuda_ok(cudaMemsetAsync(m->pos, 0, (size_t)batch * 4, m->stream)) &&
             cuda_ok(cudaMemsetAsync(m->ctx_len, 0, (size_t)batch * 4, m->stream)) &&
             cuda_ok(cudaMemcpyAsync(m->out_tokens, outs, (size_t)batch * m->max_steps * 4, cudaMemcpyHostToDevice, m->stream));
    if (!ok) rc = VSPEC_B200_ERR_CUDA;
    /* step 0 runs eagerly: it sets up every workspace and kernel attribute
     * before the graph is captured */
    if (rc == VSPEC_B200_OK) rc = enqueue_step(m, batch);
    if (rc == VSPEC_B200_OK && h_logits_out &&
        !cuda_ok(cudaMemcpyAsync(h_logits_out, m->logits, (size_t)batch * c->vocab * 4, cudaMemcpyDeviceToHost, m->stream)))
        rc = VSPEC_B200_ERR_CUDA;
    if (rc == VSPEC_B200_OK && !cuda_ok(cudaStreamSynchronize(m->stream))) rc = VSPEC_B200_ERR_CUDA;
    if (rc == VSPEC_B200_OK && steps > 1 && (m->graph_batch != batch || !m->exec)) {
        if (m->exec) { cudaGraphExecDestroy(m->exec); m->exec = NULL; }
        cudaGraph_t g = NULL;
        if (!cuda_ok(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal))) {
            rc = VSPEC_B200_ERR_CUDA;
        } else {
            const int erc = enqueue_step(m, batch);
            const cudaError_t ce = cudaStreamEndCapture(m->stream, &g);
            if (erc != VSPEC_B200_OK) rc = erc;
            else if (ce != cudaSuccess || !g || !cuda_ok(cudaGraphInstantiate(&m->exec, g, 0))) rc = VSPEC_B200_ERR_CUDA;
            if (g) cudaGraphDestroy(g);
        }
        if (rc == VSPEC_B200_OK) m->graph_batch = batch;
    }
    cudaEvent_t e0 = NULL, e1 = NULL;
    if (rc == VSPEC_B200_OK && (!cuda_ok(cudaEventCreate(&e0)) || !cuda_ok(cudaEventCreate(&e1)))) rc = VSPEC_B200_ERR_CUDA;
    /* steps 1 .. steps-1; the generation phase is the last gen_tokens steps
     * (steps prompt_len-1 .. total-2) */
    const int gen_first = prompt_len - 1;
    if (rc == VSPEC_B200_OK && gen_first == 0 && !cuda_ok(cudaEventRecord(e0, m->stream))) rc = VSPEC_B200_ERR_CUDA;
    for (int s = 1; rc == VSPEC_B200_OK && s < steps; ++s) {
        if (s == gen_first && !cuda_ok(cudaEventRecord(e0, m->stream))) { rc = VSPEC_B200_ERR_CUDA; break; }
        if (!cuda_ok(cudaGraphLaunch(m->exec, m->stream))) { rc = VSPEC_B200_ERR_CUDA; break; }
        if (h_logits_out &&
            !cuda_ok(cudaMemcpyAsync(h_logits_out + (size_t)s * batch * c->vocab, m->logits, (size_t)batch * c->vocab * 4,
                                     cudaMemcpyDeviceToHost, m->stream))) { rc = VSPEC_B200_ERR_CUDA; break; }
    }
    if (rc == VSPEC_B200_OK && !cuda_ok(cudaEventRecord(e1, m->stream))) rc = VSPEC_B200_ERR_CUDA;
    if (rc == VSPEC_B200_OK) {
        ok = cuda_ok(cudaMemcpyAsync(outs, m->out_tokens, (size_t)batch * m->max_steps * 4, cudaMemcpyDeviceToHost, m->stream)) &&
             cuda_ok(cudaStreamSynchronize(m->stream));
        if (!ok) rc = VSPEC_B200_ERR_CUDA;
    }
    if (rc == VSPEC_B200_OK) {
        for (int b = 0; b < batch; ++b) memcpy(h_tokens_out + (size_t)b * total, outs + (size_t)b * m->max_steps, (size_t)total * 4);
        if (out_gen_ms) {
            float ms = 0.f;
            cudaEventElapsedTime(&ms, e0, e1);
            *out_gen_ms = ms;
        }
    }
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    free(hp); free(hl); free(first); free(outs);
    return rc;
}

size_t vspec_b200_qwen_tensor(void* model, int kind, int layer, void* h_dst) {
    QwenModel* m = (QwenModel*)model;
    if (!m) return 0;
    const VspecB200QwenConfig* c = &m->cfg;
    const void* src = NULL;
    size_t bytes = 0;
    const int g = c->group;
    const int ba = m->bits_attn, bm = m->bits_mlp;
    if (kind == 0) { src = m->emb; bytes = (size_t)c->vocab * c->hidden * 2; }
    else if (kind == 9) { src = m->w_lm; bytes = (size_t)c->vocab * row_bytes(c->hidden, ba); }
    else if (kind == 10) { src = m->s_lm; bytes = (size_t)c->vocab * (c->hidden / g) * 2; }
    else if (kind >= 1 && kind <= 8 && layer >= 0 && layer < c->num_layers) {
        const QwenLayer* L = &m->layers[layer];
        switch (kind) {
            case 1: src = L->w_qkv; bytes = (size_t)m->qkv_n * row_bytes(c->hidden, ba); break;
            case 2: src = L->s_qkv; bytes = (size_t)m->qkv_n * (c->hidden / g) * 2; break;
            case 3: src = L->w_o; bytes = (size_t)c->hidden * row_bytes(m->q_dim, ba); break;
            case 4: src = L->s_o; bytes = (size_t)c->hidden * (m->q_dim / g) * 2; break;
            case 5: src = L->w_gu; bytes = (size_t)2 * m->inter * row_bytes(c->hidden, bm); break;
            case 6: src = L->s_gu; bytes = (size_t)2 * m->inter * (c->hidden / g) * 2; break;
            case 7: src = L->w_down; bytes = (size_t)c->hidden * row_bytes(m->inter, bm); break;
            default: src = L->s_down; bytes = (size_t)c->hidden * (m->inter / g) * 2; break;
        }
    }
    if (!src) return 0;
    if (h_dst) {
        if (!cuda_ok(cudaMemcpyAsync(h_dst, src, bytes, cudaMemcpyDeviceToHost, m->stream)) ||
            !cuda_ok(cudaStreamSynchronize(m->stream)))
            return 0;
    }
    return bytes;
}
