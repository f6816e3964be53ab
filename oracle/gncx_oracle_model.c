/*
 * gncx_oracle_model.c -- CPU oracle for whole-model decode/prefill.
 *
 * TEST INFRASTRUCTURE ONLY.  LuaJIT is not available, so the reference's
 * orchestrator (lua/gncx_streamer.lua) cannot run; this file restates its
 * forward_token (:759-965), prefill (:968-1208), sample (:1229-1273) and
 * generate (:1276-1311) for the Qwen3/Llama and Gemma(1/2) architectures,
 * calling kernels through a table that is bound either to the reference's
 * own compiled library (dlopen of oracle/_ref/*.so, the strongest pin) or to
 * the C restatement in gncx_oracle.c.  Gemma-4 extras (per-layer embeddings,
 * sliding-window layer pattern, KV sharing, post-norms) are not restated.
 */
#include "gncx_oracle.h"
#include "gncx_oracle_model.h"

#include <dlfcn.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* Kernel signatures exactly as the reference exports them (include order of
 * csrc/gncx_llm_kernels.cpp:693-2052). */
typedef void (*fn_matvec)(const uint8_t*, size_t, int32_t, const float*, const void*, int32_t, int32_t,
                          float*, void*);
typedef void (*fn_matbatch)(const uint8_t*, size_t, int32_t, const float*, int32_t, int32_t, int32_t,
                            float*, void*);
typedef void (*fn_rmsnorm)(const float*, const uint8_t*, size_t, int32_t, float, int32_t, float*, void*,
                           float*);
typedef void (*fn_rmsnorm_heads)(float*, const uint8_t*, size_t, int32_t, int32_t, int32_t, float);
typedef void (*fn_rope)(float*, float*, void*, const uint8_t*, size_t, int32_t, int32_t, int32_t, int32_t,
                        int32_t, float);
typedef void (*fn_attn)(const float*, const float*, const float*, float*, float*, int32_t, int32_t,
                        int32_t, int32_t, float, int32_t, int32_t, float*);
typedef void (*fn_glu)(const float*, const float*, int32_t, float*);
typedef void (*fn_lm_head)(const uint8_t*, size_t, int32_t, const float*, int32_t, int32_t, float, float*);
typedef void (*fn_embed)(const uint8_t*, size_t, int32_t, int32_t, float, float*);

typedef struct {
    fn_matvec matvec;
    fn_matbatch matbatch;
    fn_rmsnorm rmsnorm;
    fn_rmsnorm_heads rmsnorm_heads;
    fn_rope rope;
    fn_attn attn;
    fn_glu swiglu, geglu;
    fn_lm_head lm_head;
    fn_embed embed_q8_0, embed_q6_k, embed_bf16;
} kernel_table;

/* ---- adapters: oracle kernels behind the reference signatures ---------- */

static void a_matvec(const uint8_t* b, size_t off, int32_t t, const float* x, const void* tok, int32_t in,
                     int32_t out, float* y, void* tel) {
    (void)tok; (void)tel;
    orc_matvec(b + off, t, x, in, out, y);
}
static void a_matbatch(const uint8_t* b, size_t off, int32_t t, const float* x, int32_t B, int32_t in,
                       int32_t out, float* y, void* tel) {
    (void)tel;
    orc_matbatch(b + off, t, x, B, in, out, y);
}
static void a_rmsnorm(const float* x, const uint8_t* b, size_t off, int32_t dim, float eps, int32_t lk,
                      float* out, void* tok, float* qs) {
    (void)lk; (void)tok;
    orc_rmsnorm(x, (const float*)(b + off), dim, eps, out);
    if (qs) *qs = 1.0f;
}
static void a_rmsnorm_heads(float* v, const uint8_t* b, size_t off, int32_t has_w, int32_t nh, int32_t hd,
                            float eps) {
    orc_rmsnorm_heads(v, has_w ? (const float*)(b + off) : NULL, nh, hd, eps);
}
static void a_rope(float* q, float* k, void* tok, const uint8_t* b, size_t off, int32_t has_rf, int32_t nh,
                   int32_t nkv, int32_t hd, int32_t pos, float base) {
    (void)tok;
    orc_rope(q, k, has_rf ? (const float*)(b + off) : NULL, nh, nkv, hd, pos, base);
}
static void a_lm_head(const uint8_t* b, size_t off, int32_t t, const float* h, int32_t dim, int32_t vocab,
                      float cap, float* y) {
    orc_lm_head(b + off, t, h, dim, vocab, cap, y);
}
static void a_embed_q8_0(const uint8_t* b, size_t off, int32_t tok, int32_t dim, float s, float* out) {
    orc_embed_row(b + off, 8, tok, dim, s, out);
}
static void a_embed_q6_k(const uint8_t* b, size_t off, int32_t tok, int32_t dim, float s, float* out) {
    orc_embed_row(b + off, 14, tok, dim, s, out);
}
static void a_embed_bf16(const uint8_t* b, size_t off, int32_t tok, int32_t dim, float s, float* out) {
    orc_embed_row(b + off, 30, tok, dim, s, out);
}

static int bind_oracle(kernel_table* k) {
    k->matvec = a_matvec;
    k->matbatch = a_matbatch;
    k->rmsnorm = a_rmsnorm;
    k->rmsnorm_heads = a_rmsnorm_heads;
    k->rope = a_rope;
    k->attn = orc_attention_step;
    k->swiglu = orc_swiglu;
    k->geglu = orc_geglu;
    k->lm_head = a_lm_head;
    k->embed_q8_0 = a_embed_q8_0;
    k->embed_q6_k = a_embed_q6_k;
    k->embed_bf16 = a_embed_bf16;
    return 0;
}

static int bind_library(kernel_table* k, const char* path) {
    void* h = dlopen(path, RTLD_NOW | RTLD_LOCAL);
    if (!h) {
        fprintf(stderr, "oracle: dlopen(%s): %s\n", path, dlerror());
        return -1;
    }
#define SYM(field, name) do { *(void**)&k->field = dlsym(h, name); if (!k->field) return -2; } while (0)
    SYM(matvec, "gncx_xfold_universal_matvec");
    SYM(matbatch, "gncx_xfold_universal_matbatch");
    SYM(rmsnorm, "gncx_rmsnorm_and_encode_4phase");
    SYM(rmsnorm_heads, "gncx_rmsnorm_inplace_heads");
    SYM(rope, "gncx_apply_rope_xor11_ext");
    SYM(attn, "gncx_mqa_attention_step_ext");
    SYM(swiglu, "gncx_swiglu_activation");
    SYM(geglu, "gncx_geglu_activation");
    SYM(lm_head, "gncx_universal_lm_head_logits");
    SYM(embed_q8_0, "gncx_fetch_token_embedding_q8_0");
    SYM(embed_q6_k, "gncx_fetch_token_embedding_q6_k");
    SYM(embed_bf16, "gncx_fetch_token_embedding_bf16");
#undef SYM
    /* The reference fills its fp16 table and starts its thread pool only in
     * gncx_gla_map_readonly (csrc/gncx_llm_kernels.cpp:327-329); without that
     * call every block scale reads as 0.  The mapping is deliberately never
     * unmapped: gncx_gla_unmap shuts the pool down (:392). */
    void* (*map)(const char*, size_t*) = (void* (*)(const char*, size_t*))dlsym(h, "gncx_gla_map_readonly");
    if (!map) return -3;
    size_t sz = 0;
    if (!map(path, &sz)) return -4;
    return 0;
}

/* ---- model state -------------------------------------------------------- */

typedef struct {
    orc_model_desc d;
    kernel_table k;
    void* (*ram_alloc)(size_t); /* the bound library's arena calls (lib_memory), else NULL: */
    uint8_t* (*ram_get_ptr)(void*); /* alloc returns a handle, get_ptr its memory */
    void (*ram_free)(void*);
    void* ram_handle[32];          /* live arena blocks and their memory */
    float* ram_ptr[32];
    uint64_t* off;
    int32_t* typ;
    int32_t q_dim, kv_dim;
    float *hidden, *normed, *q, *kb, *vb, *attn, *proj, *gate, *up, *act, *logits;
    float *kc, *vc; /* [n_layers][max_seq][kv_dim] */
} model;

#define OFF(m, l, t) ((m)->off[(size_t)(l) * ORC_NT + (t)])
#define TYP(m, l, t) ((m)->typ[(size_t)(l) * ORC_NT + (t)])
#define HAS(m, l, t) (OFF(m, l, t) != UINT64_MAX)

static float* vec_alloc(model* m, size_t n) {
    if (!m->ram_alloc) return (float*)calloc(n, 4);
    for (int i = 0; i < 32; ++i) {
        if (m->ram_handle[i]) continue;
        void* h = m->ram_alloc(n * 4);
        float* p = h ? (float*)m->ram_get_ptr(h) : NULL;
        if (!p) return NULL;
        memset(p, 0, n * 4);
        m->ram_handle[i] = h;
        m->ram_ptr[i] = p;
        return p;
    }
    return NULL;
}
static void vec_free(model* m, float* p) {
    if (!p) return;
    if (!m->ram_free) {
        free(p);
        return;
    }
    for (int i = 0; i < 32; ++i)
        if (m->ram_ptr[i] == p) {
            m->ram_free(m->ram_handle[i]);
            m->ram_handle[i] = NULL;
            m->ram_ptr[i] = NULL;
            return;
        }
}

void* orc_model_create(const orc_model_desc* desc, const char* ref_lib) { return orc_model_create_ex(desc, ref_lib, 0); }

void* orc_model_create_ex(const orc_model_desc* desc, const char* ref_lib, int32_t lib_memory) {
    model* m = (model*)calloc(1, sizeof(model));
    m->d = *desc;
    if (ref_lib ? bind_library(&m->k, ref_lib) : bind_oracle(&m->k)) {
        free(m);
        return NULL;
    }
    if (lib_memory) {
        void* h = ref_lib ? dlopen(ref_lib, RTLD_NOW | RTLD_LOCAL) : NULL;  /* the handle bind_library holds */
        if (h) {
            *(void**)&m->ram_alloc = dlsym(h, "gncx_ram_alloc");
            *(void**)&m->ram_get_ptr = dlsym(h, "gncx_ram_get_ptr");
            *(void**)&m->ram_free = dlsym(h, "gncx_ram_free");
        }
        if (!m->ram_alloc || !m->ram_get_ptr || !m->ram_free) {
            free(m);
            return NULL;
        }
    }
    const size_t nt = (size_t)desc->n_layers * ORC_NT;
    m->off = (uint64_t*)malloc(nt * sizeof(uint64_t));
    m->typ = (int32_t*)malloc(nt * sizeof(int32_t));
    memcpy(m->off, desc->off, nt * sizeof(uint64_t));
    memcpy(m->typ, desc->typ, nt * sizeof(int32_t));
    m->d.off = m->off;
    m->d.typ = m->typ;
    m->q_dim = desc->n_heads * desc->head_dim;
    m->kv_dim = desc->n_kv * desc->head_dim;
    const int32_t dim = desc->dim;
    const int32_t big = dim > m->q_dim ? dim : m->q_dim;
    m->hidden = vec_alloc(m, (size_t)dim);
    m->normed = vec_alloc(m, (size_t)big);
    m->q = vec_alloc(m, (size_t)m->q_dim);
    m->kb = vec_alloc(m, (size_t)m->kv_dim);
    m->vb = vec_alloc(m, (size_t)m->kv_dim);
    m->attn = vec_alloc(m, (size_t)m->q_dim);
    m->proj = vec_alloc(m, (size_t)dim);
    m->gate = vec_alloc(m, (size_t)desc->ffn_dim);
    m->up = vec_alloc(m, (size_t)desc->ffn_dim);
    m->act = vec_alloc(m, (size_t)desc->ffn_dim);
    m->logits = vec_alloc(m, (size_t)desc->vocab);
    const size_t kvn = (size_t)desc->n_layers * desc->max_seq * m->kv_dim;
    m->kc = vec_alloc(m, kvn);
    m->vc = vec_alloc(m, kvn);
    if (!m->kc || !m->vc) {
        orc_model_destroy(m);
        return NULL;
    }
    return m;
}

void orc_model_destroy(void* h) {
    model* m = (model*)h;
    if (!m) return;
    free(m->off); free(m->typ);
    float* v[] = {m->hidden, m->normed, m->q, m->kb, m->vb, m->attn, m->proj, m->gate, m->up, m->act, m->logits,
                  m->kc, m->vc};
    for (size_t i = 0; i < sizeof(v) / sizeof(v[0]); ++i) vec_free(m, v[i]);
    free(m);
}

static float* kcache(model* m, int32_t l) { return m->kc + (size_t)l * m->d.max_seq * m->kv_dim; }
static float* vcache(model* m, int32_t l) { return m->vc + (size_t)l * m->d.max_seq * m->kv_dim; }

/* lua/gncx_streamer.lua:698-713: Qwen/Llama scale 1.0, Gemma sqrt(dim) (Lua double, passed as float). */
static void fetch_embedding(model* m, int32_t tok, float* dst) {
    const float scale = m->d.arch == ORC_ARCH_GEMMA ? (float)sqrt((double)m->d.dim) : 1.0f;
    const int32_t t = m->d.tok_embd_type;
    if (t == 8) m->k.embed_q8_0(m->d.base, m->d.tok_embd_off, tok, m->d.dim, scale, dst);
    else if (t == 14) m->k.embed_q6_k(m->d.base, m->d.tok_embd_off, tok, m->d.dim, scale, dst);
    else m->k.embed_bf16(m->d.base, m->d.tok_embd_off, tok, m->d.dim, scale, dst);
}

static float attn_scale(const model* m) { return (float)(1.0 / sqrt((double)m->d.head_dim)); }

/* lua/gncx_streamer.lua:759-965 */
const float* orc_model_forward(void* h, int32_t tok, int32_t pos) {
    model* m = (model*)h;
    const orc_model_desc* d = &m->d;
    if (pos >= d->max_seq) return NULL;
    const uint8_t* B = d->base;
    fetch_embedding(m, tok, m->hidden);
    for (int32_t l = 0; l < d->n_layers; ++l) {
        m->k.rmsnorm(m->hidden, B, OFF(m, l, T_ATTN_NORM), d->dim, d->eps, 0, m->normed, NULL, NULL);
        m->k.matvec(B, OFF(m, l, T_Q), TYP(m, l, T_Q), m->normed, NULL, d->dim, m->q_dim, m->q, NULL);
        m->k.matvec(B, OFF(m, l, T_K), TYP(m, l, T_K), m->normed, NULL, d->dim, m->kv_dim, m->kb, NULL);
        m->k.matvec(B, OFF(m, l, T_V), TYP(m, l, T_V), m->normed, NULL, d->dim, m->kv_dim, m->vb, NULL);
        if (d->arch == ORC_ARCH_QWEN) {
            if (HAS(m, l, T_Q_NORM))
                m->k.rmsnorm_heads(m->q, B, OFF(m, l, T_Q_NORM), 1, d->n_heads, d->head_dim, d->eps);
            if (HAS(m, l, T_K_NORM))
                m->k.rmsnorm_heads(m->kb, B, OFF(m, l, T_K_NORM), 1, d->n_kv, d->head_dim, d->eps);
        }
        m->k.rope(m->q, m->kb, NULL, NULL, 0, 0, d->n_heads, d->n_kv, d->head_dim, pos, d->rope_base);
        m->k.attn(m->q, m->kb, m->vb, kcache(m, l), vcache(m, l), pos, d->n_heads, d->n_kv, d->head_dim,
                  attn_scale(m), 0, 1, m->attn);
        m->k.matvec(B, OFF(m, l, T_O), TYP(m, l, T_O), m->attn, NULL, m->q_dim, d->dim, m->proj, NULL);
        for (int32_t i = 0; i < d->dim; ++i) m->hidden[i] = m->hidden[i] + m->proj[i];
        m->k.rmsnorm(m->hidden, B, OFF(m, l, T_FFN_NORM), d->dim, d->eps, 0, m->normed, NULL, NULL);
        m->k.matvec(B, OFF(m, l, T_GATE), TYP(m, l, T_GATE), m->normed, NULL, d->dim, d->ffn_dim, m->gate, NULL);
        m->k.matvec(B, OFF(m, l, T_UP), TYP(m, l, T_UP), m->normed, NULL, d->dim, d->ffn_dim, m->up, NULL);
        if (d->arch == ORC_ARCH_GEMMA) m->k.geglu(m->gate, m->up, d->ffn_dim, m->act);
        else m->k.swiglu(m->gate, m->up, d->ffn_dim, m->act);
        m->k.matvec(B, OFF(m, l, T_DOWN), TYP(m, l, T_DOWN), m->act, NULL, d->ffn_dim, d->dim, m->proj, NULL);
        for (int32_t i = 0; i < d->dim; ++i) m->hidden[i] = m->hidden[i] + m->proj[i];
    }
    m->k.rmsnorm(m->hidden, B, d->out_norm_off, d->dim, d->eps, 0, m->normed, NULL, NULL);
    m->k.lm_head(B, d->tok_embd_off, d->tok_embd_type, m->normed, d->dim, d->vocab, d->softcap, m->logits);
    return m->logits;
}

/* lua/gncx_streamer.lua:968-1208 */
const float* orc_model_prefill(void* h, const int32_t* ids, int32_t n) {
    model* m = (model*)h;
    const orc_model_desc* d = &m->d;
    if (n <= 0) return NULL;
    if (n == 1) return orc_model_forward(h, ids[0], 0);
    const uint8_t* B = d->base;
    const int32_t dim = d->dim, qd = m->q_dim, kvd = m->kv_dim, fd = d->ffn_dim;
    float* bh = vec_alloc(m, (size_t)n * dim);
    float* bn = vec_alloc(m, (size_t)n * dim);
    float* bq = vec_alloc(m, (size_t)n * qd);
    float* bk = vec_alloc(m, (size_t)n * kvd);
    float* bv = vec_alloc(m, (size_t)n * kvd);
    float* ba = vec_alloc(m, (size_t)n * qd);
    float* bp = vec_alloc(m, (size_t)n * dim);
    float* bg = vec_alloc(m, (size_t)n * fd);
    float* bu = vec_alloc(m, (size_t)n * fd);
    float* bf = vec_alloc(m, (size_t)n * fd);
    for (int32_t t = 0; t < n; ++t) fetch_embedding(m, ids[t], bh + (size_t)t * dim);
    for (int32_t l = 0; l < d->n_layers; ++l) {
        for (int32_t t = 0; t < n; ++t)
            m->k.rmsnorm(bh + (size_t)t * dim, B, OFF(m, l, T_ATTN_NORM), dim, d->eps, 0, bn + (size_t)t * dim,
                         NULL, NULL);
        m->k.matbatch(B, OFF(m, l, T_Q), TYP(m, l, T_Q), bn, n, dim, qd, bq, NULL);
        m->k.matbatch(B, OFF(m, l, T_K), TYP(m, l, T_K), bn, n, dim, kvd, bk, NULL);
        m->k.matbatch(B, OFF(m, l, T_V), TYP(m, l, T_V), bn, n, dim, kvd, bv, NULL);
        for (int32_t t = 0; t < n; ++t) {
            float* qp = bq + (size_t)t * qd;
            float* kp = bk + (size_t)t * kvd;
            float* vp = bv + (size_t)t * kvd;
            if (d->arch == ORC_ARCH_QWEN) {
                if (HAS(m, l, T_Q_NORM))
                    m->k.rmsnorm_heads(qp, B, OFF(m, l, T_Q_NORM), 1, d->n_heads, d->head_dim, d->eps);
                if (HAS(m, l, T_K_NORM))
                    m->k.rmsnorm_heads(kp, B, OFF(m, l, T_K_NORM), 1, d->n_kv, d->head_dim, d->eps);
            }
            m->k.rope(qp, kp, NULL, NULL, 0, 0, d->n_heads, d->n_kv, d->head_dim, t, d->rope_base);
            m->k.attn(qp, kp, vp, kcache(m, l), vcache(m, l), t, d->n_heads, d->n_kv, d->head_dim,
                      attn_scale(m), 0, 1, ba + (size_t)t * qd);
        }
        m->k.matbatch(B, OFF(m, l, T_O), TYP(m, l, T_O), ba, n, qd, dim, bp, NULL);
        for (size_t i = 0; i < (size_t)n * dim; ++i) bh[i] = bh[i] + bp[i];
        for (int32_t t = 0; t < n; ++t)
            m->k.rmsnorm(bh + (size_t)t * dim, B, OFF(m, l, T_FFN_NORM), dim, d->eps, 0, bn + (size_t)t * dim,
                         NULL, NULL);
        m->k.matbatch(B, OFF(m, l, T_GATE), TYP(m, l, T_GATE), bn, n, dim, fd, bg, NULL);
        m->k.matbatch(B, OFF(m, l, T_UP), TYP(m, l, T_UP), bn, n, dim, fd, bu, NULL);
        if (d->arch == ORC_ARCH_GEMMA) m->k.geglu(bg, bu, n * fd, bf);
        else m->k.swiglu(bg, bu, n * fd, bf);
        m->k.matbatch(B, OFF(m, l, T_DOWN), TYP(m, l, T_DOWN), bf, n, fd, dim, bp, NULL);
        for (size_t i = 0; i < (size_t)n * dim; ++i) bh[i] = bh[i] + bp[i];
    }
    memcpy(m->hidden, bh + (size_t)(n - 1) * dim, (size_t)dim * 4);
    float* tmp[] = {bh, bn, bq, bk, bv, ba, bp, bg, bu, bf};
    for (size_t i = 0; i < sizeof(tmp) / sizeof(tmp[0]); ++i) vec_free(m, tmp[i]);
    m->k.rmsnorm(m->hidden, B, d->out_norm_off, dim, d->eps, 0, m->normed, NULL, NULL);
    m->k.lm_head(B, d->tok_embd_off, d->tok_embd_type, m->normed, dim, d->vocab, d->softcap, m->logits);
    return m->logits;
}

/* lua/gncx_streamer.lua:1276-1311, with the tokenizer replaced by token ids.
 * Returns the number of tokens written to out_ids. */
int32_t orc_model_generate(void* h, const int32_t* prompt, int32_t n_prompt, int32_t max_new, double penalty,
                           int32_t eos_id, int32_t* out_ids) {
    model* m = (model*)h;
    if (n_prompt <= 0) return 0;
    const float* logits = orc_model_prefill(h, prompt, n_prompt);
    int32_t* all = (int32_t*)malloc(((size_t)n_prompt + max_new + 1) * 4);
    memcpy(all, prompt, (size_t)n_prompt * 4);
    int32_t n_all = n_prompt, n_out = 0, cur = n_prompt;
    for (int32_t step = 0; step < max_new; ++step) {
        if (cur >= m->d.max_seq || !logits) break;
        const int32_t nxt = orc_sample_greedy(logits, m->d.vocab, all, n_all, penalty);
        if (nxt == eos_id) break;
        out_ids[n_out++] = nxt;
        all[n_all++] = nxt;
        logits = orc_model_forward(h, nxt, cur);
        cur++;
    }
    free(all);
    return n_out;
}

const float* orc_model_logits(void* h) { return ((model*)h)->logits; }
const float* orc_model_kcache(void* h, int32_t layer) { return kcache((model*)h, layer); }
