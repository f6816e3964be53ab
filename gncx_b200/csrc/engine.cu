// engine.cu -- the model engine: GGUF load + upload in native block layout,
// decode step (forward_token + greedy sample) and batched prefill on one GPU.
//
// It restates the reference orchestrator lua/gncx_streamer.lua (forward_token
// :759-965, prefill :968-1208, sample :1229-1273, generate :1276-1311) for the
// Qwen3 / Llama / Gemma(1,2) decoder families, with the arithmetic of each step
// done by this library's kernels.  What changes is where things live:
//   * weights: one HBM arena, tensors in their GGUF block layout; q/k/v rows and
//     gate/up rows are placed back to back when their types match, so each pair
//     (triple) is one GEMV;
//   * per-token state (input token, position, penalty window, output ids) is in
//     device memory, so a whole decode step -- embedding, 36 layers, LM head,
//     argmax -- is one captured CUDA graph launch with no host round trip;
//   * the KV cache is fp32 like the reference's, laid out head-major
//     [n_kv][max_seq][head_dim] so a run of positions of one head is contiguous
//     (one bulk copy per attention chunk);
//   * tensor parallel (one process per GPU): q/k/v with the attention heads,
//     gate/up and the LM head are split by output rows, so each output
//     element is computed whole on one GPU in the 1-GPU order and the token
//     stream is the same.  Decode all-gathers (tp.cu) the attention output
//     and the GLU output, then every rank computes all of attn_output and
//     ffn_down (two exchanges per layer, at those two boundaries); prefill,
//     which is compute-bound, splits those two by rows as well and gathers
//     their results.  The logits are gathered once per token.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <map>
#include <string>
#include <vector>

#include "kernels.h"
#include <nvtx3/nvToolsExt.h>

namespace gncx {

// ---------------------------------------------------------------- GGUF (lua/gncx_gguf.lua:223-306)
struct GgufTensor {
    std::vector<uint64_t> dims;
    int32_t type = 0;
    uint64_t abs_off = 0;
    uint64_t nbytes = 0;
};

struct Gguf {
    int fd = -1;
    const uint8_t* base = nullptr;
    size_t size = 0;
    std::map<std::string, double> num;
    std::map<std::string, std::string> str;
    std::map<std::string, uint64_t> arr_len;
    std::map<std::string, GgufTensor> tensors;
    ~Gguf() {
        if (base) munmap(const_cast<uint8_t*>(base), size);
        if (fd >= 0) close(fd);
    }
};

struct Cursor {
    const uint8_t* p;
    const uint8_t* end;
    bool ok = true;
    template <class T>
    T get() {
        T v{};
        if (p + sizeof(T) > end) { ok = false; return v; }
        memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string string() {
        const uint64_t n = get<uint64_t>();
        if (!ok || p + n > end) { ok = false; return {}; }
        std::string s(reinterpret_cast<const char*>(p), n);
        p += n;
        return s;
    }
};

static bool skip_value(Cursor& c, uint32_t t, double* num_out, std::string* str_out, uint64_t* arr_n) {
    switch (t) {
        case 0: { const double v = c.get<uint8_t>(); if (num_out) *num_out = v; return c.ok; }
        case 1: { const double v = c.get<int8_t>(); if (num_out) *num_out = v; return c.ok; }
        case 2: { const double v = c.get<uint16_t>(); if (num_out) *num_out = v; return c.ok; }
        case 3: { const double v = c.get<int16_t>(); if (num_out) *num_out = v; return c.ok; }
        case 4: { const double v = c.get<uint32_t>(); if (num_out) *num_out = v; return c.ok; }
        case 5: { const double v = c.get<int32_t>(); if (num_out) *num_out = v; return c.ok; }
        case 6: { const double v = c.get<float>(); if (num_out) *num_out = v; return c.ok; }
        case 7: { const double v = c.get<uint8_t>(); if (num_out) *num_out = v; return c.ok; }
        case 8: { std::string s = c.string(); if (str_out) *str_out = s; return c.ok; }
        case 9: {
            const uint32_t et = c.get<uint32_t>();
            const uint64_t n = c.get<uint64_t>();
            if (arr_n) *arr_n = n;
            for (uint64_t i = 0; i < n && c.ok; ++i) skip_value(c, et, nullptr, nullptr, nullptr);
            return c.ok;
        }
        case 10: { const double v = (double)c.get<uint64_t>(); if (num_out) *num_out = v; return c.ok; }
        case 11: { const double v = (double)c.get<int64_t>(); if (num_out) *num_out = v; return c.ok; }
        case 12: { const double v = c.get<double>(); if (num_out) *num_out = v; return c.ok; }
        default: c.ok = false; return false;
    }
}

static bool gguf_open(const char* path, Gguf& g, std::string& err) {
    g.fd = open(path, O_RDONLY);
    if (g.fd < 0) { err = "cannot open model file"; return false; }
    struct stat st {};
    fstat(g.fd, &st);
    g.size = (size_t)st.st_size;
    void* m = mmap(nullptr, g.size, PROT_READ, MAP_PRIVATE, g.fd, 0);
    if (m == MAP_FAILED) { err = "mmap failed"; return false; }
    g.base = static_cast<const uint8_t*>(m);
    Cursor c{g.base, g.base + g.size};
    if (g.size < 24 || memcmp(g.base, "GGUF", 4) != 0) { err = "not a GGUF file"; return false; }
    c.p += 4;
    (void)c.get<uint32_t>();  // version
    const uint64_t n_tensors = c.get<uint64_t>();
    const uint64_t n_kv = c.get<uint64_t>();
    for (uint64_t i = 0; i < n_kv && c.ok; ++i) {
        const std::string key = c.string();
        const uint32_t t = c.get<uint32_t>();
        double num = 0;
        std::string s;
        uint64_t an = 0;
        skip_value(c, t, &num, &s, &an);
        if (t == 8) g.str[key] = s;
        else if (t == 9) g.arr_len[key] = an;
        else g.num[key] = num;
    }
    std::vector<std::pair<std::string, GgufTensor>> recs;
    for (uint64_t i = 0; i < n_tensors && c.ok; ++i) {
        std::string name = c.string();
        GgufTensor tr;
        const uint32_t nd = c.get<uint32_t>();
        for (uint32_t d = 0; d < nd; ++d) tr.dims.push_back(c.get<uint64_t>());
        tr.type = (int32_t)c.get<uint32_t>();
        tr.abs_off = c.get<uint64_t>();  // relative for now
        recs.emplace_back(std::move(name), std::move(tr));
    }
    if (!c.ok) { err = "truncated GGUF header"; return false; }
    uint64_t align = 32;
    auto it = g.num.find("general.alignment");
    if (it != g.num.end() && it->second > 0) align = (uint64_t)it->second;
    const uint64_t hdr = (uint64_t)(c.p - g.base);
    const uint64_t data = (hdr + align - 1) / align * align;
    for (auto& r : recs) {
        uint64_t n = 1;
        for (auto d : r.second.dims) n *= d;
        const int be = block_elems(r.second.type), bb = block_bytes(r.second.type);
        r.second.nbytes = bb ? (n / be) * (uint64_t)bb : 0;
        r.second.abs_off += data;
        if (r.second.abs_off + r.second.nbytes > g.size) { err = "tensor data past end of file: " + r.first; return false; }
        g.tensors[r.first] = r.second;
    }
    return true;
}

// ---------------------------------------------------------------- engine
struct LayerW {
    const float *attn_norm = nullptr, *ffn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
    const uint8_t *wq = nullptr, *wk = nullptr, *wv = nullptr, *wo = nullptr, *wg = nullptr, *wu = nullptr, *wd = nullptr;
    int tq = 0, tk = 0, tv = 0, to = 0, tg = 0, tu = 0, td = 0;
    bool qkv_fused = false, gu_fused = false;
    float *kc = nullptr, *vc = nullptr;
};

struct Engine {
    // hyper-parameters (lua/gncx_streamer.lua:344-441)
    int arch = 0;  // 0 qwen, 1 llama, 2 gemma
    int n_layers = 0, dim = 0, nh = 0, nkv = 0, hd = 0, ffn = 0, vocab = 0, max_seq = 0, q_dim = 0, kv_dim = 0;
    float eps = 1e-6f, rope_base = 10000.0f, softcap = 0.0f, attn_scale = 0.0f, embd_scale = 1.0f;
    int eos = -1;
    bool qk_norm = false;
    // this rank's share under tensor parallelism (the whole model when tp.size == 1)
    TpComm tp;
    int nh_l = 0, nkv_l = 0, qd_l = 0, kvd_l = 0, ffn_l = 0, dim_l = 0, voc0 = 0, voc_l = 0;
    size_t x_q = 0, x_p = 0, x_f = 0, x_l = 0;  // gather buffers (byte offsets in the exchange region)
    size_t ll_q = 0, ll_f = 0, ll_l = 0;        // one-row (decode) staging areas of the same gathers
    size_t ll_p = 0;                             // one-row staging of the out-split attn_output / ffn_down
    size_t ll_am = 0;                            // the greedy step's (value, id) swap: size x 16 bytes
    bool tp_outsplit = false;  // decode splits attn_output / ffn_down by rows too (GNCX_TP_OUTSPLIT=1)
    int x_rows = 0;                              // rows each gather buffer holds
    const uint8_t* tok_embd = nullptr;
    int embd_type = 0;
    const float* out_norm = nullptr;
    std::vector<LayerW> L;
    uint8_t* arena = nullptr;
    size_t arena_bytes = 0;
    float* kv = nullptr;
    float *rope_c = nullptr, *rope_s = nullptr;
    // decode buffers
    float *hidden = nullptr, *proj = nullptr, *qkv = nullptr, *gu = nullptr, *logits = nullptr, *normed = nullptr;
    float* logits_own = nullptr;  // logits buffer of a 1-GPU engine (tp: the gather buffer)
    uint8_t *act_d = nullptr, *act_q = nullptr, *act_f = nullptr;  // staged activation vectors
    float* part = nullptr;
    int max_splits = 0;
    bool exact = false;      // exact serial softmax in attention
    float* scores = nullptr; // [n_heads][max_splits * chunk] (decode, exact mode)
    int graph_exact = -1;
    DecodeState* st = nullptr;
    DecodeState* st_host = nullptr;  // pinned staging
    int32_t* out_ids = nullptr;
    int out_cap = 0;
    void* am_scratch = nullptr;
    int32_t* d_err = nullptr;
    int32_t* ids_dev = nullptr;
    int ids_cap = 0;
    cudaStream_t stream = nullptr;
    cudaGraphExec_t graph = nullptr;
    double penalty_graph = -1.0;
    cudaEvent_t ev[4] = {};
    double prefill_ms = 0.0, decode_ms = 0.0;
    int decode_steps = 0;
    std::string error;
    // prefill buffers (grown on demand)
    int pf_cap = 0;
    float *pf_h = nullptr, *pf_p = nullptr, *pf_qkv = nullptr, *pf_gu = nullptr, *pf_part = nullptr;
    float* pf_scores = nullptr;
    size_t pf_score_cap = 0;
    ActBlock *pf_act = nullptr, *pf_actq = nullptr, *pf_actf = nullptr;
    size_t pf_part_floats = 0;
    // persistent decode step (decode_step.cu): one launch for the layer stack
    bool step_ok = false;
    StepPlan step{};
    StepLayer* step_layers = nullptr;
    float *step_attn = nullptr, *step_proj = nullptr, *step_glu = nullptr, *step_part = nullptr;
    float* step_scores = nullptr;
    unsigned* step_sync = nullptr;
    size_t step_sync_bytes = 0;
};

// Positions per attention split in decode: 128 where the chunk's K/V rows fit
// shared memory (head_dim <= 128; 8B shape: 2.16 vs 2.20 ms/token at 64), else 64.
static int decode_chunk(int hd) {
    static const int force = getenv("GNCX_ATTN_CHUNK") ? atoi(getenv("GNCX_ATTN_CHUNK")) : 0;  // tuning override
    if (force == 32 || force == 64 || force == 128) return hd <= 128 || force < 128 ? force : 64;
    return hd <= 128 ? 128 : 64;
}
static constexpr int kPrefillChunk = 64;   // positions per chunk of the causal prefill attention kernel
static constexpr int kPrefillGroup = 256;  // prompt positions per attention launch in prefill
static constexpr int kTpMaxRows = 4096;    // prompt rows a tensor-parallel prefill gathers at once

#define CK(x)                                             \
    do {                                                  \
        const int _st = (x);                              \
        if (_st != kOk) return _st;                       \
    } while (0)
#define CU(x)                                             \
    do {                                                  \
        if ((x) != cudaSuccess) return kErrCuda;          \
    } while (0)

static int gemv(Engine* e, const uint8_t* w, int t, const uint8_t* act, const float* x, int in, int out, float* y,
                float cap = 0.0f) {
    return gemv_launch(w, t, t == kBF16 ? x : nullptr, t == kBF16 ? nullptr : act, in, out, y, cap, e->d_err,
                       e->stream);
}

// Rows [r0, r1) of `n` split over `tp` ranks in pieces of `unit` rows (the last
// rank takes what remains).
static void split_rows(int n, int tp, int rank, int unit, int& r0, int& r1) {
    const int per = ((n + tp - 1) / tp + unit - 1) / unit * unit;
    r0 = rank * per < n ? rank * per : n;
    r1 = r0 + per < n ? r0 + per : n;
}

static int gather(Engine* e, size_t buf, int rows, int row_floats, int off, int len);
static int gather_row(Engine* e, int slot);

// LM head over this rank's vocabulary rows of the staged act_d, then (tensor
// parallel, when the caller needs every logit) the all-gather that gives
// every rank all of them.
static int lm_head(Engine* e, bool gather_logits = true) {
    const uint8_t* w = e->tok_embd + (size_t)e->voc0 * row_bytes(e->embd_type, e->dim);
    CK(gemv(e, w, e->embd_type, e->act_d, e->normed, e->dim, e->voc_l, e->logits + e->voc0, e->softcap));
    return gather_logits ? gather_row(e, 2) : kOk;  // the logits slot of the one-row gathers
}


// A decode GEMV whose output y (dim rows) is the residual of the next norm:
// hidden += y, then RMSNorm with gains `norm_w` into the staged act_d (and
// normed).  The norm is its own one-CTA kernel: under programmatic dependent
// launch it is resident and waiting while the GEMV finishes, and the next
// GEMV's CTAs stream their weights while it runs.  (Running the norm in the
// GEMV's last CTA instead -- an arrival counter per launch -- measured 0.24
// ms/token slower: every CTA's exit then waits for a fence and an atomic, so
// the next kernel's CTAs start streaming later.)
static int gemv_norm(Engine* e, const uint8_t* w, int t, const uint8_t* act, const float* x, int in, float* y,
                     const float* norm_w) {
    const int D = e->dim;
    if (act && t != kBF16) CK(gemv_launch(w, t, nullptr, act, in, D, y, 0.0f, e->d_err, e->stream));
    else CK(gemv_launch(w, t, x, nullptr, in, D, y, 0.0f, e->d_err, e->stream));
    return add_norm_quant_launch(e->hidden, y, norm_w, 1, D, e->eps, ActOut{nullptr, e->act_d}, e->normed,
                                 e->stream);
}

// Split-KV decode attention through the partial + combine kernels instead of
// the register-streaming kernel (A/B override).
static bool attn_partial_env() {
    static const bool on = getenv("GNCX_ENGINE_ATTN_PARTIAL") != nullptr;
    return on;
}

static int gather(Engine* e, size_t buf, int rows, int row_floats, int off, int len) {
    return tp_gather_launch(e->tp, buf, rows, row_floats, off, len, e->d_err, e->stream);
}

// Decode's one-row gathers: attention output, GLU output, logits.
enum LlSlot { kLlAttn = 0, kLlGlu = 1, kLlLogits = 2, kLlProj = 3 };  // slot kTpLlSlots - 1: the argmax swap
static int gather_row(Engine* e, int slot) {
    TpSlices sl{};
    const int n = e->tp.size;
    size_t buf = 0, ll = 0;
    int row = 0;
    for (int q = 0; q < n; ++q) {
        if (slot == kLlAttn) { sl.off[q] = q * e->qd_l; sl.len[q] = e->qd_l; }
        else if (slot == kLlGlu) { sl.off[q] = q * e->ffn_l; sl.len[q] = e->ffn_l; }
        else if (slot == kLlProj) { sl.off[q] = q * e->dim_l; sl.len[q] = e->dim_l; }
        else { int v0, v1; split_rows(e->vocab, n, q, 4, v0, v1); sl.off[q] = v0; sl.len[q] = v1 - v0; }
    }
    if (slot == kLlAttn) { buf = e->x_q; ll = e->ll_q; row = e->q_dim; }
    else if (slot == kLlGlu) { buf = e->x_f; ll = e->ll_f; row = e->ffn; }
    else if (slot == kLlProj) { buf = e->x_p; ll = e->ll_p; row = e->dim; }
    else { buf = e->x_l; ll = e->ll_l; row = e->vocab; }
    return tp_gather_ll_launch(e->tp, buf, ll, row, sl, slot, e->d_err, e->stream);
}

// The LM head over the final norm in act_d and, if `sample`, the penalized
// greedy argmax that appends the next token and advances the position.
static int lm_head_and_sample(Engine* e, bool sample, double penalty) {
    cudaStream_t s = e->stream;
    if (sample && e->tp.size > 1) {
        // each rank takes the penalized maximum of its vocabulary slice and the
        // ranks swap (value, id) pairs: no logit crosses NVLink
        CK(lm_head(e, false));
        int32_t n_parts = 0;
        CK(argmax_partials_launch(e->logits + e->voc0, e->voc_l, e->voc0, e->st, penalty, e->am_scratch, &n_parts, s));
        CK(tp_argmax_state_launch(e->tp, e->ll_am, e->am_scratch, n_parts, e->st, e->out_ids, 1, e->d_err, s));
        return kOk;
    }
    CK(lm_head(e));
    if (sample) CK(argmax_state_launch(e->logits, e->vocab, e->st, penalty, e->out_ids, 1, e->am_scratch, s));
    return kOk;
}

// One decode step: forward(st->token at st->pos) and, if `sample`, the
// penalized argmax that appends the next token and advances the position.
static int decode_step(Engine* e, bool sample, double penalty) {
    cudaStream_t s = e->stream;
    const int D = e->dim, QD = e->q_dim, F = e->ffn;
    const int qd = e->qd_l, kvd = e->kvd_l, fl = e->ffn_l;
    const int qkv_w = qd + 2 * kvd;
    const bool tp = e->tp.size > 1;
    const int rk = e->tp.rank;
    float* gq = tp ? tp_buffer(e->tp, e->x_q) : nullptr;  // attention output (gathered)
    float* gf = tp ? tp_buffer(e->tp, e->x_f) : nullptr;  // GLU output (gathered)
    CK(dequant_launch(e->tok_embd, e->embd_type, 1, D, e->embd_scale, &e->st->token, e->hidden, s));
    if (e->step_ok && !tp) {
        // the whole layer stack as one persistent kernel; its counters start at zero
        StepPlan plan = e->step;
        plan.exact = e->exact ? 1 : 0;
        CU(cudaMemsetAsync(e->step_sync, 0, e->step_sync_bytes, s));
        CK(decode_step_launch(plan, s));
        return lm_head_and_sample(e, sample, penalty);
    }
    // layer 0's attention norm; every later norm runs in the epilogue of the
    // GEMV whose output it adds into the residual stream
    CK(add_norm_quant_launch(e->hidden, nullptr, e->L[0].attn_norm, 1, D, e->eps, ActOut{nullptr, e->act_d},
                             e->normed, s));
    for (int l = 0; l < e->n_layers; ++l) {
        const LayerW& w = e->L[l];
        const float* next_norm = l + 1 < e->n_layers ? e->L[l + 1].attn_norm : e->out_norm;
        if (w.qkv_fused) {
            CK(gemv(e, w.wq, w.tq, e->act_d, e->normed, D, qkv_w, e->qkv));
        } else {
            CK(gemv(e, w.wq, w.tq, e->act_d, e->normed, D, qd, e->qkv));
            CK(gemv(e, w.wk, w.tk, e->act_d, e->normed, D, kvd, e->qkv + qd));
            CK(gemv(e, w.wv, w.tv, e->act_d, e->normed, D, kvd, e->qkv + qd + kvd));
        }
        // the attention kernel itself norms and rotates q and the new K row and
        // writes the new K/V row to the cache (the Q/K post step, fused)
        AttnArgs a{};
        a.post_k = e->qkv + qd;
        a.post_v = e->qkv + qd + kvd;
        a.post_qn = w.q_norm;
        a.post_kn = w.k_norm;
        a.post_norm = e->qk_norm ? 1 : 0;
        a.post_eps = e->eps;
        a.rope_c = e->rope_c;
        a.rope_s = e->rope_s;
        a.q = e->qkv;
        a.q_stride = qkv_w;
        a.kc = w.kc;
        a.vc = w.vc;
        a.kv_pos_stride = e->hd;  // head-major cache: [n_kv][max_seq][head_dim]
        a.kv_head_stride = e->max_seq * e->hd;
        a.pos0 = 0;
        a.pos_dev = &e->st->pos;
        a.n_heads = e->nh_l;
        a.n_kv = e->nkv_l;
        a.hd = e->hd;
        a.scale = e->attn_scale;
        a.window = 0;
        a.chunk = decode_chunk(e->hd);
        a.max_splits = e->max_splits;
        a.part = e->part;
        if (tp) {
            a.out = gq + (size_t)rk * qd;  // this rank's heads of the gathered vector
            a.out_stride = QD;
            a.act_out = ActOut{nullptr, nullptr};
        } else {
            // the fp32 output replaces q and the O GEMV quantizes it (the
            // attention kernels that merge in-kernel write no act);
            // GNCX_ENGINE_ATTN_PARTIAL: split-KV through the partial + combine
            // kernels, the combine writing the act only
            a.out = e->exact || !attn_partial_env() ? e->qkv : nullptr;
            a.out_stride = qkv_w;
            a.act_out = a.out ? ActOut{nullptr, nullptr} : ActOut{nullptr, e->act_q};
        }
        a.prefetch_old = 1;  // cache rows below pos come from earlier tokens
        a.err = e->d_err;
        a.exact = e->exact ? 1 : 0;
        a.scores = e->scores;
        a.score_cap = e->max_splits * decode_chunk(e->hd);
        CK(attention_run(a, 1, s));
        if (tp && e->tp_outsplit) {  // gather the heads, this rank's attn_output rows, gather those
            CK(gather_row(e, kLlAttn));
            float* gpb = tp_buffer(e->tp, e->x_p);
            CK(gemv_launch(w.wo + (size_t)rk * e->dim_l * row_bytes(w.to, QD), w.to, gq, nullptr, QD, e->dim_l,
                           gpb + (size_t)rk * e->dim_l, 0.0f, e->d_err, s));
            CK(gather_row(e, kLlProj));
            CK(add_norm_quant_launch(e->hidden, gpb, w.ffn_norm, 1, D, e->eps, ActOut{nullptr, e->act_d}, e->normed,
                                     s));
        } else if (tp) {  // gather the heads, then the whole attn_output on every rank
            CK(gather_row(e, kLlAttn));
            CK(gemv_norm(e, w.wo, w.to, nullptr, gq, QD, e->proj, w.ffn_norm));
        } else if (e->exact || !attn_partial_env()) {
            CK(gemv_norm(e, w.wo, w.to, nullptr, e->qkv, QD, e->proj, w.ffn_norm));
        } else {
            CK(gemv_norm(e, w.wo, w.to, e->act_q, nullptr, QD, e->proj, w.ffn_norm));
        }
        if (w.gu_fused) {
            CK(gemv(e, w.wg, w.tg, e->act_d, e->normed, D, 2 * fl, e->gu));
        } else {
            CK(gemv(e, w.wg, w.tg, e->act_d, e->normed, D, fl, e->gu));
            CK(gemv(e, w.wu, w.tu, e->act_d, e->normed, D, fl, e->gu + fl));
        }
        if (tp) {
            CK(glu_quant_launch(e->gu, e->gu + fl, 2 * fl, fl, 1, e->arch == 2, ActOut{nullptr, nullptr}, s,
                                gf + (size_t)rk * fl, F));
            CK(gather_row(e, kLlGlu));
            if (e->tp_outsplit) {  // this rank's ffn_down rows, then every rank gathers them
                float* gpb = tp_buffer(e->tp, e->x_p);
                CK(gemv_launch(w.wd + (size_t)rk * e->dim_l * row_bytes(w.td, F), w.td, gf, nullptr, F, e->dim_l,
                               gpb + (size_t)rk * e->dim_l, 0.0f, e->d_err, s));
                CK(gather_row(e, kLlProj));
                CK(add_norm_quant_launch(e->hidden, gpb, next_norm, 1, D, e->eps, ActOut{nullptr, e->act_d},
                                         e->normed, s));
            } else {
                CK(gemv_norm(e, w.wd, w.td, nullptr, gf, F, e->proj, next_norm));  // the whole ffn_down on every rank
            }
        } else {
            CK(glu_quant_launch(e->gu, e->gu + F, 2 * F, F, 1, e->arch == 2, ActOut{nullptr, e->act_f}, s));
            CK(gemv_norm(e, w.wd, w.td, e->act_f, nullptr, F, e->proj, next_norm));
        }
    }
    return lm_head_and_sample(e, sample, penalty);
}

static int ensure_prefill(Engine* e, int B) {
    if (B <= e->pf_cap) return kOk;
    if (e->tp.size > 1 && B > e->x_rows) return kErrCapacity;  // the gather buffers hold x_rows rows
    cudaStreamSynchronize(e->stream);
    cudaFree(e->pf_h); cudaFree(e->pf_p); cudaFree(e->pf_qkv); cudaFree(e->pf_gu); cudaFree(e->pf_part);
    cudaFree(e->pf_act); cudaFree(e->pf_actq); cudaFree(e->pf_actf); cudaFree(e->pf_scores);
    e->pf_scores = nullptr;
    e->pf_cap = 0;
    const size_t D = e->dim, QKV = e->qd_l + 2 * e->kvd_l, FL = e->ffn_l;
    const int grp = B < kPrefillGroup ? B : kPrefillGroup;
    const size_t splits = (size_t)(B + kPrefillChunk - 1) / kPrefillChunk;
    e->pf_part_floats = (size_t)grp * e->nh_l * splits * attn_record_floats(e->hd);
    if (cudaMalloc(&e->pf_h, (size_t)B * D * 4) || cudaMalloc(&e->pf_p, (size_t)B * D * 4) ||
        cudaMalloc(&e->pf_qkv, (size_t)B * QKV * 4) || cudaMalloc(&e->pf_gu, (size_t)B * 2 * FL * 4) ||
        cudaMalloc(&e->pf_part, e->pf_part_floats * 4) ||
        cudaMalloc(&e->pf_act, (size_t)B * (D / 32) * sizeof(ActBlock)) ||
        cudaMalloc(&e->pf_actq, (size_t)B * (e->q_dim / 32) * sizeof(ActBlock)) ||
        cudaMalloc(&e->pf_actf, (size_t)B * (e->ffn / 32) * sizeof(ActBlock)) ||
        cudaMalloc(&e->pf_scores, (size_t)grp * e->nh_l * splits * kPrefillChunk * 4)) {
        cudaGetLastError();
        return kErrOutOfMemory;
    }
    e->pf_score_cap = splits * kPrefillChunk;
    e->pf_cap = B;
    return kOk;
}

// lua/gncx_streamer.lua:968-1208 (B >= 2): every layer runs over all prompt
// positions at once; attention is causal per position (each position sees
// the positions <= its own, exactly what the reference's per-token loop does).
static int prefill_batch(Engine* e, int B) {
    cudaStream_t s = e->stream;
    const int D = e->dim, QD = e->q_dim, F = e->ffn;
    const int qd = e->qd_l, kvd = e->kvd_l, fl = e->ffn_l, dl = e->dim_l;
    const int qkv_w = qd + 2 * kvd;
    const bool tp = e->tp.size > 1;
    const int rk = e->tp.rank;
    CK(ensure_prefill(e, B));
    float* gq = tp ? tp_buffer(e->tp, e->x_q) : nullptr;
    float* gp = tp ? tp_buffer(e->tp, e->x_p) : e->pf_p;
    float* gf = tp ? tp_buffer(e->tp, e->x_f) : nullptr;
    CK(dequant_launch(e->tok_embd, e->embd_type, B, D, e->embd_scale, e->ids_dev, e->pf_h, s));
    for (int l = 0; l < e->n_layers; ++l) {
        const LayerW& w = e->L[l];
        CK(add_norm_quant_launch(e->pf_h, l == 0 ? nullptr : gp, w.attn_norm, B, D, e->eps,
                                 ActOut{e->pf_act, nullptr}, nullptr, s));
        if (w.qkv_fused) {
            CK(matbatch_launch(w.wq, w.tq, nullptr, e->pf_act, B, D, qkv_w, e->pf_qkv, e->d_err, s, qkv_w));
        } else {
            CK(matbatch_launch(w.wq, w.tq, nullptr, e->pf_act, B, D, qd, e->pf_qkv, e->d_err, s, qkv_w));
            CK(matbatch_launch(w.wk, w.tk, nullptr, e->pf_act, B, D, kvd, e->pf_qkv + qd, e->d_err, s, qkv_w));
            CK(matbatch_launch(w.wv, w.tv, nullptr, e->pf_act, B, D, kvd, e->pf_qkv + qd + kvd, e->d_err, s, qkv_w));
        }
        CK(qkv_post_launch(e->pf_qkv, qkv_w, B, e->nh_l, e->nkv_l, e->hd, w.q_norm, w.k_norm, e->qk_norm, e->eps,
                           e->rope_c, e->rope_s, 0, nullptr, w.kc, w.vc, e->hd, (int64_t)e->max_seq * e->hd, s));
        for (int z0 = 0; z0 < B; z0 += kPrefillGroup) {
            const int nz = B - z0 < kPrefillGroup ? B - z0 : kPrefillGroup;
            AttnArgs a{};
            a.q = e->pf_qkv + (size_t)z0 * qkv_w;
            a.q_stride = qkv_w;
            a.kc = w.kc;
            a.vc = w.vc;
            a.kv_pos_stride = e->hd;
            a.kv_head_stride = e->max_seq * e->hd;
            a.pos0 = z0;
            a.pos_dev = nullptr;
            a.n_heads = e->nh_l;
            a.n_kv = e->nkv_l;
            a.hd = e->hd;
            a.scale = e->attn_scale;
            a.window = 0;
            a.chunk = kPrefillChunk;
            a.max_splits = (z0 + nz + kPrefillChunk - 1) / kPrefillChunk;
            a.part = e->pf_part;
            if (tp) {
                a.out = gq + (size_t)z0 * QD + (size_t)rk * qd;
                a.out_stride = QD;
                a.act_out = ActOut{nullptr, nullptr};
            } else {
                a.out = e->exact ? e->pf_qkv + (size_t)z0 * qkv_w : nullptr;
                a.out_stride = qkv_w;
                a.act_out = ActOut{e->pf_actq + (size_t)z0 * (QD / 32), nullptr};
            }
            a.err = e->d_err;
            a.exact = e->exact ? 1 : 0;
            a.scores = e->pf_scores;
            a.score_cap = (int)e->pf_score_cap;
            if ((size_t)nz * e->nh_l * a.max_splits * attn_record_floats(e->hd) > e->pf_part_floats)
                return kErrCapacity;
            CK(attention_run(a, nz, s));
        }
        if (tp) {
            CK(gather(e, e->x_q, B, QD, rk * qd, qd));
            CK(act_quantize_launch(gq, B, QD, e->pf_actq, s));
            CK(matbatch_launch(w.wo + (size_t)rk * dl * row_bytes(w.to, QD), w.to, nullptr, e->pf_actq, B, QD, dl,
                               gp + (size_t)rk * dl, e->d_err, s, D));
            CK(gather(e, e->x_p, B, D, rk * dl, dl));
        } else {
            CK(matbatch_launch(w.wo, w.to, nullptr, e->pf_actq, B, QD, D, e->pf_p, e->d_err, s));
        }
        CK(add_norm_quant_launch(e->pf_h, gp, w.ffn_norm, B, D, e->eps, ActOut{e->pf_act, nullptr}, nullptr, s));
        if (w.gu_fused) {
            CK(matbatch_launch(w.wg, w.tg, nullptr, e->pf_act, B, D, 2 * fl, e->pf_gu, e->d_err, s, 2 * fl));
        } else {
            CK(matbatch_launch(w.wg, w.tg, nullptr, e->pf_act, B, D, fl, e->pf_gu, e->d_err, s, 2 * fl));
            CK(matbatch_launch(w.wu, w.tu, nullptr, e->pf_act, B, D, fl, e->pf_gu + fl, e->d_err, s, 2 * fl));
        }
        if (tp) {
            CK(glu_quant_launch(e->pf_gu, e->pf_gu + fl, 2 * fl, fl, B, e->arch == 2, ActOut{nullptr, nullptr}, s,
                                gf + (size_t)rk * fl, F));
            CK(gather(e, e->x_f, B, F, rk * fl, fl));
            CK(act_quantize_launch(gf, B, F, e->pf_actf, s));
            CK(matbatch_launch(w.wd + (size_t)rk * dl * row_bytes(w.td, F), w.td, nullptr, e->pf_actf, B, F, dl,
                               gp + (size_t)rk * dl, e->d_err, s, D));
            CK(gather(e, e->x_p, B, D, rk * dl, dl));
        } else {
            CK(glu_quant_launch(e->pf_gu, e->pf_gu + F, 2 * F, F, B, e->arch == 2, ActOut{e->pf_actf, nullptr}, s));
            CK(matbatch_launch(w.wd, w.td, nullptr, e->pf_actf, B, F, D, e->pf_p, e->d_err, s));
        }
    }
    // last position: residual, final norm, LM head (:1185-1205)
    const size_t last = (size_t)(B - 1) * D;
    CU(cudaMemcpyAsync(e->hidden, e->pf_h + last, (size_t)D * 4, cudaMemcpyDeviceToDevice, s));
    CK(add_norm_quant_launch(e->hidden, gp + last, e->out_norm, 1, D, e->eps, ActOut{nullptr, e->act_d}, e->normed,
                             s));
    return lm_head(e);
}

static int upload_ids(Engine* e, const int32_t* ids, int n) {
    if (n > e->ids_cap) {
        cudaStreamSynchronize(e->stream);
        cudaFree(e->ids_dev);
        e->ids_dev = nullptr;
        if (cudaMalloc(&e->ids_dev, (size_t)n * 4) != cudaSuccess) return kErrOutOfMemory;
        e->ids_cap = n;
    }
    CU(cudaMemcpyAsync(e->ids_dev, ids, (size_t)n * 4, cudaMemcpyHostToDevice, e->stream));
    return kOk;
}

static int set_state(Engine* e, int token, int pos, const int32_t* all, int n_all, int eos, int max_out) {
    DecodeState& h = *e->st_host;
    CU(cudaStreamSynchronize(e->stream));
    memset(&h, 0, sizeof(h));
    h.token = token;
    h.pos = pos;
    h.n_all = n_all;
    h.eos = eos;
    h.max_out = max_out;
    for (int k = 0; k < n_all && k < kRecentWindow; ++k) {
        const int idx = n_all - 1 - k;  // the last kRecentWindow tokens
        h.ring[(idx) % kRecentWindow] = all[idx];
    }
    CU(cudaMemcpyAsync(e->st, &h, sizeof(h), cudaMemcpyHostToDevice, e->stream));
    return kOk;
}

static int check_device_error(Engine* e) {
    int32_t h = 0;
    CU(cudaMemcpyAsync(&h, e->d_err, 4, cudaMemcpyDeviceToHost, e->stream));
    CU(cudaStreamSynchronize(e->stream));
    if (h) {
        cudaMemsetAsync(e->d_err, 0, 4, e->stream);
        e->error = "device-side wait timed out";
        return h;
    }
    return kOk;
}

static const LayerW* layer_or_null(const Engine* e, int l) { return l < (int)e->L.size() ? &e->L[l] : nullptr; }

// Rank `rank` of `tp`: its q heads [rank*nh, ..), KV heads, ffn rows, model
// rows (prefill's attn_output / ffn_down) and vocabulary rows (LM head).
struct TpShare {
    int nh, nkv, ffn, dim, voc0, voc;
};
static int tp_share(int nh, int nkv, int hd, int dim, int ffn, int vocab, int tp, int rank, TpShare& sh,
                    std::string& err) {
    if (tp < 1 || tp > kTpMaxRanks || rank < 0 || rank >= tp) { err = "bad tensor-parallel rank/size"; return kErrInvalidArg; }
    if (nh <= 0 || nkv <= 0 || hd <= 0 || nh % nkv || nkv % tp || dim % (4 * tp) || ffn % (32 * tp)) {
        err = "tensor parallel size must divide the KV heads, hidden/4 and ffn/32";
        return kErrInvalidArg;
    }
    sh.nh = nh / tp;
    sh.nkv = nkv / tp;
    sh.ffn = ffn / tp;
    sh.dim = dim / tp;
    int v0, v1;
    split_rows(vocab, tp, rank, 4, v0, v1);
    sh.voc0 = v0;
    sh.voc = v1 - v0;
    if (sh.voc <= 0) { err = "vocabulary too small for the tensor parallel size"; return kErrInvalidArg; }
    return kOk;
}

static int setup_step(Engine* e);

// Load: read hyper-parameters, lay this rank's share of the tensors out in one
// device arena, upload.
static int engine_load(Engine* e, const char* path, int max_seq, int tp_rank, int tp_size, std::string& err) {
    Gguf g;
    if (!gguf_open(path, g, err)) return kErrInvalidArg;
    const std::string arch = g.str.count("general.architecture") ? g.str["general.architecture"] : "qwen3";
    auto num = [&](const std::string& k, double d) { auto it = g.num.find(arch + "." + k); return it == g.num.end() ? d : it->second; };
    e->arch = arch.rfind("qwen", 0) == 0 ? 0 : (arch.rfind("llama", 0) == 0 ? 1 : (arch == "gemma" ? 2 : -1));
    if (e->arch < 0) { err = "unsupported architecture: " + arch; return kErrInvalidArg; }
    e->n_layers = (int)num("block_count", 0);
    e->dim = (int)num("embedding_length", 0);
    e->nh = (int)num("attention.head_count", 0);
    e->nkv = (int)num("attention.head_count_kv", e->nh);
    e->hd = (int)num("attention.key_length", e->nh ? e->dim / e->nh : 0);
    e->ffn = (int)num("feed_forward_length", 0);
    e->eps = (float)num("attention.layer_norm_rms_epsilon", 1e-6);
    e->rope_base = (float)num("rope.freq_base", 10000.0);
    e->softcap = (float)num("final_logit_softcapping", 0.0);
    e->vocab = g.arr_len.count("tokenizer.ggml.tokens") ? (int)g.arr_len["tokenizer.ggml.tokens"] : 0;
    e->eos = g.num.count("tokenizer.ggml.eos_token_id") ? (int)g.num["tokenizer.ggml.eos_token_id"] : -1;
    e->max_seq = max_seq;
    e->q_dim = e->nh * e->hd;
    e->kv_dim = e->nkv * e->hd;
    // Lua doubles, passed to C as float (:846-862, :698-713)
    e->attn_scale = (float)(1.0 / sqrt((double)e->hd));
    e->embd_scale = e->arch == 2 ? (float)sqrt((double)e->dim) : 1.0f;
    if (!e->n_layers || !e->dim || !e->nh || !e->hd || !e->ffn || !e->vocab || max_seq <= 0) {
        err = "missing hyper-parameters";
        return kErrInvalidArg;
    }
    if (e->dim % 256 || e->q_dim % 256 || e->ffn % 256 || e->hd % 32 || e->hd > 256 || e->nh % e->nkv) {
        err = "shapes not supported (dims must be multiples of 256, head_dim a multiple of 32 up to 256)";
        return kErrInvalidArg;
    }
    // ---- this rank's share (tensor parallel: heads, ffn rows, model rows, vocabulary rows)
    const int tp = tp_size;
    {
        TpShare sh{};
        const int st = tp_share(e->nh, e->nkv, e->hd, e->dim, e->ffn, e->vocab, tp, tp_rank, sh, err);
        if (st != kOk) return st;
        e->nh_l = sh.nh;
        e->nkv_l = sh.nkv;
        e->qd_l = sh.nh * e->hd;
        e->kvd_l = sh.nkv * e->hd;
        e->ffn_l = sh.ffn;
        e->dim_l = sh.dim;
        e->voc0 = sh.voc0;
        e->voc_l = sh.voc;
    }
    // ---- arena layout
    auto T = [&](const std::string& n) -> const GgufTensor* { auto it = g.tensors.find(n); return it == g.tensors.end() ? nullptr : &it->second; };
    struct Item { uint64_t src; size_t bytes; size_t off; };
    std::vector<Item> items;
    size_t off = 0;
    auto place = [&](const GgufTensor* t, bool follow) -> size_t {
        if (!follow) off = (off + 255) & ~(size_t)255;
        const size_t o = off;
        items.push_back({t->abs_off, t->nbytes, o});
        off += t->nbytes;
        return o;
    };
    // rows [r0, r1) of a [in, out] weight (rows are contiguous, out of them)
    auto place_rows = [&](const GgufTensor* t, int r0, int r1, bool follow) -> size_t {
        if (!follow) off = (off + 255) & ~(size_t)255;
        const size_t rb = row_bytes(t->type, (int64_t)t->dims[0]);
        const size_t o = off;
        items.push_back({t->abs_off + (uint64_t)r0 * rb, (size_t)(r1 - r0) * rb, o});
        off += (size_t)(r1 - r0) * rb;
        return o;
    };
    const int rk = tp_rank;
    struct Offs { size_t an, fn, qn, kn, q, k, v, o, gt, up, dn; bool has_qn, has_kn, qkv_f, gu_f; int tq, tk, tv, to, tg, tu, td; };
    std::vector<Offs> lo(e->n_layers);
    const char* lin[] = {"attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"};
    for (int l = 0; l < e->n_layers; ++l) {
        const std::string p = "blk." + std::to_string(l) + ".";
        const GgufTensor* an = T(p + "attn_norm.weight"), *fn = T(p + "ffn_norm.weight");
        const GgufTensor* lt[7];
        const uint64_t want_out[7] = {(uint64_t)e->q_dim, (uint64_t)e->kv_dim, (uint64_t)e->kv_dim, (uint64_t)e->dim,
                                      (uint64_t)e->ffn, (uint64_t)e->ffn, (uint64_t)e->dim};
        for (int i = 0; i < 7; ++i) {
            lt[i] = T(p + lin[i] + ".weight");
            if (!lt[i]) { err = "missing tensor " + p + lin[i] + ".weight"; return kErrInvalidArg; }
            if (lt[i]->dims.size() != 2 || lt[i]->dims[1] != want_out[i]) {
                err = "unexpected shape of " + p + lin[i] + ".weight";
                return kErrInvalidArg;
            }
            const int ty = lt[i]->type;
            if (ty != kQ4_0 && ty != kQ8_0 && ty != kQ4_K && ty != kQ6_K) { err = "unsupported weight type in " + p + lin[i]; return kErrInvalidArg; }
        }
        if (!an || !fn || an->type != kF32 || fn->type != kF32) { err = "missing/non-F32 norm in " + p; return kErrInvalidArg; }
        Offs& O = lo[l];
        O.an = place(an, false);
        O.fn = place(fn, false);
        const GgufTensor* qn = T(p + "attn_q_norm.weight"), *kn = T(p + "attn_k_norm.weight");
        O.has_qn = qn && qn->type == kF32;
        O.has_kn = kn && kn->type == kF32;
        O.qn = O.has_qn ? place(qn, false) : 0;
        O.kn = O.has_kn ? place(kn, false) : 0;
        O.qkv_f = lt[0]->type == lt[1]->type && lt[1]->type == lt[2]->type;
        O.q = place_rows(lt[0], rk * e->qd_l, (rk + 1) * e->qd_l, false);
        O.k = place_rows(lt[1], rk * e->kvd_l, (rk + 1) * e->kvd_l, O.qkv_f);
        O.v = place_rows(lt[2], rk * e->kvd_l, (rk + 1) * e->kvd_l, O.qkv_f);
        // attn_output and ffn_down whole on every rank: decode computes all their
        // rows everywhere (two gathers per layer instead of four), prefill this
        // rank's rows of them (compute-bound there) and gathers
        O.o = place_rows(lt[3], 0, e->dim, false);
        O.gu_f = lt[4]->type == lt[5]->type;
        O.gt = place_rows(lt[4], rk * e->ffn_l, (rk + 1) * e->ffn_l, false);
        O.up = place_rows(lt[5], rk * e->ffn_l, (rk + 1) * e->ffn_l, O.gu_f);
        O.dn = place_rows(lt[6], 0, e->dim, false);
        O.tq = lt[0]->type; O.tk = lt[1]->type; O.tv = lt[2]->type; O.to = lt[3]->type;
        O.tg = lt[4]->type; O.tu = lt[5]->type; O.td = lt[6]->type;
    }
    const GgufTensor* emb = T("token_embd.weight");
    const GgufTensor* onorm = T("output_norm.weight");
    if (!emb || (emb->type != kQ8_0 && emb->type != kQ6_K && emb->type != kBF16)) {
        err = "token_embd.weight must be Q8_0, Q6_K or BF16";  // lua/gncx_streamer.lua:700-711
        return kErrInvalidArg;
    }
    if (!onorm || onorm->type != kF32) { err = "missing output_norm.weight"; return kErrInvalidArg; }
    const size_t emb_off = place(emb, false);
    const size_t on_off = place(onorm, false);
    e->embd_type = emb->type;
    e->arena_bytes = (off + 255) & ~(size_t)255;
    CU(cudaMalloc(&e->arena, e->arena_bytes));
    for (const Item& it : items)
        CU(cudaMemcpyAsync(e->arena + it.off, g.base + it.src, it.bytes, cudaMemcpyHostToDevice, e->stream));
    CU(cudaStreamSynchronize(e->stream));
    e->tok_embd = e->arena + emb_off;
    e->out_norm = reinterpret_cast<const float*>(e->arena + on_off);
    // ---- KV cache
    const size_t kv_layer = (size_t)max_seq * e->kvd_l;  // this rank's KV heads
    CU(cudaMalloc(&e->kv, kv_layer * 2 * e->n_layers * 4));
    CU(cudaMemsetAsync(e->kv, 0, kv_layer * 2 * e->n_layers * 4, e->stream));
    e->L.resize(e->n_layers);
    e->qk_norm = e->arch == 0;
    for (int l = 0; l < e->n_layers; ++l) {
        const Offs& O = lo[l];
        LayerW& w = e->L[l];
        w.attn_norm = reinterpret_cast<const float*>(e->arena + O.an);
        w.ffn_norm = reinterpret_cast<const float*>(e->arena + O.fn);
        w.q_norm = O.has_qn ? reinterpret_cast<const float*>(e->arena + O.qn) : nullptr;
        w.k_norm = O.has_kn ? reinterpret_cast<const float*>(e->arena + O.kn) : nullptr;
        if (e->arch == 0 && (!O.has_qn || !O.has_kn)) e->qk_norm = false;
        w.wq = e->arena + O.q; w.wk = e->arena + O.k; w.wv = e->arena + O.v; w.wo = e->arena + O.o;
        w.wg = e->arena + O.gt; w.wu = e->arena + O.up; w.wd = e->arena + O.dn;
        w.tq = O.tq; w.tk = O.tk; w.tv = O.tv; w.to = O.to; w.tg = O.tg; w.tu = O.tu; w.td = O.td;
        w.qkv_fused = O.qkv_f;
        w.gu_fused = O.gu_f;
        w.kc = e->kv + (size_t)2 * l * kv_layer;
        w.vc = w.kc + kv_layer;
    }
    // ---- RoPE table with the reference's libm calls (:1779-1796), every position
    const int half = e->hd / 2;
    std::vector<float> c((size_t)max_seq * half), sn((size_t)max_seq * half), freq(half);
    for (int i = 0; i < half; ++i) freq[i] = 1.0f / powf(e->rope_base, (float)(2 * i) / (float)e->hd);
    for (int p = 0; p < max_seq; ++p)
        for (int i = 0; i < half; ++i) {
            const float ang = (float)p * freq[i];
            c[(size_t)p * half + i] = cosf(ang);
            sn[(size_t)p * half + i] = sinf(ang);
        }
    CU(cudaMalloc(&e->rope_c, c.size() * 4));
    CU(cudaMalloc(&e->rope_s, sn.size() * 4));
    CU(cudaMemcpy(e->rope_c, c.data(), c.size() * 4, cudaMemcpyHostToDevice));
    CU(cudaMemcpy(e->rope_s, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
    // ---- decode buffers
    const size_t D = e->dim, F = e->ffn;
    e->max_splits = (max_seq + decode_chunk(e->hd) - 1) / decode_chunk(e->hd);
    CU(cudaMalloc(&e->hidden, D * 4));
    CU(cudaMalloc(&e->normed, D * 4));
    CU(cudaMalloc(&e->proj, D * 4));
    CU(cudaMalloc(&e->qkv, (size_t)(e->qd_l + 2 * e->kvd_l) * 4));
    CU(cudaMalloc(&e->gu, 2 * (size_t)e->ffn_l * 4));
    // ---- exchange region (tensor parallel): gather buffers for up to x_rows prompt rows
    {
        e->x_rows = max_seq < kTpMaxRows ? max_seq : kTpMaxRows;
        const size_t R = tp > 1 ? (size_t)e->x_rows : 0;
        e->x_q = 0;
        e->x_p = e->x_q + R * e->q_dim * 4;
        e->x_f = e->x_p + R * D * 4;
        e->x_l = e->x_f + R * F * 4;
        const size_t T = tp > 1 ? (size_t)tp : 0;
        e->ll_q = e->x_l + (tp > 1 ? (size_t)e->vocab * 4 : 0);
        e->ll_f = e->ll_q + T * e->q_dim * 8;
        e->ll_l = e->ll_f + T * F * 8;
        e->ll_p = e->ll_l + T * e->vocab * 8;
        e->ll_am = (e->ll_p + T * D * 8 + 15) & ~(size_t)15;
        const int st = tp_alloc(e->tp, tp_rank, tp, e->ll_am + T * 16);
        if (st != kOk) return st;
    }
    if (tp > 1) {
        e->logits = tp_buffer(e->tp, e->x_l);
    } else {
        CU(cudaMalloc(&e->logits_own, (size_t)e->vocab * 4));
        e->logits = e->logits_own;
    }
    CU(cudaMalloc(&e->act_d, staged_act_bytes(D)));
    CU(cudaMalloc(&e->act_q, staged_act_bytes(e->q_dim)));
    CU(cudaMalloc(&e->act_f, staged_act_bytes(F)));
    CU(cudaMalloc(&e->part, (size_t)e->nh_l * e->max_splits * attn_record_floats(e->hd) * 4));
    CU(cudaMalloc(&e->scores, (size_t)e->nh_l * e->max_splits * decode_chunk(e->hd) * 4));
    CU(cudaMalloc(&e->st, sizeof(DecodeState)));
    CU(cudaMallocHost(&e->st_host, sizeof(DecodeState)));
    CU(cudaMalloc(&e->am_scratch, argmax_state_scratch_bytes()));
    CU(cudaMalloc(&e->d_err, 4));
    CU(cudaMemset(e->d_err, 0, 4));

    e->out_cap = max_seq + 1;
    CU(cudaMalloc(&e->out_ids, (size_t)e->out_cap * 4));
    for (auto& ev : e->ev) CU(cudaEventCreate(&ev));
    (void)layer_or_null;
    return setup_step(e);
}

// Plan the persistent decode step for this model (one GPU; q/k/v and gate/up
// each stored as one matrix).  Models it does not cover keep the per-kernel
// decode, which GNCX_DECODE_PERSISTENT selects for every model when 0.
static int setup_step(Engine* e) {
    e->step_ok = false;
    if (e->tp.size > 1) return kOk;
    const char* env = getenv("GNCX_DECODE_PERSISTENT");
    if (!env || atoi(env) == 0) return kOk;
    StepPlan p{};
    std::vector<StepLayer> hl(e->n_layers);
    for (int l = 0; l < e->n_layers; ++l) {
        const LayerW& w = e->L[l];
        if (!w.qkv_fused || !w.gu_fused) return kOk;
        StepLayer& s = hl[l];
        s.wqkv = w.wq; s.wo = w.wo; s.wg = w.wg; s.wu = w.wu; s.wd = w.wd;
        s.tqkv = w.tq; s.to = w.to; s.tgu = w.tg; s.td = w.td;
        s.attn_norm = w.attn_norm; s.ffn_norm = w.ffn_norm; s.q_norm = w.q_norm; s.k_norm = w.k_norm;
        s.kc = w.kc; s.vc = w.vc;
    }
    p.n_layers = e->n_layers;
    p.dim = e->dim;
    p.nh = e->nh;
    p.nkv = e->nkv;
    p.hd = e->hd;
    p.qd = e->q_dim;
    p.kvd = e->kv_dim;
    p.ffn = e->ffn;
    p.max_seq = e->max_seq;
    p.eps = e->eps;
    p.scale = e->attn_scale;
    p.qk_norm = e->qk_norm ? 1 : 0;
    p.gelu = e->arch == 2 ? 1 : 0;
    p.ahead = 192 * 1024;
    if (const char* v = getenv("GNCX_STEP_AHEAD")) p.ahead = atoi(v);  // tuning override (bytes)
    if (decode_step_plan(p, hl.data(), device_info().max_smem_optin) != kOk) return kOk;
    const size_t R = (size_t)attn_record_floats(e->hd);
    e->step_sync_bytes = decode_step_sync_words(e->n_layers) * 4;
    CU(cudaMalloc(&e->step_layers, hl.size() * sizeof(StepLayer)));
    CU(cudaMemcpy(e->step_layers, hl.data(), hl.size() * sizeof(StepLayer), cudaMemcpyHostToDevice));
    CU(cudaMalloc(&e->step_attn, (size_t)e->q_dim * 4));
    CU(cudaMalloc(&e->step_proj, (size_t)e->dim * 4));
    CU(cudaMalloc(&e->step_glu, (size_t)e->ffn * 4));
    CU(cudaMalloc(&e->step_part, (size_t)e->nh * p.max_splits * R * 4));
    CU(cudaMalloc(&e->step_scores, (size_t)e->nh * p.score_stride * 4));
    CU(cudaMalloc(&e->step_sync, e->step_sync_bytes));
    p.layers = e->step_layers;
    p.rope_c = e->rope_c;
    p.rope_s = e->rope_s;
    p.out_norm = e->out_norm;
    p.st = e->st;
    p.hidden = e->hidden;
    p.normed = e->normed;
    p.act_out = e->act_d;
    p.qkv = e->qkv;
    p.attn = e->step_attn;
    p.proj_o = e->proj;
    p.proj_d = e->step_proj;
    p.glu = e->step_glu;
    p.part = e->step_part;
    p.scores = e->step_scores;
    p.sync = e->step_sync;
    p.err = e->d_err;
    e->step = p;
    e->step_ok = true;
    return kOk;
}

static void engine_free(Engine* e) {
    if (!e) return;
    if (e->stream) cudaStreamSynchronize(e->stream);
    if (e->graph) cudaGraphExecDestroy(e->graph);
    void* bufs[] = {e->scores, e->pf_scores, e->arena, e->kv, e->rope_c, e->rope_s, e->hidden, e->normed, e->proj, e->qkv, e->gu, e->logits_own,
                    e->act_d, e->act_q, e->act_f, e->part, e->st, e->am_scratch, e->d_err, e->out_ids, e->ids_dev,
                    e->pf_h, e->pf_p, e->pf_qkv, e->pf_gu, e->pf_part, e->pf_act, e->pf_actq, e->pf_actf,
                    e->step_layers, e->step_attn, e->step_proj, e->step_glu, e->step_part, e->step_scores,
                    e->step_sync};
    for (void* b : bufs)
        if (b) cudaFree(b);
    tp_free(e->tp);
    if (e->st_host) cudaFreeHost(e->st_host);
    for (auto& ev : e->ev)
        if (ev) cudaEventDestroy(ev);
    if (e->stream) cudaStreamDestroy(e->stream);
    delete e;
}

// Capture one decode step (forward + sample) as a graph for `penalty`.
static int build_graph(Engine* e, double penalty) {
    if (e->graph && e->penalty_graph == penalty && e->graph_exact == (int)e->exact) return kOk;
    if (e->graph) {
        cudaGraphExecDestroy(e->graph);
        e->graph = nullptr;
    }
    // One eager forward first: one-time setup (function attributes, occupancy
    // queries) happens outside the capture.  It writes the KV entry the first
    // captured step writes again with the same values.
    CK(decode_step(e, false, penalty));
    CU(cudaStreamSynchronize(e->stream));
    cudaGraph_t g = nullptr;
    CU(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
    const int st = decode_step(e, true, penalty);
    const cudaError_t ce = cudaStreamEndCapture(e->stream, &g);
    if (st != kOk) { if (g) cudaGraphDestroy(g); return st; }
    if (ce != cudaSuccess) { cudaGetLastError(); return kErrCuda; }
    const cudaError_t ie = cudaGraphInstantiate(&e->graph, g, 0);
    cudaGraphDestroy(g);
    if (ie != cudaSuccess) { cudaGetLastError(); e->graph = nullptr; return kErrCuda; }
    e->penalty_graph = penalty;
    e->graph_exact = (int)e->exact;
    return kOk;
}

}  // namespace gncx

using namespace gncx;

// ---------------------------------------------------------------- C ABI
extern "C" {

void* gncx_engine_create_tp(const char* gguf_path, int32_t max_seq_len, int32_t tp_rank, int32_t tp_size) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return nullptr;
    }
    Engine* e = new Engine();
    if (const char* v = getenv("GNCX_TP_OUTSPLIT")) e->tp_outsplit = atoi(v) != 0;
    if (cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess) {
        delete e;
        return nullptr;
    }
    std::string err;
    gemv_set_pdl(true);  // engine weights are never written while decoding
    if (engine_load(e, gguf_path, max_seq_len > 0 ? max_seq_len : 4096, tp_rank, tp_size, err) != kOk) {
        fprintf(stderr, "gncx_engine_create: %s\n", err.empty() ? "CUDA error" : err.c_str());
        engine_free(e);
        return nullptr;
    }
    return e;
}

// Host only (no GPU needed): rank `tp_rank`'s share of a model with hp = {n_heads,
// n_kv, head_dim, dim, ffn, vocab}: out = {q heads, kv heads, ffn rows, model
// rows, first vocabulary row, vocabulary rows}.  The split gncx_engine_create_tp uses.
int32_t gncx_engine_tp_share(const int32_t* hp, int32_t tp_size, int32_t tp_rank, int32_t* out) {
    if (!hp || !out) return kErrInvalidArg;
    TpShare sh{};
    std::string err;
    const int st = tp_share(hp[0], hp[1], hp[2], hp[3], hp[4], hp[5], tp_size, tp_rank, sh, err);
    if (st != kOk) return st;
    const int32_t v[6] = {sh.nh, sh.nkv, sh.ffn, sh.dim, sh.voc0, sh.voc};
    memcpy(out, v, sizeof(v));
    return kOk;
}

// This rank's exchange-region handle (GNCX_TP_HANDLE_BYTES bytes) for the other ranks.
int32_t gncx_engine_tp_handle(void* h, void* out) {
    Engine* e = static_cast<Engine*>(h);
    if (!e || !out) return kErrInvalidArg;
    if (e->tp.size == 1) return kOk;
    return tp_handle(e->tp, out);
}

// Map every rank's exchange region (handles in rank order); collective in effect:
// every rank calls it before the first prefill / forward.
int32_t gncx_engine_tp_connect(void* h, const void* handles) {
    Engine* e = static_cast<Engine*>(h);
    if (!e || !handles) return kErrInvalidArg;
    return tp_connect(e->tp, handles);
}

void* gncx_engine_create(const char* gguf_path, int32_t max_seq_len) {
    return gncx_engine_create_tp(gguf_path, max_seq_len, 0, 1);
}

void gncx_engine_destroy(void* h) { engine_free(static_cast<Engine*>(h)); }

// out[0..11] = n_layers, dim, n_heads, n_kv, head_dim, ffn, vocab, max_seq, eos, arch, embd_type, qk_norm
int32_t gncx_engine_hparams(void* h, int32_t* out) {
    Engine* e = static_cast<Engine*>(h);
    if (!e || !out) return kErrInvalidArg;
    const int32_t v[12] = {e->n_layers, e->dim, e->nh, e->nkv, e->hd, e->ffn, e->vocab, e->max_seq, e->eos, e->arch,
                           e->embd_type, e->qk_norm ? 1 : 0};
    memcpy(out, v, sizeof(v));
    return kOk;
}

// 1: exact serial softmax in attention (bit-exact with the reference up to expf
// rounding); 0 (default): split-KV softmax.
int32_t gncx_engine_set_exact(void* h, int32_t on) {
    Engine* e = static_cast<Engine*>(h);
    if (!e) return kErrInvalidArg;
    e->exact = on != 0;
    return kOk;
}

const char* gncx_engine_error(void* h) { return h ? static_cast<Engine*>(h)->error.c_str() : "null engine"; }

void* gncx_engine_stream(void* h) { return h ? static_cast<Engine*>(h)->stream : nullptr; }

// lua/gncx_streamer.lua:759-965: logits of token `id` at position `pos` (host copy if logits_out).
int32_t gncx_engine_forward_token(void* h, int32_t id, int32_t pos, float* logits_out) {
    Engine* e = static_cast<Engine*>(h);
    if (!e || id < 0 || id >= e->vocab || pos < 0 || pos >= e->max_seq || !e->tp.connected) return kErrInvalidArg;
    CK(set_state(e, id, pos, nullptr, 0, -1, 0));
    CK(decode_step(e, false, 1.0));
    if (logits_out) CU(cudaMemcpyAsync(logits_out, e->logits, (size_t)e->vocab * 4, cudaMemcpyDeviceToHost, e->stream));
    return check_device_error(e);
}

// lua/gncx_streamer.lua:968-1208: runs the prompt from position 0, fills the KV cache.
int32_t gncx_engine_prefill(void* h, const int32_t* ids, int32_t n, float* logits_out) {
    Engine* e = static_cast<Engine*>(h);
    if (!e || !ids || n <= 0 || n > e->max_seq || !e->tp.connected) return kErrInvalidArg;
    for (int i = 0; i < n; ++i)
        if (ids[i] < 0 || ids[i] >= e->vocab) return kErrInvalidArg;
    // buffers grow (and the ids travel) before the clock starts: the timing is the prefill's
    if (n > 1) {
        CK(ensure_prefill(e, n));
        CK(upload_ids(e, ids, n));
    }
    CU(cudaEventRecord(e->ev[0], e->stream));
    if (n == 1) {
        CK(set_state(e, ids[0], 0, nullptr, 0, -1, 0));
        CK(decode_step(e, false, 1.0));
    } else {
        CK(prefill_batch(e, n));
    }
    CU(cudaEventRecord(e->ev[1], e->stream));
    if (logits_out) CU(cudaMemcpyAsync(logits_out, e->logits, (size_t)e->vocab * 4, cudaMemcpyDeviceToHost, e->stream));
    const int st = check_device_error(e);
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, e->ev[0], e->ev[1]);
    e->prefill_ms = ms;
    return st;
}

// Device logits of the last forward/prefill.
const float* gncx_engine_logits(void* h) { return h ? static_cast<Engine*>(h)->logits : nullptr; }

// lua/gncx_streamer.lua:1276-1311 with token ids: prefill, then greedy decode of
// up to max_new tokens; every decode step is one CUDA graph launch driven by
// device-resident state.  Returns the number of ids written (or -status).
int32_t gncx_engine_generate(void* h, const int32_t* prompt, int32_t n_prompt, int32_t max_new, double penalty,
                             int32_t eos, int32_t* out_ids) {
    Engine* e = static_cast<Engine*>(h);
    if (!e || !prompt || n_prompt <= 0 || max_new < 0 || !out_ids) return -kErrInvalidArg;
    if (n_prompt >= e->max_seq) return 0;
    if (max_new > e->max_seq - n_prompt) max_new = e->max_seq - n_prompt;
    if (max_new == 0) return 0;
    nvtxRangePushA("gncx_prefill");
    int st = gncx_engine_prefill(h, prompt, n_prompt, nullptr);
    nvtxRangePop();
    if (st != kOk) return -st;
    if ((st = set_state(e, 0, n_prompt, prompt, n_prompt, eos, max_new)) != kOk) return -st;
    if ((st = argmax_state_launch(e->logits, e->vocab, e->st, penalty, e->out_ids, 0, e->am_scratch, e->stream)) != kOk)
        return -st;
    if ((st = build_graph(e, penalty)) != kOk) return -st;
    if (cudaEventRecord(e->ev[2], e->stream) != cudaSuccess) return -kErrCuda;
    nvtxRangePushA("gncx_decode");  // profiler ranges (no cost without a tool attached)
    for (int i = 1; i < max_new; ++i) {
        if (cudaGraphLaunch(e->graph, e->stream) != cudaSuccess) {
            nvtxRangePop();
            return -kErrCuda;
        }
    }
    nvtxRangePop();
    if (cudaEventRecord(e->ev[3], e->stream) != cudaSuccess) return -kErrCuda;
    DecodeState& hs = *e->st_host;
    if (cudaMemcpyAsync(&hs, e->st, sizeof(DecodeState), cudaMemcpyDeviceToHost, e->stream) != cudaSuccess)
        return -kErrCuda;
    if ((st = check_device_error(e)) != kOk) return -st;
    const int n_out = hs.n_out < max_new ? hs.n_out : max_new;
    if (n_out > 0 && cudaMemcpy(out_ids, e->out_ids, (size_t)n_out * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        return -kErrCuda;
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, e->ev[2], e->ev[3]);
    e->decode_ms = ms;
    e->decode_steps = max_new - 1;
    return n_out;
}

int32_t gncx_engine_decode_path(void* h) { return h && static_cast<Engine*>(h)->step_ok ? 1 : 0; }

// Device time of the last prefill and decode loop (ms) and the decode step count.
int32_t gncx_engine_timing(void* h, double* prefill_ms, double* decode_ms, int32_t* decode_steps) {
    Engine* e = static_cast<Engine*>(h);
    if (!e) return kErrInvalidArg;
    if (prefill_ms) *prefill_ms = e->prefill_ms;
    if (decode_ms) *decode_ms = e->decode_ms;
    if (decode_steps) *decode_steps = e->decode_steps;
    return kOk;
}

}  // extern "C"
