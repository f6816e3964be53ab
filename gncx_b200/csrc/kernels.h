// kernels.h -- host-side launchers for the B200 hot-path kernels (internal).
// Every launcher returns a gncx::Status; launch failures map to kErrCuda.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>
#include "act.cuh"
#include "common.cuh"

namespace gncx {

struct DeviceInfo {
    int device = -1;
    int sm_count = 0;
    int max_smem_optin = 0;
    int smem_per_sm = 0;
    int l2_bytes = 0;
};
// Properties of the current device (queried once per device).
const DeviceInfo& device_info();
// Raise kernel `k`'s dynamic shared-memory limit to at least `bytes` on the
// current device.  The attribute belongs to one device, so the limit already
// set is remembered per (kernel, device) and each device is configured once.
cudaError_t set_smem_limit(const void* k, size_t bytes);
template <class K>
inline cudaError_t set_smem_limit(K* k, size_t bytes) {
    return set_smem_limit(reinterpret_cast<const void*>(k), bytes);
}

// ---- GEMV / prefill ----
// `act` (16-byte aligned), when given, is a staged activation vector
// (staged_act_bytes(in_dim) bytes, written by act_stage_launch or a fused
// producer kernel); otherwise x is re-quantized inside the kernel.
int gemv_launch(const uint8_t* w, int32_t type, const float* x, const uint8_t* act, int32_t in_dim,
                int32_t out_dim, float* y, float softcap, int32_t* err, cudaStream_t st);
// Programmatic dependent launch for the GEMV and the fused decode kernels:
// a kernel may start (prefetching weights) before the preceding kernel on the
// stream completes; weights must not be written by that kernel.  Off by default.
void gemv_set_pdl(bool on);
bool pdl_enabled();
// yb[t * ldy + o] (ldy = out_dim when 0)
int matbatch_launch(const uint8_t* w, int32_t type, const float* xb, const ActBlock* act, int32_t batch,
                    int32_t in_dim, int32_t out_dim, float* yb, int32_t* err, cudaStream_t st, int32_t ldy = 0);
// The same on the tensor cores (tcgen05 kind::i8) for Q4_0 / Q8_0 / Q4_K;
// kErrInvalidArg when the format, shape or alignment has no such path.
int matbatch_tc_launch(const uint8_t* w, int32_t type, const ActBlock* act, int32_t batch, int32_t in_dim,
                       int32_t out_dim, float* yb, int32_t* err, cudaStream_t st, int32_t ldy);
// x[rows][in_dim] -> ActBlock[rows][in_dim/32]
int act_quantize_launch(const float* x, int32_t rows, int32_t in_dim, ActBlock* out, cudaStream_t st);
// ActBlock[in_dim/32] -> staged vector (staged_act_bytes(in_dim) bytes)
int act_stage_launch(const ActBlock* blocks, int32_t in_dim, uint8_t* staged, cudaStream_t st);
// Dequantize `rows` rows of `n` weights (row stride = row_bytes(type, n)) to fp32.
int dequant_launch(const uint8_t* w, int32_t type, int32_t rows, int32_t n, float scale, const int32_t* row_ids,
                   float* out, cudaStream_t st);

// ---- norms / rope / activations ----
// out[r] = rmsnorm(x[r]) * w, rows of `dim`; optional residual: x += res first (written back).
int rmsnorm_launch(const float* x, const float* w, int32_t rows, int32_t dim, float eps, float* out,
                   cudaStream_t st);
int rmsnorm_heads_launch(float* v, const float* w, int32_t rows, int32_t n_heads, int32_t head_dim, float eps,
                         cudaStream_t st);
// Rotate-half RoPE of `rows` vectors of n_heads heads; per-row positions
// pos0 + r (pos_list == nullptr) or pos_list[r]; cos/sin from the table
// [max_pos][head_dim/2] (host-computed with the reference's libm calls).
int rope_launch(float* v, int32_t rows, int32_t row_stride, int32_t n_heads, int32_t head_dim, int32_t pos0,
                const float* cos_tab, const float* sin_tab, cudaStream_t st);
struct RopeTab {
    float c[256];
    float s[256];
};
// One position, q (nh heads) and/or k (nkv heads); either may be null.
int rope_tab_launch(float* q, float* k, int32_t nh, int32_t nkv, int32_t hd, const RopeTab& tab, cudaStream_t st);
int absmax_launch(const float* x, int32_t n, float* out, cudaStream_t st);
int glu_launch(const float* g, const float* u, int64_t n, float* out, bool gelu, cudaStream_t st);
int softcap_launch(float* x, int64_t n, float cap, cudaStream_t st);

// ---- attention ----
// General form: n_tok queries; query z sits at position (pos_dev ? *pos_dev : pos0) + z
// and attends to its window; records [z][head][max_splits] of attn_record_floats(hd)
// floats: {max, sum of exp, -, -, o[hd]} (16-byte aligned rows).
__host__ __device__ inline int attn_record_floats(int hd) { return hd + 4; }
struct AttnArgs {
    const float* q;        // query z at q + z * q_stride
    int q_stride;
    const float* kc;
    const float* vc;
    int kv_pos_stride;     // floats between positions (reference layout: n_kv*hd; head-major: hd)
    int kv_head_stride;    // floats between kv heads (reference layout: hd; head-major: max_seq*hd)
    int pos0;
    const int* pos_dev;
    int n_heads, n_kv, hd;
    float scale;
    int window;
    int chunk;             // positions per split
    int max_splits;        // record capacity per (query, head); splits past the window exit
    float* part;
    float* out;            // may be null
    int out_stride;
    ActOut act_out;        // optional re-quantized output: blocks [z][n_heads*hd/32], or staged (one query)
    int32_t* err;
    // exact mode: scores go to `scores` [z][head][score_cap] and the softmax sum
    // and the probability-weighted V sum are formed serially in position order,
    // as the reference does (bit-exact up to the host libm's expf rounding).
    int exact;
    float* scores;
    int score_cap;         // floats per (query, head) score row; a multiple of 4
    // 1: K/V rows below the query's own position were written before the
    // preceding kernel ran (single-query decode), so a CTA may load them before
    // its dependency wait under programmatic dependent launch.  0: load nothing early.
    int prefetch_old;
    // Decode only (one query, window 0): when post_k is set, q is the QKV
    // GEMV's raw output and the kernel does what the Q/K post step does
    // otherwise -- per-head RMSNorm (post_norm, gains post_qn / post_kn, may
    // be null) and RoPE (tables [max_pos][hd/2]) of q, and of the new K row
    // post_k + kv_head * hd, which it writes with the new V row (post_v) into
    // the cache at the query's position.
    const float* post_k;
    const float* post_v;
    const float* post_qn;
    const float* post_kn;
    int post_norm;
    float post_eps;
    const float* rope_c;
    const float* rope_s;
    // One query (the drop-in step's write_kv): its own position's new K and V
    // rows, [n_kv][hd] each, or null.  attention_run stores them in the cache at
    // the query's position: the register-streaming kernel reads that position
    // from here and writes the rows itself, every other path copies them into
    // the cache before its kernels run.
    const float* new_k;
    const float* new_v;
};
int attention_run(const AttnArgs& a, int32_t n_tok, cudaStream_t st);
// True when attention_run supports these head counts and head size.
bool attention_shape_ok(int32_t n_heads, int32_t n_kv, int32_t head_dim);
int attention_geometry_chunk(int32_t len, int32_t n_kv, int sm_count);
struct AttnScratch {
    float* part;        // partial (max, sum, o[hd]) records
    int32_t capacity;   // records available
};
// exact_scores: null for the split-KV softmax, else n_heads * (window rounded up
// to 64) floats for the exact serial softmax.
int attention_launch(const float* q, float* kc, float* vc, int32_t pos, int32_t n_heads, int32_t n_kv,
                     int32_t head_dim, float scale, int32_t window, float* out, const AttnScratch& scratch,
                     int32_t* err, cudaStream_t st, float* exact_scores = nullptr, const float* new_k = nullptr,
                     const float* new_v = nullptr);
int32_t attention_scratch_records(int32_t pos, int32_t n_heads, int32_t window);

// ---- sampling ----
// Penalized greedy argmax (lua/gncx_streamer.lua:1229-1273) -> *out_idx.
int argmax_penalized_launch(const float* logits, int32_t vocab, const int32_t* recent, int32_t n_recent,
                            double penalty, int32_t* out_idx, void* scratch, cudaStream_t st);
size_t argmax_scratch_bytes(int32_t vocab);

// ---- fused engine kernels (fused.cu) ----
constexpr int kRecentWindow = 65;  // tokens the repetition penalty looks back over
struct DecodeState {
    int32_t token;     // input token of the next step
    int32_t pos;       // its position
    int32_t n_all;     // prompt + generated tokens so far
    int32_t n_out;     // generated tokens so far
    int32_t done;
    int32_t eos;
    int32_t max_out;
    int32_t pad;
    int32_t ring[kRecentWindow];  // last kRecentWindow tokens (any order)
};
// act.staged (rows == 1) or act.blocks [rows][dim/32]
int add_norm_quant_launch(float* hidden, const float* residual, const float* w, int32_t rows, int32_t dim, float eps,
                          ActOut act, float* normed, cudaStream_t st);
int qkv_post_launch(float* qkv, int32_t row_stride, int32_t rows, int32_t nh, int32_t nkv, int32_t hd,
                    const float* q_norm, const float* k_norm, bool do_norm, float eps, const float* cos_tab,
                    const float* sin_tab, int32_t pos0, const int32_t* pos_dev, float* kc, float* vc,
                    int64_t kv_pos_stride, int64_t kv_head_stride, cudaStream_t st);
// GLU of `rows` rows (gate and up `stride` floats apart between rows) into the
// re-quantized `act` and/or fp32 `out` (row r at out + r * out_stride).
int glu_quant_launch(const float* g, const float* u, int32_t stride, int32_t ffn, int32_t rows, bool gelu,
                     ActOut act, cudaStream_t st, float* out = nullptr, int32_t out_stride = 0);
constexpr int kArgmaxParts = 148;  // partial maxima of stage 1: doubles [kArgmaxParts], then ints
size_t argmax_state_scratch_bytes();
// Stage 1 only, over logits of the vocabulary ids idx0 .. idx0 + vocab: the
// per-block penalized maxima (global ids) into `scratch`; *n_parts blocks.
int argmax_partials_launch(const float* logits, int32_t vocab, int32_t idx0, const DecodeState* st, double penalty,
                           void* scratch, int32_t* n_parts, cudaStream_t s);
int argmax_state_launch(const float* logits, int32_t vocab, DecodeState* st, double penalty, int32_t* out_ids,
                        int advance_pos, void* scratch, cudaStream_t s);

// ---- persistent decode step (decode_step.cu) ----
// One decode token's layer stack as one persistent kernel (one CTA per SM,
// cooperative launch); single GPU, weights Q4_0 / Q8_0 / Q4_K / Q6_K with
// q/k/v and gate/up each stored as one matrix of one type.
constexpr int kStepMaxDim = 4096;       // hidden size (the residual stream lives in registers)
constexpr int kStepStageBytes = 73856;  // one ring stage: 32 Q4_K rows of 4096 inputs + alignment slack
constexpr int kStepStages = 2;
constexpr int kStepSyncWords = 32;      // counters per layer (phases, then per-KV-head words)
struct StepLayer {
    const uint8_t* wqkv;  // q, k, v rows back to back
    const uint8_t* wo;
    const uint8_t* wg;    // gate rows
    const uint8_t* wu;    // up rows
    const uint8_t* wd;
    int tqkv, to, tgu, td;
    const float* attn_norm;
    const float* ffn_norm;
    const float* q_norm;  // may be null
    const float* k_norm;
    float* kc;            // head-major cache [n_kv][max_seq][head_dim]
    float* vc;
    // tile geometry of the four GEMVs (q/k/v, attn_output, gate/up, ffn_down),
    // filled in by decode_step_plan
    int rows[4];          // rows per tile (gate/up: gate rows, with as many up rows)
    int wrows[4];         // rows per compute warp (gate/up: gate rows, with as many up rows)
    int tiles[4];
    int rbytes[4];        // bytes per row
    int pair_off;         // gate/up: stage offset of the up rows
};
struct StepPlan {
    const StepLayer* layers;  // device array [n_layers]
    int n_layers, dim, nh, nkv, hd, qd, kvd, ffn, max_seq;
    float eps, scale;
    int qk_norm, gelu;
    int exact;                // 1: attention in the reference's serial order (needs exact_ok)
    const float* rope_c;
    const float* rope_s;
    const float* out_norm;
    const DecodeState* st;    // the token's position
    float* hidden;            // in: the token's embedding row; out: the final residual stream
    float* normed;            // out: the final RMSNorm (fp32)
    uint8_t* act_out;         // out: the same, staged act-Q8 for the LM head
    float* qkv;               // [qd + 2 kvd]
    float* attn;              // [qd]
    float* proj_o;            // [dim]
    float* proj_d;            // [dim]
    float* glu;               // [ffn]
    float* part;              // split-KV records [nh][max_splits][hd + 4]
    float* scores;            // exact mode: scores, then softmax weights [nh][score_stride]
    unsigned* sync;           // decode_step_sync_words(n_layers) words, zero before every launch
    int32_t* err;
    int ahead;                // bytes of L2 prefetch a CTA keeps ahead of its copies
    // set by decode_step_plan
    int chunk, max_splits, stage_bytes, max_terms, exact_ok, all_q4k;
    int score_stride;         // max_seq rounded up to a multiple of 4
};
// Checks the shapes and formats and fills the geometry fields; kOk when the
// persistent kernel can run this model within max_smem bytes per CTA.
int decode_step_plan(StepPlan& p, StepLayer* host_layers, int max_smem);
size_t decode_step_sync_words(int n_layers);
int decode_step_launch(const StepPlan& p, cudaStream_t st);

// ---- tensor parallelism (tp.cu) ----
// One exchange region per rank: kTpCtlBytes of control words, then the gather
// buffers at byte offsets chosen by the caller.  Control words: flags
// [kTpMaxRanks][kTpMaxCtas] (the epoch CTA c of rank q last published here),
// this rank's epoch per gather CTA, and the layout words peers check.
constexpr int kTpMaxRanks = 8;
constexpr int kTpMaxCtas = 64;        // CTAs of one gather launch
constexpr int kTpHandleBytes = 64;    // sizeof(cudaIpcMemHandle_t)
constexpr size_t kTpCtlBytes = 4096;
constexpr int kTpEpochs = kTpMaxRanks * kTpMaxCtas;
constexpr int kTpInfo = kTpEpochs + kTpMaxCtas;  // 5 words: magic, bytes (lo, hi), rank, size
constexpr uint32_t kTpMagic = 0x58544e47u;
constexpr int kTpLlSlots = 5;
constexpr int kTpLlEpochs = 640;  // word offset: [kTpLlSlots][kTpMaxCtas] epochs of the one-row gather
static_assert(kTpInfo + 5 <= kTpLlEpochs && (kTpLlEpochs + kTpLlSlots * kTpMaxCtas) * 4 <= (int)kTpCtlBytes,
              "control words fit");
struct TpComm {
    int rank = 0, size = 1;
    bool connected = false;
    uint8_t* local = nullptr;             // this rank's region
    size_t bytes = 0;
    uint8_t* region[kTpMaxRanks] = {};    // every rank's region mapped here (region[rank] == local)
};
int tp_alloc(TpComm& c, int rank, int size, size_t bytes);
int tp_handle(const TpComm& c, void* out);          // kTpHandleBytes
int tp_connect(TpComm& c, const void* handles);     // size x kTpHandleBytes, in rank order
void tp_free(TpComm& c);
// The float buffer at byte offset `buf` of the data area, in this rank's region.
inline float* tp_buffer(const TpComm& c, size_t buf) { return reinterpret_cast<float*>(c.local + kTpCtlBytes + buf); }
// All-gather of `rows` rows of `row_floats` floats: this rank supplies floats
// [off, off + len) of every row (already in its own buffer); afterwards every
// rank's buffer holds every rank's slices.  A peer that does not arrive within
// 2 s records kErrTimeout in *err.
int tp_gather_launch(const TpComm& c, size_t buf, int32_t rows, int32_t row_floats, int32_t off, int32_t len,
                     int32_t* err, cudaStream_t st);
// Every rank's slice [off[q], off[q] + len[q]) of one gathered row.
struct TpSlices {
    int32_t off[kTpMaxRanks];
    int32_t len[kTpMaxRanks];
};
// One-row all-gather for decode: each value travels with the gather's epoch in
// one 8-byte store ({value, epoch}) into the peer's staging area at byte
// offset `ll` (size x row_floats x 8 bytes), and the receiver polls its own
// staging area until every peer value of this epoch is there -- one NVLink
// trip, no fence, no separate flag.  slot < kTpLlSlots names the gather (each
// slot keeps its own epochs; the same slot must always have the same shape).
int tp_gather_ll_launch(const TpComm& c, size_t buf, size_t ll, int32_t row_floats, const TpSlices& sl, int32_t slot,
                        int32_t* err, cudaStream_t st);
// Tensor-parallel greedy step: each rank has the penalized maxima of its
// vocabulary slice (argmax_partials_launch into `scratch`, n_parts of them);
// the ranks swap their best (value, id) -- 16 bytes each, at byte offset
// `stage` (size x 16 bytes) of every region's data area -- and every rank
// applies the overall best (larger value, then lower id: the first maximum of
// the whole vocabulary) to its decode state exactly as argmax_state_launch
// does.  Replaces an all-gather of every logit.
int tp_argmax_state_launch(const TpComm& c, size_t stage, const void* scratch, int32_t n_parts, DecodeState* st,
                           int32_t* out_ids, int advance_pos, int32_t* err, cudaStream_t s);

// ---- embedding ----
int embed_launch(const uint8_t* tensor, int32_t type, const int32_t* tokens, int32_t n_tokens, int32_t dim,
                 float scale, float* out, cudaStream_t st);

}  // namespace gncx
