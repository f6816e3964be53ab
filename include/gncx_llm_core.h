/*
 * gncx_llm_core.h -- C ABI of the B200 build of the GNC-X hot path.
 *
 * Drop-in for the reference library (csrc/gncx_llm_kernels.cpp of
 * omega-Core-Dev/gnc-x, loaded by lua/gncx_gguf.lua:72-73 and bound by the
 * ffi.cdef block of lua/gncx_streamer.lua:16-252): the entry points in the
 * first part carry the reference's names, argument order and types.
 *
 * Memory model.  Every float / byte pointer handed to a kernel entry point
 * must be reachable by the GPU: device memory, managed memory (what
 * gncx_ram_alloc* returns), or an address inside a file mapped with
 * gncx_gla_map_readonly (translated to that file's device mirror).  Telemetry
 * structs and the quant-scale out-parameter stay host memory, as in the
 * reference.  A pointer the GPU cannot reach is rejected with
 * GNCX_ERR_NOT_DEVICE_ACCESSIBLE; there is no CPU fallback.
 *
 * Errors.  The reference's kernels return void and report nothing.  Here each
 * call records a status readable with gncx_last_error(); by default every
 * reference-named call also waits for its GPU work (synchronous mode), so a
 * caller that reads results on the host, as the Lua orchestrator does, sees
 * them complete.  gncx_set_synchronous(0) makes calls stream-ordered.
 *
 * Concurrency.  Split-KV decode attention (gncx_mqa_attention_step_ext, its
 * allocation-free variant and an engine's decode step) merges its records in
 * the kernel, counting arrivals per KV head in one set of counters per GPU.
 * Keep such calls on one GPU from running at the same time on different
 * streams: use one stream per GPU for them, or order the streams.
 */
#ifndef GNCX_LLM_CORE_H
#define GNCX_LLM_CORE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#pragma pack(push, 1)
/* csrc/gncx_llm_kernels.cpp:267-271 (telemetry only; never read or written here) */
typedef struct {
    uint8_t phase_2bit;
    uint8_t diag_d;
    uint16_t abs_delta;
} GNCXCompactToken;

/* :308-313 (host memory; counters updated on the host) */
typedef struct {
    uint64_t total_macs_equivalent;
    uint64_t zero_origin_cancellations;
    uint64_t zero_weight_skips;
    uint64_t xfold_bucket_merges;
} GNCXTelemetryStats;
#pragma pack(pop)

/* ------------------------------------------------------------------------ */
/* Reference entry points (same names and signatures)                        */
/* ------------------------------------------------------------------------ */

/* GGUF file mapping: :327-404, :617-667.  map_readonly mmaps the file on the
 * host (the loader parses it there) and uploads a device mirror of it. */
void* gncx_gla_map_readonly(const char* filepath, size_t* out_size);          /* :327 */
const uint8_t* gncx_gla_get_base_ptr(void* opaque_handle);                      /* :386 */
void gncx_gla_unmap(void* opaque_handle);                                       /* :391 */
void gncx_gla_prefetch_range(const uint8_t* mmap_base, size_t offset, size_t num_bytes); /* :617 */

/* Weight arena: :481-612.  Backed by CUDA managed memory, so host loops over
 * scratch buffers (lua/gncx_streamer.lua:871-873) keep working. */
void* gncx_ram_alloc_colored(size_t total_bytes, uint8_t k, uint8_t d, uint8_t R); /* :481 */
void* gncx_ram_alloc(size_t total_bytes);                                        /* :553 */
uint8_t* gncx_ram_get_ptr(void* ram_handle);                                     /* :561 */
uint8_t gncx_ram_get_ddr3_bank(void* ram_handle);                                /* :566 */
uint8_t gncx_ram_get_l1_set(void* ram_handle);                                   /* :571 */
void gncx_ram_free(void* ram_handle);                                            /* :576 */
void gncx_ram_copy_chunk(void* ram_handle, size_t dst_offset, const uint8_t* src_base, size_t src_offset,
                         size_t num_bytes);                                      /* :602 */

/* Embedding rows: :693, :720, :765 */
void gncx_fetch_token_embedding_q8_0(const uint8_t* mmap_base, size_t tensor_abs_offset, int32_t token_id,
                                     int32_t embed_dim, float scale_factor, float* out_hidden);
void gncx_fetch_token_embedding_q6_k(const uint8_t* mmap_base, size_t tensor_abs_offset, int32_t token_id,
                                     int32_t embed_dim, float scale_factor, float* out_hidden);
void gncx_fetch_token_embedding_bf16(const uint8_t* mmap_base, size_t tensor_abs_offset, int32_t token_id,
                                     int32_t embed_dim, float scale_factor, float* out_hidden);

/* RMSNorm: :789 (out_tokens is telemetry and is not written), :895 */
void gncx_rmsnorm_and_encode_4phase(const float* input_hidden, const uint8_t* mmap_base, size_t norm_weight_offset,
                                    int32_t dim, float eps, int32_t layer_k, float* out_normed_fp32,
                                    GNCXCompactToken* out_tokens, float* out_quant_scale);
void gncx_rmsnorm_inplace_heads(float* vec, const uint8_t* mmap_base, size_t norm_weight_offset, int32_t has_weight,
                                int32_t n_heads, int32_t head_dim, float eps);

/* Quantized GEMV / prefill GEMM: :1327, :1476, :1495, :1694.
 * ggml_type 2=Q4_0, 8=Q8_0, 12=Q4_K, 14=Q6_K, 30=BF16; quantized types need
 * in_dim % 256 == 0. */
void gncx_xfold_universal_matvec(const uint8_t* mmap_base, size_t weight_abs_offset, int32_t ggml_type,
                                 const float* in_vec, const GNCXCompactToken* in_tokens, int32_t in_dim,
                                 int32_t out_dim, float* out_vec, GNCXTelemetryStats* telemetry);
void gncx_xfold_q4_0_matvec(const uint8_t* mmap_base, size_t weight_abs_offset, const float* in_vec,
                            const GNCXCompactToken* in_tokens, int32_t in_dim, int32_t out_dim, float* out_vec,
                            GNCXTelemetryStats* telemetry);
void gncx_xfold_universal_matbatch(const uint8_t* mmap_base, size_t weight_abs_offset, int32_t ggml_type,
                                   const float* in_batch, int32_t batch_size, int32_t in_dim, int32_t out_dim,
                                   float* out_batch, GNCXTelemetryStats* telemetry);
void gncx_xfold_q4_0_matbatch(const uint8_t* mmap_base, size_t weight_abs_offset, const float* in_batch,
                              int32_t batch_size, int32_t in_dim, int32_t out_dim, float* out_batch,
                              GNCXTelemetryStats* telemetry);

/* LM head over the tied embedding, optional tanh softcap: :1713, :1734 */
void gncx_universal_lm_head_logits(const uint8_t* mmap_base, size_t embd_abs_offset, int32_t ggml_type,
                                   const float* final_hidden, int32_t embed_dim, int32_t vocab_size, float softcap,
                                   float* out_logits);
void gncx_q8_0_lm_head_logits(const uint8_t* mmap_base, size_t embd_abs_offset, const float* final_hidden,
                              int32_t embed_dim, int32_t vocab_size, float* out_logits);

/* RoPE (rotate-half): :1760, :1865.  q_tokens is telemetry and is not written. */
void gncx_apply_rope_xor11_ext(float* q_vec, float* k_vec, GNCXCompactToken* q_tokens, const uint8_t* mmap_base,
                               size_t rope_freqs_offset, int32_t has_rope_freqs, int32_t n_heads, int32_t n_kv_heads,
                               int32_t head_dim, int32_t pos, float freq_base);
void gncx_apply_rope_xor11(float* q_vec, float* k_vec, GNCXCompactToken* q_tokens, int32_t n_heads,
                           int32_t n_kv_heads, int32_t head_dim, int32_t pos, float freq_base);

/* GQA/MQA decode attention over the fp32 KV cache [max_seq][n_kv][head_dim]: :1887, :1996 */
void gncx_mqa_attention_step_ext(const float* q_vec, const float* k_vec, const float* v_vec, float* k_cache_layer,
                                 float* v_cache_layer, int32_t pos, int32_t n_heads, int32_t n_kv_heads,
                                 int32_t head_dim, float attn_scale, int32_t sliding_window, int32_t write_kv,
                                 float* out_attn_vec);
void gncx_mqa_attention_step(const float* q_vec, const float* k_vec, const float* v_vec, float* k_cache_layer,
                             float* v_cache_layer, int32_t pos, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                             float* out_attn_vec);

/* GLU activations: :2018, :2038 */
void gncx_geglu_activation(const float* gate_vec, const float* up_vec, int32_t ffn_dim, float* out_ffn_vec);
void gncx_swiglu_activation(const float* gate_vec, const float* up_vec, int32_t ffn_dim, float* out_ffn_vec);

/* ------------------------------------------------------------------------ */
/* Added entry points (no counterpart in the reference): GPU plumbing        */
/* ------------------------------------------------------------------------ */

enum {
    GNCX_OK = 0,
    GNCX_ERR_INVALID_ARG = 1,
    GNCX_ERR_UNALIGNED = 2,
    GNCX_ERR_CUDA = 3,
    GNCX_ERR_NO_DEVICE = 4,
    GNCX_ERR_TIMEOUT = 5,
    GNCX_ERR_NOT_DEVICE_ACCESSIBLE = 6,
    GNCX_ERR_OUT_OF_MEMORY = 7,
    GNCX_ERR_CAPACITY = 8
};

int32_t gncx_last_error(void);               /* first error since the last clear (sticky) */
const char* gncx_last_error_message(void);
void gncx_clear_error(void);
int32_t gncx_sync(void);
/* Diagnostic builds only (libgncx_llm_core_trace.so; the product library
 * returns GNCX_ERR_INVALID_ARG): from now on every kernel launch on the
 * current device appends one 40-byte record per CTA -- grid id, kernel tag,
 * an argument, CTA index, %globaltimer at entry and exit -- to the device
 * buffer `records` (capacity records; `counter` is a device word the caller
 * zeroes).  NULL, NULL stops recording.  No reference counterpart. */
int32_t gncx_trace_enable(void* records, uint32_t* counter, uint32_t capacity);                     /* wait for queued work; returns and records its status */
void gncx_set_stream(void* cuda_stream);     /* NULL = the library's own stream */
void* gncx_get_stream(void);
void gncx_set_synchronous(int32_t on);       /* 1 (default): reference-named calls wait before returning */
/* 1: a GEMV may start streaming its weights before the preceding kernel on
 * the stream has finished (programmatic dependent launch); its activations
 * and outputs still wait.  Only valid while weights are not written by GPU
 * work queued just before the GEMV.  Default 0. */
void gncx_set_weight_prefetch(int32_t on);
/* 1: attention forms its softmax sum and weighted V sum serially in position
 * order, as the reference does (bit-exact up to expf rounding; slower at long
 * context).  0 (default): split-KV softmax, ~1e-6 relative. */
void gncx_set_exact_attention(int32_t on);
int32_t gncx_device_count(void);
int32_t gncx_set_device(int32_t device);

/* Device memory for callers without a CUDA runtime of their own (ctypes, FFI). */
void* gncx_device_alloc(size_t bytes);
void gncx_device_free(void* ptr);
int32_t gncx_memcpy(void* dst, const void* src, size_t bytes); /* any direction, synchronous */

/* Activation re-quantization to the kernels' 48-byte block records
 * ({float d; int32 sum_lo; int32 sum_hi; int32 pad; int8 qs[32]} per 32 inputs). */
int32_t gncx_act_quantize(const float* x, int32_t rows, int32_t in_dim, void* act_out);
/* GEMV from pre-quantized activations (the act-Q8 step shared by Q/K/V or gate/up). */
int32_t gncx_matvec_preq(const uint8_t* base, size_t offset, int32_t ggml_type, const void* act, int32_t in_dim,
                         int32_t out_dim, float* out_vec);
/* Block dequantization of `rows` rows of `n` weights to fp32 (bit-exact with the
 * reference's row-fetch routines for Q8_0/Q6_K/BF16). */
int32_t gncx_dequantize_rows(const uint8_t* base, size_t offset, int32_t ggml_type, int32_t rows, int32_t n,
                             float* out);
/* Penalized greedy sampling (lua/gncx_streamer.lua:1229-1273) on device logits;
 * `recent` is a host array.  Returns the token id, or -1 on error. */
int32_t gncx_sample_greedy(const float* logits, int32_t vocab, const int32_t* recent, int32_t n_recent,
                           double repeat_penalty);

/* Decode attention that allocates nothing (no counterpart in the reference).
 * Same arguments and result as gncx_mqa_attention_step_ext with the split-KV
 * softmax, plus the CUDA stream to run on (NULL = legacy default stream);
 * pointers must be device-accessible (no mapped-file translation), and the
 * call is stream-ordered (it does not wait).  Its scratch is a fixed 4 MiB
 * array per device, held until exit: n_heads * ceil(window / chunk) *
 * (head_dim + 4) * 4 bytes must fit (chunk = 16..64 positions; e.g. 32 heads
 * of 128 fit a window of ~15,800 positions), else GNCX_ERR_CAPACITY with a
 * message in gncx_last_error_message().  The first call on a device does a
 * one-time set-up (looks up the array's address) and should come before any
 * stream capture; after a cudaDeviceReset of that device the looked-up
 * address is stale and the entry point must not be called there again.  All
 * calls on a device share the array, so calls whose GPU work overlaps race
 * and must be serialised by the caller.  A call rejected with a status has
 * not written the KV cache.  Returns a status. */
/* Causal attention over a block of prompt positions (no reference
 * counterpart as one call; it replaces the per-position loop of the
 * reference's prefill, lua/gncx_streamer.lua:1079-1109, which calls
 * gncx_mqa_attention_step_ext with write_kv = 0 and no window):
 * n_tok queries at positions pos0 .. pos0 + n_tok - 1, query z attending to
 * cache rows 0 .. pos0 + z.  q and out are [n_tok][n_heads * head_dim]; the
 * caches use the reference layout [pos][n_kv][head_dim] and already hold
 * rows 0 .. pos0 + n_tok - 1.  Follows gncx_set_exact_attention.  Returns a
 * status. */
int32_t gncx_attention_prefill(const float* q, const float* k_cache, const float* v_cache, int32_t pos0,
                               int32_t n_tok, int32_t n_heads, int32_t n_kv, int32_t head_dim, float attn_scale,
                               float* out);

int32_t gncx_mqa_attention_step_noalloc(const float* q_vec, const float* k_vec, const float* v_vec,
                                        float* k_cache_layer, float* v_cache_layer, int32_t pos, int32_t n_heads,
                                        int32_t n_kv_heads, int32_t head_dim, float attn_scale,
                                        int32_t sliding_window, int32_t write_kv, float* out_attn_vec,
                                        void* cuda_stream);

/* ------------------------------------------------------------------------ */
/* Model engine: the reference orchestrator's decode loop on the GPU         */
/* ------------------------------------------------------------------------ */
/* A restatement of GNCXStreamer (lua/gncx_streamer.lua) for callers without
 * LuaJIT: the GGUF's quantized blocks are uploaded in their native layout,
 * forward_token (:759-965) runs as fused kernels, and every greedy decode
 * step of generate (:1276-1311) is one CUDA graph launch driven by state in
 * device memory.  Token ids in, token ids / logits out (no tokenizer).
 * Statuses are GNCX_* codes; gncx_engine_error() describes the last one. */
void* gncx_engine_create(const char* gguf_path, int32_t max_seq_len); /* NULL on failure (reason on stderr) */
void gncx_engine_destroy(void* engine);
/* out[12] = n_layers, dim, n_heads, n_kv_heads, head_dim, ffn_dim, vocab, max_seq, eos, arch, embd_type, qk_norm */
int32_t gncx_engine_hparams(void* engine, int32_t* out);
/* 1: exact serial softmax in attention (the reference's order); 0 (default): split-KV softmax */
int32_t gncx_engine_set_exact(void* engine, int32_t on);
const char* gncx_engine_error(void* engine);
void* gncx_engine_stream(void* engine);                 /* the engine's CUDA stream */
/* Logits of token `id` at position `pos` (KV cache entries below pos must be filled);
 * logits_out: host array of vocab floats, or NULL. */
int32_t gncx_engine_forward_token(void* engine, int32_t id, int32_t pos, float* logits_out);
/* Runs the prompt from position 0 (batched prefill); logits of the last position. */
int32_t gncx_engine_prefill(void* engine, const int32_t* ids, int32_t n, float* logits_out);
const float* gncx_engine_logits(void* engine);          /* device logits of the last forward / prefill */
/* Prefill, then penalized greedy decode of up to max_new tokens (stops at eos);
 * writes the generated ids to out_ids (host) and returns their count, or -status. */
int32_t gncx_engine_generate(void* engine, const int32_t* prompt, int32_t n_prompt, int32_t max_new,
                             double repeat_penalty, int32_t eos, int32_t* out_ids);
/* Device time (ms) of the last prefill and decode loop, and the decode step count. */
int32_t gncx_engine_timing(void* engine, double* prefill_ms, double* decode_ms, int32_t* decode_steps);
/* Which kernels run a decode step (no counterpart in the reference): 1 = the
 * whole layer stack as one persistent kernel (one GPU, a model whose shapes
 * and formats it covers); 0 = one kernel per GEMV / norm / attention step. */
int32_t gncx_engine_decode_path(void* engine);

/* Tensor parallel over the GPUs of one box (no counterpart in the reference),
 * one process per GPU, each on its own current device.  Rank r of tp_size
 * loads its share: attention heads (q/k/v rows and its KV heads), ffn
 * gate/up rows and LM-head vocabulary rows, plus attn_output and ffn_down
 * whole.  Every output element is computed whole on one GPU, in the 1-GPU
 * order, so logits and token streams equal the 1-GPU engine's.  Decode
 * all-gathers over NVLink peer memory at the attention output and the
 * ffn_down input (then every rank runs attn_output and ffn_down on all rows)
 * and once for the logits; prefill splits attn_output / ffn_down rows too.  tp_size <= 8 and
 * must divide the KV heads, hidden/4 and ffn/32.  Set-up: each rank creates
 * its engine, passes gncx_engine_tp_handle's bytes to the others (any host
 * channel), and calls gncx_engine_tp_connect with all ranks' handles in rank
 * order; then every rank makes the same prefill / forward / generate calls.
 * A peer that stops arriving makes the others' calls fail with
 * GNCX_ERR_TIMEOUT after 2 s instead of hanging.  A tensor-parallel prefill
 * takes at most min(max_seq_len, 4096) prompt tokens per call
 * (GNCX_ERR_CAPACITY beyond). */
#define GNCX_TP_HANDLE_BYTES 64
/* Host only: rank tp_rank's share of a model, hp = {n_heads, n_kv_heads,
 * head_dim, dim, ffn_dim, vocab}; out[6] = {q heads, KV heads, ffn rows,
 * model rows, first vocabulary row, vocabulary rows}, or an error status for
 * a size that does not divide the model. */
int32_t gncx_engine_tp_share(const int32_t* hp, int32_t tp_size, int32_t tp_rank, int32_t* out);
void* gncx_engine_create_tp(const char* gguf_path, int32_t max_seq_len, int32_t tp_rank, int32_t tp_size);
int32_t gncx_engine_tp_handle(void* engine, void* out /* GNCX_TP_HANDLE_BYTES */);
int32_t gncx_engine_tp_connect(void* engine, const void* handles /* tp_size * GNCX_TP_HANDLE_BYTES */);


#ifdef __cplusplus
}
#endif
#endif /* GNCX_LLM_CORE_H */
