/*
 * gncx_oracle_model.h -- whole-model CPU oracle (TEST INFRASTRUCTURE ONLY).
 * Restates lua/gncx_streamer.lua's forward_token/prefill/sample/generate over
 * either the reference's compiled kernels or the C restatement.
 */
#ifndef GNCX_ORACLE_MODEL_H
#define GNCX_ORACLE_MODEL_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { T_ATTN_NORM, T_Q, T_K, T_V, T_Q_NORM, T_K_NORM, T_O, T_FFN_NORM, T_GATE, T_UP, T_DOWN, ORC_NT };
enum { ORC_ARCH_QWEN = 0, ORC_ARCH_LLAMA = 1, ORC_ARCH_GEMMA = 2 };

typedef struct {
    int32_t n_layers, dim, n_heads, n_kv, head_dim, ffn_dim, vocab, max_seq;
    float eps, rope_base, softcap;
    int32_t arch;
    const uint8_t* base;        /* start of the GGUF file image */
    uint64_t tok_embd_off;      /* absolute file offsets */
    int32_t tok_embd_type;
    uint64_t out_norm_off;
    const uint64_t* off;        /* [n_layers][ORC_NT], UINT64_MAX = absent */
    const int32_t* typ;         /* [n_layers][ORC_NT] */
} orc_model_desc;

void* orc_model_create(const orc_model_desc* desc, const char* ref_lib /* NULL: oracle kernels */);
/* lib_memory != 0: the model's vectors and KV caches come from the bound
 * library's gncx_ram_alloc (and go back through gncx_ram_free), as the Lua
 * streamer's scratch does (lua/gncx_streamer.lua:462-464, :539-561) -- for a
 * library whose kernels need memory they can reach (the B200 library). */
void* orc_model_create_ex(const orc_model_desc* desc, const char* ref_lib, int32_t lib_memory);
void orc_model_destroy(void* m);
const float* orc_model_forward(void* m, int32_t tok, int32_t pos);
const float* orc_model_prefill(void* m, const int32_t* ids, int32_t n);
int32_t orc_model_generate(void* m, const int32_t* prompt, int32_t n_prompt, int32_t max_new, double penalty,
                           int32_t eos_id, int32_t* out_ids);
const float* orc_model_logits(void* m);
const float* orc_model_kcache(void* m, int32_t layer);

#ifdef __cplusplus
}
#endif
#endif
