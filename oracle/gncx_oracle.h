/*
 * gncx_oracle.h -- CPU oracle for the GNC-X decode/prefill hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the reference
 * CPU kernels in csrc/gncx_llm_kernels.cpp (omega-Core-Dev/gnc-x), used by
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg as the
 * checker.  Nothing in the product library links or calls it.
 *
 * Floating-point contract: every expression is evaluated in the order the
 * reference source writes it, one IEEE-754 binary32 rounding per operation
 * (the file is compiled with -ffp-contract=off).  That is the reference's
 * source-level semantics; the reference's own build script (-march=native)
 * lets GCC fuse a*b+c into FMA, which moves the last bits by ~2e-7 relative
 * depending on the build host.
 *
 * Parity pin: tests/test_oracle.py checks these functions bit-for-bit against
 * the reference sources compiled with -ffp-contract=off (oracle/_ref) and
 * against the golden vectors in tests/golden/ generated from that build.
 */
#ifndef GNCX_ORACLE_H
#define GNCX_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Per-32 activation block after re-quantization (csrc/gncx_llm_kernels.cpp:299-306). */
typedef struct {
    float   d;          /* amax / 127 */
    int32_t sum_q;      /* sum of all 32 quants */
    int32_t sum_lo;     /* sum of quants 0..15 */
    int32_t sum_hi;     /* sum of quants 16..31 */
    int8_t  qs[32];
} orc_act_block;

float orc_fp16_to_fp32(uint16_t h);
float orc_bf16_to_fp32(uint16_t b);

/* :955-995 */
void orc_act_quantize(const float* x, int32_t in_dim, orc_act_block* out);

/* Dequantize `n` consecutive weights of one row (n multiple of the block size).
 * Q8_0/Q6_K/BF16 follow the embedding-fetch routines (:693-780) with
 * scale 1.0; Q4_0 is d*(q-8) and Q4_K is (d*sc)*q - (dmin*m), the weight
 * values the dot kernels (:1021-1065, :1127-1205) integrate. */
void orc_dequant_row(const uint8_t* row, int32_t ggml_type, int32_t n, float* out);

/* :1327-1471 (universal matvec; SIMD-path arithmetic order) */
void orc_matvec(const uint8_t* w, int32_t ggml_type, const float* x,
                int32_t in_dim, int32_t out_dim, float* y);
/* :1495-1692 */
void orc_matbatch(const uint8_t* w, int32_t ggml_type, const float* xb, int32_t batch,
                  int32_t in_dim, int32_t out_dim, float* yb);
/* :1713-1732 */
void orc_lm_head(const uint8_t* w, int32_t ggml_type, const float* h, int32_t dim,
                 int32_t vocab, float softcap, float* logits);

/* :789-840 (fast path); returns the quant scale the reference would store */
void orc_rmsnorm(const float* x, const float* w, int32_t dim, float eps, float* out);
/* :895-953 (w may be NULL) */
void orc_rmsnorm_heads(float* v, const float* w, int32_t n_heads, int32_t head_dim, float eps);

/* :1779-1796 cos/sin table for one position; ff may be NULL */
void orc_rope_table(int32_t pos, int32_t head_dim, float base, const float* ff,
                    float* cos_t, float* sin_t);
/* :1760-1863 (q or k may be NULL) */
void orc_rope(float* q, float* k, const float* ff, int32_t n_heads, int32_t n_kv,
              int32_t head_dim, int32_t pos, float base);

/* :1887-1994 */
void orc_attention_step(const float* q, const float* k, const float* v, float* kc, float* vc,
                        int32_t pos, int32_t n_heads, int32_t n_kv, int32_t head_dim,
                        float scale, int32_t window, int32_t write_kv, float* out);

/* :2018-2052 */
void orc_swiglu(const float* g, const float* u, int32_t n, float* out);
void orc_geglu(const float* g, const float* u, int32_t n, float* out);

/* :693-780 */
void orc_embed_row(const uint8_t* tensor, int32_t ggml_type, int32_t token, int32_t dim,
                   float scale, float* out);

/* lua/gncx_streamer.lua:1229-1273: penalized greedy argmax (Lua doubles, strict >,
 * lowest index wins ties, penalty over the last <=65 entries of `recent`). */
int32_t orc_sample_greedy(const float* logits, int32_t vocab, const int32_t* recent,
                          int32_t n_recent, double penalty);

/* Bytes of one row of `n` weights in `ggml_type` (lua/gncx_gguf.lua:50-66). */
size_t orc_row_bytes(int32_t ggml_type, int64_t n);

#ifdef __cplusplus
}
#endif
#endif
