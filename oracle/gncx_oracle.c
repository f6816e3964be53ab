/*
 * gncx_oracle.c -- CPU oracle for the GNC-X decode/prefill hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see gncx_oracle.h).  A plain-C restatement of the
 * arithmetic in the reference's csrc/gncx_llm_kernels.cpp; each function
 * names the reference lines it follows.  Compiled with -ffp-contract=off so
 * every operation rounds exactly once, in source order.
 */
#include "gncx_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>
#include <unistd.h>

/* ---- a small parallel-for for the oracle's row loops (pthreads) -------- */

typedef void (*range_fn)(void* ctx, int32_t lo, int32_t hi);
typedef struct { range_fn fn; void* ctx; int32_t lo, hi; } range_job;

static void* range_thunk(void* p) {
    range_job* j = (range_job*)p;
    j->fn(j->ctx, j->lo, j->hi);
    return NULL;
}

static int oracle_threads(void) {
    const char* e = getenv("ORC_THREADS");
    int n = e ? atoi(e) : (int)sysconf(_SC_NPROCESSORS_ONLN);
    if (n < 1) n = 1;
    if (n > 64) n = 64;
    return n;
}

static void par_for(int32_t n, range_fn fn, void* ctx) {
    int nt = oracle_threads();
    if (n < 64 || nt == 1) { fn(ctx, 0, n); return; }
    if (nt > n) nt = n;
    pthread_t th[64];
    range_job jobs[64];
    const int32_t chunk = (n + nt - 1) / nt;
    for (int t = 0; t < nt; ++t) {
        jobs[t].fn = fn; jobs[t].ctx = ctx;
        jobs[t].lo = t * chunk;
        jobs[t].hi = (t + 1) * chunk < n ? (t + 1) * chunk : n;
        if (t) pthread_create(&th[t], NULL, range_thunk, &jobs[t]);
    }
    range_thunk(&jobs[0]);
    for (int t = 1; t < nt; ++t) pthread_join(th[t], NULL);
}

/* ---- number formats -------------------------------------------------- */

/* csrc/gncx_llm_kernels.cpp:85-112: exact IEEE half -> single, subnormals too. */
float orc_fp16_to_fp32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t expo = (h >> 10) & 0x1Fu;
    uint32_t mant = h & 0x3FFu;
    uint32_t bits;
    if (expo == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            /* normalise the subnormal: shift until the hidden bit appears */
            int32_t e = 1;
            while ((mant & 0x400u) == 0) { mant <<= 1; e--; }
            mant &= 0x3FFu;
            bits = sign | ((uint32_t)(e + 112) << 23) | (mant << 13);
        }
    } else if (expo == 31) {
        bits = sign | 0x7F800000u | (mant << 13);
    } else {
        bits = sign | ((expo + 112u) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* :114-119 */
float orc_bf16_to_fp32(uint16_t b) {
    uint32_t bits = (uint32_t)b << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

size_t orc_row_bytes(int32_t t, int64_t n) {
    switch (t) {
        case 0:  return (size_t)n * 4;          /* F32 */
        case 1:  return (size_t)n * 2;          /* F16 */
        case 30: return (size_t)n * 2;          /* BF16 */
        case 2:  return (size_t)(n / 32) * 18;  /* Q4_0 */
        case 8:  return (size_t)(n / 32) * 34;  /* Q8_0 */
        case 12: return (size_t)(n / 256) * 144;/* Q4_K */
        case 14: return (size_t)(n / 256) * 210;/* Q6_K */
        default: return 0;
    }
}

/* ---- activation re-quantization: :955-995 ----------------------------- */

void orc_act_quantize(const float* x, int32_t in_dim, orc_act_block* out) {
    const int32_t nb = in_dim / 32;
    for (int32_t b = 0; b < nb; ++b) {
        const float* src = x + (size_t)b * 32;
        orc_act_block* blk = &out[b];
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) {
            float a = fabsf(src[i]);
            if (a > amax) amax = a;
        }
        if (amax == 0.0f) {
            memset(blk, 0, sizeof(*blk));
            continue;
        }
        const float inv = 127.0f / amax;
        blk->d = amax / 127.0f;
        int32_t lo = 0, hi = 0;
        for (int i = 0; i < 16; ++i) {
            int8_t a = (int8_t)nearbyintf(src[i] * inv);
            int8_t c = (int8_t)nearbyintf(src[i + 16] * inv);
            blk->qs[i] = a;
            blk->qs[i + 16] = c;
            lo += a;
            hi += c;
        }
        blk->sum_lo = lo;
        blk->sum_hi = hi;
        blk->sum_q = lo + hi;
    }
}

/* ---- Q4_K 6-bit scale/min unpacking: :1112-1120 ------------------------ */

static inline void k4_scale_min(int j, const uint8_t* s, int* sc, int* m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* ---- dequantization -------------------------------------------------- */

void orc_dequant_row(const uint8_t* row, int32_t t, int32_t n, float* out) {
    if (t == 2) {                                   /* Q4_0: d*(q-8), :1058-1062 */
        for (int32_t b = 0; b < n / 32; ++b) {
            const uint8_t* blk = row + (size_t)b * 18;
            const float d = orc_fp16_to_fp32(rd16(blk));
            for (int j = 0; j < 16; ++j) {
                out[b * 32 + j] = d * (float)((blk[2 + j] & 0x0F) - 8);
                out[b * 32 + j + 16] = d * (float)((blk[2 + j] >> 4) - 8);
            }
        }
    } else if (t == 8) {                            /* Q8_0: q*d, :707-714 */
        for (int32_t b = 0; b < n / 32; ++b) {
            const uint8_t* blk = row + (size_t)b * 34;
            const float d = orc_fp16_to_fp32(rd16(blk)) * 1.0f;
            for (int j = 0; j < 32; ++j) out[b * 32 + j] = (float)(int8_t)blk[2 + j] * d;
        }
    } else if (t == 12) {                           /* Q4_K: (d*sc)*q - dmin*m, :1172-1175 */
        for (int32_t s = 0; s < n / 256; ++s) {
            const uint8_t* blk = row + (size_t)s * 144;
            const float d = orc_fp16_to_fp32(rd16(blk));
            const float dmin = orc_fp16_to_fp32(rd16(blk + 2));
            const uint8_t* sc = blk + 4;
            const uint8_t* qs = blk + 16;
            for (int c = 0; c < 4; ++c) {
                int s1, m1, s2, m2;
                k4_scale_min(2 * c, sc, &s1, &m1);
                k4_scale_min(2 * c + 1, sc, &s2, &m2);
                const float d1 = d * (float)s1, dm1 = dmin * (float)m1;
                const float d2 = d * (float)s2, dm2 = dmin * (float)m2;
                for (int l = 0; l < 32; ++l) {
                    out[s * 256 + c * 64 + l] = d1 * (float)(qs[c * 32 + l] & 0x0F) - dm1;
                    out[s * 256 + c * 64 + 32 + l] = d2 * (float)(qs[c * 32 + l] >> 4) - dm2;
                }
            }
        }
    } else if (t == 14) {                           /* Q6_K: (d*sc)*q, :734-759 */
        for (int32_t s = 0; s < n / 256; ++s) {
            const uint8_t* blk = row + (size_t)s * 210;
            const float d = orc_fp16_to_fp32(rd16(blk + 208)) * 1.0f;
            const uint8_t* ql = blk;
            const uint8_t* qh = blk + 128;
            const int8_t* sc = (const int8_t*)(blk + 192);
            float* y = out + (size_t)s * 256;
            for (int half = 0; half < 2; ++half) {
                for (int l = 0; l < 32; ++l) {
                    const int is = l / 16;
                    const int q1 = (int8_t)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                    const int q2 = (int8_t)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                    const int q3 = (int8_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                    const int q4 = (int8_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                    y[l] = d * (float)sc[is + 0] * (float)q1;
                    y[l + 32] = d * (float)sc[is + 2] * (float)q2;
                    y[l + 64] = d * (float)sc[is + 4] * (float)q3;
                    y[l + 96] = d * (float)sc[is + 6] * (float)q4;
                }
                y += 128; ql += 64; qh += 32; sc += 8;
            }
        }
    } else if (t == 30) {                           /* BF16, :765-780 */
        for (int32_t i = 0; i < n; ++i) out[i] = orc_bf16_to_fp32(rd16(row + 2 * (size_t)i)) * 1.0f;
    } else if (t == 0) {
        memcpy(out, row, (size_t)n * 4);
    }
}

void orc_embed_row(const uint8_t* tensor, int32_t t, int32_t token, int32_t dim, float scale,
                   float* out) {
    const uint8_t* row = tensor + (size_t)token * orc_row_bytes(t, dim);
    if (t == 8) {                                   /* :693-715 */
        for (int32_t b = 0; b < dim / 32; ++b) {
            const uint8_t* blk = row + (size_t)b * 34;
            const float d = orc_fp16_to_fp32(rd16(blk)) * scale;
            for (int j = 0; j < 32; ++j) out[b * 32 + j] = (float)(int8_t)blk[2 + j] * d;
        }
    } else if (t == 14) {                           /* :720-760 */
        for (int32_t s = 0; s < dim / 256; ++s) {
            const uint8_t* blk = row + (size_t)s * 210;
            const float d = orc_fp16_to_fp32(rd16(blk + 208)) * scale;
            const uint8_t* ql = blk;
            const uint8_t* qh = blk + 128;
            const int8_t* sc = (const int8_t*)(blk + 192);
            float* y = out + (size_t)s * 256;
            for (int half = 0; half < 2; ++half) {
                for (int l = 0; l < 32; ++l) {
                    const int is = l / 16;
                    const int q1 = (int8_t)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                    const int q2 = (int8_t)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                    const int q3 = (int8_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                    const int q4 = (int8_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                    y[l] = d * (float)sc[is + 0] * (float)q1;
                    y[l + 32] = d * (float)sc[is + 2] * (float)q2;
                    y[l + 64] = d * (float)sc[is + 4] * (float)q3;
                    y[l + 96] = d * (float)sc[is + 6] * (float)q4;
                }
                y += 128; ql += 64; qh += 32; sc += 8;
            }
        }
    } else if (t == 30) {                           /* :765-780 */
        for (int32_t i = 0; i < dim; ++i) out[i] = orc_bf16_to_fp32(rd16(row + 2 * (size_t)i)) * scale;
    }
}

/* ---- per-block dot products ------------------------------------------ */

/* Q4_0 x Q8 integer dot, :1021-1065: low nibble -> element j, high -> j+16. */
static inline int32_t dot_q4_0(const uint8_t* qs, const int8_t* x) {
    int32_t s = 0;
    for (int j = 0; j < 16; ++j) s += (qs[j] & 0x0F) * x[j] + (qs[j] >> 4) * x[j + 16];
    return s;
}

/* Q8_0 x Q8 integer dot, :1070-1107 */
static inline int32_t dot_q8_0(const int8_t* w, const int8_t* x) {
    int32_t s = 0;
    for (int j = 0; j < 32; ++j) s += w[j] * x[j];
    return s;
}

/* One Q4_K super-block against 8 act blocks, SIMD path of :1127-1178.
 * Returns ((((0 + u0) + u1) + u2) + u3) with
 * u_c = a_lo.d*(d1*dot_lo - dm1*sum_lo) + a_hi.d*(d2*dot_hi - dm2*sum_hi). */
static float sb_q4_k_matvec(const uint8_t* blk, const orc_act_block* a) {
    const float d = orc_fp16_to_fp32(rd16(blk));
    const float dmin = orc_fp16_to_fp32(rd16(blk + 2));
    const uint8_t* sc = blk + 4;
    const uint8_t* q = blk + 16;
    float total = 0.0f;
    for (int c = 0; c < 4; ++c) {
        int s1, m1, s2, m2;
        k4_scale_min(2 * c, sc, &s1, &m1);
        k4_scale_min(2 * c + 1, sc, &s2, &m2);
        const orc_act_block* lo = &a[2 * c];
        const orc_act_block* hi = &a[2 * c + 1];
        int32_t dlo = 0, dhi = 0;
        for (int l = 0; l < 32; ++l) {
            dlo += (q[l] & 0x0F) * lo->qs[l];
            dhi += (q[l] >> 4) * hi->qs[l];
        }
        const float d1 = d * (float)s1, dm1 = dmin * (float)m1;
        const float d2 = d * (float)s2, dm2 = dmin * (float)m2;
        const float ulo = lo->d * (d1 * (float)dlo - dm1 * (float)lo->sum_q);
        const float uhi = hi->d * (d2 * (float)dhi - dm2 * (float)hi->sum_q);
        total = total + (ulo + uhi);
        q += 32;
    }
    return total;
}

/* One Q6_K super-block against 8 act blocks, SIMD path of :1211-1288:
 * four lane accumulators acc_j (j = act block within the 128-half) each
 * summing float(dot - 32*sum_half) * (a_j.d * sc), folded as
 * d * ((acc0 + acc1) + (acc2 + acc3)). */
static float sb_q6_k(const uint8_t* blk, const orc_act_block* a) {
    const float d = orc_fp16_to_fp32(rd16(blk + 208));
    const uint8_t* ql = blk;
    const uint8_t* qh = blk + 128;
    const int8_t* sc = (const int8_t*)(blk + 192);
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int half = 0; half < 2; ++half) {
        const orc_act_block* a4 = a + half * 4;
        for (int is = 0; is < 2; ++is) {
            const int off = is * 16;
            int32_t dots[4] = {0, 0, 0, 0};
            for (int l = off; l < off + 16; ++l) {
                const int q1 = (ql[l] & 0x0F) | (((qh[l] >> 0) & 3) << 4);
                const int q2 = (ql[l + 32] & 0x0F) | (((qh[l] >> 2) & 3) << 4);
                const int q3 = (ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4);
                const int q4 = (ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4);
                dots[0] += q1 * a4[0].qs[l];
                dots[1] += q2 * a4[1].qs[l];
                dots[2] += q3 * a4[2].qs[l];
                dots[3] += q4 * a4[3].qs[l];
            }
            for (int j = 0; j < 4; ++j) {
                const int32_t s = is == 0 ? a4[j].sum_lo : a4[j].sum_hi;
                const int32_t diff = dots[j] - (s << 5);
                const float fsc = a4[j].d * (float)sc[is + 2 * j];
                acc[j] = acc[j] + (float)diff * fsc;
            }
        }
        ql += 64; qh += 32; sc += 8;
    }
    return d * ((acc[0] + acc[1]) + (acc[2] + acc[3]));
}

/* ---- matvec: :1327-1471 ---------------------------------------------- */

static float row_dot(const uint8_t* row, int32_t t, const orc_act_block* act, const float* x,
                     int32_t in_dim) {
    float acc = 0.0f;
    if (t == 2) {
        for (int32_t b = 0; b < in_dim / 32; ++b) {
            if (act[b].d == 0.0f) continue;
            const uint8_t* blk = row + (size_t)b * 18;
            const float w = orc_fp16_to_fp32(rd16(blk));
            const int32_t folded = dot_q4_0(blk + 2, act[b].qs) - 8 * act[b].sum_q;
            acc = acc + (float)folded * (w * act[b].d);
        }
    } else if (t == 8) {
        for (int32_t b = 0; b < in_dim / 32; ++b) {
            const uint8_t* blk = row + (size_t)b * 34;
            const float w = orc_fp16_to_fp32(rd16(blk));
            const int32_t dt = dot_q8_0((const int8_t*)(blk + 2), act[b].qs);
            acc = acc + (float)dt * (w * act[b].d);
        }
    } else if (t == 12) {
        for (int32_t s = 0; s < in_dim / 256; ++s) acc = acc + sb_q4_k_matvec(row + (size_t)s * 144, act + s * 8);
    } else if (t == 14) {
        for (int32_t s = 0; s < in_dim / 256; ++s) acc = acc + sb_q6_k(row + (size_t)s * 210, act + s * 8);
    } else if (t == 30) {                           /* :1432-1461 */
        float l4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        int32_t j = 0;
        for (; j + 3 < in_dim; j += 4)
            for (int k = 0; k < 4; ++k) l4[k] = l4[k] + orc_bf16_to_fp32(rd16(row + 2 * (size_t)(j + k))) * x[j + k];
        acc = l4[0] + l4[1] + l4[2] + l4[3];
        for (; j < in_dim; ++j) acc = acc + orc_bf16_to_fp32(rd16(row + 2 * (size_t)j)) * x[j];
    }
    return acc;
}

typedef struct {
    const uint8_t* w; int32_t t; const orc_act_block* act; const float* x; int32_t in_dim; size_t rb; float* y;
} matvec_ctx;

static void matvec_rows(void* p, int32_t lo, int32_t hi) {
    const matvec_ctx* c = (const matvec_ctx*)p;
    for (int32_t o = lo; o < hi; ++o) c->y[o] = row_dot(c->w + (size_t)o * c->rb, c->t, c->act, c->x, c->in_dim);
}

void orc_matvec(const uint8_t* w, int32_t t, const float* x, int32_t in_dim, int32_t out_dim, float* y) {
    orc_act_block* act = (orc_act_block*)calloc((size_t)(in_dim / 32) + 1, sizeof(orc_act_block));
    orc_act_quantize(x, in_dim, act);
    matvec_ctx c = {w, t, act, x, in_dim, orc_row_bytes(t, in_dim), y};
    par_for(out_dim, matvec_rows, &c);
    free(act);
}

/* ---- matbatch: :1495-1692 -------------------------------------------- */

typedef struct {
    const uint8_t* w; int32_t t; const float* xb; int32_t batch, in_dim, out_dim, nb; size_t rb;
    const orc_act_block* act; float* yb;
} matbatch_ctx;

static void matbatch_rows(void* p, int32_t lo_row, int32_t hi_row) {
    const matbatch_ctx* cx = (const matbatch_ctx*)p;
    const uint8_t* w = cx->w; const int32_t t = cx->t, batch = cx->batch, in_dim = cx->in_dim;
    const int32_t out_dim = cx->out_dim, nb = cx->nb; const size_t rb = cx->rb;
    const orc_act_block* act = cx->act; const float* xb = cx->xb; float* yb = cx->yb;
    for (int32_t o = lo_row; o < hi_row; ++o) {
        const uint8_t* row = w + (size_t)o * rb;
        for (int32_t b = 0; b < batch; ++b) {
            const orc_act_block* a = act + (size_t)b * nb;
            float acc = 0.0f;
            if (t == 2 || t == 8 || t == 14) {
                /* identical per-(token,row) order to the matvec (:1513-1545, :1620-1680);
                 * Q8_0 skips d==0 blocks here (:1664), which adds nothing either way. */
                acc = row_dot(row, t, a, NULL, in_dim);
            } else if (t == 12) {                   /* :1546-1618: acc += ((0 + lo) + hi) per chunk */
                for (int32_t s = 0; s < in_dim / 256; ++s) {
                    const uint8_t* blk = row + (size_t)s * 144;
                    const float d = orc_fp16_to_fp32(rd16(blk));
                    const float dmin = orc_fp16_to_fp32(rd16(blk + 2));
                    const uint8_t* q = blk + 16;
                    for (int c = 0; c < 4; ++c) {
                        int s1, m1, s2, m2;
                        k4_scale_min(2 * c, blk + 4, &s1, &m1);
                        k4_scale_min(2 * c + 1, blk + 4, &s2, &m2);
                        const float d1 = d * (float)s1, dm1 = dmin * (float)m1;
                        const float d2 = d * (float)s2, dm2 = dmin * (float)m2;
                        const orc_act_block* lo = &a[s * 8 + 2 * c];
                        const orc_act_block* hi = &a[s * 8 + 2 * c + 1];
                        float st = 0.0f;
                        if (lo->d != 0.0f) {
                            int32_t dl = 0;
                            for (int l = 0; l < 32; ++l) dl += (q[l] & 0x0F) * lo->qs[l];
                            st = st + lo->d * (d1 * (float)dl - dm1 * (float)lo->sum_q);
                        }
                        if (hi->d != 0.0f) {
                            int32_t dh = 0;
                            for (int l = 0; l < 32; ++l) dh += (q[l] >> 4) * hi->qs[l];
                            st = st + hi->d * (d2 * (float)dh - dm2 * (float)hi->sum_q);
                        }
                        acc = acc + st;
                        q += 32;
                    }
                }
            } else if (t == 30) {                   /* :1682-1690: scalar, one element at a time */
                const float* x = xb + (size_t)b * in_dim;
                for (int32_t j = 0; j < in_dim; ++j) acc = acc + orc_bf16_to_fp32(rd16(row + 2 * (size_t)j)) * x[j];
            }
            yb[(size_t)b * out_dim + o] = acc;
        }
    }
}

void orc_matbatch(const uint8_t* w, int32_t t, const float* xb, int32_t batch, int32_t in_dim,
                  int32_t out_dim, float* yb) {
    const int32_t nb = in_dim / 32;
    orc_act_block* act = (orc_act_block*)calloc((size_t)batch * nb + 1, sizeof(orc_act_block));
    for (int32_t b = 0; b < batch; ++b) orc_act_quantize(xb + (size_t)b * in_dim, in_dim, act + (size_t)b * nb);
    matbatch_ctx c = {w, t, xb, batch, in_dim, out_dim, nb, orc_row_bytes(t, in_dim), act, yb};
    par_for(out_dim, matbatch_rows, &c);
    free(act);
}

/* ---- LM head: :1713-1732 --------------------------------------------- */

void orc_lm_head(const uint8_t* w, int32_t t, const float* h, int32_t dim, int32_t vocab, float softcap,
                 float* logits) {
    orc_matvec(w, t, h, dim, vocab, logits);
    if (softcap > 0.0f) {
        const float inv = 1.0f / softcap;
        for (int32_t v = 0; v < vocab; ++v) logits[v] = tanhf(logits[v] * inv) * softcap;
    }
}

/* ---- RMSNorm ---------------------------------------------------------- */

/* Sum of squares as the reference forms it (:808-825, :908-925): four float
 * lanes over i = 4k+j, then the lanes widened to double and added in order,
 * then any tail element in double. */
static double sum_squares(const float* x, int32_t n) {
    float l4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int32_t i = 0;
    for (; i + 3 < n; i += 4)
        for (int k = 0; k < 4; ++k) l4[k] = l4[k] + x[i + k] * x[i + k];
    double s = (double)l4[0] + (double)l4[1] + (double)l4[2] + (double)l4[3];
    for (; i < n; ++i) {
        const double v = (double)x[i];
        s += v * v;
    }
    return s;
}

/* :789-840 */
void orc_rmsnorm(const float* x, const float* w, int32_t dim, float eps, float* out) {
    const double ss = sum_squares(x, dim);
    const float inv = 1.0f / sqrtf((float)(ss / dim) + eps);
    for (int32_t i = 0; i < dim; ++i) out[i] = x[i] * inv * w[i];
}

/* :895-953 */
void orc_rmsnorm_heads(float* v, const float* w, int32_t n_heads, int32_t hd, float eps) {
    for (int32_t h = 0; h < n_heads; ++h) {
        float* p = v + (size_t)h * hd;
        const double ss = sum_squares(p, hd);
        const float inv = 1.0f / sqrtf((float)(ss / hd) + eps);
        if (w) for (int32_t i = 0; i < hd; ++i) p[i] = p[i] * inv * w[i];
        else   for (int32_t i = 0; i < hd; ++i) p[i] = p[i] * inv;
    }
}

/* ---- RoPE: :1760-1863 -------------------------------------------------- */

void orc_rope_table(int32_t pos, int32_t hd, float base, const float* ff, float* ct, float* st) {
    for (int32_t i = 0; i < hd / 2; ++i) {
        float freq = 1.0f / powf(base, (float)(2 * i) / (float)hd);
        if (ff != NULL && ff[i] != 0.0f) freq /= ff[i];
        const float ang = (float)pos * freq;
        ct[i] = cosf(ang);
        st[i] = sinf(ang);
    }
}

static void rope_heads(float* v, int32_t nh, int32_t hd, const float* ct, const float* st) {
    const int32_t half = hd / 2;
    for (int32_t h = 0; h < nh; ++h) {
        float* p = v + (size_t)h * hd;
        for (int32_t i = 0; i < half; ++i) {
            const float x1 = p[i], x2 = p[i + half];
            p[i] = x1 * ct[i] - x2 * st[i];
            p[i + half] = x2 * ct[i] + x1 * st[i];
        }
    }
}

void orc_rope(float* q, float* k, const float* ff, int32_t nh, int32_t nkv, int32_t hd, int32_t pos,
              float base) {
    float ct[512], st[512];
    orc_rope_table(pos, hd, base, ff, ct, st);
    if (q) rope_heads(q, nh, hd, ct, st);
    if (k) rope_heads(k, nkv, hd, ct, st);
}

/* ---- decode attention: :1887-1994 ------------------------------------- */

/* q.k as the SSE loop forms it (:1925-1946): two 4-lane accumulators over
 * steps of 8, added lane-wise, reduced as (l0+l1)+(l2+l3), tail added last. */
static float qk_dot(const float* q, const float* k, int32_t hd) {
    float a0[4] = {0, 0, 0, 0}, a1[4] = {0, 0, 0, 0};
    int32_t d = 0;
    for (; d + 7 < hd; d += 8)
        for (int j = 0; j < 4; ++j) {
            a0[j] = a0[j] + q[d + j] * k[d + j];
            a1[j] = a1[j] + q[d + 4 + j] * k[d + 4 + j];
        }
    float l[4];
    for (int j = 0; j < 4; ++j) l[j] = a0[j] + a1[j];
    float dot = (l[0] + l[1]) + (l[2] + l[3]);
    for (; d < hd; ++d) dot = dot + q[d] * k[d];
    return dot;
}

typedef struct {
    const float* q; const float* kc; const float* vc; int32_t pos, t0, len, g, hd, kvd; float scale; float* out;
} attn_ctx;

static void attn_heads(void* p, int32_t h0, int32_t h1) {
    const attn_ctx* c = (const attn_ctx*)p;
    float* sc = (float*)malloc((size_t)c->len * 4);
    for (int32_t h = h0; h < h1; ++h) {
        const int32_t kh = h / c->g;
        const float* qh = c->q + (size_t)h * c->hd;
        float* o = c->out + (size_t)h * c->hd;
        float mx = -1e30f;
        for (int32_t t = c->t0; t <= c->pos; ++t) {
            const float s = qk_dot(qh, c->kc + (size_t)t * c->kvd + (size_t)kh * c->hd, c->hd) * c->scale;
            sc[t - c->t0] = s;
            if (s > mx) mx = s;
        }
        float sum = 0.0f;
        for (int32_t i = 0; i < c->len; ++i) {
            const float e = expf(sc[i] - mx);
            sc[i] = e;
            sum += e;
        }
        const float inv = 1.0f / (sum + 1e-12f);
        for (int32_t d = 0; d < c->hd; ++d) o[d] = 0.0f;
        for (int32_t t = c->t0; t <= c->pos; ++t) {
            const float wt = sc[t - c->t0] * inv;
            const float* vt = c->vc + (size_t)t * c->kvd + (size_t)kh * c->hd;
            for (int32_t d = 0; d < c->hd; ++d) o[d] = o[d] + wt * vt[d];
        }
    }
    free(sc);
}

void orc_attention_step(const float* q, const float* k, const float* v, float* kc, float* vc,
                        int32_t pos, int32_t nh, int32_t nkv, int32_t hd, float scale, int32_t window,
                        int32_t write_kv, float* out) {
    const int32_t kvd = nkv * hd;
    if (write_kv && k && v) {
        memcpy(kc + (size_t)pos * kvd, k, (size_t)kvd * 4);
        memcpy(vc + (size_t)pos * kvd, v, (size_t)kvd * 4);
    }
    const int32_t t0 = window > 0 ? (pos - window + 1 > 0 ? pos - window + 1 : 0) : 0;
    attn_ctx c = {q, kc, vc, pos, t0, pos + 1 - t0, nh / nkv, hd, kvd, scale, out};
    /* heads are independent; split them over threads only when the window is long */
    if (c.len >= 256) {
        const int32_t nt = nh;  /* one job per head is plenty */
        pthread_t th[256];
        range_job jobs[256];
        int32_t used = nt < 256 ? nt : 256;
        for (int32_t i = 0; i < used; ++i) {
            jobs[i].fn = attn_heads; jobs[i].ctx = &c;
            jobs[i].lo = (int32_t)((int64_t)nh * i / used);
            jobs[i].hi = (int32_t)((int64_t)nh * (i + 1) / used);
            if (i) pthread_create(&th[i], NULL, range_thunk, &jobs[i]);
        }
        range_thunk(&jobs[0]);
        for (int32_t i = 1; i < used; ++i) pthread_join(th[i], NULL);
    } else {
        attn_heads(&c, 0, nh);
    }
}

/* ---- GLU activations: :2018-2052 -------------------------------------- */

void orc_swiglu(const float* g, const float* u, int32_t n, float* out) {
    for (int32_t i = 0; i < n; ++i) {
        const float x = g[i];
        const float silu = x / (1.0f + expf(-x));
        out[i] = silu * u[i];
    }
}

void orc_geglu(const float* g, const float* u, int32_t n, float* out) {
    const float k0 = 0.7978845608028654f;
    for (int32_t i = 0; i < n; ++i) {
        const float x = g[i];
        const float gelu = 0.5f * x * (1.0f + tanhf(k0 * (x + 0.044715f * x * x * x)));
        out[i] = gelu * u[i];
    }
}

/* ---- greedy sampling: lua/gncx_streamer.lua:1229-1273 ----------------- */

int32_t orc_sample_greedy(const float* logits, int32_t vocab, const int32_t* recent, int32_t n_recent,
                          double penalty) {
    unsigned char* pen = (unsigned char*)calloc((size_t)vocab, 1);
    const int32_t from = n_recent - 65 > 0 ? n_recent - 65 : 0;
    for (int32_t i = from; i < n_recent; ++i)
        if (recent[i] >= 0 && recent[i] < vocab) pen[recent[i]] = 1;
    int32_t best = 0;
    double bv = -1e30;
    for (int32_t i = 0; i < vocab; ++i) {
        double v = (double)logits[i];
        if (pen[i]) v = v > 0 ? v / penalty : v * penalty;
        if (v > bv) { bv = v; best = i; }
    }
    free(pen);
    return best;
}
