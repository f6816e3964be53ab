// units.cuh -- per-256-input "unit" dot products for each GGUF block format.
//
// A unit is 256 consecutive weights of one row: one Q4_K / Q6_K super-block or
// eight Q4_0 / Q8_0 blocks.  Each function takes the unit's bytes as words
// (already shifted so word 0 starts at the unit) and the staged activations,
// and returns the term(s) the reference adds to its per-row fp32 accumulator,
// each computed with the reference's rounding order:
//   Q4_0  csrc/gncx_llm_kernels.cpp:1362-1382 (+ dot :1021-1065)
//   Q8_0  :1413-1431 (+ dot :1070-1107)
//   Q4_K  :1383-1397 (+ :1112-1120, :1127-1205, SIMD path)
//   Q6_K  :1398-1412 (+ :1211-1288, SIMD path)
#pragma once
#include "act.cuh"
#include "common.cuh"

namespace gncx {

constexpr uint32_t kLo4 = 0x0F0F0F0Fu;
constexpr uint32_t kHi4 = 0xF0F0F0F0u;
constexpr uint32_t kHi2 = 0x30303030u;

// dp4a with unsigned bytes in a and signed bytes in b.  With a = q & kHi4
// (each byte 16 x a high nibble) the sum is exactly 16 x the high-nibble dot,
// so one arithmetic shift of the sum replaces a shift per word.
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

template <int K>
__device__ __forceinline__ int byte_of(const uint32_t* w) {
    return (int)((w[K >> 2] >> ((K & 3) * 8)) & 0xFFu);
}

// 6-bit scale and min of sub-block J from the 12 packed bytes (:1112-1120).
template <int J>
__device__ __forceinline__ void k4_scale_min(const uint32_t* s, int& sc, int& m) {
    if constexpr (J < 4) {
        sc = byte_of<J>(s) & 63;
        m = byte_of<J + 4>(s) & 63;
    } else {
        sc = (byte_of<J + 4>(s) & 0x0F) | ((byte_of<J - 4>(s) >> 6) << 4);
        m = (byte_of<J + 4>(s) >> 4) | ((byte_of<J>(s) >> 6) << 4);
    }
}

// Q4_K super-block term (matvec order): ((((0 + u0) + u1) + u2) + u3),
// u_c = a_lo.d*(d1*dot_lo - dm1*sum_lo) + a_hi.d*(d2*dot_hi - dm2*sum_hi).
template <class A>
__device__ __forceinline__ float unit_q4_k(const uint32_t (&w)[36], const A& a) {
    const float d = half_bits_to_float(w[0]);
    const float dmin = half_bits_to_float(w[0] >> 16);
    const uint32_t* sc = w + 1;
    float total = 0.0f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        int s1, m1, s2, m2;
        if (c == 0) { k4_scale_min<0>(sc, s1, m1); k4_scale_min<1>(sc, s2, m2); }
        if (c == 1) { k4_scale_min<2>(sc, s1, m1); k4_scale_min<3>(sc, s2, m2); }
        if (c == 2) { k4_scale_min<4>(sc, s1, m1); k4_scale_min<5>(sc, s2, m2); }
        if (c == 3) { k4_scale_min<6>(sc, s1, m1); k4_scale_min<7>(sc, s2, m2); }
        const uint4 x0 = a.chunk(4 * c), x1 = a.chunk(4 * c + 1);
        const uint4 y0 = a.chunk(4 * c + 2), y1 = a.chunk(4 * c + 3);
        const uint32_t* q = w + 4 + 8 * c;
        int dlo = 0, dhi = 0;
        dlo = dp4a((int)(q[0] & kLo4), (int)x0.x, dlo);
        dlo = dp4a((int)(q[1] & kLo4), (int)x0.y, dlo);
        dlo = dp4a((int)(q[2] & kLo4), (int)x0.z, dlo);
        dlo = dp4a((int)(q[3] & kLo4), (int)x0.w, dlo);
        dlo = dp4a((int)(q[4] & kLo4), (int)x1.x, dlo);
        dlo = dp4a((int)(q[5] & kLo4), (int)x1.y, dlo);
        dlo = dp4a((int)(q[6] & kLo4), (int)x1.z, dlo);
        dlo = dp4a((int)(q[7] & kLo4), (int)x1.w, dlo);
        dhi = dp4a_us(q[0] & kHi4, (int)y0.x, dhi);
        dhi = dp4a_us(q[1] & kHi4, (int)y0.y, dhi);
        dhi = dp4a_us(q[2] & kHi4, (int)y0.z, dhi);
        dhi = dp4a_us(q[3] & kHi4, (int)y0.w, dhi);
        dhi = dp4a_us(q[4] & kHi4, (int)y1.x, dhi);
        dhi = dp4a_us(q[5] & kHi4, (int)y1.y, dhi);
        dhi = dp4a_us(q[6] & kHi4, (int)y1.z, dhi);
        dhi = dp4a_us(q[7] & kHi4, (int)y1.w, dhi);
        dhi >>= 4;  // exact: the sum is 16 x the high-nibble dot
        const float4 rlo = a.rec(2 * c), rhi = a.rec(2 * c + 1);  // {d, sum_lo, sum_hi, sum}
        const float d1 = fmul(d, i2f(s1)), dm1 = fmul(dmin, i2f(m1));
        const float d2 = fmul(d, i2f(s2)), dm2 = fmul(dmin, i2f(m2));
        const float ulo = fmul(rlo.x, fsub(fmul(d1, i2f(dlo)), fmul(dm1, i2f(__float_as_int(rlo.w)))));
        const float uhi = fmul(rhi.x, fsub(fmul(d2, i2f(dhi)), fmul(dm2, i2f(__float_as_int(rhi.w)))));
        total = fadd(total, fadd(ulo, uhi));
    }
    return total;
}

// Q4_K prefill order (:1546-1618): per 64-input chunk c the reference adds
// sum_t = (0 + lo) + hi to the accumulator, skipping a half whose act scale is 0.
template <class A>
__device__ __forceinline__ void unit_q4_k_batch_terms(const uint32_t (&w)[36], const A& a, float (&out)[4]) {
    const float d = half_bits_to_float(w[0]);
    const float dmin = half_bits_to_float(w[0] >> 16);
    const uint32_t* sc = w + 1;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        int s1, m1, s2, m2;
        if (c == 0) { k4_scale_min<0>(sc, s1, m1); k4_scale_min<1>(sc, s2, m2); }
        if (c == 1) { k4_scale_min<2>(sc, s1, m1); k4_scale_min<3>(sc, s2, m2); }
        if (c == 2) { k4_scale_min<4>(sc, s1, m1); k4_scale_min<5>(sc, s2, m2); }
        if (c == 3) { k4_scale_min<6>(sc, s1, m1); k4_scale_min<7>(sc, s2, m2); }
        const uint4 x0 = a.chunk(4 * c), x1 = a.chunk(4 * c + 1);
        const uint4 y0 = a.chunk(4 * c + 2), y1 = a.chunk(4 * c + 3);
        const uint32_t* q = w + 4 + 8 * c;
        int dlo = 0, dhi = 0;
        dlo = dp4a((int)(q[0] & kLo4), (int)x0.x, dlo);
        dlo = dp4a((int)(q[1] & kLo4), (int)x0.y, dlo);
        dlo = dp4a((int)(q[2] & kLo4), (int)x0.z, dlo);
        dlo = dp4a((int)(q[3] & kLo4), (int)x0.w, dlo);
        dlo = dp4a((int)(q[4] & kLo4), (int)x1.x, dlo);
        dlo = dp4a((int)(q[5] & kLo4), (int)x1.y, dlo);
        dlo = dp4a((int)(q[6] & kLo4), (int)x1.z, dlo);
        dlo = dp4a((int)(q[7] & kLo4), (int)x1.w, dlo);
        dhi = dp4a((int)((q[0] >> 4) & kLo4), (int)y0.x, dhi);
        dhi = dp4a((int)((q[1] >> 4) & kLo4), (int)y0.y, dhi);
        dhi = dp4a((int)((q[2] >> 4) & kLo4), (int)y0.z, dhi);
        dhi = dp4a((int)((q[3] >> 4) & kLo4), (int)y0.w, dhi);
        dhi = dp4a((int)((q[4] >> 4) & kLo4), (int)y1.x, dhi);
        dhi = dp4a((int)((q[5] >> 4) & kLo4), (int)y1.y, dhi);
        dhi = dp4a((int)((q[6] >> 4) & kLo4), (int)y1.z, dhi);
        dhi = dp4a((int)((q[7] >> 4) & kLo4), (int)y1.w, dhi);
        const int2 slo = a.s(2 * c), shi = a.s(2 * c + 1);
        const float alo = a.d(2 * c), ahi = a.d(2 * c + 1);
        const float d1 = fmul(d, i2f(s1)), dm1 = fmul(dmin, i2f(m1));
        const float d2 = fmul(d, i2f(s2)), dm2 = fmul(dmin, i2f(m2));
        float st = 0.0f;
        if (alo != 0.0f) st = fadd(st, fmul(alo, fsub(fmul(d1, i2f(dlo)), fmul(dm1, i2f(slo.x + slo.y)))));
        if (ahi != 0.0f) st = fadd(st, fmul(ahi, fsub(fmul(d2, i2f(dhi)), fmul(dm2, i2f(shi.x + shi.y)))));
        out[c] = st;
    }
}

// Q6_K super-block term: four lane accumulators, d * ((acc0+acc1) + (acc2+acc3)).
template <class A>
__device__ __forceinline__ float unit_q6_k(const uint32_t (&w)[53], const A& a) {
    const float d = half_bits_to_float(w[52]);
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int is = 0; is < 2; ++is) {
            int dots[4] = {0, 0, 0, 0};
            uint4 x[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) x[j] = a.chunk(2 * (4 * h + j) + is);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t W = w[16 * h + 4 * is + i];
                const uint32_t W32 = w[16 * h + 8 + 4 * is + i];
                const uint32_t H = w[32 + 8 * h + 4 * is + i];
                const uint32_t q1 = (W & kLo4) | ((H << 4) & kHi2);
                const uint32_t q2 = (W32 & kLo4) | ((H << 2) & kHi2);
                const uint32_t q3 = ((W >> 4) & kLo4) | (H & kHi2);
                const uint32_t q4 = ((W32 >> 4) & kLo4) | ((H >> 2) & kHi2);
                const uint32_t xa = i == 0 ? x[0].x : i == 1 ? x[0].y : i == 2 ? x[0].z : x[0].w;
                const uint32_t xb = i == 0 ? x[1].x : i == 1 ? x[1].y : i == 2 ? x[1].z : x[1].w;
                const uint32_t xc = i == 0 ? x[2].x : i == 1 ? x[2].y : i == 2 ? x[2].z : x[2].w;
                const uint32_t xd = i == 0 ? x[3].x : i == 1 ? x[3].y : i == 2 ? x[3].z : x[3].w;
                dots[0] = dp4a((int)q1, (int)xa, dots[0]);
                dots[1] = dp4a((int)q2, (int)xb, dots[1]);
                dots[2] = dp4a((int)q3, (int)xc, dots[2]);
                dots[3] = dp4a((int)q4, (int)xd, dots[3]);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int2 ss = a.s(4 * h + j);
                const int sh = is == 0 ? ss.x : ss.y;
                const int diff = dots[j] - (sh << 5);
                const int scb = 192 + 8 * h + is + 2 * j;
                const int sc = (int)(int8_t)((w[scb >> 2] >> ((scb & 3) * 8)) & 0xFFu);
                const float fsc = fmul(a.d(4 * h + j), i2f(sc));
                acc[j] = fadd(acc[j], fmul(i2f(diff), fsc));
            }
        }
    }
    return fmul(d, fadd(fadd(acc[0], acc[1]), fadd(acc[2], acc[3])));
}

// Eight Q4_0 block terms: (float)(dot - 8*sum_q) * (d_w * d_a), or 0 when d_a == 0
// (the reference skips those blocks; adding +0 to a never-negative-zero
// accumulator is the same).
template <int B, class A>
__device__ __forceinline__ float q4_0_block(const uint32_t (&w)[36], const A& a) {
    const float wd = half_bits_to_float(u16_at<18 * B>(w));
    const uint4 x0 = a.chunk(2 * B), x1 = a.chunk(2 * B + 1);
    const uint32_t q0 = word_at<18 * B + 2>(w), q1 = word_at<18 * B + 6>(w);
    const uint32_t q2 = word_at<18 * B + 10>(w), q3 = word_at<18 * B + 14>(w);
    int dot = 0;
    dot = dp4a((int)(q0 & kLo4), (int)x0.x, dot);
    dot = dp4a((int)(q1 & kLo4), (int)x0.y, dot);
    dot = dp4a((int)(q2 & kLo4), (int)x0.z, dot);
    dot = dp4a((int)(q3 & kLo4), (int)x0.w, dot);
    int hi = 0;
    hi = dp4a_us(q0 & kHi4, (int)x1.x, hi);
    hi = dp4a_us(q1 & kHi4, (int)x1.y, hi);
    hi = dp4a_us(q2 & kHi4, (int)x1.z, hi);
    hi = dp4a_us(q3 & kHi4, (int)x1.w, hi);
    dot += hi >> 4;  // exact: the sum is 16 x the high-nibble dot
    const float4 r = a.rec(B);  // {d, sum_lo, sum_hi, sum}
    const float ad = r.x;
    const int folded = dot - 8 * __float_as_int(r.w);
    return ad == 0.0f ? 0.0f : fmul(i2f(folded), fmul(wd, ad));
}

template <class A>
__device__ __forceinline__ void unit_q4_0(const uint32_t (&w)[36], const A& a, float (&t)[8]) {
    t[0] = q4_0_block<0>(w, a);
    t[1] = q4_0_block<1>(w, a);
    t[2] = q4_0_block<2>(w, a);
    t[3] = q4_0_block<3>(w, a);
    t[4] = q4_0_block<4>(w, a);
    t[5] = q4_0_block<5>(w, a);
    t[6] = q4_0_block<6>(w, a);
    t[7] = q4_0_block<7>(w, a);
}

// Eight Q8_0 block terms: (float)dot * (d_w * d_a).
template <int B, class A>
__device__ __forceinline__ float q8_0_block(const uint32_t (&w)[68], const A& a) {
    const float wd = half_bits_to_float(u16_at<34 * B>(w));
    const uint4 x0 = a.chunk(2 * B), x1 = a.chunk(2 * B + 1);
    int dot = 0;
    dot = dp4a((int)word_at<34 * B + 2>(w), (int)x0.x, dot);
    dot = dp4a((int)word_at<34 * B + 6>(w), (int)x0.y, dot);
    dot = dp4a((int)word_at<34 * B + 10>(w), (int)x0.z, dot);
    dot = dp4a((int)word_at<34 * B + 14>(w), (int)x0.w, dot);
    dot = dp4a((int)word_at<34 * B + 18>(w), (int)x1.x, dot);
    dot = dp4a((int)word_at<34 * B + 22>(w), (int)x1.y, dot);
    dot = dp4a((int)word_at<34 * B + 26>(w), (int)x1.z, dot);
    dot = dp4a((int)word_at<34 * B + 30>(w), (int)x1.w, dot);
    return fmul(i2f(dot), fmul(wd, a.rec(B).x));
}

template <class A>
__device__ __forceinline__ void unit_q8_0(const uint32_t (&w)[68], const A& a, float (&t)[8]) {
    t[0] = q8_0_block<0>(w, a);
    t[1] = q8_0_block<1>(w, a);
    t[2] = q8_0_block<2>(w, a);
    t[3] = q8_0_block<3>(w, a);
    t[4] = q8_0_block<4>(w, a);
    t[5] = q8_0_block<5>(w, a);
    t[6] = q8_0_block<6>(w, a);
    t[7] = q8_0_block<7>(w, a);
}

// Accessor over the staged activations of the unit being processed.
struct UnitAct {
    const ActView& a;
    int u;
    __device__ __forceinline__ uint4 chunk(int k) const { return act_chunk(a, u, k); }
    __device__ __forceinline__ float4 rec(int j) const { return act_rec(a, u * 8 + j); }
    __device__ __forceinline__ float d(int j) const { return act_rec(a, u * 8 + j).x; }
    __device__ __forceinline__ int2 s(int j) const {
        const float4 r = act_rec(a, u * 8 + j);
        return make_int2(__float_as_int(r.y), __float_as_int(r.z));
    }
};

// Format traits: unit bytes, words loaded per unit, terms per unit.
template <int T> struct Fmt;
template <> struct Fmt<kQ4_0> { static constexpr int UB = 144, NW = 36, E = 8; };
template <> struct Fmt<kQ8_0> { static constexpr int UB = 272, NW = 68, E = 8; };
template <> struct Fmt<kQ4_K> { static constexpr int UB = 144, NW = 36, E = 1; };
template <> struct Fmt<kQ6_K> { static constexpr int UB = 210, NW = 53, E = 1; };

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

// Load NW words of a unit from shared memory at byte address p.
template <int NW, bool ALIGNED>
__device__ __forceinline__ void load_unit_smem(const uint8_t* p, uint32_t (&w)[NW]) {
    const uint32_t sp = (uint32_t)__cvta_generic_to_shared(p);
    if constexpr (ALIGNED) {
        static_assert(NW % 4 == 0, "aligned unit loads need whole 16-byte chunks");
#pragma unroll
        for (int i = 0; i < NW / 4; ++i) {
            const uint4 t = lds128(sp + 16 * i);
            w[4 * i] = t.x; w[4 * i + 1] = t.y; w[4 * i + 2] = t.z; w[4 * i + 3] = t.w;
        }
    } else {
        const uint32_t a = sp & ~3u;
        const uint32_t sh = (sp & 3u) * 8u;
        uint32_t prev = lds32(a);
#pragma unroll
        for (int i = 0; i < NW; ++i) {
            const uint32_t nxt = lds32(a + 4 * (i + 1));
            w[i] = __funnelshift_r(prev, nxt, sh);
            prev = nxt;
        }
    }
}

// Compute the E terms of one unit.
template <int T, class A>
__device__ __forceinline__ void unit_terms(const uint32_t (&w)[Fmt<T>::NW], const A& a, float (&t)[Fmt<T>::E]) {
    if constexpr (T == kQ4_K) t[0] = unit_q4_k(w, a);
    else if constexpr (T == kQ6_K) t[0] = unit_q6_k(w, a);
    else if constexpr (T == kQ4_0) unit_q4_0(w, a, t);
    else unit_q8_0(w, a, t);
}

}  // namespace gncx
