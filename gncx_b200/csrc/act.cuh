// act.cuh -- activation re-quantization (fp32 -> int8 per 32 inputs) and its
// shared-memory staging layout, shared by the GEMV and prefill kernels.
//
// Quantization (csrc/gncx_llm_kernels.cpp:955-995): amax over the block,
// d = amax/127, q = nearbyint(x * (127/amax)); an all-zero block has d = 0.
#pragma once
#include "common.cuh"

namespace gncx {

// A 256-input "unit" (8 act blocks) occupies 256 bytes of quants in shared
// memory; its 16-byte chunk k (k = 2*block + half) is stored at chunk
// position k ^ (unit & 7), so eight consecutive units reading the same chunk
// hit eight different bank groups.
struct ActView {
    const int8_t* qs;  // [units*256], swizzled
    const float* d;    // [blocks]
    const int2* s;     // [blocks] (sum of quants 0..15, sum of quants 16..31)
};

__device__ __forceinline__ int act_chunk_pos(int u, int k) { return u * 256 + 16 * (k ^ (u & 7)); }

__device__ __forceinline__ uint4 act_chunk(const ActView& a, int u, int k) {
    return *reinterpret_cast<const uint4*>(a.qs + act_chunk_pos(u, k));
}

// Quantize one 32-input block; returns the 8 packed quant words.
__device__ __forceinline__ void quantize_block32(const float (&v)[32], uint32_t (&q)[8], float& d, int& lo, int& hi) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    lo = 0;
    hi = 0;
    if (amax == 0.0f) {
        d = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = 0u;
        return;
    }
    const float inv = fdiv(127.0f, amax);
    d = fdiv(amax, 127.0f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        uint32_t word = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int e = 4 * i + k;
            const int qv = __float2int_rn(fmul(v[e], inv));
            if (e < 16) lo += qv; else hi += qv;
            word |= ((uint32_t)qv & 0xFFu) << (8 * k);
        }
        q[i] = word;
    }
}

__device__ __forceinline__ void load_block32(const float* x, bool vec16, float (&v)[32]) {
    if (vec16) {
        const float4* p = reinterpret_cast<const float4*>(x);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 t = p[i];
            v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = x[i];
    }
}

// Stage act blocks for `in_dim` inputs into shared memory (thread-strided).
__device__ __forceinline__ void stage_act_fp32(const float* __restrict__ x, int in_dim, int8_t* qs, float* d,
                                               int2* s, int tid, int nthreads) {
    const int nb = in_dim >> 5;
    const bool vec = (((uintptr_t)x) & 15) == 0;
    for (int b = tid; b < nb; b += nthreads) {
        float v[32];
        load_block32(x + (size_t)b * 32, vec, v);
        uint32_t q[8];
        float dd;
        int lo, hi;
        quantize_block32(v, q, dd, lo, hi);
        const int u = b >> 3, j = b & 7;
        *reinterpret_cast<uint4*>(qs + act_chunk_pos(u, 2 * j)) = make_uint4(q[0], q[1], q[2], q[3]);
        *reinterpret_cast<uint4*>(qs + act_chunk_pos(u, 2 * j + 1)) = make_uint4(q[4], q[5], q[6], q[7]);
        d[b] = dd;
        s[b] = make_int2(lo, hi);
    }
}

__device__ __forceinline__ void stage_act_blocks(const ActBlock* __restrict__ ab, int in_dim, int8_t* qs, float* d,
                                                 int2* s, int tid, int nthreads) {
    const int nb = in_dim >> 5;
    for (int b = tid; b < nb; b += nthreads) {
        const uint4* src = reinterpret_cast<const uint4*>(ab + b);
        const uint4 h = src[0];
        const int u = b >> 3, j = b & 7;
        *reinterpret_cast<uint4*>(qs + act_chunk_pos(u, 2 * j)) = src[1];
        *reinterpret_cast<uint4*>(qs + act_chunk_pos(u, 2 * j + 1)) = src[2];
        d[b] = __uint_as_float(h.x);
        s[b] = make_int2((int)h.y, (int)h.z);
    }
}

}  // namespace gncx
