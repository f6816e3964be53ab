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
// The per-block scalars live in 16-byte records {d, sum_lo, sum_hi, sum_q},
// record j of unit u at position u*8 + (j ^ (u & 7)) (same bank spreading).
struct ActView {
    const int8_t* qs;   // [units*256], swizzled
    const float4* rec;  // [units*8], swizzled
};

__device__ __forceinline__ int act_chunk_pos(int u, int k) { return u * 256 + 16 * (k ^ (u & 7)); }
__device__ __forceinline__ int act_rec_pos(int b) { return (b & ~7) | ((b & 7) ^ ((b >> 3) & 7)); }

__device__ __forceinline__ uint4 act_chunk(const ActView& a, int u, int k) {
    const uint32_t addr = (uint32_t)__cvta_generic_to_shared(a.qs) + act_chunk_pos(u, k);
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ float4 act_rec(const ActView& a, int b) {
    const uint32_t addr = (uint32_t)__cvta_generic_to_shared(a.rec) + 16 * act_rec_pos(b);
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
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

// Quantize one quarter (8 inputs) of block b and store it into the
// shared-memory act layout; the four threads of the block run it together
// (amax and sums via shuffles).
__device__ __forceinline__ void act_quant_quarter(const float (&v)[8], bool ok, int b, int q4, int8_t* qs,
                                                  float4* rec) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    uint32_t w0 = 0, w1 = 0;
    int part = 0;
    float d = 0.0f;
    if (amax != 0.0f) {
        const float inv = fdiv(127.0f, amax);
        d = fdiv(amax, 127.0f);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int qv = __float2int_rn(fmul(v[i], inv));
            part += qv;
            if (i < 4) w0 |= ((uint32_t)qv & 0xFFu) << (8 * i);
            else w1 |= ((uint32_t)qv & 0xFFu) << (8 * (i - 4));
        }
    }
    // lanes q4 = 0,1 hold inputs 0..15, lanes 2,3 inputs 16..31
    const int pair = part + __shfl_xor_sync(0xffffffffu, part, 1);
    const int other = __shfl_xor_sync(0xffffffffu, pair, 2);
    if (ok) {
        const int u = b >> 3, j = b & 7;
        // 8-byte piece q4 of the block's 32 quants: chunk 2j + (q4 >> 1), half (q4 & 1)
        uint2* dst = reinterpret_cast<uint2*>(qs + act_chunk_pos(u, 2 * j + (q4 >> 1)) + 8 * (q4 & 1));
        *dst = make_uint2(w0, w1);
        if (q4 == 0) {
            const int lo = pair, hi = other;
            rec[act_rec_pos(b)] = make_float4(d, __int_as_float(lo), __int_as_float(hi), __int_as_float(lo + hi));
        }
    }
}

// Stage act blocks for `in_dim` inputs into shared memory.  Four threads
// quantize one 32-input block (8 inputs each).  A thread's loads for up to
// eight blocks are issued before any of them is quantized, so a long x costs
// one L2 round trip per eight blocks, not one per block.  Must be called by a
// multiple of 32 threads, all of them.  CG: x was written by other CTAs of the
// running kernel, so it is read from L2 (ld.global.cg), never from L1.
template <bool CG = false>
__device__ __forceinline__ void stage_act_fp32(const float* __restrict__ x, int in_dim, int8_t* qs, float4* rec,
                                               int tid, int nthreads) {
    constexpr int K = 8;
    const int nb = in_dim >> 5;
    const bool vec = (((uintptr_t)x) & 15) == 0;
    const int q4 = tid & 3;
    const int step = nthreads >> 2;
    const int iters = (nb + step - 1) / step;  // the same for every thread
    for (int it0 = 0; it0 < iters; it0 += K) {
        float v[K][8];
#pragma unroll
        for (int k = 0; k < K; ++k) {
            const int b = (tid >> 2) + (it0 + k) * step;
            if (it0 + k < iters && b < nb) {
                const float* src = x + (size_t)b * 32 + q4 * 8;
                if (vec) {
                    const float4 t0 = CG ? __ldcg(reinterpret_cast<const float4*>(src)) : reinterpret_cast<const float4*>(src)[0];
                    const float4 t1 = CG ? __ldcg(reinterpret_cast<const float4*>(src) + 1) : reinterpret_cast<const float4*>(src)[1];
                    v[k][0] = t0.x; v[k][1] = t0.y; v[k][2] = t0.z; v[k][3] = t0.w;
                    v[k][4] = t1.x; v[k][5] = t1.y; v[k][6] = t1.z; v[k][7] = t1.w;
                } else {
#pragma unroll
                    for (int i = 0; i < 8; ++i) v[k][i] = CG ? __ldcg(src + i) : src[i];
                }
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) v[k][i] = 0.0f;
            }
        }
#pragma unroll
        for (int k = 0; k < K; ++k) {
            if (it0 + k < iters) {  // uniform: every lane takes part in the shuffles
                const int b = (tid >> 2) + (it0 + k) * step;
                act_quant_quarter(v[k], b < nb, b, q4, qs, rec);
            }
        }
    }
}

__device__ __forceinline__ void stage_act_blocks(const ActBlock* __restrict__ ab, int in_dim, int8_t* qs, float4* rec,
                                                 int tid, int nthreads) {
    const int nb = in_dim >> 5;
    for (int b = tid; b < nb; b += nthreads) {
        const uint4* src = reinterpret_cast<const uint4*>(ab + b);
        const uint4 h = src[0];
        const int u = b >> 3, j = b & 7;
        *reinterpret_cast<uint4*>(qs + act_chunk_pos(u, 2 * j)) = src[1];
        *reinterpret_cast<uint4*>(qs + act_chunk_pos(u, 2 * j + 1)) = src[2];
        rec[act_rec_pos(b)] = make_float4(__uint_as_float(h.x), __uint_as_float(h.y), __uint_as_float(h.z),
                                          __int_as_float((int)h.y + (int)h.z));
    }
}

// Bytes of a staged activation vector: the GEMV's shared-memory act layout
// (swizzled quants, then swizzled {d, sum_lo, sum_hi, sum_q} records), which
// producers write to global memory so the GEMV loads it with one bulk copy.
__host__ __device__ inline size_t staged_act_bytes(int in_dim) { return (size_t)in_dim + (size_t)(in_dim / 32) * 16; }

// Warp-level quantization of one 32-input block (one value per lane): the
// block's quants, scale and sums.
__device__ __forceinline__ void warp_quantize(float v, int lane, int& q, float& d, int& s) {
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    q = 0;
    d = 0.0f;
    if (amax != 0.0f) {
        const float inv = fdiv(127.0f, amax);
        d = fdiv(amax, 127.0f);
        q = __float2int_rn(fmul(v, inv));
    }
    s = q;
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);  // sums of lanes 0..15 / 16..31
}

// ... stored into a staged activation vector (block b of in_dim inputs).
__device__ __forceinline__ void warp_quantize_store_staged(float v, uint8_t* staged, int in_dim, int b, int lane) {
    int q, s;
    float d;
    warp_quantize(v, lane, q, d, s);
    const int u = b >> 3, j = b & 7;
    staged[act_chunk_pos(u, 2 * j + (lane >> 4)) + (lane & 15)] = (uint8_t)(int8_t)q;
    const int hi = __shfl_sync(0xffffffffu, s, 16);
    if (lane == 0) {
        float4* rec = reinterpret_cast<float4*>(staged + in_dim);
        rec[act_rec_pos(b)] = make_float4(d, __int_as_float(s), __int_as_float(hi), __int_as_float(s + hi));
    }
}

// One warp quantizes one 32-input block held one value per lane and stores
// it as an ActBlock (same arithmetic as quantize_block32).
__device__ __forceinline__ void warp_quantize_store(float v, ActBlock* dst, int lane) {
    int q, s;
    float d;
    warp_quantize(v, lane, q, d, s);
    dst->qs[lane] = (int8_t)q;
    if (lane == 0) { dst->d = d; dst->sum_lo = s; dst->pad = 0; }
    if (lane == 16) dst->sum_hi = s;
}

// Staged or block output of a producer kernel: `staged` (one vector, the
// GEMV's shared-memory layout) when non-null, else ActBlocks.
struct ActOut {
    ActBlock* blocks;   // [rows][dim/32]
    uint8_t* staged;    // [staged_act_bytes(dim)], single row
};

__device__ __forceinline__ void act_out_store(const ActOut& o, float v, int dim, size_t row, int b, int lane) {
    if (o.staged) warp_quantize_store_staged(v, o.staged, dim, b, lane);
    else warp_quantize_store(v, o.blocks + row * (size_t)(dim >> 5) + b, lane);
}

}  // namespace gncx
