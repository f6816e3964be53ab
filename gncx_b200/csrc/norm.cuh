// norm.cuh -- the reference's RMSNorm scaling factor, reproduced exactly.
#pragma once
#include "common.cuh"

namespace gncx {

// RMSNorm (csrc/gncx_llm_kernels.cpp:789-840, :895-953).
// The reference forms sum(x^2) in four fp32 lanes over i = 4k+j (serial in k),
// widens the lanes to double and adds them in order, adds any tail in double,
// then inv = 1 / sqrtf((float)(sum/n) + eps) and y = (x * inv) * w.  The four
// serial chains are reproduced literally by four threads reading the row from
// shared memory; everything else is parallel.

__device__ __forceinline__ float lds_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    return v;
}

// Serial sum over k of xs[4k+j]^2 (one of the reference's four SSE lanes).
// The next batch's loads are issued (volatile, so in program order) before
// the current batch's adds, so only the fadd chain is serial.
__device__ __forceinline__ float lane_sumsq(const float* xs, int j, int cnt) {
    constexpr int B = 16;
    const uint32_t base = (uint32_t)__cvta_generic_to_shared(xs) + 4u * (uint32_t)j;
    float acc = 0.0f;
    const int kmain = cnt & ~(B - 1);
    if (kmain > 0) {
        float cur[B], nxt[B];
#pragma unroll
        for (int i = 0; i < B; ++i) cur[i] = lds_f32(base + 16u * i);
        for (int k = 0; k < kmain; k += B) {
            const bool more = k + B < kmain;
            if (more) {
#pragma unroll
                for (int i = 0; i < B; ++i) nxt[i] = lds_f32(base + 16u * (k + B + i));
            }
#pragma unroll
            for (int i = 0; i < B; ++i) acc = fadd(acc, fmul(cur[i], cur[i]));
            if (more) {
#pragma unroll
                for (int i = 0; i < B; ++i) cur[i] = nxt[i];
            }
        }
    }
    for (int k = kmain; k < cnt; ++k) {
        const float v = lds_f32(base + 16u * k);
        acc = fadd(acc, fmul(v, v));
    }
    return acc;
}

__device__ __forceinline__ float rms_inv(const float* xs, int n, float eps) {
    // called by all threads; returns inv in every thread
    __shared__ float s_inv;
    const int tid = threadIdx.x;
    if (tid < 32) {
        const int n4 = n & ~3;
        const float acc = tid < 4 ? lane_sumsq(xs, tid, n4 >> 2) : 0.0f;
        const float a1 = __shfl_sync(0xffffffffu, acc, 1);
        const float a2 = __shfl_sync(0xffffffffu, acc, 2);
        const float a3 = __shfl_sync(0xffffffffu, acc, 3);
        if (tid == 0) {
            double s = __dadd_rn(__dadd_rn(__dadd_rn((double)acc, (double)a1), (double)a2), (double)a3);
            for (int i = n4; i < n; ++i) {
                const double v = (double)xs[i];
                s = __dadd_rn(s, __dmul_rn(v, v));
            }
            const float ms = __double2float_rn(__ddiv_rn(s, (double)n));
            s_inv = fdiv(1.0f, __fsqrt_rn(fadd(ms, eps)));
        }
    }
    __syncthreads();
    return s_inv;
}

// The same factor from precomputed squares stored lane-major: sq[j * n4 + k]
// = x[4k+j]^2 (n = 4 * n4, n4 a multiple of 4, sq 16-byte aligned).  Lanes 0-3
// of warp 0 run the four chains with vector loads.
__device__ __forceinline__ float rms_inv_sq(const float* sq, int n4, float eps) {
    __shared__ float s_inv;
    const int tid = threadIdx.x;
    if (tid < 32) {
        float acc = 0.0f;
        if (tid < 4) {
            // a plain unrolled loop: ~5.4 cycles per element on B200, against
            // ~8 for loads pinned ahead with volatile asm and ~4.2 (the fadd
            // latency) with the values already in registers
            const float4* p = reinterpret_cast<const float4*>(sq + (size_t)tid * n4);
#pragma unroll 8
            for (int i = 0; i < (n4 >> 2); ++i) {
                const float4 v = p[i];
                acc = fadd(fadd(fadd(fadd(acc, v.x), v.y), v.z), v.w);
            }
        }
        const float a1 = __shfl_sync(0xffffffffu, acc, 1);
        const float a2 = __shfl_sync(0xffffffffu, acc, 2);
        const float a3 = __shfl_sync(0xffffffffu, acc, 3);
        if (tid == 0) {
            const double s = __dadd_rn(__dadd_rn(__dadd_rn((double)acc, (double)a1), (double)a2), (double)a3);
            const float ms = __double2float_rn(__ddiv_rn(s, (double)(4 * n4)));
            s_inv = fdiv(1.0f, __fsqrt_rn(fadd(ms, eps)));
        }
    }
    __syncthreads();
    return s_inv;
}

}  // namespace gncx
