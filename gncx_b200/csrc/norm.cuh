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

__device__ __forceinline__ float rms_inv(const float* xs, int n, float eps) {
    // called by all threads; returns inv in every thread
    __shared__ float s_inv;
    const int tid = threadIdx.x;
    if (tid < 32) {
        float acc = 0.0f;
        const int n4 = n & ~3;
        if (tid < 4) {
#pragma unroll 8
            for (int i = tid; i < n4; i += 4) {
                const float v = xs[i];
                acc = fadd(acc, fmul(v, v));
            }
        }
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

}  // namespace gncx
