// common.cuh -- shared device/host definitions for the B200 hot-path kernels.
//
// Numeric contract: the reference CPU kernels (csrc/gncx_llm_kernels.cpp of
// omega-Core-Dev/gnc-x) integrate quantized weights against activations that
// are themselves re-quantized to int8 per 32 elements, with every scale
// product rounded in fp32 in a fixed source order.  The kernels here
// reproduce that order with explicitly rounded intrinsics (__fmul_rn etc.),
// which nvcc never contracts into FMA, so results are bit-identical to the
// reference evaluated without FMA contraction.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gncx {

// ggml type ids (lua/gncx_gguf.lua:31-47)
enum GgmlType : int32_t {
    kF32 = 0, kF16 = 1, kQ4_0 = 2, kQ8_0 = 8, kQ4_K = 12, kQ6_K = 14, kBF16 = 30,
};

// Status codes returned through gncx_last_error().
enum Status : int32_t {
    kOk = 0,
    kErrInvalidArg = 1,     // null pointer, bad dimension, unsupported type
    kErrUnaligned = 2,      // a pointer the kernel needs aligned is not
    kErrCuda = 3,           // a CUDA runtime call failed
    kErrNoDevice = 4,       // no CUDA device / library used without a GPU
    kErrTimeout = 5,        // a bounded device-side wait gave up
    kErrNotHostAccessible = 6,
    kErrOutOfMemory = 7,
    kErrCapacity = 8,       // request exceeds a fixed-size buffer
};

// Bytes per block and elements per block (lua/gncx_gguf.lua:50-66).
__host__ __device__ inline int block_elems(int32_t t) {
    return (t == kQ4_K || t == kQ6_K) ? 256 : (t == kQ4_0 || t == kQ8_0) ? 32 : 1;
}
__host__ __device__ inline int block_bytes(int32_t t) {
    switch (t) {
        case kQ4_0: return 18;
        case kQ8_0: return 34;
        case kQ4_K: return 144;
        case kQ6_K: return 210;
        case kBF16: return 2;
        case kF16: return 2;
        case kF32: return 4;
        default: return 0;
    }
}
__host__ __device__ inline size_t row_bytes(int32_t t, int64_t n) {
    const int be = block_elems(t);
    return (size_t)(n / be) * (size_t)block_bytes(t);
}

// One re-quantized activation block (csrc/gncx_llm_kernels.cpp:299-306, 955-995),
// 48 bytes so it loads as three 16-byte vectors.
struct alignas(16) ActBlock {
    float d;          // amax / 127 (0 for an all-zero block)
    int32_t sum_lo;   // sum of quants 0..15
    int32_t sum_hi;   // sum of quants 16..31
    int32_t pad;
    int8_t qs[32];
};
static_assert(sizeof(ActBlock) == 48, "ActBlock layout");

// ---- exactly rounded fp32 helpers (never fused) ---------------------------
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ float i2f(int32_t v) { return __int2float_rn(v); }

__device__ __forceinline__ float half_bits_to_float(uint32_t h16) {
    return __half2float(__ushort_as_half((unsigned short)(h16 & 0xFFFFu)));
}
__device__ __forceinline__ float bf16_bits_to_float(uint32_t b16) { return __uint_as_float((b16 & 0xFFFFu) << 16); }

// Correctly rounded exp/tanh in fp32: evaluated in double and rounded once.
// The reference uses the host libm's expf/tanhf, which is within half an ulp
// of this on all but ~1e-4 of inputs.
__device__ __forceinline__ float exp_cr(float x) { return (float)exp((double)x); }
__device__ __forceinline__ float tanh_cr(float x) { return (float)tanh((double)x); }

// GLU activations (csrc/gncx_llm_kernels.cpp:2018-2052), rounding as written there.
__device__ __forceinline__ float swiglu1(float g, float u) {
    const float silu = fdiv(g, fadd(1.0f, exp_cr(-g)));
    return fmul(silu, u);
}
__device__ __forceinline__ float geglu1(float x, float u) {
    const float k0 = 0.7978845608028654f;
    const float inner = fmul(k0, fadd(x, fmul(fmul(fmul(0.044715f, x), x), x)));
    const float gelu = fmul(fmul(0.5f, x), fadd(1.0f, tanh_cr(inner)));
    return fmul(gelu, u);
}

// Bytes [off, off+4) of a little-endian word array as one word, for a
// compile-time offset.
template <int OFF>
__device__ __forceinline__ uint32_t word_at(const uint32_t* w) {
    if constexpr ((OFF & 3) == 0) {
        return w[OFF >> 2];
    } else {
        return __funnelshift_r(w[OFF >> 2], w[(OFF >> 2) + 1], (OFF & 3) * 8);
    }
}
template <int OFF>
__device__ __forceinline__ uint32_t u16_at(const uint32_t* w) {
    return (w[OFF >> 2] >> ((OFF & 3) * 8)) & 0xFFFFu;
}

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

}  // namespace gncx
