// matbatch.cu -- batched quantized GEMM for prefill (replaces
// gncx_xfold_universal_matbatch, csrc/gncx_llm_kernels.cpp:1495-1692).
//
// out[t][o] = the reference's per-(token,row) fp32 accumulation of integer
// block dots, reproduced bit for bit: each thread owns whole (token,row)
// accumulators and adds the unit terms in the reference's order (Q4_K adds
// one term per 64-input chunk here, :1546-1618; the other formats add the same
// terms as the matvec).  A CTA computes a 32-row x 32-token tile, staging one
// 256-input unit of weights and activations per step in shared memory; each
// weight unit is unpacked once into registers and reused for four tokens.
#include <cuda_runtime.h>
#include <stdlib.h>
#include "act.cuh"
#include "common.cuh"
#include "kernels.h"
#include "trace.cuh"
#include "units.cuh"

namespace gncx {

constexpr int kMbRows = 32, kMbToks = 32, kMbThreads = 256;

struct TokAct {
    const int8_t* qs;  // this token's 256 staged quants
    int swz;
    const float* dd;   // 8 block scales
    const int2* ss;    // 8 block sums
    __device__ __forceinline__ uint4 chunk(int k) const {
        return *reinterpret_cast<const uint4*>(qs + 16 * (k ^ swz));
    }
    __device__ __forceinline__ float d(int j) const { return dd[j]; }
    __device__ __forceinline__ int2 s(int j) const { return ss[j]; }
    // {d, sum_lo, sum_hi, sum} of block j, as the staged records hold them
    __device__ __forceinline__ float4 rec(int j) const {
        const int2 t = ss[j];
        return make_float4(dd[j], __int_as_float(t.x), __int_as_float(t.y), __int_as_float(t.x + t.y));
    }
};

template <int T>
__global__ void __launch_bounds__(kMbThreads) matbatch_kernel(const uint8_t* __restrict__ w, size_t rb,
                                                               const ActBlock* __restrict__ act, int batch,
                                                               int in_dim, int out_dim, float* __restrict__ y,
                                                               int ldy) {
    GNCX_TRACE_SCOPE(kTagMatbatch, out_dim);
    constexpr int UB = Fmt<T>::UB, NW = Fmt<T>::NW, E = Fmt<T>::E;
    constexpr int WS = (UB + 3) / 4 + 2;  // staged words per row (aligned cover + look-ahead)
    __shared__ __align__(16) uint32_t wsm[kMbRows * WS];
    __shared__ __align__(16) int8_t aq[kMbToks * 256];
    __shared__ float ad[kMbToks * 8];
    __shared__ int2 as[kMbToks * 8];

    const int tid = threadIdx.x;
    const int r = tid >> 3, tg = tid & 7;
    const int row0 = blockIdx.x * kMbRows, tok0 = blockIdx.y * kMbToks;
    const int nb = in_dim >> 5, upr = in_dim >> 8;
    const int grow = row0 + r;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};

    for (int u = 0; u < upr; ++u) {
        // ---- stage weights: the aligned word cover of each row's unit ----
        for (int i = tid; i < kMbRows * WS; i += kMbThreads) {
            const int rr = i / WS, k = i % WS;
            uint32_t v = 0u;
            if (row0 + rr < out_dim) {
                const uint8_t* seg = w + (size_t)(row0 + rr) * rb + (size_t)u * UB;
                const uint32_t* a = reinterpret_cast<const uint32_t*>((uintptr_t)seg & ~(uintptr_t)3);
                const int nwords = (int)((((uintptr_t)seg & 3) + UB + 3) >> 2);
                if (k < nwords) v = __ldg(a + k);
            }
            wsm[i] = v;
        }
        // ---- stage activations of 32 tokens for this unit ----
        for (int i = tid; i < kMbToks * 8; i += kMbThreads) {
            const int tt = i >> 3, j = i & 7;
            const int tok = tok0 + tt;
            uint4 h = make_uint4(0, 0, 0, 0), q0 = h, q1 = h;
            if (tok < batch) {
                const uint4* src = reinterpret_cast<const uint4*>(act + (size_t)tok * nb + u * 8 + j);
                h = src[0]; q0 = src[1]; q1 = src[2];
            }
            const int swz = (tt >> 2) & 7;
            *reinterpret_cast<uint4*>(aq + tt * 256 + 16 * ((2 * j) ^ swz)) = q0;
            *reinterpret_cast<uint4*>(aq + tt * 256 + 16 * ((2 * j + 1) ^ swz)) = q1;
            ad[i] = __uint_as_float(h.x);
            as[i] = make_int2((int)h.y, (int)h.z);
        }
        __syncthreads();
        if (grow < out_dim) {
            const uint8_t* seg = w + (size_t)grow * rb + (size_t)u * UB;
            uint32_t wv[NW];
            load_unit_smem<NW, false>(reinterpret_cast<const uint8_t*>(wsm + r * WS) + ((uintptr_t)seg & 3), wv);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int tt = tg * 4 + i;
                const TokAct ta{aq + tt * 256, (tt >> 2) & 7, ad + tt * 8, as + tt * 8};
                if constexpr (T == kQ4_K) {
                    float st[4];
                    unit_q4_k_batch_terms(wv, ta, st);
#pragma unroll
                    for (int c = 0; c < 4; ++c) acc[i] = fadd(acc[i], st[c]);
                } else {
                    float tv[E];
                    unit_terms<T>(wv, ta, tv);
#pragma unroll
                    for (int e = 0; e < E; ++e) acc[i] = fadd(acc[i], tv[e]);
                }
            }
        }
        __syncthreads();
    }
    if (grow < out_dim) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int tok = tok0 + tg * 4 + i;
            if (tok < batch) y[(size_t)tok * ldy + grow] = acc[i];
        }
    }
}

// BF16 prefill: the reference accumulates one element at a time (:1682-1690).
__global__ void matbatch_bf16_kernel(const uint8_t* __restrict__ w, const float* __restrict__ xb, int batch,
                                     int in_dim, int out_dim, float* __restrict__ y) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= (int64_t)batch * out_dim) return;
    const int t = (int)(i / out_dim), o = (int)(i % out_dim);
    const uint16_t* r = reinterpret_cast<const uint16_t*>(w + (size_t)o * in_dim * 2);
    const float* x = xb + (size_t)t * in_dim;
    float acc = 0.0f;
    for (int j = 0; j < in_dim; ++j) acc = fadd(acc, fmul(bf16_bits_to_float(__ldg(r + j)), x[j]));
    y[i] = acc;
}

int matbatch_launch(const uint8_t* w, int32_t type, const float* xb, const ActBlock* act, int32_t batch,
                    int32_t in_dim, int32_t out_dim, float* yb, int32_t* err, cudaStream_t st, int32_t ldy) {
    (void)err;
    if (ldy <= 0) ldy = out_dim;
    if (!w || !yb || batch < 0 || in_dim <= 0 || out_dim < 0) return kErrInvalidArg;
    if (batch == 0 || out_dim == 0) return kOk;
    if (type == kBF16) {
        if (!xb) return kErrInvalidArg;
        const int64_t n = (int64_t)batch * out_dim;
        if (ldy != out_dim) return kErrInvalidArg;
        matbatch_bf16_kernel<<<(int)((n + 255) / 256), 256, 0, st>>>(w, xb, batch, in_dim, out_dim, yb);
        return cudaPeekAtLastError() == cudaSuccess ? kOk : kErrCuda;
    }
    if (!act || in_dim % 256) return kErrInvalidArg;
    // Q4_0 / Q8_0 / Q4_K on the tensor cores (matbatch_tc.cu) unless disabled
    static const bool use_tc = [] {
        const char* v = getenv("GNCX_MATBATCH_TC");
        return !(v && v[0] == '0');
    }();
    if (use_tc) {
        const int r = matbatch_tc_launch(w, type, act, batch, in_dim, out_dim, yb, err, st, ldy);
        if (r != kErrInvalidArg) return r;
    }
    const size_t rb = row_bytes(type, in_dim);
    dim3 grid((out_dim + kMbRows - 1) / kMbRows, (batch + kMbToks - 1) / kMbToks);
    if (grid.y > 65535) return kErrCapacity;
    switch (type) {
        case kQ4_0: matbatch_kernel<kQ4_0><<<grid, kMbThreads, 0, st>>>(w, rb, act, batch, in_dim, out_dim, yb, ldy); break;
        case kQ8_0: matbatch_kernel<kQ8_0><<<grid, kMbThreads, 0, st>>>(w, rb, act, batch, in_dim, out_dim, yb, ldy); break;
        case kQ4_K: matbatch_kernel<kQ4_K><<<grid, kMbThreads, 0, st>>>(w, rb, act, batch, in_dim, out_dim, yb, ldy); break;
        case kQ6_K: matbatch_kernel<kQ6_K><<<grid, kMbThreads, 0, st>>>(w, rb, act, batch, in_dim, out_dim, yb, ldy); break;
        default: return kErrInvalidArg;
    }
    return cudaPeekAtLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace gncx
