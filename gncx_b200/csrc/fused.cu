// fused.cu -- the model engine's fused per-token kernels.
//
// The fusion boundaries follow the reference's operation order
// (lua/gncx_streamer.lua:780-965), so every fused result equals the unfused
// sequence bit for bit:
//   * residual add -> RMSNorm -> activation re-quantization for the next GEMV
//     (:871-873 / :906-908 then :793-803 / :876-887, and :955-995 in the GEMV);
//   * per-head Q/K RMSNorm -> RoPE -> KV-cache write (:813-862);
//   * SwiGLU / GeGLU -> re-quantization for ffn_down (:893-900);
//   * penalized greedy argmax -> decode state update (:1229-1311), so the token
//     loop runs from device memory under one captured CUDA graph per token.
#include <cuda_runtime.h>
#include <stdlib.h>
#include "act.cuh"
#include "common.cuh"
#include "kernels.h"
#include "trace.cuh"
#include "launch.cuh"
#include "norm.cuh"

namespace gncx {

static int status() { return cudaPeekAtLastError() == cudaSuccess ? kOk : kErrCuda; }

// ---------------------------------------------------------------- add + norm + quantize
// Prefill form, one CTA per row: hidden[r] += residual[r] (if given, written
// back), then y = rmsnorm(hidden[r]) * w, re-quantized to act blocks (and
// optionally stored as fp32 in normed).
__global__ void __launch_bounds__(256) add_norm_quant_kernel(float* hidden, const float* residual,
                                                             const float* __restrict__ w, int dim, float eps,
                                                             ActOut act, float* normed) {
    extern __shared__ float xs[];
    GNCX_TRACE_SCOPE(kTagAddNormQuant, gridDim.x);
    const size_t base = (size_t)blockIdx.x * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
        float v = hidden[base + i];
        if (residual) {
            v = fadd(v, residual[base + i]);
            hidden[base + i] = v;
        }
        xs[i] = v;
    }
    __syncthreads();
    const float inv = rms_inv(xs, dim, eps);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int nb = dim >> 5;
    for (int b = warp; b < nb; b += nwarps) {
        const int i = b * 32 + lane;
        const float v = fmul(fmul(xs[i], inv), w[i]);
        if (normed) normed[base + i] = v;
        act_out_store(act, v, dim, blockIdx.x, b, lane);
    }
}

// Decode form (one row, staged output, one CTA of kRowThreads): the norm gains
// are fetched before the dependency wait; each thread owns 8 consecutive
// inputs per pass, writes their squares lane-major for the four serial chains,
// and after the chains quantizes its 8 outputs (four threads per 32-input
// block).  The next kernel may launch (and prefetch its weights) meanwhile.
constexpr int kRowThreads = 512;
constexpr int kRowPasses = 2;  // dim <= kRowPasses * 8 * kRowThreads

__global__ void __launch_bounds__(kRowThreads) add_norm_quant_row_kernel(float* hidden, const float* residual,
                                                                         const float* __restrict__ w, int dim,
                                                                         float eps, uint8_t* staged, float* normed) {
    extern __shared__ __align__(16) float sq[];  // [4][dim/4]
    GNCX_TRACE_SCOPE(kTagAddNormQuantRow, dim);
    const int tid = threadIdx.x;
    const int n4 = dim >> 2;
    float g[kRowPasses][8];
#pragma unroll
    for (int ps = 0; ps < kRowPasses; ++ps) {
        const int base = (ps * kRowThreads + tid) * 8;
        if (base < dim) {
            const float4 a = __ldg(reinterpret_cast<const float4*>(w + base));
            const float4 b = __ldg(reinterpret_cast<const float4*>(w + base + 4));
            g[ps][0] = a.x; g[ps][1] = a.y; g[ps][2] = a.z; g[ps][3] = a.w;
            g[ps][4] = b.x; g[ps][5] = b.y; g[ps][6] = b.z; g[ps][7] = b.w;
        }
    }
    if (tid == 0) GNCX_TRACE_MARK(20, 0);
    pdl_launch_dependents();
    pdl_wait();
    if (tid == 0) GNCX_TRACE_MARK(21, 0);
    float x[kRowPasses][8];
#pragma unroll
    for (int ps = 0; ps < kRowPasses; ++ps) {
        const int base = (ps * kRowThreads + tid) * 8;
        if (base < dim) {
            float4* h4 = reinterpret_cast<float4*>(hidden + base);
            float4 a = h4[0], b = h4[1];
            if (residual) {
                const float4* r4 = reinterpret_cast<const float4*>(residual + base);
                const float4 ra = r4[0], rb = r4[1];
                a = make_float4(fadd(a.x, ra.x), fadd(a.y, ra.y), fadd(a.z, ra.z), fadd(a.w, ra.w));
                b = make_float4(fadd(b.x, rb.x), fadd(b.y, rb.y), fadd(b.z, rb.z), fadd(b.w, rb.w));
                h4[0] = a;
                h4[1] = b;
            }
            x[ps][0] = a.x; x[ps][1] = a.y; x[ps][2] = a.z; x[ps][3] = a.w;
            x[ps][4] = b.x; x[ps][5] = b.y; x[ps][6] = b.z; x[ps][7] = b.w;
            // inputs base+j and base+4+j belong to chain j at k = base/4 and base/4 + 1
            const int k = base >> 2;
#pragma unroll
            for (int j = 0; j < 4; ++j)
                *reinterpret_cast<float2*>(sq + (size_t)j * n4 + k) =
                    make_float2(fmul(x[ps][j], x[ps][j]), fmul(x[ps][4 + j], x[ps][4 + j]));
        }
    }
    __syncthreads();
    if (tid == 0) GNCX_TRACE_MARK(22, 0);
    const float inv = rms_inv_sq(sq, n4, eps);
    if (tid == 0) GNCX_TRACE_MARK(23, 0);
    const int q4 = tid & 3;
    float4* rec = reinterpret_cast<float4*>(staged + dim);
#pragma unroll
    for (int ps = 0; ps < kRowPasses; ++ps) {
        const int base = (ps * kRowThreads + tid) * 8;
        if (ps * kRowThreads * 8 >= dim) break;  // uniform across the CTA
        const bool ok = base < dim;
        float v[8];
        float amax = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            v[e] = ok ? fmul(fmul(x[ps][e], inv), g[ps][e]) : 0.0f;
            amax = fmaxf(amax, fabsf(v[e]));
        }
        if (ok && normed) {
            reinterpret_cast<float4*>(normed + base)[0] = make_float4(v[0], v[1], v[2], v[3]);
            reinterpret_cast<float4*>(normed + base)[1] = make_float4(v[4], v[5], v[6], v[7]);
        }
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        uint32_t w0 = 0, w1 = 0;
        int part = 0;
        float d = 0.0f;
        if (amax != 0.0f) {
            const float qi = fdiv(127.0f, amax);
            d = fdiv(amax, 127.0f);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int qv = __float2int_rn(fmul(v[e], qi));
                part += qv;
                if (e < 4) w0 |= ((uint32_t)qv & 0xFFu) << (8 * e);
                else w1 |= ((uint32_t)qv & 0xFFu) << (8 * (e - 4));
            }
        }
        const int pair = part + __shfl_xor_sync(0xffffffffu, part, 1);  // quarters 0+1 or 2+3
        const int other = __shfl_xor_sync(0xffffffffu, pair, 2);
        if (ok) {
            const int b = base >> 5;
            *reinterpret_cast<uint2*>(staged + act_chunk_pos(b >> 3, 2 * (b & 7) + (q4 >> 1)) + 8 * (q4 & 1)) =
                make_uint2(w0, w1);
            if (q4 == 0)
                rec[act_rec_pos(b)] = make_float4(d, __int_as_float(pair), __int_as_float(other),
                                                  __int_as_float(pair + other));
        }
    }
}

int add_norm_quant_launch(float* hidden, const float* residual, const float* w, int32_t rows, int32_t dim, float eps,
                          ActOut act, float* normed, cudaStream_t st) {
    if (!hidden || !w || (!act.blocks && !act.staged) || rows < 0 || dim <= 0 || (dim & 31)) return kErrInvalidArg;
    if (act.staged && (rows != 1 || (dim & 255) || ((uintptr_t)act.staged & 15))) return kErrInvalidArg;
    if (rows == 0) return kOk;
    const size_t smem = (size_t)dim * 4;
    if (smem > 200 * 1024) return kErrCapacity;
    const bool vec = ((uintptr_t)hidden & 15) == 0 && ((uintptr_t)residual & 15) == 0 && ((uintptr_t)w & 15) == 0 &&
                     ((uintptr_t)normed & 15) == 0;
    if (act.staged && vec && dim <= kRowPasses * 8 * kRowThreads) {
        if (set_smem_limit(add_norm_quant_row_kernel, smem) != cudaSuccess) return kErrCuda;
        return launch_k(add_norm_quant_row_kernel, dim3(1), dim3(kRowThreads), smem, st, hidden, residual, w, dim,
                        eps, act.staged, normed) == cudaSuccess
                   ? kOk
                   : kErrCuda;
    }
    if (set_smem_limit(add_norm_quant_kernel, smem) != cudaSuccess) return kErrCuda;
    add_norm_quant_kernel<<<rows, 256, smem, st>>>(hidden, residual, w, dim, eps, act, normed);
    return status();
}

// ---------------------------------------------------------------- Q/K norm + RoPE + KV write
// grid (n_heads + 2*n_kv, rows): q heads are normed and rotated in place, k heads
// normed, rotated and written to the cache at the row's position, v heads copied.
__global__ void qkv_post_kernel(float* qkv, int row_stride, int nh, int nkv, int hd, const float* __restrict__ qn,
                                const float* __restrict__ kn, int do_norm, float eps, const float* __restrict__ ct,
                                const float* __restrict__ stab, int pos0, const int* pos_dev, float* kc, float* vc,
                                int64_t kps, int64_t khs) {
    extern __shared__ float xs[];
    GNCX_TRACE_SCOPE(kTagQkvPost, gridDim.x);
    pdl_launch_dependents();
    pdl_wait();
    const int x = blockIdx.x, r = blockIdx.y;
    const int pos = (pos_dev ? *pos_dev : pos0) + r;
    float* row = qkv + (size_t)r * row_stride;
    const int kvd = nkv * hd, qd = nh * hd;
    if (x >= nh + nkv) {
        const int jv = x - nh - nkv;
        const float* src = row + qd + kvd + (size_t)jv * hd;
        float* dst = vc + (size_t)pos * kps + (size_t)jv * khs;
        for (int i = threadIdx.x; i < hd; i += blockDim.x) dst[i] = src[i];
        return;
    }
    const bool isq = x < nh;
    float* vec = isq ? row + (size_t)x * hd : row + qd + (size_t)(x - nh) * hd;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) xs[i] = vec[i];
    __syncthreads();
    const float* w = isq ? qn : kn;
    if (do_norm) {
        const float inv = rms_inv(xs, hd, eps);
        for (int i = threadIdx.x; i < hd; i += blockDim.x) {
            const float v = fmul(xs[i], inv);
            xs[i] = w ? fmul(v, w[i]) : v;
        }
        __syncthreads();
    }
    const int half = hd >> 1;
    float* dst = isq ? vec : kc + (size_t)pos * kps + (size_t)(x - nh) * khs;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        const float c = ct[(size_t)pos * half + i], s = stab[(size_t)pos * half + i];
        const float x1 = xs[i], x2 = xs[i + half];
        dst[i] = fsub(fmul(x1, c), fmul(x2, s));
        dst[i + half] = fadd(fmul(x2, c), fmul(x1, s));
    }
}

int qkv_post_launch(float* qkv, int32_t row_stride, int32_t rows, int32_t nh, int32_t nkv, int32_t hd,
                    const float* q_norm, const float* k_norm, bool do_norm, float eps, const float* cos_tab,
                    const float* sin_tab, int32_t pos0, const int32_t* pos_dev, float* kc, float* vc,
                    int64_t kv_pos_stride, int64_t kv_head_stride, cudaStream_t st) {
    if (!qkv || !cos_tab || !sin_tab || !kc || !vc || rows <= 0 || hd <= 0 || (hd & 1)) return kErrInvalidArg;
    const int threads = hd >= 256 ? 256 : (hd >= 128 ? 128 : 64);
    return launch_k(qkv_post_kernel, dim3(nh + 2 * nkv, rows), dim3(threads), (size_t)hd * 4, st, qkv, row_stride,
                    nh, nkv, hd, q_norm, k_norm, do_norm ? 1 : 0, eps, cos_tab, sin_tab, pos0, pos_dev, kc, vc,
                    kv_pos_stride, kv_head_stride) == cudaSuccess
               ? kOk
               : kErrCuda;
}

// ---------------------------------------------------------------- GLU + quantize
// One warp per 32-output block: out = glu(gate, up), re-quantized for ffn_down.
__global__ void glu_quant_kernel(const float* __restrict__ g, const float* __restrict__ u, int stride, int ffn,
                                 int rows, int gelu, ActOut act, float* out, int out_stride) {
    GNCX_TRACE_SCOPE(kTagGluQuant, ffn);
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x == 0) GNCX_TRACE_MARK(40, 0);
    const int lane = threadIdx.x & 31;
    const int nbf = ffn >> 5;
    const int64_t gw = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int64_t r = gw / nbf;
    if (r >= rows) return;  // whole warp
    const int b = (int)(gw % nbf);
    const size_t i = (size_t)r * stride + (size_t)b * 32 + lane;
    const float v = gelu ? geglu1(g[i], u[i]) : swiglu1(g[i], u[i]);
    if (out) out[(size_t)r * out_stride + (size_t)b * 32 + lane] = v;
    if (act.blocks || act.staged) act_out_store(act, v, ffn, (size_t)r, b, lane);
}

int glu_quant_launch(const float* g, const float* u, int32_t stride, int32_t ffn, int32_t rows, bool gelu,
                     ActOut act, cudaStream_t st, float* out, int32_t out_stride) {
    if (!g || !u || (!act.blocks && !act.staged && !out) || ffn <= 0 || (ffn & 31) || rows < 0) return kErrInvalidArg;
    if (act.staged && (rows != 1 || (ffn & 255) || ((uintptr_t)act.staged & 15))) return kErrInvalidArg;
    if (rows == 0) return kOk;
    const int64_t warps = (int64_t)rows * (ffn >> 5);
    const int64_t blocks = (warps + 7) / 8;
    return launch_k(glu_quant_kernel, dim3((unsigned)blocks), dim3(256), 0, st, g, u, stride, ffn, rows,
                    gelu ? 1 : 0, act, out, out_stride) == cudaSuccess
               ? kOk
               : kErrCuda;
}

// ---------------------------------------------------------------- argmax -> decode state
// lua/gncx_streamer.lua:1229-1273 (penalty over the last <= 65 tokens, doubles,
// first maximum wins) feeding generate (:1276-1311): the chosen token becomes
// the next input, joins the penalty window and the output; EOS stops.
constexpr int kAmThreads = 256;
constexpr int kAmBlocks = kArgmaxParts;

struct Best { double v; int i; };
__device__ __forceinline__ Best pick(Best a, Best b) {
    return (b.v > a.v || (b.v == a.v && b.i < a.i)) ? b : a;
}

__device__ Best am_block_best(Best p) {
    __shared__ double sv[kAmThreads / 32];
    __shared__ int si[kAmThreads / 32];
    for (int o = 16; o > 0; o >>= 1) {
        Best q;
        q.v = __shfl_xor_sync(0xffffffffu, p.v, o);
        q.i = __shfl_xor_sync(0xffffffffu, p.i, o);
        p = pick(p, q);
    }
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = p.v; si[threadIdx.x >> 5] = p.i; }
    __syncthreads();
    if (threadIdx.x == 0)
        for (int k = 1; k < (int)(blockDim.x >> 5); ++k) p = pick(p, Best{sv[k], si[k]});
    return p;
}

// logits[0 .. vocab) are the vocabulary ids idx0 .. idx0 + vocab (a tensor-
// parallel rank's slice); the partial results carry global ids.
__global__ void am_state_stage1(const float* __restrict__ logits, int vocab, int idx0, const DecodeState* st,
                                double penalty, double* part_v, int* part_i) {
    GNCX_TRACE_SCOPE(kTagArgmax1, vocab);
    pdl_launch_dependents();
    pdl_wait();  // the logits come from the preceding kernel
    const int per = (vocab + gridDim.x - 1) / gridDim.x;
    const int lo = blockIdx.x * per, hi = min(vocab, lo + per);
    extern __shared__ unsigned pen[];
    const int words = (per + 31) / 32;
    for (int k = threadIdx.x; k < words; k += blockDim.x) pen[k] = 0u;
    __syncthreads();
    const int n = st->n_all < kRecentWindow ? st->n_all : kRecentWindow;
    for (int k = threadIdx.x; k < n; k += blockDim.x) {
        const int t = st->ring[k] - idx0;
        if (t >= lo && t < hi) atomicOr(&pen[(t - lo) >> 5], 1u << ((t - lo) & 31));
    }
    __syncthreads();
    Best b{-1e30, 0};
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        double v = (double)logits[i];
        if ((pen[(i - lo) >> 5] >> ((i - lo) & 31)) & 1u) v = v > 0.0 ? __ddiv_rn(v, penalty) : __dmul_rn(v, penalty);
        if (v > b.v) { b.v = v; b.i = idx0 + i; }
    }
    b = am_block_best(b);
    if (threadIdx.x == 0) { part_v[blockIdx.x] = b.v; part_i[blockIdx.x] = b.i; }
}

__global__ void am_state_stage2(const double* part_v, const int* part_i, int n, DecodeState* st, int32_t* out_ids,
                                int advance_pos) {
    GNCX_TRACE_SCOPE(kTagArgmax2, n);
    pdl_launch_dependents();
    pdl_wait();
    Best b{-1e30, 0};
    for (int k = threadIdx.x; k < n; k += blockDim.x) b = pick(b, Best{part_v[k], part_i[k]});
    b = am_block_best(b);
    if (threadIdx.x == 0 && !st->done) {
        const int next = b.i;
        if (next == st->eos) {
            st->done = 1;
        } else {
            if (st->n_out < st->max_out) out_ids[st->n_out] = next;
            st->n_out += 1;
            st->ring[st->n_all % kRecentWindow] = next;
            st->n_all += 1;
            st->token = next;
            if (advance_pos) st->pos += 1;
            if (st->n_out >= st->max_out) st->done = 1;
        }
    }
}

size_t argmax_state_scratch_bytes() { return (size_t)kAmBlocks * (sizeof(double) + sizeof(int)); }

int argmax_partials_launch(const float* logits, int32_t vocab, int32_t idx0, const DecodeState* st, double penalty,
                           void* scratch, int32_t* n_parts, cudaStream_t s) {
    if (!logits || !st || !scratch || vocab <= 0 || idx0 < 0) return kErrInvalidArg;
    double* pv = reinterpret_cast<double*>(scratch);
    int* pi = reinterpret_cast<int*>(pv + kAmBlocks);
    const int blocks = vocab < kAmBlocks * 64 ? (vocab + 63) / 64 : kAmBlocks;
    const int per = (vocab + blocks - 1) / blocks;
    *n_parts = blocks;
    return launch_k(am_state_stage1, dim3(blocks), dim3(kAmThreads), (size_t)((per + 31) / 32) * 4, s, logits, vocab,
                    idx0, st, penalty, pv, pi) == cudaSuccess
               ? kOk
               : kErrCuda;
}

int argmax_state_launch(const float* logits, int32_t vocab, DecodeState* st, double penalty, int32_t* out_ids,
                        int advance_pos, void* scratch, cudaStream_t s) {
    if (!logits || !st || !out_ids || !scratch || vocab <= 0) return kErrInvalidArg;
    double* pv = reinterpret_cast<double*>(scratch);
    int* pi = reinterpret_cast<int*>(pv + kAmBlocks);
    const int blocks = vocab < kAmBlocks * 64 ? (vocab + 63) / 64 : kAmBlocks;
    const int per = (vocab + blocks - 1) / blocks;
    if (launch_k(am_state_stage1, dim3(blocks), dim3(kAmThreads), (size_t)((per + 31) / 32) * 4, s, logits, vocab, 0,
                 st, penalty, pv, pi) != cudaSuccess ||
        launch_k(am_state_stage2, dim3(1), dim3(kAmThreads), 0, s, pv, pi, blocks, st, out_ids, advance_pos) !=
            cudaSuccess)
        return kErrCuda;
    return kOk;
}

}  // namespace gncx
