// ops.cu -- the small hot-path kernels: activation quantization, block
// dequantization / embedding fetch, RMSNorm, per-head RMSNorm, RoPE, GLU
// activations, logit softcap and penalized greedy argmax.
#include <cuda_runtime.h>
#include <float.h>
#include "act.cuh"
#include "common.cuh"
#include "kernels.h"
#include "trace.cuh"
#include "launch.cuh"
#include "norm.cuh"

namespace gncx {

static int launch_status() { return cudaPeekAtLastError() == cudaSuccess ? kOk : kErrCuda; }

// ---------------- activation quantization (:955-995) ----------------
__global__ void act_quantize_kernel(const float* __restrict__ x, int rows, int in_dim, ActBlock* __restrict__ out) {
    const int nb = in_dim >> 5;
    const int64_t total = (int64_t)rows * nb;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / nb, b = i % nb;
        const float* src = x + r * in_dim + b * 32;
        float v[32];
        load_block32(src, ((uintptr_t)src & 15) == 0, v);
        uint32_t q[8];
        float d;
        int lo, hi;
        quantize_block32(v, q, d, lo, hi);
        uint4* dst = reinterpret_cast<uint4*>(out + i);
        dst[0] = make_uint4(__float_as_uint(d), (uint32_t)lo, (uint32_t)hi, 0u);
        dst[1] = make_uint4(q[0], q[1], q[2], q[3]);
        dst[2] = make_uint4(q[4], q[5], q[6], q[7]);
    }
}

int act_quantize_launch(const float* x, int32_t rows, int32_t in_dim, ActBlock* out, cudaStream_t st) {
    if (!x || !out || rows < 0 || in_dim <= 0 || (in_dim & 31)) return kErrInvalidArg;
    const int64_t total = (int64_t)rows * (in_dim >> 5);
    if (total == 0) return kOk;
    const int threads = 128;
    const int blocks = (int)((total + threads - 1) / threads < 65535 ? (total + threads - 1) / threads : 65535);
    act_quantize_kernel<<<blocks, threads, 0, st>>>(x, rows, in_dim, out);
    return launch_status();
}

__global__ void act_stage_kernel(const ActBlock* __restrict__ blocks, int in_dim, uint8_t* __restrict__ staged) {
    stage_act_blocks(blocks, in_dim, reinterpret_cast<int8_t*>(staged), reinterpret_cast<float4*>(staged + in_dim),
                     blockIdx.x * blockDim.x + threadIdx.x, gridDim.x * blockDim.x);
}

int act_stage_launch(const ActBlock* blocks, int32_t in_dim, uint8_t* staged, cudaStream_t st) {
    if (!blocks || !staged || in_dim <= 0 || (in_dim & 255) || ((uintptr_t)staged & 15)) return kErrInvalidArg;
    const int nb = in_dim >> 5;
    act_stage_kernel<<<(nb + 127) / 128, 128, 0, st>>>(blocks, in_dim, staged);
    return launch_status();
}

// ---------------- dequantization / embedding rows ----------------
// Element e of a row, following the reference fetch routines (:693-780) with
// scale factor `scale` applied to the block scale first (scale 1.0 is exact).
__device__ __forceinline__ float dequant_elem(const uint8_t* row, int32_t type, int e, float scale) {
    switch (type) {
        case kQ8_0: {
            const uint8_t* blk = row + (e >> 5) * 34;
            const float d = fmul(half_bits_to_float(blk[0] | (blk[1] << 8)), scale);
            return fmul(i2f((int8_t)blk[2 + (e & 31)]), d);
        }
        case kQ4_0: {
            const uint8_t* blk = row + (e >> 5) * 18;
            const float d = fmul(half_bits_to_float(blk[0] | (blk[1] << 8)), scale);
            const int j = e & 31;
            const int q = j < 16 ? (blk[2 + j] & 0x0F) : (blk[2 + j - 16] >> 4);
            return fmul(d, i2f(q - 8));
        }
        case kQ4_K: {
            const uint8_t* blk = row + (e >> 8) * 144;
            const float d = fmul(half_bits_to_float(blk[0] | (blk[1] << 8)), scale);
            const float dmin = fmul(half_bits_to_float(blk[2] | (blk[3] << 8)), scale);
            const uint8_t* s = blk + 4;
            const int j = e & 255, c = j >> 6, hi = (j >> 5) & 1, l = j & 31;
            const int sb = 2 * c + hi;
            int sc, m;
            if (sb < 4) { sc = s[sb] & 63; m = s[sb + 4] & 63; }
            else { sc = (s[sb + 4] & 0x0F) | ((s[sb - 4] >> 6) << 4); m = (s[sb + 4] >> 4) | ((s[sb] >> 6) << 4); }
            const int qb = blk[16 + c * 32 + l];
            const int q = hi ? (qb >> 4) : (qb & 0x0F);
            return fsub(fmul(fmul(d, i2f(sc)), i2f(q)), fmul(dmin, i2f(m)));
        }
        case kQ6_K: {
            const uint8_t* blk = row + (e >> 8) * 210;
            const float d = fmul(half_bits_to_float(blk[208] | (blk[209] << 8)), scale);
            const int j = e & 255, half = j >> 7, r = j & 127, quad = r >> 5, l = r & 31;
            const uint8_t* ql = blk + 64 * half;
            const uint8_t* qh = blk + 128 + 32 * half;
            const int8_t* sc = reinterpret_cast<const int8_t*>(blk + 192 + 8 * half);
            int q;
            if (quad == 0) q = (ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4);
            else if (quad == 1) q = (ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4);
            else if (quad == 2) q = (ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4);
            else q = (ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4);
            const int is = l / 16;
            return fmul(fmul(d, i2f(sc[is + 2 * quad])), i2f(q - 32));
        }
        case kBF16:
            return fmul(bf16_bits_to_float(row[2 * e] | (row[2 * e + 1] << 8)), scale);
        case kF16:
            return fmul(half_bits_to_float(row[2 * e] | (row[2 * e + 1] << 8)), scale);
        default: {
            const float v = __uint_as_float((uint32_t)row[4 * e] | ((uint32_t)row[4 * e + 1] << 8) |
                                            ((uint32_t)row[4 * e + 2] << 16) | ((uint32_t)row[4 * e + 3] << 24));
            return fmul(v, scale);
        }
    }
}

__global__ void dequant_kernel(const uint8_t* __restrict__ w, int32_t type, int32_t rows, int32_t n, float scale,
                               const int32_t* __restrict__ row_ids, float* __restrict__ out) {
    GNCX_TRACE_SCOPE(kTagDequant, rows);
    pdl_launch_dependents();
    pdl_wait();  // row ids (the decode step's token) come from the preceding kernel
    const size_t rb = row_bytes(type, n);
    const int64_t total = (int64_t)rows * n;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / n;
        const int e = (int)(i % n);
        const int64_t src_row = row_ids ? (int64_t)row_ids[r] : r;
        out[i] = dequant_elem(w + (size_t)src_row * rb, type, e, scale);
    }
}

int dequant_launch(const uint8_t* w, int32_t type, int32_t rows, int32_t n, float scale, const int32_t* row_ids,
                   float* out, cudaStream_t st) {
    if (!w || !out || rows < 0 || n <= 0) return kErrInvalidArg;
    if (type != kQ4_0 && type != kQ8_0 && type != kQ4_K && type != kQ6_K && type != kBF16 && type != kF16 &&
        type != kF32)
        return kErrInvalidArg;
    if (n % block_elems(type)) return kErrInvalidArg;
    const int64_t total = (int64_t)rows * n;
    if (total == 0) return kOk;
    const int threads = 256;
    const int64_t want = (total + threads - 1) / threads;
    return launch_k(dequant_kernel, dim3((unsigned)(want < 65535 ? want : 65535)), dim3(threads), 0, st, w, type, rows,
                    n, scale, row_ids, out) == cudaSuccess
               ? kOk
               : kErrCuda;
}

int embed_launch(const uint8_t* tensor, int32_t type, const int32_t* tokens, int32_t n_tokens, int32_t dim,
                 float scale, float* out, cudaStream_t st) {
    if (type != kQ8_0 && type != kQ6_K && type != kBF16) return kErrInvalidArg;
    return dequant_launch(tensor, type, n_tokens, dim, scale, tokens, out, st);
}

// ---------------- RMSNorm (:789-840, :895-953): see norm.cuh ----------------
constexpr int kNormThreads = 256;

// One CTA per (row, head); rows of `n_heads * head_dim` floats; out may alias x.
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const float* x, const float* __restrict__ w, float* out,
                                                               int n_heads, int head_dim, float eps) {
    extern __shared__ float xs[];
    const size_t base = (size_t)blockIdx.x * head_dim;  // blockIdx.x = row * n_heads + head
    for (int i = threadIdx.x; i < head_dim; i += blockDim.x) xs[i] = x[base + i];
    __syncthreads();
    const float inv = rms_inv(xs, head_dim, eps);
    for (int i = threadIdx.x; i < head_dim; i += blockDim.x) {
        const float v = fmul(xs[i], inv);
        out[base + i] = w ? fmul(v, w[i]) : v;
    }
}

int rmsnorm_launch(const float* x, const float* w, int32_t rows, int32_t dim, float eps, float* out,
                   cudaStream_t st) {
    if (!x || !w || !out || rows < 0 || dim <= 0) return kErrInvalidArg;
    if (rows == 0) return kOk;
    const size_t smem = (size_t)dim * 4;
    if (smem > 200 * 1024) return kErrCapacity;
    if (set_smem_limit(rmsnorm_kernel, smem) != cudaSuccess) return kErrCuda;
    rmsnorm_kernel<<<rows, kNormThreads, smem, st>>>(x, w, out, 1, dim, eps);
    return launch_status();
}

int rmsnorm_heads_launch(float* v, const float* w, int32_t rows, int32_t n_heads, int32_t head_dim, float eps,
                         cudaStream_t st) {
    if (!v || rows < 0 || n_heads <= 0 || head_dim <= 0) return kErrInvalidArg;
    if (rows == 0) return kOk;
    const size_t smem = (size_t)head_dim * 4;
    if (smem > 200 * 1024) return kErrCapacity;
    if (set_smem_limit(rmsnorm_kernel, smem) != cudaSuccess) return kErrCuda;
    const int threads = head_dim >= 256 ? 256 : 128;
    rmsnorm_kernel<<<rows * n_heads, threads, smem, st>>>(v, w, v, n_heads, head_dim, eps);
    return launch_status();
}

// ---------------- RoPE (:1760-1863) ----------------
// x1' = x1*c - x2*s ; x2' = x2*c + x1*s with the reference's cos/sin table.
__global__ void rope_kernel(float* v, int rows, int row_stride, int n_heads, int head_dim, int pos0,
                            const float* __restrict__ ct, const float* __restrict__ stab) {
    const int half = head_dim >> 1;
    const int64_t total = (int64_t)rows * n_heads * half;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int k = (int)(i % half);
        const int64_t rh = i / half;
        const int h = (int)(rh % n_heads);
        const int r = (int)(rh / n_heads);
        const int pos = pos0 + r;
        const float c = ct[(size_t)pos * half + k], s = stab[(size_t)pos * half + k];
        float* p = v + (size_t)r * row_stride + (size_t)h * head_dim;
        const float x1 = p[k], x2 = p[k + half];
        p[k] = fsub(fmul(x1, c), fmul(x2, s));
        p[k + half] = fadd(fmul(x2, c), fmul(x1, s));
    }
}

int rope_launch(float* v, int32_t rows, int32_t row_stride, int32_t n_heads, int32_t head_dim, int32_t pos0,
                const float* cos_tab, const float* sin_tab, cudaStream_t st) {
    if (!v || !cos_tab || !sin_tab || rows < 0 || n_heads < 0 || head_dim <= 0 || (head_dim & 1)) return kErrInvalidArg;
    const int64_t total = (int64_t)rows * n_heads * (head_dim / 2);
    if (total == 0) return kOk;
    const int threads = 256;
    const int64_t want = (total + threads - 1) / threads;
    rope_kernel<<<(int)(want < 65535 ? want : 65535), threads, 0, st>>>(v, rows, row_stride, n_heads, head_dim, pos0,
                                                                      cos_tab, sin_tab);
    return launch_status();
}

// Single-position variant for the reference-shaped entry point: the cos/sin
// table travels in the kernel parameters (head_dim/2 <= 256).
__global__ void rope_tab_kernel(float* q, float* k, int nh, int nkv, int hd, const RopeTab tab) {
    const int half = hd >> 1;
    const int total = (nh + nkv) * half;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const int h = i / half, kk = i % half;
        float* p = h < nh ? q + (size_t)h * hd : k + (size_t)(h - nh) * hd;
        if (!p) continue;
        const float c = tab.c[kk], s = tab.s[kk];
        const float x1 = p[kk], x2 = p[kk + half];
        p[kk] = fsub(fmul(x1, c), fmul(x2, s));
        p[kk + half] = fadd(fmul(x2, c), fmul(x1, s));
    }
}

int rope_tab_launch(float* q, float* k, int32_t nh, int32_t nkv, int32_t hd, const RopeTab& tab, cudaStream_t st) {
    if (hd <= 0 || (hd & 1) || hd / 2 > 256) return kErrInvalidArg;
    const int n_q = q ? nh : 0, n_k = k ? nkv : 0;
    if (n_q == 0 && n_k == 0) return kOk;
    // rows of q first, then k; a null side contributes no rows
    const int total = (n_q + n_k) * (hd / 2);
    rope_tab_kernel<<<(total + 255) / 256, 256, 0, st>>>(n_q ? q : k, n_q ? k : nullptr, n_q ? n_q : n_k, n_q ? n_k : 0,
                                                         hd, tab);
    return launch_status();
}

// max |x| over n floats -> *out (one CTA)
__global__ void absmax_kernel(const float* __restrict__ x, int n, float* out) {
    float m = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, fabsf(x[i]));
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    __shared__ float w[32];
    if ((threadIdx.x & 31) == 0) w[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < (int)(blockDim.x >> 5); ++k) m = fmaxf(m, w[k]);
        *out = fmaxf(m, w[0]);
    }
}

int absmax_launch(const float* x, int32_t n, float* out, cudaStream_t st) {
    if (!x || !out || n < 0) return kErrInvalidArg;
    absmax_kernel<<<1, 256, 0, st>>>(x, n, out);
    return launch_status();
}

// ---------------- GLU activations (:2018-2052) ----------------
__global__ void glu_kernel(const float* __restrict__ g, const float* __restrict__ u, int64_t n, float* out, int gelu) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = gelu ? geglu1(g[i], u[i]) : swiglu1(g[i], u[i]);
}

int glu_launch(const float* g, const float* u, int64_t n, float* out, bool gelu, cudaStream_t st) {
    if (!g || !u || !out || n < 0) return kErrInvalidArg;
    if (n == 0) return kOk;
    const int threads = 256;
    const int64_t want = (n + threads - 1) / threads;
    glu_kernel<<<(int)(want < 65535 ? want : 65535), threads, 0, st>>>(g, u, n, out, gelu ? 1 : 0);
    return launch_status();
}

__global__ void softcap_kernel(float* x, int64_t n, float cap) {
    const float inv = fdiv(1.0f, cap);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        x[i] = fmul(tanh_cr(fmul(x[i], inv)), cap);
}

int softcap_launch(float* x, int64_t n, float cap, cudaStream_t st) {
    if (!x || n < 0) return kErrInvalidArg;
    if (n == 0 || !(cap > 0.0f)) return kOk;
    const int threads = 256;
    const int64_t want = (n + threads - 1) / threads;
    softcap_kernel<<<(int)(want < 65535 ? want : 65535), threads, 0, st>>>(x, n, cap);
    return launch_status();
}

// ---------------- penalized greedy argmax (lua/gncx_streamer.lua:1229-1273) ----------------
// Values are compared as doubles exactly like the Lua scan: logits of the last
// <=65 recent tokens become v/p (v > 0) or v*p; the first maximum wins; the
// running best starts at (-1e30, index 0).
constexpr int kArgmaxThreads = 256;
constexpr int kArgmaxBlocks = 148;

struct BestPair { double v; int i; };

__device__ __forceinline__ BestPair better(BestPair a, BestPair b) {
    if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
    return a;
}

__device__ BestPair block_best(BestPair p) {
    __shared__ double sv[kArgmaxThreads / 32];
    __shared__ int si[kArgmaxThreads / 32];
    for (int o = 16; o > 0; o >>= 1) {
        BestPair q;
        q.v = __shfl_xor_sync(0xffffffffu, p.v, o);
        q.i = __shfl_xor_sync(0xffffffffu, p.i, o);
        p = better(p, q);
    }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) { sv[w] = p.v; si[w] = p.i; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < (int)(blockDim.x >> 5); ++k) p = better(p, BestPair{sv[k], si[k]});
    }
    return p;
}

__global__ void argmax_stage1(const float* __restrict__ logits, int vocab, const int32_t* __restrict__ recent,
                              int n_recent, double penalty, double* part_v, int* part_i) {
    const int per = (vocab + gridDim.x - 1) / gridDim.x;
    const int lo = blockIdx.x * per;
    const int hi = min(vocab, lo + per);
    extern __shared__ unsigned pen_bits[];
    const int words = (per + 31) / 32;
    for (int k = threadIdx.x; k < words; k += blockDim.x) pen_bits[k] = 0u;
    __syncthreads();
    const int from = n_recent > 65 ? n_recent - 65 : 0;
    for (int k = from + threadIdx.x; k < n_recent; k += blockDim.x) {
        const int t = recent[k];
        if (t >= lo && t < hi) atomicOr(&pen_bits[(t - lo) >> 5], 1u << ((t - lo) & 31));
    }
    __syncthreads();
    BestPair best{-1e30, 0};
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        double v = (double)logits[i];
        if ((pen_bits[(i - lo) >> 5] >> ((i - lo) & 31)) & 1u) v = v > 0.0 ? __ddiv_rn(v, penalty) : __dmul_rn(v, penalty);
        if (v > best.v) { best.v = v; best.i = i; }
    }
    best = block_best(best);
    if (threadIdx.x == 0) { part_v[blockIdx.x] = best.v; part_i[blockIdx.x] = best.i; }
}

__global__ void argmax_stage2(const double* part_v, const int* part_i, int n, int32_t* out) {
    BestPair best{-1e30, 0};
    for (int k = threadIdx.x; k < n; k += blockDim.x) best = better(best, BestPair{part_v[k], part_i[k]});
    best = block_best(best);
    if (threadIdx.x == 0) *out = best.i;
}

size_t argmax_scratch_bytes(int32_t) { return (size_t)kArgmaxBlocks * (sizeof(double) + sizeof(int)); }

int argmax_penalized_launch(const float* logits, int32_t vocab, const int32_t* recent, int32_t n_recent,
                            double penalty, int32_t* out_idx, void* scratch, cudaStream_t st) {
    if (!logits || !out_idx || !scratch || vocab <= 0 || n_recent < 0 || (n_recent > 0 && !recent)) return kErrInvalidArg;
    double* pv = reinterpret_cast<double*>(scratch);
    int* pi = reinterpret_cast<int*>(pv + kArgmaxBlocks);
    const int blocks = vocab < kArgmaxBlocks * 64 ? (vocab + 63) / 64 : kArgmaxBlocks;
    const int per = (vocab + blocks - 1) / blocks;
    const size_t smem = (size_t)((per + 31) / 32) * 4;
    argmax_stage1<<<blocks, kArgmaxThreads, smem, st>>>(logits, vocab, recent, n_recent, penalty, pv, pi);
    argmax_stage2<<<1, kArgmaxThreads, 0, st>>>(pv, pi, blocks, out_idx);
    return launch_status();
}

}  // namespace gncx
