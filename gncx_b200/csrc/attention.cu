// attention.cu -- GQA / MQA / sliding-window decode attention over an fp32 KV
// cache (replaces gncx_mqa_attention_step_ext, csrc/gncx_llm_kernels.cpp:1887-1994).
//
// Split-KV ("flash-decoding"): the window [t0, pos] is cut into chunks of up
// to 64 positions; one CTA per (chunk, KV head) pulls that chunk's K and V
// head rows into shared memory with cp.async.bulk (one 16-byte-aligned copy per
// position, rows padded by 8 floats so the 8-lane dot pattern is bank-conflict
// free), serves every query head of the group from it, and writes a partial
// record (chunk max, sum of exp, unnormalised output).  A combine kernel merges
// the records of each head.  Each K/V byte crosses HBM once.
//
// Scores are bit-identical to the reference's: its q.k is two 4-lane SSE
// accumulators over steps of 8, folded (l0+l1)+(l2+l3); lane j of an 8-lane
// group owns the chain over d = 8m + j and the fold is done with shuffles.
// The softmax sums are formed in a different order, so outputs agree with
// the reference to ~1e-6 relative.
//
// KV cache layout is the reference's: [max_seq][n_kv][head_dim] fp32 per layer.
#include <cuda_runtime.h>
#include "common.cuh"
#include "kernels.h"
#include "tma.cuh"

namespace gncx {

constexpr int kAttnThreads = 128;
constexpr int kMaxHeadDim = 256;
constexpr int kMaxChunk = 64;
constexpr int kRowPad = 8;  // floats of padding per staged K/V row

struct AttnGeom {
    int t0, len, chunk, n_splits;
};

static AttnGeom attn_geom(int32_t pos, int32_t n_kv, int32_t window, int sm_count) {
    AttnGeom g;
    g.t0 = window > 0 ? (pos - window + 1 > 0 ? pos - window + 1 : 0) : 0;
    g.len = pos + 1 - g.t0;
    int c = kMaxChunk;
    // shorter chunks when the window is small, so every SM gets ~2 CTAs
    while (c > 16 && (int64_t)((g.len + c - 1) / c) * n_kv < 2 * (int64_t)sm_count) c >>= 1;
    g.chunk = c;
    g.n_splits = (g.len + c - 1) / c;
    return g;
}

int32_t attention_scratch_records(int32_t pos, int32_t n_heads, int32_t window) {
    const int32_t t0 = window > 0 ? (pos - window + 1 > 0 ? pos - window + 1 : 0) : 0;
    const int32_t len = pos + 1 - t0;
    return n_heads * ((len + 15) / 16);  // the smallest chunk is 16 positions
}

static size_t attn_smem_bytes(int G, int hd, int chunk) {
    const int rs = hd + kRowPad;
    return 64 /*barriers*/ + (size_t)2 * chunk * rs * 4 + (size_t)G * hd * 4 + (size_t)G * chunk * 4 +
           (size_t)2 * G * 4;
}

// Partial record layout per (head, split): [0] = max, [1] = sum of exp, [2..] = o[hd]
template <bool BULK>
__global__ void __launch_bounds__(kAttnThreads) attn_partial_kernel(
    const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc, int n_heads, int n_kv,
    int hd, float scale, int t0, int len, int chunk, int n_splits, float* __restrict__ part, int32_t* err) {
    extern __shared__ __align__(128) uint8_t smraw[];
    const int G = n_heads / n_kv;
    const int kvh = blockIdx.y;
    const int split = blockIdx.x;
    const int c0 = split * chunk;
    const int cn = min(chunk, len - c0);
    const int kvd = n_kv * hd;
    const int rs = hd + kRowPad;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smraw);   // [0] = K, [1] = V
    float* ks = reinterpret_cast<float*>(smraw + 64);     // [chunk][rs]
    float* vs = ks + (size_t)chunk * rs;                  // [chunk][rs]
    float* qs = vs + (size_t)chunk * rs;                  // [G][hd]
    float* sc = qs + (size_t)G * hd;                      // [G][chunk]
    float* red = sc + (size_t)G * chunk;                  // [G][2]
    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const size_t row0 = (size_t)(t0 + c0) * kvd + (size_t)kvh * hd;

    if (BULK) {
        if (tid == 0) {
            mbar_init(&bar[0], 1);
            mbar_init(&bar[1], 1);
            fence_barrier_init();
        }
        __syncthreads();
        if (warp == 0) {
            const uint32_t bytes = (uint32_t)hd * 4;
            if (lane == 0) {
                mbar_arrive_expect_tx(&bar[0], bytes * cn);
                mbar_arrive_expect_tx(&bar[1], bytes * cn);
            }
            __syncwarp();
            for (int p = lane; p < cn; p += 32) bulk_g2s(ks + (size_t)p * rs, kc + row0 + (size_t)p * kvd, bytes, &bar[0]);
            for (int p = lane; p < cn; p += 32) bulk_g2s(vs + (size_t)p * rs, vc + row0 + (size_t)p * kvd, bytes, &bar[1]);
        }
    } else {
        for (int i = tid; i < cn * hd; i += blockDim.x) {
            const int p = i / hd, d = i % hd;
            ks[(size_t)p * rs + d] = kc[row0 + (size_t)p * kvd + d];
            vs[(size_t)p * rs + d] = vc[row0 + (size_t)p * kvd + d];
        }
    }
    for (int i = tid; i < G * hd; i += blockDim.x) qs[i] = q[(size_t)kvh * G * hd + i];
    __syncthreads();
    bool timed_out = false;
    if (BULK && !mbar_wait(&bar[0], 0)) timed_out = true;

    // ---- scores: 8 lanes per position, lane j owns the chain over d = 8m + j ----
    const int j = lane & 7, slot = lane >> 3;  // 4 positions per warp per step
    const int nm = hd >> 3;
    if (!timed_out) {
        for (int p0 = warp * 4; p0 < cn; p0 += (kAttnThreads / 32) * 4) {
            const int p = p0 + slot;
            const bool ok = p < cn;
            const float* kt = ks + (size_t)(ok ? p : 0) * rs;
            float kr[kMaxHeadDim / 8];
#pragma unroll
            for (int m = 0; m < kMaxHeadDim / 8; ++m)
                if (m < nm) kr[m] = kt[8 * m + j];
            for (int g = 0; g < G; ++g) {
                const float* qg = qs + g * hd;
                float c = 0.0f;
#pragma unroll
                for (int m = 0; m < kMaxHeadDim / 8; ++m)
                    if (m < nm) c = fadd(c, fmul(qg[8 * m + j], kr[m]));
                const float a = fadd(c, __shfl_down_sync(0xffffffffu, c, 4));
                const float b = fadd(a, __shfl_down_sync(0xffffffffu, a, 1));
                float dot = fadd(b, __shfl_down_sync(0xffffffffu, b, 2));
                if (j == 0 && ok) {
                    for (int d = nm * 8; d < hd; ++d) dot = fadd(dot, fmul(qg[d], kt[d]));
                    sc[g * chunk + p] = fmul(dot, scale);
                }
            }
        }
    }
    __syncthreads();

    // ---- per head: chunk max, exp, sum ----
    for (int g = warp; g < G; g += kAttnThreads / 32) {
        float mx = -INFINITY;
        for (int p = lane; p < cn; p += 32) mx = fmaxf(mx, sc[g * chunk + p]);
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float sum = 0.0f;
        for (int p = lane; p < cn; p += 32) {
            const float e = exp_cr(fsub(sc[g * chunk + p], mx));
            sc[g * chunk + p] = e;
            sum += e;
        }
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) { red[2 * g] = mx; red[2 * g + 1] = sum; }
    }
    // always wait (bounded) for the V copies, so none is in flight when the CTA exits
    if (BULK && !mbar_wait(&bar[1], 0)) timed_out = true;
    __syncthreads();
    if (timed_out) {
        if (tid == 0) record_error(err, kErrTimeout);
        return;
    }

    // ---- o[g][d] = sum_p e[g][p] * v[p][d] ----
    for (int d = tid; d < hd; d += blockDim.x) {
        for (int g0 = 0; g0 < G; g0 += 4) {
            float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 4
            for (int p = 0; p < cn; ++p) {
                const float v = vs[(size_t)p * rs + d];
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    if (g0 + k < G) acc[k] = fadd(acc[k], fmul(sc[(g0 + k) * chunk + p], v));
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                if (g0 + k < G) {
                    const int h = kvh * G + g0 + k;
                    float* rec = part + ((size_t)h * n_splits + split) * (hd + 2);
                    rec[2 + d] = acc[k];
                    if (d == 0) { rec[0] = red[2 * (g0 + k)]; rec[1] = red[2 * (g0 + k) + 1]; }
                }
            }
        }
    }
}

// Merge the split records of one head: out = (sum_s o_s * e^(m_s-M)) / (sum_s l_s * e^(m_s-M) + 1e-12).
__global__ void attn_combine_kernel(const float* __restrict__ part, int n_splits, int hd, float* __restrict__ out) {
    extern __shared__ float wsm[];  // [n_splits] weights
    __shared__ float s_inv;
    const int h = blockIdx.x;
    const float* rec = part + (size_t)h * n_splits * (hd + 2);
    float M = -INFINITY;
    for (int s = 0; s < n_splits; ++s) M = fmaxf(M, rec[(size_t)s * (hd + 2)]);
    for (int s = threadIdx.x; s < n_splits; s += blockDim.x) wsm[s] = exp_cr(fsub(rec[(size_t)s * (hd + 2)], M));
    __syncthreads();
    if (threadIdx.x == 0) {
        float L = 0.0f;
        for (int s = 0; s < n_splits; ++s) L = fadd(L, fmul(rec[(size_t)s * (hd + 2) + 1], wsm[s]));
        s_inv = fdiv(1.0f, fadd(L, 1e-12f));
    }
    __syncthreads();
    const float inv = s_inv;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float o = 0.0f;
        for (int s = 0; s < n_splits; ++s) o = fadd(o, fmul(rec[(size_t)s * (hd + 2) + 2 + d], wsm[s]));
        out[(size_t)h * hd + d] = fmul(o, inv);
    }
}

int attention_launch(const float* q, float* kc, float* vc, int32_t pos, int32_t n_heads, int32_t n_kv,
                     int32_t head_dim, float scale, int32_t window, float* out, const AttnScratch& scratch,
                     int32_t* err, cudaStream_t st) {
    if (!q || !kc || !vc || !out || pos < 0 || n_heads <= 0 || n_kv <= 0 || head_dim <= 0) return kErrInvalidArg;
    if (n_heads % n_kv != 0 || head_dim > kMaxHeadDim || (head_dim & 3)) return kErrInvalidArg;
    const DeviceInfo& dev = device_info();
    const AttnGeom g = attn_geom(pos, n_kv, window, dev.sm_count);
    if (!scratch.part || (int64_t)n_heads * g.n_splits > scratch.capacity) return kErrCapacity;
    const int G = n_heads / n_kv;
    const size_t smem = attn_smem_bytes(G, head_dim, g.chunk);
    if (smem > (size_t)dev.max_smem_optin) return kErrCapacity;
    const bool bulk = ((uintptr_t)kc % 16 == 0) && ((uintptr_t)vc % 16 == 0);
    dim3 grid(g.n_splits, n_kv);
    if (bulk) {
        static size_t set_bytes = 0;
        if (smem > set_bytes) {
            cudaFuncSetAttribute(attn_partial_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            set_bytes = smem;
        }
        attn_partial_kernel<true><<<grid, kAttnThreads, smem, st>>>(q, kc, vc, n_heads, n_kv, head_dim, scale, g.t0,
                                                                     g.len, g.chunk, g.n_splits, scratch.part, err);
    } else {
        static size_t set_bytes = 0;
        if (smem > set_bytes) {
            cudaFuncSetAttribute(attn_partial_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            set_bytes = smem;
        }
        attn_partial_kernel<false><<<grid, kAttnThreads, smem, st>>>(q, kc, vc, n_heads, n_kv, head_dim, scale, g.t0,
                                                                      g.len, g.chunk, g.n_splits, scratch.part, err);
    }
    const size_t csm = (size_t)g.n_splits * 4;
    if (csm > 48 * 1024)
        cudaFuncSetAttribute(attn_combine_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)csm);
    attn_combine_kernel<<<n_heads, 128, csm, st>>>(scratch.part, g.n_splits, head_dim, out);
    return cudaPeekAtLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace gncx
