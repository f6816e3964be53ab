// attention.cu -- GQA / MQA / sliding-window decode attention over an fp32 KV
// cache (replaces gncx_mqa_attention_step_ext, csrc/gncx_llm_kernels.cpp:1887-1994),
// and the causal prefill form (one query per prompt position, each attending to
// positions <= its own, as the reference's prefill calls the decode step per
// token, lua/gncx_streamer.lua:1079-1109).
//
// Split-KV ("flash-decoding"): a query's window [t0, pos] is cut into chunks;
// one CTA per (chunk, KV head, query) pulls that chunk's K and V head rows into
// shared memory with cp.async.bulk (one 16-byte-aligned copy per position, rows
// padded by 8 floats so the 8-lane dot pattern is bank-conflict free), serves
// every query head of the group from it, and writes a partial record (chunk
// max, sum of exp, unnormalised output).  A combine kernel merges the records
// of each head and can re-quantize the result for the next GEMV.  In decode,
// each K/V byte crosses HBM once.  The position may live in device memory so a
// captured CUDA graph replays every token; CTAs past the window exit at once.
//
// Scores are bit-identical to the reference's: its q.k is two 4-lane SSE
// accumulators over steps of 8, folded (l0+l1)+(l2+l3); lane j of an 8-lane
// group owns the chain over d = 8m + j and the fold is done with shuffles.
// The softmax sums are formed in a different order, so outputs agree with
// the reference to ~1e-6 relative.
//
// KV cache layout is the reference's: [max_seq][n_kv][head_dim] fp32 per layer.
#include <cuda_runtime.h>
#include "act.cuh"
#include "common.cuh"
#include "kernels.h"
#include "tma.cuh"

namespace gncx {

constexpr int kAttnThreads = 128;
constexpr int kMaxHeadDim = 256;
constexpr int kRowPad = 8;  // floats of padding per staged K/V row

static size_t attn_smem_bytes(int G, int hd, int chunk) {
    const int rs = hd + kRowPad;
    return 64 /*barriers*/ + (size_t)2 * chunk * rs * 4 + (size_t)G * hd * 4 + (size_t)G * chunk * 4 +
           (size_t)2 * G * 4;
}

__device__ __forceinline__ void attn_window(const AttnArgs& a, int z, int& t0, int& len) {
    const int pos = (a.pos_dev ? *a.pos_dev : a.pos0) + z;
    t0 = a.window > 0 ? max(0, pos - a.window + 1) : 0;
    len = pos + 1 - t0;
}

// Partial record layout per (query, head, split): [0] = max, [1] = sum of exp, [2..] = o[hd]
template <bool BULK, bool SCORES_ONLY>
__global__ void __launch_bounds__(kAttnThreads) attn_partial_kernel(const AttnArgs a) {
    extern __shared__ __align__(128) uint8_t smraw[];
    const int z = blockIdx.z;
    int t0, len;
    attn_window(a, z, t0, len);
    const int chunk = a.chunk;
    const int split = blockIdx.x;
    const int c0 = split * chunk;
    if (c0 >= len) return;  // uniform per CTA, before any barrier
    const int hd = a.hd;
    const int G = a.n_heads / a.n_kv;
    const int kvh = blockIdx.y;
    const int cn = min(chunk, len - c0);
    // head-major caches hold a chunk's positions contiguously: one bulk copy,
    // dense rows; otherwise one copy per position into padded rows
    const bool contig = a.kv_pos_stride == hd;
    const int rs = contig ? hd : hd + kRowPad;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smraw);   // [0] = K, [1] = V
    float* ks = reinterpret_cast<float*>(smraw + 64);     // [chunk][rs]
    float* vs = ks + (size_t)chunk * rs;                  // [chunk][rs]
    float* qs = vs + (size_t)chunk * rs;                  // [G][hd]
    float* sc = qs + (size_t)G * hd;                      // [G][chunk]
    float* red = sc + (size_t)G * chunk;                  // [G][2]
    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const size_t row0 = (size_t)(t0 + c0) * a.kv_pos_stride + (size_t)kvh * a.kv_head_stride;
    const size_t ps = (size_t)a.kv_pos_stride;

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
                if (!SCORES_ONLY) mbar_arrive_expect_tx(&bar[1], bytes * cn);
            }
            __syncwarp();
            if (contig) {
                if (lane == 0) {
                    bulk_g2s(ks, a.kc + row0, bytes * cn, &bar[0]);
                    if (!SCORES_ONLY) bulk_g2s(vs, a.vc + row0, bytes * cn, &bar[1]);
                }
            } else {
                for (int p = lane; p < cn; p += 32) bulk_g2s(ks + (size_t)p * rs, a.kc + row0 + p * ps, bytes, &bar[0]);
                if (!SCORES_ONLY)
                    for (int p = lane; p < cn; p += 32)
                        bulk_g2s(vs + (size_t)p * rs, a.vc + row0 + p * ps, bytes, &bar[1]);
            }
        }
    } else {
        for (int i = tid; i < cn * hd; i += blockDim.x) {
            const int p = i / hd, d = i % hd;
            ks[(size_t)p * rs + d] = a.kc[row0 + p * ps + d];
            if (!SCORES_ONLY) vs[(size_t)p * rs + d] = a.vc[row0 + p * ps + d];
        }
    }
    const float* qz = a.q + (size_t)z * a.q_stride + (size_t)kvh * G * hd;
    for (int i = tid; i < G * hd; i += blockDim.x) qs[i] = qz[i];
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
                const float x = fadd(c, __shfl_down_sync(0xffffffffu, c, 4));
                const float y = fadd(x, __shfl_down_sync(0xffffffffu, x, 1));
                float dot = fadd(y, __shfl_down_sync(0xffffffffu, y, 2));
                if (j == 0 && ok) {
                    for (int d = nm * 8; d < hd; ++d) dot = fadd(dot, fmul(qg[d], kt[d]));
                    const float sv = fmul(dot, a.scale);
                    if (SCORES_ONLY)
                        a.scores[((size_t)z * a.n_heads + kvh * G + g) * a.score_cap + c0 + p] = sv;
                    else
                        sc[g * chunk + p] = sv;
                }
            }
        }
    }
    if (SCORES_ONLY) {  // the K copies have all landed (waited above)
        if (timed_out && tid == 0) record_error(a.err, kErrTimeout);
        return;
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
        if (tid == 0) record_error(a.err, kErrTimeout);
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
                    float* rec = a.part + (((size_t)z * a.n_heads + h) * a.max_splits + split) * (hd + 2);
                    rec[2 + d] = acc[k];
                    if (d == 0) { rec[0] = red[2 * (g0 + k)]; rec[1] = red[2 * (g0 + k) + 1]; }
                }
            }
        }
    }
}

// Merge the split records of one (query, head):
// out = (sum_s o_s * e^(m_s-M)) / (sum_s l_s * e^(m_s-M) + 1e-12); optionally
// re-quantized (blockDim == hd, one warp per 32 outputs).
__global__ void attn_combine_kernel(const AttnArgs a) {
    extern __shared__ float wsm[];  // [max_splits] weights, then [max_splits] sums
    __shared__ float red[32];
    __shared__ float s_inv;
    const int h = blockIdx.x, z = blockIdx.y;
    const int hd = a.hd;
    int t0, len;
    attn_window(a, z, t0, len);
    const int n = (len + a.chunk - 1) / a.chunk;
    const float* rec = a.part + ((size_t)z * a.n_heads + h) * a.max_splits * (hd + 2);
    float* lsm = wsm + a.max_splits;
    float M = -INFINITY;
    for (int s = threadIdx.x; s < n; s += blockDim.x) {
        const float m = rec[(size_t)s * (hd + 2)];
        wsm[s] = m;
        lsm[s] = rec[(size_t)s * (hd + 2) + 1];
        M = fmaxf(M, m);
    }
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = M;
    __syncthreads();
    M = red[0];
    for (int k = 1; k < (int)(blockDim.x >> 5); ++k) M = fmaxf(M, red[k]);
    for (int s = threadIdx.x; s < n; s += blockDim.x) wsm[s] = exp_cr(fsub(wsm[s], M));
    __syncthreads();
    if (threadIdx.x == 0) {
        float L = 0.0f;
        for (int s = 0; s < n; ++s) L = fadd(L, fmul(lsm[s], wsm[s]));
        s_inv = fdiv(1.0f, fadd(L, 1e-12f));
    }
    __syncthreads();
    const float inv = s_inv;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float o = 0.0f;
#pragma unroll 8
        for (int s = 0; s < n; ++s) o = fadd(o, fmul(rec[(size_t)s * (hd + 2) + 2 + d], wsm[s]));
        o = fmul(o, inv);
        if (a.out) a.out[(size_t)z * a.out_stride + (size_t)h * hd + d] = o;
        if (a.act_out) {
            ActBlock* dst = a.act_out + (size_t)z * (a.n_heads * hd / 32) + ((size_t)h * hd + d) / 32;
            warp_quantize_store(o, dst, d & 31);
        }
    }
}

// Exact softmax * V in the reference's order (:1960-1987): max over the
// window, e_t = exp(s_t - max) (correctly rounded here; the reference uses the
// host expf), sum_exp serially over t, inv = 1/(sum_exp + 1e-12),
// out[d] += (e_t * inv) * v_t[d] serially over t.  One CTA per (query, head).
__global__ void attn_exact_kernel(const AttnArgs a) {
    const int h = blockIdx.x, z = blockIdx.y;
    const int hd = a.hd, G = a.n_heads / a.n_kv, kvh = h / G;
    int t0, len;
    attn_window(a, z, t0, len);
    float* sc = a.scores + ((size_t)z * a.n_heads + h) * a.score_cap;
    __shared__ float red[32];
    __shared__ float s_inv;
    float mx = -1e30f;  // the reference starts its running max at -1e30
    for (int t = threadIdx.x; t < len; t += blockDim.x) mx = fmaxf(mx, sc[t]);
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red[0];
    for (int k = 1; k < (int)(blockDim.x >> 5); ++k) mx = fmaxf(mx, red[k]);
    for (int t = threadIdx.x; t < len; t += blockDim.x) sc[t] = exp_cr(fsub(sc[t], mx));
    __syncthreads();
    if (threadIdx.x == 0) {
        float sum = 0.0f;
        for (int t = 0; t < len; ++t) sum = fadd(sum, sc[t]);
        s_inv = fdiv(1.0f, fadd(sum, 1e-12f));
    }
    __syncthreads();
    const float inv = s_inv;
    const float* vbase = a.vc + (size_t)t0 * a.kv_pos_stride + (size_t)kvh * a.kv_head_stride;
    const size_t ps = (size_t)a.kv_pos_stride;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float o = 0.0f;
#pragma unroll 16
        for (int t = 0; t < len; ++t) o = fadd(o, fmul(fmul(sc[t], inv), vbase[(size_t)t * ps + d]));
        if (a.out) a.out[(size_t)z * a.out_stride + (size_t)h * hd + d] = o;
        if (a.act_out) {
            ActBlock* dst = a.act_out + (size_t)z * (a.n_heads * hd / 32) + ((size_t)h * hd + d) / 32;
            warp_quantize_store(o, dst, d & 31);
        }
    }
}

int attention_geometry_chunk(int32_t len, int32_t n_kv, int sm_count) {
    int c = 64;
    // shorter chunks when the window is small, so every SM gets ~2 CTAs
    while (c > 16 && (int64_t)((len + c - 1) / c) * n_kv < 2 * (int64_t)sm_count) c >>= 1;
    return c;
}

template <bool BULK, bool SCORES_ONLY>
static void launch_partial(const AttnArgs& a, dim3 grid, size_t smem, cudaStream_t st) {
    static size_t set_bytes = 0;
    if (smem > set_bytes) {
        cudaFuncSetAttribute(attn_partial_kernel<BULK, SCORES_ONLY>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem);
        set_bytes = smem;
    }
    attn_partial_kernel<BULK, SCORES_ONLY><<<grid, kAttnThreads, smem, st>>>(a);
}

int attention_run(const AttnArgs& args, int32_t n_tok, cudaStream_t st) {
    const AttnArgs& a = args;
    if (!a.q || !a.kc || !a.vc || !a.part || a.n_heads <= 0 || a.n_kv <= 0 || a.hd <= 0 || n_tok <= 0)
        return kErrInvalidArg;
    if (a.n_heads % a.n_kv != 0 || a.hd > kMaxHeadDim || (a.hd & 3) || a.chunk <= 0 || a.max_splits <= 0)
        return kErrInvalidArg;
    if (a.act_out && (a.hd % 32 || a.hd > 1024)) return kErrInvalidArg;
    const DeviceInfo& dev = device_info();
    const int G = a.n_heads / a.n_kv;
    const size_t smem = attn_smem_bytes(G, a.hd, a.chunk);
    if (smem > (size_t)dev.max_smem_optin) return kErrCapacity;
    const bool bulk = ((uintptr_t)a.kc % 16 == 0) && ((uintptr_t)a.vc % 16 == 0);
    dim3 grid(a.max_splits, a.n_kv, n_tok);
    if (a.exact) {
        if (!a.scores || a.score_cap < a.max_splits * a.chunk) return kErrCapacity;
        if (a.act_out && a.hd > 1024) return kErrInvalidArg;
        if (bulk) launch_partial<true, true>(a, grid, smem, st);
        else launch_partial<false, true>(a, grid, smem, st);
        const int threads = (a.act_out || (a.hd % 32 == 0 && a.hd <= 1024)) ? a.hd : 128;
        attn_exact_kernel<<<dim3(a.n_heads, n_tok), threads, 0, st>>>(a);
        return cudaPeekAtLastError() == cudaSuccess ? kOk : kErrCuda;
    }
    if (bulk) launch_partial<true, false>(a, grid, smem, st);
    else launch_partial<false, false>(a, grid, smem, st);
    const size_t csm = (size_t)a.max_splits * 8;
    if (csm > 48 * 1024)
        cudaFuncSetAttribute(attn_combine_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)csm);
    const int cthreads = (a.act_out || (a.hd % 32 == 0 && a.hd <= 1024)) ? a.hd : 128;
    attn_combine_kernel<<<dim3(a.n_heads, n_tok), cthreads, csm, st>>>(a);
    return cudaPeekAtLastError() == cudaSuccess ? kOk : kErrCuda;
}

int32_t attention_scratch_records(int32_t pos, int32_t n_heads, int32_t window) {
    const int32_t t0 = window > 0 ? (pos - window + 1 > 0 ? pos - window + 1 : 0) : 0;
    const int32_t len = pos + 1 - t0;
    return n_heads * ((len + 15) / 16);  // the smallest chunk is 16 positions
}

int attention_launch(const float* q, float* kc, float* vc, int32_t pos, int32_t n_heads, int32_t n_kv,
                     int32_t head_dim, float scale, int32_t window, float* out, const AttnScratch& scratch,
                     int32_t* err, cudaStream_t st, float* exact_scores) {
    if (!q || !kc || !vc || !out || pos < 0 || n_heads <= 0 || n_kv <= 0 || head_dim <= 0) return kErrInvalidArg;
    const int32_t t0 = window > 0 ? (pos - window + 1 > 0 ? pos - window + 1 : 0) : 0;
    const int32_t len = pos + 1 - t0;
    AttnArgs a{};
    a.q = q;
    a.q_stride = n_heads * head_dim;
    a.kc = kc;
    a.vc = vc;
    a.kv_pos_stride = n_kv * head_dim;  // the reference's [pos][n_kv][head_dim]
    a.kv_head_stride = head_dim;
    a.pos0 = pos;
    a.pos_dev = nullptr;
    a.n_heads = n_heads;
    a.n_kv = n_kv;
    a.hd = head_dim;
    a.scale = scale;
    a.window = window;
    a.chunk = attention_geometry_chunk(len, n_kv, device_info().sm_count);
    a.max_splits = (len + a.chunk - 1) / a.chunk;
    if (!scratch.part || (int64_t)n_heads * a.max_splits > scratch.capacity) return kErrCapacity;
    a.part = scratch.part;
    a.out = out;
    a.out_stride = n_heads * head_dim;
    a.act_out = nullptr;
    a.err = err;
    a.exact = exact_scores != nullptr;
    a.scores = exact_scores;
    a.score_cap = a.max_splits * a.chunk;
    return attention_run(a, 1, st);
}

}  // namespace gncx
