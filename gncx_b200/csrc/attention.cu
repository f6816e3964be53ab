// attention.cu -- GQA / MQA / sliding-window decode attention over an fp32 KV
// cache (replaces gncx_mqa_attention_step_ext, csrc/gncx_llm_kernels.cpp:1887-1994),
// and the causal prefill form (one query per prompt position, each attending to
// positions <= its own, as the reference's prefill calls the decode step per
// token, lua/gncx_streamer.lua:1079-1109).
//
// Split-KV ("flash-decoding"): a query's window [t0, pos] is cut into chunks;
// one CTA per (chunk, KV head, query) stages that chunk's K and V head rows in
// shared memory (16-byte cp.async copies into rows padded by 4 floats, so that
// eight threads reading eight different rows hit eight different bank groups),
// serves every query head of the group from it, and writes a partial record
// (chunk max, sum of exp, unnormalised output).  A combine kernel merges the
// records of each (query, head) and can re-quantize the result for the next
// GEMV.  In decode each K/V byte crosses HBM once.  The position may live in device memory so a captured CUDA graph
// replays every token; CTAs past the window exit at once.
//
// Scores are bit-identical to the reference's: its q.k is two 4-lane SSE
// accumulators over steps of 8, folded (l0+l1)+(l2+l3), i.e. eight serial
// chains over d = 8m + j (j = 0..7), folded ((c0+c4)+(c1+c5))+((c2+c6)+(c3+c7));
// one thread runs the eight chains of one (position, head).  The split-KV
// softmax sums are formed in a different order from the reference's serial
// ones, so those outputs agree to ~1e-6 relative.  Exact mode keeps the
// reference's order: scores only here, then attn_exact_softmax_kernel (serial
// sum of exp over the window) and attn_exact_pv_kernel (serial sum over t of
// (e_t * inv) * v_t[d] for every output element).
//
// KV cache layout: rows of head_dim floats at kc + t * kv_pos_stride +
// kvh * kv_head_stride (the reference's [pos][n_kv][head_dim], or the engine's
// head-major [n_kv][max_seq][head_dim]).
#include <cuda_runtime.h>
#include <stdlib.h>
#include "act.cuh"
#include "attn_parts.cuh"
#include "common.cuh"
#include "kernels.h"
#include "trace.cuh"
#include "launch.cuh"
#include "norm.cuh"
#include "tma.cuh"

namespace gncx {

constexpr int kAttnThreads = 256;     // prefill / exact kernels
constexpr int kAttnMaxThreads = 512;  // the split-KV partial kernel: 512 where head_dim <= 128
constexpr int kMaxHeadDim = 256;
constexpr int kRowPad = 4;    // floats of padding per staged K/V row
constexpr int kScorePad = 8;  // floats of padding per score row
__host__ __device__ inline int attn_q_stride(int hd) { return hd + 4; }  // padded q rows

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
                 "l"(gmem)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Floats of the K/V staging area, which the position-group reduction of the
// PV step reuses as scratch (up to kAttnMaxThreads * 8 floats).
__host__ __device__ inline size_t attn_kv_floats(int hd, int chunk) {
    size_t n = (size_t)2 * chunk * (hd + kRowPad);
    if ((size_t)kAttnMaxThreads * 8 > n) n = (size_t)kAttnMaxThreads * 8;
    return (n + 3) & ~(size_t)3;  // keeps the q rows that follow 16-byte aligned
}

static size_t attn_smem_bytes(int G, int hd, int chunk) {
    const int G4 = (G + 3) & ~3;
    return attn_kv_floats(hd, chunk) * 4 + (size_t)G * attn_q_stride(hd) * 4 +
           (size_t)G * (chunk + kScorePad) * 4 + (size_t)chunk * G4 * 4 + (size_t)2 * G * 4;
}

__device__ __forceinline__ void attn_window(const AttnArgs& a, int z, int& t0, int& len) {
    const int pos = (a.pos_dev ? *a.pos_dev : a.pos0) + z;
    t0 = a.window > 0 ? max(0, pos - a.window + 1) : 0;
    len = pos + 1 - t0;
}

constexpr int kMergeBatch = 32;  // split records loaded per round trip in a merge


// Merge the n split records of head h of query z:
// out = (sum_s o_s * e^(m_s-M)) / (sum_s l_s * e^(m_s-M) + 1e-12).  The split
// sums are formed in parallel (the split-KV softmax is not in the reference's
// serial order anyway): blockDim / head_dim groups of threads each take every
// g-th split for one output column, then the groups' partial sums are added.
// `wsm` / `lsm` hold n floats each, `osm` blockDim floats; whole CTAs call it.
__device__ void attn_merge(const AttnArgs& a, int z, int h, int n, float* wsm, float* lsm, float* osm) {
    const int hd = a.hd;
    const size_t R = attn_record_floats(hd);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x, nwarps = nthr >> 5;
    __shared__ float red[32];
    __shared__ float s_max, s_inv;
    const float* rec0 = a.part + ((size_t)z * a.n_heads + h) * a.max_splits * R;
    float M = -INFINITY;
    for (int s = tid; s < n; s += nthr) {
        wsm[s] = ld_l2(rec0 + (size_t)s * R);
        lsm[s] = ld_l2(rec0 + (size_t)s * R + 1);
        M = fmaxf(M, wsm[s]);
    }
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    if (lane == 0) red[warp] = M;
    __syncthreads();
    if (tid == 0) {
        float m = red[0];
        for (int k = 1; k < nwarps; ++k) m = fmaxf(m, red[k]);
        s_max = m;
    }
    __syncthreads();
    M = s_max;
    float L = 0.0f;
    for (int s = tid; s < n; s += nthr) {
        const float wgt = exp_cr(fsub(wsm[s], M));
        wsm[s] = wgt;
        L = fadd(L, fmul(lsm[s], wgt));
    }
    for (int o = 16; o > 0; o >>= 1) L = fadd(L, __shfl_xor_sync(0xffffffffu, L, o));
    __syncthreads();  // red is reused
    if (lane == 0) red[warp] = L;
    __syncthreads();
    if (tid == 0) {
        float l = 0.0f;
        for (int k = 0; k < nwarps; ++k) l = fadd(l, red[k]);
        s_inv = fdiv(1.0f, fadd(l, 1e-12f));
    }
    const int ng = nthr / hd > 0 ? nthr / hd : 1;
    const int d = tid % hd, g = tid / hd;
    if (g < ng && d < hd) {
        const float* rec = rec0 + 4 + d;
        float o = 0.0f;
        for (int s0 = g * kMergeBatch; s0 < n; s0 += ng * kMergeBatch) {
            float v[kMergeBatch];  // a batch of records in flight at once
#pragma unroll
            for (int b = 0; b < kMergeBatch; ++b) v[b] = s0 + b < n ? ld_l2(rec + (size_t)(s0 + b) * R) : 0.0f;
#pragma unroll
            for (int b = 0; b < kMergeBatch; ++b)
                if (s0 + b < n) o = fadd(o, fmul(v[b], wsm[s0 + b]));
        }
        osm[g * hd + d] = o;
    }
    __syncthreads();
    for (int i = tid; i < hd; i += nthr) {  // whole warps: hd % 32 == 0 when act is written
        float o = osm[i];
        for (int q = 1; q < ng; ++q) o = fadd(o, osm[q * hd + i]);
        o = fmul(o, s_inv);
        if (a.out) a.out[(size_t)z * a.out_stride + (size_t)h * hd + i] = o;
        if (a.act_out.blocks || a.act_out.staged)
            act_out_store(a.act_out, o, a.n_heads * hd, (size_t)z, (h * hd + i) >> 5, i & 31);
    }
}

// ---- per-chunk building blocks shared by the split-KV kernels ----
// Scores of positions [0, cn) of a staged chunk; task t = (position t / G, head
// t % G), so the G lanes of one position read the same K row (one shared-memory
// wavefront serves eight positions).  store(g, p, q.k) receives the unscaled dot.
template <class Store>
__device__ __forceinline__ void chunk_scores(const float* ks, int rs, const float* qs, int qrs, int G, int hd, int cn,
                                             Store store) {
    const int nm = hd >> 3;
    for (int task = threadIdx.x; task < G * cn; task += blockDim.x) {
        const int p = task / G, g = task - p * G;
        const float* kr = ks + (size_t)p * rs;
        const float* qg = qs + (size_t)g * qrs;
        float c[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) c[j] = 0.0f;
#pragma unroll 4
        for (int m = 0; m < nm; ++m) {
            const float4 k0 = *reinterpret_cast<const float4*>(kr + 8 * m);
            const float4 k1 = *reinterpret_cast<const float4*>(kr + 8 * m + 4);
            const float4 q0 = *reinterpret_cast<const float4*>(qg + 8 * m);
            const float4 q1 = *reinterpret_cast<const float4*>(qg + 8 * m + 4);
            c[0] = fadd(c[0], fmul(q0.x, k0.x));
            c[1] = fadd(c[1], fmul(q0.y, k0.y));
            c[2] = fadd(c[2], fmul(q0.z, k0.z));
            c[3] = fadd(c[3], fmul(q0.w, k0.w));
            c[4] = fadd(c[4], fmul(q1.x, k1.x));
            c[5] = fadd(c[5], fmul(q1.y, k1.y));
            c[6] = fadd(c[6], fmul(q1.z, k1.z));
            c[7] = fadd(c[7], fmul(q1.w, k1.w));
        }
        float dot = fadd(fadd(fadd(c[0], c[4]), fadd(c[1], c[5])), fadd(fadd(c[2], c[6]), fadd(c[3], c[7])));
        for (int d = nm * 8; d < hd; ++d) dot = fadd(dot, fmul(qg[d], kr[d]));
        store(g, p, dot);
    }
}


// Sum acc over the npg position groups through `scr` (npg * kPvHeads * hd
// floats) and hand out(i, d, value) each (head g0 + i, column d) once.
template <class Out>
__device__ __forceinline__ void pv_reduce(const float (&acc)[kPvHeads], int ng, int hd, int d, int pg, int npg,
                                          bool active, float* scr, Out out) {
    if (npg == 1) {
        if (active)
            for (int i = 0; i < ng; ++i) out(i, d, acc[i]);
        return;
    }
    __syncthreads();  // scr may overlap the V rows other threads are still reading
    if (active)
        for (int i = 0; i < ng; ++i) scr[((size_t)pg * kPvHeads + i) * hd + d] = acc[i];
    __syncthreads();
    for (int t = threadIdx.x; t < ng * hd; t += blockDim.x) {
        const int i = t / hd, dd = t - i * hd;
        float v = scr[(size_t)i * hd + dd];
        for (int q = 1; q < npg; ++q) v += scr[((size_t)q * kPvHeads + i) * hd + dd];
        out(i, dd, v);
    }
    __syncthreads();
}


// The per-head gains and this position's rope factors of one warp's head,
// loaded into registers before the kernel's dependency wait (the gains are
// weights; the rope table is fixed; the position was set before the step).
constexpr int kPostMaxW = kMaxHeadDim / 32, kPostMaxR = kMaxHeadDim / 64;
struct HeadPost {
    float w[kPostMaxW];
    float c[kPostMaxR], s[kPostMaxR];
};
__device__ __forceinline__ void head_post_load(HeadPost& hp, int hd, const float* __restrict__ w,
                                               const float* __restrict__ ct, const float* __restrict__ st, int pos,
                                               int lane) {
    const int half = hd >> 1;
#pragma unroll
    for (int m = 0; m < kPostMaxW; ++m) {
        const int i = lane + 32 * m;
        hp.w[m] = (w && i < hd) ? __ldg(w + i) : 1.0f;
    }
#pragma unroll
    for (int m = 0; m < kPostMaxR; ++m) {
        const int i = lane + 32 * m;
        hp.c[m] = i < half ? __ldg(ct + (size_t)pos * half + i) : 0.0f;
        hp.s[m] = i < half ? __ldg(st + (size_t)pos * half + i) : 0.0f;
    }
}
// warp_head_norm_rope with the operands of head_post_load (same arithmetic).
__device__ __forceinline__ void warp_head_norm_rope_pf(float* x, int hd, const HeadPost& hp, bool has_w,
                                                       bool do_norm, float eps, int lane) {
    if (do_norm) {
        const float acc = lane < 4 ? lane_sumsq(x, lane, hd >> 2) : 0.0f;
        const float a1 = __shfl_sync(0xffffffffu, acc, 1);
        const float a2 = __shfl_sync(0xffffffffu, acc, 2);
        const float a3 = __shfl_sync(0xffffffffu, acc, 3);
        float inv = 0.0f;
        if (lane == 0) {
            const double s = __dadd_rn(__dadd_rn(__dadd_rn((double)acc, (double)a1), (double)a2), (double)a3);
            const float ms = __double2float_rn(__ddiv_rn(s, (double)hd));
            inv = fdiv(1.0f, __fsqrt_rn(fadd(ms, eps)));
        }
        inv = __shfl_sync(0xffffffffu, inv, 0);
#pragma unroll
        for (int m = 0; m < kPostMaxW; ++m) {
            const int i = lane + 32 * m;
            if (i < hd) {
                const float v = fmul(x[i], inv);
                x[i] = has_w ? fmul(v, hp.w[m]) : v;
            }
        }
        __syncwarp();
    }
    const int half = hd >> 1;
#pragma unroll
    for (int m = 0; m < kPostMaxR; ++m) {
        const int i = lane + 32 * m;
        if (i < half) {
            const float c = hp.c[m], s = hp.s[m];
            const float x1 = x[i], x2 = x[i + half];
            x[i] = fsub(fmul(x1, c), fmul(x2, s));
            x[i + half] = fadd(fmul(x2, c), fmul(x1, s));
        }
    }
    __syncwarp();
}

// Partial record per (query, head, split): [0] = max, [1] = sum of exp, [4..] = o[hd]
// BULK (split-KV, head-major cache: a chunk of one head is contiguous): K and
// V of the chunk arrive as one bulk copy (TMA) each into unpadded rows,
// completing on s_bar[0] / s_bar[1], and the scores use the warp-per-dot
// mapping that is conflict-free on unpadded rows.
// POST (split-KV decode with the fused Q/K post step): the post step's gains
// and rope factors are loaded into registers before the dependency wait (a
// separate instantiation: the registers would lower the occupancy of the
// long-window drop-in launches, which have no post step).
template <bool VEC, bool SCORES_ONLY, int NT, bool BULK, bool POST>
__global__ void __launch_bounds__(NT) attn_partial_kernel(const AttnArgs a) {
    extern __shared__ __align__(16) uint8_t smraw[];
    GNCX_TRACE_SCOPE(kTagAttnPartial, gridDim.x);
    const int z = blockIdx.z;
    int t0, len;
    attn_window(a, z, t0, len);
    const int chunk = a.chunk;
    const int split = blockIdx.x;
    const int c0 = split * chunk;
    if (c0 >= len) return;  // uniform per CTA, before any barrier
    const int hd = a.hd;
    const int G = a.n_heads / a.n_kv;
    const int G4 = (G + 3) & ~3;
    const int kvh = blockIdx.y;
    const int cn = min(chunk, len - c0);
    const int rs = BULK ? hd : hd + kRowPad;
    float* ks = reinterpret_cast<float*>(smraw);                                  // [chunk][rs]
    float* vs = ks + (size_t)chunk * rs;                                           // [chunk][rs]
    const int qrs = attn_q_stride(hd), sld = chunk + kScorePad;
    float* qs = ks + attn_kv_floats(hd, chunk);                                    // [G][qrs]
    float* sc = qs + (size_t)G * qrs;                                              // [G][sld]
    float* es = sc + (size_t)G * sld;                                              // [chunk][G4]
    float* red = es + (size_t)chunk * G4;                                          // [G][2]
    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const size_t row0 = (size_t)(t0 + c0) * a.kv_pos_stride + (size_t)kvh * a.kv_head_stride;
    const size_t ps = (size_t)a.kv_pos_stride;
    // with the fused post step the query's own row (the last of the window) is
    // made here, not loaded
    const int pn = t0 + len - 1 - (t0 + c0);  // the query's position within this chunk
    const bool own_row = a.post_k && pn >= 0 && pn < cn;
    const int n_load = own_row ? pn : cn;     // rows copied from the cache
    __shared__ __align__(8) uint64_t s_bar[2];
    if (BULK) {
        if (tid == 0) {
            mbar_init(&s_bar[0], 1);
            mbar_init(&s_bar[1], 1);
            fence_barrier_init();
            const uint32_t bytes = (uint32_t)n_load * (uint32_t)hd * 4u;
            mbar_arrive_expect_tx(&s_bar[0], bytes);
            mbar_arrive_expect_tx(&s_bar[1], bytes);
        }
        __syncthreads();
    }

    pdl_launch_dependents();
    // ---- stage K and V: rows written before the preceding kernel first (they
    // may stream in while it finishes), the rest after the dependency wait ----
    const int n_old = a.prefetch_old ? max(0, min(cn, (t0 + len - 1) - (t0 + c0))) : 0;
    auto stage_rows = [&](int pa, int pb) {
        if (BULK) {
            if (tid == 0 && pb > pa) {
                const uint32_t bytes = (uint32_t)(pb - pa) * (uint32_t)hd * 4u;
                bulk_g2s(ks + (size_t)pa * hd, a.kc + row0 + (size_t)pa * ps, bytes, &s_bar[0]);
                bulk_g2s(vs + (size_t)pa * hd, a.vc + row0 + (size_t)pa * ps, bytes, &s_bar[1]);
            }
        } else if (VEC) {
            // thread -> one 16-byte piece c of rows pa + p0, pa + p0 + step, ...
            // (16-byte cp.async: per-row bulk copies measured slower -- the
            // SM's copy engine serialises hundreds of 512-byte copies)
            const int cpr = hd >> 2, step = NT / cpr;
            const int c = tid % cpr, p0 = tid / cpr;
            if (tid < step * cpr) {
                for (int p = pa + p0; p < pb; p += step) {
                    cp_async16(ks + (size_t)p * rs + 4 * c, a.kc + row0 + p * ps + 4 * c);
                    if (!SCORES_ONLY) cp_async16(vs + (size_t)p * rs + 4 * c, a.vc + row0 + p * ps + 4 * c);
                }
            }
            cp_async_commit();
        } else {
            for (int i = tid; i < (pb - pa) * hd; i += NT) {
                const int p = pa + i / hd, d = i % hd;
                ks[(size_t)p * rs + d] = a.kc[row0 + p * ps + d];
                if (!SCORES_ONLY) vs[(size_t)p * rs + d] = a.vc[row0 + p * ps + d];
            }
        }
    };
    if (n_old > 0) stage_rows(0, n_old);
    // the post step's gains and rope factors, before the dependency wait: warp
    // `task` < G norms and rotates q head `task`, warp G the new K row
    // (split-KV only: in exact mode, whose scores-only CTAs end right after the
    // post step, loading these early measured slower: 3.92 vs 3.38 ms/token)
    HeadPost hp;
    const int n_post = a.post_k ? G + (own_row ? 1 : 0) : 0;
    const bool post_pf = POST && !SCORES_ONLY && n_post <= NT / 32;
    if constexpr (POST) {
        if (warp < n_post && post_pf)
            head_post_load(hp, hd, warp < G ? a.post_qn : a.post_kn, a.rope_c, a.rope_s, t0 + len - 1, lane);
    }
    if (tid == 0) GNCX_TRACE_MARK(10, n_old);
    pdl_wait();
    if (tid == 0) GNCX_TRACE_MARK(11, 0);
    if (n_old < n_load) stage_rows(n_old, n_load);
    const float* qz = a.q + (size_t)z * a.q_stride + (size_t)kvh * G * hd;
    for (int i = tid; i < G * hd; i += NT) qs[(size_t)(i / hd) * qrs + i % hd] = qz[i];
    if (a.post_k) {
        const int pos = t0 + len - 1;
        if (own_row) {
            const float* kz = a.post_k + (size_t)kvh * hd;
            const float* vz = a.post_v + (size_t)kvh * hd;
            for (int i = tid; i < hd; i += NT) {
                ks[(size_t)pn * rs + i] = kz[i];
                const float v = vz[i];
                if (!SCORES_ONLY) vs[(size_t)pn * rs + i] = v;
                // the cache's new V row (the caches are writable whenever post_k is set)
                const_cast<float*>(a.vc)[(size_t)pos * ps + (size_t)kvh * a.kv_head_stride + i] = v;
            }
        }
        __syncthreads();
        // warps 0..G-1: the group's q heads; warp G: the new K row
        for (int task = warp; task < G + (own_row ? 1 : 0); task += NT / 32) {
            const bool isq = task < G;
            float* x = isq ? qs + (size_t)task * qrs : ks + (size_t)pn * rs;
            if (POST && post_pf)
                warp_head_norm_rope_pf(x, hd, hp, (isq ? a.post_qn : a.post_kn) != nullptr, a.post_norm != 0,
                                       a.post_eps, lane);
            else
                warp_head_norm_rope(x, hd, isq ? a.post_qn : a.post_kn, a.post_norm != 0, a.post_eps, a.rope_c,
                                    a.rope_s, pos, lane);
            if (!isq)
                for (int i = lane; i < hd; i += 32)
                    const_cast<float*>(a.kc)[(size_t)pos * ps + (size_t)kvh * a.kv_head_stride + i] = x[i];
        }
    }
    if (tid == 0) GNCX_TRACE_MARK(12, 0);
    if (BULK) {
        if (!mbar_wait(&s_bar[0], 0)) record_error(a.err, kErrTimeout);
    } else if (VEC) {
        cp_async_wait<0>();
    }
    __syncthreads();
    if (tid == 0) GNCX_TRACE_MARK(13, 0);

    // ---- scores (the reference's eight chains per dot) ----
    if (SCORES_ONLY) {
        float* row = a.scores + ((size_t)z * a.n_heads + kvh * G) * a.score_cap + c0;
        const int cap = a.score_cap;
        const float scale = a.scale;
        chunk_scores(ks, rs, qs, qrs, G, hd, cn,
                     [&](int g, int p, float dot) { row[(size_t)g * cap + p] = fmul(dot, scale); });
        return;  // the K copies have all landed (waited above)
    }
    {
        const float scale = a.scale;
        if (BULK)
            chunk_scores_warp(ks, hd, qs, qrs, G, cn, NT / 32,
                              [&](int g, int p, float dot) { sc[g * sld + p] = fmul(dot, scale); });
        else
            chunk_scores(ks, rs, qs, qrs, G, hd, cn,
                         [&](int g, int p, float dot) { sc[g * sld + p] = fmul(dot, scale); });
    }
    __syncthreads();

    if (tid == 0) GNCX_TRACE_MARK(14, 0);
    // ---- per head: chunk max, exp (position-major copy for the PV), sum ----
    for (int g = warp; g < G; g += NT / 32) {
        float mx = -INFINITY;
        for (int p = lane; p < cn; p += 32) mx = fmaxf(mx, sc[g * sld + p]);
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float sum = 0.0f;
        for (int p = lane; p < cn; p += 32) {
            const float e = exp_cr(fsub(sc[g * sld + p], mx));
            es[(size_t)p * G4 + g] = e;
            sum += e;
        }
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) { red[2 * g] = mx; red[2 * g + 1] = sum; }
    }
    for (int i = tid; i < cn * (G4 - G); i += NT) es[(size_t)(i / (G4 - G)) * G4 + G + i % (G4 - G)] = 0.0f;
    __syncthreads();

    if (tid == 0) GNCX_TRACE_MARK(15, 0);
    if (BULK && !mbar_wait(&s_bar[1], 0)) record_error(a.err, kErrTimeout);
    // ---- o[g][d] = sum_p e[p][g] * v[p][d] ----
    const int npg = NT / hd > 0 ? NT / hd : 1;
    const int d = tid % hd, pg = tid / hd;
    const bool active = pg < npg && d < hd && tid < npg * hd;
    for (int g0 = 0; g0 < G; g0 += kPvHeads) {
        const int ng = min(kPvHeads, G - g0);
        float acc[kPvHeads];
#pragma unroll
        for (int i = 0; i < kPvHeads; ++i) acc[i] = 0.0f;
        if (active)
            for (int dd = d; dd < hd; dd += npg * hd) chunk_pv(vs, rs, es, G4, g0, ng, cn, dd, pg, npg, acc);
        pv_reduce(acc, ng, hd, d, pg, npg, active, ks, [&](int i, int dd, float v) {
            const int h = kvh * G + g0 + i;
            float* rec = a.part + (((size_t)z * a.n_heads + h) * a.max_splits + split) * attn_record_floats(hd);
            rec[4 + dd] = v;
            if (dd == 0) { rec[0] = red[2 * (g0 + i)]; rec[1] = red[2 * (g0 + i) + 1]; }
        });
    }
}

// ---- long windows: one CTA per (range of chunks, KV head) streams its chunks ----
// A CTA walks kStreamChunk-position chunks of its KV head through two
// shared-memory buffers (cp.async: chunk j + 2 is in flight while chunk j is
// scored and summed) and keeps an online softmax per query head -- running
// maximum m, sum l and unnormalised output o, rescaled by e^(m_old - m_new)
// when a chunk raises the maximum -- so loading and computing overlap inside
// the CTA and the merge sees one record per CTA instead of one per chunk.
// Records {m, l, -, -, o[hd]} like the split-KV partial kernel's; split-KV
// softmax mode (sums in a different order from the reference's serial ones,
// outputs within ~1e-6 relative).  Rows are unpadded (kv rows of head_dim
// floats), scored with eight lanes per dot.
constexpr int kStreamThreads = 256;
constexpr int kStreamChunk = 32;
constexpr int kStreamCtasPerSm = 3;  // resident together, so one CTA's loads and latency overlap the others'

__host__ __device__ inline size_t attn_stream_smem_bytes(int G, int hd) {
    const int G4 = (G + 3) & ~3;
    return ((size_t)4 * kStreamChunk * hd                      // K and V, two buffers each
            + (size_t)G * attn_q_stride(hd)                    // q heads
            + (size_t)G * (kStreamChunk + kScorePad)           // scores
            + (size_t)kStreamChunk * G4                        // exp, position-major
            + (size_t)4 * G) * 4;                              // m, l, correction per head
}

__global__ void __launch_bounds__(kStreamThreads, kStreamCtasPerSm) attn_stream_kernel(const AttnArgs a, int cpp) {
    extern __shared__ __align__(16) uint8_t smraw[];
    GNCX_TRACE_SCOPE(kTagAttnPartial, gridDim.x);
    pdl_launch_dependents();
    pdl_wait();
    const int hd = a.hd;
    const int G = a.n_heads / a.n_kv, G4 = (G + 3) & ~3;
    const int part = blockIdx.x, kvh = blockIdx.y;
    int t0, len;
    attn_window(a, 0, t0, len);
    const int n_chunks = (len + kStreamChunk - 1) / kStreamChunk;
    const int j0 = part * cpp, j1 = min(n_chunks, j0 + cpp);
    if (j0 >= j1) return;  // uniform per CTA
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = kStreamThreads / 32;
    float* kb = reinterpret_cast<float*>(smraw);                  // [2][chunk][hd]
    float* vb = kb + (size_t)2 * kStreamChunk * hd;               // [2][chunk][hd]
    const int qrs = attn_q_stride(hd), sld = kStreamChunk + kScorePad;
    float* qs = vb + (size_t)2 * kStreamChunk * hd;               // [G][qrs]
    float* sc = qs + (size_t)G * qrs;                              // [G][sld]
    float* es = sc + (size_t)G * sld;                              // [chunk][G4]
    float* st = es + (size_t)kStreamChunk * G4;                    // [G]{m, l, corr, -}
    const size_t ps = (size_t)a.kv_pos_stride;
    const float* kbase = a.kc + (size_t)t0 * ps + (size_t)kvh * a.kv_head_stride;
    const float* vbase = a.vc + (size_t)t0 * ps + (size_t)kvh * a.kv_head_stride;
    const int cpr = hd >> 2;  // 16-byte pieces per row
    auto issue = [&](int j) {
        const int c0 = j * kStreamChunk;
        const int cn = min(kStreamChunk, len - c0);
        float* kd = kb + (size_t)(j & 1) * kStreamChunk * hd;
        float* vd = vb + (size_t)(j & 1) * kStreamChunk * hd;
        for (int i = tid; i < cn * cpr; i += kStreamThreads) {
            const int pp = i / cpr, c = i - pp * cpr;
            cp_async16(kd + (size_t)pp * hd + 4 * c, kbase + (size_t)(c0 + pp) * ps + 4 * c);
            cp_async16(vd + (size_t)pp * hd + 4 * c, vbase + (size_t)(c0 + pp) * ps + 4 * c);
        }
        cp_async_commit();
    };
    issue(j0);
    if (j0 + 1 < j1) issue(j0 + 1);
    const float* qz = a.q + (size_t)kvh * G * hd;
    for (int i = tid; i < G * hd; i += kStreamThreads) qs[(size_t)(i / hd) * qrs + i % hd] = qz[i];
    if (tid < G) { st[4 * tid] = -INFINITY; st[4 * tid + 1] = 0.0f; }
    // PV mapping: thread (d, position group pg) accumulates column d of every head
    const int npg = kStreamThreads / hd;
    const int d = tid % hd, pg = tid / hd;
    float acc[kPvHeads];
#pragma unroll
    for (int i = 0; i < kPvHeads; ++i) acc[i] = 0.0f;
    const float scale = a.scale;
    for (int j = j0; j < j1; ++j) {
        if (tid == 0) GNCX_TRACE_MARK(50, j - j0);
        if (j + 1 < j1) cp_async_wait<1>(); else cp_async_wait<0>();
        __syncthreads();  // chunk j landed for every thread; qs / stats written
        if (tid == 0) GNCX_TRACE_MARK(51, j - j0);
        const int c0 = j * kStreamChunk;
        const int cn = min(kStreamChunk, len - c0);
        const float* ks = kb + (size_t)(j & 1) * kStreamChunk * hd;
        const float* vs = vb + (size_t)(j & 1) * kStreamChunk * hd;
        chunk_scores_warp(ks, hd, qs, qrs, G, cn, NW, [&](int g, int pp, float dot) { sc[g * sld + pp] = fmul(dot, scale); });
        __syncthreads();
        if (tid == 0) GNCX_TRACE_MARK(52, j - j0);
        for (int g = warp; g < G; g += NW) {
            float mx = -INFINITY;
            for (int pp = lane; pp < cn; pp += 32) mx = fmaxf(mx, sc[g * sld + pp]);
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float m_old = st[4 * g];
            const float m_new = fmaxf(m_old, mx);
            float sum = 0.0f;
            for (int pp = lane; pp < cn; pp += 32) {
                const float e = exp_cr(fsub(sc[g * sld + pp], m_new));
                es[(size_t)pp * G4 + g] = e;
                sum += e;
            }
            for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            if (lane == 0) {
                const float corr = exp_cr(fsub(m_old, m_new));  // 0 for the first chunk (m_old = -inf)
                st[4 * g] = m_new;
                st[4 * g + 1] = fadd(fmul(st[4 * g + 1], corr), sum);
                st[4 * g + 2] = corr;
            }
        }
        for (int i = tid; i < cn * (G4 - G); i += kStreamThreads)
            es[(size_t)(i / (G4 - G)) * G4 + G + i % (G4 - G)] = 0.0f;
        __syncthreads();
        if (tid == 0) GNCX_TRACE_MARK(53, j - j0);
        if (pg < npg) {
#pragma unroll
            for (int i = 0; i < kPvHeads; ++i)
                if (i < G) acc[i] = fmul(acc[i], st[4 * i + 2]);
            chunk_pv(vs, hd, es, G4, 0, G, cn, d, pg, npg, acc);
        }
        __syncthreads();  // buffer j & 1 is free again
        if (tid == 0) GNCX_TRACE_MARK(54, j - j0);
        if (j + 2 < j1) issue(j + 2);
    }
    // sum the position groups' partial outputs (through the K buffers) and
    // write this CTA's record of every head of the group
    float* scr = kb;  // [npg][kPvHeads][hd] <= 2 * kStreamChunk * hd floats
    if (pg < npg) {
#pragma unroll
        for (int i = 0; i < kPvHeads; ++i)
            if (i < G) scr[((size_t)pg * kPvHeads + i) * hd + d] = acc[i];
    }
    __syncthreads();
    const size_t R = attn_record_floats(hd);
    for (int t = tid; t < G * hd; t += kStreamThreads) {
        const int i = t / hd, dd = t - i * hd;
        float v = scr[(size_t)i * hd + dd];
        for (int q = 1; q < npg; ++q) v += scr[((size_t)q * kPvHeads + i) * hd + dd];
        float* rec = a.part + ((size_t)(kvh * G + i) * a.max_splits + part) * R;
        rec[4 + dd] = v;
        if (dd == 0) { rec[0] = st[4 * i]; rec[1] = st[4 * i + 1]; }
    }
}

// Merge the split records of one (query, head).
constexpr int kCombineThreads = 256;
__global__ void __launch_bounds__(kCombineThreads) attn_combine_kernel(const AttnArgs a) {
    extern __shared__ float wsm[];  // [max_splits] weights, [max_splits] sums, [kCombineThreads] partial outputs
    GNCX_TRACE_SCOPE(kTagAttnCombine, gridDim.x);
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x == 0) GNCX_TRACE_MARK(30, 0);
    const int h = blockIdx.x, z = blockIdx.y;
    int t0, len;
    attn_window(a, z, t0, len);
    const int n = (len + a.chunk - 1) / a.chunk;
    attn_merge(a, z, h, n, wsm, wsm + a.max_splits, wsm + 2 * a.max_splits);
}

// ---- causal prefill: one CTA per (chunk, KV head, tile of queries) ----
// Many queries share each K/V chunk, so a CTA stages the chunk once and
// serves a tile of 64 (query, head) rows of the KV head's group: scores as a
// 64 x 64 register-blocked product (4 x 4 per thread), a per-row softmax over
// the positions each query may see (position <= its own), and the PV product,
// written as the same split records the combine kernel merges.  Split-KV
// softmax mode only; window 0; chunk of 64 positions.
constexpr int kPfRows = 64;  // (query, head) rows per CTA
constexpr int kPfChunk = 64;

static size_t attn_prefill_smem_bytes(int hd) {
    const int rs = hd + kRowPad;
    return ((size_t)3 * kPfRows * rs + (size_t)2 * kPfRows * (kPfChunk + 4) + 2 * kPfRows) * 4;
}

template <int HD>
__global__ void __launch_bounds__(kAttnThreads, 1) attn_prefill_kernel(const AttnArgs a) {
    extern __shared__ __align__(16) float psm[];
    GNCX_TRACE_SCOPE(kTagAttnPrefill, gridDim.x);
    constexpr int RS = HD + kRowPad;
    constexpr int SL = kPfChunk + 4;
    const int G = a.n_heads / a.n_kv;
    const int QT = kPfRows / G;  // queries per tile
    const int split = blockIdx.x, kvh = blockIdx.y;
    const int z0 = blockIdx.z * QT;
    const int c0 = split * kPfChunk;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    pdl_launch_dependents();
    pdl_wait();
    const int pos_first = (a.pos_dev ? *a.pos_dev : a.pos0) + z0;  // query z sits at position pos0 + z
    // the tile's last valid query sees the most positions (score_cap carries n_tok here)
    const int z_last = min(z0 + QT, a.score_cap) - 1;
    const int pos_last = pos_first + (z_last - z0);
    if (c0 > pos_last) return;  // uniform: no query of the tile sees this chunk
    const int cn = min(kPfChunk, pos_last + 1 - c0);
    float* ks = psm;                                  // [64][RS]
    float* vs = ks + kPfRows * RS;                    // [64][RS]
    float* qs = vs + kPfRows * RS;                    // [64 rows][RS]
    float* sc = qs + kPfRows * RS;                    // [64 rows][SL]
    float* es = sc + kPfRows * SL;                    // [64 positions][SL] (row index fastest)
    float* red = es + kPfRows * SL;                   // [64 rows][2]
    const size_t ps = (size_t)a.kv_pos_stride;
    const size_t row0 = (size_t)c0 * ps + (size_t)kvh * a.kv_head_stride;
    // ---- stage K/V rows [c0, c0+cn) and the tile's q rows ----
    {
        constexpr int CPR = HD / 4, STEP = kAttnThreads / CPR;
        const int c = tid % CPR, p0 = tid / CPR;
        for (int p = p0; p < cn; p += STEP) {
            cp_async16(ks + p * RS + 4 * c, a.kc + row0 + p * ps + 4 * c);
            cp_async16(vs + p * RS + 4 * c, a.vc + row0 + p * ps + 4 * c);
        }
        cp_async_commit();
        for (int i = tid; i < kPfRows * (HD / 4); i += kAttnThreads) {
            const int qr = i / (HD / 4), cc = i % (HD / 4);
            const int zl = qr / G, g = qr % G;
            const int z = z0 + zl;
            float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (z <= z_last)
                v = *reinterpret_cast<const float4*>(a.q + (size_t)z * a.q_stride + (size_t)(kvh * G + g) * HD + 4 * cc);
            *reinterpret_cast<float4*>(qs + qr * RS + 4 * cc) = v;
        }
        cp_async_wait<0>();
        __syncthreads();
    }
    // ---- scores: thread (i, j) owns rows 4i..4i+3 x positions j, j+16, j+32, j+48
    // (consecutive threads read consecutive padded K rows: no bank conflicts) ----
    {
        const int i = tid >> 4, j = tid & 15;
        float acc[4][4];
#pragma unroll
        for (int x = 0; x < 4; ++x)
#pragma unroll
            for (int y = 0; y < 4; ++y) acc[x][y] = 0.0f;
#pragma unroll 2
        for (int m = 0; m < HD / 8; ++m) {
            float4 q0[4], q1[4], k0[4], k1[4];
#pragma unroll
            for (int x = 0; x < 4; ++x) {
                q0[x] = *reinterpret_cast<const float4*>(qs + (4 * i + x) * RS + 8 * m);
                q1[x] = *reinterpret_cast<const float4*>(qs + (4 * i + x) * RS + 8 * m + 4);
                k0[x] = *reinterpret_cast<const float4*>(ks + (j + 16 * x) * RS + 8 * m);
                k1[x] = *reinterpret_cast<const float4*>(ks + (j + 16 * x) * RS + 8 * m + 4);
            }
#pragma unroll
            for (int x = 0; x < 4; ++x)
#pragma unroll
                for (int y = 0; y < 4; ++y) {
                    float t = acc[x][y];
                    t = fmaf(q0[x].x, k0[y].x, t); t = fmaf(q0[x].y, k0[y].y, t);
                    t = fmaf(q0[x].z, k0[y].z, t); t = fmaf(q0[x].w, k0[y].w, t);
                    t = fmaf(q1[x].x, k1[y].x, t); t = fmaf(q1[x].y, k1[y].y, t);
                    t = fmaf(q1[x].z, k1[y].z, t); t = fmaf(q1[x].w, k1[y].w, t);
                    acc[x][y] = t;
                }
        }
#pragma unroll
        for (int x = 0; x < 4; ++x) {
            const int qr = 4 * i + x;
            const int pos_q = pos_first + qr / G;
#pragma unroll
            for (int y = 0; y < 4; ++y) {
                const int p = j + 16 * y;
                sc[qr * SL + p] = (p < cn && c0 + p <= pos_q) ? acc[x][y] * a.scale : -INFINITY;
            }
        }
    }
    __syncthreads();
    // ---- softmax per row (a warp per row, 8 rows per warp) ----
    for (int qr = warp; qr < kPfRows; qr += kAttnThreads / 32) {
        const float s0 = sc[qr * SL + lane], s1 = sc[qr * SL + lane + 32];
        float mx = fmaxf(s0, s1);
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const bool live = mx != -INFINITY;
        const float e0 = live ? exp_cr(fsub(s0, mx)) : 0.0f, e1 = live ? exp_cr(fsub(s1, mx)) : 0.0f;
        es[lane * SL + qr] = e0;
        es[(lane + 32) * SL + qr] = e1;
        float sum = e0 + e1;
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) { red[2 * qr] = mx; red[2 * qr + 1] = sum; }
    }
    __syncthreads();
    // ---- PV: thread (i, j) owns rows 4i..4i+3 x columns (HD/16)*j .. ----
    {
        constexpr int DJ = HD / 16;  // columns per thread: 8 (HD 128) or 4 (HD 64)
        const int i = tid >> 4, j = tid & 15;
        float acc[4][DJ];
#pragma unroll
        for (int x = 0; x < 4; ++x)
#pragma unroll
            for (int y = 0; y < DJ; ++y) acc[x][y] = 0.0f;
        for (int p = 0; p < cn; ++p) {
            const float4 e = *reinterpret_cast<const float4*>(es + p * SL + 4 * i);
            float v[DJ];
#pragma unroll
            for (int y = 0; y < DJ; y += 4) {
                const float4 t = *reinterpret_cast<const float4*>(vs + p * RS + DJ * j + y);
                v[y] = t.x; v[y + 1] = t.y; v[y + 2] = t.z; v[y + 3] = t.w;
            }
            const float ex[4] = {e.x, e.y, e.z, e.w};
#pragma unroll
            for (int x = 0; x < 4; ++x)
#pragma unroll
                for (int y = 0; y < DJ; ++y) acc[x][y] = fmaf(ex[x], v[y], acc[x][y]);
        }
        const size_t R = attn_record_floats(HD);
#pragma unroll
        for (int x = 0; x < 4; ++x) {
            const int qr = 4 * i + x;
            const int zl = qr / G, g = qr % G;
            const int z = z0 + zl;
            if (z > z_last || c0 > pos_first + zl) continue;  // this query does not see the chunk
            float* rec = a.part + (((size_t)z * a.n_heads + kvh * G + g) * a.max_splits + split) * R;
#pragma unroll
            for (int y = 0; y < DJ; ++y) rec[4 + DJ * j + y] = acc[x][y];
            if (j == 0) { rec[0] = red[2 * qr]; rec[1] = red[2 * qr + 1]; }
        }
    }
}

// ---- one query over a long window: rows streamed through registers ----
// Each warp walks batches of B positions of one KV head; lane l holds columns
// [l*DPL, l*DPL + DPL) of the G query heads, of the running outputs, and of
// the K and V rows it loads (one coalesced vector load per row and lane,
// straight into registers: no shared-memory staging and no CTA barrier per
// batch).  The B*G partial dot products of a batch are summed across the warp
// by a reduce-scatter butterfly that leaves lane l with the total of
// (position, head) pair l >> SH; the online softmax (running maximum m, sum l
// of e^(s - m), outputs rescaled by e^(m_old - m_new)) runs on those lanes,
// and the batch's weights reach every lane through a per-warp shared-memory
// row.  After its range, the CTA merges its warps' states and writes one
// record {m, l, -, -, o[hd]} per head, in the split-KV partial kernel's
// format, for the combine kernel.  Split-KV softmax mode (sums in a different
// order from the reference's serial ones; outputs within ~1e-6 relative).
// Many warps per SM, each with a whole batch of rows in flight, keep HBM busy
// where the chunked kernels' per-chunk barriers and phases left it idle.
constexpr int kRowsThreads = 256;
constexpr int kRowsWarps = kRowsThreads / 32;
constexpr int kRowsMaxKv = 256;     // KV heads the in-kernel merge counts arrivals for
constexpr int kRowsMaxParts = 256;  // CTAs per KV head the in-kernel merge takes

// Arrivals per KV head of the CTAs of one attn_rows_kernel launch, for the
// in-kernel merge: zero when the module loads, and atomicInc wraps each back
// to zero at the launch's last arrival.
__device__ unsigned int g_rows_arrive[kRowsMaxKv];

template <int DPL>
__device__ __forceinline__ void rows_load(const float* p, float (&r)[DPL]) {
    if constexpr (DPL == 4) {
        const float4 v = __ldcs(reinterpret_cast<const float4*>(p));
        r[0] = v.x; r[1] = v.y; r[2] = v.z; r[3] = v.w;
    } else {
        const float2 v = __ldcs(reinterpret_cast<const float2*>(p));
        r[0] = v.x; r[1] = v.y;
    }
}

// One batch of B rows of a warp (loaded in kr / vr): scores, the online
// softmax update, the weighted V sum.  Lane l ends the butterfly with pair
// l >> SH = (position p, head g) = (my / G, my % G); m and l belong to that head.
template <int DPL, int G, int B>
__device__ __forceinline__ void rows_batch(const float (&q)[G][DPL], float (&o)[G][DPL], const float (&kr)[B][DPL],
                                           const float (&vr)[B][DPL], int n_valid, float scale, float& m, float& l,
                                           float* wsh, int lane) {
    constexpr int NV = B * G;
    constexpr int LNV = NV == 1 ? 0 : NV == 2 ? 1 : NV == 4 ? 2 : NV == 8 ? 3 : NV == 16 ? 4 : 5;
    constexpr int SH = 5 - LNV;
    constexpr int LG = G == 1 ? 0 : G == 2 ? 1 : G == 4 ? 2 : 3;
    const int my = lane >> SH;
    float v[NV];
#pragma unroll
    for (int p = 0; p < B; ++p)
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float c = 0.0f;
#pragma unroll
            for (int k = 0; k < DPL; ++k) c = fmaf(q[g][k], kr[p][k], c);
            v[p * G + g] = c;
        }
    // reduce-scatter: at offset o, lanes with bit o set keep the upper half
#pragma unroll
    for (int n = NV, lvl = 0; n > 1; n >>= 1, ++lvl) {
        const int off = 16 >> lvl;
        const bool up = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < n / 2; ++i) {
            const float send = up ? v[i] : v[i + n / 2];
            const float keep = up ? v[i + n / 2] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
    }
    float sc = v[0];
#pragma unroll
    for (int off = (1 << SH) >> 1; off > 0; off >>= 1) sc += __shfl_xor_sync(0xffffffffu, sc, off);
    sc = my / G < n_valid ? sc * scale : -INFINITY;
    // the head's maximum and sum over the batch: lanes whose pairs differ in position
    float bm = sc;
#pragma unroll
    for (int off = 16; off >= (1 << (SH + LG)); off >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, off));
    const float m_new = fmaxf(m, bm);
    const float e = __expf(sc - m_new);
    const float corr = __expf(m - m_new);  // 0 while m = -inf
    float bs = e;
#pragma unroll
    for (int off = 16; off >= (1 << (SH + LG)); off >>= 1) bs += __shfl_xor_sync(0xffffffffu, bs, off);
    l = fmaf(l, corr, bs);
    m = m_new;
    if ((lane & ((1 << SH) - 1)) == 0) wsh[my] = e;
    if (lane < (G << SH) && (lane & ((1 << SH) - 1)) == 0) wsh[32 + my] = corr;
    __syncwarp();
    float w[NV], cg[G];
#pragma unroll
    for (int i = 0; i < NV; ++i) w[i] = wsh[i];
#pragma unroll
    for (int g = 0; g < G; ++g) cg[g] = wsh[32 + g];
    __syncwarp();  // wsh is rewritten by the next batch
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int k = 0; k < DPL; ++k) {
            float acc = o[g][k] * cg[g];
#pragma unroll
            for (int p = 0; p < B; ++p) acc = fmaf(w[p * G + g], vr[p][k], acc);
            o[g][k] = acc;
        }
}

// PF: the next batch's rows are loaded before the current one is computed
// (two batches of registers in flight per warp).
// POSTQ (the engine's split-KV decode): q is the QKV GEMV's raw output and the
// kernel does the Q/K post step itself -- warps 0..G-1 norm and rotate the
// group's q heads in shared memory (warp_head_norm_rope, the partial kernel's
// arithmetic), and in the CTA whose range ends the window the last warp makes
// the new K row (normed, rotated) and stores it with the new V row in the
// cache at the query's position before the CTA's loads; the launch may hold
// CTAs past the window (ranges sized for the largest window the records
// cover), which exit at once and do not arrive at the merge.
template <int DPL, int G, int B, bool PF, bool MERGE, bool POSTQ>
__global__ void __launch_bounds__(kRowsThreads, 2) attn_rows_kernel(const AttnArgs a, int ppc) {
    constexpr int HD = DPL * 32;
    constexpr int NV = B * G;  // (position, head) pairs per batch
    static_assert(NV >= 1 && NV <= 32 && (NV & (NV - 1)) == 0, "pairs per batch: a power of two up to 32");
    constexpr int LNV = NV == 1 ? 0 : NV == 2 ? 1 : NV == 4 ? 2 : NV == 8 ? 3 : NV == 16 ? 4 : 5;
    constexpr int SH = 5 - LNV;
    __shared__ __align__(16) float wsh[kRowsWarps][32 + G];   // a batch's weights, then the heads' corrections
    __shared__ float mst[kRowsWarps][G], lst[kRowsWarps][G];
    __shared__ __align__(16) float ost[kRowsWarps][G][HD];
    GNCX_TRACE_SCOPE(kTagAttnPartial, gridDim.x);
    pdl_launch_dependents();
    pdl_wait();
    const int part = blockIdx.x, kvh = blockIdx.y;
    int t0, len;
    attn_window(a, 0, t0, len);
    const int p0 = part * ppc, p1 = min(len, p0 + ppc);
    if (p0 >= p1) return;  // uniform per CTA; the launch has none (parts = ceil(len / ppc))
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const size_t ps = (size_t)a.kv_pos_stride;
    const float* kbase = a.kc + (size_t)t0 * ps + (size_t)kvh * a.kv_head_stride + lane * DPL;
    const float* vbase = a.vc + (size_t)t0 * ps + (size_t)kvh * a.kv_head_stride + lane * DPL;
    float q[G][DPL], o[G][DPL];
    if constexpr (POSTQ) {
        __shared__ __align__(16) float qs[G][HD];
        __shared__ __align__(16) float kx[HD];
        const int pos = t0 + len - 1;
        const bool own = p1 == len;  // this CTA's range ends the window
        for (int i = threadIdx.x; i < G * HD; i += kRowsThreads) qs[i / HD][i % HD] = a.q[(size_t)kvh * G * HD + i];
        if (own)
            for (int i = threadIdx.x; i < HD; i += kRowsThreads) kx[i] = a.post_k[(size_t)kvh * HD + i];
        __syncthreads();
        if (warp < G)
            warp_head_norm_rope(qs[warp], HD, a.post_qn, a.post_norm != 0, a.post_eps, a.rope_c, a.rope_s, pos, lane);
        if (own && warp == kRowsWarps - 1) {
            warp_head_norm_rope(kx, HD, a.post_kn, a.post_norm != 0, a.post_eps, a.rope_c, a.rope_s, pos, lane);
            const size_t at = (size_t)pos * ps + (size_t)kvh * a.kv_head_stride;
            for (int i = lane; i < HD; i += 32) {
                const_cast<float*>(a.kc)[at + i] = kx[i];
                const_cast<float*>(a.vc)[at + i] = a.post_v[(size_t)kvh * HD + i];
            }
        }
        __syncthreads();  // q heads ready; the new K/V rows are in the cache for this CTA's loads
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int k = 0; k < DPL; ++k) {
                q[g][k] = qs[g][lane * DPL + k];
                o[g][k] = 0.0f;
            }
    } else {
#pragma unroll
        for (int g = 0; g < G; ++g) {
            rows_load<DPL>(a.q + (size_t)(kvh * G + g) * HD + lane * DPL, q[g]);
#pragma unroll
            for (int k = 0; k < DPL; ++k) o[g][k] = 0.0f;
        }
    }
    float m = -INFINITY, l = 0.0f;
    const float scale = a.scale;
    // the query's own rows, when given, come from new_k / new_v: the warp whose
    // batch holds that position stores them in the cache before its loads, and
    // each lane later reads back only what it stored itself (program order)
    const int last = len - 1;
    if (a.new_k && last >= p0 && last < p1 && warp == ((last - p0) / B) % kRowsWarps) {
        float r[DPL];
        const size_t at = (size_t)last * ps;
        rows_load<DPL>(a.new_k + (size_t)kvh * HD + lane * DPL, r);
#pragma unroll
        for (int k = 0; k < DPL; ++k) const_cast<float*>(kbase)[at + k] = r[k];
        rows_load<DPL>(a.new_v + (size_t)kvh * HD + lane * DPL, r);
#pragma unroll
        for (int k = 0; k < DPL; ++k) const_cast<float*>(vbase)[at + k] = r[k];
    }
    // rows past the range load a valid row and get weight 0
    auto load = [&](int b0, float (&kr)[B][DPL], float (&vr)[B][DPL]) {
#pragma unroll
        for (int p = 0; p < B; ++p) rows_load<DPL>(kbase + (size_t)min(b0 + p, p1 - 1) * ps, kr[p]);
#pragma unroll
        for (int p = 0; p < B; ++p) rows_load<DPL>(vbase + (size_t)min(b0 + p, p1 - 1) * ps, vr[p]);
    };
    constexpr int kStep = kRowsWarps * B;
    int b0 = p0 + warp * B;
    if constexpr (PF) {
        float ka[B][DPL], va[B][DPL], kb[B][DPL], vb[B][DPL];
        if (b0 < p1) load(b0, ka, va);
        while (b0 < p1) {
            if (b0 + kStep < p1) load(b0 + kStep, kb, vb);
            rows_batch<DPL, G, B>(q, o, ka, va, p1 - b0, scale, m, l, wsh[warp], lane);
            b0 += kStep;
            if (b0 >= p1) break;
            if (b0 + kStep < p1) load(b0 + kStep, ka, va);
            rows_batch<DPL, G, B>(q, o, kb, vb, p1 - b0, scale, m, l, wsh[warp], lane);
            b0 += kStep;
        }
    } else {
        for (; b0 < p1; b0 += kStep) {
            float kr[B][DPL], vr[B][DPL];
            load(b0, kr, vr);
            rows_batch<DPL, G, B>(q, o, kr, vr, p1 - b0, scale, m, l, wsh[warp], lane);
        }
    }
    // merge the warps' states: lanes 0, 1 << SH, ... (G << SH) - 1 hold head g's m and l
    if (lane < (G << SH) && (lane & ((1 << SH) - 1)) == 0) {
        mst[warp][lane >> SH] = m;
        lst[warp][lane >> SH] = l;
    }
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int k = 0; k < DPL; ++k) ost[warp][g][lane * DPL + k] = o[g][k];
    __syncthreads();
    const size_t R = attn_record_floats(HD);
    for (int t = threadIdx.x; t < G * HD; t += kRowsThreads) {
        const int g = t / HD, d = t - g * HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kRowsWarps; ++w) M = fmaxf(M, mst[w][g]);
        float L = 0.0f, O = 0.0f;
#pragma unroll
        for (int w = 0; w < kRowsWarps; ++w) {
            const float f = __expf(mst[w][g] - M);  // 0 for warps with no rows (m = -inf)
            L = fmaf(lst[w][g], f, L);
            O = fmaf(ost[w][g][d], f, O);
        }
        float* rec = a.part + ((size_t)(kvh * G + g) * a.max_splits + part) * R;
        rec[4 + d] = O;
        if (d == 0) { rec[0] = M; rec[1] = L; }
    }
    if constexpr (MERGE) {
        // the last CTA of this KV head to finish merges its heads' records:
        // out = sum_r o_r e^(m_r - M) / (sum_r l_r e^(m_r - M) + 1e-12), in one
        // pass per output pair of columns with a running maximum
        __shared__ int s_last;
        __syncthreads();  // this CTA's records are written
        const unsigned n_arr = (unsigned)((len + ppc - 1) / ppc);  // the CTAs whose range meets the window
        if (threadIdx.x == 0) {
            __threadfence();
            s_last = atomicInc(&g_rows_arrive[kvh], n_arr - 1) == n_arr - 1;
        }
        __syncthreads();
        if (!s_last) return;  // uniform per CTA
        __threadfence();
        const int n = (int)n_arr;
        constexpr int kRb = 16;  // records in flight per thread
        for (int t = threadIdx.x; t < G * HD / 2; t += kRowsThreads) {
            const int g = t / (HD / 2), d = 2 * (t - g * (HD / 2));
            const float* r0 = a.part + (size_t)(kvh * G + g) * a.max_splits * R;
            float M = -INFINITY, L = 0.0f, O0 = 0.0f, O1 = 0.0f;
            for (int rb = 0; rb < n; rb += kRb) {
                float2 ml[kRb], ov[kRb];
#pragma unroll
                for (int b = 0; b < kRb; ++b) {
                    const int r = min(rb + b, n - 1);
                    ml[b] = __ldcg(reinterpret_cast<const float2*>(r0 + (size_t)r * R));
                    ov[b] = __ldcg(reinterpret_cast<const float2*>(r0 + (size_t)r * R + 4 + d));
                }
                float bm = M;
#pragma unroll
                for (int b = 0; b < kRb; ++b) bm = fmaxf(bm, ml[b].x);
                const float c = __expf(M - bm);  // 0 on the first batch
                L *= c; O0 *= c; O1 *= c;
#pragma unroll
                for (int b = 0; b < kRb; ++b) {
                    const float w = rb + b < n ? __expf(ml[b].x - bm) : 0.0f;
                    L = fmaf(ml[b].y, w, L);
                    O0 = fmaf(ov[b].x, w, O0);
                    O1 = fmaf(ov[b].y, w, O1);
                }
                M = bm;
            }
            const float inv = 1.0f / (L + 1e-12f);
            *reinterpret_cast<float2*>(a.out + (size_t)(kvh * G + g) * HD + d) = make_float2(O0 * inv, O1 * inv);
        }
    }
}

template <int DPL, int G, bool MERGE, bool POSTQ>
static cudaError_t launch_rows_g(const AttnArgs& a, dim3 grid, int ppc, int B, cudaStream_t st) {
    constexpr int BMAX = 32 / G < 8 ? 32 / G : 8;
    constexpr int BPF = BMAX >= 4 ? 4 : BMAX;
    constexpr int BPP = G >= 8 ? 2 : BPF;  // two batches of registers in flight
    if constexpr (POSTQ) {  // one batch size: the engine's decode
        return launch_k(attn_rows_kernel<DPL, G, BMAX, false, MERGE, true>, grid, dim3(kRowsThreads), 0, st, a, ppc);
    } else {
        if (B < 0)
            return launch_k(attn_rows_kernel<DPL, G, BPP, true, MERGE, false>, grid, dim3(kRowsThreads), 0, st, a, ppc);
        if (B >= BMAX)
            return launch_k(attn_rows_kernel<DPL, G, BMAX, false, MERGE, false>, grid, dim3(kRowsThreads), 0, st, a,
                            ppc);
        return launch_k(attn_rows_kernel<DPL, G, BPF, false, MERGE, false>, grid, dim3(kRowsThreads), 0, st, a, ppc);
    }
}

// head_dim 64 or 128, G in {1, 2, 4, 8}
static bool rows_ok(const AttnArgs& a) {
    const int G = a.n_heads / a.n_kv;
    return (a.hd == 128 || a.hd == 64) && (G == 1 || G == 2 || G == 4 || G == 8) &&
           (((uintptr_t)a.kc | (uintptr_t)a.vc | (uintptr_t)a.q) & (a.hd == 128 ? 15 : 7)) == 0 &&
           a.kv_pos_stride % (a.hd / 32) == 0 && a.kv_head_stride % (a.hd / 32) == 0;
}

template <bool MERGE, bool POSTQ = false>
static cudaError_t launch_rows(const AttnArgs& a, dim3 grid, int ppc, int B, cudaStream_t st) {
    const int G = a.n_heads / a.n_kv;
    if (a.hd == 128) {
        switch (G) {
            case 1: return launch_rows_g<4, 1, MERGE, POSTQ>(a, grid, ppc, B, st);
            case 2: return launch_rows_g<4, 2, MERGE, POSTQ>(a, grid, ppc, B, st);
            case 4: return launch_rows_g<4, 4, MERGE, POSTQ>(a, grid, ppc, B, st);
            default: return launch_rows_g<4, 8, MERGE, POSTQ>(a, grid, ppc, B, st);
        }
    }
    switch (G) {
        case 1: return launch_rows_g<2, 1, MERGE, POSTQ>(a, grid, ppc, B, st);
        case 2: return launch_rows_g<2, 2, MERGE, POSTQ>(a, grid, ppc, B, st);
        case 4: return launch_rows_g<2, 4, MERGE, POSTQ>(a, grid, ppc, B, st);
        default: return launch_rows_g<2, 8, MERGE, POSTQ>(a, grid, ppc, B, st);
    }
}

// ---- exact mode (:1960-1987) ----
// Softmax in the reference's order: max over the window (its running max
// starts at -1e30), e_t = exp(s_t - max) (correctly rounded here; the reference
// uses the host expf), sum_exp serially over t, inv = 1/(sum_exp + 1e-12); the
// scores are replaced by p_t = e_t * inv.  One CTA per (head, query).
constexpr int kExactThreads = 256;
__global__ void __launch_bounds__(kExactThreads) attn_exact_softmax_kernel(const AttnArgs a) {
    GNCX_TRACE_SCOPE(kTagAttnExactSoftmax, gridDim.x);
    pdl_launch_dependents();
    pdl_wait();
    const int h = blockIdx.x, z = blockIdx.y;
    int t0, len;
    attn_window(a, z, t0, len);
    float* sc = a.scores + ((size_t)z * a.n_heads + h) * a.score_cap;
    __shared__ float red[32];
    __shared__ float s_inv;
    const int tid = threadIdx.x;
    float mx = -1e30f;
    for (int t = tid; t < len; t += kExactThreads) mx = fmaxf(mx, sc[t]);
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    mx = red[0];
    for (int k = 1; k < kExactThreads / 32; ++k) mx = fmaxf(mx, red[k]);
    for (int t = tid; t < len; t += kExactThreads) sc[t] = exp_cr(fsub(sc[t], mx));
    __syncthreads();
    if (tid == 0) {
        // serial sum; the vector loads run ahead of the dependent adds
        float sum = 0.0f;
        const int n4 = ((uintptr_t)sc & 15) == 0 ? (len & ~3) : 0;
        const float4* s4 = reinterpret_cast<const float4*>(sc);
#pragma unroll 8
        for (int i = 0; i < (n4 >> 2); ++i) {
            const float4 v = s4[i];
            sum = fadd(fadd(fadd(fadd(sum, v.x), v.y), v.z), v.w);
        }
        for (int t = n4; t < len; ++t) sum = fadd(sum, sc[t]);
        s_inv = fdiv(1.0f, fadd(sum, 1e-12f));
    }
    __syncthreads();
    const float inv = s_inv;
    for (int t = tid; t < len; t += kExactThreads) sc[t] = fmul(sc[t], inv);
}

// Exact mode, one query: softmax and PV in one kernel, one CTA per (KV head,
// kFusedCols output columns).  The CTA stages its columns of every V row of
// the window in shared memory -- the rows below the query's position before
// the dependency wait when they come from earlier steps -- then, for each of
// the group's G heads, the maximum of the scores, e_t = exp(s_t - max), the
// serial sum of e_t in position order, inv = 1 / (sum + 1e-12), the weights
// e_t * inv, and thread (head, column) runs out = sum over t in order of
// weight_t * v_t[d] (csrc/gncx_llm_kernels.cpp:1960-1988).  The same
// arithmetic as attn_exact_softmax_kernel + attn_exact_pv_kernel, without
// their round trip through global memory and with V in flight early: every
// CTA of a KV group repeats the group's softmax (a few microseconds of serial
// adds, in parallel across CTAs) instead of waiting for it.
constexpr int kFusedCols = 8;
constexpr int kFusedThreads = 256;

__host__ __device__ inline size_t attn_exact_fused_smem(int G, int len) {
    return ((size_t)len * kFusedCols + (size_t)G * ((len + 3) & ~3) + 64) * 4;
}

__global__ void __launch_bounds__(kFusedThreads) attn_exact_fused_kernel(const AttnArgs a) {
    extern __shared__ __align__(16) float fsm[];
    GNCX_TRACE_SCOPE(kTagAttnExactPv, gridDim.x);
    const int hd = a.hd, G = a.n_heads / a.n_kv;
    const int ncb = hd / kFusedCols;
    const int kvh = blockIdx.x / ncb, d0 = (blockIdx.x - kvh * ncb) * kFusedCols;
    int t0, len;
    attn_window(a, 0, t0, len);
    const int lp = (len + 3) & ~3;
    float* vsl = fsm;                                // [len][kFusedCols]
    float* es = vsl + (size_t)len * kFusedCols;      // [G][lp]: scores, then e, then weights
    float* red = es + (size_t)G * lp;                // [G] max, [G] inv
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const size_t ps = (size_t)a.kv_pos_stride;
    const float* vbase = a.vc + (size_t)t0 * ps + (size_t)kvh * a.kv_head_stride + d0;
    constexpr int kPieces = kFusedCols / 4;  // 16-byte pieces per row
    auto stage_v = [&](int ta, int tb) {
        for (int i = tid; i < (tb - ta) * kPieces; i += kFusedThreads) {
            const int t = ta + i / kPieces, c = i % kPieces;
            cp_async16(vsl + (size_t)t * kFusedCols + 4 * c, vbase + (size_t)t * ps + 4 * c);
        }
        cp_async_commit();
    };
    // rows below the query's own were written before the preceding kernel ran
    const int n_old = a.prefetch_old ? len - 1 : 0;
    if (n_old > 0) stage_v(0, n_old);
    pdl_launch_dependents();
    pdl_wait();
    stage_v(n_old, len);
    const float* sc = a.scores + (size_t)(kvh * G) * a.score_cap;
    for (int i = tid; i < G * len; i += kFusedThreads) {
        const int g = i / len, t = i - g * len;
        es[(size_t)g * lp + t] = sc[(size_t)g * a.score_cap + t];
    }
    __syncthreads();
    // maxima: warp w takes heads w, w + 8, ...
    for (int g = warp; g < G; g += kFusedThreads / 32) {
        float mx = -1e30f;
        for (int t = lane; t < len; t += 32) mx = fmaxf(mx, es[(size_t)g * lp + t]);
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) red[g] = mx;
    }
    __syncthreads();
    for (int i = tid; i < G * len; i += kFusedThreads) {
        const int g = i / len, t = i - g * len;
        es[(size_t)g * lp + t] = exp_cr(fsub(es[(size_t)g * lp + t], red[g]));
    }
    __syncthreads();
    // the serial sum of each head, one thread per head
    if (tid < G) {
        const float* e = es + (size_t)tid * lp;
        float sum = 0.0f;
        const float4* e4 = reinterpret_cast<const float4*>(e);
        const int n4 = len >> 2;
#pragma unroll 8
        for (int i = 0; i < n4; ++i) {
            const float4 v = e4[i];
            sum = fadd(fadd(fadd(fadd(sum, v.x), v.y), v.z), v.w);
        }
        for (int t = n4 * 4; t < len; ++t) sum = fadd(sum, e[t]);
        red[G + tid] = fdiv(1.0f, fadd(sum, 1e-12f));
    }
    __syncthreads();
    for (int i = tid; i < G * len; i += kFusedThreads) {
        const int g = i / len, t = i - g * len;
        es[(size_t)g * lp + t] = fmul(es[(size_t)g * lp + t], red[G + g]);
    }
    cp_async_wait<0>();
    __syncthreads();
    // thread (head g, column c): the serial weighted sum over the window
    if (tid < G * kFusedCols) {
        const int g = tid / kFusedCols, c = tid - g * kFusedCols;
        const float* w = es + (size_t)g * lp;
        float acc = 0.0f;
#pragma unroll 8
        for (int t = 0; t < len; ++t) acc = fadd(acc, fmul(w[t], vsl[(size_t)t * kFusedCols + c]));
        a.out[(size_t)(kvh * G + g) * hd + d0 + c] = acc;
    }
}

// Exact mode, one query, G <= 4, windows up to 4096 positions: two kernels.
// attn_exact_softmax_reg_kernel (one CTA per head) forms the maximum, the
// exps, their serial sum and the weights p_t = e_t * inv once per head;
// attn_exact_reg_kernel (one CTA per (KV head, 8 output columns)) stages its
// columns of every V row while the softmax runs, then forms each output
// element's serial sum of p_t * v_t[d].  Every serial chain runs from
// registers: the window is cut into 32-position segments, a chain's segment
// s is held by lane s % 32 of the warp that runs the chain (one pass per 32
// segments), and the segments are added one after the other -- the running
// sum handed to the next lane by a shuffle -- so the adds are the
// reference's, in its order, with no shared-memory load on the chain.  Warp w
// of the PV kernel runs the four output columns 4 (w % 2) .. + 3 of head
// w / 2 as four interleaved chains, their products formed in registers per
// pass.  Shared memory keeps 4 floats of padding after every 32 positions (V
// rows and the weights), so that the 32 lanes' loads of their segments hit
// different banks.  8B exact-mode decode 3.20 -> 3.07 ms/token against
// attn_exact_fused_kernel, where every PV CTA formed its group's whole
// softmax (8200 double-precision exps at ~2050 positions, 16 times per KV
// head) itself; the same one-kernel design with register chains measured
// 3.23-3.54.
constexpr int kXSeg = 32;  // positions per chain segment
__host__ __device__ inline int xidx(int t) { return t + ((t >> 5) << 2); }
__host__ __device__ inline size_t attn_exact_reg_smem(int G, int len) {
    const size_t nseg = (size_t)(len + kXSeg - 1) / kXSeg;
    return (nseg * (kXSeg * kFusedCols + 4) + (size_t)G * nseg * (kXSeg + 4)) * 4;
}

// The serial sum over t < len of e[xidx(t)] (non-negative terms) by one warp:
// lane L holds segment p0 + L of 32 positions in registers, the segments are
// added one after the other (the running sum handed to the next lane by a
// shuffle), 32 segments per pass.  Positions past the window add +0, which
// leaves a sum of non-negative terms unchanged.  Returns the sum in every lane.
__device__ __forceinline__ float seg_chain_sum(const float* e, int nseg, int len, int lane) {
    float carry = 0.0f;
    for (int p0 = 0; p0 < nseg; p0 += 32) {
        const int sg = p0 + lane;
        float r[kXSeg];
#pragma unroll
        for (int q = 0; q < kXSeg / 4; ++q) {
            const float4 v = sg < nseg ? *reinterpret_cast<const float4*>(e + (size_t)sg * (kXSeg + 4) + 4 * q)
                                       : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            const int tq = sg * kXSeg + 4 * q;
            r[4 * q] = tq < len ? v.x : 0.0f;
            r[4 * q + 1] = tq + 1 < len ? v.y : 0.0f;
            r[4 * q + 2] = tq + 2 < len ? v.z : 0.0f;
            r[4 * q + 3] = tq + 3 < len ? v.w : 0.0f;
        }
        const int nr = min(32, nseg - p0);
        float ain = lane == 0 ? carry : 0.0f, last = 0.0f;
        for (int k = 0; k < nr; ++k) {  // round k: lane k's segment continues the chain
            float x = ain;
#pragma unroll
            for (int i = 0; i < kXSeg; ++i) x = fadd(x, r[i]);
            last = x;
            ain = __shfl_up_sync(0xffffffffu, x, 1);
        }
        carry = __shfl_sync(0xffffffffu, last, nr - 1);
    }
    return carry;
}

constexpr int kXPer = 16;                          // scores per thread per head held in registers
constexpr int kXMaxLen = kXPer * kFusedThreads;    // windows up to 4096 positions

// One query, one CTA per head: the maximum of the scores, e_t = exp(s_t - max)
// (every thread 16 positions, the loads all in flight at once), the serial
// sum of e_t in position order by one warp with the chain in registers
// (seg_chain_sum), inv = 1 / (sum + 1e-12), and the weights e_t * inv written
// over the scores for attn_exact_reg_kernel<G, true>.  Computing the exps once
// per head here, instead of in every CTA of the PV kernel (16 per KV head at
// head_dim 128), keeps them off each PV CTA's path.
__global__ void __launch_bounds__(kFusedThreads, 1) attn_exact_softmax_reg_kernel(const AttnArgs a) {
    __shared__ __align__(16) float es[kXMaxLen / kXSeg * (kXSeg + 4)];
    __shared__ float wmax[kFusedThreads / 32];
    __shared__ float s_inv;
    GNCX_TRACE_SCOPE(kTagAttnExactSoftmax, gridDim.x);
    pdl_launch_dependents();
    pdl_wait();
    const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int t0, len;
    attn_window(a, 0, t0, len);
    float* sc = a.scores + (size_t)h * a.score_cap;
    float v[kXPer];
#pragma unroll
    for (int k = 0; k < kXPer; ++k) {
        const int t = tid + k * kFusedThreads;
        v[k] = t < len ? ld_l2(sc + t) : -1e30f;
    }
    float mx = -1e30f;  // the reference's running max starts at -1e30
#pragma unroll
    for (int k = 0; k < kXPer; ++k) mx = fmaxf(mx, v[k]);
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) wmax[warp] = mx;
    __syncthreads();
    mx = wmax[0];
#pragma unroll
    for (int w = 1; w < kFusedThreads / 32; ++w) mx = fmaxf(mx, wmax[w]);
#pragma unroll
    for (int k = 0; k < kXPer; ++k) {
        const int t = tid + k * kFusedThreads;
        if (t < len) {
            v[k] = exp_cr(fsub(v[k], mx));
            es[xidx(t)] = v[k];
        }
    }
    __syncthreads();
    if (warp == 0) {
        const float sum = seg_chain_sum(es, (len + kXSeg - 1) / kXSeg, len, lane);
        if (lane == 0) s_inv = fdiv(1.0f, fadd(sum, 1e-12f));
    }
    __syncthreads();
    const float inv = s_inv;
#pragma unroll
    for (int k = 0; k < kXPer; ++k) {
        const int t = tid + k * kFusedThreads;
        if (t < len) sc[t] = fmul(v[k], inv);
    }
}

template <int G>
__global__ void __launch_bounds__(kFusedThreads) attn_exact_reg_kernel(const AttnArgs a) {
    extern __shared__ __align__(16) float fsm[];
    GNCX_TRACE_SCOPE(kTagAttnExactPv, gridDim.x);
    const int hd = a.hd;
    const int ncb = hd / kFusedCols;
    const int kvh = blockIdx.x / ncb, d0 = (blockIdx.x - kvh * ncb) * kFusedCols;
    int t0, len;
    attn_window(a, 0, t0, len);
    const int nseg = (len + kXSeg - 1) / kXSeg;
    const int lp = nseg * (kXSeg + 4);                            // floats per head row of es
    float* vsl = fsm;                                               // row t at t * 8 + (t / 32) * 4
    float* es = vsl + (size_t)nseg * (kXSeg * kFusedCols + 4);      // [G][lp] weights, position t at xidx(t)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const size_t ps = (size_t)a.kv_pos_stride;
    const float* vbase = a.vc + (size_t)t0 * ps + (size_t)kvh * a.kv_head_stride + d0;
    constexpr int kPieces = kFusedCols / 4;  // 16-byte pieces per row
    auto stage_v = [&](int ta, int tb) {
        for (int i = tid; i < (tb - ta) * kPieces; i += kFusedThreads) {
            const int t = ta + i / kPieces, c = i % kPieces;
            cp_async16(vsl + (size_t)t * kFusedCols + ((t >> 5) << 2) + 4 * c, vbase + (size_t)t * ps + 4 * c);
        }
        cp_async_commit();
    };
    // rows below the query's own were written before the preceding kernel ran
    const int n_old = a.prefetch_old ? len - 1 : 0;
    if (n_old > 0) stage_v(0, n_old);
    pdl_launch_dependents();
    pdl_wait();
    stage_v(n_old, len);
    if (tid == 0) GNCX_TRACE_MARK(60, 0);
    // the weights p_t, written over the scores by attn_exact_softmax_reg_kernel
    const float* sc = a.scores + (size_t)(kvh * G) * a.score_cap;
    float v[G][kXPer];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int k = 0; k < kXPer; ++k) {
            const int t = tid + k * kFusedThreads;
            v[g][k] = t < len ? ld_l2(sc + (size_t)g * a.score_cap + t) : 0.0f;
        }
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int k = 0; k < kXPer; ++k) {
            const int t = tid + k * kFusedThreads;
            if (t < len) es[(size_t)g * lp + xidx(t)] = v[g][k];
        }
    cp_async_wait<0>();
    __syncthreads();
    if (tid == 0) GNCX_TRACE_MARK(63, 0);
    // out[g][d0 + c0 + ch] = sum over t in order of w_t * v_t[d0 + c0 + ch]
    if (warp < 2 * G) {
        const int g = warp >> 1, c0 = (warp & 1) * 4;
        const float* wr = es + (size_t)g * lp;
        float carry0 = 0.0f, carry1 = 0.0f, carry2 = 0.0f, carry3 = 0.0f;
        for (int p0 = 0; p0 < nseg; p0 += 32) {
            const int sg = p0 + lane;
            const bool segok = sg < nseg;
            const float* wseg = wr + (size_t)sg * (kXSeg + 4);
            const float* vseg = vsl + (size_t)sg * (kXSeg * kFusedCols + 4) + c0;
            float p0r[kXSeg], p1r[kXSeg], p2r[kXSeg], p3r[kXSeg];
#pragma unroll
            for (int q = 0; q < kXSeg / 4; ++q) {
                const float4 w4 = segok ? *reinterpret_cast<const float4*>(wseg + 4 * q)
                                        : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int i = 4 * q + k;
                    const bool ok = segok && sg * kXSeg + i < len;
                    const float4 v4 = ok ? *reinterpret_cast<const float4*>(vseg + (size_t)i * kFusedCols)
                                         : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    const float wv = k == 0 ? w4.x : k == 1 ? w4.y : k == 2 ? w4.z : w4.w;
                    p0r[i] = ok ? fmul(wv, v4.x) : 0.0f;
                    p1r[i] = ok ? fmul(wv, v4.y) : 0.0f;
                    p2r[i] = ok ? fmul(wv, v4.z) : 0.0f;
                    p3r[i] = ok ? fmul(wv, v4.w) : 0.0f;
                }
            }
            const int nr = min(32, nseg - p0);
            float a0 = lane == 0 ? carry0 : 0.0f, a1 = lane == 0 ? carry1 : 0.0f;
            float a2 = lane == 0 ? carry2 : 0.0f, a3 = lane == 0 ? carry3 : 0.0f;
            float l0 = 0.0f, l1 = 0.0f, l2 = 0.0f, l3 = 0.0f;
            for (int k = 0; k < nr; ++k) {
                float x0 = a0, x1 = a1, x2 = a2, x3 = a3;
#pragma unroll
                for (int i = 0; i < kXSeg; ++i) {
                    x0 = fadd(x0, p0r[i]);
                    x1 = fadd(x1, p1r[i]);
                    x2 = fadd(x2, p2r[i]);
                    x3 = fadd(x3, p3r[i]);
                }
                l0 = x0; l1 = x1; l2 = x2; l3 = x3;
                a0 = __shfl_up_sync(0xffffffffu, x0, 1);
                a1 = __shfl_up_sync(0xffffffffu, x1, 1);
                a2 = __shfl_up_sync(0xffffffffu, x2, 1);
                a3 = __shfl_up_sync(0xffffffffu, x3, 1);
            }
            carry0 = __shfl_sync(0xffffffffu, l0, nr - 1);
            carry1 = __shfl_sync(0xffffffffu, l1, nr - 1);
            carry2 = __shfl_sync(0xffffffffu, l2, nr - 1);
            carry3 = __shfl_sync(0xffffffffu, l3, nr - 1);
        }
        if (lane == 0) {
            float* o = a.out + (size_t)(kvh * G + g) * hd + d0 + c0;
            o[0] = carry0;
            o[1] = carry1;
            o[2] = carry2;
            o[3] = carry3;
        }
    }
}

// out[h][d] = sum over t (serial) of p_t * v_t[d].  One CTA per (KV head,
// group of up to 8 query heads, slice of kExactSlice output columns, query);
// thread (g, d) runs one chain.  V rows and p stream through double-buffered
// shared memory in tiles of kExactTile positions.
constexpr int kExactSlice = 32;
static_assert(kExactSlice == 32, "one warp per (head, 32 columns): one act block, quantized in the PV kernel");
constexpr int kExactTile = 64;
constexpr int kExactHeads = kExactThreads / kExactSlice;  // 8
template <bool VEC>
__global__ void __launch_bounds__(kExactThreads) attn_exact_pv_kernel(const AttnArgs a) {
    GNCX_TRACE_SCOPE(kTagAttnExactPv, gridDim.x);
    pdl_launch_dependents();
    pdl_wait();
    __shared__ __align__(16) float vt[2][kExactTile][kExactSlice];
    __shared__ __align__(16) float pt[2][kExactHeads][kExactTile];
    const int slices = (a.hd + kExactSlice - 1) / kExactSlice;
    const int G = a.n_heads / a.n_kv;
    const int hgroups = (G + kExactHeads - 1) / kExactHeads;
    int bx = blockIdx.x;
    const int slice = bx % slices;
    bx /= slices;
    const int hg = bx % hgroups;
    const int kvh = bx / hgroups;
    const int z = blockIdx.y;
    const int d0 = slice * kExactSlice;
    const int g0 = hg * kExactHeads;
    const int ng = min(kExactHeads, G - g0);
    int t0, len;
    attn_window(a, z, t0, len);
    const int tid = threadIdx.x;
    const int g = tid / kExactSlice, dl = tid % kExactSlice;
    const int nd = min(kExactSlice, a.hd - d0);
    const bool active = g < ng && dl < nd;
    const float* vbase = a.vc + (size_t)t0 * a.kv_pos_stride + (size_t)kvh * a.kv_head_stride + d0;
    const size_t ps = (size_t)a.kv_pos_stride;
    const float* pbase = a.scores + ((size_t)z * a.n_heads + kvh * G + g0) * a.score_cap;
    const int n_tiles = (len + kExactTile - 1) / kExactTile;
    auto issue = [&](int tile, int buf) {
        const int tb = tile * kExactTile;
        const int tn = min(kExactTile, len - tb);
        if (VEC) {
            const int vp = nd >> 2;  // 16-byte pieces per V row slice
            for (int i = tid; i < tn * vp; i += kExactThreads) {
                const int t = i / vp, c = i - t * vp;
                cp_async16(&vt[buf][t][4 * c], vbase + (size_t)(tb + t) * ps + 4 * c);
            }
            const int pp = (tn + 3) >> 2;  // 16-byte pieces of p per head
            for (int i = tid; i < ng * pp; i += kExactThreads) {
                const int gg = i / pp, c = i - gg * pp;
                cp_async16(&pt[buf][gg][4 * c], pbase + (size_t)gg * a.score_cap + tb + 4 * c);
            }
        } else {
            for (int i = tid; i < tn * nd; i += kExactThreads) {
                const int t = i / nd, c = i - t * nd;
                vt[buf][t][c] = vbase[(size_t)(tb + t) * ps + c];
            }
            for (int i = tid; i < ng * tn; i += kExactThreads) {
                const int gg = i / tn, t = i - gg * tn;
                pt[buf][gg][t] = pbase[(size_t)gg * a.score_cap + tb + t];
            }
        }
        cp_async_commit();
    };
    float o = 0.0f;
    issue(0, 0);
    for (int tile = 0; tile < n_tiles; ++tile) {
        const int buf = tile & 1;
        if (tile + 1 < n_tiles) issue(tile + 1, buf ^ 1);
        else cp_async_commit();  // an empty group keeps the wait count uniform
        cp_async_wait<1>();
        __syncthreads();
        const int tn = min(kExactTile, len - tile * kExactTile);
        if (active) {
            const float* pp = pt[buf][g];
#pragma unroll 16
            for (int t = 0; t < tn; ++t) o = fadd(o, fmul(pp[t], vt[buf][t][dl]));
        }
        __syncthreads();  // the buffer is refilled two tiles on
    }
    if (!active) return;  // whole warps: g is the warp, and with act every lane of it is active
    const int h = kvh * G + g0 + g;
    const size_t col = (size_t)h * a.hd + d0 + dl;
    a.out[(size_t)z * a.out_stride + col] = o;
    // re-quantized for the next GEMV here: a warp holds one 32-column block of one head
    if (a.act_out.blocks || a.act_out.staged)
        act_out_store(a.act_out, o, a.n_heads * a.hd, (size_t)z, (int)(col >> 5), dl);
}

// Positions per split of the drop-in decode step: 64, halved (down to 16)
// while the window gives fewer than two CTAs per SM (splits x KV heads).
int attention_geometry_chunk(int32_t len, int32_t n_kv, int sm_count) {
    int c = 64;
    // shorter chunks when the window is small, so every SM gets ~2 CTAs
    while (c > 16 && (int64_t)((len + c - 1) / c) * n_kv < 2 * (int64_t)sm_count) c >>= 1;
    return c;
}

// 512 threads when head_dim <= 128 and the grid is at most two CTAs per SM
// (decode at a few thousand positions: one score per thread for 128 positions
// x 4 heads, four position groups in the PV; 2.26 vs 2.31 ms/token on the 8B
// shape), else 256 (long windows: more resident CTAs per SM, 136 vs 148 us at
// 32768 positions).
template <bool VEC, bool SCORES_ONLY>
static cudaError_t launch_partial(const AttnArgs& a, dim3 grid, size_t smem, cudaStream_t st) {
    static const int force = getenv("GNCX_ATTN_THREADS") ? atoi(getenv("GNCX_ATTN_THREADS")) : 0;  // tuning override
    const bool wide = force ? force == 512
                            : a.hd <= 128 && (int64_t)grid.x * grid.y * grid.z <= 2 * (int64_t)device_info().sm_count;
    // one bulk copy per chunk for K and for V where a chunk of a head is
    // contiguous (the engine's head-major cache), split-KV mode
    static const bool no_bulk = getenv("GNCX_ATTN_NO_BULK") != nullptr;  // tuning override
    const int G = a.n_heads / a.n_kv;
    const bool bulk = !no_bulk && VEC && !SCORES_ONLY && a.kv_pos_stride == a.hd && a.hd % 8 == 0 && a.hd <= 128 &&
                      (G == 1 || G == 2 || G == 4) && (((uintptr_t)a.kc | (uintptr_t)a.vc) & 15) == 0 &&
                      (a.kv_head_stride % 4) == 0;
    constexpr bool kSplit = VEC && !SCORES_ONLY;  // the instantiations with bulk / post variants
    const bool post = kSplit && a.post_k != nullptr;
    void (*k)(const AttnArgs) = nullptr;
    if (bulk && post) k = wide ? attn_partial_kernel<VEC, SCORES_ONLY, 512, kSplit, kSplit>
                               : attn_partial_kernel<VEC, SCORES_ONLY, 256, kSplit, kSplit>;
    else if (bulk) k = wide ? attn_partial_kernel<VEC, SCORES_ONLY, 512, kSplit, false>
                            : attn_partial_kernel<VEC, SCORES_ONLY, 256, kSplit, false>;
    else if (post) k = wide ? attn_partial_kernel<VEC, SCORES_ONLY, 512, false, kSplit>
                            : attn_partial_kernel<VEC, SCORES_ONLY, 256, false, kSplit>;
    else k = wide ? attn_partial_kernel<VEC, SCORES_ONLY, 512, false, false>
                  : attn_partial_kernel<VEC, SCORES_ONLY, 256, false, false>;
    const cudaError_t e = set_smem_limit(k, smem);
    if (e != cudaSuccess) return e;
    return launch_k(k, grid, dim3(wide ? 512 : 256), smem, st, a);
}

bool attention_shape_ok(int32_t n_heads, int32_t n_kv, int32_t hd) {
    return n_heads > 0 && n_kv > 0 && hd > 0 && n_heads % n_kv == 0 && hd <= kMaxHeadDim && (hd & 3) == 0;
}

// The query's new K/V rows into the cache at its position (paths whose
// kernels read that position from the cache).
static cudaError_t store_new_rows(const AttnArgs& a, cudaStream_t st) {
    const size_t row = (size_t)a.hd * 4;
    float* kd = const_cast<float*>(a.kc) + (size_t)a.pos0 * a.kv_pos_stride;
    float* vd = const_cast<float*>(a.vc) + (size_t)a.pos0 * a.kv_pos_stride;
    if (a.kv_head_stride == a.hd) {  // the heads of a position are one contiguous row
        const cudaError_t e = cudaMemcpyAsync(kd, a.new_k, a.n_kv * row, cudaMemcpyDefault, st);
        return e != cudaSuccess ? e : cudaMemcpyAsync(vd, a.new_v, a.n_kv * row, cudaMemcpyDefault, st);
    }
    const size_t pitch = (size_t)a.kv_head_stride * 4;
    const cudaError_t e = cudaMemcpy2DAsync(kd, pitch, a.new_k, row, row, a.n_kv, cudaMemcpyDefault, st);
    return e != cudaSuccess ? e : cudaMemcpy2DAsync(vd, pitch, a.new_v, row, row, a.n_kv, cudaMemcpyDefault, st);
}

int attention_run(const AttnArgs& args, int32_t n_tok, cudaStream_t st) {
    const AttnArgs& a = args;
    if (!a.q || !a.kc || !a.vc || !a.part || a.n_heads <= 0 || a.n_kv <= 0 || a.hd <= 0 || n_tok <= 0)
        return kErrInvalidArg;
    if (a.n_heads % a.n_kv != 0 || a.hd > kMaxHeadDim || (a.hd & 3) || a.chunk <= 0 || a.max_splits <= 0)
        return kErrInvalidArg;
    const bool act = a.act_out.blocks || a.act_out.staged;
    if (act && a.hd % 32) return kErrInvalidArg;
    if (a.post_k && (n_tok != 1 || !a.post_v || !a.rope_c || !a.rope_s || (a.hd & 1))) return kErrInvalidArg;
    if (a.new_k && (n_tok != 1 || !a.new_v || a.pos_dev || a.post_k)) return kErrInvalidArg;
    if (a.act_out.staged && (n_tok != 1 || (a.n_heads * a.hd) % 256 || ((uintptr_t)a.act_out.staged & 15)))
        return kErrInvalidArg;
    const DeviceInfo& dev = device_info();
    const int G = a.n_heads / a.n_kv;
    const size_t smem = attn_smem_bytes(G, a.hd, a.chunk);
    if (smem > (size_t)dev.max_smem_optin) return kErrCapacity;
    const bool vec = ((uintptr_t)a.kc % 16 == 0) && ((uintptr_t)a.vc % 16 == 0) && (a.kv_pos_stride % 4 == 0) &&
                     (a.kv_head_stride % 4 == 0);
    dim3 grid(a.max_splits, a.n_kv, n_tok);
    cudaError_t e;
    if (a.exact) {
        if (!a.scores || a.score_cap < a.max_splits * a.chunk || (a.score_cap & 3)) return kErrCapacity;
        if (!a.out) return kErrInvalidArg;
        if (a.new_k && store_new_rows(a, st) != cudaSuccess) return kErrCuda;
        e = vec ? launch_partial<true, true>(a, grid, smem, st) : launch_partial<false, true>(a, grid, smem, st);
        if (e != cudaSuccess) return kErrCuda;
        // one query whose window's V columns fit a CTA's shared memory: softmax
        // and PV fused (the output in fp32 only; no re-quantized act)
        int len1 = 0;
        if (n_tok == 1 && !a.pos_dev) {
            const int t0 = a.window > 0 ? (a.pos0 - a.window + 1 > 0 ? a.pos0 - a.window + 1 : 0) : 0;
            len1 = a.pos0 + 1 - t0;
        } else if (n_tok == 1) {
            len1 = a.score_cap;  // upper bound: the position is read on the device
        }
        // G <= 4: the register-chain kernel
        static const bool no_reg = getenv("GNCX_EXACT_SMEM_CHAINS") != nullptr;  // A/B override
        const size_t rsm = attn_exact_reg_smem(G, len1);
        if (!no_reg && n_tok == 1 && vec && !act && a.hd % kFusedCols == 0 && (G == 1 || G == 2 || G == 4) &&
            len1 > 0 && len1 <= kXMaxLen && rsm <= (size_t)dev.max_smem_optin && !getenv("GNCX_EXACT_UNFUSED")) {
            // the softmax once per head, then the PV per (KV head, 8 columns)
            void (*k)(const AttnArgs) = G == 4 ? attn_exact_reg_kernel<4>
                                        : G == 2 ? attn_exact_reg_kernel<2> : attn_exact_reg_kernel<1>;
            if (set_smem_limit(k, rsm) != cudaSuccess) return kErrCuda;
            if (launch_k(attn_exact_softmax_reg_kernel, dim3(a.n_heads), dim3(kFusedThreads), 0, st, a) != cudaSuccess)
                return kErrCuda;
            return launch_k(k, dim3(a.n_kv * (a.hd / kFusedCols)), dim3(kFusedThreads), rsm, st, a) == cudaSuccess
                       ? kOk
                       : kErrCuda;
        }
        const size_t fsm = attn_exact_fused_smem(G, len1);
        if (n_tok == 1 && vec && !act && a.hd % kFusedCols == 0 && G * kFusedCols <= kFusedThreads && len1 > 0 &&
            fsm <= (size_t)dev.max_smem_optin && !getenv("GNCX_EXACT_UNFUSED")) {
            if (set_smem_limit(attn_exact_fused_kernel, fsm) != cudaSuccess) return kErrCuda;
            return launch_k(attn_exact_fused_kernel, dim3(a.n_kv * (a.hd / kFusedCols)), dim3(kFusedThreads), fsm, st,
                            a) == cudaSuccess
                       ? kOk
                       : kErrCuda;
        }
        if (launch_k(attn_exact_softmax_kernel, dim3(a.n_heads, n_tok), dim3(kExactThreads), 0, st, a) != cudaSuccess)
            return kErrCuda;
        const int slices = (a.hd + kExactSlice - 1) / kExactSlice;
        const int hgroups = (G + kExactHeads - 1) / kExactHeads;
        const dim3 pv_grid(a.n_kv * hgroups * slices, n_tok);
        e = (vec && ((uintptr_t)a.scores & 15) == 0)
                ? launch_k(attn_exact_pv_kernel<true>, pv_grid, dim3(kExactThreads), 0, st, a)
                : launch_k(attn_exact_pv_kernel<false>, pv_grid, dim3(kExactThreads), 0, st, a);
        if (e != cudaSuccess) return kErrCuda;
        return kOk;  // the PV kernel also wrote act_out
    }
    const int Gq = a.n_heads / a.n_kv;
    // One query, window known on the host (the drop-in step): rows streamed
    // through registers, ~2 CTAs per SM, each a range of positions of one KV head
    static const bool no_rows = getenv("GNCX_ATTN_NO_ROWS") != nullptr;  // tuning overrides
    static const int rows_b = getenv("GNCX_ATTN_ROWS_B") ? atoi(getenv("GNCX_ATTN_ROWS_B")) : 8;
    static const int rows_ctas = getenv("GNCX_ATTN_ROWS_CTAS") ? atoi(getenv("GNCX_ATTN_ROWS_CTAS")) : 2;
    static const bool no_rows_merge = getenv("GNCX_ATTN_NO_ROWS_MERGE") != nullptr;
    bool rows = false, rows_merge = false;
    AttnArgs ra = a;
    dim3 rgrid;
    int rppc = 0;
    if (!no_rows && n_tok == 1 && !a.post_k && !a.pos_dev && rows_ok(a)) {
        const int t0r = a.window > 0 ? (a.pos0 - a.window + 1 > 0 ? a.pos0 - a.window + 1 : 0) : 0;
        const int lenr = a.pos0 + 1 - t0r;
        int parts = (rows_ctas > 0 ? rows_ctas : 2) * dev.sm_count / a.n_kv;
        if (parts < 1) parts = 1;
        int ppc = (lenr + parts - 1) / parts;
        const int gran = ppc >= kRowsWarps * 8 ? kRowsWarps * 8 : 8;  // whole batches for every warp
        ppc = (ppc + gran - 1) / gran * gran;
        parts = (lenr + ppc - 1) / ppc;
        if (parts <= a.max_splits) {  // one record per CTA fits the caller's record space
            rows = true;
            rgrid = dim3(parts, a.n_kv, 1);
            ra.chunk = ppc;  // the merge's "split": one CTA's range of positions
            rppc = ppc;
            // the last CTA of each KV head merges (no combine kernel) when the
            // output is fp32 only
            rows_merge = !no_rows_merge && a.out && ((uintptr_t)a.out & 7) == 0 && !act && a.n_kv <= kRowsMaxKv &&
                         parts <= kRowsMaxParts;
        }
    }
    // the register-streaming kernel reads the new rows in place (vector loads)
    // and stores them; every other path finds them in the cache
    if (a.new_k) {
        const bool in_kernel =
            rows && (((uintptr_t)a.new_k | (uintptr_t)a.new_v) & (a.hd == 128 ? 15 : 7)) == 0;
        if (!in_kernel) {
            if (store_new_rows(a, st) != cudaSuccess) return kErrCuda;
            ra.new_k = ra.new_v = nullptr;
        }
    }
    // One query over a long window (the drop-in step at thousands of
    // positions): the streaming kernel, one CTA per (range of chunks, KV head),
    // kStreamCtasPerSm resident per SM, when there are at least two chunks per CTA.
    bool stream = false;
    AttnArgs sa = a;
    dim3 sgrid;
    int cpp = 0;
    size_t ssm = 0;
    if (!rows && n_tok == 1 && !a.post_k && vec && a.hd % 8 == 0 && a.hd <= 128 && (kStreamThreads % a.hd) == 0 &&
        (Gq == 1 || Gq == 2 || Gq == 4) && !getenv("GNCX_ATTN_NO_STREAM")) {
        int t0s, lens;
        if (a.pos_dev) {
            lens = 0;  // the position lives on the device: the chunked kernel sizes itself at run time
        } else {
            t0s = a.window > 0 ? (a.pos0 - a.window + 1 > 0 ? a.pos0 - a.window + 1 : 0) : 0;
            lens = a.pos0 + 1 - t0s;
        }
        const int n_chunks = (lens + kStreamChunk - 1) / kStreamChunk;
        int parts = kStreamCtasPerSm * dev.sm_count / a.n_kv;
        if (parts < 1) parts = 1;
        ssm = attn_stream_smem_bytes(Gq, a.hd);
        if (lens > 0 && n_chunks >= 2 * parts && ssm <= (size_t)dev.max_smem_optin) {
            cpp = (n_chunks + parts - 1) / parts;
            parts = (n_chunks + cpp - 1) / cpp;
            if ((int64_t)parts <= a.max_splits) {  // one record per CTA fits the caller's record space
                stream = true;
                sgrid = dim3(parts, a.n_kv, 1);
                sa.chunk = cpp * kStreamChunk;  // the merge's "split": one CTA's range of positions
                sa.max_splits = a.max_splits;
                if (set_smem_limit(attn_stream_kernel, ssm) != cudaSuccess) return kErrCuda;
            }
        }
    }
    if (n_tok > 1 && vec && a.window == 0 && a.chunk == kPfChunk && (a.hd == 128 || a.hd == 64) &&
        kPfRows % Gq == 0 && Gq <= kPfRows && attn_prefill_smem_bytes(a.hd) <= (size_t)dev.max_smem_optin) {
        // query-tiled causal prefill; score_cap carries the query count
        AttnArgs b = a;
        b.score_cap = n_tok;
        const int qt = kPfRows / Gq;
        const dim3 pgrid(a.max_splits, a.n_kv, (n_tok + qt - 1) / qt);
        const size_t psm = attn_prefill_smem_bytes(a.hd);
        if (a.hd == 128) {
            if (set_smem_limit(attn_prefill_kernel<128>, psm) != cudaSuccess) return kErrCuda;
            e = launch_k(attn_prefill_kernel<128>, pgrid, dim3(kAttnThreads), psm, st, b);
        } else {
            if (set_smem_limit(attn_prefill_kernel<64>, psm) != cudaSuccess) return kErrCuda;
            e = launch_k(attn_prefill_kernel<64>, pgrid, dim3(kAttnThreads), psm, st, b);
        }
    } else if (rows) {
        if (rows_merge) return launch_rows<true>(ra, rgrid, rppc, rows_b, st) == cudaSuccess ? kOk : kErrCuda;
        e = launch_rows<false>(ra, rgrid, rppc, rows_b, st);
    } else if (stream) {
        e = launch_k(attn_stream_kernel, sgrid, dim3(kStreamThreads), ssm, st, sa, cpp);
    } else {
        // decode with the fused post step, fp32 output (the engine's split-KV
        // decode): the register-streaming kernel with the post step and the
        // in-kernel merge, one CTA per (split of a.chunk positions, KV head)
        // over the splits the records cover (the position is read on the
        // device; CTAs past the window exit).  The ranges depend only on the
        // caller's split size, so a tensor-parallel rank forms every head
        // exactly as one GPU does.
        static const bool no_rows_post = getenv("GNCX_ENGINE_ATTN_PARTIAL") != nullptr;  // A/B override
        if (!no_rows_post && n_tok == 1 && a.post_k && a.window == 0 && a.out && !act && rows_ok(a) &&
            ((uintptr_t)a.out & 7) == 0 && ((uintptr_t)a.post_k & 15) == 0 && a.n_kv <= kRowsMaxKv &&
            a.max_splits <= kRowsMaxParts && a.chunk % 8 == 0) {
            return launch_rows<true, true>(a, dim3(a.max_splits, a.n_kv, 1), a.chunk, 8, st) == cudaSuccess
                       ? kOk
                       : kErrCuda;
        }
        e = vec ? launch_partial<true, false>(a, grid, smem, st) : launch_partial<false, false>(a, grid, smem, st);
    }
    if (e != cudaSuccess) return kErrCuda;
    const AttnArgs& ca = rows ? ra : stream ? sa : a;
    const size_t csm = (size_t)ca.max_splits * 8 + kCombineThreads * 4;
    if (set_smem_limit(attn_combine_kernel, csm) != cudaSuccess) return kErrCuda;
    return launch_k(attn_combine_kernel, dim3(a.n_heads, n_tok), dim3(kCombineThreads), csm, st, ca) == cudaSuccess
               ? kOk
               : kErrCuda;
}

int32_t attention_scratch_records(int32_t pos, int32_t n_heads, int32_t window) {
    const int32_t t0 = window > 0 ? (pos - window + 1 > 0 ? pos - window + 1 : 0) : 0;
    const int32_t len = pos + 1 - t0;
    return n_heads * ((len + 15) / 16);  // the smallest chunk is 16 positions
}

int attention_launch(const float* q, float* kc, float* vc, int32_t pos, int32_t n_heads, int32_t n_kv,
                     int32_t head_dim, float scale, int32_t window, float* out, const AttnScratch& scratch,
                     int32_t* err, cudaStream_t st, float* exact_scores, const float* new_k,
                     const float* new_v) {
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
    a.act_out = ActOut{nullptr, nullptr};
    a.err = err;
    a.exact = exact_scores != nullptr;
    a.scores = exact_scores;
    a.score_cap = a.max_splits * a.chunk;
    a.prefetch_old = 0;  // a caller's kernel just before may have written any row
    a.new_k = new_k;
    a.new_v = new_v;
    return attention_run(a, 1, st);
}

}  // namespace gncx
