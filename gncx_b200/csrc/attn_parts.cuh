// attn_parts.cuh -- device building blocks of split-KV decode attention shared
// by the attention kernels (attention.cu) and the persistent decode-step
// kernel (decode_step.cu): the reference's score chains, the PV accumulation
// and the per-head Q/K RMSNorm + RoPE post step.
#pragma once
#include "common.cuh"
#include "norm.cuh"

namespace gncx {

// L2 load that the compiler keeps after every preceding memory barrier (a
// dependency wait, a fence): __ldcg is a pure asm the compiler may hoist.
__device__ __forceinline__ float ld_l2(const float* p) {
    float v;
    asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
    return v;
}

// The same scores from unpadded K rows (rows `hd` floats apart, as one bulk
// copy lands them): eight lanes share one (position, head) dot, lane j
// running the reference's chain j (d = 8m + j) with the query values in its
// registers, then the fold ((c0+c4)+(c1+c5))+((c2+c6)+(c3+c7)) by shuffles.
// The four (position, head) pairs of a warp are the G heads of G == 4 / 2 / 1
// consecutive... pairs in (position, head) order, so a warp reads at most
// 4 / G different K rows per step (the same row for G == 4).  hd % 8 == 0,
// hd <= 128, G in {1, 2, 4}; the first `nw` warps of the CTA take part, each
// taking every nw-th group of four pairs.
template <class Store>
__device__ __forceinline__ void chunk_scores_warp(const float* ks, int hd, const float* qs, int qrs, int G, int cn,
                                                  int nw, Store store) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int s = lane >> 3, j = lane & 7, nm = hd >> 3;
    const int g = s % G;  // this lane's head: the same for every group a warp takes (4 % G == 0)
    float qv[16];
#pragma unroll
    for (int m = 0; m < 16; ++m) qv[m] = m < nm ? qs[(size_t)g * qrs + 8 * m + j] : 0.0f;
    for (int pair0 = 4 * warp; pair0 < G * cn; pair0 += 4 * nw) {
        const int pair = pair0 + s;
        const int p = pair / G;
        const bool ok = pair < G * cn;
        const float* kr = ks + (size_t)(ok ? p : 0) * hd + j;
        float c = 0.0f;
#pragma unroll
        for (int m = 0; m < 16; ++m)
            if (m < nm) c = fadd(c, fmul(qv[m], kr[8 * m]));
        const float c4 = __shfl_down_sync(0xffffffffu, c, 4);   // lanes j < 4: c_j + c_{j+4}
        const float t = fadd(c, c4);
        const float t1 = __shfl_down_sync(0xffffffffu, t, 1);   // lanes 0, 2: (c0+c4)+(c1+c5), (c2+c6)+(c3+c7)
        const float u = fadd(t, t1);
        const float u2 = __shfl_down_sync(0xffffffffu, u, 2);
        if (ok && j == 0) store(g, p, fadd(u, u2));
    }
}

constexpr int kPvHeads = 8;  // query heads accumulated per pass over V

// acc[i] += sum over this thread's positions p = pg, pg + npg, ... of
// e[p][g0 + i] * v[p][d]; e is position-major with row stride G4 (a multiple
// of 4), so one broadcast vector load serves four heads.
__device__ __forceinline__ void chunk_pv(const float* vs, int rs, const float* es, int G4, int g0, int ng, int cn,
                                         int d, int pg, int npg, float (&acc)[kPvHeads]) {
    for (int p = pg; p < cn; p += npg) {
        const float v = vs[(size_t)p * rs + d];
        const float4 e0 = *reinterpret_cast<const float4*>(es + (size_t)p * G4 + g0);
        acc[0] = fmaf(e0.x, v, acc[0]);
        acc[1] = fmaf(e0.y, v, acc[1]);
        acc[2] = fmaf(e0.z, v, acc[2]);
        acc[3] = fmaf(e0.w, v, acc[3]);
        if (ng > 4) {
            const float4 e1 = *reinterpret_cast<const float4*>(es + (size_t)p * G4 + g0 + 4);
            acc[4] = fmaf(e1.x, v, acc[4]);
            acc[5] = fmaf(e1.y, v, acc[5]);
            acc[6] = fmaf(e1.z, v, acc[6]);
            acc[7] = fmaf(e1.w, v, acc[7]);
        }
    }
}

// One warp: per-head RMSNorm (the reference's four serial fp32 lanes over
// x[4k+j]^2, combined in double) with gain w (may be null) and rotate-half
// RoPE at `pos`, in place on x[hd] in shared memory -- the arithmetic of the
// Q/K post step (csrc/gncx_llm_kernels.cpp:895-953, :1760-1863).
__device__ __forceinline__ void warp_head_norm_rope(float* x, int hd, const float* __restrict__ w, bool do_norm,
                                                    float eps, const float* __restrict__ ct,
                                                    const float* __restrict__ stab, int pos, int lane) {
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
        for (int i = lane; i < hd; i += 32) {
            const float v = fmul(x[i], inv);
            x[i] = w ? fmul(v, w[i]) : v;
        }
        __syncwarp();
    }
    const int half = hd >> 1;
    for (int i = lane; i < half; i += 32) {
        const float c = ct[(size_t)pos * half + i], s = stab[(size_t)pos * half + i];
        const float x1 = x[i], x2 = x[i + half];
        x[i] = fsub(fmul(x1, c), fmul(x2, s));
        x[i + half] = fadd(fmul(x2, c), fmul(x1, s));
    }
    __syncwarp();
}

}  // namespace gncx
