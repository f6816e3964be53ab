// gemv.cu -- quantized GEMV (decode matvec) for Q4_0 / Q8_0 / Q4_K / Q6_K / BF16.
//
// Replaces gncx_xfold_universal_matvec (csrc/gncx_llm_kernels.cpp:1327-1471).
//
// Data flow (one persistent CTA per SM):
//   * the weight matrix stays in its native GGUF block layout in HBM;
//   * a producer warp streams (32-row x 8-unit) chunks into a ring of shared
//     memory stages with cp.async.bulk (TMA) completing on mbarriers.  Each row
//     segment is copied as its 16-byte-aligned superset, so any base/row
//     alignment works (an aligned 16-byte chunk never crosses a page);
//   * eight compute warps re-quantize x to int8 per 32 inputs once per CTA
//     (or load blocks another kernel quantized), then each lane computes one
//     256-input unit of one row with dp4a integer dots and the reference's
//     exactly-rounded fp32 scale arithmetic;
//   * the eight lanes of a row add their unit terms to the row accumulator in
//     unit order with a shuffle chain, which reproduces the reference's serial
//     per-row accumulation bit for bit.
// HBM traffic is the weight bytes once plus the (L2-resident) activation.
#include <cuda_runtime.h>
#include "act.cuh"
#include "common.cuh"
#include "kernels.h"
#include "tma.cuh"
#include "units.cuh"

namespace gncx {

constexpr int kRows = 32;           // rows per tile (4 per compute warp)
constexpr int kUnitsPerChunk = 8;   // units per row per stage (one per lane)
constexpr int kComputeWarps = 8;
constexpr int kGemvThreads = (kComputeWarps + 1) * 32;

struct GemvArgs {
    const uint8_t* w;
    size_t rb;              // bytes per row
    const float* x;         // fp32 activations (PREQ == false)
    const ActBlock* act;    // pre-quantized activations (PREQ == true)
    float* y;
    int in_dim, out_dim;
    int upr;                // units per row (in_dim / 256)
    int upc;                // units per chunk (min(8, upr))
    int n_chunks;           // ceil(upr / upc)
    int n_tiles;            // ceil(out_dim / 32)
    int slot;               // shared bytes per row slot
    int stages;
    float softcap;
    int32_t* err;
};

struct GemvSmem {
    uint64_t* full;
    uint64_t* empty;
    int8_t* qs;
    float* d;
    int2* s;
    uint8_t* stage0;
};

__host__ __device__ inline size_t gemv_act_bytes(int in_dim) {
    const int nb = in_dim / 32;
    return (size_t)in_dim + (size_t)nb * 4 + (size_t)nb * 8;
}

__host__ __device__ inline size_t gemv_smem_bytes(int in_dim, int slot, int stages) {
    size_t off = 128;  // barriers
    off += (gemv_act_bytes(in_dim) + 127) & ~(size_t)127;
    off += (size_t)stages * kRows * slot;
    return off;
}

__device__ inline GemvSmem carve(uint8_t* base, int in_dim, int stages) {
    GemvSmem s;
    s.full = reinterpret_cast<uint64_t*>(base);
    s.empty = s.full + stages;
    uint8_t* p = base + 128;
    const int nb = in_dim / 32;
    s.qs = reinterpret_cast<int8_t*>(p);
    s.d = reinterpret_cast<float*>(p + in_dim);
    s.s = reinterpret_cast<int2*>(p + in_dim + nb * 4);
    s.stage0 = base + 128 + ((gemv_act_bytes(in_dim) + 127) & ~(size_t)127);
    return s;
}

template <int T, bool ALIGNED, bool PREQ>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(const GemvArgs args) {
    constexpr int UB = Fmt<T>::UB, NW = Fmt<T>::NW, E = Fmt<T>::E;
    extern __shared__ __align__(128) uint8_t smem[];
    const GemvSmem sm = carve(smem, args.in_dim, args.stages);
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int S = args.stages;
    __shared__ int abort_flag;

    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], kComputeWarps);
        }
        abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == kComputeWarps) {
        // ---------------- producer warp ----------------
        int item = 0;
        for (int tile = blockIdx.x; tile < args.n_tiles; tile += gridDim.x) {
            const int row0 = tile * kRows;
            const int nr = min(kRows, args.out_dim - row0);
            for (int c = 0; c < args.n_chunks; ++c, ++item) {
                const int s = item % S;
                const int use = item / S;
                if (use > 0) {
                    bool ok = true;
                    if (lane == 0) ok = mbar_wait(&sm.empty[s], (use - 1) & 1);
                    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
                    if (!ok) {
                        if (lane == 0) { record_error(args.err, kErrTimeout); atomicExch(&abort_flag, 1); }
                        goto producer_done;
                    }
                }
                const int u0 = c * args.upc;
                const int nu = min(args.upc, args.upr - u0);
                uint32_t bytes = 0;
                const uint8_t* src = nullptr;
                if (lane < nr) {
                    const uint8_t* seg = args.w + (size_t)(row0 + lane) * args.rb + (size_t)u0 * UB;
                    const uintptr_t a = (uintptr_t)seg & ~(uintptr_t)15;
                    const uintptr_t e = ((uintptr_t)seg + (uintptr_t)nu * UB + 15) & ~(uintptr_t)15;
                    src = reinterpret_cast<const uint8_t*>(a);
                    bytes = (uint32_t)(e - a);
                }
                uint32_t total = bytes;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
                if (lane == 0) mbar_arrive_expect_tx(&sm.full[s], total);
                __syncwarp();
                if (lane < nr) bulk_g2s(sm.stage0 + ((size_t)s * kRows + lane) * args.slot, src, bytes, &sm.full[s]);
            }
        }
    producer_done:
        // Wait (bounded) for every copy this warp issued before the CTA may exit.
        if (lane == 0) {
            const int issued = item;
            for (int k = max(0, issued - S); k < issued; ++k) {
                if (!mbar_wait(&sm.full[k % S], (k / S) & 1)) record_error(args.err, kErrTimeout);
            }
        }
        return;
    }

    // ---------------- compute warps ----------------
    if (PREQ) stage_act_blocks(args.act, args.in_dim, sm.qs, sm.d, sm.s, tid, kComputeWarps * 32);
    else stage_act_fp32(args.x, args.in_dim, sm.qs, sm.d, sm.s, tid, kComputeWarps * 32);
    asm volatile("bar.sync 1, %0;" ::"r"(kComputeWarps * 32) : "memory");
    const ActView av{sm.qs, sm.d, sm.s};

    const int rloc = tid >> 3;       // row within tile, 0..31
    const int unit = tid & 7;        // unit within chunk
    const int gbase = lane & ~7;     // first lane of this row's group
    const float inv_cap = args.softcap > 0.0f ? fdiv(1.0f, args.softcap) : 0.0f;

    int item = 0;
    for (int tile = blockIdx.x; tile < args.n_tiles; tile += gridDim.x) {
        const int row0 = tile * kRows;
        const int nr = min(kRows, args.out_dim - row0);
        const bool row_ok = rloc < nr;
        float acc = 0.0f;
        for (int c = 0; c < args.n_chunks; ++c, ++item) {
            const int s = item % S;
            const int use = item / S;
            if (!mbar_wait(&sm.full[s], use & 1)) {
                record_error(args.err, kErrTimeout);
                atomicExch(&abort_flag, 1);
            }
            if (*(volatile int*)&abort_flag) return;
            const int u0 = c * args.upc;
            const int nu = min(args.upc, args.upr - u0);
            float t[E];
#pragma unroll
            for (int e = 0; e < E; ++e) t[e] = 0.0f;
            if (row_ok && unit < nu) {
                const uint8_t* seg = args.w + (size_t)(row0 + rloc) * args.rb + (size_t)u0 * UB;
                const uint8_t* p = sm.stage0 + ((size_t)s * kRows + rloc) * args.slot + ((uintptr_t)seg & 15) +
                                   (size_t)unit * UB;
                uint32_t wv[NW];
                load_unit_smem<NW, ALIGNED>(p, wv);
                unit_terms<T>(wv, UnitAct{av, u0 + unit}, t);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.empty[s]);
            // Serial chain over this chunk's units, in unit order.
            for (int u = 0; u < nu; ++u) {
                if (unit == u) {
#pragma unroll
                    for (int e = 0; e < E; ++e) acc = fadd(acc, t[e]);
                }
                acc = __shfl_sync(0xffffffffu, acc, gbase | u);
            }
        }
        if (row_ok && unit == 0) {
            float v = acc;
            if (args.softcap > 0.0f) v = fmul(tanh_cr(fmul(v, inv_cap)), args.softcap);
            args.y[row0 + rloc] = v;
        }
    }
}

// ---------------- BF16 (only used by Gemma-4 per-layer inputs) ----------------
// Four chains per row over inputs 4k+j, folded ((l0+l1)+l2)+l3, tail last (:1432-1461).
__global__ void gemv_bf16_kernel(const uint8_t* __restrict__ w, size_t rb, const float* __restrict__ x, int in_dim,
                                 int out_dim, float* __restrict__ y, float softcap) {
    const int gid = blockIdx.x * blockDim.x + threadIdx.x;
    const int row = gid >> 2, j = gid & 3;
    const bool ok = row < out_dim;
    const uint16_t* r = reinterpret_cast<const uint16_t*>(w + (size_t)(ok ? row : 0) * rb);
    float acc = 0.0f;
    const int n4 = in_dim & ~3;
    if (ok)
        for (int k = j; k < n4; k += 4) acc = fadd(acc, fmul(bf16_bits_to_float(__ldg(r + k)), __ldg(x + k)));
    const float l1 = __shfl_down_sync(0xffffffffu, acc, 1);
    const float l2 = __shfl_down_sync(0xffffffffu, acc, 2);
    const float l3 = __shfl_down_sync(0xffffffffu, acc, 3);
    if (ok && j == 0) {
        float v = fadd(fadd(fadd(acc, l1), l2), l3);
        for (int k = n4; k < in_dim; ++k) v = fadd(v, fmul(bf16_bits_to_float(__ldg(r + k)), __ldg(x + k)));
        if (softcap > 0.0f) v = fmul(tanh_cr(fmul(v, fdiv(1.0f, softcap))), softcap);
        y[row] = v;
    }
}

// ---------------- host launch ----------------

template <int T, bool ALIGNED, bool PREQ>
static int launch_t(const GemvArgs& a, size_t smem, int grid, cudaStream_t st) {
    auto k = gemv_kernel<T, ALIGNED, PREQ>;
    static int configured_bytes = 0;  // per instantiation, per process (single device at a time)
    if ((int)smem > configured_bytes) {
        if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return kErrCuda;
        configured_bytes = (int)smem;
    }
    k<<<grid, kGemvThreads, smem, st>>>(a);
    return cudaPeekAtLastError() == cudaSuccess ? kOk : kErrCuda;
}

template <int T>
static int launch_fmt(const GemvArgs& a, bool aligned, bool preq, size_t smem, int grid, cudaStream_t st) {
    if (aligned) {
        if constexpr (T != kQ6_K) {
            return preq ? launch_t<T, true, true>(a, smem, grid, st) : launch_t<T, true, false>(a, smem, grid, st);
        }
    }
    return preq ? launch_t<T, false, true>(a, smem, grid, st) : launch_t<T, false, false>(a, smem, grid, st);
}

int gemv_launch(const uint8_t* w, int32_t type, const float* x, const ActBlock* act, int32_t in_dim,
                int32_t out_dim, float* y, float softcap, int32_t* err, cudaStream_t st) {
    if (!w || !y || (!x && !act) || in_dim <= 0 || out_dim < 0) return kErrInvalidArg;
    if (out_dim == 0) return kOk;
    const DeviceInfo& dev = device_info();
    if (type == kBF16) {
        if (!x) return kErrInvalidArg;
        const int threads = 256;
        const int blocks = (int)(((int64_t)out_dim * 4 + threads - 1) / threads);
        gemv_bf16_kernel<<<blocks, threads, 0, st>>>(w, (size_t)in_dim * 2, x, in_dim, out_dim, y, softcap);
        return cudaPeekAtLastError() == cudaSuccess ? kOk : kErrCuda;
    }
    if (type != kQ4_0 && type != kQ8_0 && type != kQ4_K && type != kQ6_K) return kErrInvalidArg;
    if (in_dim % 256 != 0) return kErrInvalidArg;
    int ub = 0;
    switch (type) {
        case kQ4_0: ub = Fmt<kQ4_0>::UB; break;
        case kQ8_0: ub = Fmt<kQ8_0>::UB; break;
        case kQ4_K: ub = Fmt<kQ4_K>::UB; break;
        default: ub = Fmt<kQ6_K>::UB; break;
    }
    GemvArgs a{};
    a.w = w;
    a.rb = row_bytes(type, in_dim);
    a.x = x;
    a.act = act;
    a.y = y;
    a.in_dim = in_dim;
    a.out_dim = out_dim;
    a.upr = in_dim / 256;
    a.upc = a.upr < kUnitsPerChunk ? a.upr : kUnitsPerChunk;
    a.n_chunks = (a.upr + a.upc - 1) / a.upc;
    a.n_tiles = (out_dim + kRows - 1) / kRows;
    a.slot = ((a.upc * ub + 15) & ~15) + 32;
    a.softcap = softcap;
    a.err = err;
    const size_t budget = (size_t)dev.max_smem_optin;
    int stages = 4;
    while (stages > 2 && gemv_smem_bytes(in_dim, a.slot, stages) > budget) --stages;
    if (gemv_smem_bytes(in_dim, a.slot, stages) > budget) return kErrCapacity;
    a.stages = stages;
    const size_t smem = gemv_smem_bytes(in_dim, a.slot, stages);
    const int grid = a.n_tiles < dev.sm_count ? a.n_tiles : dev.sm_count;
    const bool aligned = ((uintptr_t)w % 16 == 0) && (a.rb % 16 == 0) && (ub % 16 == 0);
    const bool preq = act != nullptr;
    switch (type) {
        case kQ4_0: return launch_fmt<kQ4_0>(a, aligned, preq, smem, grid, st);
        case kQ8_0: return launch_fmt<kQ8_0>(a, aligned, preq, smem, grid, st);
        case kQ4_K: return launch_fmt<kQ4_K>(a, aligned, preq, smem, grid, st);
        default: return launch_fmt<kQ6_K>(a, aligned, preq, smem, grid, st);
    }
}

}  // namespace gncx
