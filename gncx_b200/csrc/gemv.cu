// gemv.cu -- quantized GEMV (decode matvec) for Q4_0 / Q8_0 / Q4_K / Q6_K / BF16.
//
// Replaces gncx_xfold_universal_matvec (csrc/gncx_llm_kernels.cpp:1327-1471).
//
// Data flow (persistent CTAs, one or two per SM):
//   * the weight matrix stays in its native GGUF block layout in HBM;
//   * tiles of consecutive whole rows go to the CTAs round robin, so the
//     CTAs stream neighbouring tiles at the same time (DRAM page locality:
//     one contiguous row range per CTA measured 3 % slower on the LM head);
//   * a producer warp streams a CTA's tiles into a ring of shared-memory
//     stages, one cp.async.bulk (TMA) per tile completing on an mbarrier.
//     Each tile is copied as its 16-byte-aligned superset, so any base/row
//     alignment works (an aligned 16-byte chunk never crosses a page);
//   * the compute warps re-quantize x to int8 per 32 inputs once per CTA, or
//     bulk-copy a vector the producing kernel already quantized in the same
//     shared-memory layout ("staged" act); each lane then computes one or two
//     256-input units of one row with dp4a integer dots and the reference's
//     exactly-rounded fp32 scale arithmetic;
//   * the lanes of a row park their unit terms in shared memory and the row's
//     first lane adds them to the row accumulator in unit order, which
//     reproduces the reference's serial per-row accumulation bit for bit.
// HBM traffic is the weight bytes once plus the (L2-resident) activation.
#include <cuda_runtime.h>
#include <stdlib.h>
#include "act.cuh"
#include "common.cuh"
#include "kernels.h"
#include "trace.cuh"
#include "launch.cuh"
#include "tma.cuh"
#include "units.cuh"

namespace gncx {

constexpr int kMaxUnitsPerLane = 2;
constexpr size_t kGemvSmemCap = 200 * 1024;

struct GemvArgs {
    const uint8_t* w;
    size_t rb;              // bytes per row
    const float* x;         // fp32 activations (PREQ == false)
    const uint8_t* act;     // staged activations (PREQ == true): staged_act_bytes(in_dim)
    float* y;
    int in_dim, out_dim;
    int upr;                // units (256 inputs) per row
    int lpr;                // lanes per row (power of two, <= 32); lane j owns units j, j + lpr
    int rows;               // rows per tile = compute threads / lpr
    int stage_bytes;        // shared bytes per stage (rows * rb + 32)
    int stages;
    float softcap;
    int32_t* err;
};

struct GemvSmem {
    uint64_t* full;
    uint64_t* empty;
    uint64_t* act_bar;
    int8_t* qs;
    float4* rec;
    float* red;      // [CW][64 * E] unit terms awaiting the serial row sum
    uint8_t* stage0;
};

__host__ __device__ inline size_t gemv_act_bytes(int in_dim) {
    const int nb = in_dim / 32;
    return (size_t)in_dim + (size_t)nb * 16;
}

__host__ __device__ inline size_t gemv_red_bytes(int cw, int e) { return (size_t)cw * 64 * e * 4; }

__host__ __device__ inline size_t gemv_smem_bytes(int in_dim, int stage_bytes, int stages, size_t red_bytes) {
    size_t off = 128;  // barriers
    off += (gemv_act_bytes(in_dim) + 127) & ~(size_t)127;
    off += red_bytes;
    off += (size_t)stages * stage_bytes;
    return off;
}

__device__ inline GemvSmem carve(uint8_t* base, int in_dim, int stages, size_t red_bytes) {
    GemvSmem s;
    s.full = reinterpret_cast<uint64_t*>(base);
    s.empty = s.full + stages;
    s.act_bar = s.empty + stages;
    uint8_t* p = base + 128;
    s.qs = reinterpret_cast<int8_t*>(p);
    s.rec = reinterpret_cast<float4*>(p + in_dim);
    p += (gemv_act_bytes(in_dim) + 127) & ~(size_t)127;
    s.red = reinterpret_cast<float*>(p);
    s.stage0 = p + red_bytes;
    return s;
}


// One pipeline stage = one tile of `rows` consecutive whole rows, which are
// contiguous in memory and arrive with a single bulk copy (its 16-byte-aligned
// superset; an aligned 16-byte chunk never crosses a page).  CW compute warps
// + 1 producer warp.  With programmatic dependent launch the producer streams
// weights before the preceding kernel on the stream has finished; everything
// that touches x or y waits for it (griddepcontrol.wait).
template <int T, bool ALIGNED, bool PREQ, int CW>
__global__ void __launch_bounds__((CW + 1) * 32, 1) gemv_kernel(const GemvArgs args) {
    constexpr int UB = Fmt<T>::UB, NW = Fmt<T>::NW, E = Fmt<T>::E;
    constexpr int CT = CW * 32;
    extern __shared__ __align__(128) uint8_t smem[];
    GNCX_TRACE_SCOPE(kTagGemv, args.out_dim);
    const GemvSmem sm = carve(smem, args.in_dim, args.stages, gemv_red_bytes(CW, E));
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int S = args.stages;
    const int R = args.rows;
    const int n_tiles = (args.out_dim + R - 1) / R;  // tiles blockIdx.x, + gridDim.x, ...
    __shared__ int abort_flag;

    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], CW);
        }
        mbar_init(sm.act_bar, 1);
        abort_flag = 0;
        GNCX_TRACE_MARK(5, 0);
        fence_barrier_init();
        GNCX_TRACE_MARK(6, 0);
    }
    __syncthreads();
    if (tid == CW * 32) GNCX_TRACE_MARK(7, 0);
    pdl_launch_dependents();
    if (tid == CW * 32) GNCX_TRACE_MARK(8, 0);

    if (warp == CW) {
        // ---------------- producer warp: one bulk copy per tile ----------------
        int item = 0;
        if (lane == 0) {
            for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++item) {
                const int s = item % S;
                const int use = item / S;
                if (use > 0 && !mbar_wait(&sm.empty[s], (use - 1) & 1)) {
                    record_error(args.err, kErrTimeout);
                    atomicExch(&abort_flag, 1);
                    break;
                }
                const int row0 = tile * R;
                const int nr = min(R, args.out_dim - row0);
                const uint8_t* seg = args.w + (size_t)row0 * args.rb;
                const uintptr_t a = (uintptr_t)seg & ~(uintptr_t)15;
                const uintptr_t e = ((uintptr_t)seg + (uintptr_t)nr * args.rb + 15) & ~(uintptr_t)15;
                mbar_arrive_expect_tx(&sm.full[s], (uint32_t)(e - a));
                bulk_g2s(sm.stage0 + (size_t)s * args.stage_bytes, reinterpret_cast<const void*>(a), (uint32_t)(e - a),
                         &sm.full[s]);
                GNCX_TRACE_MARK(4, tile);
            }
            // Wait (bounded) for every copy issued before the CTA may exit.
            const int issued = item;
            for (int k = max(0, issued - S); k < issued; ++k)
                if (!mbar_wait(&sm.full[k % S], (k / S) & 1)) record_error(args.err, kErrTimeout);
        }
        return;
    }

    // ---------------- compute warps ----------------
    pdl_wait();  // x / act and y belong to the preceding kernel's world from here on
    if (tid == 0) GNCX_TRACE_MARK(1, 0);
    if (PREQ) {
        // the staged vector is already in the shared-memory layout: one bulk copy
        if (tid == 0) {
            const uint32_t bytes = (uint32_t)gemv_act_bytes(args.in_dim);
            mbar_arrive_expect_tx(sm.act_bar, bytes);
            bulk_g2s(sm.qs, args.act, bytes, sm.act_bar);
        }
        if (!mbar_wait(sm.act_bar, 0)) {
            record_error(args.err, kErrTimeout);
            atomicExch(&abort_flag, 1);
        }
    } else {
        stage_act_fp32(args.x, args.in_dim, sm.qs, sm.rec, tid, CT);
    }
    asm volatile("bar.sync 1, %0;" ::"r"(CT) : "memory");
    if (tid == 0) GNCX_TRACE_MARK(2, 0);
    const ActView av{sm.qs, sm.rec};

    const int lpr = args.lpr;
    const int rloc = tid / lpr;          // row within tile
    const int j = tid - rloc * lpr;      // lane within the row group
    const int upr = args.upr;
    const int n_terms = upr * E;                           // terms per row
    float* const red_w = sm.red + (size_t)warp * 64 * E;   // this warp's rows
    const int rbase = (lane / lpr) * n_terms;
    const float inv_cap = args.softcap > 0.0f ? fdiv(1.0f, args.softcap) : 0.0f;

    int item = 0;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++item) {
        const int s = item % S;
        const int use = item / S;
        if (!mbar_wait(&sm.full[s], use & 1)) {
            record_error(args.err, kErrTimeout);
            atomicExch(&abort_flag, 1);
        }
        if (*(volatile int*)&abort_flag) return;
        if (tid == 0) GNCX_TRACE_MARK(3, tile);
        const int row0 = tile * R;
        const int nr = min(R, args.out_dim - row0);
        const bool row_ok = rloc < nr;
        const uint8_t* tile_src = args.w + (size_t)row0 * args.rb;
        const uint8_t* row_smem = sm.stage0 + (size_t)s * args.stage_bytes + ((uintptr_t)tile_src & 15) +
                                  (size_t)rloc * args.rb;
        float t[kMaxUnitsPerLane][E];
#pragma unroll
        for (int k = 0; k < kMaxUnitsPerLane; ++k) {
#pragma unroll
            for (int e = 0; e < E; ++e) t[k][e] = 0.0f;
            const int u = j + k * lpr;
            if (row_ok && u < upr) {
                uint32_t wv[NW];
                load_unit_smem<NW, ALIGNED>(row_smem + (size_t)u * UB, wv);
                unit_terms<T>(wv, UnitAct{av, u}, t[k]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty[s]);
        // Park the terms (row-major, unit order), then the row's first lane adds
        // them serially: unit u = k*lpr + j, terms e = 0..E-1 within a unit.
#pragma unroll
        for (int k = 0; k < kMaxUnitsPerLane; ++k) {
            const int u = j + k * lpr;
            if (u < upr) {
                float* dst = red_w + rbase + u * E;
                if constexpr (E % 4 == 0) {
#pragma unroll
                    for (int e = 0; e < E; e += 4)
                        *reinterpret_cast<float4*>(dst + e) = make_float4(t[k][e], t[k][e + 1], t[k][e + 2], t[k][e + 3]);
                } else {
#pragma unroll
                    for (int e = 0; e < E; ++e) dst[e] = t[k][e];
                }
            }
        }
        __syncwarp();
        if (row_ok && j == 0) {
            float acc = 0.0f;
            const float* rp = red_w + rbase;
            if ((n_terms & 3) == 0) {
#pragma unroll 4
                for (int i = 0; i < n_terms; i += 4) {
                    const float4 v4 = *reinterpret_cast<const float4*>(rp + i);
                    acc = fadd(fadd(fadd(fadd(acc, v4.x), v4.y), v4.z), v4.w);
                }
            } else {
                for (int i = 0; i < n_terms; ++i) acc = fadd(acc, rp[i]);
            }
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

static bool g_pdl = false;
void gemv_set_pdl(bool on) { g_pdl = on; }
bool pdl_enabled() { return g_pdl; }

// Tuning overrides (GNCX_GEMV_WARPS = 4|8, GNCX_GEMV_STAGES = 2..4); read once.
static int env_int(const char* name, int dflt) {
    const char* v = getenv(name);
    return v ? atoi(v) : dflt;
}

template <int T, bool ALIGNED, bool PREQ, int CW>
static int launch_t(const GemvArgs& a, size_t smem, int, cudaStream_t st) {
    auto k = gemv_kernel<T, ALIGNED, PREQ, CW>;
    static size_t occ_smem = 0;  // occupancy per instantiation (devices of one model alike)
    static int occ_blocks = 1;
    if (set_smem_limit(k, smem) != cudaSuccess) return kErrCuda;
    if (smem != occ_smem) {  // resident CTAs per SM for this shared-memory size (registers included)
        int nb = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, k, (CW + 1) * 32, smem) != cudaSuccess) nb = 1;
        occ_blocks = nb < 1 ? 1 : nb;
        occ_smem = smem;
    }
    const int max_grid = device_info().sm_count * occ_blocks;
    const int n_tiles = (a.out_dim + a.rows - 1) / a.rows;
    const int grid = n_tiles < max_grid ? n_tiles : max_grid;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3((CW + 1) * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = g_pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k, a) == cudaSuccess ? kOk : kErrCuda;
}

template <int T, int CW>
static int launch_fmt(const GemvArgs& a, bool aligned, bool preq, size_t smem, int grid, cudaStream_t st) {
    if (aligned) {
        if constexpr (T != kQ6_K) {
            return preq ? launch_t<T, true, true, CW>(a, smem, grid, st) : launch_t<T, true, false, CW>(a, smem, grid, st);
        }
    }
    return preq ? launch_t<T, false, true, CW>(a, smem, grid, st) : launch_t<T, false, false, CW>(a, smem, grid, st);
}

template <int T>
static int launch_cw(const GemvArgs& a, int cw, bool aligned, bool preq, size_t smem, int grid, cudaStream_t st) {
    return cw == 8 ? launch_fmt<T, 8>(a, aligned, preq, smem, grid, st)
                   : launch_fmt<T, 4>(a, aligned, preq, smem, grid, st);
}

int gemv_launch(const uint8_t* w, int32_t type, const float* x, const uint8_t* act, int32_t in_dim,
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
    if (act && ((uintptr_t)act & 15)) return kErrInvalidArg;  // bulk-copied
    int ub = 0, terms = 1;
    switch (type) {
        case kQ4_0: ub = Fmt<kQ4_0>::UB; terms = Fmt<kQ4_0>::E; break;
        case kQ8_0: ub = Fmt<kQ8_0>::UB; terms = Fmt<kQ8_0>::E; break;
        case kQ4_K: ub = Fmt<kQ4_K>::UB; terms = Fmt<kQ4_K>::E; break;
        default: ub = Fmt<kQ6_K>::UB; terms = Fmt<kQ6_K>::E; break;
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
    // lanes per row: smallest power of two with <= 2 units per lane
    int lpr = 1;
    while (lpr < 32 && lpr * kMaxUnitsPerLane < a.upr) lpr <<= 1;
    if (lpr * kMaxUnitsPerLane < a.upr) return kErrCapacity;  // in_dim > 16384
    a.lpr = lpr;
    a.softcap = softcap;
    a.err = err;
    // Leave room beside each CTA for the small kernels that run between GEMVs,
    // so the next GEMV's CTAs become resident (and prefetch) while they run.
    const size_t budget = (size_t)dev.max_smem_optin < kGemvSmemCap ? (size_t)dev.max_smem_optin : kGemvSmemCap;
    static const int force_cw = env_int("GNCX_GEMV_WARPS", 0);
    static const int max_stages = env_int("GNCX_GEMV_STAGES", 2);
    // Two stages: the CTA stays small enough that the next kernel's CTAs (the
    // next GEMV's producer, the small kernels between GEMVs) become resident
    // and start while it runs -- measured faster than deeper rings in decode
    // (2.20 vs 2.34 ms/token, 8B shape) and in the GEMV sweep.  8 compute
    // warps, except for very tall matrices (at least 16 tiles of 8 warps per
    // SM, e.g. the LM head): there 4 warps and half-size tiles let two CTAs
    // share an SM (151936x4096 Q4_K: 6090 vs 5910 GB/s).
    int cw = 8;
    if (force_cw == 4 || force_cw == 8) cw = force_cw;
    else if ((out_dim + 256 / lpr - 1) / (256 / lpr) >= 16 * dev.sm_count) cw = 4;
    int stages = 0;
    for (;; cw >>= 1) {
        a.rows = cw * 32 / lpr;
        a.stage_bytes = (int)((((size_t)a.rows * a.rb + 15) & ~(size_t)15) + 32);
        stages = max_stages < 2 ? 2 : (max_stages > 4 ? 4 : max_stages);
        while (stages > 2 && gemv_smem_bytes(in_dim, a.stage_bytes, stages, gemv_red_bytes(cw, terms)) > budget)
            --stages;
        if (gemv_smem_bytes(in_dim, a.stage_bytes, stages, gemv_red_bytes(cw, terms)) <= budget || cw == 4) break;
    }
    const size_t smem = gemv_smem_bytes(in_dim, a.stage_bytes, stages, gemv_red_bytes(cw, terms));
    if (smem > budget) return kErrCapacity;
    a.stages = stages;
    const int grid = 0;  // chosen from the occupancy of the instantiation
    const bool aligned = ((uintptr_t)w % 16 == 0) && (a.rb % 16 == 0) && (ub % 16 == 0);
    const bool preq = act != nullptr;
    switch (type) {
        case kQ4_0: return launch_cw<kQ4_0>(a, cw, aligned, preq, smem, grid, st);
        case kQ8_0: return launch_cw<kQ8_0>(a, cw, aligned, preq, smem, grid, st);
        case kQ4_K: return launch_cw<kQ4_K>(a, cw, aligned, preq, smem, grid, st);
        default: return launch_cw<kQ6_K>(a, cw, aligned, preq, smem, grid, st);
    }
}

}  // namespace gncx
