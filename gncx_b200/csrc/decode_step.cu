// decode_step.cu -- one decode token's transformer layers as ONE persistent
// kernel (single GPU).
//
// The multi-kernel decode (one launch per GEMV / norm / attention / GLU, ~255
// launches per token) loses most of its time at kernel boundaries: every small
// kernel drains, the next one fills its weight pipeline again, and the HBM
// stream stops while the latency-bound steps in between (the RMSNorm's serial
// fp32 chains, attention, the split merge) run.  Here one CTA per SM runs the
// whole layer stack (lua/gncx_streamer.lua:759-965, forward_token, without the
// LM head):
//
//   * a producer warp per CTA walks the CTA's share of every weight tile of
//     every layer, and of every attention chunk's K (and V) rows, in the order
//     the CTA consumes them, and streams them into a ring of shared-memory
//     stages with one bulk copy (TMA) per tile on mbarriers.  Weights do not
//     depend on the token, so the stream runs ahead across layer and phase
//     boundaries; it also asks L2 for the bytes `ahead` of its copies
//     (cp.async.bulk.prefetch.L2), so HBM stays busy while the compute warps
//     wait on a dependency;
//   * eight compute warps run the phases of each layer in the reference's
//     order -- QKV GEMV, attention (Q/K RMSNorm + RoPE + KV-cache write fused),
//     O GEMV, residual add + RMSNorm, gate/up GEMV with the GLU in its
//     epilogue, down GEMV, residual add + RMSNorm of the next layer -- and
//     meet at counters in global memory (release/acquire, bounded waits)
//     where a phase needs the whole output of the previous one;
//   * every CTA keeps its own copy of the residual stream in registers and
//     redoes the residual add, the RMSNorm and the act-Q8 quantization of the
//     next GEMV's input itself (a few microseconds of serial fp32 in every
//     CTA instead of one more grid-wide exchange), so the quantized vector
//     never leaves shared memory.
//
// Attention, two modes:
//   * split-KV: one work item per (chunk of positions, KV head) writes a
//     partial record per query head; the CTA that finishes a KV group's last
//     chunk merges the group's heads;
//   * exact (the reference's order, csrc/gncx_llm_kernels.cpp:1887-1994):
//     chunk items write the scores; the last CTA of a KV group forms each
//     head's softmax with the serial sum of exp in position order; then one
//     item per (KV head, 8 output columns) runs the serial sum over positions
//     of (e_t * inv) * v_t[d] for each of its (head, column) pairs.
//
// Arithmetic is that of the multi-kernel path, function by function: the same
// unit dot products (units.cuh) with the per-row serial sum in unit order, the
// same RMSNorm chains and act-Q8, the same attention score chains and post
// step (attn_parts.cuh); exact mode is the same computation as the exact
// attention kernels; split-KV mode differs only in its chunking (64 positions
// at head_dim 128) and the merge's summation order.
#include <cuda_runtime.h>
#include <stdlib.h>
#include "act.cuh"
#include "attn_parts.cuh"
#include "common.cuh"
#include "kernels.h"
#include "norm.cuh"
#include "tma.cuh"
#include "trace.cuh"
#include "units.cuh"

namespace gncx {

constexpr int kStepCW = 8;                  // compute warps
constexpr int kStepCT = kStepCW * 32;       // compute threads
constexpr int kStepThreads = kStepCT + 32;  // + the producer warp
constexpr int kStepHPass = 8 * kStepCT;     // residual elements per register pass (8 per thread)
constexpr int kStepMaxPasses = kStepMaxDim / kStepHPass;
static_assert(kStepMaxPasses * kStepHPass == kStepMaxDim, "residual passes");
constexpr int kStepMergeBatch = 16;         // split records in flight per thread in the merge

// Counter words of a layer: phases, then per KV head the split-KV / score
// arrivals (kSyGroup + kvh) and the exact softmax's completion (kSyReady + kvh).
enum StepSync { kSyQkv = 0, kSyAttn = 1, kSyO = 2, kSyGu = 3, kSyDown = 4, kSyGroup = 8, kSyReady = 20 };
constexpr int kStepMaxKv = kSyReady - kSyGroup;
static_assert(kSyReady + kStepMaxKv <= kStepSyncWords, "sync words");
enum StepPhase { kPhQkv = 0, kPhAttn = 1, kPhO = 2, kPhGu = 3, kPhDown = 4, kPhCount = 5 };
constexpr int kPvCols = 8;      // exact mode: output columns of one PV item
constexpr int kPvChunk = 256;   // exact mode: positions staged per PV step
constexpr int kSmBlock = 512;   // exact mode: exp values staged per serial-sum block

// ---------------------------------------------------------------- geometry
// A GEMV tile is kStepCW x (rows per warp) whole consecutive rows; within a
// warp, `lpr` lanes share a row (lane j owns units j and j + lpr, as in the
// per-kernel GEMV), so a warp finishes its rows on its own -- no barrier of
// the compute warps per tile.
__host__ __device__ inline int step_lpr(int upr) {
    int l = 1;
    while (l < 32 && 2 * l < upr) l <<= 1;
    return l;
}

// Rows each compute warp takes per tile (gate/up: gate rows plus as many up
// rows), limited by the lanes and by the tile fitting one stage; 0 when the
// row does not fit.
__host__ __device__ inline int step_warp_rows(int type, int in, int stage_bytes, bool pair) {
    const int upr = in / 256;
    const int lpr = step_lpr(upr);
    if (2 * lpr < upr) return 0;  // more than 16384 inputs
    const size_t rb = row_bytes(type, in);
    int r = 32 / lpr;
    if (pair) {
        const int fit = 2 * (int)(((size_t)stage_bytes - 96) / (2 * rb * kStepCW));
        r = (r < fit ? r : fit) & ~1;
    } else {
        const int fit = (int)(((size_t)stage_bytes - 32) / (rb * kStepCW));
        r = r < fit ? r : fit;
    }
    return r;
}

// Byte offset of the up rows inside a gate/up stage.
__host__ __device__ inline int step_pair_offset(int rows, size_t rb) {
    return (int)(((size_t)rows * rb + 32 + 15) & ~(size_t)15);
}

__host__ __device__ inline int step_attn_chunk(int hd, int stage_bytes) {
    int c = stage_bytes / (hd * 4);
    c = c > 128 ? 128 : c;
    return c & ~15;
}

__host__ __device__ inline int step_max_in(const StepPlan& p) {
    int m = p.dim > p.qd ? p.dim : p.qd;
    return m > p.ffn ? m : p.ffn;
}

struct StepSmem {
    uint64_t* full;
    uint64_t* empty;
    int8_t* qs;       // staged act-Q8 of the current GEMV input
    float4* rec;
    float* red;       // [kStepCW][64 * max_terms] unit terms awaiting the serial row sums
    float* scratch;   // norm squares / attention work area (union)
    uint8_t* ring;
};

__host__ __device__ inline size_t step_act_bytes(int max_in) {
    return ((size_t)max_in + (size_t)(max_in / 32) * 16 + 127) & ~(size_t)127;
}
// A warp's rows cover at most 32 lanes x 2 units: 64 units of terms.
__host__ __device__ inline size_t step_red_bytes(int max_terms) { return (size_t)kStepCW * 64 * max_terms * 4; }

// Floats of the split-KV work area for G query heads per KV head.
__host__ __device__ inline size_t step_attn_floats(int G, int hd, int chunk, int max_splits) {
    const int G4 = (G + 3) & ~3;
    size_t n = (size_t)G * (hd + 4)             // q heads
               + (size_t)G * (chunk + 8)        // scores
               + (size_t)chunk * G4             // exp, position-major
               + 2 * (size_t)G + 8              // per-head max / sum, merge factors
               + (size_t)kStepCT / hd * kPvHeads * hd  // PV partials of the position groups
               + 2 * (size_t)G * max_splits;    // merge weights and sums
    return (n + 3) & ~(size_t)3;
}

// Floats of the exact-mode work areas: q heads + the serial-sum staging
// ([G][kSmBlock]); the PV step's two buffers of kPvChunk positions.
__host__ __device__ inline size_t step_exact_floats(int G, int hd) {
    const size_t sm = (size_t)G * (hd + 4) + (size_t)G * kSmBlock;
    const size_t pv = 2 * ((size_t)kPvChunk * kPvCols + (size_t)G * kPvChunk);
    return sm > pv ? sm : pv;
}

__host__ __device__ inline size_t step_scratch_bytes(const StepPlan& p) {
    const int G = p.nh / p.nkv;
    size_t a = step_attn_floats(G, p.hd, p.chunk, p.max_splits) * 4;
    const size_t x = step_exact_floats(G, p.hd) * 4;
    const size_t sq = (size_t)p.dim * 4;
    a = a > x ? a : x;
    a = a > sq ? a : sq;
    return (a + 127) & ~(size_t)127;
}

__host__ __device__ inline size_t step_smem_bytes(const StepPlan& p) {
    return 256 + step_act_bytes(step_max_in(p)) + step_red_bytes(p.max_terms) + step_scratch_bytes(p) +
           (size_t)kStepStages * p.stage_bytes;
}

__device__ inline StepSmem step_carve(uint8_t* base, const StepPlan& p) {
    StepSmem s;
    s.full = reinterpret_cast<uint64_t*>(base);
    s.empty = s.full + kStepStages;
    uint8_t* q = base + 256;
    const int max_in = step_max_in(p);
    s.qs = reinterpret_cast<int8_t*>(q);
    s.rec = reinterpret_cast<float4*>(q + max_in);
    q += step_act_bytes(max_in);
    s.red = reinterpret_cast<float*>(q);
    q += step_red_bytes(p.max_terms);
    s.scratch = reinterpret_cast<float*>(q);
    q += step_scratch_bytes(p);
    s.ring = q;
    return s;
}

// ---------------------------------------------------------------- the work list
// Per-token geometry every thread derives from the plan.
struct StepGeo {
    int G;          // CTAs
    int cta;
    int pos, len;   // the token's position and window length
    int n_split;    // attention chunks
    int n_items;    // attention chunk items: chunks x KV heads
};

__device__ __forceinline__ int step_rows_of(const StepPlan& p, int ph) {
    switch (ph) {
        case kPhQkv: return p.qd + 2 * p.kvd;
        case kPhO: return p.dim;
        case kPhGu: return p.ffn;
        default: return p.dim;
    }
}
__device__ __forceinline__ int step_in_of(const StepPlan& p, int ph) {
    switch (ph) {
        case kPhQkv: return p.dim;
        case kPhO: return p.qd;
        case kPhGu: return p.dim;
        default: return p.ffn;
    }
}
__device__ __forceinline__ int step_type_of(const StepLayer& L, int ph) {
    switch (ph) {
        case kPhQkv: return L.tqkv;
        case kPhO: return L.to;
        case kPhGu: return L.tgu;
        default: return L.td;
    }
}
__device__ __forceinline__ const uint8_t* step_w_of(const StepLayer& L, int ph) {
    switch (ph) {
        case kPhQkv: return L.wqkv;
        case kPhO: return L.wo;
        case kPhGu: return L.wg;
        default: return L.wd;
    }
}

// Index of a GEMV phase in the layer's tile geometry.
__device__ __forceinline__ int step_gi(int ph) { return ph == kPhQkv ? 0 : ph - 1; }

__device__ __forceinline__ uint32_t span16(const uint8_t* src, uint32_t n) {
    if (n == 0) return 0;
    const uintptr_t a = (uintptr_t)src & ~(uintptr_t)15;
    const uintptr_t e = ((uintptr_t)src + n + 15) & ~(uintptr_t)15;
    return (uint32_t)(e - a);
}

// The producer's position in the ring: the stage to fill next and how many
// times the ring has wrapped (the empty barrier's phase to wait for).
struct StepRing {
    int s = 0;
    uint32_t round = 0;
    int n = 0;  // entries issued
};

// ---------------------------------------------------------------- synchronisation
__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(kStepCT) : "memory"); }

// Barrier of the compute warps that also ANDs a predicate over them: every
// thread leaves with the same answer (a shared flag read after a plain barrier
// could already hold a later call's value).
__device__ __forceinline__ bool cbar_and(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(kStepCT)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ int ld_volatile_i32(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

// Spinning threads look at the abort flag (a global word every CTA's threads
// would otherwise hammer) and their deadline only once per this many cycles.
constexpr long long kPollCycles = 16384;

// Thread 0 of the compute warps publishes this CTA's part of a phase (after
// the barrier every compute thread's stores of it are ordered before).
__device__ __forceinline__ void step_signal(unsigned* ctr, int tid) {
    cbar();
    if (tid == 0) {
        __threadfence();
        atomicAdd(ctr, 1u);
    }
}

// All compute threads: wait until *ctr >= target (bounded; a wait that gives
// up, or an abort raised by another CTA, ends the CTA's work -- uniformly, so
// no compute thread is left at a barrier).
__device__ bool step_wait(const unsigned* ctr, unsigned target, int* abort_flag, int32_t* err, int tid) {
    int ok = 1;
    if (tid == 0 && ld_acquire_u32(ctr) < target) {
        const long long t0 = clock64();
        long long next = t0 + kPollCycles;
        while (ld_acquire_u32(ctr) < target) {
            const long long now = clock64();
            if (now < next) continue;
            next = now + kPollCycles;
            if (ld_volatile_i32(abort_flag)) { ok = 0; break; }
            if (now - t0 > kWaitCycles) {
                record_error(err, kErrTimeout);
                atomicExch(abort_flag, 1);
                ok = 0;
                break;
            }
        }
    }
    return cbar_and(ok != 0);
}

// Wait on a ring stage (every compute thread).  A wait that gives up raises
// the abort and returns anyway: the threads go on through the same barriers
// (on stale data) to the next counter wait, which ends the CTA uniformly.
// Once the abort is raised later stage waits return at once.
__device__ __forceinline__ void step_stage_wait(uint64_t* bar, uint32_t parity, int* abort_flag, int32_t* err) {
    if (mbar_try_wait(bar, parity)) return;
    const long long t0 = clock64();
    long long next = t0 + kPollCycles;
    while (!mbar_try_wait(bar, parity)) {
        const long long now = clock64();
        if (now < next) continue;
        next = now + kPollCycles;
        if (ld_volatile_i32(abort_flag)) return;
        if (now - t0 > kWaitCycles) {
            record_error(err, kErrTimeout);
            atomicExch(abort_flag, 1);
            return;
        }
    }
}

// ---------------------------------------------------------------- timeline marks
// Diagnostic builds (-DGNCX_TRACE) record, per CTA and layer, %globaltimer at
// the phase boundaries of the compute warps (thread 0) into the trace buffer:
// one block of records per CTA, reserved with one atomic at kernel start.
constexpr int kStepMarks = 16;
constexpr int kStepTraceEntries = 2048;  // ring entries per CTA traced (producer and consumer)
#ifdef GNCX_TRACE
__device__ TraceRec* step_trace_block(unsigned n) {
    if (!g_trace_rec) return nullptr;
    const unsigned i = atomicAdd(g_trace_n, n);
    return i + n <= g_trace_cap ? g_trace_rec + i : nullptr;
}
__device__ __forceinline__ TraceRec*& step_cblk() {
    __shared__ TraceRec* blk;
    return blk;
}
#define STEP_CUSE(idx, t0v)                                  \
    do {                                                     \
        if (threadIdx.x == 0) STEP_ENTRY_REC(step_cblk(), kTagStepUse, (idx), (t0v)); \
    } while (0)
#define STEP_ENTRY_DECL(name) TraceRec* name = nullptr
#define STEP_ENTRY_INIT(name) name = step_trace_block(kStepTraceEntries)
#define STEP_ENTRY_T0(v) const unsigned long long v = trace_clock()
#define STEP_ENTRY_REC(blk, tag, idx, t0v)                                                      \
    do {                                                                                        \
        if ((blk) && (idx) < kStepTraceEntries) {                                               \
            const unsigned long long t1_ = trace_clock();                                       \
            trace_fill((blk)[idx], (tag), (uint32_t)(idx), (t0v), t1_, 0);                      \
        }                                                                                       \
    } while (0)
#define STEP_TRACE_DECL TraceRec* tblk = nullptr
#define STEP_TRACE_INIT(nl)                                                   \
    do {                                                                      \
        if (tid == 0 && g_trace_rec) {                                        \
            const unsigned n_ = (unsigned)(nl) * kStepMarks;                  \
            const unsigned i_ = atomicAdd(g_trace_n, n_);                     \
            if (i_ + n_ <= g_trace_cap) tblk = g_trace_rec + i_;              \
        }                                                                     \
    } while (0)
#define STEP_MARK(m, l)                                                                                  \
    do {                                                                                                 \
        if (tblk) {                                                                                      \
            const unsigned long long t_ = trace_clock();                                                 \
            trace_fill(tblk[(l) * kStepMarks + (m)], kTagStep, (uint32_t)((m) | ((l) << 8)), t_, t_, 1); \
        }                                                                                                \
    } while (0)
#else
#define STEP_TRACE_DECL \
    do {                \
    } while (0)
#define STEP_TRACE_INIT(nl) \
    do {                    \
    } while (0)
#define STEP_MARK(m, l) \
    do {                \
    } while (0)
#define STEP_ENTRY_DECL(name) \
    do {                      \
    } while (0)
#define STEP_ENTRY_INIT(name) \
    do {                      \
    } while (0)
#define STEP_ENTRY_T0(v) \
    do {                 \
    } while (0)
#define STEP_ENTRY_REC(blk, tag, idx, t0v) \
    do {                                   \
    } while (0)
#define STEP_CUSE(idx, t0v) \
    do {                    \
    } while (0)
#endif

// ---------------------------------------------------------------- residual stream + RMSNorm
struct StepResid {
    float h[kStepMaxPasses][8];  // elements (pass * kStepCT + tid) * 8 + e
};

__device__ __forceinline__ void step_load_gains(const float* __restrict__ w, int dim, int tid,
                                                float (&g)[kStepMaxPasses][8]) {
#pragma unroll
    for (int ps = 0; ps < kStepMaxPasses; ++ps) {
        const int base = (ps * kStepCT + tid) * 8;
        if (base < dim) {
            const float4 a = __ldg(reinterpret_cast<const float4*>(w + base));
            const float4 b = __ldg(reinterpret_cast<const float4*>(w + base + 4));
            g[ps][0] = a.x; g[ps][1] = a.y; g[ps][2] = a.z; g[ps][3] = a.w;
            g[ps][4] = b.x; g[ps][5] = b.y; g[ps][6] = b.z; g[ps][7] = b.w;
        }
    }
}

// h += y (y written by other CTAs: read from L2), the reference's
// hidden[i] = hidden[i] + proj[i] (lua/gncx_streamer.lua:871-873, :906-908).
__device__ __forceinline__ void step_add_residual(StepResid& r, const float* y, int dim, int tid) {
#pragma unroll
    for (int ps = 0; ps < kStepMaxPasses; ++ps) {
        const int base = (ps * kStepCT + tid) * 8;
        if (base < dim) {
            const float4 a = __ldcg(reinterpret_cast<const float4*>(y + base));
            const float4 b = __ldcg(reinterpret_cast<const float4*>(y + base + 4));
            float* h = r.h[ps];
            h[0] = fadd(h[0], a.x); h[1] = fadd(h[1], a.y); h[2] = fadd(h[2], a.z); h[3] = fadd(h[3], a.w);
            h[4] = fadd(h[4], b.x); h[5] = fadd(h[5], b.y); h[6] = fadd(h[6], b.z); h[7] = fadd(h[7], b.w);
        }
    }
}

// RMSNorm of the residual with gains g into the act-Q8 staging area (and,
// when `normed` is set, the fp32 result): the reference's four serial fp32
// lanes over x[4k+j]^2 combined in double (csrc/gncx_llm_kernels.cpp:789-840),
// then y = (x * inv) * w quantized per 32 inputs (:955-995).  Same arithmetic
// as add_norm_quant_row_kernel.
__device__ __noinline__ void step_norm_quant(const StepResid& r, const float (&g)[kStepMaxPasses][8], int dim, float eps,
                                const StepSmem& sm, float* normed, int tid) {
    __shared__ float s_inv;
    float* sq = sm.scratch;  // [4][dim/4]
    const int n4 = dim >> 2;
#pragma unroll
    for (int ps = 0; ps < kStepMaxPasses; ++ps) {
        const int base = (ps * kStepCT + tid) * 8;
        if (base < dim) {
            const int k = base >> 2;
#pragma unroll
            for (int j = 0; j < 4; ++j)
                *reinterpret_cast<float2*>(sq + (size_t)j * n4 + k) =
                    make_float2(fmul(r.h[ps][j], r.h[ps][j]), fmul(r.h[ps][4 + j], r.h[ps][4 + j]));
        }
    }
    cbar();
    if (tid < 32) {
        float acc = 0.0f;
        if (tid < 4) {
            const float4* p = reinterpret_cast<const float4*>(sq + (size_t)tid * n4);
#pragma unroll 8
            for (int i = 0; i < (n4 >> 2); ++i) {
                const float4 v = p[i];
                acc = fadd(fadd(fadd(fadd(acc, v.x), v.y), v.z), v.w);
            }
        }
        const float a1 = __shfl_sync(0xffffffffu, acc, 1);
        const float a2 = __shfl_sync(0xffffffffu, acc, 2);
        const float a3 = __shfl_sync(0xffffffffu, acc, 3);
        if (tid == 0) {
            const double s = __dadd_rn(__dadd_rn(__dadd_rn((double)acc, (double)a1), (double)a2), (double)a3);
            const float ms = __double2float_rn(__ddiv_rn(s, (double)dim));
            s_inv = fdiv(1.0f, __fsqrt_rn(fadd(ms, eps)));
        }
    }
    cbar();
    const float inv = s_inv;
    const int q4 = tid & 3;
#pragma unroll
    for (int ps = 0; ps < kStepMaxPasses; ++ps) {
        const int base = (ps * kStepCT + tid) * 8;
        if (ps * kStepHPass >= dim) break;  // uniform
        const bool ok = base < dim;
        float v[8];
        float amax = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            v[e] = ok ? fmul(fmul(r.h[ps][e], inv), g[ps][e]) : 0.0f;
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
        const int pair = part + __shfl_xor_sync(0xffffffffu, part, 1);
        const int other = __shfl_xor_sync(0xffffffffu, pair, 2);
        if (ok) {
            const int b = base >> 5;
            *reinterpret_cast<uint2*>(sm.qs + act_chunk_pos(b >> 3, 2 * (b & 7) + (q4 >> 1)) + 8 * (q4 & 1)) =
                make_uint2(w0, w1);
            if (q4 == 0)
                sm.rec[act_rec_pos(b)] =
                    make_float4(d, __int_as_float(pair), __int_as_float(other), __int_as_float(pair + other));
        }
    }
    cbar();
}

// act-Q8 staging of an fp32 vector other CTAs wrote (one shared copy, as above).
__device__ __noinline__ void step_stage_act(const float* x, int n, const StepSmem& sm, int tid) {
    stage_act_fp32<true>(x, n, sm.qs, sm.rec, tid, kStepCT);
    cbar();
}

// ---------------------------------------------------------------- GEMV tiles
// This lane's units (j and j + lpr) of the row at `rowp` in a stage, their
// terms parked in the row's slots of the warp's term area.
template <int T>
__device__ __forceinline__ void step_lane_units(const uint8_t* rowp, int j, int lpr, int upr, const ActView& av,
                                                float* terms) {
    constexpr int UB = Fmt<T>::UB, NW = Fmt<T>::NW, E = Fmt<T>::E;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int u = j + k * lpr;
        if (u < upr) {
            uint32_t w[NW];
            load_unit_smem<NW, T != kQ6_K>(rowp + (size_t)u * UB, w);
            float t[E];
            unit_terms<T>(w, UnitAct{av, u}, t);
            float* dst = terms + (size_t)u * E;
            if constexpr (E % 4 == 0) {
#pragma unroll
                for (int e = 0; e < E; e += 4)
                    *reinterpret_cast<float4*>(dst + e) = make_float4(t[e], t[e + 1], t[e + 2], t[e + 3]);
            } else {
#pragma unroll
                for (int e = 0; e < E; ++e) dst[e] = t[e];
            }
        }
    }
}

// The reference's per-row serial accumulation over the row's terms in order.
__device__ __forceinline__ float step_row_sum(const float* terms, int n) {
    float acc = 0.0f;
    if ((n & 3) == 0) {
#pragma unroll 4
        for (int i = 0; i < n; i += 4) {
            const float4 v4 = *reinterpret_cast<const float4*>(terms + i);
            acc = fadd(fadd(fadd(fadd(acc, v4.x), v4.y), v4.z), v4.w);
        }
    } else {
        for (int i = 0; i < n; ++i) acc = fadd(acc, terms[i]);
    }
    return acc;
}

__host__ __device__ __forceinline__ int type_terms(int t) { return (t == kQ4_0 || t == kQ8_0) ? 8 : 1; }

// One GEMV phase of this CTA: tiles cta, cta + G, ... of the matrix, outputs
// to y (rows) -- or, for the gate/up phase, glu(gate row, up row) to y.
// Each warp takes its rows of a tile and finishes them alone: units into its
// term area, the stage released, then each row's first lane adds the row's
// terms in unit order (and, for gate/up, takes the up row's sum from the
// lane that formed it).  FMT: the one format of every matrix, or 0.
//
// Not inlined: the four GEMV phases of a layer share one copy of this code,
// which stays in the instruction caches across phases (inlined copies, one
// per call site, were fetched cold at the start of every phase).
template <int FMT>
__device__ __noinline__ void step_gemv_phase(const StepPlan& p, const StepLayer& L, const StepGeo& g, int ph, const StepSmem& sm,
                                int& item, float* y, int* abort_flag, int tid) {
    const int lane = tid & 31, warp = tid >> 5;
    const int gi = step_gi(ph);
    const int rows = L.rows[gi];
    const int wr = L.wrows[gi];
    const int n_tiles = L.tiles[gi];
    const int type = FMT ? FMT : step_type_of(L, ph);
    const int upr = step_in_of(p, ph) / 256;
    const int lpr = step_lpr(upr);
    const size_t rb = (size_t)L.rbytes[gi];
    const int n_rows = step_rows_of(p, ph);
    const int E = type_terms(type);
    const ActView av{sm.qs, sm.rec};
    const uint8_t* w = step_w_of(L, ph);
    const bool pair = ph == kPhGu;
    const int rloc = lane / lpr, j = lane - rloc * lpr;
    const int hp = pair ? wr / 2 : wr;         // output rows of this warp per tile
    const bool up = pair && rloc >= hp;         // this lane's row is an up row
    const int orow = warp * hp + (up ? rloc - hp : rloc);  // output row within the tile
    float* terms = sm.red + (size_t)warp * 64 * p.max_terms + (size_t)rloc * upr * E;
    for (int tile = g.cta; tile < n_tiles; tile += g.G, ++item) {
        const int s = item & (kStepStages - 1);
        const uint32_t par = (uint32_t)(item / kStepStages) & 1u;
        STEP_ENTRY_T0(ct0);
        step_stage_wait(&sm.full[s], par, abort_flag, p.err);
        STEP_CUSE(item, ct0);
        const int r0 = tile * rows;
        const int nr = min(rows, n_rows - r0);
        const bool valid = rloc < wr && orow < nr;
        const uint8_t* stage = sm.ring + (size_t)s * p.stage_bytes;
        const uint8_t* src = (up ? L.wu : w) + (size_t)r0 * rb;
        const uint8_t* rowp = stage + (up ? L.pair_off : 0) + ((uintptr_t)src & 15) + (size_t)orow * rb;
        if (valid) {
            if constexpr (FMT != 0) {
                step_lane_units<FMT>(rowp, j, lpr, upr, av, terms);
            } else {
                switch (type) {
                    case kQ4_K: step_lane_units<kQ4_K>(rowp, j, lpr, upr, av, terms); break;
                    case kQ6_K: step_lane_units<kQ6_K>(rowp, j, lpr, upr, av, terms); break;
                    case kQ4_0: step_lane_units<kQ4_0>(rowp, j, lpr, upr, av, terms); break;
                    default: step_lane_units<kQ8_0>(rowp, j, lpr, upr, av, terms); break;
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty[s]);
        const float acc = (valid && j == 0) ? step_row_sum(terms, upr * E) : 0.0f;
        if (pair) {
            const float uacc = __shfl_down_sync(0xffffffffu, acc, hp * lpr);
            if (valid && j == 0 && !up) y[r0 + orow] = p.gelu ? geglu1(acc, uacc) : swiglu1(acc, uacc);
        } else if (valid && j == 0) {
            y[r0 + orow] = acc;
        }
        __syncwarp();  // the term area is rewritten by the next tile
    }
}

// ---------------------------------------------------------------- attention
// The start of a chunk item shared by both attention modes: the group's q
// heads normed and rotated into qs (the Q/K post step, overlapping the K copy
// in flight), the K stage waited for, and -- in the chunk holding the
// token's own position -- the new K row made in the stage (normed, rotated)
// and the new K and V rows written to the cache.  Returns the K stage.
__device__ __forceinline__ float* step_chunk_prologue(const StepPlan& p, const StepLayer& L, const StepGeo& g,
                                                      int kvh, int pn, bool own, float* qs, int qrs, int kitem,
                                                      const StepSmem& sm, int* abort_flag, int tid) {
    const int sK = kitem & (kStepStages - 1);
    const uint32_t parK = (uint32_t)(kitem / kStepStages) & 1u;
    const int lane = tid & 31, warp = tid >> 5;
    const int hd = p.hd;
    const int G = p.nh / p.nkv;
    const float* qkv = p.qkv;
    for (int task = warp; task < G; task += kStepCW) {
        float* x = qs + (size_t)task * qrs;
        const float* src = qkv + (size_t)(kvh * G + task) * hd;
        for (int i = lane; i < hd; i += 32) x[i] = __ldcg(src + i);
        __syncwarp();
        warp_head_norm_rope(x, hd, L.q_norm, p.qk_norm != 0, p.eps, p.rope_c, p.rope_s, g.pos, lane);
    }
    STEP_ENTRY_T0(ct0);
    step_stage_wait(&sm.full[sK], parK, abort_flag, p.err);
    STEP_CUSE(kitem, ct0);
    float* ks = reinterpret_cast<float*>(sm.ring + (size_t)sK * p.stage_bytes);
    const int kw = G % kStepCW;  // the warp that makes the new K row
    if (own && warp == kw) {
        float* x = ks + (size_t)pn * hd;
        const float* src = qkv + p.qd + (size_t)kvh * hd;
        const float* vsrc = qkv + p.qd + p.kvd + (size_t)kvh * hd;
        float* vdst = L.vc + ((size_t)kvh * p.max_seq + g.pos) * hd;
        for (int i = lane; i < hd; i += 32) {
            x[i] = __ldcg(src + i);
            vdst[i] = __ldcg(vsrc + i);  // the cache's new V row
        }
        __syncwarp();
        warp_head_norm_rope(x, hd, L.k_norm, p.qk_norm != 0, p.eps, p.rope_c, p.rope_s, g.pos, lane);
        float* kdst = L.kc + ((size_t)kvh * p.max_seq + g.pos) * hd;
        for (int i = lane; i < hd; i += 32) kdst[i] = x[i];
        // generic writes into a stage the TMA unit overwrites later
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    return ks;
}

// Arrival of a chunk item at its KV group's counter; true in the CTA whose
// item was the group's last (every compute thread gets the same answer).
__device__ __forceinline__ bool step_group_arrive(unsigned* ctr, unsigned n, int tid) {
    bool last = true;
    if (tid == 0) {
        __threadfence();
        const unsigned old = atomicAdd(ctr, 1u);
        last = old == n - 1;
        if (last) __threadfence();
    }
    return cbar_and(last);
}

// One split-KV work item: chunk `split` of KV head `kvh`; K rows in ring
// entry `item`, V rows in `item + 1`.  Writes the partial records of the
// group's G heads; the CTA that finishes a group's last chunk merges the
// group's heads into p.attn.
__device__ void step_attn_item(const StepPlan& p, const StepLayer& L, const StepGeo& g, int it, const StepSmem& sm,
                               int& item, unsigned* sync_l, int* abort_flag, int tid) {
    const int lane = tid & 31, warp = tid >> 5;
    const int hd = p.hd, C = p.chunk;
    const int G = p.nh / p.nkv, G4 = (G + 3) & ~3;
    const int split = it / p.nkv, kvh = it - split * p.nkv;
    const int c0 = split * C;
    const int cn = min(C, g.len - c0);
    const int pn = g.pos - c0;
    const bool own = pn < cn;  // this chunk holds the token's own position
    const int qrs = hd + 4, sld = C + 8;
    float* qs = sm.scratch;                          // [G][qrs]
    float* sc = qs + (size_t)G * qrs;                // [G][sld]
    float* es = sc + (size_t)G * sld;                // [C][G4]
    float* red2 = es + (size_t)C * G4;               // [G][2], then merge factors
    float* pvs = red2 + 2 * G + 8;                   // [npg][kPvHeads][hd]
    const int npg = kStepCT / hd;
    float* wsm = pvs + (size_t)npg * kPvHeads * hd;  // [G][max_splits]
    float* lsm = wsm + (size_t)G * p.max_splits;     // [G][max_splits]
    const int sK = item & (kStepStages - 1);
    const int vitem = item + 1;
    const int sV = vitem & (kStepStages - 1);
    const uint32_t parV = (uint32_t)(vitem / kStepStages) & 1u;
    float* ks = step_chunk_prologue(p, L, g, kvh, pn, own, qs, qrs, item, sm, abort_flag, tid);
    item += 2;
    float* vs = reinterpret_cast<float*>(sm.ring + (size_t)sV * p.stage_bytes);
    cbar();
    {
        const float scale = p.scale;
        chunk_scores_warp(ks, hd, qs, qrs, G, cn, kStepCW,
                          [&](int gg, int pp, float dot) { sc[gg * sld + pp] = fmul(dot, scale); });
    }
    cbar();
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[sK]);
    // per head: chunk max, exp (position-major for the PV), sum
    for (int gg = warp; gg < G; gg += kStepCW) {
        float mx = -INFINITY;
        for (int pp = lane; pp < cn; pp += 32) mx = fmaxf(mx, sc[gg * sld + pp]);
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float sum = 0.0f;
        for (int pp = lane; pp < cn; pp += 32) {
            const float e = exp_cr(fsub(sc[gg * sld + pp], mx));
            es[(size_t)pp * G4 + gg] = e;
            sum += e;
        }
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) { red2[2 * gg] = mx; red2[2 * gg + 1] = sum; }
    }
    for (int i = tid; i < cn * (G4 - G); i += kStepCT) es[(size_t)(i / (G4 - G)) * G4 + G + i % (G4 - G)] = 0.0f;
    STEP_ENTRY_T0(vt0);
    step_stage_wait(&sm.full[sV], parV, abort_flag, p.err);
    STEP_CUSE(vitem, vt0);
    if (own) {
        const float* vsrc = p.qkv + p.qd + p.kvd + (size_t)kvh * hd;
        for (int i = tid; i < hd; i += kStepCT) vs[(size_t)pn * hd + i] = __ldcg(vsrc + i);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    cbar();
    // o[g][d] = sum_p e[p][g] v[p][d], position groups summed through pvs
    const int d = tid % hd, pgi = tid / hd;
    const bool active = pgi < npg;
    const size_t R = attn_record_floats(hd);
    for (int g0 = 0; g0 < G; g0 += kPvHeads) {
        const int ng = min(kPvHeads, G - g0);
        float acc[kPvHeads];
#pragma unroll
        for (int i = 0; i < kPvHeads; ++i) acc[i] = 0.0f;
        if (active) {
            chunk_pv(vs, hd, es, G4, g0, ng, cn, d, pgi, npg, acc);
#pragma unroll
            for (int i = 0; i < kPvHeads; ++i)
                if (i < ng) pvs[((size_t)pgi * kPvHeads + i) * hd + d] = acc[i];
        }
        cbar();
        for (int t = tid; t < ng * hd; t += kStepCT) {
            const int i = t / hd, dd = t - i * hd;
            float v = pvs[(size_t)i * hd + dd];
            for (int q = 1; q < npg; ++q) v += pvs[((size_t)q * kPvHeads + i) * hd + dd];
            const int h = kvh * G + g0 + i;
            float* rec = p.part + ((size_t)h * p.max_splits + split) * R;
            rec[4 + dd] = v;
            if (dd == 0) { rec[0] = red2[2 * (g0 + i)]; rec[1] = red2[2 * (g0 + i) + 1]; }
        }
        cbar();
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[sV]);
    if (!step_group_arrive(&sync_l[kSyGroup + kvh], (unsigned)g.n_split, tid)) return;
    // merge the group's heads: one warp per head forms the weights, then
    // every thread takes (head, column) pairs
    const int n = g.n_split;
    float* sinv = red2 + 2 * G;  // [G] (8 floats reserved)
    for (int w = warp; w < G; w += kStepCW) {
        const float* rec0 = p.part + (size_t)(kvh * G + w) * p.max_splits * R;
        float* wv = wsm + (size_t)w * p.max_splits;
        float* lv = lsm + (size_t)w * p.max_splits;
        float M = -INFINITY;
        for (int s2 = lane; s2 < n; s2 += 32) {
            const float m = ld_l2(rec0 + (size_t)s2 * R);
            wv[s2] = m;
            lv[s2] = ld_l2(rec0 + (size_t)s2 * R + 1);
            M = fmaxf(M, m);
        }
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float Ls = 0.0f;
        for (int s2 = lane; s2 < n; s2 += 32) {
            const float wgt = exp_cr(fsub(wv[s2], M));
            wv[s2] = wgt;
            Ls = fadd(Ls, fmul(lv[s2], wgt));
        }
        for (int o = 16; o > 0; o >>= 1) Ls = fadd(Ls, __shfl_xor_sync(0xffffffffu, Ls, o));
        if (lane == 0) sinv[w] = fdiv(1.0f, fadd(Ls, 1e-12f));
    }
    cbar();
    for (int t = tid; t < G * hd; t += kStepCT) {
        const int w = t / hd, dd = t - w * hd;
        const float* col = p.part + (size_t)(kvh * G + w) * p.max_splits * R + 4 + dd;
        const float* wv = wsm + (size_t)w * p.max_splits;
        float o = 0.0f;
        for (int s0 = 0; s0 < n; s0 += kStepMergeBatch) {
            float v[kStepMergeBatch];
#pragma unroll
            for (int b = 0; b < kStepMergeBatch; ++b) v[b] = s0 + b < n ? ld_l2(col + (size_t)(s0 + b) * R) : 0.0f;
#pragma unroll
            for (int b = 0; b < kStepMergeBatch; ++b)
                if (s0 + b < n) o = fadd(o, fmul(v[b], wv[s0 + b]));
        }
        p.attn[(size_t)(kvh * G + w) * hd + dd] = fmul(o, sinv[w]);
    }
    step_signal(&sync_l[kSyAttn], tid);
}

// Exact mode, the softmax of the G heads of KV group kvh (the last chunk
// item's CTA): per head the maximum, e_t = exp(s_t - max), the serial sum of
// e_t in position order, inv = 1 / (sum + 1e-12) and the weights e_t * inv
// written over the scores -- csrc/gncx_llm_kernels.cpp:1960-1967, and the same
// computation as attn_exact_softmax_kernel.
__device__ void step_exact_softmax(const StepPlan& p, const StepGeo& g, int kvh, const StepSmem& sm, int tid) {
    const int lane = tid & 31, warp = tid >> 5;
    const int G = p.nh / p.nkv;
    float* eb_all = sm.scratch + (size_t)G * (p.hd + 4);
    for (int w = warp; w < G; w += kStepCW) {
        float* row = p.scores + (size_t)(kvh * G + w) * p.score_stride;
        float* eb = eb_all + (size_t)w * kSmBlock;
        float mx = -1e30f;
        for (int t = lane; t < g.len; t += 32) mx = fmaxf(mx, ld_l2(row + t));
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float sum = 0.0f;
        for (int t0 = 0; t0 < g.len; t0 += kSmBlock) {
            const int n = min(kSmBlock, g.len - t0);
            for (int i = lane; i < n; i += 32) {
                const float e = exp_cr(fsub(ld_l2(row + t0 + i), mx));
                eb[i] = e;
                row[t0 + i] = e;
            }
            __syncwarp();
            if (lane == 0) {
#pragma unroll 8
                for (int i = 0; i < n; ++i) sum = fadd(sum, eb[i]);
            }
            __syncwarp();
        }
        float inv = lane == 0 ? fdiv(1.0f, fadd(sum, 1e-12f)) : 0.0f;
        inv = __shfl_sync(0xffffffffu, inv, 0);
        // each lane rescales the positions it wrote (t = lane mod 32)
        for (int t = lane; t < g.len; t += 32) row[t] = fmul(row[t], inv);
    }
}

// Exact mode, one chunk item: the scores of the group's G heads over chunk
// `split` (K rows in ring entry `item`) written to p.scores; the last item of
// the group runs the group's softmax and raises its ready counter.
__device__ void step_exact_scores_item(const StepPlan& p, const StepLayer& L, const StepGeo& g, int it,
                                       const StepSmem& sm, int& item, unsigned* sync_l, int* abort_flag, int tid) {
    const int lane = tid & 31;
    const int hd = p.hd, C = p.chunk;
    const int G = p.nh / p.nkv;
    const int split = it / p.nkv, kvh = it - split * p.nkv;
    const int c0 = split * C;
    const int cn = min(C, g.len - c0);
    const int pn = g.pos - c0;
    const bool own = pn < cn;
    const int qrs = hd + 4;
    float* qs = sm.scratch;  // [G][qrs]
    const int sK = item & (kStepStages - 1);
    float* ks = step_chunk_prologue(p, L, g, kvh, pn, own, qs, qrs, item, sm, abort_flag, tid);
    item += 1;
    cbar();
    {
        const float scale = p.scale;
        float* srow = p.scores + (size_t)kvh * G * p.score_stride + c0;
        const int ms = p.score_stride;
        chunk_scores_warp(ks, hd, qs, qrs, G, cn, kStepCW,
                          [&](int gg, int pp, float dot) { srow[(size_t)gg * ms + pp] = fmul(dot, scale); });
    }
    cbar();
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[sK]);
    if (!step_group_arrive(&sync_l[kSyGroup + kvh], (unsigned)g.n_split, tid)) return;
    step_exact_softmax(p, g, kvh, sm, tid);
    step_signal(&sync_l[kSyReady + kvh], tid);
}

__device__ __forceinline__ void cp_async16_cg(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
                 "l"(gmem)
                 : "memory");
}

// Exact mode, one PV item: output columns [d0, d0 + kPvCols) of the G heads of
// KV group kvh.  Thread (head w, column c) of warp 0 runs
// out = sum over t, in order, of (weight_t * v_t[d]) (csrc/gncx_llm_kernels.cpp
// :1969-1988); V columns and weights stream through two shared-memory buffers
// of kPvChunk positions, copied by every compute thread.
__device__ void step_exact_pv_item(const StepPlan& p, const StepLayer& L, const StepGeo& g, int kvh, int d0,
                                   const StepSmem& sm, int tid) {
    const int G = p.nh / p.nkv;
    const int hd = p.hd;
    const size_t bufn = (size_t)kPvChunk * kPvCols + (size_t)G * kPvChunk;
    const float* vbase = L.vc + (size_t)kvh * p.max_seq * hd + d0;
    const float* wbase = p.scores + (size_t)kvh * G * p.score_stride;
    const int nk = (g.len + kPvChunk - 1) / kPvChunk;
    auto stage = [&](int k) {
        float* vb = sm.scratch + (size_t)(k & 1) * bufn;
        float* wb = vb + (size_t)kPvChunk * kPvCols;
        const int t0 = k * kPvChunk;
        const int n = min(kPvChunk, g.len - t0);
        for (int i = tid; i < n * (kPvCols / 4); i += kStepCT) {
            const int t = i / (kPvCols / 4), c = i - t * (kPvCols / 4);
            cp_async16_cg(vb + (size_t)t * kPvCols + 4 * c, vbase + (size_t)(t0 + t) * hd + 4 * c);
        }
        // weights in 16-byte pieces from L2 (rows are rewritten every layer, so
        // never through L1); a piece past the window reads the row's padding
        const int n4 = (n + 3) >> 2;
        for (int i = tid; i < G * n4; i += kStepCT) {
            const int w = i / n4, t = i - w * n4;
            cp_async16_cg(wb + (size_t)w * kPvChunk + 4 * t, wbase + (size_t)w * p.score_stride + t0 + 4 * t);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    const int w = tid / kPvCols, c = tid - w * kPvCols;
    const bool chain = tid < G * kPvCols;
    float acc = 0.0f;
    stage(0);
    for (int k = 0; k < nk; ++k) {
        if (k + 1 < nk) {
            stage(k + 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        cbar();
        if (chain) {
            const float* vb = sm.scratch + (size_t)(k & 1) * bufn;
            const float* wb = vb + (size_t)kPvChunk * kPvCols + (size_t)w * kPvChunk;
            const int n = min(kPvChunk, g.len - k * kPvChunk);
#pragma unroll 8
            for (int t = 0; t < n; ++t) acc = fadd(acc, fmul(wb[t], vb[(size_t)t * kPvCols + c]));
        }
        cbar();
    }
    if (chain) p.attn[(size_t)(kvh * G + w) * hd + d0 + c] = acc;
}

// ---------------------------------------------------------------- the producer
// One ring entry: wait until the stage is free, then one bulk copy per byte
// range (each range's 16-byte-aligned superset; range 1 at stage offset
// off1).  False when the wait gave up (the CTA is aborting).
__device__ __forceinline__ bool step_issue(const StepSmem& sm, const StepPlan& p, StepRing& rg, const uint8_t* src0,
                                           uint32_t n0, const uint8_t* src1, uint32_t n1, uint32_t off1,
                                           int* abort_flag) {
    const int s = rg.s;
    if (rg.round > 0) {
        const uint32_t par = (rg.round - 1) & 1u;
        if (!mbar_try_wait(&sm.empty[s], par)) {
            const long long t0 = clock64();
            long long next = t0 + kPollCycles;
            while (!mbar_try_wait(&sm.empty[s], par)) {
                const long long now = clock64();
                if (now < next) continue;
                next = now + kPollCycles;
                if (ld_volatile_i32(abort_flag)) return false;
                if (now - t0 > kWaitCycles) {
                    record_error(p.err, kErrTimeout);
                    atomicExch(abort_flag, 1);
                    return false;
                }
            }
        }
    }
    const uint32_t b0 = span16(src0, n0), b1 = span16(src1, n1);
    uint8_t* stage = sm.ring + (size_t)s * p.stage_bytes;
    mbar_arrive_expect_tx(&sm.full[s], b0 + b1);
    if (b0) bulk_g2s(stage, reinterpret_cast<const void*>((uintptr_t)src0 & ~(uintptr_t)15), b0, &sm.full[s]);
    if (b1) bulk_g2s(stage + off1, reinterpret_cast<const void*>((uintptr_t)src1 & ~(uintptr_t)15), b1, &sm.full[s]);
    ++rg.n;
    if (++rg.s == kStepStages) {
        rg.s = 0;
        ++rg.round;
    }
    return true;
}

// The CTA's tiles of one GEMV phase of layer L.
__device__ __forceinline__ bool step_issue_gemv(const StepSmem& sm, const StepPlan& p, const StepLayer& L,
                                                const StepGeo& g, int ph, StepRing& rg, int* abort_flag) {
    const int gi = step_gi(ph);
    const int rows = L.rows[gi];
    const size_t rb = (size_t)L.rbytes[gi];
    const int n_rows = step_rows_of(p, ph);
    const uint8_t* w = step_w_of(L, ph);
    const bool pair = ph == kPhGu;
    for (int tile = g.cta; tile < L.tiles[gi]; tile += g.G) {
        const int r0 = tile * rows;
        const uint32_t n = (uint32_t)((size_t)min(rows, n_rows - r0) * rb);
        if (!step_issue(sm, p, rg, w + (size_t)r0 * rb, n, pair ? L.wu + (size_t)r0 * rb : nullptr, pair ? n : 0u,
                        (uint32_t)L.pair_off, abort_flag))
            return false;
    }
    return true;
}

// The producer warp's lane 0: every ring entry of the CTA, in the order the
// compute warps consume them.  Returns after every copy it issued has landed.
template <bool EXACT>
__device__ void step_producer(const StepSmem& sm, const StepPlan& p, const StepGeo& g, int* abort_flag) {
    StepRing rg;
    bool ok = true;
    for (int l = 0; l < p.n_layers && ok; ++l) {
        const StepLayer L = p.layers[l];
        ok = step_issue_gemv(sm, p, L, g, kPhQkv, rg, abort_flag);
        for (int it = g.cta; it < g.n_items && ok; it += g.G) {
            const int split = it / p.nkv, kvh = it - split * p.nkv;
            const int c0 = split * p.chunk;
            // the chunk holding the token's own position loads the rows below
            // it; its own row is made in the kernel
            const uint32_t n = (uint32_t)(c0 + p.chunk > g.pos ? g.pos - c0 : p.chunk) * (uint32_t)p.hd * 4u;
            const size_t off = ((size_t)kvh * p.max_seq + c0) * p.hd;
            ok = step_issue(sm, p, rg, reinterpret_cast<const uint8_t*>(L.kc + off), n, nullptr, 0u, 0u, abort_flag);
            if (!EXACT && ok)
                ok = step_issue(sm, p, rg, reinterpret_cast<const uint8_t*>(L.vc + off), n, nullptr, 0u, 0u, abort_flag);
        }
        ok = ok && step_issue_gemv(sm, p, L, g, kPhO, rg, abort_flag);
        ok = ok && step_issue_gemv(sm, p, L, g, kPhGu, rg, abort_flag);
        ok = ok && step_issue_gemv(sm, p, L, g, kPhDown, rg, abort_flag);
    }
    // every copy issued has landed before the CTA may exit
    for (int k = rg.n > kStepStages ? rg.n - kStepStages : 0; k < rg.n; ++k)
        if (!mbar_wait(&sm.full[k % kStepStages], (uint32_t)(k / kStepStages) & 1u)) record_error(p.err, kErrTimeout);
}

// ---------------------------------------------------------------- the kernel
template <bool EXACT, int FMT>
__global__ void __launch_bounds__(kStepThreads, 1) decode_step_kernel(const StepPlan p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const StepSmem sm = step_carve(smem, p);
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    int* abort_flag = reinterpret_cast<int*>(p.sync + (size_t)p.n_layers * kStepSyncWords);
    StepGeo g;
    g.G = gridDim.x;
    g.cta = blockIdx.x;
    g.pos = p.st->pos;
    g.len = g.pos + 1;
    g.n_split = (g.len + p.chunk - 1) / p.chunk;
    g.n_items = g.n_split * p.nkv;
    if (tid == 0) {
        for (int i = 0; i < kStepStages; ++i) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], kStepCW);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == kStepCW) {
        if (lane == 0) step_producer<EXACT>(sm, p, g, abort_flag);
        return;
    }

    // ---------------- compute warps ----------------
    STEP_TRACE_DECL;
    STEP_TRACE_INIT(p.n_layers);
#ifdef GNCX_TRACE
    if (tid == 0) step_cblk() = step_trace_block(kStepTraceEntries);
#endif
    StepResid r;
    const int dim = p.dim;
#pragma unroll
    for (int ps = 0; ps < kStepMaxPasses; ++ps) {
        const int base = (ps * kStepCT + tid) * 8;
        if (base < dim) {
            const float4 a = __ldcg(reinterpret_cast<const float4*>(p.hidden + base));
            const float4 b = __ldcg(reinterpret_cast<const float4*>(p.hidden + base + 4));
            float* h = r.h[ps];
            h[0] = a.x; h[1] = a.y; h[2] = a.z; h[3] = a.w; h[4] = b.x; h[5] = b.y; h[6] = b.z; h[7] = b.w;
        }
    }
    int item = 0;
    float gn[kStepMaxPasses][8];
    const unsigned G = (unsigned)g.G;
    const int n_pv = p.nkv * (p.hd / kPvCols);  // exact mode PV items
    for (int l = 0; l < p.n_layers; ++l) {
        const StepLayer L = p.layers[l];
        unsigned* sy = p.sync + (size_t)l * kStepSyncWords;
        // ---- residual add (the previous layer's ffn_down) + attention RMSNorm
        STEP_MARK(0, l);
        step_load_gains(L.attn_norm, dim, tid, gn);
        if (l > 0) {
            if (!step_wait(p.sync + (size_t)(l - 1) * kStepSyncWords + kSyDown, G, abort_flag, p.err, tid)) return;
            step_add_residual(r, p.proj_d, dim, tid);
        }
        STEP_MARK(1, l);
        step_norm_quant(r, gn, dim, p.eps, sm, nullptr, tid);
        STEP_MARK(2, l);
        // ---- QKV GEMV
        step_gemv_phase<FMT>(p, L, g, kPhQkv, sm, item, p.qkv, abort_flag, tid);
        step_signal(&sy[kSyQkv], tid);
        STEP_MARK(3, l);
        // ---- attention
        if (!step_wait(&sy[kSyQkv], G, abort_flag, p.err, tid)) return;
        STEP_MARK(4, l);
        unsigned attn_target = (unsigned)p.nkv;
        if constexpr (!EXACT) {
            for (int it = g.cta; it < g.n_items; it += g.G) step_attn_item(p, L, g, it, sm, item, sy, abort_flag, tid);
        } else {
            for (int it = g.cta; it < g.n_items; it += g.G)
                step_exact_scores_item(p, L, g, it, sm, item, sy, abort_flag, tid);
            // PV items from the last CTA down, away from the chunk items
            const int ncb = p.hd / kPvCols;
            for (int it = g.G - 1 - g.cta; it < n_pv; it += g.G) {
                const int kvh = it / ncb;
                if (!step_wait(&sy[kSyReady + kvh], 1u, abort_flag, p.err, tid)) return;
                step_exact_pv_item(p, L, g, kvh, (it - kvh * ncb) * kPvCols, sm, tid);
                step_signal(&sy[kSyAttn], tid);
            }
            attn_target = (unsigned)n_pv;
        }
        STEP_MARK(5, l);
        // ---- O GEMV on the re-quantized attention output
        if (!step_wait(&sy[kSyAttn], attn_target, abort_flag, p.err, tid)) return;
        STEP_MARK(6, l);
        step_stage_act(p.attn, p.qd, sm, tid);
        STEP_MARK(12, l);
        step_gemv_phase<FMT>(p, L, g, kPhO, sm, item, p.proj_o, abort_flag, tid);
        step_signal(&sy[kSyO], tid);
        STEP_MARK(7, l);
        // ---- residual add + ffn RMSNorm
        step_load_gains(L.ffn_norm, dim, tid, gn);
        if (!step_wait(&sy[kSyO], G, abort_flag, p.err, tid)) return;
        STEP_MARK(8, l);
        step_add_residual(r, p.proj_o, dim, tid);
        step_norm_quant(r, gn, dim, p.eps, sm, nullptr, tid);
        STEP_MARK(9, l);
        // ---- gate/up GEMV with the GLU in its epilogue
        step_gemv_phase<FMT>(p, L, g, kPhGu, sm, item, p.glu, abort_flag, tid);
        step_signal(&sy[kSyGu], tid);
        STEP_MARK(10, l);
        // ---- ffn_down on the re-quantized GLU output
        if (!step_wait(&sy[kSyGu], G, abort_flag, p.err, tid)) return;
        STEP_MARK(11, l);
        step_stage_act(p.glu, p.ffn, sm, tid);
        STEP_MARK(13, l);
        step_gemv_phase<FMT>(p, L, g, kPhDown, sm, item, p.proj_d, abort_flag, tid);
        step_signal(&sy[kSyDown], tid);
    }
    // ---- final residual add + output norm: CTA 0 writes the LM head's input
    if (g.cta != 0) return;
    step_load_gains(p.out_norm, dim, tid, gn);
    if (!step_wait(p.sync + (size_t)(p.n_layers - 1) * kStepSyncWords + kSyDown, G, abort_flag, p.err, tid)) return;
    step_add_residual(r, p.proj_d, dim, tid);
    step_norm_quant(r, gn, dim, p.eps, sm, p.normed, tid);
    // the staged act vector: the quants, then the block records (in shared
    // memory the records sit after the largest input's quants)
    {
        const uint4* q = reinterpret_cast<const uint4*>(sm.qs);
        uint4* dq = reinterpret_cast<uint4*>(p.act_out);
        for (int i = tid; i < dim / 16; i += kStepCT) dq[i] = q[i];
        float4* dr = reinterpret_cast<float4*>(p.act_out + dim);
        for (int i = tid; i < dim / 32; i += kStepCT) dr[i] = sm.rec[i];
    }
#pragma unroll
    for (int ps = 0; ps < kStepMaxPasses; ++ps) {
        const int base = (ps * kStepCT + tid) * 8;
        if (base < dim) {
            reinterpret_cast<float4*>(p.hidden + base)[0] = make_float4(r.h[ps][0], r.h[ps][1], r.h[ps][2], r.h[ps][3]);
            reinterpret_cast<float4*>(p.hidden + base)[1] = make_float4(r.h[ps][4], r.h[ps][5], r.h[ps][6], r.h[ps][7]);
        }
    }
}

// ---------------------------------------------------------------- host side
static bool fmt_ok(int t, int in) {
    if (t != kQ4_0 && t != kQ8_0 && t != kQ4_K && t != kQ6_K) return false;
    if (in % 256) return false;
    return row_bytes(t, in) % 16 == 0 || t == kQ6_K;
}

int decode_step_plan(StepPlan& p, StepLayer* host_layers, int max_smem) {
    if (p.n_layers <= 0 || p.dim <= 0 || p.dim > kStepMaxDim || p.dim % 256 || p.nh <= 0 || p.nkv <= 0 ||
        p.nh % p.nkv || p.max_seq <= 0)
        return kErrInvalidArg;
    const int G = p.nh / p.nkv;
    if (!(G == 1 || G == 2 || G == 4) || p.hd % kPvCols || p.hd > 128 || p.hd < 32 || kStepCT % p.hd ||
        p.nkv > kStepMaxKv)
        return kErrInvalidArg;
    if (p.qd != p.nh * p.hd || p.kvd != p.nkv * p.hd || p.qd % 256 || p.ffn % 256) return kErrInvalidArg;
    p.stage_bytes = kStepStageBytes;
    p.chunk = step_attn_chunk(p.hd, p.stage_bytes);
    if (p.chunk < 16) return kErrInvalidArg;
    p.max_splits = (p.max_seq + p.chunk - 1) / p.chunk;
    p.exact_ok = 1;
    p.score_stride = (p.max_seq + 3) & ~3;
    int max_terms = 1;
    bool all_q4k = true;
    for (int l = 0; l < p.n_layers; ++l) {
        StepLayer& L = host_layers[l];
        const int ts[4] = {L.tqkv, L.to, L.tgu, L.td};
        const int ins[4] = {p.dim, p.qd, p.dim, p.ffn};
        const int outs[4] = {p.qd + 2 * p.kvd, p.dim, p.ffn, p.dim};
        for (int i = 0; i < 4; ++i) {
            if (!fmt_ok(ts[i], ins[i])) return kErrInvalidArg;
            const int wr = step_warp_rows(ts[i], ins[i], p.stage_bytes, i == 2);
            if (wr < (i == 2 ? 2 : 1)) return kErrCapacity;
            L.wrows[i] = i == 2 ? wr / 2 * 2 : wr;
            L.rows[i] = kStepCW * (i == 2 ? wr / 2 : wr);
            L.tiles[i] = (outs[i] + L.rows[i] - 1) / L.rows[i];
            L.rbytes[i] = (int)row_bytes(ts[i], ins[i]);
            const int e = type_terms(ts[i]);
            max_terms = e > max_terms ? e : max_terms;
            all_q4k = all_q4k && ts[i] == kQ4_K;
        }
        L.pair_off = step_pair_offset(L.rows[2], (size_t)L.rbytes[2]);
        // the 16-byte unit loads of the aligned formats need 16-byte aligned rows
        const uintptr_t ptrs[5] = {(uintptr_t)L.wqkv, (uintptr_t)L.wo, (uintptr_t)L.wg, (uintptr_t)L.wu,
                                   (uintptr_t)L.wd};
        const int pt[5] = {L.tqkv, L.to, L.tgu, L.tgu, L.td};
        for (int i = 0; i < 5; ++i)
            if (pt[i] != kQ6_K && ptrs[i] % 16) return kErrUnaligned;
        if (((uintptr_t)L.kc | (uintptr_t)L.vc) % 16) return kErrUnaligned;
    }
    p.max_terms = max_terms;
    p.all_q4k = all_q4k ? 1 : 0;
    return step_smem_bytes(p) <= (size_t)max_smem ? kOk : kErrCapacity;
}

size_t decode_step_sync_words(int n_layers) { return (size_t)(n_layers + 1) * kStepSyncWords; }

template <bool EXACT, int FMT>
static int step_launch_t(const StepPlan& p, cudaStream_t st) {
    auto k = decode_step_kernel<EXACT, FMT>;
    const size_t smem = step_smem_bytes(p);
    if (set_smem_limit(k, smem) != cudaSuccess) return kErrCuda;
    const DeviceInfo& dev = device_info();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(dev.sm_count);
    cfg.blockDim = dim3(kStepThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once: they wait on one another
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, p) == cudaSuccess ? kOk : kErrCuda;
}

int decode_step_launch(const StepPlan& p, cudaStream_t st) {
    if (p.exact) return p.all_q4k ? step_launch_t<true, kQ4_K>(p, st) : step_launch_t<true, 0>(p, st);
    return p.all_q4k ? step_launch_t<false, kQ4_K>(p, st) : step_launch_t<false, 0>(p, st);
}

}  // namespace gncx
