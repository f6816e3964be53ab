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
#include "units.cuh"

namespace gncx {

constexpr int kStepCW = 8;                  // compute warps
constexpr int kStepCT = kStepCW * 32;       // compute threads
constexpr int kStepThreads = kStepCT + 32;  // + the producer warp
constexpr int kStepMaxUnits = kStepCT;      // 256-input units per GEMV tile: one per compute thread
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
// Whole rows per tile of a matrix with `in` inputs: at most one unit per
// compute thread and the rows' bytes (+ alignment slack) within a stage;
// `pair` tiles hold that many gate rows and as many up rows.
__host__ __device__ inline int step_tile_rows(int type, int in, int stage_bytes, bool pair) {
    const int upr = in / 256;
    const size_t rb = row_bytes(type, in);
    int r;
    if (pair) {
        r = (kStepMaxUnits / 2) / upr;
        const int fit = (int)(((size_t)stage_bytes - 96) / (2 * rb));
        r = r < fit ? r : fit;
    } else {
        r = kStepMaxUnits / upr;
        const int fit = (int)(((size_t)stage_bytes - 32) / rb);
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
    float* red;       // [2][kStepMaxUnits * max_terms] unit terms awaiting the serial row sums
    float* scratch;   // norm squares / attention work area (union)
    uint8_t* ring;
};

__host__ __device__ inline size_t step_act_bytes(int max_in) {
    return ((size_t)max_in + (size_t)(max_in / 32) * 16 + 127) & ~(size_t)127;
}
__host__ __device__ inline size_t step_red_bytes(int max_terms) { return (size_t)2 * kStepMaxUnits * max_terms * 4; }

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
           (size_t)p.stages * p.stage_bytes;
}

__device__ inline StepSmem step_carve(uint8_t* base, const StepPlan& p) {
    StepSmem s;
    s.full = reinterpret_cast<uint64_t*>(base);
    s.empty = s.full + kStepMaxStages;
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
// One ring entry: up to two byte ranges (a gate/up tile has two), each copied
// as its 16-byte-aligned superset; range 1 lands at stage offset `off1`.
struct StepEntry {
    const uint8_t* src0;
    uint32_t n0;
    const uint8_t* src1;
    uint32_t n1;
    uint32_t off1;
};

// Per-token geometry every thread derives from the plan.
struct StepGeo {
    int G;          // CTAs
    int cta;
    int pos, len;   // the token's position and window length
    int n_split;    // attention chunks
    int n_items;    // attention chunk items: chunks x KV heads
};

__device__ __forceinline__ int step_mine(int n_total, const StepGeo& g) {
    return n_total > g.cta ? (n_total - g.cta + g.G - 1) / g.G : 0;
}

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

// Tiles of a GEMV phase.
__device__ __forceinline__ int step_tiles(const StepPlan& p, const StepLayer& L, int ph, int& rows) {
    rows = step_tile_rows(step_type_of(L, ph), step_in_of(p, ph), p.stage_bytes, ph == kPhGu);
    const int n = step_rows_of(p, ph);
    return (n + rows - 1) / rows;
}

// Ring entries per attention chunk item: K and V (split-KV) or K only (exact
// mode, whose PV step loads V itself).
__device__ __forceinline__ int step_attn_per_item(const StepPlan& p) { return p.exact ? 1 : 2; }

// Ring entries of this CTA in phase `ph` of a layer.
__device__ __forceinline__ int step_entries(const StepPlan& p, const StepLayer& L, const StepGeo& g, int ph) {
    if (ph == kPhAttn) return step_attn_per_item(p) * step_mine(g.n_items, g);
    int rows;
    return step_mine(step_tiles(p, L, ph, rows), g);
}

__device__ StepEntry step_describe(const StepPlan& p, const StepLayer& L, const StepGeo& g, int ph, int k) {
    StepEntry e{nullptr, 0u, nullptr, 0u, 0u};
    if (ph == kPhAttn) {
        const int per = step_attn_per_item(p);
        const int item = g.cta + (k / per) * g.G;
        const bool is_v = per == 2 && (k & 1);
        const int split = item / p.nkv, kvh = item - split * p.nkv;
        const int c0 = split * p.chunk;
        // the chunk holding the token's own position loads the rows below it;
        // its own row is made in the kernel
        const int n_load = c0 + p.chunk > g.pos ? g.pos - c0 : p.chunk;
        const float* cache = is_v ? L.vc : L.kc;
        e.src0 = reinterpret_cast<const uint8_t*>(cache + ((size_t)kvh * p.max_seq + c0) * p.hd);
        e.n0 = (uint32_t)n_load * (uint32_t)p.hd * 4u;
        return e;
    }
    int rows;
    step_tiles(p, L, ph, rows);
    const int tile = g.cta + k * g.G;
    const int r0 = tile * rows;
    const int n_rows = step_rows_of(p, ph);
    const int nr = min(rows, n_rows - r0);
    const int type = step_type_of(L, ph);
    const size_t rb = row_bytes(type, step_in_of(p, ph));
    e.src0 = step_w_of(L, ph) + (size_t)r0 * rb;
    e.n0 = (uint32_t)((size_t)nr * rb);
    if (ph == kPhGu) {
        e.src1 = L.wu + (size_t)r0 * rb;
        e.n1 = e.n0;
        e.off1 = (uint32_t)step_pair_offset(rows, rb);
    }
    return e;
}

__device__ __forceinline__ uint32_t span16(const uint8_t* src, uint32_t n) {
    if (n == 0) return 0;
    const uintptr_t a = (uintptr_t)src & ~(uintptr_t)15;
    const uintptr_t e = ((uintptr_t)src + n + 15) & ~(uintptr_t)15;
    return (uint32_t)(e - a);
}

struct StepCursor {
    int l, ph, k, n;  // layer, phase, entry within the phase, entries in the phase
};

__device__ void step_settle(const StepPlan& p, const StepGeo& g, StepCursor& c) {
    while (c.l < p.n_layers) {
        if (c.k < c.n) return;
        c.k = 0;
        if (++c.ph == kPhCount) {
            c.ph = 0;
            ++c.l;
            if (c.l >= p.n_layers) return;
        }
        const StepLayer L = p.layers[c.l];
        c.n = step_entries(p, L, g, c.ph);
    }
}

__device__ StepCursor step_first(const StepPlan& p, const StepGeo& g) {
    StepCursor c{0, 0, 0, 0};
    const StepLayer L = p.layers[0];
    c.n = step_entries(p, L, g, 0);
    step_settle(p, g, c);
    return c;
}

__device__ __forceinline__ void step_next(const StepPlan& p, const StepGeo& g, StepCursor& c) {
    ++c.k;
    step_settle(p, g, c);
}

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
        while (ld_acquire_u32(ctr) < target) {
            if (ld_volatile_i32(abort_flag)) { ok = 0; break; }
            if (clock64() - t0 > kWaitCycles) {
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
    while (!mbar_try_wait(bar, parity)) {
        if (ld_volatile_i32(abort_flag)) return;
        if (clock64() - t0 > kWaitCycles) {
            record_error(err, kErrTimeout);
            atomicExch(abort_flag, 1);
            return;
        }
    }
}

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
__device__ void step_norm_quant(const StepResid& r, const float (&g)[kStepMaxPasses][8], int dim, float eps,
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

// ---------------------------------------------------------------- GEMV tiles
template <int T>
__device__ __forceinline__ void step_units(const uint8_t* r0p, const uint8_t* r1p, int split, int rb, int nr, int upr,
                                           const ActView& av, float* red, int tid) {
    constexpr int UB = Fmt<T>::UB, NW = Fmt<T>::NW, E = Fmt<T>::E;
    if (tid < nr * upr) {
        const int r = tid / upr, u = tid - r * upr;
        const uint8_t* rp = r < split ? r0p + (size_t)r * rb : r1p + (size_t)(r - split) * rb;
        uint32_t w[NW];
        load_unit_smem<NW, T != kQ6_K>(rp + (size_t)u * UB, w);
        float t[E];
        unit_terms<T>(w, UnitAct{av, u}, t);
        float* dst = red + (size_t)tid * E;
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
__device__ void step_gemv_phase(const StepPlan& p, const StepLayer& L, const StepGeo& g, int ph, const StepSmem& sm,
                                int& item, int& red_buf, float* y, int* abort_flag, int tid) {
    const int lane = tid & 31;
    int rows;
    const int n_tiles = step_tiles(p, L, ph, rows);
    const int type = step_type_of(L, ph);
    const int in = step_in_of(p, ph);
    const int upr = in / 256;
    const size_t rb = row_bytes(type, in);
    const int n_rows = step_rows_of(p, ph);
    const int E = type_terms(type);
    const ActView av{sm.qs, sm.rec};
    const uint8_t* w = step_w_of(L, ph);
    const bool pair = ph == kPhGu;
    for (int tile = g.cta; tile < n_tiles; tile += g.G, ++item) {
        const int s = item % p.stages;
        const uint32_t par = (uint32_t)(item / p.stages) & 1u;
        step_stage_wait(&sm.full[s], par, abort_flag, p.err);
        const int r0 = tile * rows;
        const int nr = min(rows, n_rows - r0);
        uint8_t* stage = sm.ring + (size_t)s * p.stage_bytes;
        const uint8_t* src0 = w + (size_t)r0 * rb;
        const uint8_t* r0p = stage + ((uintptr_t)src0 & 15);
        const uint8_t* r1p = r0p;
        int split = nr;
        int nr_all = nr;
        if (pair) {
            const uint8_t* src1 = L.wu + (size_t)r0 * rb;
            r1p = stage + step_pair_offset(rows, rb) + ((uintptr_t)src1 & 15);
            nr_all = 2 * nr;
        }
        float* red = sm.red + (size_t)red_buf * kStepMaxUnits * p.max_terms;
        switch (type) {
            case kQ4_K: step_units<kQ4_K>(r0p, r1p, split, (int)rb, nr_all, upr, av, red, tid); break;
            case kQ6_K: step_units<kQ6_K>(r0p, r1p, split, (int)rb, nr_all, upr, av, red, tid); break;
            case kQ4_0: step_units<kQ4_0>(r0p, r1p, split, (int)rb, nr_all, upr, av, red, tid); break;
            default: step_units<kQ8_0>(r0p, r1p, split, (int)rb, nr_all, upr, av, red, tid); break;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty[s]);
        cbar();
        const int nt = upr * E;
        if (tid < nr) {
            if (pair) {
                const float gv = step_row_sum(red + (size_t)tid * nt, nt);
                const float uv = step_row_sum(red + (size_t)(nr + tid) * nt, nt);
                y[r0 + tid] = p.gelu ? geglu1(gv, uv) : swiglu1(gv, uv);
            } else {
                y[r0 + tid] = step_row_sum(red + (size_t)tid * nt, nt);
            }
        }
        red_buf ^= 1;
    }
}

// ---------------------------------------------------------------- attention
// The start of a chunk item shared by both attention modes: the group's q
// heads normed and rotated into qs (the Q/K post step, overlapping the K copy
// in flight), the K stage waited for, and -- in the chunk holding the
// token's own position -- the new K row made in the stage (normed, rotated)
// and the new K and V rows written to the cache.  Returns the K stage.
__device__ __forceinline__ float* step_chunk_prologue(const StepPlan& p, const StepLayer& L, const StepGeo& g,
                                                      int kvh, int pn, bool own, float* qs, int qrs, int sK,
                                                      uint32_t parK, const StepSmem& sm, int* abort_flag, int tid) {
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
    step_stage_wait(&sm.full[sK], parK, abort_flag, p.err);
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
    const int sK = item % p.stages;
    const uint32_t parK = (uint32_t)(item / p.stages) & 1u;
    const int sV = (item + 1) % p.stages;
    const uint32_t parV = (uint32_t)((item + 1) / p.stages) & 1u;
    item += 2;
    float* ks = step_chunk_prologue(p, L, g, kvh, pn, own, qs, qrs, sK, parK, sm, abort_flag, tid);
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
    step_stage_wait(&sm.full[sV], parV, abort_flag, p.err);
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
    const int sK = item % p.stages;
    const uint32_t parK = (uint32_t)(item / p.stages) & 1u;
    item += 1;
    float* ks = step_chunk_prologue(p, L, g, kvh, pn, own, qs, qrs, sK, parK, sm, abort_flag, tid);
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

// ---------------------------------------------------------------- the kernel
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
        for (int i = 0; i < p.stages; ++i) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], kStepCW);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == kStepCW) {
        // ---------------- producer: the CTA's weight tiles and K/V chunks, in order ----------------
        if (lane != 0) return;
        StepCursor c = step_first(p, g);
        StepCursor pf = c;
        uint32_t ahead = 0;
        int item = 0;
        const uint32_t want_ahead = (uint32_t)p.ahead;
        while (c.l < p.n_layers) {
            if (want_ahead) {
                while (pf.l < p.n_layers && ahead < want_ahead) {
                    const StepLayer Lp = p.layers[pf.l];
                    const StepEntry e = step_describe(p, Lp, g, pf.ph, pf.k);
                    const uint32_t b0 = span16(e.src0, e.n0), b1 = span16(e.src1, e.n1);
                    if (b0) bulk_prefetch_l2(reinterpret_cast<const void*>((uintptr_t)e.src0 & ~(uintptr_t)15), b0);
                    if (b1) bulk_prefetch_l2(reinterpret_cast<const void*>((uintptr_t)e.src1 & ~(uintptr_t)15), b1);
                    ahead += b0 + b1;
                    step_next(p, g, pf);
                }
            }
            const StepLayer L = p.layers[c.l];
            const StepEntry e = step_describe(p, L, g, c.ph, c.k);
            const int s = item % p.stages;
            const int use = item / p.stages;
            if (use > 0) {
                const uint32_t par = (uint32_t)(use - 1) & 1u;
                bool ok = mbar_try_wait(&sm.empty[s], par);
                if (!ok) {
                    const long long t0 = clock64();
                    while (!(ok = mbar_try_wait(&sm.empty[s], par))) {
                        if (ld_volatile_i32(abort_flag)) break;
                        if (clock64() - t0 > kWaitCycles) {
                            record_error(p.err, kErrTimeout);
                            atomicExch(abort_flag, 1);
                            break;
                        }
                    }
                }
                if (!ok) break;
            }
            const uint32_t b0 = span16(e.src0, e.n0), b1 = span16(e.src1, e.n1);
            uint8_t* stage = sm.ring + (size_t)s * p.stage_bytes;
            mbar_arrive_expect_tx(&sm.full[s], b0 + b1);
            if (b0) bulk_g2s(stage, reinterpret_cast<const void*>((uintptr_t)e.src0 & ~(uintptr_t)15), b0, &sm.full[s]);
            if (b1)
                bulk_g2s(stage + e.off1, reinterpret_cast<const void*>((uintptr_t)e.src1 & ~(uintptr_t)15), b1,
                         &sm.full[s]);
            if (want_ahead) ahead = ahead > b0 + b1 ? ahead - (b0 + b1) : 0;
            ++item;
            step_next(p, g, c);
        }
        // every copy issued has landed before the CTA may exit
        for (int k = item > p.stages ? item - p.stages : 0; k < item; ++k)
            if (!mbar_wait(&sm.full[k % p.stages], (uint32_t)(k / p.stages) & 1u)) record_error(p.err, kErrTimeout);
        return;
    }

    // ---------------- compute warps ----------------
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
    int item = 0, red_buf = 0;
    float gn[kStepMaxPasses][8];
    const unsigned G = (unsigned)g.G;
    const int n_pv = p.nkv * (p.hd / kPvCols);  // exact mode PV items
    for (int l = 0; l < p.n_layers; ++l) {
        const StepLayer L = p.layers[l];
        unsigned* sy = p.sync + (size_t)l * kStepSyncWords;
        // ---- residual add (the previous layer's ffn_down) + attention RMSNorm
        step_load_gains(L.attn_norm, dim, tid, gn);
        if (l > 0) {
            if (!step_wait(p.sync + (size_t)(l - 1) * kStepSyncWords + kSyDown, G, abort_flag, p.err, tid)) return;
            step_add_residual(r, p.proj_d, dim, tid);
        }
        step_norm_quant(r, gn, dim, p.eps, sm, nullptr, tid);
        // ---- QKV GEMV
        step_gemv_phase(p, L, g, kPhQkv, sm, item, red_buf, p.qkv, abort_flag, tid);
        step_signal(&sy[kSyQkv], tid);
        // ---- attention
        if (!step_wait(&sy[kSyQkv], G, abort_flag, p.err, tid)) return;
        unsigned attn_target = (unsigned)p.nkv;
        if (!p.exact) {
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
        // ---- O GEMV on the re-quantized attention output
        if (!step_wait(&sy[kSyAttn], attn_target, abort_flag, p.err, tid)) return;
        stage_act_fp32<true>(p.attn, p.qd, sm.qs, sm.rec, tid, kStepCT);
        cbar();
        step_gemv_phase(p, L, g, kPhO, sm, item, red_buf, p.proj_o, abort_flag, tid);
        step_signal(&sy[kSyO], tid);
        // ---- residual add + ffn RMSNorm
        step_load_gains(L.ffn_norm, dim, tid, gn);
        if (!step_wait(&sy[kSyO], G, abort_flag, p.err, tid)) return;
        step_add_residual(r, p.proj_o, dim, tid);
        step_norm_quant(r, gn, dim, p.eps, sm, nullptr, tid);
        // ---- gate/up GEMV with the GLU in its epilogue
        step_gemv_phase(p, L, g, kPhGu, sm, item, red_buf, p.glu, abort_flag, tid);
        step_signal(&sy[kSyGu], tid);
        // ---- ffn_down on the re-quantized GLU output
        if (!step_wait(&sy[kSyGu], G, abort_flag, p.err, tid)) return;
        stage_act_fp32<true>(p.glu, p.ffn, sm.qs, sm.rec, tid, kStepCT);
        cbar();
        step_gemv_phase(p, L, g, kPhDown, sm, item, red_buf, p.proj_d, abort_flag, tid);
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

int decode_step_plan(StepPlan& p, const StepLayer* host_layers, int max_smem) {
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
    for (int l = 0; l < p.n_layers; ++l) {
        const StepLayer& L = host_layers[l];
        const int ts[4] = {L.tqkv, L.to, L.tgu, L.td};
        const int ins[4] = {p.dim, p.qd, p.dim, p.ffn};
        for (int i = 0; i < 4; ++i) {
            if (!fmt_ok(ts[i], ins[i])) return kErrInvalidArg;
            if (step_tile_rows(ts[i], ins[i], p.stage_bytes, i == 2) < 1) return kErrCapacity;
            const int e = type_terms(ts[i]);
            max_terms = e > max_terms ? e : max_terms;
        }
        // the 16-byte unit loads of the aligned formats need 16-byte aligned rows
        const uintptr_t ptrs[5] = {(uintptr_t)L.wqkv, (uintptr_t)L.wo, (uintptr_t)L.wg, (uintptr_t)L.wu,
                                   (uintptr_t)L.wd};
        const int pt[5] = {L.tqkv, L.to, L.tgu, L.tgu, L.td};
        for (int i = 0; i < 5; ++i)
            if (pt[i] != kQ6_K && ptrs[i] % 16) return kErrUnaligned;
        if (((uintptr_t)L.kc | (uintptr_t)L.vc) % 16) return kErrUnaligned;
    }
    p.max_terms = max_terms;
    for (int s = kStepMaxStages; s >= 2; --s) {
        p.stages = s;
        if (step_smem_bytes(p) <= (size_t)max_smem) return kOk;
    }
    return kErrCapacity;
}

size_t decode_step_sync_words(int n_layers) { return (size_t)(n_layers + 1) * kStepSyncWords; }

int decode_step_launch(const StepPlan& p, cudaStream_t st) {
    const size_t smem = step_smem_bytes(p);
    if (set_smem_limit(decode_step_kernel, smem) != cudaSuccess) return kErrCuda;
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
    return cudaLaunchKernelEx(&cfg, decode_step_kernel, p) == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace gncx
