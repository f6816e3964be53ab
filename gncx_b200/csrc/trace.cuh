// trace.cuh -- optional kernel timeline records for diagnostic builds.
//
// Built with -DGNCX_TRACE (python -m gncx_b200.build --trace writes the
// separate library libgncx_llm_core_trace.so; the product library has none of
// this), every kernel that opens a GNCX_TRACE_SCOPE appends one record per
// CTA when thread 0 leaves it: the grid id, the kernel's tag and an argument
// (e.g. a GEMV's row count), the CTA index, and %globaltimer at thread 0's
// entry and exit.  gncx_trace_enable() hands the library a device buffer;
// grouping the records by grid id gives each launch's first start and last
// end as they ran inside CUDA graphs and under programmatic dependent launch,
// which a serialising profiler cannot show.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace gncx {

enum TraceTag : uint32_t {
    kTagGemv = 1, kTagGemvBf16, kTagMatbatch, kTagMatbatchTc, kTagAttnPartial, kTagAttnCombine, kTagAttnPrefill,
    kTagAttnExactSoftmax, kTagAttnExactPv, kTagAddNormQuant, kTagAddNormQuantRow, kTagQkvPost, kTagGluQuant,
    kTagArgmax1, kTagArgmax2, kTagDequant, kTagActQuant, kTagActStage, kTagTpGather, kTagTpGatherLl, kTagOther,
    kTagStep,  // the persistent decode step's phase marks: aux = mark | layer << 8
    kTagStepIssue,  // its producer, per ring entry: t0 before the slot wait, t1 after the copy is issued
    kTagStepUse,    // its compute warps, per ring entry: t0 before the stage wait, t1 when the data is there
};

struct TraceRec {
    unsigned long long grid, t0, t1;
    uint32_t tag, aux, cta, pad;  // pad: odd (1) = an instant mark; even = a CTA span, SM cycles x 2
};
static_assert(sizeof(TraceRec) == 40, "trace record layout");

// Registers a translation unit's binder (capi.cu keeps the list).
int trace_register(void (*bind)(TraceRec*, unsigned*, unsigned));

}  // namespace gncx

#ifdef GNCX_TRACE
namespace gncx {
namespace {
__device__ TraceRec* g_trace_rec = nullptr;
__device__ unsigned* g_trace_n = nullptr;
__device__ unsigned g_trace_cap = 0;

__device__ __forceinline__ unsigned long long trace_clock() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

constexpr int kTraceMarks = 32;  // instant marks a CTA keeps in shared memory until it leaves

__device__ __forceinline__ TraceRec* trace_marks() {
    __shared__ TraceRec marks[kTraceMarks];
    return marks;
}
__device__ __forceinline__ unsigned* trace_mark_count() {
    __shared__ unsigned count;
    return &count;
}

__device__ __forceinline__ void trace_fill(TraceRec& r, uint32_t tag, uint32_t aux, unsigned long long t0,
                                           unsigned long long t1, uint32_t kind) {
    unsigned long long grid;
    asm volatile("mov.u64 %0, %%gridid;" : "=l"(grid));
    r.grid = grid;
    r.t0 = t0;
    r.t1 = t1;
    r.tag = tag;
    r.aux = aux;
    r.cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    r.pad = kind;
}

// Constructed by every thread at kernel entry (the first statement); thread 0
// flushes the CTA's span record and its instant marks when it leaves.
struct TraceScope {
    unsigned long long t0;
    long long c0;  // SM cycles at entry: the span record's pad carries the cycles spent
    uint32_t tag, aux;
    __device__ TraceScope(uint32_t tg, uint32_t ax) : tag(tg), aux(ax) {
        t0 = trace_clock();
        c0 = clock64();
        if (threadIdx.x == 0) *trace_mark_count() = 0;
        __syncthreads();
    }
    __device__ ~TraceScope() {
        if (threadIdx.x != 0 || !g_trace_rec) return;
        const unsigned long long t1 = trace_clock();
        const long long c1 = clock64();
        const unsigned nm = min(*(volatile unsigned*)trace_mark_count(), (unsigned)kTraceMarks);
        const unsigned i = atomicAdd(g_trace_n, 1u + nm);
        if (i + nm >= g_trace_cap) return;
        trace_fill(g_trace_rec[i], tag, aux, t0, t1, 0);
        g_trace_rec[i].pad = (uint32_t)((c1 - c0) << 1);  // even: a span (cycles x 2); marks carry 1
        for (unsigned k = 0; k < nm; ++k) g_trace_rec[i + 1 + k] = trace_marks()[k];
    }
};

// One instant record (t0 == t1) from the calling thread, e.g. a phase boundary
// inside a kernel; `tag` distinguishes the phase.  Kept in shared memory (no
// global round trip on the measured path) and written out with the CTA's span.
__device__ __forceinline__ void trace_mark(uint32_t tag, uint32_t aux) {
    const unsigned long long t = trace_clock();
    const unsigned k = atomicAdd_block(trace_mark_count(), 1u);
    if (k < kTraceMarks) trace_fill(trace_marks()[k], tag, aux, t, t, 1);
}

void trace_bind_tu(TraceRec* rec, unsigned* n, unsigned cap) {
    cudaMemcpyToSymbol(g_trace_rec, &rec, sizeof(rec));
    cudaMemcpyToSymbol(g_trace_n, &n, sizeof(n));
    cudaMemcpyToSymbol(g_trace_cap, &cap, sizeof(cap));
}
const int g_trace_registered = trace_register(&trace_bind_tu);
}  // namespace
}  // namespace gncx
#define GNCX_TRACE_SCOPE(tag, aux) ::gncx::TraceScope _gncx_trace_scope((tag), (uint32_t)(aux))
#define GNCX_TRACE_MARK(tag, aux) ::gncx::trace_mark((tag), (uint32_t)(aux))
#else
#define GNCX_TRACE_MARK(tag, aux) \
    do {                         \
    } while (0)
#define GNCX_TRACE_SCOPE(tag, aux) \
    do {                          \
    } while (0)
#endif
