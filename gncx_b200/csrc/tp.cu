// tp.cu -- tensor-parallel exchange between the GPUs of one NVLink/NVSwitch box.
//
// The decoder is split Megatron-style with every output element computed whole
// on one GPU (weights split by output rows), so after each split GEMV or
// attention the ranks all-gather the pieces of one fp32 vector.  The all-gather is this
// file's own kernel over peer memory: each rank owns one exchange region
// (cudaMalloc, shared with the other processes through CUDA IPC handles); a
// rank writes its slice straight into every peer's region with NVLink stores,
// then publishes an epoch number in each peer's control words, then waits
// (bounded) for every peer's epoch in its own.
//
// Why no buffer is overwritten while a peer still reads it: the exchange
// points of a step alternate between buffers, and a rank can only write the
// next use of a buffer into a peer after it has seen that peer's epoch for a
// later exchange, which the peer publishes after the kernels that read the
// buffer have finished (stream order).
#include <cuda_runtime.h>
#include <string.h>

#include "kernels.h"
#include "trace.cuh"
#include "launch.cuh"
#include "tma.cuh"

namespace gncx {

namespace {

constexpr int kTpThreads = 256;
constexpr unsigned long long kTpWaitNs = 2000000000ull;  // 2 s: a peer that never arrives is an error

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

struct GatherArgs {
    uint8_t* region[kTpMaxRanks];  // every rank's exchange region as mapped in this process
    int rank, size;
    size_t buf;                    // byte offset of the gathered buffer within a region
    int rows, row_floats;          // rows x row_floats floats
    int off, len;                  // this rank's slice of every row
    int32_t* err;
};

// CTA c copies its share of this rank's slice into every peer, then tells
// each peer "CTA c of rank r is done" (flags[r][c] = its epoch) and waits
// until CTA c of every peer has told it the same.  Every rank launches the
// same grid for the same gather, so when all CTAs are through, every peer's
// slice has landed here.  No cross-CTA counter, one system fence per CTA.
__global__ void __launch_bounds__(kTpThreads) tp_gather_kernel(const GatherArgs a) {
    GNCX_TRACE_SCOPE(kTagTpGather, a.rows);
    pdl_launch_dependents();  // the next kernel may start streaming its weights
    pdl_wait();               // the slice comes from the preceding kernel
    const float* src = reinterpret_cast<const float*>(a.region[a.rank] + a.buf);
    const bool vec = ((a.off | a.len | a.row_floats) & 3) == 0;
    const int per_row = vec ? a.len >> 2 : a.len;
    const size_t items = (size_t)a.rows * per_row;
    const size_t per_cta = (items + gridDim.x - 1) / gridDim.x;
    const size_t i0 = (size_t)blockIdx.x * per_cta;
    const size_t i1 = i0 + per_cta < items ? i0 + per_cta : items;
    for (size_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
        const size_t r = i / per_row, c = i - r * per_row;
        if (vec) {
            const size_t o = r * a.row_floats + a.off + 4 * c;
            const float4 v = *reinterpret_cast<const float4*>(src + o);
            for (int q = 0; q < a.size; ++q)
                if (q != a.rank) *reinterpret_cast<float4*>(reinterpret_cast<float*>(a.region[q] + a.buf) + o) = v;
        } else {
            const size_t o = r * a.row_floats + a.off + c;
            const float v = src[o];
            for (int q = 0; q < a.size; ++q)
                if (q != a.rank) reinterpret_cast<float*>(a.region[q] + a.buf)[o] = v;
        }
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    __threadfence_system();  // the CTA's peer stores (ordered before by the barrier) before its flags
    uint32_t* ctl = reinterpret_cast<uint32_t*>(a.region[a.rank]);
    const int cta = blockIdx.x;
    const uint32_t ep = ctl[kTpEpochs + cta] + 1u;
    ctl[kTpEpochs + cta] = ep;
    for (int q = 0; q < a.size; ++q)
        if (q != a.rank) st_release_sys(reinterpret_cast<uint32_t*>(a.region[q]) + a.rank * kTpMaxCtas + cta, ep);
    if (*(volatile int32_t*)a.err != 0) return;  // a rank already gave up: do not wait again
    const unsigned long long t0 = global_ns();
    for (int q = 0; q < a.size; ++q) {
        if (q == a.rank) continue;
        const uint32_t* f = ctl + q * kTpMaxCtas + cta;
        while ((int32_t)(ld_acquire_sys(f) - ep) < 0) {
            if (global_ns() - t0 > kTpWaitNs) {
                record_error(a.err, kErrTimeout);
                return;
            }
        }
    }
}

struct LlArgs {
    uint8_t* region[kTpMaxRanks];
    int rank, size, slot;
    size_t buf, ll;  // byte offsets (data area) of the gathered row and of the staging area
    int row_floats;
    TpSlices sl;
    int32_t* err;
};

__global__ void __launch_bounds__(kTpThreads) tp_ll_gather_kernel(const LlArgs a) {
    GNCX_TRACE_SCOPE(kTagTpGatherLl, a.row_floats);
    pdl_launch_dependents();
    pdl_wait();  // this rank's slice comes from the preceding kernel
    __shared__ uint32_t s_ep;
    uint32_t* ctl = reinterpret_cast<uint32_t*>(a.region[a.rank]);
    if (threadIdx.x == 0) {
        // every CTA of every launch of this slot counts the same launches, so
        // the epochs agree across CTAs and ranks
        uint32_t* e = ctl + kTpLlEpochs + a.slot * kTpMaxCtas + blockIdx.x;
        s_ep = *e + 1u;
        *e = s_ep;
    }
    __syncthreads();
    const uint32_t ep = s_ep;
    const int gid = blockIdx.x * blockDim.x + threadIdx.x, stride = gridDim.x * blockDim.x;
    float* row = reinterpret_cast<float*>(a.region[a.rank] + kTpCtlBytes + a.buf);
    // send: {value, epoch} words into every peer's staging row of this rank
    const int o_me = a.sl.off[a.rank], n_me = a.sl.len[a.rank];
    for (int i = gid; i < n_me; i += stride) {
        const uint64_t w = ((uint64_t)ep << 32) | __float_as_uint(row[o_me + i]);
        for (int q = 0; q < a.size; ++q) {
            if (q == a.rank) continue;
            uint64_t* dst = reinterpret_cast<uint64_t*>(a.region[q] + kTpCtlBytes + a.ll) +
                            (size_t)a.rank * a.row_floats + o_me + i;
            asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(dst), "l"(w) : "memory");
        }
    }
    if (threadIdx.x == 0) GNCX_TRACE_MARK(50, 0);  // sends issued
    // receive: poll this rank's staging rows until each peer value carries the epoch
    if (*(volatile int32_t*)a.err != 0) return;  // a rank already gave up: do not wait again
    const unsigned long long t0 = global_ns();
    const uint64_t* st = reinterpret_cast<const uint64_t*>(a.region[a.rank] + kTpCtlBytes + a.ll);
    for (int q = 0; q < a.size; ++q) {
        if (q == a.rank) continue;
        const int o = a.sl.off[q], n = a.sl.len[q];
        for (int j = gid; j < n; j += stride) {
            const uint64_t* p = st + (size_t)q * a.row_floats + o + j;
            uint64_t w;
            for (;;) {
                asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
                if ((uint32_t)(w >> 32) == ep) break;
                if (global_ns() - t0 > kTpWaitNs) {
                    record_error(a.err, kErrTimeout);
                    return;
                }
            }
            row[o + j] = __uint_as_float((uint32_t)w);
        }
    }
    if (threadIdx.x == 0) GNCX_TRACE_MARK(51, 0);  // every peer value of this thread's share arrived
}

// ---- the greedy step over a split vocabulary ----
constexpr int kAmSlot = kTpLlSlots - 1;  // epoch slot of the (value, id) swap
struct AmArgs {
    uint8_t* region[kTpMaxRanks];
    int rank, size;
    size_t stage;  // data-area byte offset of size x 16-byte entries {word0: id | epoch << 32, word1: value}
    const double* part_v;
    const int* part_i;
    int n;
    DecodeState* st;
    int32_t* out_ids;
    int advance_pos;
    int32_t* err;
};

__device__ __forceinline__ bool am_better(double v, int i, double bv, int bi) {
    return v > bv || (v == bv && i < bi);  // the first maximum wins (lua/gncx_streamer.lua:1229-1273)
}

__global__ void __launch_bounds__(kTpThreads) tp_argmax_state_kernel(const AmArgs a) {
    GNCX_TRACE_SCOPE(kTagArgmax2, a.n);
    pdl_launch_dependents();
    pdl_wait();  // the partial maxima come from the preceding kernel
    __shared__ double sv[kTpThreads / 32];
    __shared__ int si[kTpThreads / 32];
    double bv = -1e30;
    int bi = 0;
    for (int k = threadIdx.x; k < a.n; k += blockDim.x)
        if (am_better(a.part_v[k], a.part_i[k], bv, bi)) { bv = a.part_v[k]; bi = a.part_i[k]; }
    for (int o = 16; o > 0; o >>= 1) {
        const double v = __shfl_xor_sync(0xffffffffu, bv, o);
        const int i = __shfl_xor_sync(0xffffffffu, bi, o);
        if (am_better(v, i, bv, bi)) { bv = v; bi = i; }
    }
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x != 0) return;
    for (int k = 1; k < kTpThreads / 32; ++k)
        if (am_better(sv[k], si[k], bv, bi)) { bv = sv[k]; bi = si[k]; }
    // swap: the value first, a system fence, then the (id, epoch) word the peers poll
    uint32_t* ctl = reinterpret_cast<uint32_t*>(a.region[a.rank]);
    uint32_t* epw = ctl + kTpLlEpochs + kAmSlot * kTpMaxCtas;
    const uint32_t ep = *epw + 1u;
    *epw = ep;
    for (int q = 0; q < a.size; ++q) {
        if (q == a.rank) continue;
        uint64_t* dst = reinterpret_cast<uint64_t*>(a.region[q] + kTpCtlBytes + a.stage) + 2 * a.rank;
        asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(dst + 1), "l"((uint64_t)__double_as_longlong(bv))
                     : "memory");
    }
    __threadfence_system();
    for (int q = 0; q < a.size; ++q) {
        if (q == a.rank) continue;
        uint64_t* dst = reinterpret_cast<uint64_t*>(a.region[q] + kTpCtlBytes + a.stage) + 2 * a.rank;
        const uint64_t w0 = ((uint64_t)ep << 32) | (uint32_t)bi;
        asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(dst), "l"(w0) : "memory");
    }
    if (*(volatile int32_t*)a.err != 0) return;  // a rank already gave up: do not wait again
    const unsigned long long t0 = global_ns();
    const uint64_t* mine = reinterpret_cast<const uint64_t*>(a.region[a.rank] + kTpCtlBytes + a.stage);
    for (int q = 0; q < a.size; ++q) {
        if (q == a.rank) continue;
        uint64_t w0;
        for (;;) {
            asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(w0) : "l"(mine + 2 * q) : "memory");
            if ((uint32_t)(w0 >> 32) == ep) break;
            if (global_ns() - t0 > kTpWaitNs) {
                record_error(a.err, kErrTimeout);
                return;
            }
        }
        uint64_t w1;
        asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(w1) : "l"(mine + 2 * q + 1) : "memory");
        const double v = __longlong_as_double((long long)w1);
        const int i = (int)(uint32_t)w0;
        if (am_better(v, i, bv, bi)) { bv = v; bi = i; }
    }
    // the decode state update of argmax_state_launch (generate, :1276-1311)
    DecodeState* st = a.st;
    if (!st->done) {
        const int next = bi;
        if (next == st->eos) {
            st->done = 1;
        } else {
            if (st->n_out < st->max_out) a.out_ids[st->n_out] = next;
            st->n_out += 1;
            st->ring[st->n_all % kRecentWindow] = next;
            st->n_all += 1;
            st->token = next;
            if (a.advance_pos) st->pos += 1;
            if (st->n_out >= st->max_out) st->done = 1;
        }
    }
}

}  // namespace

int tp_argmax_state_launch(const TpComm& c, size_t stage, const void* scratch, int32_t n_parts, DecodeState* st,
                           int32_t* out_ids, int advance_pos, int32_t* err, cudaStream_t s) {
    if (!c.connected || !scratch || !st || !out_ids || !err || n_parts <= 0 || n_parts > kArgmaxParts || (stage & 15))
        return kErrInvalidArg;
    AmArgs a{};
    for (int q = 0; q < kTpMaxRanks; ++q) a.region[q] = c.region[q];
    a.rank = c.rank;
    a.size = c.size;
    a.stage = stage;
    a.part_v = reinterpret_cast<const double*>(scratch);
    a.part_i = reinterpret_cast<const int*>(a.part_v + kArgmaxParts);
    a.n = n_parts;
    a.st = st;
    a.out_ids = out_ids;
    a.advance_pos = advance_pos;
    a.err = err;
    return launch_k(tp_argmax_state_kernel, dim3(1), dim3(kTpThreads), 0, s, a) == cudaSuccess ? kOk : kErrCuda;
}

int tp_gather_ll_launch(const TpComm& c, size_t buf, size_t ll, int32_t row_floats, const TpSlices& sl, int32_t slot,
                        int32_t* err, cudaStream_t st) {
    if (c.size == 1) return kOk;
    if (!c.connected || !err || slot < 0 || slot >= kTpLlSlots || row_floats <= 0) return kErrInvalidArg;
    int most = 0;
    for (int q = 0; q < c.size; ++q) {
        if (sl.off[q] < 0 || sl.len[q] < 0 || sl.off[q] + sl.len[q] > row_floats) return kErrInvalidArg;
        most = sl.len[q] > most ? sl.len[q] : most;
    }
    LlArgs a{};
    for (int q = 0; q < kTpMaxRanks; ++q) a.region[q] = c.region[q];
    a.rank = c.rank;
    a.size = c.size;
    a.slot = slot;
    a.buf = buf;
    a.ll = ll;
    a.row_floats = row_floats;
    a.sl = sl;
    a.err = err;
    // one thread per 4 values of the largest slice (a fixed grid per slot shape)
    int blocks = (most + 4 * kTpThreads - 1) / (4 * kTpThreads);
    if (blocks > kTpMaxCtas) blocks = kTpMaxCtas;
    if (blocks < 1) blocks = 1;
    return launch_k(tp_ll_gather_kernel, dim3(blocks), dim3(kTpThreads), 0, st, a) == cudaSuccess ? kOk : kErrCuda;
}

int tp_alloc(TpComm& c, int rank, int size, size_t bytes) {
    if (size < 1 || size > kTpMaxRanks || rank < 0 || rank >= size) return kErrInvalidArg;
    c.rank = rank;
    c.size = size;
    c.bytes = (bytes + kTpCtlBytes + 255) & ~(size_t)255;
    if (cudaMalloc(&c.local, c.bytes) != cudaSuccess) {
        cudaGetLastError();
        c.local = nullptr;
        return kErrOutOfMemory;
    }
    if (cudaMemset(c.local, 0, c.bytes) != cudaSuccess) return kErrCuda;
    // layout words, checked by every peer before it writes into this region
    const uint32_t info[5] = {kTpMagic, (uint32_t)c.bytes, (uint32_t)((uint64_t)c.bytes >> 32), (uint32_t)rank,
                              (uint32_t)size};
    if (cudaMemcpy(reinterpret_cast<uint32_t*>(c.local) + kTpInfo, info, sizeof(info), cudaMemcpyHostToDevice) !=
            cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess)
        return kErrCuda;
    for (auto& p : c.region) p = nullptr;
    c.region[rank] = c.local;
    c.connected = size == 1;
    return kOk;
}

int tp_handle(const TpComm& c, void* out) {
    if (!c.local || !out) return kErrInvalidArg;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, c.local) != cudaSuccess) return kErrCuda;
    static_assert(sizeof(h) == kTpHandleBytes, "IPC handle size");
    memcpy(out, &h, sizeof(h));
    return kOk;
}

int tp_connect(TpComm& c, const void* handles) {
    if (!c.local || !handles) return kErrInvalidArg;
    if (c.connected) return kOk;
    for (int q = 0; q < c.size; ++q) {
        if (q == c.rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)q * kTpHandleBytes, sizeof(h));
        void* p = nullptr;
        if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            return kErrCuda;
        }
        c.region[q] = static_cast<uint8_t*>(p);
        // The peer's region must have this region's size and belong to rank q
        // of the same group: the gather writes at this region's offsets.
        uint32_t info[5] = {};
        if (cudaMemcpy(info, static_cast<uint32_t*>(p) + kTpInfo, sizeof(info), cudaMemcpyDeviceToHost) !=
            cudaSuccess)
            return kErrCuda;
        const uint64_t bytes = (uint64_t)info[1] | ((uint64_t)info[2] << 32);
        if (info[0] != kTpMagic || bytes != c.bytes || info[3] != (uint32_t)q || info[4] != (uint32_t)c.size)
            return kErrInvalidArg;
    }
    c.connected = true;
    return kOk;
}

void tp_free(TpComm& c) {
    for (int q = 0; q < kTpMaxRanks; ++q)
        if (q != c.rank && c.region[q]) cudaIpcCloseMemHandle(c.region[q]);
    if (c.local) cudaFree(c.local);
    c = TpComm{};
}

int tp_gather_launch(const TpComm& c, size_t buf, int32_t rows, int32_t row_floats, int32_t off, int32_t len,
                     int32_t* err, cudaStream_t st) {
    if (c.size == 1) return kOk;
    if (!c.connected || rows < 0 || off < 0 || len < 0 || off + len > row_floats || !err) return kErrInvalidArg;
    if (rows == 0) return kOk;
    GatherArgs a{};
    for (int q = 0; q < kTpMaxRanks; ++q) a.region[q] = c.region[q];
    a.rank = c.rank;
    a.size = c.size;
    a.buf = buf + kTpCtlBytes;
    a.rows = rows;
    a.row_floats = row_floats;
    a.off = off;
    a.len = len;
    a.err = err;
    // one CTA per 1024 float4 (each thread moves 4), at most kTpMaxCtas
    const size_t items = (size_t)rows * ((len + 3) / 4);
    size_t blocks = (items + 4 * kTpThreads - 1) / (4 * kTpThreads);
    if (blocks > (size_t)kTpMaxCtas) blocks = kTpMaxCtas;
    if (blocks < 1) blocks = 1;
    return launch_k(tp_gather_kernel, dim3((unsigned)blocks), dim3(kTpThreads), 0, st, a) == cudaSuccess ? kOk
                                                                                                        : kErrCuda;
}

}  // namespace gncx
