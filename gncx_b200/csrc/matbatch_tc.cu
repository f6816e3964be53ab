// matbatch_tc.cu -- prefill GEMM (gncx_xfold_universal_matbatch,
// csrc/gncx_llm_kernels.cpp:1495-1692) on the 5th-generation tensor cores.
//
// The reference's integer block dots are exact in any order, but it applies
// fp32 scales per 32-input block and adds the block terms to each
// (token, row) accumulator serially.  So the tensor cores produce one int32
// dot per (row, token, block) -- `tcgen05.mma kind::i8` with K = 32, each
// block into a fresh TMEM accumulator -- and CUDA cores finish every term
// with the reference's fp32 rounding order (the same formulas as the CUDA-core
// path in matbatch.cu, so results are bit-identical to it and to the
// reference).
//
// CTA tile: 128 weight rows (TMEM lanes) x 32 tokens (TMEM columns), the
// whole reduction dimension streamed one 256-input unit at a time:
//   * loader warps (4): each thread unpacks one row's unit (nibbles / int8
//     quants) into int8 K-major core matrices (8 rows x 16 bytes) and its
//     per-block scales; they also stage the tokens' int8 quants and scales;
//   * MMA warp: one thread issues the 8 block MMAs of a unit into one half of
//     TMEM (8 x 32 columns) and commits them to mbarriers;
//   * epilogue warps (8): warp w reads TMEM lanes 32(w%4).. (its rows) and
//     16 of the 32 token columns, one block at a time, and accumulates the
//     block terms.  The independent products of two tokens go through one
//     packed `mul.rn.f32x2`; every sum stays a scalar __fadd_rn / __fsub_rn
//     (a packed product feeding a packed sum may be fused into an FMA, which
//     would not round like the reference).
// The operand tiles (A, B) sit in a two-stage ring the MMA releases as soon
// as it has read them; the scales sit in a separate four-stage ring the
// epilogue releases, so the loaders run up to three units ahead of the
// epilogue.  The loaders fetch the next unit's weight bytes while unpacking
// the current one and copy token quants with cp.async.  Units alternate
// between the two TMEM halves, so the tensor cores, the loaders and the
// epilogue overlap.  Every wait is bounded; on a timeout the kernel records an
// error, skips the remaining work and still releases TMEM.
#include <cuda_runtime.h>
#include "act.cuh"
#include "common.cuh"
#include "kernels.h"
#include "trace.cuh"
#include "tma.cuh"
#include "units.cuh"

namespace gncx {

constexpr int kTcM = 128;        // weight rows per tile
constexpr int kTcN = 32;         // tokens per tile
constexpr int kTcCols = 512;     // TMEM columns: 2 halves x 8 blocks x kTcN
constexpr int kTcEpiWarps = 8;   // two per TMEM lane quadrant, 16 tokens each
constexpr int kTcLoadWarps = 4;
constexpr int kTcThreads = (kTcEpiWarps + kTcLoadWarps + 1) * 32;
constexpr int kTcMmaWarp = kTcEpiWarps + kTcLoadWarps;

// shared memory: operand stages (A + B tiles, free once the unit's MMAs have
// read them) and scale stages (per-block weight and token scales, free once
// the epilogue has applied them) in separate rings, so the loaders can run
// kTcScaleStages - 1 units ahead of the epilogue
constexpr int kTcA = 16 * 16 * 128;     // 16 K-chunks x 16 row groups x (8 rows x 16 B)
constexpr int kTcB = 16 * 4 * 128;      // 16 K-chunks x 4 token groups x (8 tokens x 16 B)
constexpr int kTcWS = 8 * kTcM * 8;     // per block, per row: float2
constexpr int kTcAS = 8 * kTcN * 8;     // per block and token {d_a, sum q}, token pairs side by side
constexpr int kTcOpStage = kTcA + kTcB;
constexpr int kTcScStage = kTcWS + kTcAS;
constexpr int kTcOpStages = 2;
constexpr int kTcScaleStages = 4;
constexpr int kTcSmem = kTcOpStages * kTcOpStage + kTcScaleStages * kTcScStage + 256;
// More than half of an SM's shared memory, so one CTA per SM owns all of TMEM.
constexpr int kTcSmemAlloc = kTcSmem > 120 * 1024 ? kTcSmem : 120 * 1024;

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    // K-major, no swizzle: core matrices of 8 rows x 16 bytes; lbo = bytes
    // between the two K core matrices of a K=32 slice, sbo = bytes between
    // 8-row groups; version 1 (sm_100).
    uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    return d;
}

// kind::i8: s32 accumulate, signed A and B, both K-major, N = kTcN, M = kTcM.
constexpr uint32_t kTcIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTcN >> 3) << 17) |
                              ((uint32_t)(kTcM >> 4) << 24);

__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t da, uint64_t db) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(kTcIdesc), "r"(0));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 32 consecutive TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, int (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Byte offset of (row or token r, 16-byte K-chunk kc) in an operand tile whose
// 8-row groups are 128 bytes apart and whose K-chunks are `kstride` apart.
__device__ __forceinline__ int tile_off(int r, int kc, int kstride) { return kc * kstride + (r >> 3) * 128 + (r & 7) * 16; }

// Unpack one weight row's unit into 16 int8 K-chunks (input order) and its
// block scales.  q: the unit's bytes as words (16-byte aligned source).
template <int T>
__device__ __forceinline__ void tc_unpack(const uint32_t* q, uint8_t* a_tile, int r, float2* ws) {
    if constexpr (T == kQ4_K) {
        const float d = half_bits_to_float(q[0]), dmin = half_bits_to_float(q[0] >> 16);
        const uint32_t* sc = q + 1;
        int s[8], m[8];
        k4_scale_min<0>(sc, s[0], m[0]); k4_scale_min<1>(sc, s[1], m[1]);
        k4_scale_min<2>(sc, s[2], m[2]); k4_scale_min<3>(sc, s[3], m[3]);
        k4_scale_min<4>(sc, s[4], m[4]); k4_scale_min<5>(sc, s[5], m[5]);
        k4_scale_min<6>(sc, s[6], m[6]); k4_scale_min<7>(sc, s[7], m[7]);
#pragma unroll
        for (int j = 0; j < 8; ++j) ws[j * kTcM + r] = make_float2(fmul(d, i2f(s[j])), fmul(dmin, i2f(m[j])));
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint32_t* w = q + 4 + 8 * c;  // qs[32c .. 32c+31]
#pragma unroll
            for (int h = 0; h < 2; ++h) {       // qs[32c + 16h .. +15]
                const uint32_t w0 = w[4 * h], w1 = w[4 * h + 1], w2 = w[4 * h + 2], w3 = w[4 * h + 3];
                *reinterpret_cast<uint4*>(a_tile + tile_off(r, 4 * c + h, 2048)) =
                    make_uint4(w0 & kLo4, w1 & kLo4, w2 & kLo4, w3 & kLo4);
                *reinterpret_cast<uint4*>(a_tile + tile_off(r, 4 * c + 2 + h, 2048)) =
                    make_uint4((w0 >> 4) & kLo4, (w1 >> 4) & kLo4, (w2 >> 4) & kLo4, (w3 >> 4) & kLo4);
            }
        }
    } else if constexpr (T == kQ4_0) {
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            const int o = 18 * b;  // byte offset of block b in the unit
            auto wat = [&](int off) {  // 4 bytes at byte offset off
                const int wi = off >> 2, sh = (off & 3) * 8;
                return sh ? __funnelshift_r(q[wi], q[wi + 1], sh) : q[wi];
            };
            const uint32_t hb = wat(o);
            ws[b * kTcM + r] = make_float2(half_bits_to_float(hb & 0xFFFFu), 0.0f);
            const uint32_t w0 = wat(o + 2), w1 = wat(o + 6), w2 = wat(o + 10), w3 = wat(o + 14);
            *reinterpret_cast<uint4*>(a_tile + tile_off(r, 2 * b, 2048)) =
                make_uint4(w0 & kLo4, w1 & kLo4, w2 & kLo4, w3 & kLo4);
            *reinterpret_cast<uint4*>(a_tile + tile_off(r, 2 * b + 1, 2048)) =
                make_uint4((w0 >> 4) & kLo4, (w1 >> 4) & kLo4, (w2 >> 4) & kLo4, (w3 >> 4) & kLo4);
        }
    } else {  // kQ8_0
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            const int o = 34 * b;
            auto wat = [&](int off) {
                const int wi = off >> 2, sh = (off & 3) * 8;
                return sh ? __funnelshift_r(q[wi], q[wi + 1], sh) : q[wi];
            };
            ws[b * kTcM + r] = make_float2(half_bits_to_float(wat(o) & 0xFFFFu), 0.0f);
            *reinterpret_cast<uint4*>(a_tile + tile_off(r, 2 * b, 2048)) =
                make_uint4(wat(o + 2), wat(o + 6), wat(o + 10), wat(o + 14));
            *reinterpret_cast<uint4*>(a_tile + tile_off(r, 2 * b + 1, 2048)) =
                make_uint4(wat(o + 18), wat(o + 22), wat(o + 26), wat(o + 30));
        }
    }
}

template <int T> struct TcFmt;
template <> struct TcFmt<kQ4_0> { static constexpr int UB = 144; };
template <> struct TcFmt<kQ8_0> { static constexpr int UB = 272; };
template <> struct TcFmt<kQ4_K> { static constexpr int UB = 144; };

__device__ __forceinline__ void cp_async16_tc(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}

// 16 consecutive TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}

// Two fp32 values as one packed operand, and back.
__device__ __forceinline__ unsigned long long pk2(float a, float b) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void upk2(unsigned long long v, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
// Two independent IEEE round-to-nearest products in one instruction.  Only
// products go through the packed form: a packed product feeding a packed add
// or subtract may be fused into a packed FMA by the backend (measured: the
// all-packed epilogue differed from the scalar one in 64 % of outputs, the
// packed-product form in none), so every sum stays a scalar __fadd_rn /
// __fsub_rn, which is never contracted.
__device__ __forceinline__ unsigned long long mul2_rn(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm volatile("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

template <int T>
__global__ void __launch_bounds__(kTcThreads, 1) matbatch_tc_kernel(const uint8_t* __restrict__ w, size_t rb,
                                                                    const ActBlock* __restrict__ act, int batch,
                                                                    int in_dim, int out_dim, float* __restrict__ y,
                                                                    int ldy, int32_t* err) {
    GNCX_TRACE_SCOPE(kTagMatbatchTc, out_dim);
    constexpr int UB = TcFmt<T>::UB;
    constexpr int NQ = UB / 16;           // 16-byte pieces of a row's unit
    constexpr int NE = kTcEpiWarps * 32;  // epilogue threads
    constexpr int NL = kTcLoadWarps * 32; // loader threads
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* sc_base = smem + kTcOpStages * kTcOpStage;
    uint64_t* full = reinterpret_cast<uint64_t*>(sc_base + kTcScaleStages * kTcScStage);  // operands loaded
    uint64_t* empty = full + kTcOpStages;       // operands consumed by the MMAs
    uint64_t* sfull = empty + kTcOpStages;      // scales written
    uint64_t* sempty = sfull + kTcScaleStages;  // scales applied by the epilogue
    uint64_t* accf = sempty + kTcScaleStages;
    uint64_t* acce = accf + 2;
    uint64_t* done = acce + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    __shared__ int abort_flag;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tok0 = blockIdx.x * kTcN;  // token tiles vary fastest: CTAs that share a weight tile run together
    const int row0 = blockIdx.y * kTcM;
    const int upr = in_dim >> 8, nb = in_dim >> 5;

    if (tid == 0) {
        for (int i = 0; i < kTcOpStages; ++i) {
            mbar_init(&full[i], NL);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < kTcScaleStages; ++i) {
            mbar_init(&sfull[i], NL);
            mbar_init(&sempty[i], NE);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&accf[i], 1);
            mbar_init(&acce[i], NE);
        }
        mbar_init(done, 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == kTcMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTcCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto stage_a = [&](int s) { return smem + s * kTcOpStage; };
    auto stage_b = [&](int s) { return smem + s * kTcOpStage + kTcA; };
    auto stage_ws = [&](int q) { return reinterpret_cast<float2*>(sc_base + q * kTcScStage); };
    auto stage_as = [&](int q) { return sc_base + q * kTcScStage + kTcWS; };
    auto fail = [&]() {
        record_error(err, kErrTimeout);
        atomicExch(&abort_flag, 1);
    };

    if (warp >= kTcEpiWarps && warp < kTcMmaWarp) {
        // ---------------- loaders: thread r owns weight row r of the tile ----------------
        const int r = tid - NE;
        const int grow = row0 + r;
        const bool row_ok = grow < out_dim;
        const uint4* wrow = reinterpret_cast<const uint4*>(w + (size_t)(row_ok ? grow : 0) * rb);
        uint32_t q[4 * NQ + 1];
        auto fetch = [&](int u) {  // the next unit's raw bytes, in flight while this one is unpacked
#pragma unroll
            for (int i = 0; i < NQ; ++i) {
                const uint4 v = row_ok ? __ldg(wrow + (size_t)u * NQ + i) : make_uint4(0, 0, 0, 0);
                q[4 * i] = v.x; q[4 * i + 1] = v.y; q[4 * i + 2] = v.z; q[4 * i + 3] = v.w;
            }
            q[4 * NQ] = 0u;
        };
        fetch(0);
        for (int u = 0; u < upr; ++u) {
            const int s = u & (kTcOpStages - 1);                     // operand stage
            const int ss = u & (kTcScaleStages - 1);                 // scale stage
            if (u >= kTcOpStages && !mbar_wait(&empty[s], ((u / kTcOpStages) - 1) & 1)) fail();
            if (u >= kTcScaleStages && !mbar_wait(&sempty[ss], ((u / kTcScaleStages) - 1) & 1)) fail();
            if (*(volatile int*)&abort_flag) break;
            // tokens' quants straight into the B tile (asynchronous), then their scalars
            uint8_t* bt = stage_b(s);
            for (int p = r; p < kTcN * 16; p += NL) {
                const int t = p >> 4, kc = p & 15;
                const int tok = tok0 + t;
                uint8_t* dst = bt + tile_off(t, kc, 512);
                if (tok < batch)
                    cp_async16_tc(dst, reinterpret_cast<const uint8_t*>(act + (size_t)tok * nb + u * 8 + (kc >> 1)) +
                                           16 + 16 * (kc & 1));
                else
                    *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
            uint4 hdr[(kTcN * 8 + NL - 1) / NL];
#pragma unroll
            for (int k = 0; k < (kTcN * 8 + NL - 1) / NL; ++k) {
                const int p = r + k * NL;
                const int b = p / kTcN, t = p % kTcN;
                hdr[k] = (p < kTcN * 8 && tok0 + t < batch)
                             ? *reinterpret_cast<const uint4*>(act + (size_t)(tok0 + t) * nb + u * 8 + b)
                             : make_uint4(0, 0, 0, 0);
            }
            constexpr bool kAhead = NQ <= 9;  // a second copy of a Q8_0 unit does not fit in registers
            uint32_t cur[kAhead ? 4 * NQ + 1 : 1];
            if constexpr (kAhead) {
#pragma unroll
                for (int i = 0; i < 4 * NQ + 1; ++i) cur[i] = q[i];
                if (u + 1 < upr) fetch(u + 1);
            }
            if (row_ok) {
                tc_unpack<T>(kAhead ? cur : q, stage_a(s), r, stage_ws(ss));
            } else {
                for (int kc = 0; kc < 16; ++kc)
                    *reinterpret_cast<uint4*>(stage_a(s) + tile_off(r, kc, 2048)) = make_uint4(0, 0, 0, 0);
                for (int j = 0; j < 8; ++j) stage_ws(ss)[j * kTcM + r] = make_float2(0.0f, 0.0f);
            }
            if constexpr (!kAhead) {
                if (u + 1 < upr) fetch(u + 1);
            }
            uint8_t* as = stage_as(ss);
#pragma unroll
            for (int k = 0; k < (kTcN * 8 + NL - 1) / NL; ++k) {
                const int p = r + k * NL;
                if (p < kTcN * 8) {
                    const int b = p / kTcN, t = p % kTcN;
                    const float ad = __uint_as_float(hdr[k].x), sq = i2f((int)hdr[k].y + (int)hdr[k].z);
                    // token pairs side by side for the packed products:
                    // Q4_K, per 64-input chunk and token pair: {d_lo x2, S_lo x2}, {d_hi x2, S_hi x2};
                    // Q4_0 / Q8_0, per block and token pair: {d_a x2, sum q x2}
                    float* af = reinterpret_cast<float*>(as);
                    const int slot = (T == kQ4_K) ? (((b >> 1) * (kTcN / 2) + (t >> 1)) * 8 + (b & 1) * 4)
                                                  : ((b * (kTcN / 2) + (t >> 1)) * 4);
                    af[slot + (t & 1)] = ad;
                    af[slot + 2 + (t & 1)] = sq;
                }
            }
            asm volatile("cp.async.wait_all;" ::: "memory");
            fence_async_smem();  // the tensor cores read these tiles through the async proxy
            mbar_arrive(&full[s]);
            mbar_arrive(&sfull[ss]);
        }
    } else if (warp == kTcMmaWarp) {
        // ---------------- MMA issue (one thread) ----------------
        if (lane == 0) {
            int issued = 0;
            for (int u = 0; u < upr; ++u) {
                const int s = u & (kTcOpStages - 1), hb = u & 1;
                if (!mbar_wait(&full[s], (u / kTcOpStages) & 1)) fail();
                if (u >= 2 && !mbar_wait(&acce[hb], ((u >> 1) - 1) & 1)) fail();
                if (*(volatile int*)&abort_flag) break;
                tc_fence_after();
                const uint32_t a0 = smem_u32(stage_a(s)), b0 = smem_u32(stage_b(s));
#pragma unroll
                for (int kb = 0; kb < 8; ++kb)
                    umma_i8(tmem + (uint32_t)((hb * 8 + kb) * kTcN), umma_desc(a0 + 2 * kb * 2048, 2048, 128),
                            umma_desc(b0 + 2 * kb * 512, 512, 128));
                umma_commit(&accf[hb]);
                umma_commit(&empty[s]);
                ++issued;
            }
            // nothing may still write TMEM when it is released
            if (issued > 0) {
                umma_commit(done);
                if (!mbar_wait(done, 0)) record_error(err, kErrTimeout);
            }
        }
        __syncwarp();
    } else {
        // ---- epilogue: warp w reads TMEM lanes 32*(w%4).. (its rows), tokens 16*(w/4) .. +15 ----
        constexpr int TN = kTcN / (kTcEpiWarps / 4);  // tokens per thread
        const int quad = warp & 3, half = warp >> 2;
        const int r = quad * 32 + lane;
        const int t0 = half * TN;
        const uint32_t tlane = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)t0;
        float acc[TN];
#pragma unroll
        for (int t = 0; t < TN; ++t) acc[t] = 0.0f;
        for (int u = 0; u < upr; ++u) {
            const int q = u & (kTcScaleStages - 1), hb = u & 1;
            // accf: this unit's dots are in TMEM; sfull: its scales are written
            // (the scale stage cannot be refilled before this warp releases it)
            if (!mbar_wait(&accf[hb], (u >> 1) & 1) || !mbar_wait(&sfull[q], (u / kTcScaleStages) & 1)) fail();
            if (*(volatile int*)&abort_flag) break;
            tc_fence_after();
            const float2* ws = stage_ws(q);
            const uint8_t* as = stage_as(q);
            if constexpr (T == kQ4_K) {
                // per 64-input chunk c: st = (0 + lo) + hi, a half skipped when its act scale
                // is 0 (:1546-1618).  Adding such a half instead changes nothing for finite
                // weight scales: it is a zero whose sign the row accumulator (never -0)
                // absorbs, so both halves are always added.
#pragma unroll 1
                for (int c = 0; c < 4; ++c) {
                    int dl[TN], dh[TN];
                    tmem_ld16(tlane + (uint32_t)((hb * 8 + 2 * c) * kTcN), dl);
                    tmem_ld16(tlane + (uint32_t)((hb * 8 + 2 * c + 1) * kTcN), dh);
                    tmem_wait_ld();
                    const float2 w1 = ws[(2 * c) * kTcM + r], w2 = ws[(2 * c + 1) * kTcM + r];
                    const unsigned long long W1X = pk2(w1.x, w1.x), W1Y = pk2(w1.y, w1.y);
                    const unsigned long long W2X = pk2(w2.x, w2.x), W2Y = pk2(w2.y, w2.y);
                    const float4* a4 = reinterpret_cast<const float4*>(as) + (c * (kTcN / 2) + t0 / 2) * 2;
#pragma unroll
                    for (int tp = 0; tp < TN / 2; ++tp) {
                        const float4 L = a4[2 * tp], H = a4[2 * tp + 1];  // {d x2, S x2} of the lo / hi half
                        // lo = d_lo * ((d1 * dot_lo) - (dm1 * S_lo)), hi likewise, for two tokens
                        float p1a, p1b, p2a, p2b, p3a, p3b, p4a, p4b;
                        upk2(mul2_rn(W1X, pk2(i2f(dl[2 * tp]), i2f(dl[2 * tp + 1]))), p1a, p1b);
                        upk2(mul2_rn(W1Y, pk2(L.z, L.w)), p2a, p2b);
                        upk2(mul2_rn(W2X, pk2(i2f(dh[2 * tp]), i2f(dh[2 * tp + 1]))), p3a, p3b);
                        upk2(mul2_rn(W2Y, pk2(H.z, H.w)), p4a, p4b);
                        float loa, lob, hia, hib;
                        upk2(mul2_rn(pk2(L.x, L.y), pk2(fsub(p1a, p2a), fsub(p1b, p2b))), loa, lob);
                        upk2(mul2_rn(pk2(H.x, H.y), pk2(fsub(p3a, p4a), fsub(p3b, p4b))), hia, hib);
                        acc[2 * tp] = fadd(acc[2 * tp], fadd(loa, hia));
                        acc[2 * tp + 1] = fadd(acc[2 * tp + 1], fadd(lob, hib));
                    }
                }
            } else {
#pragma unroll 1
                for (int b = 0; b < 8; ++b) {
                    int dv[TN];
                    tmem_ld16(tlane + (uint32_t)((hb * 8 + b) * kTcN), dv);
                    tmem_wait_ld();
                    const float wd = ws[b * kTcM + r].x;
                    const unsigned long long WD = pk2(wd, wd);
                    const float4* a4 = reinterpret_cast<const float4*>(as) + b * (kTcN / 2) + t0 / 2;
#pragma unroll
                    for (int tp = 0; tp < TN / 2; ++tp) {
                        const float4 a = a4[tp];  // {d_a x2, sum q x2}
                        int f0 = dv[2 * tp], f1 = dv[2 * tp + 1];
                        if constexpr (T == kQ4_0) {
                            // (float)(dot - 8*sum_q) * (d_w * d_a); a block with d_a == 0 has a zero
                            // dot and sum, so it adds +0 like the reference's skip
                            f0 -= 8 * __float2int_rn(a.z);
                            f1 -= 8 * __float2int_rn(a.w);
                        }
                        float ta, tb;
                        upk2(mul2_rn(pk2(i2f(f0), i2f(f1)), mul2_rn(WD, pk2(a.x, a.y))), ta, tb);
                        acc[2 * tp] = fadd(acc[2 * tp], ta);
                        acc[2 * tp + 1] = fadd(acc[2 * tp + 1], tb);
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&acce[hb]);
            mbar_arrive(&sempty[q]);
        }
        const int grow = row0 + r;
        if (grow < out_dim && !*(volatile int*)&abort_flag) {
#pragma unroll
            for (int t = 0; t < TN; ++t)
                if (tok0 + t0 + t < batch) y[(size_t)(tok0 + t0 + t) * ldy + grow] = acc[t];
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kTcMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcCols) : "memory");
    }
}

template <int T>
static int launch_tc(const uint8_t* w, size_t rb, const ActBlock* act, int batch, int in_dim, int out_dim, float* y,
                     int ldy, int32_t* err, cudaStream_t st) {
    if (set_smem_limit(matbatch_tc_kernel<T>, kTcSmemAlloc) != cudaSuccess) return kErrCuda;
    const dim3 grid((batch + kTcN - 1) / kTcN, (out_dim + kTcM - 1) / kTcM);
    matbatch_tc_kernel<T><<<grid, kTcThreads, kTcSmemAlloc, st>>>(w, rb, act, batch, in_dim, out_dim, y, ldy, err);
    return cudaPeekAtLastError() == cudaSuccess ? kOk : kErrCuda;
}

// Returns kErrInvalidArg when the shape or format has no tensor-core path
// (the caller then uses the CUDA-core kernel).
int matbatch_tc_launch(const uint8_t* w, int32_t type, const ActBlock* act, int32_t batch, int32_t in_dim,
                       int32_t out_dim, float* y, int32_t* err, cudaStream_t st, int32_t ldy) {
    if (!w || !act || !y || batch <= 0 || out_dim <= 0 || in_dim <= 0 || (in_dim & 255)) return kErrInvalidArg;
    if (type != kQ4_K && type != kQ4_0 && type != kQ8_0) return kErrInvalidArg;
    const size_t rb = row_bytes(type, in_dim);
    if (((uintptr_t)w & 15) || (rb & 15) || ((uintptr_t)act & 15)) return kErrInvalidArg;
    if ((batch + kTcN - 1) / kTcN > 2147483647 || (out_dim + kTcM - 1) / kTcM > 65535) return kErrInvalidArg;
    if (ldy <= 0) ldy = out_dim;
    if (device_info().max_smem_optin < kTcSmemAlloc) return kErrInvalidArg;
    switch (type) {
        case kQ4_K: return launch_tc<kQ4_K>(w, rb, act, batch, in_dim, out_dim, y, ldy, err, st);
        case kQ4_0: return launch_tc<kQ4_0>(w, rb, act, batch, in_dim, out_dim, y, ldy, err, st);
        default: return launch_tc<kQ8_0>(w, rb, act, batch, in_dim, out_dim, y, ldy, err, st);
    }
}

}  // namespace gncx
