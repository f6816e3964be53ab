// noalloc.cu -- a decode-attention entry point that allocates nothing.
//
// gncx_mqa_attention_step_noalloc runs the same split-KV attention as
// gncx_mqa_attention_step_ext, but its partial-softmax records live in a
// fixed array in this file instead of the library's growable workspace, and
// it touches none of the library's lazily created state (stream, error word,
// workspace).  It is for callers that may not allocate GPU memory once they
// are running: a host that pre-plans every allocation (a serving process
// with a fixed memory budget), or code running where an allocation would
// synchronise the device.
//
// Limit: kNoAllocScratchBytes of records, i.e. n_heads * splits * (head_dim + 4)
// floats, splits = ceil(window / chunk) with chunk = 16..64 positions; a call
// that needs more is rejected with GNCX_ERR_CAPACITY and a message.
//
// Set-up: the first call on a device (with that device current) looks up the
// array's device address with cudaGetSymbolAddress; make that first call
// before any stream capture.  Every later call on the device reuses it.  A
// cudaDeviceReset discards the device's copy of the array; the cached address
// is then stale, so a process that resets a device must not call this entry
// point on that device again.
//
// Sharing: all calls on a device share the one array and leave their records
// in it.  Nothing in it needs to start at zero: every record the merge reads
// is written earlier in the same call.  Calls whose GPU work overlaps (on
// different streams, or from different threads without ordering) race on the
// array and must be serialised by the caller.
#include <cuda_runtime.h>
#include <stdio.h>
#include <mutex>
#include "kernels.h"

namespace gncx {

// Internal: records a status in the library's error state (capi.cu).
void record_api_error(int32_t code, const char* message);

constexpr size_t kNoAllocScratchBytes = (size_t)4 << 20;  // 4 MiB per device, held until exit
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[kMaxDevices];

// Device address of the scratch array on the current device (looked up once).
static int32_t noalloc_scratch(void** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return kErrNoDevice;
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            return kErrCuda;
        }
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return kOk;
}

}  // namespace gncx

using namespace gncx;

extern "C" int32_t gncx_mqa_attention_step_noalloc(const float* q_vec, const float* k_vec, const float* v_vec,
                                                   float* k_cache_layer, float* v_cache_layer, int32_t pos,
                                                   int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                                                   float attn_scale, int32_t sliding_window, int32_t write_kv,
                                                   float* out_attn_vec, void* cuda_stream) {
    // Everything the launch would reject is rejected here, before the KV-cache
    // write, so a refused call leaves the caller's cache untouched.
    if (!q_vec || !k_cache_layer || !v_cache_layer || !out_attn_vec || pos < 0 ||
        !attention_shape_ok(n_heads, n_kv_heads, head_dim)) {
        record_api_error(kErrInvalidArg,
                         "gncx_mqa_attention_step_noalloc: null pointer, bad dimension, n_heads not a multiple of "
                         "n_kv_heads, or head_dim not a multiple of 4 up to 256");
        return kErrInvalidArg;
    }
    void* scratch = nullptr;
    int32_t st = noalloc_scratch(&scratch);
    if (st != kOk) {
        record_api_error(st, "gncx_mqa_attention_step_noalloc: scratch set-up failed (cudaGetSymbolAddress)");
        return st;
    }
    int sms = 0, dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        cudaGetLastError();
        record_api_error(kErrCuda, "gncx_mqa_attention_step_noalloc: device query failed");
        return kErrCuda;
    }
    const int32_t t0 = sliding_window > 0 ? (pos - sliding_window + 1 > 0 ? pos - sliding_window + 1 : 0) : 0;
    const int32_t len = pos + 1 - t0;
    const int chunk = attention_geometry_chunk(len, n_kv_heads, sms);
    const int64_t splits = (len + chunk - 1) / chunk;
    const int64_t rec_bytes = (int64_t)attn_record_floats(head_dim) * 4;
    const int64_t need = (int64_t)n_heads * splits * rec_bytes;
    if (need > (int64_t)kNoAllocScratchBytes) {
        char msg[256];
        snprintf(msg, sizeof(msg),
                 "gncx_mqa_attention_step_noalloc: this window needs %lld bytes of scratch; the fixed array holds %zu",
                 (long long)need, kNoAllocScratchBytes);
        record_api_error(kErrCapacity, msg);
        return kErrCapacity;
    }
    cudaStream_t s = static_cast<cudaStream_t>(cuda_stream);
    const size_t kvd = (size_t)n_kv_heads * head_dim;
    if (write_kv && k_vec && v_vec) {  // csrc/gncx_llm_kernels.cpp:1903-1907
        if (cudaMemcpyAsync(k_cache_layer + (size_t)pos * kvd, k_vec, kvd * 4, cudaMemcpyDefault, s) != cudaSuccess ||
            cudaMemcpyAsync(v_cache_layer + (size_t)pos * kvd, v_vec, kvd * 4, cudaMemcpyDefault, s) != cudaSuccess) {
            cudaGetLastError();
            record_api_error(kErrCuda, "gncx_mqa_attention_step_noalloc: KV write failed");
            return kErrCuda;
        }
    }
    const int32_t capacity = (int32_t)(kNoAllocScratchBytes / rec_bytes);
    st = attention_launch(q_vec, k_cache_layer, v_cache_layer, pos, n_heads, n_kv_heads, head_dim, attn_scale,
                          sliding_window, out_attn_vec, AttnScratch{static_cast<float*>(scratch), capacity}, nullptr,
                          s, nullptr);
    if (st != kOk) record_api_error(st, "gncx_mqa_attention_step_noalloc: launch failed");
    return st;
}
