// capi.cu -- the C ABI (include/gncx_llm_core.h): reference-named entry points
// over device pointers plus the runtime they need (stream, status, workspace,
// host-mapping -> device-mirror registry, managed-memory arena).
#include <cuda_runtime.h>
#include <fcntl.h>
#include <math.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/gncx_llm_core.h"
#include "kernels.h"
#include "trace.cuh"

namespace gncx {

// ---------------------------------------------------------------- runtime state
struct Mapping {
    const uint8_t* host;
    size_t size;
    uint8_t* dev;
};

struct Runtime {
    int device = -1;
    cudaStream_t own = nullptr;
    cudaStream_t stream = nullptr;
    bool synchronous = true;
    int32_t* d_err = nullptr;
    int32_t* h_err = nullptr;  // pinned
    uint8_t* ws = nullptr;
    size_t ws_bytes = 0;
    std::vector<Mapping> maps;
};

static Runtime g_rt;
static std::mutex g_maps_mu;
static int32_t g_status = kOk;
static std::string g_message;

static std::mutex g_status_mu;  // entry points in other threads (the no-alloc one) report here too

static void set_error(int32_t code, const char* what) {
    std::lock_guard<std::mutex> lock(g_status_mu);
    if (code == kOk || g_status != kOk) return;
    g_status = code;
    g_message = what ? what : "";
}

static const char* cuda_msg(cudaError_t e) { return cudaGetErrorString(e); }

// Status of an entry point defined in another file of the library.
void record_api_error(int32_t code, const char* message) { set_error(code, message); }

static DeviceInfo g_info[64];

const DeviceInfo& device_info() {
    int dev = 0;
    cudaGetDevice(&dev);
    DeviceInfo& d = g_info[dev & 63];
    if (d.device != dev) {
        d.device = dev;
        cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        cudaDeviceGetAttribute(&d.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
        cudaDeviceGetAttribute(&d.l2_bytes, cudaDevAttrL2CacheSize, dev);
    }
    return d;
}

// Timeline-record binders of the translation units built with tracing.
static std::vector<void (*)(TraceRec*, unsigned*, unsigned)>& trace_binders() {
    static std::vector<void (*)(TraceRec*, unsigned*, unsigned)> v;
    return v;
}
int trace_register(void (*bind)(TraceRec*, unsigned*, unsigned)) {
    trace_binders().push_back(bind);
    return (int)trace_binders().size();
}

cudaError_t set_smem_limit(const void* k, size_t bytes) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, size_t> done;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorNoDevice;
    std::lock_guard<std::mutex> lock(mu);
    size_t& have = done[std::make_pair(k, dev)];
    if (bytes <= have || bytes <= 48 * 1024) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) have = bytes;
    return e;
}

// Initialise on first use: pick up the current device, create the library
// stream and the device error word.  Returns a status.
static int32_t ensure_init() {
    int dev = -1;
    if (g_rt.device >= 0) {
        if (cudaGetDevice(&dev) == cudaSuccess && dev == g_rt.device) return kOk;
    }
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0) {
        cudaGetLastError();
        set_error(kErrNoDevice, "gncx: no CUDA device is available (this library has no CPU path)");
        return kErrNoDevice;
    }
    if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
    if (g_rt.device != dev) {
        g_rt = Runtime{};
        g_rt.device = dev;
        if ((e = cudaStreamCreateWithFlags(&g_rt.own, cudaStreamNonBlocking)) != cudaSuccess ||
            (e = cudaMalloc(&g_rt.d_err, sizeof(int32_t))) != cudaSuccess ||
            (e = cudaMallocHost(&g_rt.h_err, sizeof(int32_t))) != cudaSuccess) {
            set_error(kErrCuda, cuda_msg(e));
            g_rt.device = -1;
            return kErrCuda;
        }
        cudaMemset(g_rt.d_err, 0, sizeof(int32_t));
        g_rt.stream = g_rt.own;
        device_info();
    }
    return kOk;
}

static cudaStream_t stream() { return g_rt.stream; }

// Growable device workspace, used in stream order.
static uint8_t* workspace(size_t bytes) {
    if (bytes <= g_rt.ws_bytes) return g_rt.ws;
    if (g_rt.ws) {
        cudaStreamSynchronize(g_rt.stream);
        cudaFree(g_rt.ws);
        g_rt.ws = nullptr;
        g_rt.ws_bytes = 0;
    }
    size_t want = bytes < ((size_t)1 << 20) ? ((size_t)1 << 20) : bytes;
    want = (want + 0xFFFFF) & ~(size_t)0xFFFFF;
    if (cudaMalloc(&g_rt.ws, want) != cudaSuccess) {
        cudaGetLastError();
        set_error(kErrOutOfMemory, "gncx: workspace allocation failed");
        return nullptr;
    }
    g_rt.ws_bytes = want;
    return g_rt.ws;
}

static size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

// Translate an address inside a gncx_gla_map_readonly mapping to its device mirror.
static const void* xlate(const void* p) {
    if (!p) return p;
    std::lock_guard<std::mutex> lk(g_maps_mu);
    const uint8_t* b = static_cast<const uint8_t*>(p);
    for (const Mapping& m : g_rt.maps)
        if (b >= m.host && b < m.host + m.size) return m.dev + (b - m.host);
    return p;
}
template <class T>
static T* xl(T* p) { return const_cast<T*>(static_cast<const T*>(xlate(p))); }

// The GPU must be able to dereference p.
static int32_t check_dev(const void* p, const char* name) {
    if (!p) {
        std::string m = std::string("gncx: null pointer: ") + name;
        set_error(kErrInvalidArg, m.c_str());
        return kErrInvalidArg;
    }
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        a.type = cudaMemoryTypeUnregistered;
    }
    if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged ||
        (a.type == cudaMemoryTypeHost && a.devicePointer != nullptr))
        return kOk;
    std::string m = std::string("gncx: pointer is not device-accessible: ") + name;
    set_error(kErrNotHostAccessible, m.c_str());
    return kErrNotHostAccessible;
}

// Record a launch status; in synchronous mode also wait and collect device-side errors.
static int32_t finish(int32_t st, bool force_sync = false) {
    if (st != kOk) {
        cudaError_t e = cudaGetLastError();
        set_error(st, st == kErrCuda ? cuda_msg(e) : "gncx: invalid argument or unsupported shape/type");
        return st;
    }
    if (!(g_rt.synchronous || force_sync)) return kOk;
    cudaMemcpyAsync(g_rt.h_err, g_rt.d_err, sizeof(int32_t), cudaMemcpyDeviceToHost, g_rt.stream);
    cudaError_t e = cudaStreamSynchronize(g_rt.stream);
    if (e != cudaSuccess) {
        set_error(kErrCuda, cuda_msg(e));
        return kErrCuda;
    }
    if (*g_rt.h_err != kOk) {
        const int32_t code = *g_rt.h_err;
        cudaMemsetAsync(g_rt.d_err, 0, sizeof(int32_t), g_rt.stream);
        set_error(code, code == kErrTimeout ? "gncx: a device-side wait timed out" : "gncx: device-side error");
        return code;
    }
    return kOk;
}

#define GNCX_BEGIN()                      \
    if (ensure_init() != kOk) return;     \
    (void)0
// True when the GPU can read p (device, managed or mapped pinned memory); no error recorded.
static bool dev_accessible(const void* p) {
    cudaPointerAttributes a;
    if (!p || cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged ||
           (a.type == cudaMemoryTypeHost && a.devicePointer == p);
}

#define GNCX_CHECK(p)                                \
    if (check_dev((p), #p) != kOk) return;           \
    (void)0

// ---------------------------------------------------------------- GLA mapping
struct GlaHandle {
    int fd = -1;
    const uint8_t* base = nullptr;
    size_t size = 0;
    uint8_t* dev = nullptr;
};

// ---------------------------------------------------------------- arena
struct RamHandle {
    uint8_t* ptr = nullptr;
    size_t bytes = 0;
};

static void telemetry_add(GNCXTelemetryStats* t, int64_t batch, int32_t in_dim, int32_t out_dim) {
    // csrc/gncx_llm_kernels.cpp:1464-1470, :1687-1691 (counters are synthetic there too;
    // zero_origin_cancellations needs the telemetry token encoding, which is not produced here)
    if (!t) return;
    const uint64_t macs = (uint64_t)batch * (uint64_t)in_dim * (uint64_t)out_dim;
    t->total_macs_equivalent += macs;
    t->zero_weight_skips += macs / 15;
    t->xfold_bucket_merges += (uint64_t)batch * ((uint64_t)in_dim / 32) * (uint64_t)out_dim;
}

}  // namespace gncx

using namespace gncx;

extern "C" {

// ---------------------------------------------------------------- status / plumbing
int32_t gncx_last_error(void) { return g_status; }
const char* gncx_last_error_message(void) { return g_message.c_str(); }
void gncx_clear_error(void) {
    std::lock_guard<std::mutex> lock(g_status_mu);
    g_status = kOk;
    g_message.clear();
}

int32_t gncx_trace_enable(void* records, uint32_t* counter, uint32_t capacity) {
    if (ensure_init() != kOk) return g_status;
    if (trace_binders().empty()) {
        set_error(kErrInvalidArg, "gncx_trace_enable: this library was built without timeline tracing");
        return kErrInvalidArg;
    }
    if ((records == nullptr) != (counter == nullptr)) {
        set_error(kErrInvalidArg, "gncx_trace_enable: records and counter go together");
        return kErrInvalidArg;
    }
    for (auto bind : trace_binders()) bind(static_cast<TraceRec*>(records), counter, records ? capacity : 0);
    const cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        set_error(kErrCuda, cuda_msg(e));
        return kErrCuda;
    }
    return kOk;
}

int32_t gncx_sync(void) {
    if (ensure_init() != kOk) return g_status;
    return finish(kOk, true);
}

void gncx_set_stream(void* s) {
    if (ensure_init() != kOk) return;
    cudaStreamSynchronize(g_rt.stream);
    g_rt.stream = s ? static_cast<cudaStream_t>(s) : g_rt.own;
}

void* gncx_get_stream(void) {
    if (ensure_init() != kOk) return nullptr;
    return g_rt.stream;
}

void gncx_set_synchronous(int32_t on) { g_rt.synchronous = on != 0; }

void gncx_set_weight_prefetch(int32_t on) { gemv_set_pdl(on != 0); }

static bool g_exact_attention = false;
void gncx_set_exact_attention(int32_t on) { g_exact_attention = on != 0; }

int32_t gncx_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

int32_t gncx_set_device(int32_t device) {
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) {
        set_error(kErrCuda, cuda_msg(e));
        return kErrCuda;
    }
    return ensure_init();
}

void* gncx_device_alloc(size_t bytes) {
    if (ensure_init() != kOk) return nullptr;
    void* p = nullptr;
    if (cudaMalloc(&p, bytes ? bytes : 1) != cudaSuccess) {
        cudaGetLastError();
        set_error(kErrOutOfMemory, "gncx: cudaMalloc failed");
        return nullptr;
    }
    return p;
}

void gncx_device_free(void* p) {
    if (p) cudaFree(p);
}

int32_t gncx_memcpy(void* dst, const void* src, size_t bytes) {
    if (ensure_init() != kOk) return g_status;
    if (bytes == 0) return kOk;
    cudaStreamSynchronize(g_rt.stream);
    cudaError_t e = cudaMemcpy(dst, xlate(src), bytes, cudaMemcpyDefault);
    if (e != cudaSuccess) {
        set_error(kErrCuda, cuda_msg(e));
        return kErrCuda;
    }
    return kOk;
}

// ---------------------------------------------------------------- GLA file mapping
void* gncx_gla_map_readonly(const char* filepath, size_t* out_size) {
    if (ensure_init() != kOk) return nullptr;
    if (!filepath) {
        set_error(kErrInvalidArg, "gncx: null path");
        return nullptr;
    }
    const int fd = open(filepath, O_RDONLY);
    if (fd < 0) return nullptr;  // as the reference: NULL when the file cannot be opened
    struct stat st {};
    fstat(fd, &st);
    const size_t size = (size_t)st.st_size;
    void* base = size ? mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0) : nullptr;
    if (size && (base == MAP_FAILED || base == nullptr)) {
        close(fd);
        return nullptr;
    }
    if (size) madvise(base, size, MADV_WILLNEED);
    GlaHandle* h = new GlaHandle();
    h->fd = fd;
    h->base = static_cast<const uint8_t*>(base);
    h->size = size;
    if (size) {
        cudaError_t e = cudaMalloc(&h->dev, size);
        if (e == cudaSuccess) e = cudaMemcpy(h->dev, base, size, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            set_error(kErrOutOfMemory, cuda_msg(e));
            if (h->dev) cudaFree(h->dev);
            munmap(base, size);
            close(fd);
            delete h;
            return nullptr;
        }
        std::lock_guard<std::mutex> lk(g_maps_mu);
        g_rt.maps.push_back(Mapping{h->base, size, h->dev});
    }
    if (out_size) *out_size = size;
    return h;
}

const uint8_t* gncx_gla_get_base_ptr(void* opaque) {
    return opaque ? static_cast<GlaHandle*>(opaque)->base : nullptr;
}

void gncx_gla_unmap(void* opaque) {
    if (!opaque) return;
    GlaHandle* h = static_cast<GlaHandle*>(opaque);
    {
        std::lock_guard<std::mutex> lk(g_maps_mu);
        for (size_t i = 0; i < g_rt.maps.size(); ++i)
            if (g_rt.maps[i].host == h->base) {
                g_rt.maps.erase(g_rt.maps.begin() + (long)i);
                break;
            }
    }
    if (h->dev) {
        cudaStreamSynchronize(g_rt.stream);
        cudaFree(h->dev);
    }
    if (h->base) munmap(const_cast<uint8_t*>(h->base), h->size);
    if (h->fd >= 0) close(h->fd);
    delete h;
}

void gncx_gla_prefetch_range(const uint8_t* mmap_base, size_t offset, size_t num_bytes) {
    // The whole file already has a device mirror; only advise the host pages.
    if (!mmap_base || !num_bytes) return;
    const uintptr_t a = (uintptr_t)(mmap_base + offset) & ~(uintptr_t)4095;
    madvise(reinterpret_cast<void*>(a), num_bytes + ((uintptr_t)(mmap_base + offset) - a), MADV_WILLNEED);
}

// ---------------------------------------------------------------- arena
void* gncx_ram_alloc_colored(size_t total_bytes, uint8_t, uint8_t, uint8_t) {
    if (ensure_init() != kOk) return nullptr;
    if (total_bytes == 0) total_bytes = 64;
    RamHandle* h = new RamHandle();
    if (cudaMallocManaged(&h->ptr, total_bytes) != cudaSuccess) {
        cudaGetLastError();
        set_error(kErrOutOfMemory, "gncx: cudaMallocManaged failed");
        delete h;
        return nullptr;
    }
    h->bytes = total_bytes;
    return h;
}

void* gncx_ram_alloc(size_t total_bytes) { return gncx_ram_alloc_colored(total_bytes, 0, 0, 0); }

uint8_t* gncx_ram_get_ptr(void* h) { return h ? static_cast<RamHandle*>(h)->ptr : nullptr; }

// Address bits the reference reports (:566-574); the colouring itself is DDR3-specific.
uint8_t gncx_ram_get_ddr3_bank(void* h) {
    return h ? (uint8_t)(((uintptr_t) static_cast<RamHandle*>(h)->ptr >> 14) & 0x7u) : 0;
}
uint8_t gncx_ram_get_l1_set(void* h) {
    return h ? (uint8_t)(((uintptr_t) static_cast<RamHandle*>(h)->ptr >> 6) & 0x3Fu) : 0;
}

void gncx_ram_free(void* h) {
    if (!h) return;
    RamHandle* r = static_cast<RamHandle*>(h);
    if (g_rt.stream) cudaStreamSynchronize(g_rt.stream);
    cudaFree(r->ptr);
    delete r;
}

void gncx_ram_copy_chunk(void* h, size_t dst_offset, const uint8_t* src_base, size_t src_offset, size_t num_bytes) {
    if (!h || !src_base || num_bytes == 0) return;
    GNCX_BEGIN();
    RamHandle* r = static_cast<RamHandle*>(h);
    if (dst_offset + num_bytes > r->bytes) {
        set_error(kErrInvalidArg, "gncx_ram_copy_chunk: copy exceeds the arena");
        return;
    }
    cudaStreamSynchronize(g_rt.stream);
    cudaError_t e = cudaMemcpy(r->ptr + dst_offset, src_base + src_offset, num_bytes, cudaMemcpyDefault);
    if (e != cudaSuccess) set_error(kErrCuda, cuda_msg(e));
}

// ---------------------------------------------------------------- embeddings
static void fetch_embedding(const uint8_t* base, size_t off, int32_t type, int32_t token, int32_t dim, float scale,
                            float* out) {
    GNCX_BEGIN();
    const uint8_t* w = xl(base);
    GNCX_CHECK(w);
    GNCX_CHECK(out);
    if (token < 0 || dim <= 0) {
        finish(kErrInvalidArg);
        return;
    }
    const uint8_t* row = w + off + (size_t)token * row_bytes(type, dim);
    finish(dequant_launch(row, type, 1, dim, scale, nullptr, out, stream()));
}

void gncx_fetch_token_embedding_q8_0(const uint8_t* b, size_t off, int32_t tok, int32_t dim, float s, float* out) {
    fetch_embedding(b, off, kQ8_0, tok, dim, s, out);
}
void gncx_fetch_token_embedding_q6_k(const uint8_t* b, size_t off, int32_t tok, int32_t dim, float s, float* out) {
    fetch_embedding(b, off, kQ6_K, tok, dim, s, out);
}
void gncx_fetch_token_embedding_bf16(const uint8_t* b, size_t off, int32_t tok, int32_t dim, float s, float* out) {
    fetch_embedding(b, off, kBF16, tok, dim, s, out);
}

// ---------------------------------------------------------------- RMSNorm
static const int64_t kRepunits[18] = {1LL, 11LL, 111LL, 1111LL, 11111LL, 111111LL, 1111111LL, 11111111LL,
                                      111111111LL, 1111111111LL, 11111111111LL, 111111111111LL, 1111111111111LL,
                                      11111111111111LL, 111111111111111LL, 1111111111111111LL,
                                      11111111111111111LL, 111111111111111111LL};

void gncx_rmsnorm_and_encode_4phase(const float* in, const uint8_t* base, size_t w_off, int32_t dim, float eps,
                                    int32_t layer_k, float* out, GNCXCompactToken* out_tokens, float* out_scale) {
    GNCX_BEGIN();
    const float* x = xl(in);
    const uint8_t* b = xl(base);
    GNCX_CHECK(x);
    GNCX_CHECK(b);
    GNCX_CHECK(out);
    const float* w = reinterpret_cast<const float*>(b + w_off);
    int32_t st = rmsnorm_launch(x, w, 1, dim, eps, out, stream());
    if (st == kOk && out_scale) {
        if (!out_tokens) {
            *out_scale = 1.0f;  // :836-840
        } else {
            // :842-855: scale_to_fp = max(1e-9, max|y|) / (9 * repunit(k))
            float* d = reinterpret_cast<float*>(workspace(256));
            if (!d) return;
            st = absmax_launch(out, dim, d, stream());
            float m = 0.0f;
            if (st == kOk && cudaMemcpyAsync(&m, d, 4, cudaMemcpyDeviceToHost, stream()) == cudaSuccess &&
                cudaStreamSynchronize(stream()) == cudaSuccess) {
                const float max_abs = m > 1e-9f ? m : 1e-9f;
                const int lk = layer_k < 0 ? 0 : (layer_k > 17 ? 17 : layer_k);
                *out_scale = max_abs / (float)(9 * kRepunits[lk]);
            }
        }
    }
    finish(st);
}

void gncx_rmsnorm_inplace_heads(float* vec, const uint8_t* base, size_t w_off, int32_t has_weight, int32_t n_heads,
                                int32_t head_dim, float eps) {
    GNCX_BEGIN();
    float* v = xl(vec);
    GNCX_CHECK(v);
    const float* w = nullptr;
    if (has_weight) {
        const uint8_t* b = xl(base);
        GNCX_CHECK(b);
        w = reinterpret_cast<const float*>(b + w_off);
    }
    finish(rmsnorm_heads_launch(v, w, 1, n_heads, head_dim, eps, stream()));
}

// ---------------------------------------------------------------- GEMV / GEMM
void gncx_xfold_universal_matvec(const uint8_t* base, size_t off, int32_t type, const float* in_vec,
                                 const GNCXCompactToken*, int32_t in_dim, int32_t out_dim, float* out_vec,
                                 GNCXTelemetryStats* telemetry) {
    GNCX_BEGIN();
    const uint8_t* b = xl(base);
    const float* x = xl(in_vec);
    GNCX_CHECK(b);
    GNCX_CHECK(x);
    GNCX_CHECK(out_vec);
    const int32_t st = gemv_launch(b + off, type, x, nullptr, in_dim, out_dim, out_vec, 0.0f, g_rt.d_err, stream());
    if (st == kOk) telemetry_add(telemetry, 1, in_dim, out_dim);
    finish(st);
}

void gncx_xfold_q4_0_matvec(const uint8_t* base, size_t off, const float* in_vec, const GNCXCompactToken* tok,
                            int32_t in_dim, int32_t out_dim, float* out_vec, GNCXTelemetryStats* telemetry) {
    gncx_xfold_universal_matvec(base, off, kQ4_0, in_vec, tok, in_dim, out_dim, out_vec, telemetry);
}

void gncx_xfold_universal_matbatch(const uint8_t* base, size_t off, int32_t type, const float* in_batch,
                                   int32_t batch, int32_t in_dim, int32_t out_dim, float* out_batch,
                                   GNCXTelemetryStats* telemetry) {
    GNCX_BEGIN();
    const uint8_t* b = xl(base);
    const float* x = xl(in_batch);
    GNCX_CHECK(b);
    GNCX_CHECK(x);
    GNCX_CHECK(out_batch);
    if (batch <= 0 || in_dim <= 0 || (in_dim & 31)) {
        finish(batch == 0 ? kOk : kErrInvalidArg);
        return;
    }
    int32_t st = kOk;
    const ActBlock* act = nullptr;
    if (type != kBF16) {
        ActBlock* a = reinterpret_cast<ActBlock*>(workspace((size_t)batch * (in_dim / 32) * sizeof(ActBlock)));
        if (!a) return;
        st = act_quantize_launch(x, batch, in_dim, a, stream());
        act = a;
    }
    if (st == kOk) st = matbatch_launch(b + off, type, x, act, batch, in_dim, out_dim, out_batch, g_rt.d_err, stream());
    if (st == kOk) telemetry_add(telemetry, batch, in_dim, out_dim);
    finish(st);
}

void gncx_xfold_q4_0_matbatch(const uint8_t* base, size_t off, const float* in_batch, int32_t batch, int32_t in_dim,
                              int32_t out_dim, float* out_batch, GNCXTelemetryStats* telemetry) {
    gncx_xfold_universal_matbatch(base, off, kQ4_0, in_batch, batch, in_dim, out_dim, out_batch, telemetry);
}

void gncx_universal_lm_head_logits(const uint8_t* base, size_t off, int32_t type, const float* h, int32_t dim,
                                   int32_t vocab, float softcap, float* logits) {
    GNCX_BEGIN();
    const uint8_t* b = xl(base);
    const float* x = xl(h);
    GNCX_CHECK(b);
    GNCX_CHECK(x);
    GNCX_CHECK(logits);
    finish(gemv_launch(b + off, type, x, nullptr, dim, vocab, logits, softcap, g_rt.d_err, stream()));
}

void gncx_q8_0_lm_head_logits(const uint8_t* base, size_t off, const float* h, int32_t dim, int32_t vocab,
                              float* logits) {
    gncx_universal_lm_head_logits(base, off, kQ8_0, h, dim, vocab, 0.0f, logits);
}

// ---------------------------------------------------------------- RoPE
// The cos/sin table is computed on the host with the same libm calls as the
// reference (:1779-1796: powf, cosf, sinf in float), exactly once per call.
static int32_t rope_table_host(int32_t pos, int32_t hd, float base, const float* ff, RopeTab& t) {
    const int32_t half = hd / 2;
    if (half > 256) return kErrInvalidArg;
    for (int32_t i = 0; i < half; ++i) {
        float freq = 1.0f / powf(base, (float)(2 * i) / (float)hd);
        if (ff && ff[i] != 0.0f) freq /= ff[i];
        const float ang = (float)pos * freq;
        t.c[i] = cosf(ang);
        t.s[i] = sinf(ang);
    }
    return kOk;
}

void gncx_apply_rope_xor11_ext(float* q_vec, float* k_vec, GNCXCompactToken*, const uint8_t* base,
                               size_t rope_freqs_off, int32_t has_rope_freqs, int32_t n_heads, int32_t n_kv,
                               int32_t hd, int32_t pos, float freq_base) {
    GNCX_BEGIN();
    float* q = xl(q_vec);
    float* k = xl(k_vec);
    if (q) GNCX_CHECK(q);
    if (k) GNCX_CHECK(k);
    if (hd <= 0 || (hd & 1) || hd / 2 > 256) {
        finish(kErrInvalidArg);
        return;
    }
    float ff[256];
    const float* ffp = nullptr;
    if (has_rope_freqs) {
        const uint8_t* b = xl(base);
        GNCX_CHECK(b);
        if (cudaMemcpy(ff, b + rope_freqs_off, (size_t)(hd / 2) * 4, cudaMemcpyDefault) != cudaSuccess) {
            finish(kErrCuda);
            return;
        }
        ffp = ff;
    }
    static RopeTab tab;
    rope_table_host(pos, hd, freq_base, ffp, tab);
    finish(rope_tab_launch(q, k, n_heads, n_kv, hd, tab, stream()));
}

void gncx_apply_rope_xor11(float* q_vec, float* k_vec, GNCXCompactToken* tok, int32_t n_heads, int32_t n_kv,
                           int32_t hd, int32_t pos, float freq_base) {
    gncx_apply_rope_xor11_ext(q_vec, k_vec, tok, nullptr, 0, 0, n_heads, n_kv, hd, pos, freq_base);
}

// ---------------------------------------------------------------- attention
void gncx_mqa_attention_step_ext(const float* q_vec, const float* k_vec, const float* v_vec, float* k_cache,
                                 float* v_cache, int32_t pos, int32_t n_heads, int32_t n_kv, int32_t hd,
                                 float attn_scale, int32_t window, int32_t write_kv, float* out) {
    GNCX_BEGIN();
    const float* q = xl(q_vec);
    float* kc = xl(k_cache);
    float* vc = xl(v_cache);
    GNCX_CHECK(q);
    GNCX_CHECK(kc);
    GNCX_CHECK(vc);
    GNCX_CHECK(out);
    if (pos < 0 || !attention_shape_ok(n_heads, n_kv, hd)) {  // rejected before the KV write
        finish(kErrInvalidArg);
        return;
    }
    const size_t kvd = (size_t)n_kv * hd;
    const float* nk = nullptr;
    const float* nv = nullptr;
    if (write_kv && k_vec && v_vec) {  // :1903-1907
        const float* k = xl(k_vec);
        const float* v = xl(v_vec);
        if (dev_accessible(k) && dev_accessible(v)) {
            nk = k;  // the attention launch stores them in the cache
            nv = v;
        } else {
            cudaMemcpyAsync(kc + (size_t)pos * kvd, k, kvd * 4, cudaMemcpyDefault, stream());
            cudaMemcpyAsync(vc + (size_t)pos * kvd, v, kvd * 4, cudaMemcpyDefault, stream());
        }
    }
    const int32_t recs = attention_scratch_records(pos, n_heads, window);
    const size_t part_bytes = align256((size_t)recs * attn_record_floats(hd) * 4);
    const size_t score_floats = (size_t)n_heads * (((size_t)pos + 1 + 63) / 64 * 64);
    uint8_t* ws = workspace(part_bytes + (g_exact_attention ? score_floats * 4 : 0));
    if (!ws) return;
    float* part = reinterpret_cast<float*>(ws);
    float* scores = g_exact_attention ? reinterpret_cast<float*>(ws + part_bytes) : nullptr;
    finish(attention_launch(q, kc, vc, pos, n_heads, n_kv, hd, attn_scale, window, out, AttnScratch{part, recs},
                            g_rt.d_err, stream(), scores, nk, nv));
}

// Causal attention of a block of prompt positions: the reference's prefill
// calls gncx_mqa_attention_step_ext once per position (write_kv = 0, no
// window; lua/gncx_streamer.lua:1079-1109); here every query of the block
// runs in one launch per group of kPfGroup positions.
constexpr int kPfGroup = 256;
constexpr int kPfChunkApi = 64;
int32_t gncx_attention_prefill(const float* q, const float* k_cache, const float* v_cache, int32_t pos0, int32_t n_tok,
                               int32_t n_heads, int32_t n_kv, int32_t hd, float attn_scale, float* out) {
    if (ensure_init() != kOk) return g_status;
    const float* qq = xl(q);
    const float* kc = xl(k_cache);
    const float* vc = xl(v_cache);
    if (check_dev(qq, "q") || check_dev(kc, "k_cache") || check_dev(vc, "v_cache") || check_dev(out, "out"))
        return g_status;
    if (pos0 < 0 || n_tok <= 0 || !attention_shape_ok(n_heads, n_kv, hd)) {
        set_error(kErrInvalidArg, "gncx_attention_prefill: bad position, count or head shape");
        return kErrInvalidArg;
    }
    const int32_t last = pos0 + n_tok - 1;
    const size_t splits = (size_t)(last + kPfChunkApi) / kPfChunkApi;
    const size_t grp = n_tok < kPfGroup ? (size_t)n_tok : (size_t)kPfGroup;
    const size_t part_bytes = align256(grp * n_heads * splits * attn_record_floats(hd) * 4);
    const size_t score_bytes = g_exact_attention ? grp * n_heads * splits * kPfChunkApi * 4 : 0;
    uint8_t* ws = workspace(part_bytes + score_bytes);
    if (!ws) return g_status;
    const int32_t qd = n_heads * hd;
    for (int32_t z0 = 0; z0 < n_tok; z0 += kPfGroup) {
        const int32_t nz = n_tok - z0 < kPfGroup ? n_tok - z0 : kPfGroup;
        AttnArgs a{};
        a.q = qq + (size_t)z0 * qd;
        a.q_stride = qd;
        a.kc = kc;
        a.vc = vc;
        a.kv_pos_stride = n_kv * hd;  // the reference's [pos][n_kv][head_dim]
        a.kv_head_stride = hd;
        a.pos0 = pos0 + z0;
        a.n_heads = n_heads;
        a.n_kv = n_kv;
        a.hd = hd;
        a.scale = attn_scale;
        a.chunk = kPfChunkApi;
        a.max_splits = (pos0 + z0 + nz + kPfChunkApi - 1) / kPfChunkApi;
        a.part = reinterpret_cast<float*>(ws);
        a.out = out + (size_t)z0 * qd;
        a.out_stride = qd;
        a.err = g_rt.d_err;
        a.exact = g_exact_attention ? 1 : 0;
        a.scores = g_exact_attention ? reinterpret_cast<float*>(ws + part_bytes) : nullptr;
        a.score_cap = a.max_splits * kPfChunkApi;
        const int st = attention_run(a, nz, stream());
        if (st != kOk) return finish(st);
    }
    return finish(kOk);
}

void gncx_mqa_attention_step(const float* q_vec, const float* k_vec, const float* v_vec, float* k_cache,
                             float* v_cache, int32_t pos, int32_t n_heads, int32_t n_kv, int32_t hd, float* out) {
    const float scale = 1.0f / sqrtf((float)hd);  // :2008
    gncx_mqa_attention_step_ext(q_vec, k_vec, v_vec, k_cache, v_cache, pos, n_heads, n_kv, hd, scale, 0, 1, out);
}

// ---------------------------------------------------------------- GLU
static void glu(const float* g, const float* u, int32_t n, float* out, bool gelu) {
    GNCX_BEGIN();
    const float* gg = xl(g);
    const float* uu = xl(u);
    GNCX_CHECK(gg);
    GNCX_CHECK(uu);
    GNCX_CHECK(out);
    finish(glu_launch(gg, uu, n, out, gelu, stream()));
}
void gncx_geglu_activation(const float* g, const float* u, int32_t n, float* out) { glu(g, u, n, out, true); }
void gncx_swiglu_activation(const float* g, const float* u, int32_t n, float* out) { glu(g, u, n, out, false); }

// ---------------------------------------------------------------- added entry points
int32_t gncx_act_quantize(const float* x, int32_t rows, int32_t in_dim, void* act_out) {
    if (ensure_init() != kOk) return g_status;
    const float* xx = xl(x);
    if (check_dev(xx, "x") || check_dev(act_out, "act_out")) return g_status;
    return finish(act_quantize_launch(xx, rows, in_dim, static_cast<ActBlock*>(act_out), stream()));
}

int32_t gncx_matvec_preq(const uint8_t* base, size_t off, int32_t type, const void* act, int32_t in_dim,
                         int32_t out_dim, float* out_vec) {
    if (ensure_init() != kOk) return g_status;
    const uint8_t* b = xl(base);
    if (check_dev(b, "base") || check_dev(act, "act") || check_dev(out_vec, "out_vec")) return g_status;
    if (type == kBF16 || in_dim <= 0 || (in_dim & 255)) return finish(kErrInvalidArg);
    uint8_t* staged = workspace(staged_act_bytes(in_dim));
    if (!staged) return g_status;
    int32_t st = act_stage_launch(static_cast<const ActBlock*>(act), in_dim, staged, stream());
    if (st == kOk) st = gemv_launch(b + off, type, nullptr, staged, in_dim, out_dim, out_vec, 0.0f, g_rt.d_err, stream());
    return finish(st);
}

int32_t gncx_dequantize_rows(const uint8_t* base, size_t off, int32_t type, int32_t rows, int32_t n, float* out) {
    if (ensure_init() != kOk) return g_status;
    const uint8_t* b = xl(base);
    if (check_dev(b, "base") || check_dev(out, "out")) return g_status;
    return finish(dequant_launch(b + off, type, rows, n, 1.0f, nullptr, out, stream()));
}

int32_t gncx_sample_greedy(const float* logits, int32_t vocab, const int32_t* recent, int32_t n_recent,
                           double penalty) {
    if (ensure_init() != kOk) return -1;
    const float* lg = xl(logits);
    if (check_dev(lg, "logits")) return -1;
    if (vocab <= 0 || n_recent < 0) {
        finish(kErrInvalidArg);
        return -1;
    }
    const int32_t keep = n_recent > 65 ? 65 : n_recent;  // the last <=65 tokens matter
    const size_t o_rec = 0, o_idx = align256((size_t)keep * 4 + 4), o_scr = o_idx + 256;
    uint8_t* ws = workspace(o_scr + argmax_scratch_bytes(vocab));
    if (!ws) return -1;
    int32_t* d_rec = reinterpret_cast<int32_t*>(ws + o_rec);
    int32_t* d_idx = reinterpret_cast<int32_t*>(ws + o_idx);
    if (keep > 0) cudaMemcpyAsync(d_rec, recent + (n_recent - keep), (size_t)keep * 4, cudaMemcpyHostToDevice, stream());
    int32_t st = argmax_penalized_launch(lg, vocab, d_rec, keep, penalty, d_idx, ws + o_scr, stream());
    int32_t idx = -1;
    if (st == kOk) cudaMemcpyAsync(&idx, d_idx, 4, cudaMemcpyDeviceToHost, stream());
    if (finish(st, true) != kOk) return -1;
    return idx;
}

}  // extern "C"
