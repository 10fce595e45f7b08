// C ABI of libb200q.so (declared in include/b200q.h): per-device state, the
// resident weight cache behind the host-pointer drop-ins, and the drop-in and
// device-pointer entry points.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <utility>
#include <vector>

#include "common.cuh"
#include "internal.h"

namespace b200q {

namespace {

std::mutex g_dev_mu;
std::vector<Device*> g_devs;
int g_act_mode = 0;  // 0 = not yet read from the environment
int g_pdl = -1;
thread_local int t_last_error = B200Q_OK;

int env_act_mode() {
    const char* e = std::getenv("B200Q_ACT");
    if (e && (std::strcmp(e, "x8") == 0 || std::strcmp(e, "X8") == 0 || std::strcmp(e, "1") == 0)) return B200Q_ACT_X8;
    return B200Q_ACT_X16;
}

bool env_flag(const char* name, bool dflt) {
    const char* e = std::getenv(name);
    if (!e || !*e) return dflt;
    return !(std::strcmp(e, "0") == 0 || std::strcmp(e, "false") == 0 || std::strcmp(e, "off") == 0);
}

}  // namespace

void set_last_error(int status) { t_last_error = status; }

bool pdl_enabled() {
    if (g_pdl < 0) g_pdl = env_flag("B200Q_PDL", true) ? 1 : 0;
    return g_pdl == 1;
}

Device* device_state(int dev, int* err) {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (dev < 0) {
        *err = B200Q_ENODEV;
        return nullptr;
    }
    if (static_cast<int>(g_devs.size()) <= dev) g_devs.resize(dev + 1, nullptr);
    if (g_devs[dev]) return g_devs[dev];
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) {
        *err = B200Q_ENODEV;
        return nullptr;
    }
    if (prop.major != 10) {  // built for sm_100a only
        *err = B200Q_ENODEV;
        return nullptr;
    }
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(dev);
    Device* d = new Device();
    d->id = dev;
    d->num_sms = prop.multiProcessorCount;
    int* h = nullptr;
    if (cudaHostAlloc(reinterpret_cast<void**>(&h), 64, cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) {
        delete d;
        if (prev >= 0) cudaSetDevice(prev);
        *err = B200Q_ENOMEM;
        return nullptr;
    }
    std::memset(h, 0, 64);
    int* dptr = nullptr;
    if (cudaHostGetDevicePointer(reinterpret_cast<void**>(&dptr), h, 0) != cudaSuccess) {
        cudaFreeHost(h);
        delete d;
        if (prev >= 0) cudaSetDevice(prev);
        *err = B200Q_ECUDA;
        return nullptr;
    }
    d->status_host = h;
    d->status = dptr;
    if (prev >= 0 && prev != dev) cudaSetDevice(prev);
    g_devs[dev] = d;
    *err = B200Q_OK;
    return d;
}

Device* device_state_if_present(int dev) {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (dev < 0 || dev >= static_cast<int>(g_devs.size())) return nullptr;
    return g_devs[dev];
}

int current_device_state(Device** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return B200Q_ENODEV;
    int err = B200Q_OK;
    *out = device_state(dev, &err);
    return *out ? B200Q_OK : err;
}

// ---------------------------------------------------------------------------
// Resident weight cache for the host-pointer drop-ins. The reference engine
// borrows weight pointers for the lifetime of its graph and never mutates
// them (model_graph.cpp:3387-3427); the drop-ins therefore upload each
// packed matrix once per device, keyed by (device, host address, bytes).
// B200Q_WEIGHT_CACHE=0 disables residency (upload on every call).
// ---------------------------------------------------------------------------
namespace {

struct WeightEntry {
    void* dptr = nullptr;
    size_t bytes = 0;
    uint64_t fingerprint = 0;
};

// FNV-1a over the size and three 64-byte samples (start, middle, end) of a
// host matrix: a cheap guard against a freed buffer's address being reused
// for different weights. It does not detect in-place edits of the middle of
// a buffer; callers that mutate or free weights call b200q_weight_cache_evict.
uint64_t fingerprint(const void* host, size_t bytes) {
    const uint8_t* p = static_cast<const uint8_t*>(host);
    uint64_t h = 1469598103934665603ull ^ bytes;
    auto mix = [&](size_t off) {
        const size_t end = std::min(bytes, off + 64);
        for (size_t i = off; i < end; ++i) h = (h ^ p[i]) * 1099511628211ull;
    };
    mix(0);
    if (bytes > 128) mix(bytes / 2 - 32);
    if (bytes > 64) mix(bytes - 64);
    return h;
}
std::mutex g_w_mu;
std::map<std::pair<int, const void*>, WeightEntry> g_weights;
long long g_weight_bytes = 0;

int upload_weights(int dev, const void* host, size_t bytes, void** out) {
    void* d = nullptr;
    // +16: kernels copy 16-byte-aligned windows around rows.
    if (cudaMalloc(&d, bytes + 16) != cudaSuccess) return B200Q_ENOMEM;
    if (cudaMemcpy(d, host, bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(d);
        return B200Q_ECUDA;
    }
    *out = d;
    (void)dev;
    return B200Q_OK;
}

int weights_for(int dev, const void* host, size_t bytes, void** dptr, bool* temporary) {
    *temporary = false;
    if (!env_flag("B200Q_WEIGHT_CACHE", true)) {
        *temporary = true;
        return upload_weights(dev, host, bytes, dptr);
    }
    std::lock_guard<std::mutex> lk(g_w_mu);
    auto key = std::make_pair(dev, host);
    auto it = g_weights.find(key);
    const uint64_t fp = fingerprint(host, bytes);
    if (it != g_weights.end()) {
        if (it->second.bytes == bytes && it->second.fingerprint == fp) {
            *dptr = it->second.dptr;
            return B200Q_OK;
        }
        cudaFree(it->second.dptr);
        g_weight_bytes -= static_cast<long long>(it->second.bytes);
        g_weights.erase(it);
    }
    void* d = nullptr;
    int rc = upload_weights(dev, host, bytes, &d);
    if (rc != B200Q_OK) return rc;
    g_weights[key] = WeightEntry{d, bytes, fp};
    g_weight_bytes += static_cast<long long>(bytes);
    *dptr = d;
    return B200Q_OK;
}

// Per host thread, per device: a stream and staging buffers for x / y.
struct Staging {
    int dev = -1;
    cudaStream_t stream = nullptr;
    float* dx = nullptr;
    size_t xcap = 0;
    float* dy = nullptr;
    size_t ycap = 0;
    void* db = nullptr;  // generic device bytes (repack / dequant staging)
    size_t bcap = 0;
    void* db2 = nullptr;
    size_t bcap2 = 0;
};
thread_local std::vector<Staging> t_staging;

Staging* staging_for(int dev) {
    for (auto& s : t_staging)
        if (s.dev == dev) return &s;
    Staging s;
    s.dev = dev;
    if (cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking) != cudaSuccess) return nullptr;
    t_staging.push_back(s);
    return &t_staging.back();
}

int ensure_cap(float** p, size_t* cap, size_t floats) {
    if (*cap >= floats) return B200Q_OK;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    size_t want = floats < 4096 ? 4096 : floats;
    if (cudaMalloc(reinterpret_cast<void**>(p), want * sizeof(float)) != cudaSuccess) return B200Q_ENOMEM;
    *cap = want;
    return B200Q_OK;
}

int ensure_bytes(void** p, size_t* cap, size_t bytes) {
    if (*cap >= bytes) return B200Q_OK;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    const size_t want = std::max<size_t>(bytes + 16, 1u << 16);
    if (cudaMalloc(p, want) != cudaSuccess) return B200Q_ENOMEM;
    *cap = want;
    return B200Q_OK;
}

// Device copy of a cached host matrix, if one is resident and covers
// `need` bytes (no upload).
void* cached_weights(int dev, const void* host, size_t need) {
    std::lock_guard<std::mutex> lk(g_w_mu);
    auto it = g_weights.find(std::make_pair(dev, host));
    if (it != g_weights.end() && it->second.bytes >= need) return it->second.dptr;
    return nullptr;
}

int act_mode_now() {
    if (g_act_mode == 0) g_act_mode = env_act_mode();
    return g_act_mode;
}

// The device address of page-locked host memory allocated or registered
// through CUDA (cudaHostAlloc / cudaMallocHost / cudaHostRegister), else
// nullptr. Only such memory qualifies: ordinary pageable memory is refused
// by cudaHostGetFlags even where the device could reach it otherwise.
void* mapped_host(const void* p) {
    unsigned int flags = 0;
    void* d = nullptr;
    if (cudaHostGetFlags(&flags, const_cast<void*>(p)) != cudaSuccess ||
        cudaHostGetDevicePointer(&d, const_cast<void*>(p), 0) != cudaSuccess) {
        cudaGetLastError();  // clear: p is not CUDA page-locked memory
        return nullptr;
    }
    return d;
}

// Drop-in calls on page-locked buffers replay a CUDA graph of their two
// launches (staging kernel, GEMV): one launch call instead of two on the
// host's critical path. Keyed by everything the graph bakes in; a key is
// captured the second time it is seen (the first call sizes the scratch on
// the direct path). B200Q_DROPIN_GRAPHS=0 disables.
using GraphKey = std::tuple<int, int, int, int, int, int, const void*, const void*, const void*, void*>;
thread_local std::map<GraphKey, cudaGraphExec_t> t_graphs;
thread_local std::map<GraphKey, int> t_graph_seen;
constexpr size_t kMaxDropinGraphs = 512;

bool dropin_graphs_enabled() {
    static const bool on = env_flag("B200Q_DROPIN_GRAPHS", true);
    return on;
}

// Launch (or capture and launch) the staged drop-in; returns false when the
// caller should take the direct path instead.
bool dropin_graph_launch(const GraphKey& key, Staging* s, int qtype, int act, const void* dw, const float* x_mapped,
                         float* y_mapped, int m, int k, int n, Device* dev, int* rc) {
    auto it = t_graphs.find(key);
    if (it == t_graphs.end()) {
        if (t_graph_seen.size() >= 8 * kMaxDropinGraphs) t_graph_seen.clear();  // call sites seen once
        if (++t_graph_seen[key] < 2) return false;
        if (t_graphs.size() >= kMaxDropinGraphs) {
            for (auto& kv : t_graphs) cudaGraphExecDestroy(kv.second);
            t_graphs.clear();
            t_graph_seen.clear();
        }
        cudaGraph_t g = nullptr;
        if (cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        int r = launch_stage_host_rows(x_mapped, s->dx, static_cast<long long>(m) * k, s->stream);
        if (r == B200Q_OK)
            r = launch_gemv(qtype, act, dw, s->dx, y_mapped, m, k, n, k, n, nullptr, dev, s->stream, pdl_enabled(),
                            B200Q_WEIGHTS_STATIC);
        const bool ended = cudaStreamEndCapture(s->stream, &g) == cudaSuccess;
        cudaGraphExec_t ex = nullptr;
        if (r == B200Q_OK && ended && g && cudaGraphInstantiate(&ex, g, 0) != cudaSuccess) ex = nullptr;
        if (g) cudaGraphDestroy(g);
        if (!ex) {
            cudaGetLastError();
            t_graph_seen[key] = -1000000;  // this key stays on the direct path
            return false;
        }
        it = t_graphs.emplace(key, ex).first;
    }
    *rc = cudaGraphLaunch(it->second, s->stream) == cudaSuccess ? B200Q_OK : B200Q_ECUDA;
    return true;
}

// Host-pointer matmul through the device: the body of every drop-in. x and
// y in page-locked host memory are read and written in place by the GPU
// (a staging kernel for x, the GEMV's own stores for y); pageable buffers go
// through DMA copies to and from device staging.
int dropin(int qtype, const float* x, const void* w, float* y, int m, int k, int n) {
    if (!x || !w || !y || m <= 0 || k <= 0 || n <= 0) return B200Q_EINVAL;
    const long long rb = row_bytes_of(qtype, k);
    if (rb < 0) return B200Q_ESHAPE;
    Device* dev = nullptr;
    int rc = current_device_state(&dev);
    if (rc != B200Q_OK) return rc;
    Staging* s = staging_for(dev->id);
    if (!s) return B200Q_ECUDA;
    void* dw = nullptr;
    bool temporary = false;
    rc = weights_for(dev->id, w, static_cast<size_t>(rb) * n, &dw, &temporary);
    if (rc != B200Q_OK) return rc;
    rc = ensure_cap(&s->dx, &s->xcap, static_cast<size_t>(m) * k);
    if (rc == B200Q_OK) rc = ensure_cap(&s->dy, &s->ycap, static_cast<size_t>(m) * n);
    const int act = act_mode_now();
    const float* x_mapped = static_cast<const float*>(mapped_host(x));
    // y straight to host memory only on the GEMV route (the tile path's
    // epilogue and split-K reduction stay on device memory)
    float* y_mapped = uses_tile_path(qtype, act, m, 0) ? nullptr : static_cast<float*>(mapped_host(y));
    bool launched = false;
    if (rc == B200Q_OK) {
        *dev->status_host = 0;
        if (x_mapped && y_mapped && !temporary && dropin_graphs_enabled()) {
            const GraphKey key(dev->id, qtype, act, m, k, n, dw, x_mapped, s->dx, y_mapped);
            launched = dropin_graph_launch(key, s, qtype, act, dw, x_mapped, y_mapped, m, k, n, dev, &rc);
        }
        if (!launched) {
            if (x_mapped)
                rc = launch_stage_host_rows(x_mapped, s->dx, static_cast<long long>(m) * k, s->stream);
            else if (cudaMemcpyAsync(s->dx, x, sizeof(float) * m * k, cudaMemcpyHostToDevice, s->stream) !=
                     cudaSuccess)
                rc = B200Q_ECUDA;
        }
    }
    if (rc == B200Q_OK && !launched)
        rc = launch_gemv(qtype, act, dw, s->dx, y_mapped ? y_mapped : s->dy, m, k, n, k, n, nullptr, dev, s->stream,
                         pdl_enabled(), B200Q_WEIGHTS_STATIC);
    if (rc == B200Q_OK && !y_mapped) {
        if (cudaMemcpyAsync(y, s->dy, sizeof(float) * m * n, cudaMemcpyDeviceToHost, s->stream) != cudaSuccess)
            rc = B200Q_ECUDA;
    }
    if (cudaStreamSynchronize(s->stream) != cudaSuccess && rc == B200Q_OK) rc = B200Q_ECUDA;
    if (rc == B200Q_OK && *dev->status_host != 0) rc = B200Q_ETIMEOUT;
    if (temporary) cudaFree(dw);
    return rc;
}

}  // namespace
}  // namespace b200q

using namespace b200q;

extern "C" {

// ---- drop-ins: matvec ------------------------------------------------------
#define B200Q_MATVEC(name, qt)                                          \
    void name(const float* x, const void* a, float* y, int k, int n) { \
        set_last_error(dropin(qt, x, a, y, 1, k, n));                  \
    }
B200Q_MATVEC(simd_matvec_q4k, QT_Q4_K)
B200Q_MATVEC(simd_matvec_q4k_r4, QT_Q4_K_R4)
B200Q_MATVEC(simd_matvec_q6k, QT_Q6_K)
B200Q_MATVEC(simd_matvec_q6k_r4, QT_Q6_K_R4)
B200Q_MATVEC(simd_matvec_q6k_lm, QT_Q6_K_LM)
B200Q_MATVEC(simd_matvec_q8_0, QT_Q8_0)
B200Q_MATVEC(simd_matvec_q4_0, QT_Q4_0)
#undef B200Q_MATVEC

// ---- drop-ins: matmul ------------------------------------------------------
#define B200Q_MATMUL(name, qt)                                                 \
    void name(const float* x, const void* a, float* y, int m, int k, int n) { \
        set_last_error(dropin(qt, x, a, y, m, k, n));                         \
    }
B200Q_MATMUL(simd_matmul_q4k, QT_Q4_K)
B200Q_MATMUL(simd_matmul_q4k_r4, QT_Q4_K_R4)
B200Q_MATMUL(simd_matmul_q6k, QT_Q6_K)
B200Q_MATMUL(simd_matmul_q6k_r4, QT_Q6_K_R4)
B200Q_MATMUL(simd_matmul_q8_0, QT_Q8_0)
B200Q_MATMUL(simd_matmul_q4_0, QT_Q4_0)
#undef B200Q_MATMUL

// ---- device-pointer API ----------------------------------------------------
int b200q_matmul_ex(int qtype, int act_mode, const float* x, const void* w, float* y, int m, int k, int n, int flags,
                    void* stream) {
    Device* dev = nullptr;
    int rc = current_device_state(&dev);
    if (rc == B200Q_OK)
        rc = launch_gemv(qtype, act_mode, w, x, y, m, k, n, k, n, nullptr, dev, static_cast<cudaStream_t>(stream),
                         pdl_enabled(), flags);
    set_last_error(rc);
    return rc;
}

int b200q_matmul(int qtype, int act_mode, const float* x, const void* w, float* y, int m, int k, int n,
                 void* stream) {
    return b200q_matmul_ex(qtype, act_mode, x, w, y, m, k, n, 0, stream);
}

// model_graph.cpp:731-747 (matvec_quant): the graph dispatches a quantized
// linear by qtype and zero-fills y for a qtype it has no kernel for.
int b200q_matvec_quant(const void* w_quant, int qtype, const float* x, float* y, int cols, int rows, void* stream) {
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    int rc = B200Q_OK;
    FmtInfo f;
    if (!y || rows <= 0) {
        rc = B200Q_EINVAL;
    } else if (!fmt_info(qtype, f)) {
        rc = cudaMemsetAsync(y, 0, static_cast<size_t>(rows) * sizeof(float), st) == cudaSuccess ? B200Q_OK
                                                                                                  : B200Q_ECUDA;
    } else {
        Device* dev = nullptr;
        rc = current_device_state(&dev);
        if (rc == B200Q_OK)
            rc = launch_gemv(qtype, act_mode_now(), w_quant, x, y, 1, cols, rows, cols, rows, nullptr, dev, st,
                             pdl_enabled(), 0);
    }
    set_last_error(rc);
    return rc;
}

// model_graph.cpp:749-760 (matvec_dispatch): fp32 weights when present, else
// the quantized weights when qtype > 0, else a zeroed y.
int b200q_matvec_dispatch(const float* w_f32, const void* w_quant, int qtype, const float* x, float* y, int rows,
                          int cols, void* stream) {
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (w_f32) {
        const int rc = launch_matvec_f32(w_f32, x, y, rows, cols, st);
        set_last_error(rc);
        return rc;
    }
    if (w_quant && qtype > 0) return b200q_matvec_quant(w_quant, qtype, x, y, cols, rows, stream);
    int rc = B200Q_EINVAL;
    if (y && rows > 0)
        rc = cudaMemsetAsync(y, 0, static_cast<size_t>(rows) * sizeof(float), st) == cudaSuccess ? B200Q_OK
                                                                                                  : B200Q_ECUDA;
    set_last_error(rc);
    return rc;
}

int b200q_matvec_isums(int qtype, int act_mode, const float* x, const void* w, float* y, int* isums, int k, int n,
                       void* stream) {
    if (!isums) return B200Q_EINVAL;
    Device* dev = nullptr;
    int rc = current_device_state(&dev);
    if (rc == B200Q_OK)
        rc = launch_gemv(qtype, act_mode, w, x, y, 1, k, n, k, n, reinterpret_cast<int32_t*>(isums), dev,
                         static_cast<cudaStream_t>(stream), false);
    set_last_error(rc);
    return rc;
}

// ---- layout repacks ----------------------------------------------------------
int b200q_repack(int dst_qtype, const void* src, void* dst, int k, int n, void* stream) {
    const int rc = launch_repack(dst_qtype, src, dst, k, n, static_cast<cudaStream_t>(stream));
    set_last_error(rc);
    return rc;
}

namespace {
// Host-pointer repack: upload, repack on the device, download. Returns 1 on
// success, 0 otherwise (quantized_matmul.cpp:250-300 return convention).
int host_repack(int dst_qtype, int src_block, int dst_block, const void* src, void* dst, int k, int n) {
    if (!src || !dst || k <= 0 || n <= 0 || k % 256) {
        set_last_error(B200Q_EINVAL);
        return 0;
    }
    Device* dev = nullptr;
    int rc = current_device_state(&dev);
    Staging* s = rc == B200Q_OK ? staging_for(dev->id) : nullptr;
    if (!s) {
        set_last_error(rc == B200Q_OK ? B200Q_ECUDA : rc);
        return 0;
    }
    const size_t in_bytes = static_cast<size_t>(k / 256) * src_block * n;
    const size_t out_bytes = static_cast<size_t>(k / 256) * dst_block * n;
    rc = ensure_bytes(&s->db, &s->bcap, in_bytes);
    if (rc == B200Q_OK) rc = ensure_bytes(&s->db2, &s->bcap2, out_bytes);
    if (rc == B200Q_OK && cudaMemcpyAsync(s->db, src, in_bytes, cudaMemcpyHostToDevice, s->stream) != cudaSuccess)
        rc = B200Q_ECUDA;
    if (rc == B200Q_OK) rc = launch_repack(dst_qtype, s->db, s->db2, k, n, s->stream);
    if (rc == B200Q_OK && cudaMemcpyAsync(dst, s->db2, out_bytes, cudaMemcpyDeviceToHost, s->stream) != cudaSuccess)
        rc = B200Q_ECUDA;
    if (cudaStreamSynchronize(s->stream) != cudaSuccess && rc == B200Q_OK) rc = B200Q_ECUDA;
    set_last_error(rc);
    return rc == B200Q_OK ? 1 : 0;
}
}  // namespace

int simd_repack_q4k_r4(const void* src_q4k, void* dst_q4k_r4, int k, int n) {
    return host_repack(QT_Q4_K_R4, 144, 144, src_q4k, dst_q4k_r4, k, n);
}
int simd_repack_q6k_r4(const void* src_q6k, void* dst_q6k_r4, int k, int n) {
    return host_repack(QT_Q6_K_R4, 210, 210, src_q6k, dst_q6k_r4, k, n);
}
int simd_repack_q6k_lm(const void* src_q6k, void* dst_q6k_lm, int k, int n) {
    return host_repack(QT_Q6_K_LM, 210, 276, src_q6k, dst_q6k_lm, k, n);
}

// ---- row dequantization -------------------------------------------------------
// ---- decode-step glue ----------------------------------------------------------
int b200q_add_rmsnorm(float* residual, const float* delta, const float* gamma, float* out, int n, int rows, float eps,
                      void* stream) {
    const int rc = launch_add_rmsnorm(residual, delta, gamma, out, n, rows, eps, static_cast<cudaStream_t>(stream));
    set_last_error(rc);
    return rc;
}

int b200q_rope_kv(float* q, float* k, const float* v, int batch, int n_heads, int n_kv_heads, int head_dim, int pos,
                  float theta, void* k_cache, void* v_cache, int max_ctx, void* stream) {
    const int rc = launch_rope_kv(q, k, v, batch, n_heads, n_kv_heads, head_dim, pos, theta, k_cache, v_cache, max_ctx,
                                  static_cast<cudaStream_t>(stream));
    set_last_error(rc);
    return rc;
}

int b200q_attention_decode(const float* q, const void* k_cache, const void* v_cache, float* out, int batch,
                           int n_heads, int n_kv_heads, int head_dim, int ctx_len, int max_ctx, void* stream) {
    Device* dev = nullptr;
    int rc = current_device_state(&dev);
    if (rc == B200Q_OK)
        rc = launch_attention(q, k_cache, v_cache, out, batch, n_heads, n_kv_heads, head_dim, ctx_len, max_ctx, dev,
                              static_cast<cudaStream_t>(stream));
    set_last_error(rc);
    return rc;
}

long long b200q_xq_row_bytes(int k, int act_mode) {
    if (k <= 0 || k % 32 || (act_mode != B200Q_ACT_X8 && act_mode != B200Q_ACT_X16)) return B200Q_EINVAL;
    return xq_bytes_per_row(k, act_mode);
}

int b200q_add_rmsnorm_q(float* residual, const float* delta, const float* gamma, float* out, void* xq, int act_mode,
                        int n, int rows, float eps, void* stream) {
    const int rc = !xq ? B200Q_EINVAL
                       : launch_add_rmsnorm(residual, delta, gamma, out, n, rows, eps,
                                            static_cast<cudaStream_t>(stream), xq, act_mode);
    set_last_error(rc);
    return rc;
}

int b200q_attention_decode_q(const float* q, const void* k_cache, const void* v_cache, float* out, void* xq,
                             int act_mode, int batch, int n_heads, int n_kv_heads, int head_dim, int ctx_len,
                             int max_ctx, void* stream) {
    Device* dev = nullptr;
    int rc = !xq ? B200Q_EINVAL : current_device_state(&dev);
    if (rc == B200Q_OK)
        rc = launch_attention(q, k_cache, v_cache, out, batch, n_heads, n_kv_heads, head_dim, ctx_len, max_ctx, dev,
                              static_cast<cudaStream_t>(stream), xq, act_mode);
    set_last_error(rc);
    return rc;
}

int b200q_rope_attention_decode(const float* q, const float* k, const float* v, int batch, int n_heads, int n_kv_heads,
                                int head_dim, int pos, float theta, void* k_cache, void* v_cache, int max_ctx,
                                float* out, void* xq, int act_mode, void* stream) {
    Device* dev = nullptr;
    int rc = current_device_state(&dev);
    if (rc == B200Q_OK)
        rc = launch_rope_attention(q, k, v, batch, 1, n_heads, n_kv_heads, head_dim, pos, theta, k_cache, v_cache,
                                   max_ctx, out, xq, act_mode, dev, static_cast<cudaStream_t>(stream));
    set_last_error(rc);
    return rc;
}

int b200q_rope_attention_decode_tokens(const float* q, const float* k, const float* v, int batch, int n_tokens,
                                       int n_heads, int n_kv_heads, int head_dim, int pos0, float theta, void* k_cache,
                                       void* v_cache, int max_ctx, float* out, void* xq, int act_mode,
                                       long long q_stride, long long kv_stride, void* stream) {
    Device* dev = nullptr;
    int rc = current_device_state(&dev);
    if (rc == B200Q_OK)
        rc = launch_rope_attention(q, k, v, batch, n_tokens, n_heads, n_kv_heads, head_dim, pos0, theta, k_cache,
                                   v_cache, max_ctx, out, xq, act_mode, dev, static_cast<cudaStream_t>(stream),
                                   q_stride, kv_stride);
    set_last_error(rc);
    return rc;
}

int b200q_rope_attention_decode_paged(const float* q, const float* k, const float* v, int batch, int n_tokens,
                                      int n_heads, int n_kv_heads, int head_dim, int pos, float theta, int kv_mode,
                                      void* k_pages, void* v_pages, float* k_scales, float* v_scales, int n_slots,
                                      int page_size, const int* page_table, int pages_per_seq, float* out, void* xq,
                                      int act_mode, long long q_stride, long long kv_stride, void* stream) {
    Device* dev = nullptr;
    int rc = current_device_state(&dev);
    if (rc == B200Q_OK)
        rc = launch_rope_attention_paged(q, k, v, batch, n_tokens, n_heads, n_kv_heads, head_dim, pos, theta, kv_mode,
                                         k_pages, v_pages, k_scales, v_scales, n_slots, page_size, page_table,
                                         pages_per_seq, out, xq, act_mode, dev, static_cast<cudaStream_t>(stream),
                                         q_stride, kv_stride);
    set_last_error(rc);
    return rc;
}

int b200q_swiglu_q(const float* gate, const float* up, void* xq, int act_mode, int n, void* stream) {
    int rc = B200Q_OK;
    if (!gate || !up || !xq || n <= 0 || (act_mode != B200Q_ACT_X8 && act_mode != B200Q_ACT_X16)) rc = B200Q_EINVAL;
    else if (reinterpret_cast<uintptr_t>(xq) & 15u) rc = B200Q_EALIGN;
    else rc = launch_swiglu_quantize(act_mode, gate, up, n, static_cast<uint8_t*>(xq),
                                     static_cast<cudaStream_t>(stream), pdl_enabled());
    set_last_error(rc);
    return rc;
}

int b200q_matmul_xq(int qtype, int act_mode, const void* xq, const void* w, float* y, int m, int k, int n, float alpha,
                    float beta, int flags, void* stream) {
    Device* dev = nullptr;
    int rc = current_device_state(&dev);
    if (rc == B200Q_OK && (reinterpret_cast<uintptr_t>(xq) & 15u)) rc = B200Q_EALIGN;
    if (rc == B200Q_OK) rc = gemv_check_shape(qtype, act_mode, k, n, dev);
    if (rc == B200Q_OK)
        rc = gemv_from_xq(qtype, act_mode, w, static_cast<const uint8_t*>(xq), xq_bytes_per_row(k, act_mode), y, m, k,
                          n, n, alpha, beta, nullptr, dev, static_cast<cudaStream_t>(stream), pdl_enabled(), flags);
    set_last_error(rc);
    return rc;
}

int b200q_gemv_plan(int qtype, int act_mode, int k, int n, int rows_per_launch, int fused_quantize, int num_sms,
                    long long* out, int out_len) {
    return gemv_plan_info(qtype, act_mode, k, n, rows_per_launch, fused_quantize != 0, num_sms, out, out_len);
}

int b200q_matmul_norm(int qtype, int act_mode, const float* x, const float* gamma, float eps, const void* w, float* y,
                      int k, int n, float alpha, float beta, int flags, void* stream) {
    Device* dev = nullptr;
    int rc = current_device_state(&dev);
    if (rc == B200Q_OK && (reinterpret_cast<uintptr_t>(x) & 15u)) rc = B200Q_EALIGN;
    if (rc == B200Q_OK) rc = gemv_check_shape(qtype, act_mode, k, n, dev);
    if (rc == B200Q_OK)
        rc = gemv_norm_f32(qtype, act_mode, w, x, gamma, eps, y, k, n, alpha, beta, dev,
                           static_cast<cudaStream_t>(stream), pdl_enabled(), flags);
    set_last_error(rc);
    return rc;
}

int b200q_matmul_swiglu(int qtype, int act_mode, const float* gate, const float* up, const void* w, float* y, int k,
                        int n, float alpha, float beta, int flags, void* stream) {
    Device* dev = nullptr;
    int rc = current_device_state(&dev);
    if (rc == B200Q_OK && (reinterpret_cast<uintptr_t>(gate) & 15u)) rc = B200Q_EALIGN;
    if (rc == B200Q_OK) rc = gemv_check_shape(qtype, act_mode, k, n, dev);
    if (rc == B200Q_OK)
        rc = gemv_swiglu_f32(qtype, act_mode, w, gate, up, y, k, n, alpha, beta, dev, static_cast<cudaStream_t>(stream),
                             pdl_enabled(), flags);
    set_last_error(rc);
    return rc;
}

int b200q_swiglu_rows(const float* gate_up, float* out, int rows, int n, void* stream) {
    const int rc = launch_swiglu_rows(gate_up, out, rows, n, static_cast<cudaStream_t>(stream));
    set_last_error(rc);
    return rc;
}

int b200q_swiglu(const float* gate, const float* up, float* out, long long n, void* stream) {
    const int rc = launch_swiglu(gate, up, out, n, static_cast<cudaStream_t>(stream));
    set_last_error(rc);
    return rc;
}

int b200q_unshard_rows(const float* in, float* out, int shards, int rows, int cols, void* stream) {
    const int rc = launch_unshard_rows(in, out, shards, rows, cols, static_cast<cudaStream_t>(stream));
    set_last_error(rc);
    return rc;
}

// ---- multi-GPU: IPC-shared buffers and the peer all-gather ----------------------
static_assert(sizeof(cudaIpcMemHandle_t) <= B200Q_IPC_HANDLE_BYTES, "IPC handle size");

int b200q_ipc_alloc(long long bytes, void** dptr, void* handle) {
    int rc = B200Q_OK;
    if (bytes <= 0 || !dptr || !handle) rc = B200Q_EINVAL;
    void* p = nullptr;
    if (rc == B200Q_OK && cudaMalloc(&p, static_cast<size_t>(bytes)) != cudaSuccess) rc = B200Q_ENOMEM;
    // zeroed (flags start at 0) before the handle can reach another process
    if (rc == B200Q_OK && (cudaMemset(p, 0, static_cast<size_t>(bytes)) != cudaSuccess ||
                           cudaDeviceSynchronize() != cudaSuccess))
        rc = B200Q_ECUDA;
    cudaIpcMemHandle_t h;
    if (rc == B200Q_OK && cudaIpcGetMemHandle(&h, p) != cudaSuccess) rc = B200Q_ECUDA;
    if (rc == B200Q_OK) {
        std::memset(handle, 0, B200Q_IPC_HANDLE_BYTES);
        std::memcpy(handle, &h, sizeof(h));
        *dptr = p;
    } else if (p) {
        cudaFree(p);
    }
    set_last_error(rc);
    return rc;
}

int b200q_ipc_open(const void* handle, void** dptr) {
    int rc = (!handle || !dptr) ? B200Q_EINVAL : B200Q_OK;
    if (rc == B200Q_OK) {
        cudaIpcMemHandle_t h;
        std::memcpy(&h, handle, sizeof(h));
        if (cudaIpcOpenMemHandle(dptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) rc = B200Q_ECUDA;
    }
    set_last_error(rc);
    return rc;
}

int b200q_ipc_close(void* dptr) {
    const int rc = !dptr ? B200Q_EINVAL : (cudaIpcCloseMemHandle(dptr) == cudaSuccess ? B200Q_OK : B200Q_ECUDA);
    set_last_error(rc);
    return rc;
}

int b200q_ipc_free(void* dptr) {
    const int rc = !dptr ? B200Q_EINVAL : (cudaFree(dptr) == cudaSuccess ? B200Q_OK : B200Q_ECUDA);
    set_last_error(rc);
    return rc;
}

int b200q_allgather_peer(const float* local, int rows, int n_local, void* const* bases, long long data_offset,
                         long long flags_offset, int rank, int world, void* counters, int slot, void* xq, int act_mode,
                         void* stream) {
    Device* dev = nullptr;
    int rc = current_device_state(&dev);
    if (rc == B200Q_OK)
        rc = launch_allgather_peer(local, rows, n_local, bases, data_offset, flags_offset, rank, world,
                                   static_cast<uint32_t*>(counters), slot, dev, static_cast<cudaStream_t>(stream), xq,
                                   act_mode);
    set_last_error(rc);
    return rc;
}

int b200q_quantize_rows(int act_mode, const float* x, int rows, int k, void* xq, void* stream) {
    int rc = (!x || !xq || rows <= 0 || k <= 0) ? B200Q_EINVAL : B200Q_OK;
    if (rc == B200Q_OK && (reinterpret_cast<uintptr_t>(xq) & 15u)) rc = B200Q_EALIGN;
    if (rc == B200Q_OK) rc = launch_quantize_rows(act_mode, x, rows, k, static_cast<uint8_t*>(xq),
                                                  static_cast<cudaStream_t>(stream), pdl_enabled());
    set_last_error(rc);
    return rc;
}

int b200q_dequantize_rows(int qtype, const void* w, const int* rows, int nrows, float* out, int k, int n, void* stream) {
    const int rc = launch_dequant_rows(qtype, w, rows, nrows, out, k, n, true, static_cast<cudaStream_t>(stream));
    set_last_error(rc);
    return rc;
}

int simd_dequantize_row(const void* quant_data, int qtype, int row, float* out, int k) {
    FmtInfo f;
    if (!quant_data || !out || row < 0 || k <= 0 || !fmt_info(qtype, f) || k % f.elems) {
        set_last_error(B200Q_EINVAL);
        return 0;
    }
    Device* dev = nullptr;
    int rc = current_device_state(&dev);
    Staging* s = rc == B200Q_OK ? staging_for(dev->id) : nullptr;
    if (!s) {
        set_last_error(rc == B200Q_OK ? B200Q_ECUDA : rc);
        return 0;
    }
    // Bytes the reference addressing reads for this row: the row itself, or
    // its whole 4-row group for the R4 layouts (group = row / 4).
    const size_t rb = static_cast<size_t>(k / f.elems) * f.bytes;
    const size_t off = f.r4 ? static_cast<size_t>(row / 4) * 4 * rb : static_cast<size_t>(row) * rb;
    const size_t len = f.r4 ? 4 * rb : rb;
    const int local_row = f.r4 ? row % 4 : 0;
    const void* dw = cached_weights(dev->id, quant_data, off + len);
    int rows_host[1] = {dw ? row : local_row};
    rc = ensure_bytes(&s->db, &s->bcap, (dw ? 0 : len) + 16);
    if (rc == B200Q_OK) rc = ensure_cap(&s->dy, &s->ycap, static_cast<size_t>(k));
    uint8_t* dbytes = static_cast<uint8_t*>(s->db);
    int* drow = reinterpret_cast<int*>(dbytes);
    uint8_t* dsrc = dbytes + 16;
    if (rc == B200Q_OK && !dw &&
        cudaMemcpyAsync(dsrc, static_cast<const uint8_t*>(quant_data) + off, len, cudaMemcpyHostToDevice, s->stream) !=
            cudaSuccess)
        rc = B200Q_ECUDA;
    if (rc == B200Q_OK && cudaMemcpyAsync(drow, rows_host, sizeof(int), cudaMemcpyHostToDevice, s->stream) != cudaSuccess)
        rc = B200Q_ECUDA;
    if (rc == B200Q_OK)
        rc = launch_dequant_rows(qtype, dw ? dw : static_cast<const void*>(dsrc), drow, 1, s->dy, k, dw ? 0 : 4, false,
                                 s->stream);
    if (rc == B200Q_OK && cudaMemcpyAsync(out, s->dy, sizeof(float) * k, cudaMemcpyDeviceToHost, s->stream) != cudaSuccess)
        rc = B200Q_ECUDA;
    if (cudaStreamSynchronize(s->stream) != cudaSuccess && rc == B200Q_OK) rc = B200Q_ECUDA;
    set_last_error(rc);
    return rc == B200Q_OK ? 1 : 0;
}

// ---- fused multi-matrix matvec (one activation quantization) -----------------
int b200q_fused_matvec(int act_mode, const float* x, int cols, int count, const void* const* w, const int* qtypes,
                       float* const* y, const int* rows, int flags, void* stream) {
    Device* dev = nullptr;
    int rc = current_device_state(&dev);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (rc == B200Q_OK && (!x || !w || !qtypes || !y || !rows || count <= 0 || cols <= 0)) rc = B200Q_EINVAL;
    for (int i = 0; rc == B200Q_OK && i < count; ++i) {
        if (!w[i] || !y[i] || rows[i] <= 0) rc = B200Q_EINVAL;
        else rc = gemv_check_shape(qtypes[i], act_mode, cols, rows[i], dev);
    }
    const uint8_t* xq = nullptr;
    long long xq_row = 0;
    if (rc == B200Q_OK) rc = quantize_activations(act_mode, x, cols, 1, cols, dev, st, pdl_enabled(), 1, &xq, &xq_row);
    for (int i = 0; rc == B200Q_OK && i < count; ++i)
        rc = gemv_from_xq(qtypes[i], act_mode, w[i], xq, xq_row, y[i], 1, cols, rows[i], rows[i], 1.0f, 0.0f, nullptr,
                          dev, st, pdl_enabled(), flags);
    set_last_error(rc);
    return rc;
}

namespace {
bool fused_supported(int q) { return q == QT_Q4_K || q == QT_Q4_K_R4 || q == QT_Q6_K || q == QT_Q6_K_R4; }

// Host-pointer fused matvec: count matrices sharing x (quantized_matmul.cpp:
// 1855-1942). Returns 1 on success, 0 on invalid arguments (outputs untouched).
int host_fused(const float* x, int cols, int count, const void* const* data, const int* qt, float* const* outs,
               const int* rows) {
    if (!x || cols <= 0) return 0;
    for (int i = 0; i < count; ++i)
        if (!data[i] || !outs[i] || rows[i] <= 0 || !fused_supported(qt[i]) || row_bytes_of(qt[i], cols) < 0) return 0;
    Device* dev = nullptr;
    int rc = current_device_state(&dev);
    Staging* s = rc == B200Q_OK ? staging_for(dev->id) : nullptr;
    if (!s) {
        set_last_error(rc == B200Q_OK ? B200Q_ECUDA : rc);
        return 0;
    }
    const void* dws[4];
    float* dys[4];
    size_t total_rows = 0;
    for (int i = 0; i < count; ++i) total_rows += static_cast<size_t>(rows[i]);
    rc = ensure_cap(&s->dx, &s->xcap, static_cast<size_t>(cols));
    if (rc == B200Q_OK) rc = ensure_cap(&s->dy, &s->ycap, total_rows);
    size_t o = 0;
    for (int i = 0; rc == B200Q_OK && i < count; ++i) {
        bool temporary = false;
        void* dw = nullptr;
        rc = weights_for(dev->id, data[i], static_cast<size_t>(row_bytes_of(qt[i], cols)) * rows[i], &dw, &temporary);
        if (temporary) {  // residency disabled: keep the upload for this call only
            cudaStreamSynchronize(s->stream);
        }
        dws[i] = dw;
        dys[i] = s->dy + o;
        o += static_cast<size_t>(rows[i]);
    }
    if (rc == B200Q_OK && cudaMemcpyAsync(s->dx, x, sizeof(float) * cols, cudaMemcpyHostToDevice, s->stream) != cudaSuccess)
        rc = B200Q_ECUDA;
    if (rc == B200Q_OK) {
        *dev->status_host = 0;
        rc = b200q_fused_matvec(act_mode_now(), s->dx, cols, count, dws, qt, dys, rows, B200Q_WEIGHTS_STATIC, s->stream);
    }
    for (int i = 0; rc == B200Q_OK && i < count; ++i)
        if (cudaMemcpyAsync(outs[i], dys[i], sizeof(float) * rows[i], cudaMemcpyDeviceToHost, s->stream) != cudaSuccess)
            rc = B200Q_ECUDA;
    if (cudaStreamSynchronize(s->stream) != cudaSuccess && rc == B200Q_OK) rc = B200Q_ECUDA;
    if (rc == B200Q_OK && *dev->status_host != 0) rc = B200Q_ETIMEOUT;
    set_last_error(rc);
    return rc == B200Q_OK ? 1 : 0;
}
}  // namespace

int simd_fused_qkv_matvec_quant(const float* x, const void* q_data, int q_qtype, float* q_out, int q_rows,
                                const void* k_data, int k_qtype, float* k_out, int k_rows, const void* v_data,
                                int v_qtype, float* v_out, int v_rows, int cols) {
    const void* d[3] = {q_data, k_data, v_data};
    const int qt[3] = {q_qtype, k_qtype, v_qtype};
    float* o[3] = {q_out, k_out, v_out};
    const int r[3] = {q_rows, k_rows, v_rows};
    return host_fused(x, cols, 3, d, qt, o, r);
}

int simd_fused_quad_matvec_quant(const float* x, const void* a_data, int a_qtype, float* a_out, int a_rows,
                                 const void* b_data, int b_qtype, float* b_out, int b_rows, const void* c_data,
                                 int c_qtype, float* c_out, int c_rows, const void* d_data, int d_qtype, float* d_out,
                                 int d_rows, int cols) {
    const void* d[4] = {a_data, b_data, c_data, d_data};
    const int qt[4] = {a_qtype, b_qtype, c_qtype, d_qtype};
    float* o[4] = {a_out, b_out, c_out, d_out};
    const int r[4] = {a_rows, b_rows, c_rows, d_rows};
    return host_fused(x, cols, 4, d, qt, o, r);
}

// ---- fused SwiGLU expert and MoE FFN -------------------------------------------
int b200q_expert_swiglu(int act_mode, const float* x, int in_dim, const void* gate, int gq, int hidden, const void* up,
                        int uq, const void* down, int dq, int out_dim, float* out, float alpha, float beta, int flags,
                        void* stream) {
    Device* dev = nullptr;
    int rc = current_device_state(&dev);
    if (rc == B200Q_OK)
        rc = expert_swiglu(act_mode, x, in_dim, gate, gq, hidden, up, uq, down, dq, out_dim, out, alpha, beta, dev,
                           static_cast<cudaStream_t>(stream), pdl_enabled(), flags);
    set_last_error(rc);
    return rc;
}

int b200q_moe_ffn(int act_mode, const float* x, int in_dim, const int* expert_indices, const float* expert_weights,
                  int top_k, const void* const* gate_ptrs, int gq, int hidden, const void* const* up_ptrs, int uq,
                  const void* const* down_ptrs, int dq, int out_dim, float* out, int write_mode, int flags,
                  void* stream) {
    Device* dev = nullptr;
    int rc = current_device_state(&dev);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (rc == B200Q_OK && (!x || !out || top_k <= 0 || !expert_indices || !expert_weights)) rc = B200Q_EINVAL;
    // Experts with a non-positive weight or a missing matrix are skipped;
    // write_mode 0 overwrites out (zero when no expert contributes), other
    // values accumulate into it (quantized_matmul.cpp:2426-2525).
    bool have = write_mode != 0;
    for (int e = 0; rc == B200Q_OK && e < top_k; ++e) {
        const int idx = expert_indices[e];
        const float w = expert_weights[e];
        if (!(w > 0.0f) || idx < 0) continue;
        if (!gate_ptrs[idx] || !up_ptrs[idx] || !down_ptrs[idx]) continue;
        rc = expert_swiglu(act_mode, x, in_dim, gate_ptrs[idx], gq, hidden, up_ptrs[idx], uq, down_ptrs[idx], dq, out_dim,
                           out, w, have ? 1.0f : 0.0f, dev, st, pdl_enabled(), flags);
        have = true;
    }
    if (rc == B200Q_OK && !have && cudaMemsetAsync(out, 0, sizeof(float) * out_dim, st) != cudaSuccess) rc = B200Q_ECUDA;
    set_last_error(rc);
    return rc;
}

namespace {
bool ffn_supported(int q) { return fused_supported(q) || q == QT_Q6_K_LM || q == QT_Q8_0; }

// Upload one expert's three matrices (resident cache) and return device
// pointers.
int resolve_expert(int dev, const void* g, int gq, const void* u, int uq, const void* d, int dq, int in_dim,
                   int hidden, int out_dim, const void** dg, const void** du, const void** dd) {
    bool t = false;
    void* p = nullptr;
    int rc = weights_for(dev, g, static_cast<size_t>(row_bytes_of(gq, in_dim)) * hidden, &p, &t);
    *dg = p;
    if (rc == B200Q_OK) rc = weights_for(dev, u, static_cast<size_t>(row_bytes_of(uq, in_dim)) * hidden, &p, &t);
    *du = p;
    if (rc == B200Q_OK) rc = weights_for(dev, d, static_cast<size_t>(row_bytes_of(dq, hidden)) * out_dim, &p, &t);
    *dd = p;
    return rc;
}
}  // namespace

void simd_fused_expert_swiglu(const float* x, int in_dim, const void* gate_data, int gate_qtype, int hidden_dim,
                              const void* up_data, int up_qtype, const void* down_data, int down_qtype, int out_dim,
                              float* output) {
    if (!x || !output || in_dim <= 0 || hidden_dim <= 0 || out_dim <= 0 || !gate_data || !up_data || !down_data ||
        !ffn_supported(gate_qtype) || !ffn_supported(up_qtype) || !ffn_supported(down_qtype) ||
        row_bytes_of(gate_qtype, in_dim) < 0 || row_bytes_of(up_qtype, in_dim) < 0 ||
        row_bytes_of(down_qtype, hidden_dim) < 0) {
        set_last_error(B200Q_EINVAL);
        return;
    }
    Device* dev = nullptr;
    int rc = current_device_state(&dev);
    Staging* s = rc == B200Q_OK ? staging_for(dev->id) : nullptr;
    if (!s) {
        set_last_error(rc == B200Q_OK ? B200Q_ECUDA : rc);
        return;
    }
    const void *dg = nullptr, *du = nullptr, *dd = nullptr;
    rc = resolve_expert(dev->id, gate_data, gate_qtype, up_data, up_qtype, down_data, down_qtype, in_dim, hidden_dim,
                        out_dim, &dg, &du, &dd);
    if (rc == B200Q_OK) rc = ensure_cap(&s->dx, &s->xcap, static_cast<size_t>(in_dim));
    if (rc == B200Q_OK) rc = ensure_cap(&s->dy, &s->ycap, static_cast<size_t>(out_dim));
    if (rc == B200Q_OK && cudaMemcpyAsync(s->dx, x, sizeof(float) * in_dim, cudaMemcpyHostToDevice, s->stream) != cudaSuccess)
        rc = B200Q_ECUDA;
    if (rc == B200Q_OK) {
        *dev->status_host = 0;
        rc = expert_swiglu(act_mode_now(), s->dx, in_dim, dg, gate_qtype, hidden_dim, du, up_qtype, dd, down_qtype,
                           out_dim, s->dy, 1.0f, 0.0f, dev, s->stream, pdl_enabled(), B200Q_WEIGHTS_STATIC);
    }
    if (rc == B200Q_OK &&
        cudaMemcpyAsync(output, s->dy, sizeof(float) * out_dim, cudaMemcpyDeviceToHost, s->stream) != cudaSuccess)
        rc = B200Q_ECUDA;
    if (cudaStreamSynchronize(s->stream) != cudaSuccess && rc == B200Q_OK) rc = B200Q_ECUDA;
    if (rc == B200Q_OK && *dev->status_host != 0) rc = B200Q_ETIMEOUT;
    set_last_error(rc);
}

void simd_fused_moe_ffn(const float* x, int in_dim, const int* expert_indices, const float* expert_weights, int top_k,
                        const void* const* gate_data_ptrs, int gate_qtype, int hidden_dim,
                        const void* const* up_data_ptrs, int up_qtype, const void* const* down_data_ptrs,
                        int down_qtype, int out_dim, float* output, int write_mode) {
    if (!x || !output || top_k <= 0 || !expert_indices || !expert_weights || !gate_data_ptrs || !up_data_ptrs ||
        !down_data_ptrs || in_dim <= 0 || hidden_dim <= 0 || out_dim <= 0 || !ffn_supported(gate_qtype) ||
        !ffn_supported(up_qtype) || !ffn_supported(down_qtype)) {
        set_last_error(B200Q_EINVAL);
        return;
    }
    Device* dev = nullptr;
    int rc = current_device_state(&dev);
    Staging* s = rc == B200Q_OK ? staging_for(dev->id) : nullptr;
    if (!s) {
        set_last_error(rc == B200Q_OK ? B200Q_ECUDA : rc);
        return;
    }
    rc = ensure_cap(&s->dx, &s->xcap, static_cast<size_t>(in_dim));
    if (rc == B200Q_OK) rc = ensure_cap(&s->dy, &s->ycap, static_cast<size_t>(out_dim));
    if (rc == B200Q_OK && cudaMemcpyAsync(s->dx, x, sizeof(float) * in_dim, cudaMemcpyHostToDevice, s->stream) != cudaSuccess)
        rc = B200Q_ECUDA;
    if (rc == B200Q_OK && write_mode != 0 &&
        cudaMemcpyAsync(s->dy, output, sizeof(float) * out_dim, cudaMemcpyHostToDevice, s->stream) != cudaSuccess)
        rc = B200Q_ECUDA;
    // Resolve each contributing expert's device copies (same skip rules).
    std::vector<const void*> g(top_k, nullptr), u(top_k, nullptr), d(top_k, nullptr);
    std::vector<int> idx(top_k);
    for (int e = 0; rc == B200Q_OK && e < top_k; ++e) {
        idx[e] = e;
        const int i = expert_indices[e];
        if (!(expert_weights[e] > 0.0f) || i < 0) continue;
        if (!gate_data_ptrs[i] || !up_data_ptrs[i] || !down_data_ptrs[i]) continue;
        rc = resolve_expert(dev->id, gate_data_ptrs[i], gate_qtype, up_data_ptrs[i], up_qtype, down_data_ptrs[i],
                            down_qtype, in_dim, hidden_dim, out_dim, &g[e], &u[e], &d[e]);
    }
    if (rc == B200Q_OK) {
        *dev->status_host = 0;
        rc = b200q_moe_ffn(act_mode_now(), s->dx, in_dim, idx.data(), expert_weights, top_k, g.data(), gate_qtype,
                           hidden_dim, u.data(), up_qtype, d.data(), down_qtype, out_dim, s->dy, write_mode,
                           B200Q_WEIGHTS_STATIC, s->stream);
    }
    if (rc == B200Q_OK &&
        cudaMemcpyAsync(output, s->dy, sizeof(float) * out_dim, cudaMemcpyDeviceToHost, s->stream) != cudaSuccess)
        rc = B200Q_ECUDA;
    if (cudaStreamSynchronize(s->stream) != cudaSuccess && rc == B200Q_OK) rc = B200Q_ECUDA;
    if (rc == B200Q_OK && *dev->status_host != 0) rc = B200Q_ETIMEOUT;
    set_last_error(rc);
}

// ---- controls ----------------------------------------------------------------
int b200q_set_act_mode(int act_mode) {
    const int prev = act_mode_now();
    if (act_mode == B200Q_ACT_X8 || act_mode == B200Q_ACT_X16) g_act_mode = act_mode;
    return prev;
}

int b200q_get_act_mode(void) { return act_mode_now(); }

int b200q_last_error(void) { return t_last_error; }

const char* b200q_status_string(int status) {
    switch (status) {
        case B200Q_OK: return "ok";
        case B200Q_EINVAL: return "invalid argument";
        case B200Q_EQTYPE: return "unsupported qtype";
        case B200Q_ESHAPE: return "unsupported shape";
        case B200Q_EALIGN: return "pointer not 16-byte aligned";
        case B200Q_ECUDA: return "CUDA runtime error";
        case B200Q_ENOMEM: return "device allocation failed";
        case B200Q_ETIMEOUT: return "kernel pipeline wait timed out";
        case B200Q_ENODEV: return "no usable sm_100 device";
        case B200Q_ECAPTURE: return "scratch must grow during stream capture";
        case B200Q_ESCRATCH: return "request larger than the fixed no-alloc scratch";
        case B200Q_EPAGE: return "page table entry names no page or one outside the pool";
        default: return "unknown status";
    }
}

int b200q_device_status(int device) {
    if (device < 0) return B200Q_ENODEV;
    // Reads only what exists: the host-mapped word of the regular entry
    // points and the word inside b200q_matvec_noalloc's fixed array; neither
    // is created here, so this allocates nothing.
    int v = noalloc_take_status(device);
    if (v < 0) return v;
    if (Device* d = device_state_if_present(device)) {
        v |= *d->status_host;
        *d->status_host = 0;
    }
    return v;
}

long long b200q_set_peer_wait_ns(long long ns) { return set_peer_wait_ns(ns); }

void b200q_weight_cache_clear(void) {
    std::lock_guard<std::mutex> lk(g_w_mu);
    for (auto& kv : g_weights) {
        int prev = -1;
        cudaGetDevice(&prev);
        cudaSetDevice(kv.first.first);
        cudaFree(kv.second.dptr);
        if (prev >= 0) cudaSetDevice(prev);
    }
    g_weights.clear();
    g_weight_bytes = 0;
}

int b200q_weight_cache_evict(const void* host_ptr) {
    std::lock_guard<std::mutex> lk(g_w_mu);
    int freed = 0;
    for (auto it = g_weights.begin(); it != g_weights.end();) {
        if (it->first.second == host_ptr) {
            int prev = -1;
            cudaGetDevice(&prev);
            cudaSetDevice(it->first.first);
            cudaFree(it->second.dptr);
            if (prev >= 0) cudaSetDevice(prev);
            g_weight_bytes -= static_cast<long long>(it->second.bytes);
            it = g_weights.erase(it);
            freed = 1;
        } else {
            ++it;
        }
    }
    return freed;
}

long long b200q_weight_cache_bytes(void) {
    std::lock_guard<std::mutex> lk(g_w_mu);
    return g_weight_bytes;
}

int b200q_set_pdl(int enable) {
    const int prev = pdl_enabled() ? 1 : 0;
    g_pdl = enable ? 1 : 0;
    return prev;
}

const char* b200q_version(void) { return "b200q 0.1 (sm_100a)"; }

}  // extern "C"
