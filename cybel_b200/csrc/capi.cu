// C ABI of libb200q.so (declared in include/b200q.h): per-device state, the
// resident weight cache behind the host-pointer drop-ins, and the drop-in and
// device-pointer entry points.
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
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
};
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
    if (it != g_weights.end()) {
        if (it->second.bytes == bytes) {
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
    g_weights[key] = WeightEntry{d, bytes};
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

int act_mode_now() {
    if (g_act_mode == 0) g_act_mode = env_act_mode();
    return g_act_mode;
}

// Host-pointer matmul through the device: the body of every drop-in.
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
    if (rc == B200Q_OK) {
        *dev->status_host = 0;
        if (cudaMemcpyAsync(s->dx, x, sizeof(float) * m * k, cudaMemcpyHostToDevice, s->stream) != cudaSuccess)
            rc = B200Q_ECUDA;
    }
    if (rc == B200Q_OK)
        rc = launch_gemv(qtype, act_mode_now(), dw, s->dx, s->dy, m, k, n, k, n, nullptr, dev, s->stream, pdl_enabled(),
                         B200Q_WEIGHTS_STATIC);
    if (rc == B200Q_OK) {
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
        default: return "unknown status";
    }
}

int b200q_device_status(int device) {
    int err = B200Q_OK;
    Device* d = device_state(device, &err);
    if (!d) return err;
    const int v = *d->status_host;
    *d->status_host = 0;
    return v;
}

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
