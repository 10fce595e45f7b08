// b200q_matvec_noalloc: the decode matvec without any allocation.
//
// Some callers cannot let a library allocate device memory inside a call:
// an engine whose caching allocator or memory pool owns all of HBM after
// start-up (a cudaMalloc there fails or fragments the pool), a decode loop
// with a latency budget that cannot absorb cudaMalloc/cudaFree (cudaFree
// synchronises the device), and embedders that account for every byte of
// device memory before serving starts. The regular entry points size a
// per-stream scratch buffer on first use; this one instead keeps its only
// scratch -- the quantized activation row and a status word -- in a fixed
// array that is part of the library's device image, so every GPU that loads
// the library holds it (B200Q_NOALLOC_SCRATCH_BYTES) until the process exits.
//
// Set-up: the first call on a device (with that device current) resolves the
// array's device address with cudaGetSymbolAddress and reads the device's
// attributes; make that first call before any stream capture. Later calls
// only launch work: a memset of the status word, the activation quantizer
// and the GEMV kernel.
//
// Every call on every stream shares the one array and it keeps the last
// call's contents: calls that overlap on the GPU (different streams, or
// different host threads without ordering) race on it.
#include <mutex>

#include "gemv.cuh"
#include "internal.h"

namespace b200q {
namespace {

constexpr size_t kStatusBytes = 256;  // status word, padded to keep the codes 256-byte aligned
constexpr size_t kCodeBytes = B200Q_NOALLOC_SCRATCH_BYTES - kStatusBytes;
constexpr int kMaxDevices = 64;

// The array's name is a host-side stand-in: the device address is obtained
// per device with cudaGetSymbolAddress.
static __device__ __align__(256) uint8_t g_noalloc_scratch[B200Q_NOALLOC_SCRATCH_BYTES];

struct NoAllocDevice {
    bool ready = false;
    uint8_t* base = nullptr;  // device address of g_noalloc_scratch on this device
    Device dev;               // status points into the array; no host-mapped word
};

std::mutex g_mu;
NoAllocDevice g_devices[kMaxDevices];

int setup_current_device(NoAllocDevice** out) {
    int d = -1;
    if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= kMaxDevices) return B200Q_ENODEV;
    std::lock_guard<std::mutex> lk(g_mu);
    NoAllocDevice& s = g_devices[d];
    if (!s.ready) {
        int major = 0, sms = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, d) != cudaSuccess || major != 10)
            return B200Q_ENODEV;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, d) != cudaSuccess || sms <= 0)
            return B200Q_ENODEV;
        void* ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr) return B200Q_ECUDA;
        s.base = static_cast<uint8_t*>(ptr);
        s.dev.id = d;
        s.dev.num_sms = sms;
        s.dev.status = reinterpret_cast<volatile int*>(s.base);
        s.ready = true;
    }
    *out = &s;
    return B200Q_OK;
}

template <int DIG>
cudaError_t launch_quantize_row(const float* x, int k, uint8_t* xq, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>((k / 32 + 127) / 128));
    cfg.blockDim = dim3(128);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, b200q_quantize_act_kernel<DIG>, x, static_cast<long long>(k), 1, k, xq);
}

int matvec_noalloc(int qtype, int act_mode, const float* x, const void* w, float* y, int k, int n,
                   cudaStream_t st) {
    if (!x || !w || !y || k <= 0 || n <= 0) return B200Q_EINVAL;
    if (act_mode != B200Q_ACT_X8 && act_mode != B200Q_ACT_X16) return B200Q_EINVAL;
    if ((reinterpret_cast<uintptr_t>(w) & 15u) || (reinterpret_cast<uintptr_t>(x) & 15u)) return B200Q_EALIGN;
    if (k % 32) return B200Q_ESHAPE;
    const long long xq_row = xq_bytes_per_row(k, act_mode);
    if (xq_row > static_cast<long long>(kCodeBytes)) return B200Q_ESCRATCH;
    NoAllocDevice* s = nullptr;
    int rc = setup_current_device(&s);
    if (rc != B200Q_OK) return rc;
    rc = gemv_check_shape(qtype, act_mode, k, n, &s->dev);
    if (rc != B200Q_OK) return rc;
    uint8_t* xq = s->base + kStatusBytes;
    if (cudaMemsetAsync(s->base, 0, sizeof(int), st) != cudaSuccess) return B200Q_ECUDA;
    const bool pdl = pdl_enabled();
    const cudaError_t e = act_mode == B200Q_ACT_X8 ? launch_quantize_row<1>(x, k, xq, st, pdl)
                                                   : launch_quantize_row<2>(x, k, xq, st, pdl);
    if (e != cudaSuccess) return B200Q_ECUDA;
    return gemv_from_xq(qtype, act_mode, w, xq, xq_row, y, 1, k, n, n, 1.0f, 0.0f, nullptr, &s->dev, st, pdl, 0);
}

}  // namespace

int noalloc_take_status(int device) {
    if (device < 0 || device >= kMaxDevices) return 0;
    uint8_t* base = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!g_devices[device].ready) return 0;
        base = g_devices[device].base;
    }
    // A synchronous copy of the word out of the fixed array and a reset to
    // zero (no allocation); the caller reads it after the call's stream has
    // finished.
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) return B200Q_ECUDA;
    if (prev != device && cudaSetDevice(device) != cudaSuccess) return B200Q_ECUDA;
    int v = 0;
    cudaError_t e = cudaMemcpy(&v, base, sizeof(int), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && v != 0) e = cudaMemset(base, 0, sizeof(int));
    if (prev != device) cudaSetDevice(prev);
    return e == cudaSuccess ? v : B200Q_ECUDA;
}

}  // namespace b200q

extern "C" int b200q_matvec_noalloc(int qtype, int act_mode, const float* x, const void* w, float* y, int k, int n,
                                    void* stream) {
    const int rc = b200q::matvec_noalloc(qtype, act_mode, x, w, y, k, n, static_cast<cudaStream_t>(stream));
    b200q::set_last_error(rc);
    return rc;
}
