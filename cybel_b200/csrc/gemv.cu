// Launch planning and dispatch for the decode GEMV kernels (gemv.cuh).
#include <algorithm>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>
#include <utility>

#include "gemv.cuh"
#include "internal.h"

namespace b200q {

bool fmt_info(int qtype, FmtInfo& f) {
    switch (qtype) {
        case QT_Q4_K: f = {256, 144, 2, 16, 32, false}; return true;
        case QT_Q4_K_R4: f = {256, 144, 2, 16, 32, true}; return true;
        case QT_Q6_K: f = {256, 210, 8, 4, 16, false}; return true;
        case QT_Q6_K_R4: f = {256, 210, 8, 4, 16, true}; return true;
        case QT_Q6_K_LM: f = {256, 276, 8, 4, 16, false}; return true;
        case QT_Q8_0: f = {32, 34, 1, 64, 32, false}; return true;
        case QT_Q4_0: f = {32, 18, 1, 64, 32, false}; return true;
        default: return false;
    }
}

long long row_bytes_of(int qtype, int k) {
    FmtInfo f;
    if (!fmt_info(qtype, f) || k <= 0 || k % f.elems) return -1;
    return static_cast<long long>(k / f.elems) * f.bytes;
}

namespace {

int env_int(const char* name, int dflt) {
    const char* e = std::getenv(name);
    if (!e || !*e) return dflt;
    const int v = std::atoi(e);
    return v > 0 ? v : dflt;
}

// The same, accepting 0.
int env_int0(const char* name, int dflt) {
    const char* e = std::getenv(name);
    if (!e || !*e) return dflt;
    const int v = std::atoi(e);
    return v >= 0 ? v : dflt;
}

// Ring + bookkeeping per CTA (one CTA per SM; B200Q_GEMV_SMEM_KB overrides):
// the full 220 KB for long rows (k >= 8192), 200 KB below, where fewer
// weight bytes queued ahead of the next kernel's loads measured faster
// (4096-element rows: 8% per matvec, the Llama-3-8B decode step 2.5%).
constexpr int kSmemBudgetKB = 220;
constexpr int kSmemBudgetShortKB = 200;
// Preferred bytes per stage (B200Q_STAGE_KB overrides). Walker groups take
// alternate stages, so a stage is a unit of work for a group, not for all
// warps; below ~16 KB the bulk copies in flight per SM (limited in number)
// no longer cover the HBM latency. Measured against 32 KB: the same on the
// x8 4096x14336 matvec, x16 4% faster, the Llama-3-8B decode step 5%
// faster, 4096x4096 matrices 3-5% slower.
constexpr int kStageTargetKB = 48;
constexpr int kStageMax = 96 * 1024;      // largest stage
constexpr int kMaxStages = 48;
// Weight bytes issued at CTA start, before the activations are requested
// (B200Q_GEMV_PREFETCH_KB): about what drains while the CTA waits for the
// preceding kernel, so that little is still queued ahead of the activation
// copy; the rest of the ring follows that copy.
constexpr int kPrefetchKB = 64;

struct Plan {
    GemvParams p;
    int threads;
    int smem;
    int grid;
    long long x_bytes;  // staged activation codes, past the ring
    int dev = -1;       // device id the launch targets (set by the caller)
};

// Rows a consumer warp carries per iteration (kRowsPerIter in gemv.cuh).
int rows_per_iter(int MR) { return MR == 1 ? 2 : 1; }

// fq: the GEMV quantizes fp32 activations itself; they (and, with norm, the
// RMSNorm gains) are first copied into the last nx ring slots.
int make_plan(int qtype, int dig, int k, int n, int MR, int num_sms, Plan& pl, bool fq = false, bool norm = false) {
    FmtInfo f;
    if (!fmt_info(qtype, f)) return B200Q_EQTYPE;
    if (k <= 0 || n <= 0) return B200Q_EINVAL;
    if (k % f.elems) return B200Q_ESHAPE;
    const int nb = k / f.elems;
    const long long rb = static_cast<long long>(nb) * f.bytes;
    const int S = (nb + f.blocks_per_slice - 1) / f.blocks_per_slice;
    // kGemvWarps in gemv.cuh; x16 takes 14 only for tall matrices (measured:
    // 14 warps were faster from ~8K rows, slower on 4096-row matrices)
    int max_warps = (dig == 1 && MR == 1) ? 16 : ((dig == 2 && MR == 1 && n >= 8192) ? 14 : 12);
    if (S > max_warps) return B200Q_ESHAPE;
    // B200Q_GEMV_WARPS caps the warps (never below one per k-slice).
    static const int warps_cap = env_int("B200Q_GEMV_WARPS", 0);
    if (warps_cap > 0) max_warps = std::max(S, std::min(max_warps, warps_cap));
    static const int smem_env = env_int("B200Q_GEMV_SMEM_KB", 0);
    const int smem_budget = std::min(227, smem_env > 0 ? smem_env : (k >= 8192 ? kSmemBudgetKB : kSmemBudgetShortKB)) *
                            1024;
    static const int target = env_int("B200Q_STAGE_KB", kStageTargetKB) * 1024;
    static const int prefetch = env_int0("B200Q_GEMV_PREFETCH_KB", kPrefetchKB) * 1024;
    const int U = rows_per_iter(MR);
    const int walkers = std::max(1, max_warps / S);
    const int n_quads = (n + 3) / 4;
    const int grid = std::min(num_sms, n_quads);
    const int rows_cta = 4 * ((n_quads + grid - 1) / grid);
    // Rows per stage: whole U-row steps (whole 4-row groups for R4) totalling
    // about `target` bytes, but no more than the CTA's rows.
    int R = U * static_cast<int>(std::max<long long>(1, (target + U * rb / 2) / (U * rb)));
    R = std::min(R, std::max(U, (rows_cta + U - 1) / U * U));
    if (f.r4) R = (R + 3) / 4 * 4;
    // A stage copies the 16-byte-aligned window around its rows: at most
    // rows * rb + 30 bytes; kSlotPad also covers the 4-byte over-read of the
    // unaligned word loads.
    constexpr int kSlotPad = 48;
    if (R * rb + kSlotPad > kStageMax) {
        R = f.r4 ? 4 : std::max<int>(1, static_cast<int>((kStageMax - kSlotPad) / rb));
        if (R * rb + kSlotPad > kStageMax) return B200Q_ESHAPE;
    }
    // One walker per U rows of a stage, then as many groups as that leaves.
    int SW = std::max(1, std::min(walkers, (R + U - 1) / U));
    // x8 with long rows: SW divides the walkers, so every consumer warp
    // walks (measured on 4096x14336: 8.8 against 9.4 us; on shorter rows and
    // in x16 the undivided split measured faster)
    if (dig == 1 && k >= 8192)
        while (SW > 1 && walkers % SW) --SW;
    int G = std::max(1, walkers / SW);
    const int stage_stride = static_cast<int>(((R * rb + kSlotPad) + 127) / 128 * 128);
    const int part_bytes = rows_cta * MR * S * 4;
    const long long x_bytes = static_cast<long long>(MR) * xs_row_bytes(k, dig);
    // full + empty barriers per slot, x and x-done barriers, x flag, per-warp sums
    const long long book = static_cast<long long>(kMaxStages) * 16 + 20 + kGemvMaxWarps * 4 + part_bytes + 64;
    const long long room = smem_budget - x_bytes - book;
    int NS = static_cast<int>(std::min<long long>(kMaxStages, room > 0 ? room / stage_stride : 0));
    if (NS < 2) return B200Q_ESHAPE;
    // Stage s and s + NS must belong to the same walker group (each group
    // then meets its slots' barrier phases in order): NS is a multiple of G.
    if (NS < G) G = NS;
    NS -= NS % G;
    const long long fq_bytes = fq ? static_cast<long long>(MR + (norm ? 1 : 0)) * k * 4 : 0;
    const int nx = static_cast<int>((fq_bytes + stage_stride - 1) / stage_stride);
    if (nx > NS) return B200Q_ESHAPE;  // the fp32 rows must fit in the ring
    const int WR = G * SW;
    const int x_off = NS * stage_stride;
    const int PD = std::max(0, std::min(NS, prefetch / stage_stride));
    GemvParams& p = pl.p;
    p = GemvParams{};
    p.row_bytes = rb;
    p.k = k;
    p.n = n;
    p.nb = nb;
    p.S = S;
    p.WR = WR;
    p.G = G;
    p.SW = SW;
    p.R = R;
    p.NS = NS;
    p.stage_stride = stage_stride;
    p.PD = PD;
    p.x_off = x_off;
    p.nx = nx;
    p.n_quads = n_quads;
    p.rows_cta = rows_cta;
    pl.x_bytes = x_bytes;
    pl.threads = (S * WR + 1) * 32;
    pl.smem = static_cast<int>(x_off + x_bytes + NS * 16 + 20 + kGemvMaxWarps * 4 + part_bytes + 16);
    pl.grid = grid;
    return B200Q_OK;
}

template <int QT, int DIG, int MR, bool DBG, bool FQ>
cudaError_t launch_kernel(const Plan& pl, cudaStream_t st, bool pdl) {
    auto kern = b200q_gemv_kernel<QT, DIG, MR, DBG, FQ>;
    // Raise the dynamic shared-memory limit once per kernel instance and
    // device: the attribute belongs to the device context, so a process that
    // drives several GPUs sets it on each (bit per device id below 64; ids
    // beyond that set it on every launch).
    static std::mutex mu;
    static uint64_t configured = 0;
    {
        std::lock_guard<std::mutex> lk(mu);
        const uint64_t bit = (pl.dev >= 0 && pl.dev < 64) ? (1ull << pl.dev) : 0;
        if (!bit || !(configured & bit)) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
            if (e != cudaSuccess) return e;
            configured |= bit;
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3(pl.threads);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, kern, pl.p);
}

// Most activation rows one launch carries, per qtype and mode (the Q4_K
// lanes hold four activation runs, so they carry fewer rows).
int max_rows_per_launch(int qtype, int dig) {
    const bool q4k = qtype == QT_Q4_K || qtype == QT_Q4_K_R4;
    if (dig == 1) return q4k ? 2 : 4;
    return q4k ? 1 : 2;
}

template <int QT, bool FQ>
cudaError_t dispatch_qt(int dig, int MR, bool dbg, const Plan& pl, cudaStream_t st, bool pdl) {
    constexpr bool q4k = QT == QT_Q4_K || QT == QT_Q4_K_R4;
    if (dbg)
        return dig == 1 ? launch_kernel<QT, 1, 1, true, FQ>(pl, st, pdl) : launch_kernel<QT, 2, 1, true, FQ>(pl, st, pdl);
    if (dig == 1) {
        if constexpr (!q4k) {
            if (MR == 4) return launch_kernel<QT, 1, 4, false, FQ>(pl, st, pdl);
        }
        if (MR == 2) return launch_kernel<QT, 1, 2, false, FQ>(pl, st, pdl);
        return launch_kernel<QT, 1, 1, false, FQ>(pl, st, pdl);
    }
    if constexpr (!q4k) {
        if (MR == 2) return launch_kernel<QT, 2, 2, false, FQ>(pl, st, pdl);
    }
    return launch_kernel<QT, 2, 1, false, FQ>(pl, st, pdl);
}

template <bool FQ>
cudaError_t dispatch(int qtype, int dig, int MR, bool dbg, const Plan& pl, cudaStream_t st, bool pdl) {
    switch (qtype) {
        case QT_Q4_K: return dispatch_qt<QT_Q4_K, FQ>(dig, MR, dbg, pl, st, pdl);
        case QT_Q4_K_R4: return dispatch_qt<QT_Q4_K_R4, FQ>(dig, MR, dbg, pl, st, pdl);
        case QT_Q6_K: return dispatch_qt<QT_Q6_K, FQ>(dig, MR, dbg, pl, st, pdl);
        case QT_Q6_K_R4: return dispatch_qt<QT_Q6_K_R4, FQ>(dig, MR, dbg, pl, st, pdl);
        case QT_Q6_K_LM: return dispatch_qt<QT_Q6_K_LM, FQ>(dig, MR, dbg, pl, st, pdl);
        case QT_Q8_0: return dispatch_qt<QT_Q8_0, FQ>(dig, MR, dbg, pl, st, pdl);
        case QT_Q4_0: return dispatch_qt<QT_Q4_0, FQ>(dig, MR, dbg, pl, st, pdl);
        default: return cudaErrorInvalidValue;
    }
}

// Activation scratch: growable buffers per (device, stream, slot); calls on
// one stream are ordered, so they can share them. Slots let one call keep
// several quantized vectors alive (e.g. x and the SwiGLU hidden vector).
struct Scratch {
    void* ptr = nullptr;
    size_t bytes = 0;
};
std::mutex g_scratch_mu;
std::map<std::tuple<int, cudaStream_t, int>, Scratch> g_scratch;

}  // namespace

int scratch_for(Device* dev, cudaStream_t st, int slot, size_t bytes, void** out, bool zero) {
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    Scratch& s = g_scratch[std::make_tuple(dev->id, st, slot)];
    if (s.bytes < bytes) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone)
            return B200Q_ECAPTURE;  // size the scratch with one call before capturing
        if (s.ptr) {
            cudaStreamSynchronize(st);
            cudaFree(s.ptr);
            s.ptr = nullptr;
            s.bytes = 0;
        }
        const size_t want = std::max<size_t>(bytes, 1u << 20);
        if (cudaMalloc(&s.ptr, want) != cudaSuccess) return B200Q_ENOMEM;
        s.bytes = want;
        // Every byte of the allocation, not just the bytes asked for: a later
        // call may use more of it without reallocating.
        if (zero && cudaMemsetAsync(s.ptr, 0, want, st) != cudaSuccess) return B200Q_ECUDA;
    }
    *out = s.ptr;
    return B200Q_OK;
}

namespace {

template <int DIG>
cudaError_t launch_quantize(const float* x, long long x_stride, int m, int k, uint8_t* xq, cudaStream_t st, bool pdl) {
    const long long threads = static_cast<long long>(m) * (k / 4);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>((threads + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, b200q_quantize_act_quads_kernel<DIG>, x, x_stride, m, k, xq);
}

}  // namespace

int launch_quantize_rows(int act_mode, const float* x, int rows, int k, uint8_t* xq, cudaStream_t st, bool pdl) {
    if (act_mode != B200Q_ACT_X8 && act_mode != B200Q_ACT_X16) return B200Q_EINVAL;
    if ((reinterpret_cast<uintptr_t>(x) & 15u)) return B200Q_EALIGN;
    if (k % 32) return B200Q_ESHAPE;
    const cudaError_t e = act_mode == B200Q_ACT_X8 ? launch_quantize<1>(x, k, rows, k, xq, st, pdl)
                                                   : launch_quantize<2>(x, k, rows, k, xq, st, pdl);
    return e == cudaSuccess ? B200Q_OK : B200Q_ECUDA;
}

int quantize_activations(int act_mode, const float* x, long long x_stride, int m, int k, Device* dev, cudaStream_t st,
                         bool pdl, int slot, const uint8_t** xq_out, long long* xq_row_out) {
    if (!x || m <= 0 || k <= 0 || !dev) return B200Q_EINVAL;
    if (act_mode != B200Q_ACT_X8 && act_mode != B200Q_ACT_X16) return B200Q_EINVAL;
    if ((reinterpret_cast<uintptr_t>(x) & 15u) || (x_stride & 3)) return B200Q_EALIGN;
    if (k % 32) return B200Q_ESHAPE;
    const int dig = act_mode == B200Q_ACT_X8 ? 1 : 2;
    const long long xq_row = xq_row_bytes(k, dig);
    void* xq = nullptr;
    const int rcs = scratch_for(dev, st, slot, static_cast<size_t>(xq_row) * m, &xq);
    if (rcs != B200Q_OK) return rcs;
    const cudaError_t e = dig == 1 ? launch_quantize<1>(x, x_stride, m, k, static_cast<uint8_t*>(xq), st, pdl)
                                   : launch_quantize<2>(x, x_stride, m, k, static_cast<uint8_t*>(xq), st, pdl);
    if (e != cudaSuccess) return B200Q_ECUDA;
    *xq_out = static_cast<const uint8_t*>(xq);
    *xq_row_out = xq_row;
    return B200Q_OK;
}

namespace {

// y = alpha * (W x) + beta * y over m activation rows in chunks of at most
// max_rows_per_launch rows: from codes (xq, quantized by a preceding kernel)
// or, when xf is given, from fp32 rows that the GEMV quantizes itself.
int gemv_rows(int qtype, int act_mode, const void* w, const uint8_t* xq, long long xq_row, const float* xf,
              long long xf_stride, float* y, int m, int k, int n, long long y_stride, float alpha, float beta,
              int32_t* isums, Device* dev, cudaStream_t st, bool pdl, int flags, const float* gamma = nullptr,
              float eps = 0.0f, const float* xu = nullptr) {
    if (!w || (!xq && !xf) || !y || m <= 0 || k <= 0 || n <= 0 || !dev) return B200Q_EINVAL;
    if (act_mode != B200Q_ACT_X8 && act_mode != B200Q_ACT_X16) return B200Q_EINVAL;
    if (reinterpret_cast<uintptr_t>(w) & 15u) return B200Q_EALIGN;
    if (xf && ((reinterpret_cast<uintptr_t>(xf) & 15u) || (xf_stride & 3))) return B200Q_EALIGN;
    if (isums && m != 1) return B200Q_EINVAL;
    const int dig = act_mode == B200Q_ACT_X8 ? 1 : 2;
    const int mr_max = max_rows_per_launch(qtype, dig);
    for (int m0 = 0; m0 < m;) {
        const int left = m - m0;
        const int MR = isums ? 1 : (left >= mr_max ? mr_max : (left >= 2 && mr_max >= 2 ? 2 : 1));
        Plan pl;
        // (the planner's extra fp32 row holds the RMSNorm gains or the up row)
        const int rc = make_plan(qtype, dig, k, n, MR, dev->num_sms, pl, xf != nullptr, gamma != nullptr || xu != nullptr);
        if (rc != B200Q_OK) return rc;
        pl.p.W = static_cast<const uint8_t*>(w);
        pl.dev = dev->id;
        if (xf) {
            pl.p.xf = xf + m0 * xf_stride;
            pl.p.xf_stride = xf_stride;
            if (gamma) {
                // One group per lane covers the whole row.
                if (MR != 1 || k > 32 * 32 * pl.p.S * pl.p.WR) return B200Q_ESHAPE;
                pl.p.gamma = gamma;
                pl.p.eps = eps;
            }
            if (xu) {
                if (MR != 1 || gamma) return B200Q_EINVAL;
                pl.p.xu = xu;
            }
        } else {
            pl.p.xq = xq + m0 * xq_row;
            pl.p.xq_stride = xq_row;
        }
        pl.p.y = y + m0 * y_stride;
        pl.p.y_stride = y_stride;
        pl.p.dbg = isums;
        pl.p.status = dev->status;
        pl.p.w_static = (flags & B200Q_WEIGHTS_STATIC) ? 1 : 0;
        pl.p.alpha = alpha;
        pl.p.beta = beta;
        const cudaError_t e = xf ? dispatch<true>(qtype, dig, MR, isums != nullptr, pl, st, pdl)
                                 : dispatch<false>(qtype, dig, MR, isums != nullptr, pl, st, pdl);
        if (e != cudaSuccess) return B200Q_ECUDA;
        m0 += MR;
    }
    return B200Q_OK;
}

}  // namespace

int gemv_from_xq(int qtype, int act_mode, const void* w, const uint8_t* xq, long long xq_row, float* y, int m, int k,
                 int n, long long y_stride, float alpha, float beta, int32_t* isums, Device* dev, cudaStream_t st,
                 bool pdl, int flags) {
    if (!xq) return B200Q_EINVAL;
    return gemv_rows(qtype, act_mode, w, xq, xq_row, nullptr, 0, y, m, k, n, y_stride, alpha, beta, isums, dev, st,
                     pdl, flags);
}

int gemv_from_f32(int qtype, int act_mode, const void* w, const float* x, long long x_stride, float* y, int m, int k,
                  int n, long long y_stride, float alpha, float beta, int32_t* isums, Device* dev, cudaStream_t st,
                  bool pdl, int flags) {
    if (!x) return B200Q_EINVAL;
    return gemv_rows(qtype, act_mode, w, nullptr, 0, x, x_stride, y, m, k, n, y_stride, alpha, beta, isums, dev, st,
                     pdl, flags);
}

int gemv_norm_f32(int qtype, int act_mode, const void* w, const float* x, const float* gamma, float eps, float* y,
                  int k, int n, float alpha, float beta, Device* dev, cudaStream_t st, bool pdl, int flags) {
    if (!x || !gamma) return B200Q_EINVAL;
    if (reinterpret_cast<uintptr_t>(gamma) & 15u) return B200Q_EALIGN;
    if (!(eps >= 0.0f)) return B200Q_EINVAL;
    return gemv_rows(qtype, act_mode, w, nullptr, 0, x, k, y, 1, k, n, n, alpha, beta, nullptr, dev, st, pdl, flags,
                     gamma, eps);
}

int gemv_swiglu_f32(int qtype, int act_mode, const void* w, const float* gate, const float* up, float* y, int k, int n,
                    float alpha, float beta, Device* dev, cudaStream_t st, bool pdl, int flags) {
    if (!gate || !up) return B200Q_EINVAL;
    if (reinterpret_cast<uintptr_t>(up) & 15u) return B200Q_EALIGN;
    return gemv_rows(qtype, act_mode, w, nullptr, 0, gate, k, y, 1, k, n, n, alpha, beta, nullptr, dev, st, pdl, flags,
                     nullptr, 0.0f, up);
}

int gemv_plan_info(int qtype, int act_mode, int k, int n, int mr, bool fq, int num_sms, long long* out, int out_len) {
    if (act_mode != B200Q_ACT_X8 && act_mode != B200Q_ACT_X16) return B200Q_EINVAL;
    if (!out || out_len < kPlanInfoFields || num_sms <= 0) return B200Q_EINVAL;
    FmtInfo f;
    if (!fmt_info(qtype, f)) return B200Q_EQTYPE;
    const int dig = act_mode == B200Q_ACT_X8 ? 1 : 2;
    // Only the row counts a launch is ever made with: 1, 2 and (where the
    // format's lanes carry it) 4, up to max_rows_per_launch.
    if (mr < 1 || mr == 3 || mr > max_rows_per_launch(qtype, dig)) return B200Q_EINVAL;
    Plan pl;
    const int rc = make_plan(qtype, dig, k, n, mr, num_sms, pl, fq);
    if (rc != B200Q_OK) return rc;
    const GemvParams& p = pl.p;
    const long long v[kPlanInfoFields] = {pl.threads, pl.smem, pl.grid, p.S, p.WR, p.G, p.SW, p.R, p.NS,
                                          p.stage_stride, p.PD, p.x_off, pl.x_bytes, p.row_bytes, p.rows_cta};
    for (int i = 0; i < kPlanInfoFields; ++i) out[i] = v[i];
    return B200Q_OK;
}

int gemv_check_shape(int qtype, int act_mode, int k, int n, Device* dev) {
    if (act_mode != B200Q_ACT_X8 && act_mode != B200Q_ACT_X16) return B200Q_EINVAL;
    if (k % 32) return B200Q_ESHAPE;
    Plan probe;
    return make_plan(qtype, act_mode == B200Q_ACT_X8 ? 1 : 2, k, n, 1, dev->num_sms, probe);
}

// B200Q_ACT_F16 always takes the tile path (fp16 activations). Q4_K batches
// of at least B200Q_TILE_MIN_M rows (default 8) take it too, where the tile
// kernel streams W once for the whole batch: x8 with fp16 activations (more
// accurate than int8 codes), x16 with the precise variant (fp16 activations
// plus their fp16 rounding residues, within the x16 accuracy).
int uses_tile_path(int qtype, int act_mode, int m, int flags) {
    static const int min_m = env_int("B200Q_TILE_MIN_M", 8);
    if (qtype != QT_Q4_K) return 0;
    if (act_mode == B200Q_ACT_F16) return 1;
    const int from = (flags & B200Q_TILE_FROM_2) ? 2 : min_m;
    if (from <= 0 || m < from) return 0;
    if (act_mode == B200Q_ACT_X8) return 1;
    if (act_mode == B200Q_ACT_X16) return 2;
    return 0;
}

int launch_gemv(int qtype, int act_mode, const void* w, const float* x, float* y, int m, int k, int n,
                long long x_stride, long long y_stride, int32_t* isums, Device* dev, cudaStream_t st, bool pdl,
                int flags) {
    if (!w || !x || !y || m <= 0 || k <= 0 || n <= 0 || !dev) return B200Q_EINVAL;
    if ((reinterpret_cast<uintptr_t>(w) & 15u) || (reinterpret_cast<uintptr_t>(x) & 15u) || (x_stride & 3))
        return B200Q_EALIGN;
    if (isums && m != 1) return B200Q_EINVAL;
    const int tile = isums ? 0 : uses_tile_path(qtype, act_mode, m, flags);
    if (tile) {
        // Batches of up to tile_max_rows activation rows per tile-kernel call.
        const int step = tile_max_rows(tile == 2);
        for (int r0 = 0; r0 < m; r0 += step) {
            const int rc = launch_tile(qtype, w, x + r0 * x_stride, x_stride, y + r0 * y_stride,
                                       std::min(step, m - r0), k, n, y_stride, dev, st, pdl, tile == 2);
            if (rc != B200Q_OK) return rc;
        }
        return B200Q_OK;
    }
    if (act_mode == B200Q_ACT_F16) return B200Q_EQTYPE;
    int rc = gemv_check_shape(qtype, act_mode, k, n, dev);  // validate before any launch
    if (rc != B200Q_OK) return rc;
    // One launch per chunk of rows: the GEMV quantizes x itself, unless its
    // staging does not fit (B200Q_GEMV_FUSED_QUANT=0 selects the separate
    // quantizer kernel).
    static const bool fused = [] {
        const char* e = std::getenv("B200Q_GEMV_FUSED_QUANT");
        return !(e && e[0] == '0');
    }();
    Plan probe;
    const int dig = act_mode == B200Q_ACT_X8 ? 1 : 2;
    if (fused && make_plan(qtype, dig, k, n, 1, dev->num_sms, probe, true) == B200Q_OK &&
        (isums || m == 1 ||
         make_plan(qtype, dig, k, n, std::min(m, max_rows_per_launch(qtype, dig)), dev->num_sms, probe, true) == B200Q_OK))
        return gemv_from_f32(qtype, act_mode, w, x, x_stride, y, m, k, n, y_stride, 1.0f, 0.0f, isums, dev, st, pdl,
                             flags);
    const uint8_t* xq = nullptr;
    long long xq_row = 0;
    rc = quantize_activations(act_mode, x, x_stride, m, k, dev, st, pdl, 0, &xq, &xq_row);
    if (rc != B200Q_OK) return rc;
    return gemv_from_xq(qtype, act_mode, w, xq, xq_row, y, m, k, n, y_stride, 1.0f, 0.0f, isums, dev, st, pdl, flags);
}

}  // namespace b200q

namespace b200q {
long long xq_bytes_per_row(int k, int act_mode) { return xq_row_bytes(k, act_mode == B200Q_ACT_X8 ? 1 : 2); }
}  // namespace b200q
