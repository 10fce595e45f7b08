// Layout repacks, row dequantization and the fused-op glue kernels
// (SwiGLU + activation quantization), with their device-pointer entry points.
#include <algorithm>

#include "gemv.cuh"
#include "internal.h"

namespace b200q {

namespace {

// ---------------------------------------------------------------------------
// Repacks (quantized_matmul.cpp:250-365).
// ---------------------------------------------------------------------------

// R4: rows grouped by 4, block-major inside a group ([g][b][r][B]); the n % 4
// tail rows are copied canonically after the full groups. One thread per
// output 16-bit word (block sizes are even).
__global__ void b200q_repack_r4_kernel(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst, long long words,
                                 long long row_bytes, int block_bytes, int n) {
    const long long o = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (o >= words) return;
    const long long ob = 2 * o;
    const long long grouped = static_cast<long long>(n / 4) * 4 * row_bytes;
    long long sb = ob;
    if (ob < grouped) {
        const long long g = ob / (4 * row_bytes);
        const long long rem = ob - g * 4 * row_bytes;
        const long long b = rem / (4 * block_bytes);
        const long long rem2 = rem - b * 4 * block_bytes;
        const long long r = rem2 / block_bytes;
        const long long byte = rem2 - r * block_bytes;
        sb = (4 * g + r) * row_bytes + b * block_bytes + byte;
    }
    dst[o] = src[sb / 2];
}

// Q6_K -> Q6_K_LM: 256 int8 codes (6-bit value - 32) in element order, the
// 16 int8 scales, and d as fp32 (276 bytes per block). One warp per block.
__global__ void b200q_repack_q6k_lm_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, long long blocks) {
    const long long blk = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
    const int lane = threadIdx.x & 31;
    if (blk >= blocks) return;
    const uint8_t* b = src + blk * 210;
    uint8_t* o = dst + blk * 276;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int e = lane * 8 + i;
        const int g = e / 32, j = e % 32;
        const int ql_shift = (g % 4) >= 2 ? 4 : 0;
        const int lo = (b[(g / 4) * 64 + (g % 2) * 32 + j] >> ql_shift) & 0x0F;
        const int hi = (b[128 + (g / 4) * 32 + j] >> ((g % 4) * 2)) & 0x03;
        o[e] = static_cast<uint8_t>(static_cast<int8_t>((lo | (hi << 4)) - 32));
    }
    if (lane < 16) o[256 + lane] = b[192 + lane];
    if (lane == 0) {
        const float d = half_bits_to_float(static_cast<uint32_t>(b[208]) | (static_cast<uint32_t>(b[209]) << 8));
        const uint32_t bits = __float_as_uint(d);
        o[272] = bits & 0xFF;
        o[273] = (bits >> 8) & 0xFF;
        o[274] = (bits >> 16) & 0xFF;
        o[275] = bits >> 24;
    }
}

// ---------------------------------------------------------------------------
// Row dequantization (simd_dequantize_row, quantized_matmul.cpp:2179-2296):
// w = (a * code) - b in fp32, with the products and difference rounded
// separately (no contraction), exactly like the reference.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t rd16(const uint8_t* p) {
    return static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8);
}

__device__ float dequant_element(int qtype, const uint8_t* blk, int e) {
    switch (qtype) {
        case QT_Q4_0: {
            const float d = half_bits_to_float(rd16(blk));
            const int q = e < 16 ? (blk[2 + e] & 0x0F) : (blk[2 + e - 16] >> 4);
            return __fmul_rn(d, static_cast<float>(q - 8));
        }
        case QT_Q8_0: {
            const float d = half_bits_to_float(rd16(blk));
            return __fmul_rn(d, static_cast<float>(static_cast<int8_t>(blk[2 + e])));
        }
        case QT_Q4_K:
        case QT_Q4_K_R4: {
            const float d = half_bits_to_float(rd16(blk));
            const float dmin = half_bits_to_float(rd16(blk + 2));
            const uint8_t* s = blk + 4;
            const int j = e / 32, i = e % 32;
            int sc, mn;
            if (j < 4) {
                sc = s[j] & 63;
                mn = s[j + 4] & 63;
            } else {
                sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 2) & 0x30);
                mn = (s[j + 4] >> 4) | ((s[j] >> 2) & 0x30);
            }
            const uint8_t byte = blk[16 + (j / 2) * 32 + i];
            const int q = (j & 1) ? (byte >> 4) : (byte & 0x0F);
            const float dsc = __fmul_rn(d, static_cast<float>(sc));
            const float dmn = __fmul_rn(dmin, static_cast<float>(mn));
            return __fsub_rn(__fmul_rn(dsc, static_cast<float>(q)), dmn);
        }
        case QT_Q6_K:
        case QT_Q6_K_R4: {
            const int g = e / 32, i = e % 32;
            const int ql_shift = (g % 4) >= 2 ? 4 : 0;
            const int lo = (blk[(g / 4) * 64 + (g % 2) * 32 + i] >> ql_shift) & 0x0F;
            const int hi = (blk[128 + (g / 4) * 32 + i] >> ((g % 4) * 2)) & 0x03;
            const float d = half_bits_to_float(rd16(blk + 208));
            const float scale = __fmul_rn(d, static_cast<float>(static_cast<int8_t>(blk[192 + g * 2 + i / 16])));
            return __fmul_rn(scale, static_cast<float>((lo | (hi << 4)) - 32));
        }
        case QT_Q6_K_LM: {
            const float d = __uint_as_float(rd16(blk + 272) | (rd16(blk + 274) << 16));
            const float scale = __fmul_rn(d, static_cast<float>(static_cast<int8_t>(blk[256 + e / 16])));
            return __fmul_rn(scale, static_cast<float>(static_cast<int8_t>(blk[e])));
        }
    }
    return 0.0f;
}

// One thread per output element. `tail_canonical` selects the R4 addressing
// of the layout (tail rows canonical, needs n) or the reference's
// (group = row / 4 for every row; simd_dequantize_row has no n).
__global__ void b200q_dequant_rows_kernel(int qtype, const uint8_t* __restrict__ w, const int* __restrict__ rows, int nrows,
                                    float* __restrict__ out, int k, int n, int elems, int bbytes, int tail_canonical) {
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<long long>(nrows) * k) return;
    const int r = static_cast<int>(i / k), c = static_cast<int>(i % k);
    const int row = rows[r];
    const int b = c / elems, e = c % elems;
    const long long rb = static_cast<long long>(k / elems) * bbytes;
    long long off;
    const bool r4 = qtype == QT_Q4_K_R4 || qtype == QT_Q6_K_R4;
    if (r4 && (!tail_canonical || row < (n / 4) * 4))
        off = static_cast<long long>(row / 4) * 4 * rb + static_cast<long long>(b * 4 + row % 4) * bbytes;
    else
        off = row * rb + static_cast<long long>(b) * bbytes;
    out[i] = dequant_element(qtype, w + off, e);
}

// ---------------------------------------------------------------------------
// SwiGLU + activation quantization: h = silu(g) * u, quantized per 32 for the
// down projection (the SiLU(gate) * up step of quantized_matmul.cpp:2380-2412).
// ---------------------------------------------------------------------------
template <int DIG>
__global__ void __launch_bounds__(256) b200q_swiglu_quantize_kernel(const float* __restrict__ g, const float* __restrict__ u,
                                                              int hidden, uint8_t* __restrict__ xq) {
    griddep_launch_dependents();
    griddep_wait();
    // four elements per thread; the 8 threads of a 32-element group quantize
    // it together (quantize_quad); hidden % 32 == 0 keeps groups whole
    const int q4 = blockIdx.x * blockDim.x + threadIdx.x;
    const bool valid = q4 < hidden / 4;
    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (valid) {
        const float4 gv = __ldg(reinterpret_cast<const float4*>(g) + q4);
        const float4 uv = __ldg(reinterpret_cast<const float4*>(u) + q4);
        v = make_float4(gv.x / (1.0f + expf(-gv.x)) * uv.x, gv.y / (1.0f + expf(-gv.y)) * uv.y,
                        gv.z / (1.0f + expf(-gv.z)) * uv.z, gv.w / (1.0f + expf(-gv.w)) * uv.w);
    }
    quantize_quad<DIG>(v, valid, xq, hidden, q4);
}

cudaLaunchConfig_t make_cfg(unsigned grid, unsigned block, cudaStream_t st, bool pdl, cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.stream = st;
    if (pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cfg;
}

}  // namespace

int launch_repack(int dst_qtype, const void* src, void* dst, int k, int n, cudaStream_t st) {
    if (!src || !dst || k <= 0 || n <= 0 || k % 256) return B200Q_EINVAL;
    if ((reinterpret_cast<uintptr_t>(src) & 1u) || (reinterpret_cast<uintptr_t>(dst) & 1u)) return B200Q_EALIGN;
    if (dst_qtype == QT_Q4_K_R4 || dst_qtype == QT_Q6_K_R4) {
        const int bb = dst_qtype == QT_Q4_K_R4 ? 144 : 210;
        const long long rb = static_cast<long long>(k / 256) * bb;
        const long long words = rb * n / 2;
        b200q_repack_r4_kernel<<<static_cast<unsigned>((words + 255) / 256), 256, 0, st>>>(
            static_cast<const uint16_t*>(src), static_cast<uint16_t*>(dst), words, rb, bb, n);
    } else if (dst_qtype == QT_Q6_K_LM) {
        const long long blocks = static_cast<long long>(k / 256) * n;
        b200q_repack_q6k_lm_kernel<<<static_cast<unsigned>((blocks * 32 + 255) / 256), 256, 0, st>>>(
            static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst), blocks);
    } else {
        return B200Q_EQTYPE;
    }
    return cudaGetLastError() == cudaSuccess ? B200Q_OK : B200Q_ECUDA;
}

int launch_dequant_rows(int qtype, const void* w, const int* rows, int nrows, float* out, int k, int n,
                        bool tail_canonical, cudaStream_t st) {
    FmtInfo f;
    if (!fmt_info(qtype, f)) return B200Q_EQTYPE;
    if (!w || !rows || !out || nrows <= 0 || k <= 0) return B200Q_EINVAL;
    if (k % f.elems) return B200Q_ESHAPE;
    const long long total = static_cast<long long>(nrows) * k;
    b200q_dequant_rows_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, st>>>(
        qtype, static_cast<const uint8_t*>(w), rows, nrows, out, k, n, f.elems, f.bytes, tail_canonical ? 1 : 0);
    return cudaGetLastError() == cudaSuccess ? B200Q_OK : B200Q_ECUDA;
}

int launch_swiglu_quantize(int act_mode, const float* g, const float* u, int hidden, uint8_t* xq, cudaStream_t st,
                           bool pdl) {
    if (hidden % 32) return B200Q_ESHAPE;
    cudaLaunchAttribute attr[1];
    if ((reinterpret_cast<uintptr_t>(g) & 15u) || (reinterpret_cast<uintptr_t>(u) & 15u)) return B200Q_EALIGN;
    cudaLaunchConfig_t cfg = make_cfg(static_cast<unsigned>((hidden / 4 + 255) / 256), 256, st, pdl, attr);
    const cudaError_t e = act_mode == B200Q_ACT_X8 ? cudaLaunchKernelEx(&cfg, b200q_swiglu_quantize_kernel<1>, g, u, hidden, xq)
                                                   : cudaLaunchKernelEx(&cfg, b200q_swiglu_quantize_kernel<2>, g, u, hidden, xq);
    return e == cudaSuccess ? B200Q_OK : B200Q_ECUDA;
}

// Fused SwiGLU expert FFN on device buffers (quantized_matmul.cpp:2307-2416):
// out = alpha * down(silu(gate x) * (up x)) + beta * out. Scratch slots 1..3
// hold the quantized x, the gate/up outputs and the quantized hidden vector.
int expert_swiglu(int act_mode, const float* x, int in_dim, const void* gate, int gq, int hidden, const void* up, int uq,
                  const void* down, int dq, int out_dim, float* out, float alpha, float beta, Device* dev,
                  cudaStream_t st, bool pdl, int flags) {
    if (!x || !gate || !up || !down || !out || in_dim <= 0 || hidden <= 0 || out_dim <= 0) return B200Q_EINVAL;
    int rc = gemv_check_shape(gq, act_mode, in_dim, hidden, dev);
    if (rc == B200Q_OK) rc = gemv_check_shape(uq, act_mode, in_dim, hidden, dev);
    if (rc == B200Q_OK) rc = gemv_check_shape(dq, act_mode, hidden, out_dim, dev);
    if (rc != B200Q_OK) return rc;
    void* gu = nullptr;
    rc = scratch_for(dev, st, 2, static_cast<size_t>(hidden) * 2 * sizeof(float), &gu);
    if (rc != B200Q_OK) return rc;
    void* hq = nullptr;
    rc = scratch_for(dev, st, 3, static_cast<size_t>(xq_bytes_per_row(hidden, act_mode)), &hq);
    if (rc != B200Q_OK) return rc;
    float* gbuf = static_cast<float*>(gu);
    float* ubuf = gbuf + hidden;
    const uint8_t* xq = nullptr;
    long long xq_row = 0;
    rc = quantize_activations(act_mode, x, in_dim, 1, in_dim, dev, st, pdl, 1, &xq, &xq_row);
    if (rc == B200Q_OK)
        rc = gemv_from_xq(gq, act_mode, gate, xq, xq_row, gbuf, 1, in_dim, hidden, hidden, 1.0f, 0.0f, nullptr, dev, st,
                          pdl, flags);
    if (rc == B200Q_OK)
        rc = gemv_from_xq(uq, act_mode, up, xq, xq_row, ubuf, 1, in_dim, hidden, hidden, 1.0f, 0.0f, nullptr, dev, st,
                          pdl, flags);
    if (rc == B200Q_OK) rc = launch_swiglu_quantize(act_mode, gbuf, ubuf, hidden, static_cast<uint8_t*>(hq), st, pdl);
    if (rc == B200Q_OK)
        rc = gemv_from_xq(dq, act_mode, down, static_cast<const uint8_t*>(hq), xq_bytes_per_row(hidden, act_mode), out,
                          1, hidden, out_dim, out_dim, alpha, beta, nullptr, dev, st, pdl, flags);
    return rc;
}

// ---------------------------------------------------------------------------
// The graph-side dispatch of model_graph.cpp:731-790 on device pointers.
// ---------------------------------------------------------------------------
namespace {

// y = W x for fp32 weights [rows][cols] (matvec_f32, model_graph.cpp:700-727):
// one warp per row, coalesced 16-byte loads when the rows allow them, fp32
// accumulation, warp-shuffle reduction.
__global__ void __launch_bounds__(256) b200q_matvec_f32_kernel(const float* __restrict__ W, const float* __restrict__ x,
                                                         float* __restrict__ y, int rows, int cols, int vec4) {
    const long long warp = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= rows) return;
    const float* w = W + warp * cols;
    float acc = 0.0f;
    if (vec4) {
        const float4* w4 = reinterpret_cast<const float4*>(w);
        const float4* x4 = reinterpret_cast<const float4*>(x);
        for (int i = lane; i < cols / 4; i += 32) {
            const float4 a = __ldg(w4 + i), b = __ldg(x4 + i);
            acc = fmaf(a.x, b.x, acc);
            acc = fmaf(a.y, b.y, acc);
            acc = fmaf(a.z, b.z, acc);
            acc = fmaf(a.w, b.w, acc);
        }
    } else {
        for (int i = lane; i < cols; i += 32) acc = fmaf(__ldg(w + i), __ldg(x + i), acc);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) y[warp] = acc;
}

}  // namespace

namespace {

// dst[0..n) = src[0..n) where src is page-locked host memory mapped into the
// device's address space: the drop-ins' activation upload without a DMA
// copy (whose setup costs several microseconds). Launched without the
// programmatic-launch attribute, so all earlier work on the stream is done;
// it lets the GEMV launched behind it start at once, which streams its
// first weight stages while these PCIe reads are in flight and waits for
// this grid before it reads dst.
__global__ void b200q_stage_host_rows_kernel(const float* __restrict__ src, float* __restrict__ dst, long long n,
                                             int vec4) {
    griddep_launch_dependents();
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (vec4) {
        if (i < n / 4) reinterpret_cast<float4*>(dst)[i] = reinterpret_cast<const float4*>(src)[i];
    } else if (i < n) {
        dst[i] = src[i];
    }
}

}  // namespace

int launch_stage_host_rows(const float* src_mapped, float* dst, long long n, cudaStream_t st) {
    if (!src_mapped || !dst || n <= 0) return B200Q_EINVAL;
    const int vec4 = (n % 4 == 0) && !(reinterpret_cast<uintptr_t>(src_mapped) & 15u) &&
                     !(reinterpret_cast<uintptr_t>(dst) & 15u);
    const long long items = vec4 ? n / 4 : n;
    b200q_stage_host_rows_kernel<<<static_cast<unsigned>((items + 255) / 256), 256, 0, st>>>(src_mapped, dst, n, vec4);
    return cudaGetLastError() == cudaSuccess ? B200Q_OK : B200Q_ECUDA;
}

int launch_matvec_f32(const float* W, const float* x, float* y, int rows, int cols, cudaStream_t st) {
    if (!W || !x || !y || rows <= 0 || cols <= 0) return B200Q_EINVAL;
    const int vec4 = (cols % 4 == 0) && !(reinterpret_cast<uintptr_t>(W) & 15u) && !(reinterpret_cast<uintptr_t>(x) & 15u);
    const long long threads = static_cast<long long>(rows) * 32;
    b200q_matvec_f32_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, st>>>(W, x, y, rows, cols, vec4);
    return cudaGetLastError() == cudaSuccess ? B200Q_OK : B200Q_ECUDA;
}

}  // namespace b200q
