// Decode GEMV for GGUF block formats on sm_100a.
//
// y[m][row] = sum_k dequant(W)[row][k] * x[m][k] for m < MR activation rows,
// the operation of simd_matvec_* / simd_matmul_* in
// JSBuild/src/verso/Anvil/core/native/quantized_matmul.cpp:1536-2154, on the
// same canonical (and R4 / LM) block layouts.
//
// Design (one persistent CTA per SM, 16 warps):
//  * Each CTA streams its contiguous slab of weight rows into a ring of
//    shared-memory stages with 1-D bulk copies (cp.async.bulk, no multicast)
//    that complete on mbarriers. Weights are touched once, with an L2
//    evict-first policy. No warp is set aside for this: thread 0 issues the
//    first stages, and the warp that finishes a slot last refills it.
//  * Activations are quantized per 32-element group (int8 "x8", or int16
//    split in two byte planes "x16"). They are staged once per CTA in shared
//    memory of their own, past the ring: FQ instances (one launch per
//    matvec) bulk-copy the fp32 rows into ring slots and quantize them there,
//    one group per lane; code instances copy the codes a preceding kernel
//    wrote. Each lane then keeps the codes of its k-slice in registers for
//    all its rows.
//  * Programmatic dependent launch: the GEMV streams its first (static)
//    weight stages while the preceding kernel runs and waits for it only
//    before reading the activations, whose copy is requested before the rest
//    of the ring, so the weight traffic does not delay it.
//  * Per row a lane decodes its weight codes from shared memory and forms
//    exact integer dot sums with dp4a; each group sum is scaled in fp32 by
//    the weight and activation scales; partials are reduced per warp with
//    shuffles and across slices through shared memory in a fixed order.
//  * Every pipeline wait is bounded (%globaltimer); on timeout the kernel
//    records STATUS_TIMEOUT, stops consuming, and still reaches every
//    barrier, so nothing hangs.
#pragma once

#include "common.cuh"

namespace b200q {

// Consumer warps per CTA (one more warp is the producer). With 17 warps a
// thread may hold up to 96 registers (each SM sub-partition runs 5 warps);
// with 13-15, up to 128 -- the heavier instantiations take fewer: x16 up to
// 14 (the planner uses 14 for matrices of >= 8192 rows, 12 below: measured),
// several activation rows 12.
template <int DIG, int MR>
constexpr int kGemvWarps = (DIG == 1 && MR == 1) ? 16 : ((DIG == 2 && MR == 1) ? 14 : 12);
constexpr int kGemvMaxWarps = 16;
// Rows a consumer warp carries per iteration (independent chains, and the
// loop and reduction overhead shared between them).
template <int DIG, int MR>
constexpr int kRowsPerIter = MR == 1 ? 2 : 1;

struct GemvParams {
    const uint8_t* W;      // packed weight rows (device, 16-byte aligned)
    const uint8_t* xq;     // [MR] quantized activation rows (b200q_quantize_act_kernel layout)
    long long xq_stride;   // bytes between quantized rows
    const float* xf;       // [MR] fp32 activation rows, quantized in the kernel (FQ instances)
    long long xf_stride;   // floats between fp32 rows
    const float* gamma;    // FQ with MR == 1: RMSNorm weights; x is normalized before quantizing
    const float* xu;       // FQ with MR == 1: up row; silu(x) * xu is quantized (SwiGLU inside the GEMV)
    float eps;             // RMSNorm epsilon
    float* y;              // [MR][y_stride] fp32 outputs
    int32_t* dbg;          // optional [n][k/G] integer group sums (MR == 1 only)
    volatile int* status;  // status word (host-mapped); kernels store STATUS_* values
    long long row_bytes;   // bytes per packed row
    long long y_stride;    // floats between output rows
    int k, n;
    int nb;                // blocks per row
    int S;                 // slices per row (consumer warps per row)
    int WR;                // row walkers per slice (G groups x SW)
    int G;                 // walker groups: stage s belongs to group s % G
    int SW;                // walkers per slice in a group; they split a stage's rows
    int R;                 // rows per stage
    int NS;                // ring stages
    int stage_stride;      // bytes between ring slots (multiple of 128)
    int PD;                // stages issued at CTA start, before the activations are requested
    int x_off;             // byte offset of the staged activation codes (just past the ring)
    int nx;                // FQ: ring slots (at the ring's end) that first hold the fp32 rows (and gamma)
    int n_quads;           // ceil(n / 4)
    int rows_cta;          // most rows any CTA owns
    int w_static;          // weights not written by the preceding kernel: stream them before the grid dependency resolves
    float alpha, beta;     // y = alpha * (W x) + beta * y
};



// ---------------------------------------------------------------------------
// Per-format lane geometry. A warp covers kBlocksPerSlice consecutive blocks
// of a row; kLanesPerBlock lanes share a block. Each lane holds kRuns runs of
// kRun activation elements (kRun = 16 means its 32-element quantization
// group is split with lane^1).
// ---------------------------------------------------------------------------
template <int QT>
struct Fmt;

template <>
struct Fmt<QT_Q4_K> {
    // Lane p (0, 1) of a block holds sub-blocks 2p, 2p+1 (qs pair p, scale
    // encoding "lower") and 2p+4, 2p+5 (qs pair p+2, "upper").
    static constexpr int kElems = 256, kBytes = 144, kBlocksPerLane = 1, kLanesPerBlock = 2, kBlocksPerSlice = 16;
    static constexpr int kRun = 32, kRuns = 4, kGroup = 32, kGroupsPerLane = 4;
    static constexpr bool kR4 = false;
    // Lane l takes block l % 16 and half l / 16: each quarter-warp of a
    // 128-bit shared load then reads 8 blocks 144 B apart (bank offsets 4b),
    // conflict-free.
    __device__ static int lane_part(int lane) { return lane >> 4; }
    __device__ static int lane_block(int lane) { return lane & 15; }
    __device__ static int sub(int p, int r) { return 2 * p + r + (r >= 2 ? 2 : 0); }
    __device__ static int run_start(int blk, int p, int r) { return blk * 256 + sub(p, r) * 32; }
    __device__ static int group_index(int blk, int p, int r) { return blk * 8 + sub(p, r); }
};
template <>
struct Fmt<QT_Q4_K_R4> : Fmt<QT_Q4_K> {
    static constexpr bool kR4 = true;
};

template <>
struct Fmt<QT_Q6_K> {
    static constexpr int kElems = 256, kBytes = 210, kBlocksPerLane = 1, kLanesPerBlock = 8, kBlocksPerSlice = 4;
    static constexpr int kRun = 16, kRuns = 2, kGroup = 16, kGroupsPerLane = 2;
    static constexpr bool kR4 = false;
    __device__ static int lane_part(int lane) { return lane % kLanesPerBlock; }
    __device__ static int lane_block(int lane) { return (lane / kLanesPerBlock) * kBlocksPerLane; }
    // lane t = 4h + 2c + i16 holds groups g = 4h + c (r = 0) and 4h + c + 2 (r = 1).
    __device__ static int grp(int t, int r) { return 4 * (t >> 2) + ((t >> 1) & 1) + 2 * r; }
    __device__ static int run_start(int blk, int t, int r) { return blk * 256 + grp(t, r) * 32 + (t & 1) * 16; }
    __device__ static int group_index(int blk, int t, int r) { return blk * 16 + 2 * grp(t, r) + (t & 1); }
};
template <>
struct Fmt<QT_Q6_K_R4> : Fmt<QT_Q6_K> {
    static constexpr bool kR4 = true;
};

template <>
struct Fmt<QT_Q8_0> {
    // Lane l holds two consecutive blocks (2l, 2l+1 of its slice).
    static constexpr int kElems = 32, kBytes = 34, kLanesPerBlock = 1, kBlocksPerLane = 2, kBlocksPerSlice = 64;
    static constexpr int kRun = 32, kRuns = 2, kGroup = 32, kGroupsPerLane = 2;
    static constexpr bool kR4 = false;
    __device__ static int lane_part(int lane) { return lane % kLanesPerBlock; }
    __device__ static int lane_block(int lane) { return (lane / kLanesPerBlock) * kBlocksPerLane; }
    __device__ static int run_start(int blk, int, int r) { return (blk + r) * 32; }
    __device__ static int group_index(int blk, int, int r) { return blk + r; }
};
template <>
struct Fmt<QT_Q4_0> : Fmt<QT_Q8_0> {
    static constexpr int kBytes = 18;
};

template <>
struct Fmt<QT_Q6_K_LM> {
    static constexpr int kElems = 256, kBytes = 276, kBlocksPerLane = 1, kLanesPerBlock = 8, kBlocksPerSlice = 4;
    static constexpr int kRun = 32, kRuns = 1, kGroup = 16, kGroupsPerLane = 2;
    static constexpr bool kR4 = false;
    __device__ static int lane_part(int lane) { return lane % kLanesPerBlock; }
    __device__ static int lane_block(int lane) { return (lane / kLanesPerBlock) * kBlocksPerLane; }
    __device__ static int run_start(int blk, int t, int) { return blk * 256 + t * 32; }
    __device__ static int group_index(int blk, int t, int r) { return blk * 16 + 2 * t + r; }
};

// ---------------------------------------------------------------------------
// One lane's activation codes: a run of RUN consecutive elements of a
// quantized row (per 32-element group: int8 "x8" codes, or int16 "x16" codes
// split in a signed high byte plane and an unsigned low byte plane).
// ---------------------------------------------------------------------------
template <int DIG, int RUN>
struct XRun {
    uint32_t hi[RUN / 4];  // packed signed bytes (x8: the code; x16: high byte)
    uint32_t lo[DIG == 2 ? RUN / 4 : 1];  // packed unsigned low bytes (x16 only)
    float d;               // group scale
    int sum;               // sum of the codes in this run
    float fsum;            // the same sum as a float (exact: |sum| < 2^20)
};

__device__ __forceinline__ int round_half_even_small(float v) {
    // v in (-2^22, 2^22): adding 1.5*2^23 rounds to an integer with RNE.
    const float t = __fadd_rn(v, 12582912.0f);
    return __float_as_int(t) - 0x4B400000;
}

// Activation rows quantized once per call by b200q_quantize_act_kernel, in the
// layout the GEMV lanes read: per row, k signed code bytes (x8: the code;
// x16: its high byte), k unsigned low bytes (x16 only), k/32 fp32 group
// scales and k/32 int32 group code sums; xq_row_bytes(k, DIG) bytes per row.
__host__ __device__ constexpr long long xq_row_bytes(int k, int dig) {
    return ((static_cast<long long>(k) * dig + (k / 32) * 8) + 15) / 16 * 16;
}

// The same row as the GEMV stages it in shared memory: each code plane has
// 16 bytes of padding after every 256 codes, so the lanes of a warp (whose
// runs lie 256 codes apart) read their runs without bank conflicts.
// Plane length, byte offset of code e within a plane, and the row size:
__host__ __device__ constexpr int xs_plane_bytes(int k) { return k + 16 * ((k + 255) / 256); }
__host__ __device__ constexpr int xs_code_offset(int e) { return e + 16 * (e >> 8); }
__host__ __device__ constexpr int xs_row_bytes(int k, int dig) {
    return (dig * xs_plane_bytes(k) + (k / 32) * 8 + 15) / 16 * 16;
}

// Quantize one 32-element group v into a quantized row at `base` (group g
// of a row of k elements). The arithmetic is restated in the oracle as
// orc_quantize_act: amax, iscale = QMAX / amax (IEEE division),
// q = rint(x * iscale) (one rounded multiply, half-even), d = amax / QMAX.
template <int DIG>
__device__ __forceinline__ void quantize_group(const float (&v)[32], uint8_t* base, int k, int g) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    constexpr float QMAX = DIG == 1 ? 127.0f : 32767.0f;
    const float iscale = amax > 0.0f ? __fdiv_rn(QMAX, amax) : 0.0f;
    int sum = 0;
    uint32_t hw[8], lw[8];
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        uint32_t h = 0, l = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int q = round_half_even_small(__fmul_rn(v[4 * w + j], iscale));
            sum += q;
            if (DIG == 1) {
                h |= (static_cast<uint32_t>(q) & 0xFFu) << (8 * j);
            } else {
                h |= (static_cast<uint32_t>(q >> 8) & 0xFFu) << (8 * j);
                l |= (static_cast<uint32_t>(q) & 0xFFu) << (8 * j);
            }
        }
        hw[w] = h;
        lw[w] = l;
    }
    uint4* dh = reinterpret_cast<uint4*>(base + g * 32);
    dh[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    dh[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
    if (DIG == 2) {
        uint4* dl = reinterpret_cast<uint4*>(base + k + g * 32);
        dl[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        dl[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
    }
    float* gd = reinterpret_cast<float*>(base + static_cast<long long>(k) * DIG);
    gd[g] = amax > 0.0f ? __fdiv_rn(amax, QMAX) : 0.0f;
    reinterpret_cast<int*>(gd + k / 32)[g] = sum;
}

__device__ __forceinline__ void load_group(const float* p, float (&v)[32]) {
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
        const float4 f = __ldg(reinterpret_cast<const float4*>(p + i));
        v[i] = f.x;
        v[i + 1] = f.y;
        v[i + 2] = f.z;
        v[i + 3] = f.w;
    }
}

// One thread per 32-element group of m activation rows.
template <int DIG>
__global__ void __launch_bounds__(128) b200q_quantize_act_kernel(const float* __restrict__ x, long long x_stride, int m, int k,
                                                           uint8_t* __restrict__ xq) {
    // Let the GEMV behind this kernel launch now, so it can stream its
    // weights while this grid waits for x; x may be produced by the
    // preceding kernel in the stream.
    griddep_launch_dependents();
    griddep_wait();
    const int groups = k / 32;
    const long long gid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (gid >= static_cast<long long>(groups) * m) return;
    const int row = static_cast<int>(gid / groups), g = static_cast<int>(gid % groups);
    float v[32];
    load_group(x + row * x_stride + g * 32, v);
    quantize_group<DIG>(v, xq + row * xq_row_bytes(k, DIG), k, g);
}

// The same quantization with four elements per thread: the 8 threads of a
// 32-element group meet through warp shuffles for amax and the code sum, so
// a row of k elements is quantized by k/4 threads in one short step (the
// launch latency of this kernel sits between x's producer and the GEMV).
// Writes exactly what quantize_group writes. blockDim.x must be a multiple
// of 32.
// Quantize elements [4 q4, 4 q4 + 4) of a row held by this thread (v) into
// the quantized row at `base` (row of k elements). The 8 lanes holding one
// 32-element group must be the aligned lanes 8j .. 8j+7 of the warp, and every
// lane of the warp must call (valid == false for lanes without data; their
// v is ignored and nothing is stored).
template <int DIG>
__device__ __forceinline__ void quantize_quad(float4 v, bool valid, uint8_t* base, int k, int q4) {
    if (!valid) v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    constexpr float QMAX = DIG == 1 ? 127.0f : 32767.0f;
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
    const float iscale = amax > 0.0f ? __fdiv_rn(QMAX, amax) : 0.0f;
    const int c0 = round_half_even_small(__fmul_rn(v.x, iscale));
    const int c1 = round_half_even_small(__fmul_rn(v.y, iscale));
    const int c2 = round_half_even_small(__fmul_rn(v.z, iscale));
    const int c3 = round_half_even_small(__fmul_rn(v.w, iscale));
    int sum = c0 + c1 + c2 + c3;
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    sum += __shfl_xor_sync(0xffffffffu, sum, 4);
    if (!valid) return;
    uint32_t h, l = 0;
    if (DIG == 1) {
        h = (static_cast<uint32_t>(c0) & 0xFFu) | ((static_cast<uint32_t>(c1) & 0xFFu) << 8) |
            ((static_cast<uint32_t>(c2) & 0xFFu) << 16) | (static_cast<uint32_t>(c3) << 24);
    } else {
        h = (static_cast<uint32_t>(c0 >> 8) & 0xFFu) | ((static_cast<uint32_t>(c1 >> 8) & 0xFFu) << 8) |
            ((static_cast<uint32_t>(c2 >> 8) & 0xFFu) << 16) | (static_cast<uint32_t>(c3 >> 8) << 24);
        l = (static_cast<uint32_t>(c0) & 0xFFu) | ((static_cast<uint32_t>(c1) & 0xFFu) << 8) |
            ((static_cast<uint32_t>(c2) & 0xFFu) << 16) | (static_cast<uint32_t>(c3) << 24);
    }
    reinterpret_cast<uint32_t*>(base)[q4] = h;
    if (DIG == 2) reinterpret_cast<uint32_t*>(base + k)[q4] = l;
    if ((q4 & 7) == 0) {
        float* gd = reinterpret_cast<float*>(base + static_cast<long long>(k) * DIG);
        gd[q4 >> 3] = amax > 0.0f ? __fdiv_rn(amax, QMAX) : 0.0f;
        reinterpret_cast<int*>(gd + k / 32)[q4 >> 3] = sum;
    }
}

template <int DIG>
__global__ void __launch_bounds__(256) b200q_quantize_act_quads_kernel(const float* __restrict__ x, long long x_stride, int m,
                                                                  int k, uint8_t* __restrict__ xq) {
    griddep_launch_dependents();
    griddep_wait();
    const int quads = k >> 2;
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const bool valid = i < static_cast<long long>(m) * quads;  // groups never straddle the end
    const int row = valid ? static_cast<int>(i / quads) : 0;
    const int q4 = valid ? static_cast<int>(i - static_cast<long long>(row) * quads) : 0;
    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (valid) v = __ldg(reinterpret_cast<const float4*>(x + row * x_stride) + q4);
    quantize_quad<DIG>(v, valid, xq + row * xq_row_bytes(k, DIG), k, q4);
}

// One lane's run of RUN codes starting at element e (a multiple of 16) of a
// quantized row. The run's code sum is recomputed from the bytes when the
// run is half a group.
template <int DIG, int RUN>
__device__ __forceinline__ void load_run(const uint8_t* row, int k, int e, XRun<DIG, RUN>& out) {
    const uint4* h = reinterpret_cast<const uint4*>(row + e);
#pragma unroll
    for (int i = 0; i < RUN / 16; ++i) {
        const uint4 v = __ldg(h + i);
        out.hi[4 * i] = v.x;
        out.hi[4 * i + 1] = v.y;
        out.hi[4 * i + 2] = v.z;
        out.hi[4 * i + 3] = v.w;
    }
    if (DIG == 2) {
        const uint4* l = reinterpret_cast<const uint4*>(row + k + e);
#pragma unroll
        for (int i = 0; i < RUN / 16; ++i) {
            const uint4 v = __ldg(l + i);
            out.lo[4 * i] = v.x;
            out.lo[4 * i + 1] = v.y;
            out.lo[4 * i + 2] = v.z;
            out.lo[4 * i + 3] = v.w;
        }
    }
    const float* gd = reinterpret_cast<const float*>(row + static_cast<long long>(k) * DIG);
    out.d = __ldg(gd + e / 32);
    if (RUN == 32) {
        out.sum = __ldg(reinterpret_cast<const int*>(gd + k / 32) + e / 32);
    } else {
        int hs = 0, ls = 0;
#pragma unroll
        for (int w = 0; w < RUN / 4; ++w) {
            hs = dp4a_ss(out.hi[w], 0x01010101u, hs);
            if (DIG == 2) ls = dp4a_uu(out.lo[w], 0x01010101u, ls);
        }
        out.sum = DIG == 2 ? hs * 256 + ls : hs;
    }
    out.fsum = static_cast<float>(out.sum);
}

// Exact float of a signed integer |v| < 2^22 without a convert instruction:
// add it to the mantissa of 1.5 * 2^23 and subtract 1.5 * 2^23.
__device__ __forceinline__ float i2f_small(int v) { return __int_as_float(v + 0x4B400000) - 12582912.0f; }

// Float of a dot sum kept as two digit sums (x16: 256 * hi + lo, each
// |.| < 2^21), rounded once.
template <int DIG>
__device__ __forceinline__ float digits_to_float(int hi, int lo) {
    return DIG == 2 ? fmaf(256.0f, i2f_small(hi), i2f_small(lo)) : i2f_small(hi);
}

// Exact float of a small non-negative integer (< 2^23) without a convert:
// place it in the mantissa of 2^23 and subtract 2^23.
__device__ __forceinline__ float small_uint_to_float(uint32_t v) {
    return __uint_as_float(0x4B000000u | v) - 8388608.0f;
}

// sum_i code_i * q_i for four packed weight bytes (unsigned codes 0..255 or
// signed codes) against one activation word pair.
template <int DIG, bool SIGNED_W>
__device__ __forceinline__ void dot4(uint32_t w, uint32_t xh, uint32_t xl, int& acc_hi, int& acc_lo) {
    if (SIGNED_W) {
        acc_hi = dp4a_ss(w, xh, acc_hi);
        if (DIG == 2) acc_lo = dp4a_su(w, xl, acc_lo);
    } else {
        acc_hi = dp4a_us(w, xh, acc_hi);
        if (DIG == 2) acc_lo = dp4a_uu(w, xl, acc_lo);
    }
}

template <int DIG>
__device__ __forceinline__ int combine_digits(int hi, int lo) {
    return DIG == 2 ? hi * 256 + lo : hi;
}

// ---------------------------------------------------------------------------
// Per-format row dot: one lane's contribution for one weight row, for MR
// activation rows. `ba` is the shared-memory byte address of the lane's
// block. Group integer sums go to `isum` (used by the debug path).
// ---------------------------------------------------------------------------
template <int QT, int DIG, int MR>
struct RowDot;

// Exact float of byte 0 / byte 1 of v: the byte placed in the mantissa of
// 2^23 with one byte permute, then 2^23 subtracted.
__device__ __forceinline__ float byte0_to_float(uint32_t v) {
    return __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7540)) - 8388608.0f;
}
__device__ __forceinline__ float byte1_to_float(uint32_t v) {
    return __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7541)) - 8388608.0f;
}

// Q4_K (quantized_matmul.cpp:411-515, scale decode :423-437). Lane p of a
// block reads qs pairs p and p+2 (bytes [32p, 32p+32) and [64+32p, 96+32p)):
// sub-blocks 2p and 2p+4 are their low nibbles, 2p+1 and 2p+5 the high
// nibbles. High nibbles are masked in place (0xF0 per byte), so their dp4a
// sums come out x16 and the 1/16 is folded into the activation scale
// (xdd). Scales and mins of the lane's four sub-blocks need no selects:
// pair p uses the "lower" 6-bit encoding, pair p+2 the "upper" one.
template <int DIG, int MR>
struct Q4KDot {
    using X = XRun<DIG, 32>;
    __device__ static void run(uint32_t ba, int p, const X (&x)[MR][4], const float (&xdd)[MR][4],
                               const float (&xsd)[MR][4], float (&acc)[MR], int (&isum)[4]) {
        const uint4 h = lds128(ba);
        const uint32_t qa = ba + 16u + 32u * p;
        const uint4 a0 = lds128(qa), a1 = lds128(qa + 16u);
        const uint4 b0 = lds128(qa + 64u), b1 = lds128(qa + 80u);
        const float d = half_bits_to_float(h.x);
        const float dmin = half_bits_to_float(h.x >> 16);
        const uint32_t sh = 16u * p;
        const uint32_t A = h.y >> sh, B = h.z >> sh, C = h.w >> sh;
        const uint32_t scl = A & 0x3F3Fu, mnl = B & 0x3F3Fu;
        const uint32_t sch = (C & 0x0F0Fu) | ((A >> 2) & 0x3030u);
        const uint32_t mnh = ((C >> 4) & 0x0F0Fu) | ((B >> 2) & 0x3030u);
        const float sc[4] = {byte0_to_float(scl), byte1_to_float(scl), byte0_to_float(sch), byte1_to_float(sch)};
        const float mn[4] = {byte0_to_float(mnl), byte1_to_float(mnl), byte0_to_float(mnh), byte1_to_float(mnh)};
        const uint32_t qw[2][8] = {{a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w},
                                   {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w}};
#pragma unroll
        for (int m = 0; m < MR; ++m) {
            int hs[4] = {0, 0, 0, 0}, ls[4] = {0, 0, 0, 0};
#pragma unroll
            for (int pr = 0; pr < 2; ++pr) {
#pragma unroll
                for (int w = 0; w < 8; ++w) {
                    const uint32_t lo = qw[pr][w] & 0x0F0F0F0Fu;
                    const uint32_t hi16 = qw[pr][w] & 0xF0F0F0F0u;
                    dot4<DIG, false>(lo, x[m][2 * pr].hi[w], DIG == 2 ? x[m][2 * pr].lo[w] : 0u, hs[2 * pr], ls[2 * pr]);
                    dot4<DIG, false>(hi16, x[m][2 * pr + 1].hi[w], DIG == 2 ? x[m][2 * pr + 1].lo[w] : 0u, hs[2 * pr + 1],
                                     ls[2 * pr + 1]);
                }
            }
            if (m == 0) {
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int v = combine_digits<DIG>(hs[r], ls[r]);
                    isum[r] = (r & 1) ? (v >> 4) : v;
                }
            }
            float S = 0.0f, M = 0.0f;
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                S = fmaf(sc[r], xdd[m][r] * digits_to_float<DIG>(hs[r], ls[r]), S);
                M = fmaf(mn[r], xsd[m][r], M);
            }
            acc[m] = fmaf(d, S, fmaf(-dmin, M, acc[m]));
        }
    }
};

// Q6_K (quantized_matmul.cpp:683-775). Lane t = 4h + 2c + i16 reads the 16
// ql bytes at 64h + 32c + 16*i16 (groups 4h+c low nibbles, 4h+c+2 high
// nibbles) and the 16 qh bytes at 128 + 32h + 16*i16.
template <int DIG, int MR>
struct Q6KDot {
    using X = XRun<DIG, 16>;
    __device__ static void run(uint32_t ba, int t, const X (&x)[MR][2], float (&acc)[MR], int (&isum)[4]) {
        const int h = t >> 2, c = (t >> 1) & 1, i16 = t & 1;
        uint32_t ql[4], qh[4];
        lds_words_unaligned<4>(ba + 64u * h + 32u * c + 16u * i16, ql);
        lds_words_unaligned<4>(ba + 128u + 32u * h + 16u * i16, qh);
        const int g0 = 4 * h + c, g1 = g0 + 2;
        const float d = half_bits_to_float(lds_u16(ba + 208u));
        const float s0 = d * i2f_small(lds_s8(ba + 192u + 2u * g0 + i16));
        const float s1 = d * i2f_small(lds_s8(ba + 192u + 2u * g1 + i16));
        const uint32_t sh0 = 2u * c, sh1 = 2u * c + 4u;
        uint32_t u0[4], u1[4];
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            u0[w] = (ql[w] & 0x0F0F0F0Fu) | (((qh[w] >> sh0) & 0x03030303u) << 4);
            u1[w] = ((ql[w] >> 4) & 0x0F0F0F0Fu) | (((qh[w] >> sh1) & 0x03030303u) << 4);
        }
#pragma unroll
        for (int m = 0; m < MR; ++m) {
            int a_hi = 0, a_lo = 0, b_hi = 0, b_lo = 0;
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                dot4<DIG, false>(u0[w], x[m][0].hi[w], DIG == 2 ? x[m][0].lo[w] : 0u, a_hi, a_lo);
                dot4<DIG, false>(u1[w], x[m][1].hi[w], DIG == 2 ? x[m][1].lo[w] : 0u, b_hi, b_lo);
            }
            // codes are stored +32: subtract 32 * sum(q) to get sum((c-32) * q)
            const int ia = combine_digits<DIG>(a_hi, a_lo) - 32 * x[m][0].sum;
            const int ib = combine_digits<DIG>(b_hi, b_lo) - 32 * x[m][1].sum;
            if (m == 0) {
                isum[0] = ia;
                isum[1] = ib;
            }
            const float fa = fmaf(-32.0f, x[m][0].fsum, digits_to_float<DIG>(a_hi, a_lo));
            const float fb = fmaf(-32.0f, x[m][1].fsum, digits_to_float<DIG>(b_hi, b_lo));
            float a = acc[m];
            a = fmaf(s0, x[m][0].d * fa, a);
            a = fmaf(s1, x[m][1].d * fb, a);
            acc[m] = a;
        }
    }
};

// Q8_0 (quantized_matmul.cpp:1041-1081): fp16 d then 32 int8 codes. The
// lane's two blocks are consecutive; `v1` is false when the second lies past
// the end of the row (its contribution is dropped).
template <int DIG, int MR>
struct Q80Dot {
    using X = XRun<DIG, 32>;
    __device__ static void run(uint32_t ba, bool v1, const X (&x)[MR][2], float (&acc)[MR], int (&isum)[4]) {
        uint32_t q[2][8];
        lds_words_unaligned<8>(ba + 2u, q[0]);
        lds_words_unaligned<8>(ba + 36u, q[1]);
        const float d[2] = {half_bits_to_float(lds_u16(ba)), v1 ? half_bits_to_float(lds_u16(ba + 34u)) : 0.0f};
#pragma unroll
        for (int m = 0; m < MR; ++m) {
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                int a_hi = 0, a_lo = 0;
#pragma unroll
                for (int w = 0; w < 8; ++w)
                    dot4<DIG, true>(q[b][w], x[m][b].hi[w], DIG == 2 ? x[m][b].lo[w] : 0u, a_hi, a_lo);
                if (m == 0) isum[b] = combine_digits<DIG>(a_hi, a_lo);
                acc[m] = fmaf(d[b], x[m][b].d * digits_to_float<DIG>(a_hi, a_lo), acc[m]);
            }
        }
    }
};

// Q4_0 (ggml type 2): fp16 d then 16 bytes; element i < 16 is the low
// nibble of byte i, element 16 + i the high nibble; value d * (q - 8). Two
// consecutive blocks per lane, as for Q8_0.
template <int DIG, int MR>
struct Q40Dot {
    using X = XRun<DIG, 32>;
    __device__ static void run(uint32_t ba, bool v1, const X (&x)[MR][2], float (&acc)[MR], int (&isum)[4]) {
        uint32_t q[2][4];
        lds_words_unaligned<4>(ba + 2u, q[0]);
        lds_words_unaligned<4>(ba + 20u, q[1]);
        const float d[2] = {half_bits_to_float(lds_u16(ba)), v1 ? half_bits_to_float(lds_u16(ba + 18u)) : 0.0f};
#pragma unroll
        for (int m = 0; m < MR; ++m) {
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                int a_hi = 0, a_lo = 0;
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    const uint32_t lo = q[b][w] & 0x0F0F0F0Fu;
                    const uint32_t hi = (q[b][w] >> 4) & 0x0F0F0F0Fu;
                    dot4<DIG, false>(lo, x[m][b].hi[w], DIG == 2 ? x[m][b].lo[w] : 0u, a_hi, a_lo);
                    dot4<DIG, false>(hi, x[m][b].hi[4 + w], DIG == 2 ? x[m][b].lo[4 + w] : 0u, a_hi, a_lo);
                }
                if (m == 0) isum[b] = combine_digits<DIG>(a_hi, a_lo) - 8 * x[m][b].sum;
                const float fa = fmaf(-8.0f, x[m][b].fsum, digits_to_float<DIG>(a_hi, a_lo));
                acc[m] = fmaf(d[b], x[m][b].d * fa, acc[m]);
            }
        }
    }
};

// Q6_K_LM (quantized_matmul.cpp:302-365, 1083-1154): 256 int8 codes in
// element order, 16 int8 scales, fp32 d. Lane t holds elements [32t, 32t+32)
// (scale groups 2t and 2t+1).
template <int DIG, int MR>
struct Q6KLMDot {
    using X = XRun<DIG, 32>;
    __device__ static void run(uint32_t ba, int t, const X (&x)[MR][1], float (&acc)[MR], int (&isum)[4]) {
        uint32_t q[8];
#pragma unroll
        for (int w = 0; w < 8; ++w) q[w] = lds32(ba + 32u * t + 4u * w);
        const uint32_t scw = lds_u16(ba + 256u + 2u * t);
        float dd;
        {
            const uint32_t db = lds32(ba + 272u);
            dd = __uint_as_float(db);
        }
        const float s0 = dd * i2f_small(static_cast<int8_t>(scw & 0xFFu));
        const float s1 = dd * i2f_small(static_cast<int8_t>((scw >> 8) & 0xFFu));
#pragma unroll
        for (int m = 0; m < MR; ++m) {
            int a_hi = 0, a_lo = 0, b_hi = 0, b_lo = 0;
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                dot4<DIG, true>(q[w], x[m][0].hi[w], DIG == 2 ? x[m][0].lo[w] : 0u, a_hi, a_lo);
                dot4<DIG, true>(q[4 + w], x[m][0].hi[4 + w], DIG == 2 ? x[m][0].lo[4 + w] : 0u, b_hi, b_lo);
            }
            const int ia = combine_digits<DIG>(a_hi, a_lo);
            const int ib = combine_digits<DIG>(b_hi, b_lo);
            if (m == 0) {
                isum[0] = ia;
                isum[1] = ib;
            }
            acc[m] = fmaf(s0, x[m][0].d * digits_to_float<DIG>(a_hi, a_lo), acc[m]);
            acc[m] = fmaf(s1, x[m][0].d * digits_to_float<DIG>(b_hi, b_lo), acc[m]);
        }
    }
};

// Byte offset of (row, blk) inside a stage whose first row is `r0` (a
// multiple of 4 for the R4 layouts).
template <int QT>
__device__ __forceinline__ uint32_t stage_offset(int row, int r0, int blk, uint32_t row_bytes, int n) {
    using F = Fmt<QT>;
    if (F::kR4) {
        const int full4 = (n / 4) * 4;
        if (row < full4)
            return static_cast<uint32_t>((row & ~3) - r0) * row_bytes + static_cast<uint32_t>(blk * 4 + (row & 3)) * F::kBytes;
    }
    return static_cast<uint32_t>(row - r0) * row_bytes + static_cast<uint32_t>(blk) * F::kBytes;
}

// Sum V values across the warp, V in {1, 2, 4}: the first log2(V) butterfly
// levels trade halves of the value set (each lane keeps one half), the rest
// reduce the survivor. On return, lane (i >> 1) * 16 + (i & 1) * 8 ... more
// precisely the lane whose bits 4..(5 - log2 V) spell index i holds sum i;
// warp_sum_lane(i) gives it.
template <int V>
__device__ __forceinline__ float warp_sum_multi(float (&v)[V], int lane) {
    if constexpr (V == 1) {
        float a = v[0];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
        return a;
    } else if constexpr (V == 2) {
        const bool hi = (lane & 16) != 0;
        float a = (hi ? v[1] : v[0]) + __shfl_xor_sync(0xffffffffu, hi ? v[0] : v[1], 16);
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
        return a;
    } else {
        const bool h16 = (lane & 16) != 0;
        const float b0 = (h16 ? v[2] : v[0]) + __shfl_xor_sync(0xffffffffu, h16 ? v[0] : v[2], 16);
        const float b1 = (h16 ? v[3] : v[1]) + __shfl_xor_sync(0xffffffffu, h16 ? v[1] : v[3], 16);
        const bool h8 = (lane & 8) != 0;
        float a = (h8 ? b1 : b0) + __shfl_xor_sync(0xffffffffu, h8 ? b0 : b1, 8);
#pragma unroll
        for (int off = 4; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
        return a;
    }
}
// Lane holding sum i after warp_sum_multi<V>.
template <int V>
__device__ __forceinline__ int warp_sum_lane(int i) {
    return V == 1 ? 0 : (V == 2 ? 16 * i : 16 * (i >> 1) + 8 * (i & 1));
}

// One lane's run of RUN codes starting at element e of a staged row (padded
// layout) at shared-memory byte address `row`.
template <int DIG, int RUN>
__device__ __forceinline__ void load_run_smem(uint32_t row, int k, int e, XRun<DIG, RUN>& out) {
    const uint32_t kp = static_cast<uint32_t>(xs_plane_bytes(k));
    const uint32_t ce = static_cast<uint32_t>(xs_code_offset(e));  // a run never crosses a 256-code boundary
#pragma unroll
    for (int i = 0; i < RUN / 16; ++i) {
        const uint4 v = lds128(row + ce + 16u * i);
        out.hi[4 * i] = v.x;
        out.hi[4 * i + 1] = v.y;
        out.hi[4 * i + 2] = v.z;
        out.hi[4 * i + 3] = v.w;
    }
    if (DIG == 2) {
#pragma unroll
        for (int i = 0; i < RUN / 16; ++i) {
            const uint4 v = lds128(row + kp + ce + 16u * i);
            out.lo[4 * i] = v.x;
            out.lo[4 * i + 1] = v.y;
            out.lo[4 * i + 2] = v.z;
            out.lo[4 * i + 3] = v.w;
        }
    }
    const uint32_t gd = row + kp * DIG;
    out.d = __uint_as_float(lds32(gd + 4u * static_cast<uint32_t>(e / 32)));
    if (RUN == 32) {
        out.sum = static_cast<int>(lds32(gd + 4u * static_cast<uint32_t>(k / 32 + e / 32)));
    } else {
        int hs = 0, ls = 0;
#pragma unroll
        for (int w = 0; w < RUN / 4; ++w) {
            hs = dp4a_ss(out.hi[w], 0x01010101u, hs);
            if (DIG == 2) ls = dp4a_uu(out.lo[w], 0x01010101u, ls);
        }
        out.sum = DIG == 2 ? hs * 256 + ls : hs;
    }
    out.fsum = static_cast<float>(out.sum);
}

// Stage MR rows of activation codes a preceding kernel wrote (xq layout) in
// shared memory (xs, generic pointer; rows xs_row bytes apart in the padded
// layout), using all warps, four 16-byte words per thread per trip.
// `on_issued` runs on thread 0 once its first loads are issued (the weight
// stages held back until then are issued behind them).
template <int DIG, int MR, class OnIssued>
__device__ __forceinline__ void stage_codes(const GemvParams& p, uint8_t* xs, int xs_row, int warp, int lane,
                                            int nwarps, OnIssued on_issued) {
    const int kp = xs_plane_bytes(p.k);
    const int nthreads = nwarps * 32, tid = warp * 32 + lane;
    bool first = true;
    constexpr int B = 4;  // 16-byte words a thread loads per trip
    const int words = static_cast<int>(xq_row_bytes(p.k, DIG) >> 4);
    const int code_words = (DIG * p.k) >> 4;
    const int total = MR * words;
    for (int i0 = tid; i0 < total; i0 += B * nthreads) {
        uint4 v[B];
#pragma unroll
        for (int b = 0; b < B; ++b) {
            const int i = i0 + b * nthreads;
            if (i < total) {
                const int row = i / words, w = i - row * words;
                v[b] = __ldg(reinterpret_cast<const uint4*>(p.xq + row * p.xq_stride) + w);
            }
        }
        if (first && tid == 0) on_issued();
        first = false;
#pragma unroll
        for (int b = 0; b < B; ++b) {
            const int i = i0 + b * nthreads;
            if (i < total) {
                const int row = i / words, w = i - row * words;
                int off;
                if (w < code_words) {
                    const int plane = (16 * w) / p.k, e = 16 * w - plane * p.k;
                    off = plane * kp + xs_code_offset(e);
                } else {
                    off = DIG * kp + (16 * w - DIG * p.k);
                }
                *reinterpret_cast<uint4*>(xs + row * xs_row + off) = v[b];
            }
        }
    }
    if (first && tid == 0) on_issued();
}

// Quantize the fp32 rows staged in shared memory (xf4: MR rows of k, then
// the RMSNorm gains when `norm`, or the up row when `swiglu`) into the
// padded code rows at xs, one
// 32-element group per lane: the arithmetic of quantize_group (amax,
// iscale = QMAX / amax by IEEE division, one rounded multiply, half-even
// codes, d = amax / QMAX, the group's code sum), one division each per
// group. A lane reads its group's eight float4 in an order rotated by its
// group index and stores each code word at the matching position, so the
// lanes of a quarter-warp (groups 128 B apart) use different banks. With
// `norm` (one row, one group per lane covering it -- host-checked) the row
// is first scaled by 1 / sqrt(sum(x^2) / k + eps) and by the gains, the sum
// of squares reduced per warp into `red` and summed in warp order.
template <int DIG, int MR>
__device__ __forceinline__ void quantize_staged_rows(const GemvParams& p, const float4* xf4, bool norm, bool swiglu,
                                                     uint8_t* xs, int xs_row, float* red, int warp, int lane,
                                                     int nwarps) {
    const int nthreads = nwarps * 32;
    const int kp = xs_plane_bytes(p.k);
    const int groups = p.k >> 5;
    const int total_g = MR * groups;
    constexpr float QMAX = DIG == 1 ? 127.0f : 32767.0f;
    for (int g0 = warp * 32; g0 < total_g || (norm && g0 == warp * 32); g0 += nthreads) {
        const int g = g0 + lane;
        const bool valid = g < total_g;
        float4 f[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
            f[i] = valid ? xf4[g * 8 + ((i + g) & 7)] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (norm) {
            float ss = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                ss = fmaf(f[i].x, f[i].x, ss);
                ss = fmaf(f[i].y, f[i].y, ss);
                ss = fmaf(f[i].z, f[i].z, ss);
                ss = fmaf(f[i].w, f[i].w, ss);
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if (lane == 0) red[warp] = ss;
            named_bar_sync(2, static_cast<uint32_t>(nthreads));
            float tot = 0.0f;
            for (int w = 0; w < nwarps; ++w) tot += red[w];
            const float inv_rms = 1.0f / sqrtf(tot / static_cast<float>(p.k) + p.eps);
            if (valid) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float4 gm = xf4[total_g * 8 + g * 8 + ((i + g) & 7)];
                    f[i] = make_float4(f[i].x * inv_rms * gm.x, f[i].y * inv_rms * gm.y, f[i].z * inv_rms * gm.z,
                                       f[i].w * inv_rms * gm.w);
                }
            }
        }
        if (swiglu && valid) {  // silu(gate) * up, as b200q_swiglu_quantize_kernel forms it
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float4 u = xf4[total_g * 8 + g * 8 + ((i + g) & 7)];
                f[i] = make_float4(f[i].x / (1.0f + expf(-f[i].x)) * u.x, f[i].y / (1.0f + expf(-f[i].y)) * u.y,
                                   f[i].z / (1.0f + expf(-f[i].z)) * u.z, f[i].w / (1.0f + expf(-f[i].w)) * u.w);
            }
        }
        if (valid) {
            float m4[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
                m4[i] = fmaxf(fmaxf(fabsf(f[i].x), fabsf(f[i].y)), fmaxf(fabsf(f[i].z), fabsf(f[i].w)));
            const float amax = fmaxf(fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])),
                                     fmaxf(fmaxf(m4[4], m4[5]), fmaxf(m4[6], m4[7])));
            const float iscale = amax > 0.0f ? __fdiv_rn(QMAX, amax) : 0.0f;
            const int row = g / groups, gi = g - row * groups;
            uint8_t* xrow = xs + row * xs_row;
            int ws[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int c0 = round_half_even_small(__fmul_rn(f[i].x, iscale));
                const int c1 = round_half_even_small(__fmul_rn(f[i].y, iscale));
                const int c2 = round_half_even_small(__fmul_rn(f[i].z, iscale));
                const int c3 = round_half_even_small(__fmul_rn(f[i].w, iscale));
                ws[i] = (c0 + c1) + (c2 + c3);
                const int off = xs_code_offset(gi * 32) + 4 * ((i + g) & 7);
                if (DIG == 1) {
                    *reinterpret_cast<uint32_t*>(xrow + off) =
                        __byte_perm(__byte_perm(c0, c1, 0x0040), __byte_perm(c2, c3, 0x0040), 0x5410);
                } else {
                    *reinterpret_cast<uint32_t*>(xrow + off) =
                        __byte_perm(__byte_perm(c0, c1, 0x0051), __byte_perm(c2, c3, 0x0051), 0x5410);
                    *reinterpret_cast<uint32_t*>(xrow + kp + off) =
                        __byte_perm(__byte_perm(c0, c1, 0x0040), __byte_perm(c2, c3, 0x0040), 0x5410);
                }
            }
            float* gd = reinterpret_cast<float*>(xrow + DIG * kp);
            gd[gi] = amax > 0.0f ? __fdiv_rn(amax, QMAX) : 0.0f;
            reinterpret_cast<int*>(gd + groups)[gi] =
                ((ws[0] + ws[1]) + (ws[2] + ws[3])) + ((ws[4] + ws[5]) + (ws[6] + ws[7]));
        }
        if (norm) break;
    }
}

// ---------------------------------------------------------------------------
// The kernel: one CTA per SM streams a contiguous slab of rows through a
// ring of NS shared-memory stages of R rows (1-D bulk copies, L2
// evict-first, no multicast; stages stay >= ~16 KB, since the copies in
// flight per SM are limited in number). Warp NW (the producer) issues every
// copy. The NW consumer warps are S k-slices x WR walkers, in G groups of SW
// walkers; stage s belongs to group s % G, whose S x SW warps take their
// slice of its rows, U rows at a time, the SW walkers of a slice
// interleaved, and release it with one arrival each on the slot's empty
// barrier.
//
// The order of the requests is chosen for the memory system, whose queues
// serve them roughly in order (a request waits behind the bytes requested
// before it): the producer issues PD weight stages at CTA start (before the
// grid dependency resolves, when the weights are static), then -- once the
// activations may be read -- their copy first and the rest of the ring
// behind it. FQ instances bring the fp32 rows (and the RMSNorm gains) in
// with one bulk copy per row into the last nx ring slots; the consumers
// quantize them there into the codes area (which has its own bytes past the
// ring) and hand the slots back to the producer (xdone). Code instances copy
// the codes with plain loads; the producer issues the ring's remaining
// stages once thread 0 has issued its loads (a shared-memory flag; a bounded
// wait that only paces, never fails).
// ---------------------------------------------------------------------------
template <int QT, int DIG, int MR, bool DBG, bool FQ>
__global__ void __launch_bounds__(kGemvWarps<DIG, MR> * 32 + 32, 1) b200q_gemv_kernel(const GemvParams p) {
    using F = Fmt<QT>;
    constexpr int RUN = F::kRun;
    constexpr int RUNS = F::kRuns;
    constexpr int NG = F::kGroupsPerLane;
    using X = XRun<DIG, RUN>;

    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int nwarps = p.S * p.WR;
    const int nthreads = nwarps * 32;

    // Layout: ring | staged activation codes | full barriers | empty
    // barriers | x barrier | x-done barrier | x-loads flag | per-warp sums
    // (RMSNorm) | slice partials.
    uint8_t* ring = smem;
    uint8_t* xs = smem + p.x_off;
    const int xs_row = xs_row_bytes(p.k, DIG);
    uint64_t* full = reinterpret_cast<uint64_t*>(xs + MR * xs_row);
    uint64_t* empty = full + p.NS;
    uint64_t* xbar = empty + p.NS;
    uint64_t* xdone = xbar + 1;
    uint32_t* xflag = reinterpret_cast<uint32_t*>(xdone + 1);
    float* red = reinterpret_cast<float*>(xflag + 1);
    float* part = red + kGemvMaxWarps;  // [rows of this CTA][MR][S]

    // Contiguous slab of rows per CTA, balanced to one row (to one 4-row
    // group for the R4 layouts).
    const int unit = F::kR4 ? 4 : 1;
    const int n_units = F::kR4 ? p.n_quads : p.n;
    const int u0 = static_cast<int>(static_cast<long long>(blockIdx.x) * n_units / gridDim.x);
    const int u1 = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * n_units / gridDim.x);
    const int r_begin = u0 * unit;
    const int r_end = min(u1 * unit, p.n);
    const int n_stages = r_end > r_begin ? (r_end - r_begin + p.R - 1) / p.R : 0;
    const int free_slots = p.NS - (FQ ? p.nx : 0);  // slots the weights have before the activations are staged
    const bool norm = FQ && MR == 1 && p.gamma != nullptr;
    const bool swiglu = FQ && MR == 1 && p.xu != nullptr;  // never together with norm (host-checked)
    float* xf_s = reinterpret_cast<float*>(ring + static_cast<size_t>(free_slots) * p.stage_stride);  // FQ fp32 rows

    if (tid == 0) {
        for (int i = 0; i < p.NS; ++i) {
            mbar_init(smem_addr(full + i), 1);
            mbar_init(smem_addr(empty + i), static_cast<uint32_t>(p.S * p.SW));
        }
        mbar_init(smem_addr(xbar), 1);
        mbar_init(smem_addr(xdone), static_cast<uint32_t>(nwarps));
        *xflag = 0u;
        fence_mbar_init();
    }
    __syncthreads();
    // Let the next kernel in the stream launch as soon as SMs free up; it
    // still waits (griddepcontrol.wait) for this grid before touching its
    // own inputs.
    griddep_launch_dependents();

    if (warp == nwarps) {
        // ---------------- producer ----------------
        if (lane == 0 && n_stages > 0) {
            const uint64_t pol = l2_policy_evict_first();
            // Stage s into its slot: the 16-byte-aligned window around the
            // stage's rows (consumers add (r0 * row_bytes) & 15 to find the
            // first row).
            auto issue = [&](int s) {
                const int slot = s % p.NS;
                const int r0 = r_begin + s * p.R;
                const int rows = min(p.R, r_end - r0);
                const long long b0 = (r0 * p.row_bytes) & ~15ll;
                const long long b1 = ((r0 + rows) * p.row_bytes + 15) & ~15ll;
                const uint32_t bytes = static_cast<uint32_t>(b1 - b0);
                const uint32_t fb = smem_addr(full + slot);
                mbar_arrive_expect_tx(fb, bytes);
                bulk_g2s(smem_addr(ring + static_cast<size_t>(slot) * p.stage_stride), p.W + b0, bytes, fb, pol);
            };
            const uint32_t x_bytes = static_cast<uint32_t>(MR * p.k * 4);
            const uint32_t g_bytes = (norm || swiglu) ? static_cast<uint32_t>(p.k * 4) : 0u;
            const int first_batch = min(n_stages, min(p.PD, free_slots));
            const int pre_fill = min(n_stages, free_slots);
            const int ring_fill = min(n_stages, p.NS);
            auto start = [&]() {
                for (int s = 0; s < first_batch; ++s) issue(s);
                if (FQ) {
                    mbar_arrive_expect_tx(smem_addr(xbar), x_bytes + g_bytes);
                    if (norm) bulk_g2s(smem_addr(xf_s + MR * p.k), p.gamma, g_bytes, smem_addr(xbar), pol);
                }
            };
            // Weights (and gains) may stream before the preceding kernel
            // finishes only when the caller declared them static.
            if (p.w_static) start();
            griddep_wait();
            if (!p.w_static) start();
            bool ok = true;
            if (FQ) {
                for (int m = 0; m < MR; ++m)
                    bulk_g2s(smem_addr(xf_s + m * p.k), p.xf + m * p.xf_stride, static_cast<uint32_t>(p.k * 4),
                             smem_addr(xbar), pol);
                if (swiglu)  // the up row, written by the preceding kernel like x
                    bulk_g2s(smem_addr(xf_s + MR * p.k), p.xu, g_bytes, smem_addr(xbar), pol);
                for (int s = first_batch; s < pre_fill; ++s) issue(s);
                // The fp32 slots return once every consumer warp has quantized.
                ok = mbar_wait_bounded(smem_addr(xdone), 0u);
                if (ok)
                    for (int s = pre_fill; s < ring_fill; ++s) issue(s);
            } else {
                // Pacing only: proceed after ~20 us even if the flag never comes.
                const uint64_t t0 = global_timer_ns();
                while (lds_volatile(smem_addr(xflag)) == 0u && global_timer_ns() - t0 < 20000ull) {
                }
                for (int s = first_batch; s < ring_fill; ++s) issue(s);
            }
            int issued = ok ? ring_fill : first_batch;
            for (int s = ring_fill; s < n_stages && ok; ++s) {
                const int slot = s % p.NS;
                if (!mbar_wait_bounded(smem_addr(empty + slot), static_cast<uint32_t>(((s / p.NS) - 1) & 1))) {
                    ok = false;
                    break;
                }
                issue(s);
                issued = s + 1;
            }
            if (!ok) *p.status = STATUS_TIMEOUT;
            // Do not let the CTA retire with copies in flight: wait (bounded)
            // for the last stages issued.
            for (int s = max(0, issued - p.NS); s < issued; ++s)
                (void)mbar_wait_bounded(smem_addr(full + s % p.NS), static_cast<uint32_t>((s / p.NS) & 1));
            if (FQ) (void)mbar_wait_bounded(smem_addr(xbar), 0u);
        }
        return;
    }

    // ---------------- consumers ----------------
    // The activations (fp32 rows, or their codes) are written by the
    // preceding kernel. Stage them once per CTA, then every lane takes its
    // runs into registers.
    griddep_wait();
    if constexpr (FQ) {
        if (!mbar_wait_spin_bounded(smem_addr(xbar), 0u) && tid == 0) *p.status = STATUS_TIMEOUT;
        quantize_staged_rows<DIG, MR>(p, reinterpret_cast<const float4*>(xf_s), norm, swiglu, xs, xs_row, red, warp,
                                      lane, nwarps);
        // The fp32 slots go back to the weights: order this thread's reads of
        // them before the bulk copies that overwrite them.
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(xdone));
    } else {
        stage_codes<DIG, MR>(p, xs, xs_row, warp, lane, nwarps, [&]() { sts_volatile(smem_addr(xflag), 1u); });
    }
    named_bar_sync(1, static_cast<uint32_t>(nthreads));

    const int slice = warp % p.S;
    const int walker = warp / p.S;
    const int group = walker / p.SW, sub = walker - group * p.SW;
    const int t = F::lane_part(lane);
    const int blk = slice * F::kBlocksPerSlice + F::lane_block(lane);
    const bool active = blk < p.nb;
    const bool active1 = blk + 1 < p.nb;  // second block of a two-block lane
    const int blk_c = active ? blk : 0;

    X x[MR][RUNS];
    float xdd[MR][RUNS];  // group scale (with the x16 factor of in-place high nibbles folded in)
    float xsd[MR][RUNS];  // group scale * group code sum (Q4_K mins)
    const uint32_t xs_addr = smem_addr(xs);
#pragma unroll
    for (int m = 0; m < MR; ++m) {
#pragma unroll
        for (int r = 0; r < RUNS; ++r) {
            const int e = F::run_start(blk_c, t, r);
            load_run_smem<DIG, RUN>(xs_addr + static_cast<uint32_t>(m * xs_row), p.k, e < p.k ? e : 0, x[m][r]);
            xdd[m][r] = ((QT == QT_Q4_K || QT == QT_Q4_K_R4) && (r & 1)) ? x[m][r].d * 0.0625f : x[m][r].d;
            xsd[m][r] = x[m][r].d * x[m][r].fsum;
        }
    }

    constexpr int U = kRowsPerIter<DIG, MR>;
    constexpr int V = U * MR;
    bool ok = true;
    const uint32_t ring_base = smem_addr(ring);
    const uint32_t rb32 = static_cast<uint32_t>(p.row_bytes);
    for (int s = group; s < n_stages; s += p.G) {
        const int slot = s % p.NS;
        const uint32_t use = static_cast<uint32_t>(s / p.NS);
        const int r0 = r_begin + s * p.R;
        const int rows = min(p.R, r_end - r0);
        if (ok && !mbar_wait_spin_bounded(smem_addr(full + slot), use & 1u)) {
            if (lane == 0) *p.status = STATUS_TIMEOUT;
            ok = false;
        }
        const uint32_t sbase = ring_base + static_cast<uint32_t>(slot) * static_cast<uint32_t>(p.stage_stride) +
                               static_cast<uint32_t>((r0 * p.row_bytes) & 15ll);
        for (int rl0 = sub * U; rl0 < rows; rl0 += p.SW * U) {
            float acc[U][MR];
            int isum[U][4];
#pragma unroll
            for (int u = 0; u < U; ++u) {
#pragma unroll
                for (int m = 0; m < MR; ++m) acc[u][m] = 0.0f;
            }
            if (ok) {
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    // A short last group repeats its last row; the copy's
                    // results are discarded.
                    const int row = r0 + min(rl0 + u, rows - 1);
                    const uint32_t ba = sbase + stage_offset<QT>(row, r0, blk_c, rb32, p.n);
                    if constexpr (QT == QT_Q4_K || QT == QT_Q4_K_R4) {
                        Q4KDot<DIG, MR>::run(ba, t, x, xdd, xsd, acc[u], isum[u]);
                    } else if constexpr (QT == QT_Q6_K || QT == QT_Q6_K_R4) {
                        Q6KDot<DIG, MR>::run(ba, t, x, acc[u], isum[u]);
                    } else if constexpr (QT == QT_Q8_0) {
                        Q80Dot<DIG, MR>::run(ba, active1, x, acc[u], isum[u]);
                    } else if constexpr (QT == QT_Q4_0) {
                        Q40Dot<DIG, MR>::run(ba, active1, x, acc[u], isum[u]);
                    } else if constexpr (QT == QT_Q6_K_LM) {
                        Q6KLMDot<DIG, MR>::run(ba, t, x, acc[u], isum[u]);
                    }
                }
                if constexpr (DBG) {
                    if (active) {
                        const int ng = p.k / F::kGroup;
#pragma unroll
                        for (int u = 0; u < U; ++u) {
                            if (rl0 + u < rows) {
#pragma unroll
                                for (int r = 0; r < NG; ++r)
                                    if (F::kBlocksPerLane == 1 || r == 0 || active1)
                                        p.dbg[static_cast<long long>(r0 + rl0 + u) * ng + F::group_index(blk, t, r)] =
                                            isum[u][r];
                            }
                        }
                    }
                }
            }
            float v[V];
#pragma unroll
            for (int u = 0; u < U; ++u) {
#pragma unroll
                for (int m = 0; m < MR; ++m) v[u * MR + m] = active ? acc[u][m] : 0.0f;
            }
            const float tot = warp_sum_multi<V>(v, lane);
#pragma unroll
            for (int i = 0; i < V; ++i) {
                const int u = i / MR, m = i % MR;
                if (lane == warp_sum_lane<V>(i) && rl0 + u < rows)
                    part[((r0 - r_begin + rl0 + u) * MR + m) * p.S + slice] = tot;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(empty + slot));
    }
    // One barrier for the consumers: sum the slice partials of every row in
    // a fixed order and write y (rows a timed-out wait skipped are flagged
    // through the status word).
    named_bar_sync(1, static_cast<uint32_t>(nthreads));
    for (int i = tid; i < (r_end - r_begin) * MR; i += nthreads) {
        const int rl = i / MR, m = i % MR;
        const float* pp = part + (rl * MR + m) * p.S;
        float v = 0.0f;
        for (int j = 0; j < p.S; ++j) v += pp[j];
        float* yp = p.y + m * p.y_stride + r_begin + rl;
        *yp = p.beta != 0.0f ? fmaf(p.alpha, v, p.beta * *yp) : p.alpha * v;
    }
}

}  // namespace b200q
