// Decode GEMV for GGUF block formats on sm_100a.
//
// y[m][row] = sum_k dequant(W)[row][k] * x[m][k] for m < MR activation rows,
// the operation of simd_matvec_* / simd_matmul_* in
// JSBuild/src/verso/Anvil/core/native/quantized_matmul.cpp:1536-2154, on the
// same canonical (and R4 / LM) block layouts.
//
// Design (one persistent CTA per SM):
//  * A producer warp streams each CTA's contiguous slab of weight rows into a
//    ring of shared-memory stages with 1-D bulk copies (cp.async.bulk, no
//    multicast) that complete on mbarriers. Weights are touched once, with an
//    L2 evict-first policy.
//  * Consumer warps own a fixed k-slice of the row ("slice") and walk rows.
//    Each lane quantizes its own piece of x into registers at start-up
//    (per 32-element group: int8 "x8" or int16 split in two byte planes
//    "x16"), so activations never travel through memory again.
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

constexpr int kGemvMaxConsumerWarps = 16;
constexpr int kGemvMaxThreads = (kGemvMaxConsumerWarps + 1) * 32;

struct GemvParams {
    const uint8_t* W;      // packed weight rows (device, 16-byte aligned)
    const float* x;        // [MR][x_stride] fp32 activations (device, 16-byte aligned)
    float* y;              // [MR][y_stride] fp32 outputs
    int32_t* dbg;          // optional [n][k/G] integer group sums (MR == 1 only)
    volatile int* status;  // status word (host-mapped); kernels store STATUS_* values
    long long row_bytes;   // bytes per packed row
    long long x_stride;    // floats between activation rows
    long long y_stride;    // floats between output rows
    int k, n;
    int nb;                // blocks per row
    int S;                 // slices per row (consumer warps per row)
    int WR;                // row walkers per slice
    int R;                 // rows per stage
    int NS;                // ring stages
    int stage_stride;      // bytes between ring slots (multiple of 128)
    int n_quads;           // ceil(n / 4)
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
    static constexpr int kElems = 256, kBytes = 144, kLanesPerBlock = 4, kBlocksPerSlice = 8;
    static constexpr int kRun = 32, kRuns = 2, kGroup = 32;
    static constexpr bool kR4 = false;
    __device__ static int run_start(int blk, int t, int r) { return blk * 256 + t * 64 + r * 32; }
    __device__ static int group_index(int blk, int t, int r) { return blk * 8 + 2 * t + r; }
};
template <>
struct Fmt<QT_Q4_K_R4> : Fmt<QT_Q4_K> {
    static constexpr bool kR4 = true;
};

template <>
struct Fmt<QT_Q6_K> {
    static constexpr int kElems = 256, kBytes = 210, kLanesPerBlock = 8, kBlocksPerSlice = 4;
    static constexpr int kRun = 16, kRuns = 2, kGroup = 16;
    static constexpr bool kR4 = false;
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
    static constexpr int kElems = 32, kBytes = 34, kLanesPerBlock = 1, kBlocksPerSlice = 32;
    static constexpr int kRun = 32, kRuns = 1, kGroup = 32;
    static constexpr bool kR4 = false;
    __device__ static int run_start(int blk, int, int) { return blk * 32; }
    __device__ static int group_index(int blk, int, int) { return blk; }
};
template <>
struct Fmt<QT_Q4_0> : Fmt<QT_Q8_0> {
    static constexpr int kBytes = 18;
};

template <>
struct Fmt<QT_Q6_K_LM> {
    static constexpr int kElems = 256, kBytes = 276, kLanesPerBlock = 8, kBlocksPerSlice = 4;
    static constexpr int kRun = 32, kRuns = 1, kGroup = 16;
    static constexpr bool kR4 = false;
    __device__ static int run_start(int blk, int t, int) { return blk * 256 + t * 32; }
    __device__ static int group_index(int blk, int t, int r) { return blk * 16 + 2 * t + r; }
};

// ---------------------------------------------------------------------------
// Activation quantization of one lane's run (restated in the oracle as
// orc_quantize_act): per 32-element group, amax, iscale = QMAX/amax (IEEE),
// q = rint(x * iscale) (one rounded multiply, half-even), d = amax/QMAX.
// ---------------------------------------------------------------------------
template <int DIG, int RUN>
struct XRun {
    uint32_t hi[RUN / 4];  // packed signed bytes (x8: the code; x16: high byte)
    uint32_t lo[DIG == 2 ? RUN / 4 : 1];  // packed unsigned low bytes (x16 only)
    float d;               // group scale
    int sum;               // sum of the codes in this run
};

__device__ __forceinline__ int round_half_even_small(float v) {
    // v in (-2^22, 2^22): adding 1.5*2^23 rounds to an integer with RNE.
    const float t = __fadd_rn(v, 12582912.0f);
    return __float_as_int(t) - 0x4B400000;
}

template <int DIG, int RUN>
__device__ __forceinline__ void quantize_run(const float* xp, bool active, XRun<DIG, RUN>& out) {
    float v[RUN];
#pragma unroll
    for (int i = 0; i < RUN; i += 4) {
        float4 f = active ? __ldg(reinterpret_cast<const float4*>(xp + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
        v[i] = f.x;
        v[i + 1] = f.y;
        v[i + 2] = f.z;
        v[i + 3] = f.w;
    }
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < RUN; ++i) amax = fmaxf(amax, fabsf(v[i]));
    if (RUN == 16) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    constexpr float QMAX = DIG == 1 ? 127.0f : 32767.0f;
    const float iscale = amax > 0.0f ? __fdiv_rn(QMAX, amax) : 0.0f;
    out.d = amax > 0.0f ? __fdiv_rn(amax, QMAX) : 0.0f;
    int s = 0;
#pragma unroll
    for (int w = 0; w < RUN / 4; ++w) {
        uint32_t hw = 0, lw = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int q = round_half_even_small(__fmul_rn(v[4 * w + j], iscale));
            s += q;
            if (DIG == 1) {
                hw |= (static_cast<uint32_t>(q) & 0xFFu) << (8 * j);
            } else {
                hw |= (static_cast<uint32_t>(q >> 8) & 0xFFu) << (8 * j);
                lw |= (static_cast<uint32_t>(q) & 0xFFu) << (8 * j);
            }
        }
        out.hi[w] = hw;
        if (DIG == 2) out.lo[w] = lw;
    }
    out.sum = s;
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

// Q4_K (quantized_matmul.cpp:411-515). Lane t of a block holds sub-blocks
// 2t (low nibbles) and 2t+1 (high nibbles) of qs bytes [32t, 32t+32).
template <int DIG, int MR>
struct Q4KDot {
    using X = XRun<DIG, 32>;
    __device__ static void run(uint32_t ba, int t, const X (&x)[MR][2], const float (&xsd)[MR][2], float (&acc)[MR],
                               int (&isum)[2]) {
        const uint4 h = lds128(ba);
        const uint4 qa = lds128(ba + 16u + 32u * t);
        const uint4 qb = lds128(ba + 32u + 32u * t);
        const float d = half_bits_to_float(h.x);
        const float dmin = half_bits_to_float(h.x >> 16);
        const uint32_t sh = (t & 1) * 16;
        const uint32_t w0 = h.y >> sh, w1 = h.z >> sh, w2 = h.w >> sh;
        const bool upper = t >= 2;
        const uint32_t sc2 = upper ? ((w2 & 0x0F0Fu) | ((w0 >> 2) & 0x3030u)) : (w0 & 0x3F3Fu);
        const uint32_t mn2 = upper ? (((w2 >> 4) & 0x0F0Fu) | ((w1 >> 2) & 0x3030u)) : (w1 & 0x3F3Fu);
        const float dsc0 = d * static_cast<float>(sc2 & 0xFFu);
        const float dsc1 = d * static_cast<float>((sc2 >> 8) & 0xFFu);
        const float dmn0 = dmin * static_cast<float>(mn2 & 0xFFu);
        const float dmn1 = dmin * static_cast<float>((mn2 >> 8) & 0xFFu);
        const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        uint32_t lo[8], hi[8];
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            lo[w] = q[w] & 0x0F0F0F0Fu;
            hi[w] = (q[w] >> 4) & 0x0F0F0F0Fu;
        }
#pragma unroll
        for (int m = 0; m < MR; ++m) {
            int a_hi = 0, a_lo = 0, b_hi = 0, b_lo = 0;
#pragma unroll
            for (int w = 0; w < 8; ++w) {
                dot4<DIG, false>(lo[w], x[m][0].hi[w], DIG == 2 ? x[m][0].lo[w] : 0u, a_hi, a_lo);
                dot4<DIG, false>(hi[w], x[m][1].hi[w], DIG == 2 ? x[m][1].lo[w] : 0u, b_hi, b_lo);
            }
            const int ia = combine_digits<DIG>(a_hi, a_lo);
            const int ib = combine_digits<DIG>(b_hi, b_lo);
            if (m == 0) {
                isum[0] = ia;
                isum[1] = ib;
            }
            float a = acc[m];
            a = fmaf(dsc0, x[m][0].d * static_cast<float>(ia), a);
            a = fmaf(-dmn0, xsd[m][0], a);
            a = fmaf(dsc1, x[m][1].d * static_cast<float>(ib), a);
            a = fmaf(-dmn1, xsd[m][1], a);
            acc[m] = a;
        }
    }
};

// Q6_K (quantized_matmul.cpp:683-775). Lane t = 4h + 2c + i16 reads the 16
// ql bytes at 64h + 32c + 16*i16 (groups 4h+c low nibbles, 4h+c+2 high
// nibbles) and the 16 qh bytes at 128 + 32h + 16*i16.
template <int DIG, int MR>
struct Q6KDot {
    using X = XRun<DIG, 16>;
    __device__ static void run(uint32_t ba, int t, const X (&x)[MR][2], float (&acc)[MR], int (&isum)[2]) {
        const int h = t >> 2, c = (t >> 1) & 1, i16 = t & 1;
        uint32_t ql[4], qh[4];
        lds_words_unaligned<4>(ba + 64u * h + 32u * c + 16u * i16, ql);
        lds_words_unaligned<4>(ba + 128u + 32u * h + 16u * i16, qh);
        const int g0 = 4 * h + c, g1 = g0 + 2;
        const float d = half_bits_to_float(lds_u16(ba + 208u));
        const float s0 = d * static_cast<float>(lds_s8(ba + 192u + 2u * g0 + i16));
        const float s1 = d * static_cast<float>(lds_s8(ba + 192u + 2u * g1 + i16));
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
            float a = acc[m];
            a = fmaf(s0, x[m][0].d * static_cast<float>(ia), a);
            a = fmaf(s1, x[m][1].d * static_cast<float>(ib), a);
            acc[m] = a;
        }
    }
};

// Q8_0 (quantized_matmul.cpp:1041-1081): fp16 d then 32 int8 codes.
template <int DIG, int MR>
struct Q80Dot {
    using X = XRun<DIG, 32>;
    __device__ static void run(uint32_t ba, const X (&x)[MR][1], float (&acc)[MR], int (&isum)[2]) {
        uint32_t q[8];
        lds_words_unaligned<8>(ba + 2u, q);
        const float d = half_bits_to_float(lds_u16(ba));
#pragma unroll
        for (int m = 0; m < MR; ++m) {
            int a_hi = 0, a_lo = 0;
#pragma unroll
            for (int w = 0; w < 8; ++w) dot4<DIG, true>(q[w], x[m][0].hi[w], DIG == 2 ? x[m][0].lo[w] : 0u, a_hi, a_lo);
            const int ia = combine_digits<DIG>(a_hi, a_lo);
            if (m == 0) isum[0] = ia;
            acc[m] = fmaf(d, x[m][0].d * static_cast<float>(ia), acc[m]);
        }
    }
};

// Q4_0 (ggml type 2): fp16 d then 16 bytes; element i < 16 is the low
// nibble of byte i, element 16 + i the high nibble; value d * (q - 8).
template <int DIG, int MR>
struct Q40Dot {
    using X = XRun<DIG, 32>;
    __device__ static void run(uint32_t ba, const X (&x)[MR][1], float (&acc)[MR], int (&isum)[2]) {
        uint32_t q[4];
        lds_words_unaligned<4>(ba + 2u, q);
        const float d = half_bits_to_float(lds_u16(ba));
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            lo[w] = q[w] & 0x0F0F0F0Fu;
            hi[w] = (q[w] >> 4) & 0x0F0F0F0Fu;
        }
#pragma unroll
        for (int m = 0; m < MR; ++m) {
            int a_hi = 0, a_lo = 0;
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                dot4<DIG, false>(lo[w], x[m][0].hi[w], DIG == 2 ? x[m][0].lo[w] : 0u, a_hi, a_lo);
                dot4<DIG, false>(hi[w], x[m][0].hi[4 + w], DIG == 2 ? x[m][0].lo[4 + w] : 0u, a_hi, a_lo);
            }
            const int ia = combine_digits<DIG>(a_hi, a_lo) - 8 * x[m][0].sum;
            if (m == 0) isum[0] = ia;
            acc[m] = fmaf(d, x[m][0].d * static_cast<float>(ia), acc[m]);
        }
    }
};

// Q6_K_LM (quantized_matmul.cpp:302-365, 1083-1154): 256 int8 codes in
// element order, 16 int8 scales, fp32 d. Lane t holds elements [32t, 32t+32)
// (scale groups 2t and 2t+1).
template <int DIG, int MR>
struct Q6KLMDot {
    using X = XRun<DIG, 32>;
    __device__ static void run(uint32_t ba, int t, const X (&x)[MR][1], float (&acc)[MR], int (&isum)[2]) {
        uint32_t q[8];
#pragma unroll
        for (int w = 0; w < 8; ++w) q[w] = lds32(ba + 32u * t + 4u * w);
        const uint32_t scw = lds_u16(ba + 256u + 2u * t);
        float dd;
        {
            const uint32_t db = lds32(ba + 272u);
            dd = __uint_as_float(db);
        }
        const float s0 = dd * static_cast<float>(static_cast<int8_t>(scw & 0xFFu));
        const float s1 = dd * static_cast<float>(static_cast<int8_t>((scw >> 8) & 0xFFu));
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
            acc[m] = fmaf(s0, x[m][0].d * static_cast<float>(ia), acc[m]);
            acc[m] = fmaf(s1, x[m][0].d * static_cast<float>(ib), acc[m]);
        }
    }
};

// Byte offset of (row, blk) inside a stage whose first row is `r0`
// (a multiple of 4 for the R4 layouts).
template <int QT>
__device__ __forceinline__ uint32_t stage_offset(int row, int r0, int blk, long long row_bytes, int n) {
    using F = Fmt<QT>;
    if (F::kR4) {
        const int full4 = (n / 4) * 4;
        if (row < full4) {
            const int g0 = row & ~3;
            return static_cast<uint32_t>((g0 - r0) * row_bytes) + static_cast<uint32_t>((blk * 4 + (row & 3)) * F::kBytes);
        }
    }
    return static_cast<uint32_t>((row - r0) * row_bytes) + static_cast<uint32_t>(blk * F::kBytes);
}

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------
template <int QT, int DIG, int MR, bool DBG>
__global__ void __launch_bounds__(kGemvMaxThreads, 1) gemv_kernel(const GemvParams p) {
    using F = Fmt<QT>;
    constexpr int RUN = F::kRun;
    constexpr int RUNS = F::kRuns;
    using X = XRun<DIG, RUN>;

    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int n_cons_warps = p.S * p.WR;
    const int n_cons_threads = n_cons_warps * 32;

    uint8_t* ring = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + static_cast<size_t>(p.NS) * p.stage_stride);
    uint64_t* empty = full + p.NS;
    float* part = reinterpret_cast<float*>(empty + p.NS);  // [2][R][MR][S]
    volatile int* abort_flag = reinterpret_cast<volatile int*>(part + 2 * p.R * MR * p.S);

    const int q0 = static_cast<int>(static_cast<long long>(blockIdx.x) * p.n_quads / gridDim.x);
    const int q1 = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * p.n_quads / gridDim.x);
    const int r_begin = q0 * 4;
    const int r_end = min(q1 * 4, p.n);
    const int n_stages = r_end > r_begin ? (r_end - r_begin + p.R - 1) / p.R : 0;

    if (tid == 0) {
        for (int i = 0; i < p.NS; ++i) {
            mbar_init(smem_addr(full + i), 1);
            mbar_init(smem_addr(empty + i), static_cast<uint32_t>(n_cons_warps));
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == n_cons_warps) {
        // ---------------- producer ----------------
        if (lane == 0 && n_stages > 0) {
            const uint64_t pol = l2_policy_evict_first();
            int issued = 0;
            for (int s = 0; s < n_stages; ++s) {
                const int slot = s % p.NS;
                const uint32_t use = static_cast<uint32_t>(s / p.NS);
                if (*abort_flag) break;
                if (!mbar_wait_bounded(smem_addr(empty + slot), (use & 1u) ^ 1u)) {
                    *p.status = STATUS_TIMEOUT;
                    *abort_flag = 1;
                    break;
                }
                // Copy the 16-byte-aligned window around the stage's rows;
                // consumers add (r0 * row_bytes) & 15 to find the first row.
                const int r0 = r_begin + s * p.R;
                const int rows = min(p.R, r_end - r0);
                const long long b0 = (r0 * p.row_bytes) & ~15ll;
                const long long b1 = ((r0 + rows) * p.row_bytes + 15) & ~15ll;
                const uint32_t bytes = static_cast<uint32_t>(b1 - b0);
                const uint32_t fb = smem_addr(full + slot);
                mbar_arrive_expect_tx(fb, bytes);
                bulk_g2s(smem_addr(ring + static_cast<size_t>(slot) * p.stage_stride), p.W + b0, bytes, fb, pol);
                issued = s + 1;
            }
            // Do not let the CTA retire with copies in flight: wait (bounded)
            // for the last stages issued.
            for (int s = max(0, issued - p.NS); s < issued; ++s) {
                const int slot = s % p.NS;
                const uint32_t use = static_cast<uint32_t>(s / p.NS);
                (void)mbar_wait_bounded(smem_addr(full + slot), use & 1u);
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    const int slice = warp % p.S;
    const int walker = warp / p.S;
    const int t = lane % F::kLanesPerBlock;
    const int blk = slice * F::kBlocksPerSlice + lane / F::kLanesPerBlock;
    const bool active = blk < p.nb;

    // Activations may be written by the preceding kernel in the stream.
    griddep_wait();

    X x[MR][RUNS];
    float xsd[MR][RUNS];
#pragma unroll
    for (int m = 0; m < MR; ++m) {
#pragma unroll
        for (int r = 0; r < RUNS; ++r) {
            const int e = active ? F::run_start(blk, t, r) : 0;
            quantize_run<DIG, RUN>(p.x + m * p.x_stride + e, active, x[m][r]);
            xsd[m][r] = x[m][r].d * static_cast<float>(x[m][r].sum);
        }
    }

    const uint32_t ring_base = smem_addr(ring);
    for (int s = 0; s < n_stages; ++s) {
        const int slot = s % p.NS;
        const uint32_t use = static_cast<uint32_t>(s / p.NS);
        const int r0 = r_begin + s * p.R;
        const int rows = min(p.R, r_end - r0);
        const int buf = s & 1;
        bool ok = !*abort_flag;
        if (ok && !mbar_wait_bounded(smem_addr(full + slot), use & 1u)) {
            if (lane == 0) *p.status = STATUS_TIMEOUT;
            *abort_flag = 1;
            ok = false;
        }
        const uint32_t sbase = ring_base + static_cast<uint32_t>(slot) * static_cast<uint32_t>(p.stage_stride) +
                               static_cast<uint32_t>((r0 * p.row_bytes) & 15ll);
        for (int rl = walker; rl < rows; rl += p.WR) {
            const int row = r0 + rl;
            float acc[MR];
#pragma unroll
            for (int m = 0; m < MR; ++m) acc[m] = 0.0f;
            int isum[2] = {0, 0};
            if (ok && active) {
                const uint32_t ba = sbase + stage_offset<QT>(row, r0, blk, p.row_bytes, p.n);
                if constexpr (QT == QT_Q4_K || QT == QT_Q4_K_R4) {
                    Q4KDot<DIG, MR>::run(ba, t, x, xsd, acc, isum);
                } else if constexpr (QT == QT_Q6_K || QT == QT_Q6_K_R4) {
                    Q6KDot<DIG, MR>::run(ba, t, x, acc, isum);
                } else if constexpr (QT == QT_Q8_0) {
                    Q80Dot<DIG, MR>::run(ba, x, acc, isum);
                } else if constexpr (QT == QT_Q4_0) {
                    Q40Dot<DIG, MR>::run(ba, x, acc, isum);
                } else if constexpr (QT == QT_Q6_K_LM) {
                    Q6KLMDot<DIG, MR>::run(ba, t, x, acc, isum);
                }
                if constexpr (DBG) {
                    const int ng = p.k / F::kGroup;
#pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        const bool has = (QT == QT_Q8_0 || QT == QT_Q4_0) ? (r == 0) : true;
                        if (has) p.dbg[static_cast<long long>(row) * ng + F::group_index(blk, t, r)] = isum[r];
                    }
                }
            }
#pragma unroll
            for (int m = 0; m < MR; ++m) {
                float v = acc[m];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
                if (lane == 0) part[((buf * p.R + rl) * MR + m) * p.S + slice] = v;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(empty + slot));
        named_bar_sync(1, static_cast<uint32_t>(n_cons_threads));
        for (int i = tid; i < rows * MR; i += n_cons_threads) {
            const int rl = i / MR, m = i % MR;
            const float* pp = part + ((buf * p.R + rl) * MR + m) * p.S;
            float v = 0.0f;
            for (int j = 0; j < p.S; ++j) v += pp[j];
            p.y[m * p.y_stride + r0 + rl] = v;
        }
    }
    griddep_launch_dependents();
}

}  // namespace b200q
