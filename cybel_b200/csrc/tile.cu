// Tile kernel for 8-128 activation rows (speculative verify / prefill):
// Y[m][n] = X[m][k] W[n][k]^T on the 5th-generation tensor cores.
//
// The reference reaches M > 1 through simd_matmul_* (quantized_matmul.cpp:
// 1944-2154), a per-(row, activation) loop of the same fp32 dot products that
// re-streams W once per activation row. On B200 the batch turns the op into a
// small GEMM that streams W once:
//
//  * A = a 128-row tile of the weights, dequantized in shared memory to fp16:
//    each element is the reference's fp32 dequantized value
//    (quantized_matmul.cpp:1323-1375: (d*sc)*q - dmin*mn, each step rounded
//    to fp32) rounded once more to fp16. B = the activations rounded to fp16,
//    prepared once per call in the UMMA K-major layout. D = fp32 accumulators
//    in tensor memory (M = 128 lanes x NP columns).
//  * Warp 0 streams the packed Q4_K weights with 2-D TMA (one 128-row x
//    144-byte box = one 256-element block column per copy) and the fp16
//    activation chunks with 1-D bulk copies; one thread of warp 1 issues
//    tcgen05.mma (M=128, N=NP, K=16) and commits to mbarriers that free the
//    chunk slots; warps 2-9 dequantize 64-element chunks into the canonical
//    no-swizzle K-major layout, then read the accumulators back with
//    tcgen05.ld and write fp32 outputs.
//  * Split-K across CTAs when the tile count alone cannot fill the SMs;
//    partials are summed in a fixed order by a second kernel (deterministic).
//  * Every pipeline wait is bounded (status word on timeout); tensor memory
//    is allocated and freed by warp 1 on every path. No multicast.
#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace b200q {

namespace {

constexpr int kTileRows = 128;   // MMA M (weight rows per CTA)
constexpr int kChunkK = 64;      // K elements per pipeline chunk
constexpr int kBlockBytes = 144; // Q4_K super-block
constexpr int kNSW = 3;          // packed-weight slots (one 256-element block column each)
constexpr int kNSC = 4;          // fp16 chunk slots
constexpr int kDeqWarps = 8;
constexpr int kDeqThreads = kDeqWarps * 32;
constexpr int kThreads = (2 + kDeqWarps) * 32;
constexpr int kPackedBytes = kTileRows * kBlockBytes;  // 18432
constexpr int kW16Bytes = kTileRows * kChunkK * 2;     // 16384

__host__ __device__ constexpr int x16_chunk_bytes(int np) { return np * kChunkK * 2; }

struct TileParams {
    const uint8_t* x16;   // [k/64 chunks][canonical NP x 64 fp16]
    float* out;           // [splits][m][n] partials, or y itself (one split, y_stride == n)
    volatile int* status;
    int n, m;
    int nblocks;          // k / 256
    int splits;           // K splits (gridDim.y)
};

// ---- tcgen05 / TMA wrappers ------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t holder, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(holder), "r"(cols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
__device__ __forceinline__ void tc_mma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                           uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(accum)
        : "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major, no swizzle. The UMMA canonical
// layout is built from 8-row x 16-byte core matrices (128 contiguous bytes);
// SBO = byte distance between 8-row groups, LBO = byte distance between the
// two 8-element K groups that one K=16 instruction reads.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100
    return d;                              // base offset 0, layout SWIZZLE_NONE
}

// Instruction descriptor: kind::f16 with fp16 A and B, fp32 D, both K-major,
// M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_f16(int n) {
    return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(kTileRows >> 4) << 24);
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Byte E of a word of nibbles (each byte < 16) as a float: the byte is
// placed in the low mantissa bits of 2^23 and 2^23 is subtracted (exact).
template <int E>
__device__ __forceinline__ float nib_to_float(uint32_t m) {
    return __int_as_float(__byte_perm(m, 0x4B000000u, 0x7540u + E)) - 8388608.0f;
}

// ---- the kernel -------------------------------------------------------------
template <int NP>
__global__ void __launch_bounds__(kThreads, 1)
    tile_q4k_kernel(const __grid_constant__ CUtensorMap wmap, const TileParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    constexpr int XB = x16_chunk_bytes(NP);
    constexpr int kSlot = kW16Bytes + XB;
    constexpr uint32_t kTmemCols = NP < 32 ? 32 : NP;
    uint8_t* packed = smem;                        // [kNSW][18432]
    uint8_t* chunks = smem + kNSW * kPackedBytes;  // [kNSC][W16 | X16]
    uint64_t* bars = reinterpret_cast<uint64_t*>(chunks + kNSC * kSlot);
    uint64_t* wfull = bars;             // [kNSW] packed block column landed (TMA)
    uint64_t* wempty = bars + kNSW;     // [kNSW] all dequantizers done with it
    uint64_t* xfull = bars + 2 * kNSW;  // [kNSC] fp16 activation chunk landed
    uint64_t* cready = xfull + kNSC;    // [kNSC] fp16 weight chunk written
    uint64_t* cfree = cready + kNSC;    // [kNSC] MMAs reading the chunk done
    uint64_t* accfull = cfree + kNSC;   // accumulators final
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(accfull + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.x * kTileRows;
    const int split = blockIdx.y;
    const int b_begin = static_cast<int>(static_cast<long long>(split) * p.nblocks / p.splits);
    const int b_end = static_cast<int>(static_cast<long long>(split + 1) * p.nblocks / p.splits);
    const int nchunks = (b_end - b_begin) * 4;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kNSW; ++i) {
            mbar_init(smem_addr(wfull + i), 1);
            mbar_init(smem_addr(wempty + i), kDeqThreads);
        }
        for (int i = 0; i < kNSC; ++i) {
            mbar_init(smem_addr(xfull + i), 1);
            mbar_init(smem_addr(cready + i), kDeqThreads);
            mbar_init(smem_addr(cfree + i), 1);
        }
        mbar_init(smem_addr(accfull), 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_addr(tmem_holder), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_d = *tmem_holder;
    griddep_launch_dependents();

    bool ok = true;
    if (warp == 0) {
        // ---------------- producer ----------------
        if (lane == 0) {
            griddep_wait();  // the fp16 activations come from the preceding prep kernel
            for (int c = 0; c < nchunks; ++c) {
                const int bl = c >> 2;
                if ((c & 3) == 0) {
                    const int s = bl % kNSW;
                    if (!mbar_wait_bounded(smem_addr(wempty + s), ((bl / kNSW) & 1) ^ 1)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(smem_addr(wfull + s), kPackedBytes);
                    tma_load_2d(smem_addr(packed + s * kPackedBytes), &wmap, (b_begin + bl) * kBlockBytes, row0,
                                smem_addr(wfull + s));
                }
                const int cs = c % kNSC;
                if (!mbar_wait_bounded(smem_addr(cfree + cs), ((c / kNSC) & 1) ^ 1)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(smem_addr(xfull + cs), XB);
                bulk_load(smem_addr(chunks + cs * kSlot + kW16Bytes),
                          p.x16 + static_cast<long long>(b_begin * 4 + c) * XB, XB, smem_addr(xfull + cs));
            }
            if (!ok) *p.status = STATUS_TIMEOUT;
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16(NP);
            for (int c = 0; c < nchunks; ++c) {
                const int cs = c % kNSC;
                const uint32_t par = (c / kNSC) & 1;
                if (!mbar_wait_bounded(smem_addr(cready + cs), par) || !mbar_wait_bounded(smem_addr(xfull + cs), par)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t wa = smem_addr(chunks + cs * kSlot);
                const uint32_t xa = wa + kW16Bytes;
#pragma unroll
                for (int s = 0; s < kChunkK / 16; ++s) {
                    const uint64_t da = smem_desc(wa + s * 2 * (kTileRows * 16), kTileRows * 16, 128);
                    const uint64_t db = smem_desc(xa + s * 2 * (NP * 16), NP * 16, 128);
                    tc_mma_f16(tmem_d, da, db, idesc, (c > 0 || s > 0) ? 1u : 0u);
                }
                tc_commit(smem_addr(cfree + cs));
            }
            if (ok) tc_commit(smem_addr(accfull));
            else *p.status = STATUS_TIMEOUT;
        }
    } else {
        // ---------------- dequantizers (warps 2..9), then the epilogue ----------------
        const int dt = threadIdx.x - 64;
        const int t = dt & (kTileRows - 1);  // tile row
        const int h = dt >> 7;               // 0: sub-block 2q (low nibbles), 1: sub-block 2q+1 (high)
        for (int c = 0; c < nchunks; ++c) {
            const int bl = c >> 2, q = c & 3;
            const int s = bl % kNSW;
            if (q == 0 && !mbar_wait_bounded(smem_addr(wfull + s), (bl / kNSW) & 1)) {
                ok = false;
                break;
            }
            const int cs = c % kNSC;
            if (!mbar_wait_bounded(smem_addr(cfree + cs), ((c / kNSC) & 1) ^ 1)) {
                ok = false;
                break;
            }
            // Row t, elements [64q + 32h, 64q + 32h + 32) of the block = sub-block
            // j = 2q + h: the low (h = 0) or high (h = 1) nibbles of qs bytes
            // [32q, 32q + 32) (quantized_matmul.cpp:1323-1375 layout).
            const uint32_t blk = smem_addr(packed + s * kPackedBytes + t * kBlockBytes);
            const uint4 hd = lds128(blk);
            const uint4 qa = lds128(blk + 16u + 32u * q);
            const uint4 qb = lds128(blk + 32u + 32u * q);
            const float d = half_bits_to_float(hd.x & 0xFFFFu), dmin = half_bits_to_float(hd.x >> 16);
            // 6-bit scale/min of sub-block j = 2q + h (byte h of the pair).
            const uint32_t sh = 16u * (q & 1) + 8u * h;
            const uint32_t w0 = hd.y >> sh, w1 = hd.z >> sh, w2 = hd.w >> sh;
            uint32_t sc, mn;
            if (q < 2) {
                sc = w0 & 0x3Fu;
                mn = w1 & 0x3Fu;
            } else {
                sc = (w2 & 0x0Fu) | ((w0 >> 2) & 0x30u);
                mn = ((w2 >> 4) & 0x0Fu) | ((w1 >> 2) & 0x30u);
            }
            const float dsc = __fmul_rn(d, static_cast<float>(sc));
            const float dmn = __fmul_rn(dmin, static_cast<float>(mn));
            const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
            const uint32_t wbase = smem_addr(chunks + cs * kSlot) + (t >> 3) * 128 + (t & 7) * 16;
#pragma unroll
            for (int g = 0; g < 4; ++g) {  // K group j = 4h + g covers qs bytes 8g .. 8g+7
                const uint32_t lo = h ? (qw[2 * g] >> 4) & 0x0F0F0F0Fu : qw[2 * g] & 0x0F0F0F0Fu;
                const uint32_t hi = h ? (qw[2 * g + 1] >> 4) & 0x0F0F0F0Fu : qw[2 * g + 1] & 0x0F0F0F0Fu;
                float v[8];
                v[0] = nib_to_float<0>(lo);
                v[1] = nib_to_float<1>(lo);
                v[2] = nib_to_float<2>(lo);
                v[3] = nib_to_float<3>(lo);
                v[4] = nib_to_float<0>(hi);
                v[5] = nib_to_float<1>(hi);
                v[6] = nib_to_float<2>(hi);
                v[7] = nib_to_float<3>(hi);
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] = __fsub_rn(__fmul_rn(dsc, v[e]), dmn);
                const uint32_t a = wbase + (4 * h + g) * (kTileRows * 16);
                asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(pack_h2(v[0], v[1])),
                             "r"(pack_h2(v[2], v[3])), "r"(pack_h2(v[4], v[5])), "r"(pack_h2(v[6], v[7]))
                             : "memory");
            }
            fence_proxy_async_smem();
            mbar_arrive(smem_addr(cready + cs));
            if (q == 3) mbar_arrive(smem_addr(wempty + s));
        }
        if (!ok) *p.status = STATUS_TIMEOUT;
        // ---- epilogue: TMEM lane = tile row; warp w reads lanes 32*(w%4) ----
        const bool acc_ok = ok && nchunks > 0 && mbar_wait_bounded(smem_addr(accfull), 0);
        __syncwarp();
        tc_fence_after();
        const int lane_base = 32 * (warp & 3);
        const int row = row0 + lane_base + lane;
        float* dst = p.out + static_cast<long long>(split) * p.m * p.n;
        for (int c0 = 8 * h; c0 < NP; c0 += 16) {
            uint32_t v[8];
            const uint32_t taddr = tmem_d + (static_cast<uint32_t>(lane_base) << 16) + static_cast<uint32_t>(c0);
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                : "r"(taddr));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (row < p.n) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int mm = c0 + i;
                    if (mm < p.m) dst[static_cast<long long>(mm) * p.n + row] = acc_ok ? __uint_as_float(v[i]) : 0.0f;
                }
            }
        }
    }
    // Teardown: every warp is done with tensor memory before warp 1 frees it.
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_d, kTmemCols);
    }
}

// X (fp32, m rows of k, row stride x_stride) -> fp16 chunks in the UMMA
// K-major canonical layout. Chunk c holds K elements [64c, 64c + 64) of NP
// rows (rows >= m are zero): row r, K group j (8 elements), element e at byte
// j * NP*16 + (r / 8) * 128 + (r % 8) * 16 + 2e.
template <int NP>
__global__ void prep_x16_kernel(const float* __restrict__ x, long long x_stride, int m, int k,
                                uint8_t* __restrict__ x16) {
    griddep_launch_dependents();
    griddep_wait();
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;  // one (K group, row)
    const long long groups = static_cast<long long>(k / 8) * NP;
    if (i >= groups) return;
    const int r = static_cast<int>(i % NP);
    const long long g8 = i / NP;  // global K group
    const int c = static_cast<int>(g8 >> 3), j = static_cast<int>(g8 & 7);
    uint4 out = make_uint4(0u, 0u, 0u, 0u);
    if (r < m) {
        const float* src = x + static_cast<long long>(r) * x_stride + g8 * 8;
        const float4 a = __ldg(reinterpret_cast<const float4*>(src));
        const float4 b = __ldg(reinterpret_cast<const float4*>(src + 4));
        out = make_uint4(pack_h2(a.x, a.y), pack_h2(a.z, a.w), pack_h2(b.x, b.y), pack_h2(b.z, b.w));
    }
    *reinterpret_cast<uint4*>(x16 + static_cast<long long>(c) * x16_chunk_bytes(NP) + j * (NP * 16) + (r >> 3) * 128 +
                              (r & 7) * 16) = out;
}

// y[m][row] = sum over splits of part[split][m][row], in split order.
__global__ void reduce_splits_kernel(const float* __restrict__ part, float* __restrict__ y, int m, int n, int splits,
                                     long long y_stride) {
    griddep_launch_dependents();
    griddep_wait();
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const long long total = static_cast<long long>(m) * n;
    if (i >= total) return;
    float v = 0.0f;
    for (int s = 0; s < splits; ++s) v += part[static_cast<long long>(s) * total + i];
    y[(i / n) * y_stride + (i % n)] = v;
}

template <int NP>
constexpr int smem_bytes() {
    return kNSW * kPackedBytes + kNSC * (kW16Bytes + x16_chunk_bytes(NP)) + (2 * kNSW + 3 * kNSC + 1) * 8 + 16;
}

cudaLaunchConfig_t cfg_of(dim3 grid, dim3 block, int smem, cudaStream_t st, bool pdl, cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    if (pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cfg;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point, so the
// library does not link libcuda directly (it loads on machines without a
// driver, e.g. for symbol checks).
using EncodeTiledFn = decltype(&cuTensorMapEncodeTiled);

EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = []() -> EncodeTiledFn {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return nullptr;
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

// One-time (per device) opt-in to the kernel's dynamic shared memory.
template <int NP>
int configure_tile(int dev_id) {
    static std::mutex mu;
    static uint64_t done = 0;  // bit per device id < 64
    std::lock_guard<std::mutex> lk(mu);
    const uint64_t bit = dev_id < 64 ? (1ull << dev_id) : 0;
    if (bit && (done & bit)) return B200Q_OK;
    if (cudaFuncSetAttribute(tile_q4k_kernel<NP>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes<NP>()) !=
        cudaSuccess)
        return B200Q_ECUDA;
    done |= bit;
    return B200Q_OK;
}

int splits_for(int k, int n, int num_sms) {
    const int tiles = (n + kTileRows - 1) / kTileRows;
    return std::max(1, std::min(k / 256, num_sms / tiles));
}

template <int NP>
int launch_np(const void* w, const float* x, long long x_stride, float* y, int m, int k, int n, long long y_stride,
              Device* dev, cudaStream_t st, bool pdl) {
    const int nblocks = k / 256;
    const int tiles = (n + kTileRows - 1) / kTileRows;
    const int splits = splits_for(k, n, dev->num_sms);
    const bool direct = splits == 1 && y_stride == n;
    void* x16 = nullptr;
    void* part = nullptr;
    int rc = scratch_for(dev, st, kScratchTileX, static_cast<size_t>(k / kChunkK) * x16_chunk_bytes(NP), &x16);
    if (rc == B200Q_OK && !direct)
        rc = scratch_for(dev, st, kScratchTilePart, static_cast<size_t>(splits) * m * n * sizeof(float), &part);
    if (rc == B200Q_OK) rc = configure_tile<NP>(dev->id);
    if (rc != B200Q_OK) return rc;
    // Tensor map over the packed weights: [n rows][row bytes] of bytes; box =
    // 128 rows x 144 bytes (one block column); rows past n read as zeros.
    CUtensorMap map;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(nblocks) * kBlockBytes, static_cast<cuuint64_t>(n)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(nblocks) * kBlockBytes};
    const cuuint32_t box[2] = {kBlockBytes, kTileRows};
    const cuuint32_t estr[2] = {1, 1};
    const EncodeTiledFn encode = encode_tiled_fn();
    if (!encode ||
        encode(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(w), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return B200Q_ECUDA;
    cudaLaunchAttribute attr[1];
    {
        const long long groups = static_cast<long long>(k / 8) * NP;
        cudaLaunchConfig_t c = cfg_of(dim3(static_cast<unsigned>((groups + 255) / 256)), dim3(256), 0, st, pdl, attr);
        if (cudaLaunchKernelEx(&c, prep_x16_kernel<NP>, x, x_stride, m, k, static_cast<uint8_t*>(x16)) != cudaSuccess)
            return B200Q_ECUDA;
    }
    {
        TileParams tp{};
        tp.x16 = static_cast<const uint8_t*>(x16);
        tp.out = direct ? y : static_cast<float*>(part);
        tp.status = dev->status;
        tp.n = n;
        tp.m = m;
        tp.nblocks = nblocks;
        tp.splits = splits;
        cudaLaunchConfig_t c = cfg_of(dim3(tiles, splits), dim3(kThreads), smem_bytes<NP>(), st, pdl, attr);
        if (cudaLaunchKernelEx(&c, tile_q4k_kernel<NP>, map, tp) != cudaSuccess) return B200Q_ECUDA;
    }
    if (!direct) {
        const long long total = static_cast<long long>(m) * n;
        cudaLaunchConfig_t c = cfg_of(dim3(static_cast<unsigned>((total + 255) / 256)), dim3(256), 0, st, pdl, attr);
        if (cudaLaunchKernelEx(&c, reduce_splits_kernel, static_cast<const float*>(part), y, m, n, splits, y_stride) !=
            cudaSuccess)
            return B200Q_ECUDA;
    }
    return B200Q_OK;
}

}  // namespace

int tile_kernel_launches(int k, int n, long long y_stride, int num_sms) {
    return (splits_for(k, n, num_sms) == 1 && y_stride == n) ? 2 : 3;
}

int launch_tile(int qtype, const void* w, const float* x, long long x_stride, float* y, int m, int k, int n,
                long long y_stride, Device* dev, cudaStream_t st, bool pdl) {
    if (!w || !x || !y || m <= 0 || k <= 0 || n <= 0 || !dev) return B200Q_EINVAL;
    if (qtype != QT_Q4_K) return B200Q_EQTYPE;
    if (m > kTileMaxM || k % 256) return B200Q_ESHAPE;
    if ((reinterpret_cast<uintptr_t>(w) & 15u) || (reinterpret_cast<uintptr_t>(x) & 15u) || (x_stride & 3))
        return B200Q_EALIGN;
    if (m <= 16) return launch_np<16>(w, x, x_stride, y, m, k, n, y_stride, dev, st, pdl);
    if (m <= 32) return launch_np<32>(w, x, x_stride, y, m, k, n, y_stride, dev, st, pdl);
    if (m <= 64) return launch_np<64>(w, x, x_stride, y, m, k, n, y_stride, dev, st, pdl);
    return launch_np<128>(w, x, x_stride, y, m, k, n, y_stride, dev, st, pdl);
}

}  // namespace b200q
