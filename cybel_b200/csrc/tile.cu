// Tile kernel for 8-128 activation rows (speculative verify / prefill):
// Y[m][n] = X[m][k] W[n][k]^T on the 5th-generation tensor cores.
//
// The reference reaches M > 1 through simd_matmul_* (quantized_matmul.cpp:
// 1944-2154), a per-(row, activation) loop of the same fp32 dot products that
// re-streams W once per activation row. On B200 the batch turns the op into a
// small GEMM that streams W once. For a Q4_K row, block b, sub-block j:
//
//     w_i = d_b * sc_j * q_i - dmin_b * mn_j        (quantized_matmul.cpp:1323-1375)
//     y   = sum_b ( d_b * sum_i (sc_j q_i) x_i  -  dmin_b * sum_j mn_j sx_j ),
//           sx_j = sum_{i in j} x_i
//
// so the tensor cores work on exact small integers:
//  * A = sc_j * q_i (<= 945, exact in fp16), dequantized in shared memory with
//    one packed half2 FMA per two nibbles; B = the activations in fp16 (with
//    the precise variant, a second pass on the fp16 rounding residue of x).
//    One 256-element block accumulates in tensor memory as D1[row][m]
//    (tcgen05.mma kind::f16, M = 128 rows, N = NP columns, K = 16).
//  * A2 = mn_j (fp16, exact) against B2 = sx_j (hi and lo fp16 parts) gives
//    D2[row][m] = sum_j mn_j sx_j with one more K = 16 MMA per block.
//  * Epilogue warps read D1 and D2 back (tcgen05.ld) per block and
//    accumulate d_b D1 - dmin_b D2 in fp32 registers; two tensor-memory
//    buffers let the MMAs of block b+1 run while block b is read.
//  * Three lanes of warp 0 stream, each with its own ring, the packed weights
//    (2-D TMA, one 128-row x 144-byte box per block column), the prepared
//    activation chunks and the per-block sub-block sums (1-D bulk copies);
//    one thread of warp 1 issues the MMAs; warps 2-9 dequantize;
//    warps 10-17 run the epilogue. Split-K across CTAs when the row tiles
//    alone cannot fill the SMs; partials are reduced in a fixed order.
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

constexpr int kTileRows = 128;     // MMA M (weight rows per CTA)
constexpr int kChunkK = 64;        // K elements per pipeline chunk
constexpr int kBlockBytes = 144;   // Q4_K super-block
constexpr int kNSW = 4;            // packed-weight slots (one 256-element block column each)
constexpr int kNSA = 4;            // dequantized A chunk slots
constexpr int kDeqWarps = 8;
constexpr int kEpiWarps = 8;
constexpr int kDeqThreads = kDeqWarps * 32;
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr int kThreads = (2 + kDeqWarps + kEpiWarps) * 32;
constexpr int kPackedBytes = kTileRows * kBlockBytes;  // 18432
constexpr int kABytes = kTileRows * kChunkK * 2;       // 16384
constexpr int kA2Bytes = kTileRows * 16 * 2;           // 4096: mins tile, 128 x 16 fp16

// Activation bytes of one 64-element chunk: NP rows x 64 fp16, twice for
// the precise variant (hi K-groups, then lo K-groups).
__host__ __device__ constexpr int xchunk_bytes(int np, bool prec) { return np * kChunkK * 2 * (prec ? 2 : 1); }
// Bytes of one block's B2 tile (NP rows x 16 fp16: sx hi, then sx lo).
__host__ __device__ constexpr int b2_bytes(int np) { return np * 16 * 2; }

struct TileParams {
    const uint8_t* xc;    // [k/64][xchunk_bytes] activation chunks (UMMA K-major layout)
    const uint8_t* b2;    // [k/256][b2_bytes] per-block sub-block sums
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

// Two nibble codes (bytes 2i, 2i+1 of a word of nibbles, each < 16) times a
// sub-block scale sc as an exact half2: the bytes become the halves
// 1024 + q (0x64 as their high byte), and fma(1024 + q, sc, -1024 sc) =
// q * sc is exactly representable (<= 945), so the one rounding is exact.
template <int PAIR>
__device__ __forceinline__ uint32_t nib_pair_times(uint32_t m, __half2 sc2, __half2 off2) {
    const uint32_t h = __byte_perm(m, 0x64646464u, PAIR == 0 ? 0x5140u : 0x5342u);
    const __half2 r = __hfma2(*reinterpret_cast<const __half2*>(&h), sc2, off2);
    return *reinterpret_cast<const uint32_t*>(&r);
}

__device__ __forceinline__ uint32_t tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
        : "r"(taddr));
    return 0;
}

// ---- the kernel -------------------------------------------------------------
// Shared-memory map (bytes): packed slots | A chunk slots | activation
// chunk ring (as deep as 64 KB allows, 4..16 chunks, so its loads run far
// ahead) | per-block A2 (mins) tiles x2 | B2 tiles x2 | d/dmin per row x2 |
// barriers | tensor-memory address.
template <int NP, bool PREC>
struct TileSmem {
    static constexpr int XB = xchunk_bytes(NP, PREC);
    static constexpr int NSX = (64 * 1024 / XB) < 4 ? 4 : ((64 * 1024 / XB) > 16 ? 16 : (64 * 1024 / XB));
    static constexpr int kPacked = 0;
    static constexpr int kA = kPacked + kNSW * kPackedBytes;
    static constexpr int kX = kA + kNSA * kABytes;
    static constexpr int kA2 = kX + NSX * XB;
    static constexpr int kB2 = kA2 + 2 * kA2Bytes;
    static constexpr int kDD = kB2 + 2 * b2_bytes(NP);
    static constexpr int kBars = kDD + 2 * kTileRows * 8;
    static constexpr int kNumBars = 2 * kNSW + 2 * kNSA + 2 * NSX + 4 * 2;
    static constexpr int kTmemHolder = kBars + kNumBars * 8;
    static constexpr int kTotal = kTmemHolder + 16;
};

template <int NP, bool PREC>
__global__ void __launch_bounds__(kThreads, 1)
    tile_q4k_kernel(const __grid_constant__ CUtensorMap wmap, const TileParams p) {
    using SM = TileSmem<NP, PREC>;
    extern __shared__ __align__(1024) uint8_t smem[];
    constexpr int XB = SM::XB;
    constexpr uint32_t kTmemCols = 4 * NP;  // 2 buffers x (D1, D2); NP >= 16 -> >= 64 columns
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::kBars);
    constexpr int NSX = SM::NSX;
    uint64_t* wfull = bars;                 // [kNSW] packed block column landed (TMA)
    uint64_t* wempty = wfull + kNSW;        // [kNSW] dequantizers done with it
    uint64_t* cready = wempty + kNSW;       // [kNSA] A chunk written
    uint64_t* cfree = cready + kNSA;        // [kNSA] MMAs reading the A chunk done
    uint64_t* xfull = cfree + kNSA;         // [NSX] activation chunk landed
    uint64_t* xfree = xfull + NSX;          // [NSX] MMAs reading the activation chunk done
    uint64_t* mfull = xfree + NSX;          // [2] B2 tile landed
    uint64_t* mready = mfull + 2;           // [2] A2 tile and d/dmin written
    uint64_t* accfull = mready + 2;         // [2] block MMAs done (D1, D2 final)
    uint64_t* accempty = accfull + 2;       // [2] epilogue done with the buffer
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + SM::kTmemHolder);
    float* dd = reinterpret_cast<float*>(smem + SM::kDD);  // [2][128][2] d, dmin

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.x * kTileRows;
    const int split = blockIdx.y;
    const int b_begin = static_cast<int>(static_cast<long long>(split) * p.nblocks / p.splits);
    const int b_end = static_cast<int>(static_cast<long long>(split + 1) * p.nblocks / p.splits);
    const int nblk = b_end - b_begin;
    const int nchunks = nblk * 4;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kNSW; ++i) {
            mbar_init(smem_addr(wfull + i), 1);
            mbar_init(smem_addr(wempty + i), kDeqThreads);
        }
        for (int i = 0; i < kNSA; ++i) {
            mbar_init(smem_addr(cready + i), kDeqThreads);
            mbar_init(smem_addr(cfree + i), 1);
        }
        for (int i = 0; i < NSX; ++i) {
            mbar_init(smem_addr(xfull + i), 1);
            mbar_init(smem_addr(xfree + i), 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(smem_addr(mfull + i), 1);
            mbar_init(smem_addr(mready + i), kTileRows);
            mbar_init(smem_addr(accfull + i), 1);
            mbar_init(smem_addr(accempty + i), kEpiThreads);
        }
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_addr(tmem_holder), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;
    griddep_launch_dependents();

    bool ok = true;
    if (warp == 0) {
        // ---------------- producers ----------------
        // lane 0: packed block columns; lane 1: activation chunks; lane 2: B2
        // tiles -- independent rings, so no one waits behind another.
        if (lane < 3) griddep_wait();  // the activation tiles come from the preceding prep kernels
        if (lane == 0) {
            for (int bl = 0; bl < nblk && ok; ++bl) {
                const int s = bl % kNSW;
                ok = mbar_wait_bounded(smem_addr(wempty + s), ((bl / kNSW) & 1) ^ 1);
                if (!ok) break;
                mbar_arrive_expect_tx(smem_addr(wfull + s), kPackedBytes);
                tma_load_2d(smem_addr(smem + SM::kPacked + s * kPackedBytes), &wmap, (b_begin + bl) * kBlockBytes, row0,
                            smem_addr(wfull + s));
            }
        } else if (lane == 1) {
            for (int c = 0; c < nchunks && ok; ++c) {
                const int xs = c % NSX;
                ok = mbar_wait_bounded(smem_addr(xfree + xs), ((c / NSX) & 1) ^ 1);
                if (!ok) break;
                mbar_arrive_expect_tx(smem_addr(xfull + xs), XB);
                bulk_load(smem_addr(smem + SM::kX + xs * XB), p.xc + static_cast<long long>(b_begin * 4 + c) * XB, XB,
                          smem_addr(xfull + xs));
            }
        } else if (lane == 2) {
            // B2 of block bl: its buffer is free once the epilogue of block
            // bl - 2 is done (which follows that block's MMAs).
            for (int bl = 0; bl < nblk && ok; ++bl) {
                const int mb = bl & 1;
                ok = mbar_wait_bounded(smem_addr(accempty + mb), ((bl >> 1) & 1) ^ 1);
                if (!ok) break;
                mbar_arrive_expect_tx(smem_addr(mfull + mb), b2_bytes(NP));
                bulk_load(smem_addr(smem + SM::kB2 + mb * b2_bytes(NP)),
                          p.b2 + static_cast<long long>(b_begin + bl) * b2_bytes(NP), b2_bytes(NP), smem_addr(mfull + mb));
            }
        }
        if (!ok) *p.status = STATUS_TIMEOUT;
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16(NP);
            for (int bl = 0; bl < nblk && ok; ++bl) {
                const int mb = bl & 1;
                const uint32_t d1 = tmem_base + static_cast<uint32_t>(mb * 2 * NP);
                const uint32_t d2 = d1 + NP;
                ok = mbar_wait_bounded(smem_addr(accempty + mb), ((bl >> 1) & 1) ^ 1);
                if (!ok) break;
                tc_fence_after();
                for (int q = 0; q < 4 && ok; ++q) {
                    const int c = bl * 4 + q;
                    const int cs = c % kNSA, xs = c % NSX;
                    ok = mbar_wait_bounded(smem_addr(cready + cs), (c / kNSA) & 1) &&
                         mbar_wait_bounded(smem_addr(xfull + xs), (c / NSX) & 1);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t wa = smem_addr(smem + SM::kA + cs * kABytes);
                    const uint32_t xa = smem_addr(smem + SM::kX + xs * XB);
#pragma unroll
                    for (int s = 0; s < kChunkK / 16; ++s) {
                        const uint64_t da = smem_desc(wa + s * 2 * (kTileRows * 16), kTileRows * 16, 128);
                        const uint64_t db = smem_desc(xa + s * 2 * (NP * 16), NP * 16, 128);
                        tc_mma_f16(d1, da, db, idesc, (q > 0 || s > 0) ? 1u : 0u);
                        if constexpr (PREC) {  // the rounding residue of x, same A
                            const uint64_t dl = smem_desc(xa + 8 * (NP * 16) + s * 2 * (NP * 16), NP * 16, 128);
                            tc_mma_f16(d1, da, dl, idesc, 1u);
                        }
                    }
                    tc_commit(smem_addr(cfree + cs));
                    tc_commit(smem_addr(xfree + xs));
                }
                if (!ok) break;
                // mins: D2 = A2 (mn) x B2 (sx hi | sx lo), one K = 16 step
                ok = mbar_wait_bounded(smem_addr(mready + mb), (bl >> 1) & 1) &&
                     mbar_wait_bounded(smem_addr(mfull + mb), (bl >> 1) & 1);
                if (!ok) break;
                tc_fence_after();
                const uint64_t da2 = smem_desc(smem_addr(smem + SM::kA2 + mb * kA2Bytes), kTileRows * 16, 128);
                const uint64_t db2 = smem_desc(smem_addr(smem + SM::kB2 + mb * b2_bytes(NP)), NP * 16, 128);
                tc_mma_f16(d2, da2, db2, idesc, 0u);
                tc_commit(smem_addr(accfull + mb));
            }
            if (!ok) *p.status = STATUS_TIMEOUT;
        }
    } else if (warp < 2 + kDeqWarps) {
        // ---------------- dequantizers (warps 2..9) ----------------
        const int dt = threadIdx.x - 64;
        const int t = dt & (kTileRows - 1);  // tile row
        const int h = dt >> 7;               // 0: sub-block 2q (low nibbles), 1: sub-block 2q+1 (high)
        for (int c = 0; c < nchunks && ok; ++c) {
            const int bl = c >> 2, q = c & 3;
            const int s = bl % kNSW;
            if (q == 0) {
                ok = mbar_wait_bounded(smem_addr(wfull + s), (bl / kNSW) & 1);
                if (!ok) break;
            }
            const int cs = c % kNSA;
            ok = mbar_wait_bounded(smem_addr(cfree + cs), ((c / kNSA) & 1) ^ 1);
            if (!ok) break;
            // Row t of block column bl (quantized_matmul.cpp:1323-1375 layout):
            // d, dmin (fp16), 12 scale bytes, 128 nibble bytes; this chunk is
            // sub-blocks 2q (low nibbles) and 2q+1 (high) of qs[32q, 32q+32).
            const uint32_t blk = smem_addr(smem + SM::kPacked + s * kPackedBytes + t * kBlockBytes);
            const uint4 hd = lds128(blk);
            const uint4 qa = lds128(blk + 16u + 32u * q);
            const uint4 qb = lds128(blk + 32u + 32u * q);
            const int j = 2 * q + h;  // sub-block
            const uint32_t sb_lo = (j < 4 ? hd.y : hd.w) >> (8 * (j & 3));
            const uint32_t sc = j < 4 ? (sb_lo & 63u) : ((sb_lo & 15u) | ((hd.y >> (8 * (j & 3)) >> 2) & 0x30u));
            const __half2 sc2 = __half2half2(__int2half_rn(static_cast<int>(sc)));
            const __half2 off2 = __half2half2(__int2half_rn(-1024 * static_cast<int>(sc)));
            const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
            const uint32_t wbase = smem_addr(smem + SM::kA + cs * kABytes) + (t >> 3) * 128 + (t & 7) * 16;
#pragma unroll
            for (int g = 0; g < 4; ++g) {  // K group 4h + g: qs bytes 8g .. 8g+7 of the pair
                const uint32_t lo = h ? (qw[2 * g] >> 4) & 0x0F0F0F0Fu : qw[2 * g] & 0x0F0F0F0Fu;
                const uint32_t hi = h ? (qw[2 * g + 1] >> 4) & 0x0F0F0F0Fu : qw[2 * g + 1] & 0x0F0F0F0Fu;
                const uint32_t a = wbase + (4 * h + g) * (kTileRows * 16);
                asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a),
                             "r"(nib_pair_times<0>(lo, sc2, off2)), "r"(nib_pair_times<1>(lo, sc2, off2)),
                             "r"(nib_pair_times<0>(hi, sc2, off2)), "r"(nib_pair_times<1>(hi, sc2, off2))
                             : "memory");
            }
            fence_proxy_async_smem();
            mbar_arrive(smem_addr(cready + cs));
            if (q == 3) {
                if (h == 0) {
                    // The block's mins tile A2 (row t: mn_0..7, twice, as fp16)
                    // and its d / dmin, into buffer bl & 1 once the epilogue of
                    // block bl - 2 has released it.
                    const int mb = bl & 1;
                    ok = mbar_wait_bounded(smem_addr(accempty + mb), ((bl >> 1) & 1) ^ 1);
                    if (!ok) break;
                    uint32_t mnw[4];
#pragma unroll
                    for (int jj = 0; jj < 8; jj += 2) {
                        uint32_t m2[2];
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int jx = jj + e;
                            const uint32_t shz = 8 * (jx & 3);
                            m2[e] = jx < 4 ? ((hd.z >> shz) & 63u)
                                           : (((hd.w >> shz) >> 4) & 15u) | (((hd.z >> shz) >> 2) & 0x30u);
                        }
                        const __half2 hm = __halves2half2(__int2half_rn(static_cast<int>(m2[0])),
                                                          __int2half_rn(static_cast<int>(m2[1])));
                        mnw[jj / 2] = *reinterpret_cast<const uint32_t*>(&hm);
                    }
                    const uint32_t a2 = smem_addr(smem + SM::kA2 + mb * kA2Bytes) + (t >> 3) * 128 + (t & 7) * 16;
#pragma unroll
                    for (int kg = 0; kg < 2; ++kg)
                        asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a2 + kg * (kTileRows * 16)),
                                     "r"(mnw[0]), "r"(mnw[1]), "r"(mnw[2]), "r"(mnw[3])
                                     : "memory");
                    dd[(mb * kTileRows + t) * 2] = half_bits_to_float(hd.x & 0xFFFFu);
                    dd[(mb * kTileRows + t) * 2 + 1] = half_bits_to_float(hd.x >> 16);
                    fence_proxy_async_smem();
                    mbar_arrive(smem_addr(mready + mb));
                }
                mbar_arrive(smem_addr(wempty + s));
            }
        }
        if (!ok) *p.status = STATUS_TIMEOUT;
    } else {
        // ---------------- epilogue (warps 10..17) ----------------
        constexpr int NH = NP / 2;
        const int ew = warp - 2 - kDeqWarps;
        const int lane_base = 32 * (warp & 3);
        const int ch = ew >> 2;  // column half
        const int row = lane_base + lane;
        float acc[NH];
#pragma unroll
        for (int i = 0; i < NH; ++i) acc[i] = 0.0f;
        for (int bl = 0; bl < nblk && ok; ++bl) {
            const int mb = bl & 1;
            ok = mbar_wait_bounded(smem_addr(accfull + mb), (bl >> 1) & 1) &&
                 mbar_wait_bounded(smem_addr(mready + mb), (bl >> 1) & 1);
            __syncwarp();
            if (!ok) break;
            tc_fence_after();
            const float d = dd[(mb * kTileRows + row) * 2];
            const float dmin = dd[(mb * kTileRows + row) * 2 + 1];
            const uint32_t tcol = tmem_base + (static_cast<uint32_t>(lane_base) << 16) +
                                  static_cast<uint32_t>(mb * 2 * NP + ch * NH);
#pragma unroll
            for (int cc = 0; cc < NH; cc += 8) {
                uint32_t v1[8], v2[8];
                tmem_ld8(tcol + cc, v1);
                tmem_ld8(tcol + NP + cc, v2);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    acc[cc + i] = fmaf(d, __uint_as_float(v1[i]), fmaf(-dmin, __uint_as_float(v2[i]), acc[cc + i]));
            }
            tc_fence_before();
            mbar_arrive(smem_addr(accempty + mb));
        }
        if (!ok) *p.status = STATUS_TIMEOUT;
        float* dst = p.out + static_cast<long long>(split) * p.m * p.n;
        if (row0 + row < p.n) {
#pragma unroll
            for (int i = 0; i < NH; ++i) {
                const int mm = ch * NH + i;
                if (mm < p.m) dst[static_cast<long long>(mm) * p.n + row0 + row] = ok ? acc[i] : 0.0f;
            }
        }
    }
    // Teardown: every warp is done with tensor memory before warp 1 frees it.
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

// Activation rows (fp32, m rows of k at stride x_stride) -> fp16 chunks in
// the UMMA K-major canonical layout: chunk c holds K elements [64c, 64c+64)
// of NP rows (rows >= m are zero): row r, K group j (8 elements), element e
// at byte j * NP*16 + (r / 8) * 128 + (r % 8) * 16 + 2e. With PREC the
// rounding residues fp16(x - fp16(x)) follow as K groups 8..15.
template <int NP, bool PREC>
__global__ void prep_x_kernel(const float* __restrict__ x, long long x_stride, int m, int k,
                              uint8_t* __restrict__ xc) {
    griddep_launch_dependents();
    griddep_wait();
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;  // one (K group, row)
    const long long groups = static_cast<long long>(k / 8) * NP;
    if (i >= groups) return;
    const int r = static_cast<int>(i % NP);
    const long long g8 = i / NP;  // global K group
    const int c = static_cast<int>(g8 >> 3), j = static_cast<int>(g8 & 7);
    uint32_t hw[4] = {0u, 0u, 0u, 0u}, lw[4] = {0u, 0u, 0u, 0u};
    if (r < m) {
        const float* src = x + static_cast<long long>(r) * x_stride + g8 * 8;
        const float4 a = __ldg(reinterpret_cast<const float4*>(src));
        const float4 b = __ldg(reinterpret_cast<const float4*>(src + 4));
        const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const __half2 hh = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
            hw[e] = *reinterpret_cast<const uint32_t*>(&hh);
            if constexpr (PREC) {
                const float2 hf = __half22float2(hh);
                lw[e] = pack_h2(v[2 * e] - hf.x, v[2 * e + 1] - hf.y);
            }
        }
    }
    uint8_t* dst = xc + static_cast<long long>(c) * xchunk_bytes(NP, PREC) + j * (NP * 16) + (r >> 3) * 128 + (r & 7) * 16;
    *reinterpret_cast<uint4*>(dst) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    if constexpr (PREC) *reinterpret_cast<uint4*>(dst + 8 * (NP * 16)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
}

// Per block and row: the 8 sub-block sums sx_j of the fp16 activations the
// MMAs see (fp16(x), plus the residues with PREC), summed in fp32 in element
// order, stored as fp16 hi and lo parts: K group 0 = hi, K group 1 = lo.
template <int NP, bool PREC>
__global__ void prep_b2_kernel(const float* __restrict__ x, long long x_stride, int m, int k,
                               uint8_t* __restrict__ b2) {
    griddep_launch_dependents();
    griddep_wait();
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;  // one (block, row, sub-block)
    const long long total = static_cast<long long>(k / 256) * NP * 8;
    if (i >= total) return;
    const int jsb = static_cast<int>(i & 7);
    const int r = static_cast<int>((i >> 3) % NP);
    const long long bl = (i >> 3) / NP;
    float sx = 0.0f;
    if (r < m) {
        const float* src = x + static_cast<long long>(r) * x_stride + bl * 256 + jsb * 32;
#pragma unroll 8
        for (int e = 0; e < 32; ++e) {
            const float v = __ldg(src + e);
            const float hv = __half2float(__float2half_rn(v));
            sx += PREC ? hv + __half2float(__float2half_rn(v - hv)) : hv;
        }
    }
    const __half hi = __float2half_rn(sx);
    const __half lo = __float2half_rn(sx - __half2float(hi));
    uint8_t* base = b2 + bl * b2_bytes(NP) + (r >> 3) * 128 + (r & 7) * 16 + jsb * 2;
    *reinterpret_cast<__half*>(base) = hi;
    *reinterpret_cast<__half*>(base + NP * 16) = lo;
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
template <int NP, bool PREC>
int configure_tile(int dev_id) {
    static std::mutex mu;
    static uint64_t done = 0;  // bit per device id < 64
    std::lock_guard<std::mutex> lk(mu);
    const uint64_t bit = dev_id < 64 ? (1ull << dev_id) : 0;
    if (bit && (done & bit)) return B200Q_OK;
    if (cudaFuncSetAttribute(tile_q4k_kernel<NP, PREC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             TileSmem<NP, PREC>::kTotal) != cudaSuccess)
        return B200Q_ECUDA;
    done |= bit;
    return B200Q_OK;
}

int splits_for(int k, int n, int num_sms) {
    const int tiles = (n + kTileRows - 1) / kTileRows;
    return std::max(1, std::min(k / 256, num_sms / tiles));
}

template <int NP, bool PREC>
int launch_np(const void* w, const float* x, long long x_stride, float* y, int m, int k, int n, long long y_stride,
              Device* dev, cudaStream_t st, bool pdl) {
    static_assert(TileSmem<NP, PREC>::kTotal <= 227 * 1024, "tile kernel shared memory");
    const int nblocks = k / 256;
    const int tiles = (n + kTileRows - 1) / kTileRows;
    const int splits = splits_for(k, n, dev->num_sms);
    const bool direct = splits == 1 && y_stride == n;
    void* xc = nullptr;
    void* b2 = nullptr;
    void* part = nullptr;
    int rc = scratch_for(dev, st, kScratchTileX, static_cast<size_t>(k / kChunkK) * xchunk_bytes(NP, PREC), &xc);
    if (rc == B200Q_OK)
        rc = scratch_for(dev, st, kScratchTileB2, static_cast<size_t>(nblocks) * b2_bytes(NP), &b2);
    if (rc == B200Q_OK && !direct)
        rc = scratch_for(dev, st, kScratchTilePart, static_cast<size_t>(splits) * m * n * sizeof(float), &part);
    if (rc == B200Q_OK) rc = configure_tile<NP, PREC>(dev->id);
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
        if (cudaLaunchKernelEx(&c, prep_x_kernel<NP, PREC>, x, x_stride, m, k, static_cast<uint8_t*>(xc)) !=
            cudaSuccess)
            return B200Q_ECUDA;
        const long long sums = static_cast<long long>(nblocks) * NP * 8;
        cudaLaunchConfig_t c2 = cfg_of(dim3(static_cast<unsigned>((sums + 255) / 256)), dim3(256), 0, st, pdl, attr);
        if (cudaLaunchKernelEx(&c2, prep_b2_kernel<NP, PREC>, x, x_stride, m, k, static_cast<uint8_t*>(b2)) !=
            cudaSuccess)
            return B200Q_ECUDA;
    }
    {
        TileParams tp{};
        tp.xc = static_cast<const uint8_t*>(xc);
        tp.b2 = static_cast<const uint8_t*>(b2);
        tp.out = direct ? y : static_cast<float*>(part);
        tp.status = dev->status;
        tp.n = n;
        tp.m = m;
        tp.nblocks = nblocks;
        tp.splits = splits;
        cudaLaunchConfig_t c =
            cfg_of(dim3(tiles, splits), dim3(kThreads), TileSmem<NP, PREC>::kTotal, st, pdl, attr);
        if (cudaLaunchKernelEx(&c, tile_q4k_kernel<NP, PREC>, map, tp) != cudaSuccess) return B200Q_ECUDA;
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
    return (splits_for(k, n, num_sms) == 1 && y_stride == n) ? 3 : 4;
}

int tile_max_rows(bool precise) { return precise ? 64 : kTileMaxM; }

int launch_tile(int qtype, const void* w, const float* x, long long x_stride, float* y, int m, int k, int n,
                long long y_stride, Device* dev, cudaStream_t st, bool pdl, bool precise) {
    if (!w || !x || !y || m <= 0 || k <= 0 || n <= 0 || !dev) return B200Q_EINVAL;
    if (qtype != QT_Q4_K) return B200Q_EQTYPE;
    if (m > tile_max_rows(precise) || k % 256) return B200Q_ESHAPE;
    if ((reinterpret_cast<uintptr_t>(w) & 15u) || (reinterpret_cast<uintptr_t>(x) & 15u) || (x_stride & 3))
        return B200Q_EALIGN;
    if (precise) {
        if (m <= 16) return launch_np<16, true>(w, x, x_stride, y, m, k, n, y_stride, dev, st, pdl);
        if (m <= 32) return launch_np<32, true>(w, x, x_stride, y, m, k, n, y_stride, dev, st, pdl);
        return launch_np<64, true>(w, x, x_stride, y, m, k, n, y_stride, dev, st, pdl);
    }
    if (m <= 16) return launch_np<16, false>(w, x, x_stride, y, m, k, n, y_stride, dev, st, pdl);
    if (m <= 32) return launch_np<32, false>(w, x, x_stride, y, m, k, n, y_stride, dev, st, pdl);
    if (m <= 64) return launch_np<64, false>(w, x, x_stride, y, m, k, n, y_stride, dev, st, pdl);
    return launch_np<128, false>(w, x, x_stride, y, m, k, n, y_stride, dev, st, pdl);
}

}  // namespace b200q
