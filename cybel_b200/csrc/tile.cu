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
//  * A = sc_j * q_i (<= 945, exact in fp16): dequant warps place nibble pairs
//    into fp16 with one AND-OR each and scale them with one packed FMA, then
//    store a block's 128 rows x 256 K into tensor memory (tcgen05.st); the
//    MMAs read A from there (kind::f16, M = 128 rows, N = NP columns,
//    K = 16). B = the activations in fp16 from shared memory (with the
//    precise variant, a second pass on the fp16 rounding residue of x).
//  * A2 = mn_j (fp16, exact) against B2 = sx_j (hi and lo fp16 parts) gives
//    D2[row][m] = sum_j mn_j sx_j with one more K = 16 MMA per block.
//  * Epilogue warps read D1 and D2 back (tcgen05.ld) per block and
//    accumulate d_b D1 - dmin_b D2 in fp32 registers; two tensor-memory
//    buffers let the MMAs of block b+1 run while block b is read.
//  * Roles have warps of their own: MMA issuers (4 at N = 16, 2 at N = 32,
//    each a share of the block's K-steps into its own accumulator), a packed
//    weight producer (2-D TMA, one 128-row x 144-byte box per block column),
//    an activation producer (chunk + B2 tile per block, 1-D bulk copies, up
//    to 6 blocks ahead), 8 dequant warps (two groups of four taking
//    alternate blocks) and 8 epilogue warps. Measured on
//    B200: an M = 128, K = 16 MMA occupies the tensor core ~45 cycles at
//    N <= 64 (~N/2 beyond), but a single issuing thread sharing its
//    scheduler with busy warps issues one only every ~150 cycles, hence
//    several issuers; lanes of one warp waiting on different barriers
//    advance in lockstep, hence one warp per producer.
//    Split-K across CTAs when the row tiles alone cannot fill the SMs;
//    partials are reduced in a fixed order.
//  * Every pipeline wait is bounded (status word on timeout); tensor memory
//    is allocated and freed by warp 0 on every path. No multicast.
#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace b200q {

namespace {

constexpr int kTileRows = 128;     // MMA M (weight rows per CTA)
constexpr int kChunkK = 256;       // K elements per pipeline chunk (one block)
constexpr int kBlockBytes = 144;   // Q4_K super-block
constexpr int kNSW = 3;            // packed-weight slots (one 256-element block column each)
constexpr int kEpiWarps = 8;
// Dequant warps: 8 in two groups of four; a group expands every other block,
// each warp all four quarters of its 32 rows, so one group's tensor-memory
// stores and barrier waits overlap the other's arithmetic (8% faster at
// 14336 x 4096, m = 8, than all eight warps on every block, two quarters
// each). Measured no faster: sixteen warps of one quarter each (the dequant
// work then takes more of the schedulers' issue slots from the MMA issuers),
// and handing each A slot to the MMAs in two halves (K-steps 0-7 once
// quarters 0-1 are stored).
__host__ __device__ constexpr int deq_warps(int) { return 8; }
// MMA issuers: the same thread-starvation argument again. Warps 0-3 each
// issue a share of every block's K-steps into their own accumulator (summed
// by the epilogue in a fixed order), so four schedulers feed the tensor core:
// 4 issuers at N = 16, 2 at N = 32, 1 beyond (longer MMAs; tensor-memory room).
// Warps: MMA issuers 0 .. NI-1, the weight producer NI, the activation
// producer NI+1, then the dequant and epilogue warps (any 4 consecutive warps
// cover the 4 tensor-memory lane quarters). Each waiting role has a warp of
// its own: lanes of one warp that wait on different barriers advance in
// lockstep, which had tied the activation loads to the dequant warps' pace.
__host__ __device__ constexpr int mma_issuers(int np) { return np == 16 ? 4 : (np == 32 ? 2 : 1); }
__host__ __device__ constexpr int first_deq_warp(int np) { return mma_issuers(np) + 2; }
__host__ __device__ constexpr int tile_threads(int np) { return (first_deq_warp(np) + deq_warps(np) + kEpiWarps) * 32; }
constexpr int kPackedBytes = kTileRows * kBlockBytes;  // 18432
constexpr int kA2Bytes = kTileRows * 16 * 2;           // 4096: mins tile, 128 x 16 fp16
constexpr int kSmemLimit = 227 * 1024;

// Activation bytes of one 256-element chunk: NP rows x 256 fp16, twice for
// the precise variant (hi K-groups 0..31, then lo K-groups 32..63).
__host__ __device__ constexpr int xchunk_bytes(int np, bool prec) { return np * kChunkK * 2 * (prec ? 2 : 1); }
// Bytes of one block's B2 tile (NP rows x 16 fp16: sx hi, then sx lo).
__host__ __device__ constexpr int b2_bytes(int np) { return np * 16 * 2; }

struct TileParams {
    const uint8_t* xc;    // [k/256][xchunk_bytes] activation chunks (UMMA K-major layout)
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

// Nibbles in place as fp16: OR-ing 0x6400 (1024.0) into a half whose low
// bits hold a nibble code q gives 1024 + q (bits 0-3) or 1024 + 16 q (bits
// 4-7), exactly. One AND-OR per pair of codes; then
//     fma(1024 + q, sc, -1024 sc) = fma(1024 + 16 q, sc / 16, -64 sc) = q sc,
// exactly representable (<= 945, sc / 16 has 6 significant bits), so the
// one rounding of each packed FMA is exact.
__device__ __forceinline__ uint32_t nib_times(uint32_t h, __half2 sc2, __half2 off2) {
    const __half2 r = __hfma2(*reinterpret_cast<const __half2*>(&h), sc2, off2);
    return *reinterpret_cast<const uint32_t*>(&r);
}

// MMA with A from tensor memory (lane = row of A, two fp16 per column) and
// B from shared memory.
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc,
                                              uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(db), "r"(idesc), "r"(accum)
        : "memory");
}

// 32 consecutive columns of this warp's 32 lanes (one register each).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
        "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
        "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}

__device__ __forceinline__ uint32_t tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
        : "r"(taddr));
    return 0;
}

// ---- the kernel -------------------------------------------------------------
// Tensor memory (512 columns): D buffers from column 0 (per buffer the
// issuers' D1 parts then D2, NP columns each; two buffers for NP <= 64, one
// for NP = 128), A block slots from column 256 (128 columns = 128 rows x 256
// fp16 each).
// Shared memory (bytes): packed slots | activation slots (chunk + B2 tile,
// 2..6 blocks deep) | per-block A2 (mins) tiles x4 | d/dmin per row x4 |
// barriers | tensor-memory address.
// A block slots in tensor memory: three where the accumulators leave room
// (N = 16 with at most two issuers: 96 columns of accumulators), else two.
// (Measured at N = 16: two issuers and three slots ran slower than four
// issuers and two slots, so the latter is used; so did four issuers with one
// accumulator buffer and three slots, 19.1 against 18.5 us at 14336 x 4096.)
__host__ __device__ constexpr int a_slots(int np) { return (np == 16 && mma_issuers(np) <= 2) ? 3 : 2; }
constexpr int kNM = 4;              // per-block mins tile / d, dmin buffers (the epilogue releases them)
constexpr uint32_t kTmemCols = 512;
// First tensor-memory column of the A slots.
__host__ __device__ constexpr uint32_t a_base(int np) { return a_slots(np) == 3 ? 128u : 256u; }
constexpr uint32_t kAColsPerChunk = kChunkK / 2;

template <int NP, bool PREC>
struct TileSmem {
    static constexpr int XB = xchunk_bytes(NP, PREC);
    static constexpr int kDBufs = NP <= 64 ? 2 : 1;
    static constexpr int kBufCols = (mma_issuers(NP) + 1) * NP;
    static constexpr int kPacked = 0;
    static constexpr int kXSlot = XB + b2_bytes(NP);  // activation chunk, then the block's B2 tile
    static constexpr int kFixed = kNSW * kPackedBytes + kNM * kA2Bytes + kNM * kTileRows * 8 + 1024;
    static constexpr int NSX = ((kSmemLimit - kFixed) / kXSlot) > 6 ? 6 : ((kSmemLimit - kFixed) / kXSlot);
    static constexpr int kX = kPacked + kNSW * kPackedBytes;  // multiple of 1024
    static constexpr int kA2 = kX + NSX * kXSlot;
    static constexpr int kDD = kA2 + kNM * kA2Bytes;
    static constexpr int kBars = kDD + kNM * kTileRows * 8;
    static constexpr int kNS = a_slots(NP);
    static constexpr uint32_t kABase = a_base(NP);
    static constexpr int kNumBars = 2 * kNSW + 2 * kNS + 2 * NSX + 2 * 2 + 2 * kNM;  // see the kernel
    static constexpr int kTmemHolder = kBars + kNumBars * 8;
    static constexpr int kTotal = kTmemHolder + 16;
    static_assert(NSX >= 2 && kTotal <= kSmemLimit, "tile kernel shared memory");
    static_assert(kDBufs * kBufCols <= static_cast<int>(a_base(NP)) &&
                  a_base(NP) + a_slots(NP) * kAColsPerChunk <= kTmemCols, "tensor memory columns");
};

// Roles: lane 0 of warps 0..NI-1 issues the MMAs; warp NI lane 0 streams
// packed block columns (2-D TMA), lane 1 the activation chunks and per-block
// B2 tiles (bulk copies); the next 8 warps dequantize into tensor memory; the
// last 8 warps run the epilogue.
//
// Slot s holds one block: A in tensor memory columns kABase + 128 s, the
// activation chunk (and B2 tile) in shared memory. Its "full" barrier
// completes when the dequant warps have arrived (their tensor-memory
// stores waited for and fenced) and the activation bytes have landed: the
// MMA issuers wait once and commit once per block (16 MMAs between them,
// 32 with PREC); issuer 0 adds the block's mins MMA (A2 and d/dmin written
// by the last dequant warp group).
template <int NP, bool PREC>
__global__ void __launch_bounds__(tile_threads(NP), 1)
    b200q_tile_q4k_kernel(const __grid_constant__ CUtensorMap wmap, const TileParams p) {
    using SM = TileSmem<NP, PREC>;
    extern __shared__ __align__(1024) uint8_t smem[];
    constexpr int XB = SM::XB;
    constexpr int DB = SM::kDBufs;
    constexpr int DW = deq_warps(NP);
    constexpr int NI = mma_issuers(NP);
    constexpr int BC = SM::kBufCols;
    constexpr int kProdWarp = NI;       // packed weights
    constexpr int kXWarp = NI + 1;      // activation chunks and B2 tiles
    constexpr int NSX = SM::NSX;
    constexpr int kFirstDeqWarp = first_deq_warp(NP);
    constexpr int kRanges = 2;  // qs quarters per dequant pass
    constexpr int kNS = SM::kNS;
    constexpr uint32_t kABase = SM::kABase;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::kBars);
    uint64_t* wfull = bars;                 // [kNSW] packed block column landed (TMA)
    uint64_t* wempty = wfull + kNSW;        // [kNSW] dequant warps done with it
    uint64_t* full = wempty + kNSW;         // [kNS] A block stored in tensor memory
    uint64_t* empty = full + kNS;           // [kNS] MMAs reading the A slot done
    uint64_t* xfull = empty + kNS;          // [NSX] activation chunk and B2 landed
    uint64_t* xfree = xfull + SM::NSX;      // [NSX] MMAs reading the activation slot done
    uint64_t* mready = xfree + SM::NSX;     // [kNM] A2 and d/dmin of the block written
    uint64_t* accfull = mready + kNM;       // [2] block MMAs done (D1, D2 final)
    uint64_t* accempty = accfull + 2;       // [2] epilogue done with the D buffer
    uint64_t* dfree = accempty + 2;         // [kNM] epilogue done with A2/d/dmin buffer bl % kNM
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + SM::kTmemHolder);
    float* dd = reinterpret_cast<float*>(smem + SM::kDD);  // [kNM][128][2] d, dmin

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.x * kTileRows;
    const int split = blockIdx.y;
    const int b_begin = static_cast<int>(static_cast<long long>(split) * p.nblocks / p.splits);
    const int b_end = static_cast<int>(static_cast<long long>(split + 1) * p.nblocks / p.splits);
    const int nblk = b_end - b_begin;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kNSW; ++i) {
            mbar_init(smem_addr(wfull + i), 1);
            mbar_init(smem_addr(wempty + i), 4);  // the four warps of the block's dequant group
        }
        for (int i = 0; i < kNS; ++i) {
            mbar_init(smem_addr(full + i), 4);
            mbar_init(smem_addr(empty + i), NI);
        }
        for (int i = 0; i < SM::NSX; ++i) {
            mbar_init(smem_addr(xfull + i), 1);
            mbar_init(smem_addr(xfree + i), NI);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(smem_addr(accfull + i), NI);
            mbar_init(smem_addr(accempty + i), kEpiWarps);
        }
        for (int i = 0; i < kNM; ++i) {
            mbar_init(smem_addr(mready + i), 4);
            mbar_init(smem_addr(dfree + i), kEpiWarps);
        }
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_addr(tmem_holder), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;
    griddep_launch_dependents();

    bool ok = true;
    if (warp == kProdWarp) {
        // ---------------- packed weight producer ----------------
        if (lane == 0) {
            for (int bl = 0; bl < nblk && ok; ++bl) {
                const int s = bl % kNSW;
                ok = mbar_wait_bounded(smem_addr(wempty + s), ((bl / kNSW) & 1) ^ 1);
                if (!ok) break;
                mbar_arrive_expect_tx(smem_addr(wfull + s), kPackedBytes);
                tma_load_2d(smem_addr(smem + SM::kPacked + s * kPackedBytes), &wmap, (b_begin + bl) * kBlockBytes, row0,
                            smem_addr(wfull + s));
            }
            if (!ok) *p.status = STATUS_TIMEOUT;
        }
    } else if (warp == kXWarp) {
        // ---------------- activation producer ----------------
        if (lane == 0) {
            griddep_wait();  // the activation chunks and B2 tiles come from the preceding prep kernel
            for (int bl = 0; bl < nblk && ok; ++bl) {
                const int xs = bl % NSX;
                ok = mbar_wait_bounded(smem_addr(xfree + xs), ((bl / NSX) & 1) ^ 1);
                if (!ok) break;
                const uint32_t fb = smem_addr(xfull + xs);
                const uint32_t dst = smem_addr(smem + SM::kX + xs * SM::kXSlot);
                mbar_arrive_expect_tx(fb, SM::kXSlot);
                bulk_load(dst, p.xc + static_cast<long long>(b_begin + bl) * XB, XB, fb);
                bulk_load(dst + XB, p.b2 + static_cast<long long>(b_begin + bl) * b2_bytes(NP), b2_bytes(NP), fb);
            }
            if (!ok) *p.status = STATUS_TIMEOUT;
        }
    } else if (warp < NI) {
        // ---------------- MMA issuers ----------------
        if (lane == 0) {
            constexpr int KS = (kChunkK / 16) / NI;  // K-steps per issuer
            const int k0 = warp * KS;
            constexpr uint32_t idesc = idesc_f16(NP);
            // Descriptors of slot 0 / buffer 0; others are fixed byte offsets
            // (>> 4 into the address field, which cannot carry: < 256 KB).
            const uint64_t dX0 = smem_desc(smem_addr(smem + SM::kX), NP * 16, 128);
            const uint64_t dA20 = smem_desc(smem_addr(smem + SM::kA2), kTileRows * 16, 128);
            const uint64_t dB20 = smem_desc(smem_addr(smem + SM::kX + XB), NP * 16, 128);
            for (int bl = 0; bl < nblk && ok; ++bl) {
                const int mb = bl % DB, hb = bl % kNM;
                const uint32_t d1 = tmem_base + static_cast<uint32_t>(mb * BC + warp * NP);
                const uint32_t d2 = tmem_base + static_cast<uint32_t>(mb * BC + NI * NP);
                ok = mbar_wait_bounded(smem_addr(accempty + mb), ((bl / DB) & 1) ^ 1);
                if (!ok) break;
                tc_fence_after();
                const int s = bl % kNS, xs = bl % NSX;
                ok = mbar_wait_bounded(smem_addr(full + s), (bl / kNS) & 1) &&
                     mbar_wait_bounded(smem_addr(xfull + xs), (bl / NSX) & 1);
                if (!ok) break;
                tc_fence_after();
                const uint32_t ta = tmem_base + kABase + static_cast<uint32_t>(s) * kAColsPerChunk;
                const uint64_t dx = dX0 + static_cast<uint64_t>((xs * SM::kXSlot) >> 4);
#pragma unroll
                for (int i = 0; i < KS; ++i) {
                    const int kk = k0 + i;
                    tc_mma_f16_ts(d1, ta + 8u * kk, dx + ((kk * 2 * NP * 16) >> 4), idesc, i > 0 ? 1u : 0u);
                    if constexpr (PREC)  // the rounding residue of x (K groups 32..63), same A
                        tc_mma_f16_ts(d1, ta + 8u * kk, dx + (((32 + kk * 2) * NP * 16) >> 4), idesc, 1u);
                }
                if (warp == 0)  // mins: D2 = A2 (mn) x B2 (sx hi | sx lo), one K = 16 step
                    tc_mma_f16(d2, dA20 + ((hb * kA2Bytes) >> 4), dB20 + ((xs * SM::kXSlot) >> 4), idesc, 0u);
                tc_commit(smem_addr(empty + s));
                tc_commit(smem_addr(xfree + xs));
                tc_commit(smem_addr(accfull + mb));
            }
            if (!ok) *p.status = STATUS_TIMEOUT;
        }
    } else if (warp < kFirstDeqWarp + DW) {
        // ---------------- dequantizers (warps NI+2 .. NI+DW+1) ----------------
        // Groups of four warps take alternate blocks (group g: blocks g,
        // g + DW/4, ...), so one group's tensor-memory stores and barrier
        // waits overlap the other's arithmetic. A warp reaches tensor-memory
        // lanes 32 (warp % 4) .. + 31, so thread (t, g) takes tile row t =
        // 32 (warp % 4) + lane of its group's blocks and all four quarters h
        // of it, qs bytes [32h, 32h+32), kRanges per pass: sub-block 2h (low
        // nibbles) into slot columns 32h .. 32h+15, sub-block 2h+1 (high
        // nibbles) into 32h+16 .. 32h+31 (two consecutive K elements per
        // column); then row t of the block's mins tile A2 and its d/dmin.
        constexpr int kGroups = DW / 4;
        constexpr int kPasses = 4 / kRanges;
        const int t = 32 * (warp & 3) + lane;
        const int grp = (warp - kFirstDeqWarp) >> 2;
        const uint32_t lane_addr = static_cast<uint32_t>(32 * (warp & 3)) << 16;
        for (int bl = grp; bl < nblk && ok; bl += kGroups) {
            const int s = bl % kNS, ws = bl % kNSW, hb = bl % kNM;
            ok = mbar_wait_bounded(smem_addr(empty + s), ((bl / kNS) & 1) ^ 1) &&
                 mbar_wait_bounded(smem_addr(wfull + ws), (bl / kNSW) & 1) &&
                 mbar_wait_bounded(smem_addr(dfree + hb), ((bl / kNM) & 1) ^ 1);
            ok = __all_sync(0xFFFFFFFFu, ok);  // warp-uniform: the tensor-memory store is warp-collective
            if (!ok) break;
            // Row t of block column bl (quantized_matmul.cpp:1323-1375 layout):
            // d, dmin (fp16), 12 scale bytes, 128 nibble bytes.
            const uint32_t blk = smem_addr(smem + SM::kPacked + ws * kPackedBytes + t * kBlockBytes);
            const uint4 hd = lds128(blk);
#pragma unroll
            for (int pass = 0; pass < kPasses; ++pass) {
                // A pass's quarters' bytes first, then their fp16 products, then
                // the tensor-memory stores, so the quarters' load and arithmetic
                // latencies overlap.
                uint32_t qw[kRanges][8];
#pragma unroll
                for (int u = 0; u < kRanges; ++u) {
                    const int h = pass + u * kPasses;
                    const uint4 qa = lds128(blk + 16u + 32u * h);
                    const uint4 qb = lds128(blk + 32u + 32u * h);
                    qw[u][0] = qa.x; qw[u][1] = qa.y; qw[u][2] = qa.z; qw[u][3] = qa.w;
                    qw[u][4] = qb.x; qw[u][5] = qb.y; qw[u][6] = qb.z; qw[u][7] = qb.w;
                }
                uint32_t r[kRanges][32];
#pragma unroll
                for (int u = 0; u < kRanges; ++u) {
                    const int h = pass + u * kPasses;
                    __half2 sc2[2], off2[2];
#pragma unroll
                    for (int half = 0; half < 2; ++half) {  // sub-block j = 2h + half
                        const int j = 2 * h + half;
                        const uint32_t sb_lo = (j < 4 ? hd.y : hd.w) >> (8 * (j & 3));
                        const uint32_t sc = j < 4 ? (sb_lo & 63u) : ((sb_lo & 15u) | ((hd.y >> (8 * (j & 3)) >> 2) & 0x30u));
                        // low nibbles: (1024 + q) sc - 1024 sc; high: (1024 + 16 q) sc/16 - 64 sc
                        sc2[half] = __float2half2_rn(half ? static_cast<float>(sc) * 0.0625f : static_cast<float>(sc));
                        off2[half] = __float2half2_rn(-static_cast<float>(sc) * (half ? 64.0f : 1024.0f));
                    }
#pragma unroll
                    for (int w8 = 0; w8 < 8; ++w8) {  // bytes 4 w8 .. 4 w8 + 3: elements e0..e3 of both sub-blocks
                        // Column pairs hold elements (e0, e2) and (e1, e3); the
                        // activation chunks use the same order.
                        const uint32_t w = qw[u][w8], w_8 = qw[u][w8] >> 8;
                        r[u][2 * w8] = nib_times((w & 0x000F000Fu) | 0x64006400u, sc2[0], off2[0]);
                        r[u][2 * w8 + 1] = nib_times((w_8 & 0x000F000Fu) | 0x64006400u, sc2[0], off2[0]);
                        r[u][16 + 2 * w8] = nib_times((w & 0x00F000F0u) | 0x64006400u, sc2[1], off2[1]);
                        r[u][16 + 2 * w8 + 1] = nib_times((w_8 & 0x00F000F0u) | 0x64006400u, sc2[1], off2[1]);
                    }
                }
#pragma unroll
                for (int u = 0; u < kRanges; ++u) {
                    const int h = pass + u * kPasses;
                    tmem_st32(tmem_base + lane_addr + kABase + static_cast<uint32_t>(s) * kAColsPerChunk + 32u * h, r[u]);
                }
            }
            {
                // The block's mins tile A2 (row t: mn_0..7, twice, as fp16)
                // and its d / dmin, into buffer bl % kNM (released by the
                // epilogue of block bl - kNM, waited for above).
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
                const uint32_t a2 = smem_addr(smem + SM::kA2 + hb * kA2Bytes) + (t >> 3) * 128 + (t & 7) * 16;
#pragma unroll
                for (int kg = 0; kg < 2; ++kg)
                    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a2 + kg * (kTileRows * 16)),
                                 "r"(mnw[0]), "r"(mnw[1]), "r"(mnw[2]), "r"(mnw[3])
                                 : "memory");
                dd[(hb * kTileRows + t) * 2] = half_bits_to_float(hd.x & 0xFFFFu);
                dd[(hb * kTileRows + t) * 2 + 1] = half_bits_to_float(hd.x >> 16);
                fence_proxy_async_smem();
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(smem_addr(full + s));
                mbar_arrive(smem_addr(wempty + ws));
                mbar_arrive(smem_addr(mready + hb));
            }
        }
        if (!ok) *p.status = STATUS_TIMEOUT;
    } else {
        // ---------------- epilogue (the last 8 warps) ----------------
        constexpr int NH = NP / 2;
        const int ew = warp - kFirstDeqWarp - DW;
        const int lane_base = 32 * (warp & 3);
        const int ch = ew >> 2;  // column half
        const int row = lane_base + lane;
        float acc[NH];
#pragma unroll
        for (int i = 0; i < NH; ++i) acc[i] = 0.0f;
        for (int bl = 0; bl < nblk && ok; ++bl) {
            const int mb = bl % DB, hb = bl % kNM;
            ok = mbar_wait_bounded(smem_addr(accfull + mb), (bl / DB) & 1) &&
                 mbar_wait_bounded(smem_addr(mready + hb), (bl / kNM) & 1);
            ok = __all_sync(0xFFFFFFFFu, ok);  // tcgen05.ld below is warp-collective
            if (!ok) break;
            tc_fence_after();
            const float d = dd[(hb * kTileRows + row) * 2];
            const float dmin = dd[(hb * kTileRows + row) * 2 + 1];
            const uint32_t tcol = tmem_base + (static_cast<uint32_t>(lane_base) << 16) +
                                  static_cast<uint32_t>(mb * BC + ch * NH);
#pragma unroll
            for (int cc = 0; cc < NH; cc += 8) {
                uint32_t v1[NI][8], v2[8];
#pragma unroll
                for (int a = 0; a < NI; ++a) tmem_ld8(tcol + a * NP + cc, v1[a]);
                tmem_ld8(tcol + NI * NP + cc, v2);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    float dsum = __uint_as_float(v1[0][i]);
#pragma unroll
                    for (int a = 1; a < NI; ++a) dsum += __uint_as_float(v1[a][i]);
                    acc[cc + i] = fmaf(d, dsum, fmaf(-dmin, __uint_as_float(v2[i]), acc[cc + i]));
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(smem_addr(accempty + mb));
                mbar_arrive(smem_addr(dfree + hb));
            }
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
    // Teardown: every warp is done with tensor memory before warp 0 frees it.
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

// Activation rows (fp32, m rows of k at stride x_stride) -> fp16 chunks in
// the UMMA K-major canonical layout, and the per-block sub-block sums (B2),
// in one pass. Chunk c holds K elements [256c, 256c+256) of NP rows (rows >=
// m are zero): row r, K group j (8 elements), element e at byte
// j * NP*16 + (r / 8) * 128 + (r % 8) * 16 + 2 pos(e), where pos swaps
// elements 1 and 2 of each group of 4 (the order in which the dequantizers
// pair nibbles). With PREC the rounding residues fp16(x - fp16(x)) follow as
// K groups 32..63. B2 of block c, row r: K group 0 = the 8 sub-block sums
// sx_j of the fp16 activations the MMAs see (plus the residues with PREC),
// rounded to fp16 (hi), K group 1 = their fp16 remainders (lo).
// Thread (c, r, j): four consecutive threads cover one 32-element sub-block
// of row r and add their partial sums with two shuffles.
template <int NP, bool PREC>
__global__ void b200q_prep_x_kernel(const float* __restrict__ x, long long x_stride, int m, int k,
                              uint8_t* __restrict__ xc, uint8_t* __restrict__ b2) {
    griddep_launch_dependents();
    griddep_wait();
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const long long groups = static_cast<long long>(k / 8) * NP;  // a multiple of 32 (k % 256 == 0)
    if (i >= groups) return;                                        // whole warps
    const int j = static_cast<int>(i & 31);                         // K group within the block
    const int r = static_cast<int>((i >> 5) % NP);
    const long long c = (i >> 5) / NP;                              // block / chunk
    uint32_t hw[4] = {0u, 0u, 0u, 0u}, lw[4] = {0u, 0u, 0u, 0u};
    float part = 0.0f;
    if (r < m) {
        const float* src = x + static_cast<long long>(r) * x_stride + c * 256 + j * 8;
        const float4 a = __ldg(reinterpret_cast<const float4*>(src));
        const float4 bq = __ldg(reinterpret_cast<const float4*>(src + 4));
        // K order within each group of 4 is (0, 2, 1, 3), as in the A columns.
        const float v[8] = {a.x, a.z, a.y, a.w, bq.x, bq.z, bq.y, bq.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const __half2 hh = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
            hw[e] = *reinterpret_cast<const uint32_t*>(&hh);
            const float2 hf = __half22float2(hh);
            part += hf.x + hf.y;
            if constexpr (PREC) {
                const __half2 ll = __floats2half2_rn(v[2 * e] - hf.x, v[2 * e + 1] - hf.y);
                lw[e] = *reinterpret_cast<const uint32_t*>(&ll);
                const float2 lf = __half22float2(ll);
                part += lf.x + lf.y;
            }
        }
    }
    part += __shfl_xor_sync(0xffffffffu, part, 1);
    part += __shfl_xor_sync(0xffffffffu, part, 2);
    uint8_t* dst = xc + c * xchunk_bytes(NP, PREC) + j * (NP * 16) + (r >> 3) * 128 + (r & 7) * 16;
    *reinterpret_cast<uint4*>(dst) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    if constexpr (PREC) *reinterpret_cast<uint4*>(dst + 32 * (NP * 16)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    if ((j & 3) == 0) {
        const __half hi = __float2half_rn(part);
        const __half lo = __float2half_rn(part - __half2float(hi));
        uint8_t* base = b2 + c * b2_bytes(NP) + (r >> 3) * 128 + (r & 7) * 16 + (j >> 2) * 2;
        *reinterpret_cast<__half*>(base) = hi;
        *reinterpret_cast<__half*>(base + NP * 16) = lo;
    }
}

// y[m][row] = sum over splits of part[split][m][row], in split order.
__global__ void b200q_reduce_splits_kernel(const float* __restrict__ part, float* __restrict__ y, int m, int n, int splits,
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
    if (cudaFuncSetAttribute(b200q_tile_q4k_kernel<NP, PREC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
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
        if (cudaLaunchKernelEx(&c, b200q_prep_x_kernel<NP, PREC>, x, x_stride, m, k, static_cast<uint8_t*>(xc),
                               static_cast<uint8_t*>(b2)) != cudaSuccess)
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
            cfg_of(dim3(tiles, splits), dim3(tile_threads(NP)), TileSmem<NP, PREC>::kTotal, st, pdl, attr);
        if (cudaLaunchKernelEx(&c, b200q_tile_q4k_kernel<NP, PREC>, map, tp) != cudaSuccess) return B200Q_ECUDA;
    }
    if (!direct) {
        const long long total = static_cast<long long>(m) * n;
        cudaLaunchConfig_t c = cfg_of(dim3(static_cast<unsigned>((total + 255) / 256)), dim3(256), 0, st, pdl, attr);
        if (cudaLaunchKernelEx(&c, b200q_reduce_splits_kernel, static_cast<const float*>(part), y, m, n, splits, y_stride) !=
            cudaSuccess)
            return B200Q_ECUDA;
    }
    return B200Q_OK;
}

}  // namespace

int tile_kernel_launches(int k, int n, long long y_stride, int num_sms) {
    return (splits_for(k, n, num_sms) == 1 && y_stride == n) ? 2 : 3;
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
