// One-kernel all-gather over NVLink peer memory for the row-sharded decode.
//
// Each rank owns one device buffer, shared with the other ranks of the node
// through CUDA IPC (cudaIpcGetMemHandle / cudaIpcOpenMemHandle, plain peer
// mappings -- no multicast objects). A buffer holds, per gather "slot", a
// receive area [rows][world * n_local] floats and a row of world flags.
// b200q_allgather_peer, run by every rank on its own GPU:
//  * block p (p = 0 .. world-1) writes this rank's rows into rank
//    (rank + p) % world's receive area at column rank * n_local (plain
//    128-bit stores through the peer mapping; p = 0 is the local copy), makes
//    them visible system-wide, and release-stores its sequence number into
//    that rank's flag [slot][rank];
//  * block 0 then waits until every other rank's flag for this slot has
//    reached the sequence number (acquire loads, bounded by a %globaltimer
//    limit; on timeout it records STATUS_TIMEOUT and returns);
//  * optionally every block waits and then quantizes a share of the gathered
//    rows into the GEMV's activation codes, so the projection that consumes
//    the gathered vector needs no quantizer launch of its own.
// Sequence numbers live in a per-(slot, block) device counter each block
// increments itself, so a CUDA graph replays them correctly. A slot's
// receive area may be reused by the next gather on that slot once its
// consumers have run: a rank can only write into a peer for the next use of
// a slot after the peer has contributed to every gather in between.
#include "gemv.cuh"
#include "internal.h"

namespace b200q {

namespace {

constexpr int kPeerThreads = 512;
constexpr int kMaxWorld = 16;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

struct PeerArgs {
    uint8_t* bases[kMaxWorld];  // each rank's shared buffer, as mapped on this GPU
    long long data_offset;      // bytes: the slot's receive area in every buffer
    long long flags_offset;     // bytes: the slot's flag row in every buffer
    int rank, world, rows, n_local, slot;
    uint8_t* xq;                // optional: gathered rows quantized here (GEMV activation codes)
    unsigned long long wait_ns; // longest wait for the other ranks' flags (%globaltimer ns)
};

// Library-wide limit of the flag wait (b200q_set_peer_wait_ns).
unsigned long long g_peer_wait_ns = kWaitTimeoutNs;

template <int DIG>
__global__ void __launch_bounds__(kPeerThreads) b200q_allgather_peer_kernel(const float* __restrict__ local,
                                                                      uint32_t* __restrict__ counters,
                                                                      volatile int* status, const PeerArgs a) {
    griddep_launch_dependents();
    griddep_wait();
    __shared__ uint32_t seq_s;
    const int p = blockIdx.x;
    const int dest = (a.rank + p) % a.world;
    if (threadIdx.x == 0) {
        uint32_t* c = counters + a.slot * kMaxWorld + p;
        seq_s = *c + 1u;
        *c = seq_s;
    }
    __syncthreads();
    const uint32_t seq = seq_s;
    float* dst = reinterpret_cast<float*>(a.bases[dest] + a.data_offset);
    const int q = a.n_local / 4;  // float4 per row chunk
    const long long row_pitch = static_cast<long long>(a.world) * a.n_local;
    for (int i = threadIdx.x; i < a.rows * q; i += blockDim.x) {
        const int r = i / q, j = i - r * q;
        const float4 v = *reinterpret_cast<const float4*>(local + static_cast<long long>(r) * a.n_local + 4 * j);
        *reinterpret_cast<float4*>(dst + r * row_pitch + static_cast<long long>(a.rank) * a.n_local + 4 * j) = v;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        st_release_sys(reinterpret_cast<uint32_t*>(a.bases[dest] + a.flags_offset) + a.rank, seq);
    }
    if (DIG == 0 && p != 0) return;
    // Wait for every other rank's rows of this slot (block 0 only, unless
    // every block then quantizes a share of the gathered rows).
    if (threadIdx.x < a.world && threadIdx.x != a.rank) {
        const uint32_t* f = reinterpret_cast<const uint32_t*>(a.bases[a.rank] + a.flags_offset) + threadIdx.x;
        const uint64_t t0 = global_timer_ns();
        uint32_t polls = 0;
        while (static_cast<int32_t>(ld_acquire_sys(f) - seq) < 0) {
            if ((++polls & 1023u) == 0 && global_timer_ns() - t0 > a.wait_ns) {
                *status = STATUS_TIMEOUT;
                break;
            }
        }
    }
    __syncthreads();
    if constexpr (DIG > 0) {
        // Quantize the gathered [rows][k] into the GEMV's activation layout,
        // four elements per thread over all blocks (k % 128 == 0, so a warp's
        // quads are all in range or all out).
        const int k = a.world * a.n_local;
        const int quads = k / 4;
        const float* full = reinterpret_cast<const float*>(a.bases[a.rank] + a.data_offset);
        const int total = a.rows * quads;
        for (int i = p * blockDim.x + threadIdx.x; i - static_cast<int>(threadIdx.x & 31) < total;
             i += gridDim.x * blockDim.x) {
            const bool valid = i < total;
            const int r = valid ? i / quads : 0, q4 = valid ? i - r * quads : 0;
            float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (valid) v = *reinterpret_cast<const float4*>(full + static_cast<long long>(r) * k + 4 * q4);
            quantize_quad<DIG>(v, valid, a.xq + static_cast<long long>(r) * xq_row_bytes(k, DIG), k, q4);
        }
    }
}

}  // namespace

int launch_allgather_peer(const float* local, int rows, int n_local, void* const* bases, long long data_offset,
                          long long flags_offset, int rank, int world, uint32_t* counters, int slot, Device* dev,
                          cudaStream_t st, void* xq, int act_mode) {
    if (!local || !bases || !counters || !dev || rows <= 0 || n_local <= 0 || slot < 0) return B200Q_EINVAL;
    if (xq && act_mode != B200Q_ACT_X8 && act_mode != B200Q_ACT_X16) return B200Q_EINVAL;
    if (xq && ((world * n_local) % 128 || (reinterpret_cast<uintptr_t>(xq) & 15u))) return B200Q_ESHAPE;
    if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world) return B200Q_EINVAL;
    if (n_local % 4 || (reinterpret_cast<uintptr_t>(local) & 15u) || (data_offset & 15) || (flags_offset & 3))
        return B200Q_EALIGN;
    PeerArgs a{};
    for (int i = 0; i < world; ++i) {
        if (!bases[i]) return B200Q_EINVAL;
        a.bases[i] = static_cast<uint8_t*>(bases[i]);
    }
    a.data_offset = data_offset;
    a.flags_offset = flags_offset;
    a.rank = rank;
    a.world = world;
    a.rows = rows;
    a.n_local = n_local;
    a.slot = slot;
    a.xq = static_cast<uint8_t*>(xq);
    a.wait_ns = g_peer_wait_ns;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(world);
    cfg.blockDim = dim3(kPeerThreads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (pdl_enabled()) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    cudaError_t e;
    if (!xq) e = cudaLaunchKernelEx(&cfg, b200q_allgather_peer_kernel<0>, local, counters, dev->status, a);
    else if (act_mode == B200Q_ACT_X8) e = cudaLaunchKernelEx(&cfg, b200q_allgather_peer_kernel<1>, local, counters, dev->status, a);
    else e = cudaLaunchKernelEx(&cfg, b200q_allgather_peer_kernel<2>, local, counters, dev->status, a);
    return e == cudaSuccess ? B200Q_OK : B200Q_ECUDA;
}

int peer_counter_slots() { return kMaxWorld; }

long long set_peer_wait_ns(long long ns) {
    const long long prev = static_cast<long long>(g_peer_wait_ns);
    if (ns > 0) g_peer_wait_ns = static_cast<unsigned long long>(ns);
    return prev;
}

}  // namespace b200q
