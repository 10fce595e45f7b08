// Shared device helpers for the sm_100a GGUF kernels: qtype ids, status
// codes, mbarrier / bulk-copy PTX wrappers with bounded waits, and dp4a forms.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace b200q {

// GGUF / engine qtype ids (quantized_matmul.cpp:39-44; Q4_0 is ggml type 2).
constexpr int QT_Q4_0 = 2;
constexpr int QT_Q8_0 = 8;
constexpr int QT_Q4_K = 12;
constexpr int QT_Q6_K = 14;
constexpr int QT_Q4_K_R4 = 112;
constexpr int QT_Q6_K_R4 = 114;
constexpr int QT_Q6_K_LM = 214;

// Device status word bits (set by kernels, read by the host).
constexpr int STATUS_TIMEOUT = 1;   // a bounded wait gave up
constexpr int STATUS_BAD_PAGE = 2;  // a page table named no page (or one past the pool) for a needed row

// Longest a kernel waits on one pipeline barrier before it records
// STATUS_TIMEOUT and stops consuming (ns of %globaltimer).
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;
// Hard cap on try_wait polls, independent of the timer.
constexpr uint32_t kWaitMaxPolls = 1u << 28;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// try_wait with a suspend-time hint: a waiting thread is parked until the
// phase completes (or ~kSuspendHintNs elapse) instead of spinning.
constexpr uint32_t kSuspendHintNs = 20000;

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(kSuspendHintNs)
        : "memory");
    return ok != 0;
}

// Non-blocking test of a phase (never suspends the thread).
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait by polling test_wait (the thread is never suspended, so it resumes
// as soon as the phase completes); false on timeout. For waits that are
// usually short and on the critical path.
__device__ __forceinline__ bool mbar_wait_spin_bounded(uint32_t bar, uint32_t parity) {
    if (mbar_test_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 1; it < kWaitMaxPolls; ++it) {
        if (mbar_test_wait(bar, parity)) return true;
        if ((it & 63u) == 0u && global_timer_ns() - t0 > kWaitTimeoutNs) return false;
    }
    return false;
}

// Wait for the phase with the given parity to complete; false on timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 1; it < kWaitMaxPolls; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 7u) == 0u && global_timer_ns() - t0 > kWaitTimeoutNs) return false;
    }
    return false;
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// 1-D bulk copy global -> this CTA's shared memory, completing on an
// mbarrier. No multicast. dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(policy)
        : "memory");
}

// Order this thread's generic-proxy shared-memory accesses before later
// async-proxy (bulk copy) writes to the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Store / poll a shared-memory word as a compiler barrier too: loads
// written before the store are issued before it.
__device__ __forceinline__ void sts_volatile(uint32_t a, uint32_t v) {
    asm volatile("st.volatile.shared.u32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t lds_volatile(uint32_t a) {
    uint32_t v;
    asm volatile("ld.volatile.shared.u32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
    return v;
}

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t a) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ int lds_s8(uint32_t a) {
    short v;
    asm volatile("ld.shared.s8 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}

// NW consecutive 32-bit words starting at a byte address that is only
// 2-byte aligned: aligned loads plus funnel shifts.
template <int NW>
__device__ __forceinline__ void lds_words_unaligned(uint32_t a, uint32_t* out) {
    const uint32_t base = a & ~3u;
    const uint32_t sh = (a & 3u) * 8u;
    uint32_t w[NW + 1];
#pragma unroll
    for (int i = 0; i <= NW; ++i) w[i] = lds32(base + 4u * i);
#pragma unroll
    for (int i = 0; i < NW; ++i) out[i] = __funnelshift_r(w[i], w[i + 1], sh);
}

// dp4a in the four signedness combinations (PTX dp4a.atype.btype).
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_su(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ float half_bits_to_float(uint32_t h16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h16 & 0xFFFFu)));
}

}  // namespace b200q
