// Decode-step glue around the quantized linears: residual add + RMSNorm,
// RoPE with the KV-cache append, and GQA attention of one query token over
// the cache. These are the non-matvec stages of the reference's single-token
// decode graph (JSBuild/src/verso/Anvil/core/native/model_graph.cpp:
// rmsnorm_inplace 674-693, apply_rope_with_dim 1222-1323, the fused GQA
// attention that follows), restated for one B200 so that a whole layer stack
// runs on the device and can be captured in one CUDA graph.
//
//  * b200q_add_rmsnorm_kernel: one CTA per row; residual += delta, out = residual *
//    (1 / sqrt(mean(residual^2) + eps)) * gamma (the reference's formula).
//  * b200q_rope_kv_kernel: interleaved pairs (2p, 2p+1) rotated by pos *
//    theta^(-2p / head_dim), as the reference; the rotated k and v are
//    written to fp16 caches [sequence][kv_head][max_ctx][head_dim].
//  * attention: split over the context (flash-decoding): one CTA per
//    (kv head, 128-position chunk) scores the G = n_heads / n_kv_heads query
//    heads of the group against the chunk, keeps the chunk's max and
//    exp-sum, and accumulates exp-weighted V; a second kernel merges the
//    chunks with the usual max rescaling.
// All kernels take part in programmatic dependent launch (trigger first,
// wait for the preceding kernel before reading its outputs).
#include <cuda_fp16.h>

#include <algorithm>

#include <type_traits>

#include "gemv.cuh"
#include "internal.h"

namespace b200q {

namespace {

constexpr int kNormThreads = 1024;
constexpr int kAttnChunk = 64;   // cache positions per attention CTA
constexpr int kAttnWarps = 8;    // warps per attention CTA
constexpr int kHeadDim = 128;    // head_dim the attention kernels are built for
constexpr int kMaxGroup = 8;     // query heads per kv head

// One CTA per row of `rows` rows of n elements. DIG > 0: the normed row is
// also quantized (x8 / x16 codes, the GEMV's activation layout) into xq, so
// the projections that follow read codes directly (out may then be null).
template <int DIG>
__global__ void __launch_bounds__(kNormThreads) b200q_add_rmsnorm_kernel(float* __restrict__ res,
                                                                   const float* __restrict__ delta,
                                                                   const float* __restrict__ gamma,
                                                                   float* __restrict__ out, uint8_t* __restrict__ xq,
                                                                   int n, float eps) {
    griddep_launch_dependents();
    griddep_wait();
    res += static_cast<long long>(blockIdx.x) * n;
    if (out) out += static_cast<long long>(blockIdx.x) * n;
    if (delta) delta += static_cast<long long>(blockIdx.x) * n;
    if (DIG) xq += static_cast<long long>(blockIdx.x) * xq_row_bytes(n, DIG);
    __shared__ float red[kNormThreads / 32];
    float ss = 0.0f;
    for (int i = 4 * threadIdx.x; i < n; i += 4 * kNormThreads) {
        float4 r = *reinterpret_cast<const float4*>(res + i);
        if (delta) {
            const float4 d = *reinterpret_cast<const float4*>(delta + i);
            r.x += d.x;
            r.y += d.y;
            r.z += d.z;
            r.w += d.w;
            *reinterpret_cast<float4*>(res + i) = r;
        }
        ss = fmaf(r.x, r.x, ss);
        ss = fmaf(r.y, r.y, ss);
        ss = fmaf(r.z, r.z, ss);
        ss = fmaf(r.w, r.w, ss);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < kNormThreads / 32 ? red[threadIdx.x] : 0.0f;
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float inv_rms = 1.0f / sqrtf(red[0] / static_cast<float>(n) + eps);
    // n % 128 == 0 when quantizing: a warp's 128 elements are all in range or
    // all out of range in every pass, as quantize_quad needs.
    const int passes = (n + 4 * kNormThreads - 1) / (4 * kNormThreads);
    for (int pass = 0; pass < passes; ++pass) {
        const int i = 4 * threadIdx.x + pass * 4 * kNormThreads;
        const bool valid = i < n;
        float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (valid) {
            const float4 r = *reinterpret_cast<const float4*>(res + i);
            const float4 g = *reinterpret_cast<const float4*>(gamma + i);
            o = make_float4(r.x * inv_rms * g.x, r.y * inv_rms * g.y, r.z * inv_rms * g.z, r.w * inv_rms * g.w);
            if (out) *reinterpret_cast<float4*>(out + i) = o;
        }
        if constexpr (DIG > 0) {
            if (i - 4 * (threadIdx.x & 31) < n) quantize_quad<DIG>(o, valid, xq, n, i >> 2);  // warp-uniform
        }
    }
}

// The same for n <= 4 * 4 * kNormThreads with the row held in registers:
// residual, delta and gamma are loaded together once (one round trip
// instead of a second pass over the residual after the reduction).
constexpr int kNormRegVec = 4;  // float4 per thread
template <int DIG>
__global__ void __launch_bounds__(kNormThreads) b200q_add_rmsnorm_reg_kernel(float* __restrict__ res,
                                                                       const float* __restrict__ delta,
                                                                       const float* __restrict__ gamma,
                                                                       float* __restrict__ out,
                                                                       uint8_t* __restrict__ xq, int n, float eps) {
    griddep_launch_dependents();
    griddep_wait();
    res += static_cast<long long>(blockIdx.x) * n;
    if (out) out += static_cast<long long>(blockIdx.x) * n;
    if (delta) delta += static_cast<long long>(blockIdx.x) * n;
    if (DIG) xq += static_cast<long long>(blockIdx.x) * xq_row_bytes(n, DIG);
    __shared__ float red[kNormThreads / 32];
    float4 r[kNormRegVec], g[kNormRegVec];
#pragma unroll
    for (int u = 0; u < kNormRegVec; ++u) {
        const int i = 4 * (threadIdx.x + u * kNormThreads);
        const bool valid = i < n;
        r[u] = valid ? *reinterpret_cast<const float4*>(res + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        g[u] = valid ? *reinterpret_cast<const float4*>(gamma + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (delta && valid) {
            const float4 d = *reinterpret_cast<const float4*>(delta + i);
            r[u].x += d.x;
            r[u].y += d.y;
            r[u].z += d.z;
            r[u].w += d.w;
        }
    }
    float ss = 0.0f;
#pragma unroll
    for (int u = 0; u < kNormRegVec; ++u) {
        const int i = 4 * (threadIdx.x + u * kNormThreads);
        if (delta && i < n) *reinterpret_cast<float4*>(res + i) = r[u];
        ss = fmaf(r[u].x, r[u].x, ss);
        ss = fmaf(r[u].y, r[u].y, ss);
        ss = fmaf(r[u].z, r[u].z, ss);
        ss = fmaf(r[u].w, r[u].w, ss);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < kNormThreads / 32 ? red[threadIdx.x] : 0.0f;
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float inv_rms = 1.0f / sqrtf(red[0] / static_cast<float>(n) + eps);
#pragma unroll
    for (int u = 0; u < kNormRegVec; ++u) {
        const int i = 4 * (threadIdx.x + u * kNormThreads);
        const bool valid = i < n;
        const float4 o = valid ? make_float4(r[u].x * inv_rms * g[u].x, r[u].y * inv_rms * g[u].y,
                                             r[u].z * inv_rms * g[u].z, r[u].w * inv_rms * g[u].w)
                               : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (out && valid) *reinterpret_cast<float4*>(out + i) = o;
        if constexpr (DIG > 0) {
            // n % 128 == 0: a warp's 128 elements are all in range or all out.
            if (i - 4 * (threadIdx.x & 31) < n) quantize_quad<DIG>(o, valid, xq, n, i >> 2);
        }
    }
}

// Threads [0, (n_heads + n_kv) * hd/2): one rotation pair each; threads
// [that, + n_kv * hd): one v element each. blockIdx.y = sequence of the
// batch (its own q/k/v rows and cache).
__global__ void b200q_rope_kv_kernel(float* __restrict__ q, float* __restrict__ k, const float* __restrict__ v, int n_heads,
                               int n_kv, int hd, int pos, float log2_theta, __half* __restrict__ kc,
                               __half* __restrict__ vc, int max_ctx) {
    griddep_launch_dependents();
    griddep_wait();
    const int b = blockIdx.y;
    q += static_cast<long long>(b) * n_heads * hd;
    k += static_cast<long long>(b) * n_kv * hd;
    v += static_cast<long long>(b) * n_kv * hd;
    kc += static_cast<long long>(b) * n_kv * max_ctx * hd;
    vc += static_cast<long long>(b) * n_kv * max_ctx * hd;
    const int half_dim = hd / 2;
    const int n_pairs = (n_heads + n_kv) * half_dim;
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t < n_pairs) {
        const int head = t / half_dim, p = t - head * half_dim;
        const float inv_freq = exp2f(-2.0f * static_cast<float>(p) / static_cast<float>(hd) * log2_theta);
        float s, c;
        sincosf(static_cast<float>(pos) * inv_freq, &s, &c);
        float* ptr = head < n_heads ? q + head * hd : k + (head - n_heads) * hd;
        const float x0 = ptr[2 * p], x1 = ptr[2 * p + 1];
        const float r0 = x0 * c - x1 * s, r1 = x0 * s + x1 * c;
        ptr[2 * p] = r0;
        ptr[2 * p + 1] = r1;
        if (head >= n_heads) {
            __half* dst = kc + (static_cast<long long>(head - n_heads) * max_ctx + pos) * hd + 2 * p;
            *reinterpret_cast<__half2*>(dst) = __floats2half2_rn(r0, r1);
        }
    } else if (t < n_pairs + n_kv * hd) {
        const int e = t - n_pairs, kvh = e / hd, d = e - kvh * hd;
        vc[(static_cast<long long>(kvh) * max_ctx + pos) * hd + d] = __float2half_rn(v[e]);
    }
}

// Partial record per (query head, chunk): o[kHeadDim], m, l.
constexpr int kPartStride = kHeadDim + 4;  // numerators, max, sum, pad: 16-byte records

// One CTA per (kv head, kAttnChunk positions, sequence), kAttnWarps warps.
// Scores: warp w takes positions w, w + kAttnWarps, ...; a lane holds 4 of
// the 128 dims of the K row (one 8-byte load) and the G query heads' dot
// products are reduced across the warp. Exp-weighted V: the same position
// split, each lane accumulating its 4 dims for the G heads in registers,
// then a reduction over the warps through shared memory. All loads of a
// warp's positions are issued before their arithmetic.
__global__ void __launch_bounds__(kAttnWarps * 32) b200q_attn_chunk_kernel(const float* __restrict__ q,
                                                                     const __half* __restrict__ kc,
                                                                     const __half* __restrict__ vc,
                                                                     float* __restrict__ part, int n_heads, int n_kv,
                                                                     int ctx, int max_ctx, float scale) {
    griddep_launch_dependents();
    griddep_wait();
    constexpr int PW = kAttnChunk / kAttnWarps;  // positions per warp
    __shared__ __align__(16) float qs[kMaxGroup][kHeadDim];
    __shared__ __align__(16) float sc[kMaxGroup][kAttnChunk];
    __shared__ __align__(16) float ml[kMaxGroup][2];
    __shared__ __align__(16) float red[kAttnWarps][kMaxGroup * kHeadDim];  // float4 stores
    const int kvh = blockIdx.x, c = blockIdx.y, n_chunks = gridDim.y, b = blockIdx.z;
    const int G = n_heads / n_kv;
    q += static_cast<long long>(b) * n_heads * kHeadDim;
    kc += static_cast<long long>(b) * n_kv * max_ctx * kHeadDim;
    vc += static_cast<long long>(b) * n_kv * max_ctx * kHeadDim;
    part += static_cast<long long>(b) * n_heads * n_chunks * kPartStride;
    const int p0 = c * kAttnChunk;
    const int np = min(kAttnChunk, ctx - p0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < G * kHeadDim; i += blockDim.x)
        qs[i / kHeadDim][i % kHeadDim] = q[(kvh * G) * kHeadDim + i] * scale;
    __syncthreads();
    const long long row0 = static_cast<long long>(kvh) * max_ctx + p0;
    {
        uint2 kr[PW];
#pragma unroll
        for (int j = 0; j < PW; ++j) {
            const int p = warp + j * kAttnWarps;
            kr[j] = p < np ? *reinterpret_cast<const uint2*>(kc + (row0 + p) * kHeadDim + 4 * lane) : make_uint2(0u, 0u);
        }
#pragma unroll
        for (int j = 0; j < PW; ++j) {
            const int p = warp + j * kAttnWarps;
            const float2 k01 = __half22float2(*reinterpret_cast<const __half2*>(&kr[j].x));
            const float2 k23 = __half22float2(*reinterpret_cast<const __half2*>(&kr[j].y));
            for (int g = 0; g < G; ++g) {
                const float* qg = qs[g] + 4 * lane;
                float d = qg[0] * k01.x + qg[1] * k01.y + qg[2] * k23.x + qg[3] * k23.y;
#pragma unroll
                for (int o = 16; o; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
                if (lane == 0 && p < np) sc[g][p] = d;
            }
        }
    }
    __syncthreads();
    // Chunk max and exp-sum per query head (warp w takes heads w, w + kAttnWarps).
    for (int g = warp; g < G; g += kAttnWarps) {
        float m = -INFINITY;
        for (int p = lane; p < np; p += 32) m = fmaxf(m, sc[g][p]);
#pragma unroll
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float l = 0.0f;
        for (int p = lane; p < np; p += 32) {
            const float e = expf(sc[g][p] - m);
            sc[g][p] = e;
            l += e;
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        if (lane == 0) {
            ml[g][0] = m;
            ml[g][1] = l;
        }
    }
    __syncthreads();
    // Exp-weighted V over this warp's positions; lane = 4 dims.
    float acc[kMaxGroup][4];
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) acc[g][0] = acc[g][1] = acc[g][2] = acc[g][3] = 0.0f;
    {
        uint2 vr[PW];
#pragma unroll
        for (int j = 0; j < PW; ++j) {
            const int p = warp + j * kAttnWarps;
            vr[j] = p < np ? *reinterpret_cast<const uint2*>(vc + (row0 + p) * kHeadDim + 4 * lane) : make_uint2(0u, 0u);
        }
#pragma unroll
        for (int j = 0; j < PW; ++j) {
            const int p = warp + j * kAttnWarps;
            if (p >= np) break;
            const float2 v01 = __half22float2(*reinterpret_cast<const __half2*>(&vr[j].x));
            const float2 v23 = __half22float2(*reinterpret_cast<const __half2*>(&vr[j].y));
#pragma unroll
            for (int g = 0; g < kMaxGroup; ++g) {
                if (g < G) {
                    const float e = sc[g][p];
                    acc[g][0] = fmaf(e, v01.x, acc[g][0]);
                    acc[g][1] = fmaf(e, v01.y, acc[g][1]);
                    acc[g][2] = fmaf(e, v23.x, acc[g][2]);
                    acc[g][3] = fmaf(e, v23.y, acc[g][3]);
                }
            }
        }
    }
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) {
        if (g < G)
            *reinterpret_cast<float4*>(&red[warp][g * kHeadDim + 4 * lane]) =
                make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < G * kHeadDim; i += blockDim.x) {
        float o = 0.0f;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) o += red[w][i];
        const int g = i / kHeadDim, d = i - g * kHeadDim;
        float* rec = part + (static_cast<long long>(kvh * G + g) * n_chunks + c) * kPartStride;
        rec[d] = o;
        if (d == 0) {
            rec[kHeadDim] = ml[g][0];
            rec[kHeadDim + 1] = ml[g][1];
        }
    }
}

// Quantize one 32-element group held one element per lane (lane i holds
// element e = 32 g + i of a row of k) into the quantized row at base: the
// arithmetic of quantize_group, with amax and the code sum by shuffles.
template <int DIG>
__device__ __forceinline__ void quantize_lane_group(float v, uint8_t* base, int k, int e) {
    constexpr float QMAX = DIG == 1 ? 127.0f : 32767.0f;
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float iscale = amax > 0.0f ? __fdiv_rn(QMAX, amax) : 0.0f;
    const int c = round_half_even_small(__fmul_rn(v, iscale));
    int sum = c;
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (DIG == 1) {
        base[e] = static_cast<uint8_t>(c & 0xFF);
    } else {
        base[e] = static_cast<uint8_t>((c >> 8) & 0xFF);
        base[k + e] = static_cast<uint8_t>(c & 0xFF);
    }
    if ((e & 31) == 0) {
        float* gd = reinterpret_cast<float*>(base + static_cast<long long>(k) * DIG);
        gd[e >> 5] = amax > 0.0f ? __fdiv_rn(amax, QMAX) : 0.0f;
        reinterpret_cast<int*>(gd + k / 32)[e >> 5] = sum;
    }
}

// DIG > 0: the attention output row of each sequence (n_heads * head_dim
// elements) is also quantized into xq for the o projection (out may be null).
template <int DIG>
__global__ void __launch_bounds__(kHeadDim) b200q_attn_combine_kernel(const float* __restrict__ part, float* __restrict__ out,
                                                                uint8_t* __restrict__ xq, int n_chunks) {
    griddep_launch_dependents();
    griddep_wait();
    __shared__ float wsh[kHeadDim];  // chunk weights exp(m_c - M), one tile of chunks
    __shared__ float lsh[kHeadDim];  // l_c * weight
    __shared__ float msh[kHeadDim / 32];
    const int h = blockIdx.x, d = threadIdx.x, b = blockIdx.y, n_heads = gridDim.x;
    const float* rec = part + (static_cast<long long>(b) * n_heads + h) * n_chunks * kPartStride;
    float m = -INFINITY;
    for (int c = d; c < n_chunks; c += kHeadDim) m = fmaxf(m, rec[c * kPartStride + kHeadDim]);
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((d & 31) == 0) msh[d >> 5] = m;
    __syncthreads();
    float M = msh[0];
#pragma unroll
    for (int w = 1; w < kHeadDim / 32; ++w) M = fmaxf(M, msh[w]);
    float L = 0.0f, acc = 0.0f;
    for (int c0 = 0; c0 < n_chunks; c0 += kHeadDim) {
        const int nt = min(kHeadDim, n_chunks - c0);
        __syncthreads();
        if (d < nt) {
            const float w = expf(rec[(c0 + d) * kPartStride + kHeadDim] - M);
            wsh[d] = w;
            lsh[d] = rec[(c0 + d) * kPartStride + kHeadDim + 1] * w;
        }
        __syncthreads();
#pragma unroll 8
        for (int t = 0; t < nt; ++t) {
            acc = fmaf(rec[(c0 + t) * kPartStride + d], wsh[t], acc);
            L += lsh[t];
        }
    }
    const float v = acc / L;
    if (out) out[static_cast<long long>(b) * n_heads * kHeadDim + h * kHeadDim + d] = v;
    if constexpr (DIG > 0) {
        const int k = n_heads * kHeadDim;
        quantize_lane_group<DIG>(v, xq + static_cast<long long>(b) * xq_row_bytes(k, DIG), k, h * kHeadDim + d);
    }
}

// Where a sequence's cached keys and values live (template KVM):
//  * KV_CONTIG: fp16 [seq][kv_head][max_ctx][head_dim] (one contiguous cache);
//  * KV_PAGED: fp16 pages of `page` positions, [slot][kv_head][page][head_dim],
//    the slot of each of a sequence's pages taken from its page table
//    (model_graph.cpp:1413-1449 keeps pages of 4096 tokens per layer);
//  * KV_PAGED_Q8: the same pages holding int8 codes plus one fp32 scale per
//    (slot, kv head, position): the reference's q8 KV mode
//    (model_graph.cpp:507-513, 1539-1576): scale = amax / 127 (1 / 127 for an
//    all-zero row), code = clamp(round(x * (1 / scale)), -127, 127).
constexpr int KV_CONTIG = 0, KV_PAGED = 1, KV_PAGED_Q8 = 2;

struct KvArgs {
    void* k;              // cache or page pool (fp16, or int8 codes for Q8)
    void* v;
    float* ks;            // Q8: scale pools [slot][kv_head][page]
    float* vs;
    const int* table;     // paged: [seq][pages_per_seq] slot of each page, -1 = none
    int pages_per_seq;
    int page;             // positions per page
    int n_slots;          // pages in the pool
    int max_ctx;          // contiguous: positions per sequence
    volatile int* status; // STATUS_BAD_PAGE is recorded here
};

// Element offset of (sequence b, kv head h, position p) in the caches (the
// offset / kHeadDim indexes the Q8 scales), or -1 where the page table names
// no page: the reference scores such a position -1e9 and skips its value
// (model_graph.cpp:1790-1795, 1896-1897); a slot past the pool is treated
// the same and recorded as STATUS_BAD_PAGE.
template <int KVM>
__device__ __forceinline__ long long kv_row(const KvArgs& a, int b, int h, int n_kv, int p) {
    if constexpr (KVM == KV_CONTIG) {
        return ((static_cast<long long>(b) * n_kv + h) * a.max_ctx + p) * kHeadDim;
    } else {
        const int slot = __ldg(a.table + static_cast<long long>(b) * a.pages_per_seq + p / a.page);
        if (slot < 0 || slot >= a.n_slots) {
            if (slot >= a.n_slots) *a.status = STATUS_BAD_PAGE;
            return -1;
        }
        return ((static_cast<long long>(slot) * n_kv + h) * a.page + (p % a.page)) * kHeadDim;
    }
}

constexpr float kMaskedScore = -1e9f;  // the reference's score for a position without a page

// One lane's four cached elements of a row (raw) and their values.
template <int KVM>
struct KvLane {
    using Raw = typename std::conditional<KVM == KV_PAGED_Q8, uint32_t, uint2>::type;
    __device__ static Raw load(const void* base, long long row, int lane) {
        if constexpr (KVM == KV_PAGED_Q8)
            return *reinterpret_cast<const uint32_t*>(static_cast<const int8_t*>(base) + row + 4 * lane);
        else
            return *reinterpret_cast<const uint2*>(static_cast<const __half*>(base) + row + 4 * lane);
    }
    // fp16: the values; Q8: the codes (the scale is applied by the caller,
    // to the dot product for keys and to the softmax weight for values, as
    // model_graph.cpp:1790-1812 and 1894-1915 do).
    __device__ static float4 value(Raw r) {
        if constexpr (KVM == KV_PAGED_Q8) {
            return make_float4(static_cast<float>(static_cast<int8_t>(r & 0xFFu)),
                               static_cast<float>(static_cast<int8_t>((r >> 8) & 0xFFu)),
                               static_cast<float>(static_cast<int8_t>((r >> 16) & 0xFFu)),
                               static_cast<float>(static_cast<int8_t>(r >> 24)));
        } else {
            const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&r.x));
            const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&r.y));
            return make_float4(a.x, a.y, b.x, b.y);
        }
    }
};

// Q8 codes of four values of a 128-element row held by the 32 lanes of a
// warp (lane l: elements 4l .. 4l+3), packed little-endian, and the row's
// scale in *scale.
__device__ __forceinline__ uint32_t q8_row_codes(float4 x, float* scale_out) {
    float amax = fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w)));
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : __fdiv_rn(1.0f, 127.0f);
    const float inv = __fdiv_rn(1.0f, scale);
    auto code = [&](float e) {
        const int c = static_cast<int>(roundf(__fmul_rn(e, inv)));
        return static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(max(-127, min(127, c)))));
    };
    *scale_out = scale;
    return code(x.x) | (code(x.y) << 8) | (code(x.z) << 16) | (code(x.w) << 24);
}

// Pair i (elements 2i, 2i+1) of a head rotated to position pos
// (apply_rope_with_dim, model_graph.cpp:1222-1323: angle pos * theta^(-2i / d)).
// Explicitly rounded products and sums, so every caller gets the same bits.
__device__ __forceinline__ float2 rope_pair(float x0, float x1, int pos, int i, float log2_theta) {
    const float inv_freq = exp2f(-2.0f * static_cast<float>(i) / static_cast<float>(kHeadDim) * log2_theta);
    float s, c;
    sincosf(static_cast<float>(pos) * inv_freq, &s, &c);
    return make_float2(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s)), __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c)));
}

// Lane l's elements 4l .. 4l+3 of key row `kin` rotated to position pos.
__device__ __forceinline__ float4 rope_lane(const float* kin, int pos, int lane, float log2_theta) {
    const float4 x = *reinterpret_cast<const float4*>(kin + 4 * lane);
    const float2 a = rope_pair(x.x, x.y, pos, 2 * lane, log2_theta);
    const float2 b = rope_pair(x.z, x.w, pos, 2 * lane + 1, log2_theta);
    return make_float4(a.x, a.y, b.x, b.y);
}

// A lane's four elements in the cache's storage form (fp16 pairs, or Q8
// codes with the row scale in *scale).
template <int KVM>
__device__ __forceinline__ typename KvLane<KVM>::Raw to_stored(float4 x, float* scale) {
    if constexpr (KVM == KV_PAGED_Q8) {
        return q8_row_codes(x, scale);
    } else {
        const __half2 a = __floats2half2_rn(x.x, x.y), b = __floats2half2_rn(x.z, x.w);
        uint2 r;
        r.x = *reinterpret_cast<const uint32_t*>(&a);
        r.y = *reinterpret_cast<const uint32_t*>(&b);
        *scale = 1.0f;
        return r;
    }
}

// Fused decode attention (the RoPE and attention stages of the reference's
// decode graph, model_graph.cpp:1222-1323 and the GQA attention after it,
// in one launch). blockIdx.z = s * n_tok + t: token t of sequence s, at
// position pos + t. n_tok = 1 is the ordinary decode step of a batch of
// sequences; n_tok > 1 runs several consecutive tokens of each sequence
// (the rows a speculative verify feeds through the stack in one pass), each
// attending causally over the cache and the tokens before it.
//  * every CTA rotates its kv head's G query heads into shared memory,
//    scaled by 1 / sqrt(head_dim);
//  * the CTA whose chunk holds its token's position appends the rotated key
//    and the value there (fp16, or Q8 codes and scales);
//  * positions written by this launch (pos .. pos + t) are not read back
//    from the cache: each CTA forms those rows from the q/k/v inputs in the
//    cache's storage form, bit-identical to what is stored; older positions
//    are loaded before the wait on the preceding kernel;
//  * each CTA scores and weights its kAttnChunk positions like
//    b200q_attn_chunk_kernel and writes its partial records;
//  * the CTA that finishes last for a (kv head, token) -- an arrival
//    counter, reset by that CTA -- merges the chunks (max rescaling) and
//    writes the output rows and, with DIG > 0, their x8 / x16 codes. No CTA
//    waits for another (threadfence-reduction pattern).
template <int G, int DIG, int KVM>
__global__ void __launch_bounds__(kAttnWarps * 32, 2) b200q_attn_decode_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v, const KvArgs kv,
    float* __restrict__ part, int* __restrict__ counters, float* __restrict__ out, uint8_t* __restrict__ xq,
    int n_heads, int n_kv, int pos, int n_tok, long long q_stride, long long kv_stride, float log2_theta,
    float scale) {
    griddep_launch_dependents();
    using KL = KvLane<KVM>;
    using Raw = typename KL::Raw;
    constexpr bool Q8 = KVM == KV_PAGED_Q8;
    constexpr int PW = kAttnChunk / kAttnWarps;  // positions per warp
    constexpr int HALF = kHeadDim / 2;
    // Keys are scored position-major: lane l of a warp takes position slot
    // l / 4 of the warp's PW positions over the quarter l % 4 of the head
    // dimension (QD elements, KW 32-bit words of stored form), so a dot
    // product needs two shuffle levels instead of five. Values stay
    // dimension-major (lane l: elements 4l .. 4l+3 of each of the PW rows).
    static_assert(PW * 4 == 32, "one position slot per four lanes");
    constexpr int QD = kHeadDim / 4;
    constexpr int KW = Q8 ? QD / 4 : QD / 2;         // words per lane quarter: 8 (Q8) or 16 (fp16)
    constexpr int ROWW = Q8 ? kHeadDim / 4 : kHeadDim / 2;  // words per stored row
    constexpr int QPAD = QD + 4;  // query quarters padded so the 4 quarters fall on distinct banks
    // 16-byte aligned: qs, red and the staged rows are accessed as float4 / uint4.
    __shared__ __align__(16) float qs[G][4][QPAD];
    __shared__ float ml[kAttnWarps][G][2];  // per warp and head: max, exp-sum
    // red (after the PV phase) shares its storage with the key rows this
    // launch writes (read in the score phase only).
    constexpr int kRedBytes = kAttnWarps * G * kHeadDim * 4;
    constexpr int kFreshBytes = kAttnChunk * ROWW * 4;
    __shared__ __align__(16) unsigned char shared_rows[kRedBytes > kFreshBytes ? kRedBytes : kFreshBytes];
    __shared__ float fresh_ks[kAttnChunk];
    __shared__ float merge_l[kAttnWarps];
    __shared__ int is_last;
    float (*red)[G * kHeadDim] = reinterpret_cast<float (*)[G * kHeadDim]>(shared_rows);
    uint32_t (*fresh_k)[ROWW] = reinterpret_cast<uint32_t (*)[ROWW]>(shared_rows);
    const int kvh = blockIdx.x, c = blockIdx.y, b = blockIdx.z;  // b: the (sequence, token) row
    const int seq = b / n_tok, tok = b - seq * n_tok;
    const int my_pos = pos + tok;
    const int n_chunks = my_pos / kAttnChunk + 1;  // this token's chunks (gridDim.y covers the last token)
    if (c >= n_chunks) return;
    const int ctx = my_pos + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // q, k and v rows (one per (sequence, token)) lie q_stride / kv_stride
    // floats apart: packed, or rows of one q|k|v projection output.
    const float* k_seq = k + static_cast<long long>(seq) * n_tok * kv_stride + kvh * kHeadDim;  // token 0's k row
    const float* v_seq = v + static_cast<long long>(seq) * n_tok * kv_stride + kvh * kHeadDim;
    const long long tok_stride = kv_stride;
    q += static_cast<long long>(b) * q_stride + kvh * G * kHeadDim;
    part += (static_cast<long long>(b) * n_heads + kvh * G) * gridDim.y * kPartStride;  // records [g][chunk]
    const int p0 = c * kAttnChunk;
    const int np = min(kAttnChunk, ctx - p0);
    const int kp = warp + (lane >> 2) * kAttnWarps;  // this lane's key position in the chunk
    const int qd = lane & 3;                          // and its quarter of the head dimension
    // Rows before pos were written by earlier steps: load them before
    // waiting for the preceding kernel (the projection that produces q, k,
    // v), so the loads overlap its tail.
    uint4 kq[KW / 4];
    float kscale = 0.0f;
    bool k_live = false;
#pragma unroll
    for (int w = 0; w < KW / 4; ++w) kq[w] = make_uint4(0u, 0u, 0u, 0u);
    {
        const long long row = kp < np && p0 + kp < pos ? kv_row<KVM>(kv, seq, kvh, n_kv, p0 + kp) : -1;
        if (row >= 0) {
            const uint4* src = reinterpret_cast<const uint4*>(static_cast<const unsigned char*>(kv.k) +
                                                              (row + qd * QD) * (Q8 ? 1 : 2));
#pragma unroll
            for (int w = 0; w < KW / 4; ++w) kq[w] = src[w];
            if constexpr (Q8) kscale = kv.ks[row / kHeadDim];
            k_live = true;
        }
    }
    Raw vr[PW];
    float vsc[PW];
    uint32_t v_live = 0;  // bit j: this warp's position j has a value row
#pragma unroll
    for (int j = 0; j < PW; ++j) {
        const int p = warp + j * kAttnWarps;
        vr[j] = Raw{};
        vsc[j] = 0.0f;
        const long long row = p < np && p0 + p < pos ? kv_row<KVM>(kv, seq, kvh, n_kv, p0 + p) : -1;
        if (row >= 0) {
            v_live |= 1u << j;
            vr[j] = KL::load(kv.v, row, lane);
            if constexpr (Q8) vsc[j] = kv.vs[row / kHeadDim];
        }
    }
    griddep_wait();
    for (int i = threadIdx.x; i < G * HALF; i += blockDim.x) {
        const int g = i / HALF, p = i - g * HALF;
        const float2 r = rope_pair(q[g * kHeadDim + 2 * p], q[g * kHeadDim + 2 * p + 1], my_pos, p, log2_theta);
        const int e = 2 * p;
        qs[g][e / QD][e % QD] = r.x * scale;
        qs[g][e / QD][e % QD + 1] = r.y * scale;
    }
    // This launch's own positions (pos .. my_pos): rows formed from the
    // inputs in the cache's storage form (bit-identical to what is stored);
    // keys staged in shared memory for the position-major score phase.
#pragma unroll
    for (int j = 0; j < PW; ++j) {
        const int p = warp + j * kAttnWarps;
        const int pp = p0 + p;
        if (p < np && pp >= pos && kv_row<KVM>(kv, seq, kvh, n_kv, pp) >= 0) {  // warp-uniform
            const long long t = pp - pos;
            float ks;
            const Raw kr = to_stored<KVM>(rope_lane(k_seq + t * tok_stride, pp, lane, log2_theta), &ks);
            if constexpr (Q8) fresh_k[p][lane] = kr;
            else *reinterpret_cast<uint2*>(&fresh_k[p][2 * lane]) = kr;
            if (lane == 0) fresh_ks[p] = ks;
            vr[j] = to_stored<KVM>(*reinterpret_cast<const float4*>(v_seq + t * tok_stride + 4 * lane), &vsc[j]);
            v_live |= 1u << j;
        }
    }
    if (c == n_chunks - 1) {  // this chunk holds my_pos: append its rotated key and value
        const long long prow = kv_row<KVM>(kv, seq, kvh, n_kv, my_pos);
        if (prow < 0) {
            if (threadIdx.x == 0) *kv.status = STATUS_BAD_PAGE;  // no page to append to
        } else if (warp < 2) {  // warp 0: the key, warp 1: the value (lane l: elements 4l .. 4l+3)
            const float* src = (warp == 0 ? k_seq : v_seq) + tok * tok_stride;
            const float4 x = warp == 0 ? rope_lane(src, my_pos, lane, log2_theta)
                                       : *reinterpret_cast<const float4*>(src + 4 * lane);
            float sc_row;
            const Raw r = to_stored<KVM>(x, &sc_row);
            if constexpr (Q8) {
                *reinterpret_cast<uint32_t*>(static_cast<int8_t*>(warp == 0 ? kv.k : kv.v) + prow + 4 * lane) = r;
                if (lane == 0) (warp == 0 ? kv.ks : kv.vs)[prow / kHeadDim] = sc_row;
            } else {
                *reinterpret_cast<uint2*>(static_cast<__half*>(warp == 0 ? kv.k : kv.v) + prow + 4 * lane) = r;
            }
        }
    }
    __syncthreads();  // the rotated queries and the staged key rows are visible to the CTA
    // Scores: lane group l / 4 holds the G dot products of its position;
    // positions past the context score -inf (excluded), positions without a
    // page kMaskedScore (counted, as in the reference).
    float d[G];
    {
        if (kp < np && p0 + kp >= pos && kv_row<KVM>(kv, seq, kvh, n_kv, p0 + kp) >= 0) {
            const uint4* src = reinterpret_cast<const uint4*>(&fresh_k[kp][qd * KW]);
#pragma unroll
            for (int w = 0; w < KW / 4; ++w) kq[w] = src[w];
            kscale = fresh_ks[kp];
            k_live = true;
        }
        const uint32_t* kw = reinterpret_cast<const uint32_t*>(kq);
#pragma unroll
        for (int g = 0; g < G; ++g) d[g] = 0.0f;
#pragma unroll
        for (int i = 0; i < QD / 4; ++i) {  // elements 4i .. 4i+3 of the quarter
            float4 x;
            if constexpr (Q8) {
                const uint32_t r = kw[i];
                x = make_float4(static_cast<float>(static_cast<int8_t>(r & 0xFFu)),
                                static_cast<float>(static_cast<int8_t>((r >> 8) & 0xFFu)),
                                static_cast<float>(static_cast<int8_t>((r >> 16) & 0xFFu)),
                                static_cast<float>(static_cast<int8_t>(r >> 24)));
            } else {
                const uint32_t r0 = kw[2 * i], r1 = kw[2 * i + 1];
                const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&r0));
                const float2 bb = __half22float2(*reinterpret_cast<const __half2*>(&r1));
                x = make_float4(a.x, a.y, bb.x, bb.y);
            }
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float4 qg = *reinterpret_cast<const float4*>(&qs[g][qd][4 * i]);
                d[g] = fmaf(qg.x, x.x, fmaf(qg.y, x.y, fmaf(qg.z, x.z, fmaf(qg.w, x.w, d[g]))));
            }
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
            d[g] += __shfl_xor_sync(0xffffffffu, d[g], 1);
            d[g] += __shfl_xor_sync(0xffffffffu, d[g], 2);
            if constexpr (Q8) d[g] *= kscale;
            if (!k_live) d[g] = kMaskedScore;
            if (kp >= np) d[g] = -INFINITY;
        }
    }
    // Chunk softmax: each warp's maximum over its PW positions (lane groups
    // differ in lane bits 2..4), one barrier, the chunk maximum from the
    // warps' maxima; then each warp's exp-weighted values.
#pragma unroll
    for (int g = 0; g < G; ++g) {
        float m = d[g];
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
        if (lane == 0) ml[warp][g][0] = m;  // -inf only when none of the warp's positions is in the context
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < G; ++g) {
        float m = ml[0][g][0];  // the chunk maximum (position 0 of a chunk is always in the context)
#pragma unroll
        for (int w = 1; w < kAttnWarps; ++w) m = fmaxf(m, ml[w][g][0]);
        d[g] = d[g] == -INFINITY ? 0.0f : expf(d[g] - m);
        float l = d[g];
        l += __shfl_xor_sync(0xffffffffu, l, 4);
        l += __shfl_xor_sync(0xffffffffu, l, 8);
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        if (lane == 0) ml[warp][g][1] = l;
    }
    float acc[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g][0] = acc[g][1] = acc[g][2] = acc[g][3] = 0.0f;
#pragma unroll
    for (int j = 0; j < PW; ++j) {
        const float4 vf = KL::value(vr[j]);  // zero without a row
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float e = __shfl_sync(0xffffffffu, d[g], 4 * j);  // slot j's weight
            if constexpr (Q8) e *= vsc[j];
            acc[g][0] = fmaf(e, vf.x, acc[g][0]);
            acc[g][1] = fmaf(e, vf.y, acc[g][1]);
            acc[g][2] = fmaf(e, vf.z, acc[g][2]);
            acc[g][3] = fmaf(e, vf.w, acc[g][3]);
        }
    }
#pragma unroll
    for (int g = 0; g < G; ++g)
        *reinterpret_cast<float4*>(&red[warp][g * kHeadDim + 4 * lane]) =
            make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
    __syncthreads();
    // The chunk's record per query head: the warps' sums.
    for (int i = threadIdx.x; i < G * kHeadDim; i += blockDim.x) {
        const int g = i / kHeadDim, dd = i - g * kHeadDim;
        float o = 0.0f;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) o += red[w][i];
        float* rec = part + (static_cast<long long>(g) * n_chunks + c) * kPartStride;
        rec[dd] = o;
        if (dd == 0) {
            float m = ml[0][g][0], l = 0.0f;
#pragma unroll
            for (int w = 0; w < kAttnWarps; ++w) {
                m = fmaxf(m, ml[w][g][0]);
                l += ml[w][g][1];
            }
            rec[kHeadDim] = m;
            rec[kHeadDim + 1] = l;
        }
    }
    // Release the records (the barrier orders the CTA's stores before the
    // releasing atomic of thread 0) and count the arrival; the last CTA's
    // thread 0 acquires the other CTAs' records the same way.
    __syncthreads();
    if (threadIdx.x == 0) {
        int prev;
        asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;"
                     : "=r"(prev)
                     : "l"(counters + b * n_kv + kvh)
                     : "memory");
        is_last = prev == n_chunks - 1;
    }
    __syncthreads();
    if (!is_last) return;
    // Merge: S = kAttnWarps / G warps per query head g, warp s of a head
    // taking chunks s, s + S, ...; each lane holds 4 output dims. The first
    // 16 of a warp's records are loaded together with the chunk maxima.
    {
        constexpr int S = kAttnWarps / G;
        constexpr int B8 = 16;
        const int g = warp % G, s = warp / G;
        const float* rec = part + static_cast<long long>(g) * n_chunks * kPartStride;
        float4 x[B8];
        float2 mlc[B8];
#pragma unroll
        for (int t = 0; t < B8; ++t) {
            const int cc = s + t * S;
            x[t] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            mlc[t] = make_float2(-INFINITY, 0.0f);
            if (cc < n_chunks) {
                const float* r = rec + cc * kPartStride;
                x[t] = __ldcg(reinterpret_cast<const float4*>(r + 4 * lane));
                mlc[t] = __ldcg(reinterpret_cast<const float2*>(r + kHeadDim));
            }
        }
        float M = -INFINITY;
        for (int cc = lane; cc < n_chunks; cc += 32) M = fmaxf(M, __ldcg(rec + cc * kPartStride + kHeadDim));
#pragma unroll
        for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float L = 0.0f;
        float4 a = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
        for (int t = 0; t < B8; ++t) {
            const float w = mlc[t].x == -INFINITY ? 0.0f : expf(mlc[t].x - M);
            L = fmaf(mlc[t].y, w, L);
            a.x = fmaf(x[t].x, w, a.x);
            a.y = fmaf(x[t].y, w, a.y);
            a.z = fmaf(x[t].z, w, a.z);
            a.w = fmaf(x[t].w, w, a.w);
        }
#pragma unroll 8
        for (int cc = s + B8 * S; cc < n_chunks; cc += S) {
            const float* r = rec + cc * kPartStride;
            const float2 m2 = __ldcg(reinterpret_cast<const float2*>(r + kHeadDim));
            const float4 y = __ldcg(reinterpret_cast<const float4*>(r + 4 * lane));
            const float w = expf(m2.x - M);
            L = fmaf(m2.y, w, L);
            a.x = fmaf(y.x, w, a.x);
            a.y = fmaf(y.y, w, a.y);
            a.z = fmaf(y.z, w, a.z);
            a.w = fmaf(y.w, w, a.w);
        }
        if constexpr (S > 1) {
            *reinterpret_cast<float4*>(&red[warp][4 * lane]) = a;
            if (lane == 0) merge_l[warp] = L;
            __syncthreads();
            if (s == 0) {
#pragma unroll
                for (int t = 1; t < S; ++t) {
                    const float4 y = *reinterpret_cast<const float4*>(&red[warp + t * G][4 * lane]);
                    a.x += y.x;
                    a.y += y.y;
                    a.z += y.z;
                    a.w += y.w;
                    L += merge_l[warp + t * G];
                }
            }
        }
        if (s == 0) {
            const float4 res = make_float4(a.x / L, a.y / L, a.z / L, a.w / L);
            const int head = kvh * G + g;
            if (out)
                *reinterpret_cast<float4*>(out + (static_cast<long long>(b) * n_heads + head) * kHeadDim + 4 * lane) =
                    res;
            if constexpr (DIG > 0) {
                const int kk = n_heads * kHeadDim;
                quantize_quad<DIG>(res, true, xq + static_cast<long long>(b) * xq_row_bytes(kk, DIG), kk,
                                   head * (kHeadDim / 4) + lane);
            }
        }
    }
    if (threadIdx.x == 0) counters[b * n_kv + kvh] = 0;  // ready for the next launch
}

// out = silu(gate) * up, element-wise (the SiLU * up step of
// quantized_matmul.cpp:2380-2412, as the fused expert kernel computes it).
__global__ void b200q_swiglu_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ out,
                              long long n) {
    griddep_launch_dependents();
    griddep_wait();
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float gv = g[i];
    out[i] = gv / (1.0f + expf(-gv)) * u[i];
}

// out[r][j] = silu(gu[r][j]) * gu[r][n + j] for rows of [gate n | up n]: the
// SiLU * up step for several rows of one gate/up projection output.
__global__ void b200q_swiglu_rows_kernel(const float* __restrict__ gu, float* __restrict__ out, int rows, int n) {
    griddep_launch_dependents();
    griddep_wait();
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<long long>(rows) * n) return;
    const long long r = i / n, j = i - r * n;
    const float gv = gu[r * 2 * n + j];
    out[i] = gv / (1.0f + expf(-gv)) * gu[r * 2 * n + n + j];
}

// out[r][s * cols + j] = in[s][r][j]: the row-major [rows][shards * cols]
// view of an all-gather of per-shard [rows][cols] blocks.
__global__ void b200q_unshard_rows_kernel(const float* __restrict__ in, float* __restrict__ out, int shards, int rows,
                                    int cols) {
    griddep_launch_dependents();
    griddep_wait();
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const long long total = static_cast<long long>(shards) * rows * cols;
    if (i >= total) return;
    const int j = static_cast<int>(i % cols);
    const long long t = i / cols;
    const int r = static_cast<int>(t % rows), s = static_cast<int>(t / rows);
    out[(static_cast<long long>(r) * shards + s) * cols + j] = in[i];
}

cudaLaunchConfig_t pdl_cfg(dim3 grid, dim3 block, cudaStream_t st, cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = st;
    if (pdl_enabled()) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cfg;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int launch_add_rmsnorm(float* res, const float* delta, const float* gamma, float* out, int n, int rows, float eps,
                       cudaStream_t st, void* xq, int act_mode) {
    if (!res || !gamma || (!out && !xq) || n <= 0 || rows <= 0) return B200Q_EINVAL;
    if (n % 4 || (xq && n % 128)) return B200Q_ESHAPE;
    if (xq && act_mode != B200Q_ACT_X8 && act_mode != B200Q_ACT_X16) return B200Q_EINVAL;
    if (!aligned16(res) || !aligned16(gamma) || (out && !aligned16(out)) || (delta && !aligned16(delta)) ||
        (xq && !aligned16(xq)))
        return B200Q_EALIGN;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_cfg(dim3(rows), dim3(kNormThreads), st, attr);
    uint8_t* q = static_cast<uint8_t*>(xq);
    cudaError_t e;
    if (n <= 4 * kNormRegVec * kNormThreads) {
        if (!xq) e = cudaLaunchKernelEx(&cfg, b200q_add_rmsnorm_reg_kernel<0>, res, delta, gamma, out, q, n, eps);
        else if (act_mode == B200Q_ACT_X8)
            e = cudaLaunchKernelEx(&cfg, b200q_add_rmsnorm_reg_kernel<1>, res, delta, gamma, out, q, n, eps);
        else e = cudaLaunchKernelEx(&cfg, b200q_add_rmsnorm_reg_kernel<2>, res, delta, gamma, out, q, n, eps);
    } else if (!xq) {
        e = cudaLaunchKernelEx(&cfg, b200q_add_rmsnorm_kernel<0>, res, delta, gamma, out, q, n, eps);
    } else if (act_mode == B200Q_ACT_X8) {
        e = cudaLaunchKernelEx(&cfg, b200q_add_rmsnorm_kernel<1>, res, delta, gamma, out, q, n, eps);
    } else {
        e = cudaLaunchKernelEx(&cfg, b200q_add_rmsnorm_kernel<2>, res, delta, gamma, out, q, n, eps);
    }
    return e == cudaSuccess ? B200Q_OK : B200Q_ECUDA;
}

int launch_rope_kv(float* q, float* k, const float* v, int batch, int n_heads, int n_kv, int hd, int pos, float theta,
                   void* kc, void* vc, int max_ctx, cudaStream_t st) {
    if (!q || !k || !v || !kc || !vc || batch <= 0 || n_heads <= 0 || n_kv <= 0 || hd <= 0 || max_ctx <= 0)
        return B200Q_EINVAL;
    if (hd % 2 || n_heads % n_kv || pos < 0 || pos >= max_ctx || !(theta > 0.0f)) return B200Q_ESHAPE;
    if ((reinterpret_cast<uintptr_t>(kc) & 3u) || (reinterpret_cast<uintptr_t>(vc) & 1u)) return B200Q_EALIGN;
    const int threads = (n_heads + n_kv) * (hd / 2) + n_kv * hd;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_cfg(dim3((threads + 255) / 256, batch), dim3(256), st, attr);
    return cudaLaunchKernelEx(&cfg, b200q_rope_kv_kernel, q, k, v, n_heads, n_kv, hd, pos, log2f(theta),
                              static_cast<__half*>(kc), static_cast<__half*>(vc), max_ctx) == cudaSuccess
               ? B200Q_OK
               : B200Q_ECUDA;
}

int launch_attention(const float* q, const void* kc, const void* vc, float* out, int batch, int n_heads, int n_kv,
                     int hd, int ctx, int max_ctx, Device* dev, cudaStream_t st, void* xq, int act_mode) {
    if (!q || !kc || !vc || (!out && !xq) || batch <= 0 || n_heads <= 0 || n_kv <= 0 || ctx <= 0 || !dev)
        return B200Q_EINVAL;
    if (xq && act_mode != B200Q_ACT_X8 && act_mode != B200Q_ACT_X16) return B200Q_EINVAL;
    if (xq && (reinterpret_cast<uintptr_t>(xq) & 15u)) return B200Q_EALIGN;
    if (hd != kHeadDim || n_heads % n_kv || n_heads / n_kv > kMaxGroup || ctx > max_ctx) return B200Q_ESHAPE;
    if ((reinterpret_cast<uintptr_t>(kc) & 7u) || (reinterpret_cast<uintptr_t>(vc) & 1u)) return B200Q_EALIGN;
    const int n_chunks = (ctx + kAttnChunk - 1) / kAttnChunk;
    void* part = nullptr;
    int rc = scratch_for(dev, st, kScratchAttn,
                         static_cast<size_t>(batch) * n_heads * n_chunks * kPartStride * sizeof(float), &part);
    if (rc != B200Q_OK) return rc;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_cfg(dim3(n_kv, n_chunks, batch), dim3(kAttnWarps * 32), st, attr);
    if (cudaLaunchKernelEx(&cfg, b200q_attn_chunk_kernel, q, static_cast<const __half*>(kc), static_cast<const __half*>(vc),
                           static_cast<float*>(part), n_heads, n_kv, ctx, max_ctx,
                           1.0f / sqrtf(static_cast<float>(hd))) != cudaSuccess)
        return B200Q_ECUDA;
    cudaLaunchConfig_t cfg2 = pdl_cfg(dim3(n_heads, batch), dim3(kHeadDim), st, attr);
    const float* pp = static_cast<const float*>(part);
    uint8_t* qx = static_cast<uint8_t*>(xq);
    cudaError_t e;
    if (!xq) e = cudaLaunchKernelEx(&cfg2, b200q_attn_combine_kernel<0>, pp, out, qx, n_chunks);
    else if (act_mode == B200Q_ACT_X8) e = cudaLaunchKernelEx(&cfg2, b200q_attn_combine_kernel<1>, pp, out, qx, n_chunks);
    else e = cudaLaunchKernelEx(&cfg2, b200q_attn_combine_kernel<2>, pp, out, qx, n_chunks);
    return e == cudaSuccess ? B200Q_OK : B200Q_ECUDA;
}

namespace {

// Shared by the contiguous and paged entry points: checks the head shapes and
// outputs, takes the scratch, and launches b200q_attn_decode_kernel<G, DIG, KVM>.
int launch_attention(int kvm, const KvArgs& kv, const float* q, const float* k, const float* v, int batch,
                     int n_tok, int n_heads, int n_kv, int hd, int pos, float theta, float* out, void* xq,
                     int act_mode, Device* dev, cudaStream_t st, long long q_stride = 0, long long kv_stride = 0) {
    if (!q || !k || !v || (!out && !xq) || batch <= 0 || n_tok <= 0 || n_heads <= 0 || n_kv <= 0 || !dev)
        return B200Q_EINVAL;
    if (xq && act_mode != B200Q_ACT_X8 && act_mode != B200Q_ACT_X16) return B200Q_EINVAL;
    if (hd != kHeadDim || n_heads % n_kv || pos < 0 || !(theta > 0.0f)) return B200Q_ESHAPE;
    const long long rows = static_cast<long long>(batch) * n_tok;
    if (rows > 65535) return B200Q_ESHAPE;
    const int G = n_heads / n_kv;
    if (G != 1 && G != 2 && G != 4 && G != 8) return B200Q_ESHAPE;
    if (q_stride == 0) q_stride = static_cast<long long>(n_heads) * kHeadDim;
    if (kv_stride == 0) kv_stride = static_cast<long long>(n_kv) * kHeadDim;
    if (q_stride < static_cast<long long>(n_heads) * kHeadDim || kv_stride < static_cast<long long>(n_kv) * kHeadDim)
        return B200Q_ESHAPE;
    if ((out && !aligned16(out)) || (xq && !aligned16(xq)) || !aligned16(k) || !aligned16(v) || (kv_stride & 3))
        return B200Q_EALIGN;
    const int n_chunks = (pos + n_tok - 1) / kAttnChunk + 1;  // the last token's
    void* part = nullptr;
    void* cnt = nullptr;
    int rc = scratch_for(dev, st, kScratchAttn,
                         static_cast<size_t>(rows) * n_heads * n_chunks * kPartStride * sizeof(float), &part);
    // Arrival counters: zero when allocated (all of the buffer, so a later
    // call with more rows finds its counters zero too); the merging CTA
    // resets its counter after each launch.
    if (rc == B200Q_OK)
        rc = scratch_for(dev, st, kScratchAttnCnt, static_cast<size_t>(rows) * n_kv * sizeof(int), &cnt, true);
    if (rc != B200Q_OK) return rc;
    KvArgs a = kv;
    a.status = dev->status;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg =
        pdl_cfg(dim3(n_kv, n_chunks, static_cast<unsigned>(rows)), dim3(kAttnWarps * 32), st, attr);
    const int dig = !xq ? 0 : (act_mode == B200Q_ACT_X8 ? 1 : 2);
    auto go = [&](auto kern) {
        return cudaLaunchKernelEx(&cfg, kern, q, k, v, a, static_cast<float*>(part), static_cast<int*>(cnt), out,
                                  static_cast<uint8_t*>(xq), n_heads, n_kv, pos, n_tok, q_stride, kv_stride,
                                  log2f(theta), 1.0f / sqrtf(static_cast<float>(hd)));
    };
    cudaError_t e = cudaErrorInvalidValue;
#define B200Q_ATTN_KVM(GG, DD)                                                          \
    if (kvm == KV_CONTIG) e = go(b200q_attn_decode_kernel<GG, DD, KV_CONTIG>);            \
    else if (kvm == KV_PAGED) e = go(b200q_attn_decode_kernel<GG, DD, KV_PAGED>);         \
    else e = go(b200q_attn_decode_kernel<GG, DD, KV_PAGED_Q8>);
#define B200Q_ATTN_CASE(GG)                  \
    if (G == GG) {                           \
        if (dig == 0) { B200Q_ATTN_KVM(GG, 0) } \
        else if (dig == 1) { B200Q_ATTN_KVM(GG, 1) } \
        else { B200Q_ATTN_KVM(GG, 2) }          \
    }
    B200Q_ATTN_CASE(1)
    B200Q_ATTN_CASE(2)
    B200Q_ATTN_CASE(4)
    B200Q_ATTN_CASE(8)
#undef B200Q_ATTN_CASE
#undef B200Q_ATTN_KVM
    return e == cudaSuccess ? B200Q_OK : B200Q_ECUDA;
}

}  // namespace

int launch_rope_attention(const float* q, const float* k, const float* v, int batch, int n_tok, int n_heads, int n_kv,
                          int hd, int pos, float theta, void* kc, void* vc, int max_ctx, float* out, void* xq,
                          int act_mode, Device* dev, cudaStream_t st, long long q_stride, long long kv_stride) {
    if (!kc || !vc || max_ctx <= 0 || n_tok <= 0) return B200Q_EINVAL;
    if (static_cast<long long>(pos) + n_tok > max_ctx) return B200Q_ESHAPE;
    if (!aligned16(kc) || !aligned16(vc)) return B200Q_EALIGN;  // key rows are read 16 bytes a lane
    KvArgs kv{};
    kv.k = kc;
    kv.v = vc;
    kv.max_ctx = max_ctx;
    return launch_attention(KV_CONTIG, kv, q, k, v, batch, n_tok, n_heads, n_kv, hd, pos, theta, out, xq, act_mode,
                            dev, st, q_stride, kv_stride);
}

int launch_rope_attention_paged(const float* q, const float* k, const float* v, int batch, int n_tok, int n_heads,
                                int n_kv, int hd, int pos, float theta, int kv_mode, void* k_pages, void* v_pages,
                                float* k_scales, float* v_scales, int n_slots, int page_size, const int* page_table,
                                int pages_per_seq, float* out, void* xq, int act_mode, Device* dev, cudaStream_t st,
                                long long q_stride, long long kv_stride) {
    const bool q8 = kv_mode == B200Q_KV_Q8;
    if ((kv_mode != B200Q_KV_F16 && !q8) || !k_pages || !v_pages || !page_table || n_slots <= 0 || page_size <= 0 ||
        pages_per_seq <= 0 || n_tok <= 0 || (q8 && (!k_scales || !v_scales)))
        return B200Q_EINVAL;
    if (static_cast<long long>(pos) + n_tok > static_cast<long long>(pages_per_seq) * page_size) return B200Q_ESHAPE;
    if (!aligned16(k_pages) || !aligned16(v_pages) ||  // key rows are read 16 bytes a lane
        (reinterpret_cast<uintptr_t>(page_table) & 3u) ||
        (q8 && ((reinterpret_cast<uintptr_t>(k_scales) & 3u) || (reinterpret_cast<uintptr_t>(v_scales) & 3u))))
        return B200Q_EALIGN;
    KvArgs kv{};
    kv.k = k_pages;
    kv.v = v_pages;
    kv.ks = k_scales;
    kv.vs = v_scales;
    kv.table = page_table;
    kv.pages_per_seq = pages_per_seq;
    kv.page = page_size;
    kv.n_slots = n_slots;
    return launch_attention(q8 ? KV_PAGED_Q8 : KV_PAGED, kv, q, k, v, batch, n_tok, n_heads, n_kv, hd, pos, theta, out,
                            xq, act_mode, dev, st, q_stride, kv_stride);
}

int launch_swiglu(const float* g, const float* u, float* out, long long n, cudaStream_t st) {
    if (!g || !u || !out || n <= 0) return B200Q_EINVAL;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_cfg(dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), st, attr);
    return cudaLaunchKernelEx(&cfg, b200q_swiglu_kernel, g, u, out, n) == cudaSuccess ? B200Q_OK : B200Q_ECUDA;
}

int launch_swiglu_rows(const float* gu, float* out, int rows, int n, cudaStream_t st) {
    if (!gu || !out || rows <= 0 || n <= 0) return B200Q_EINVAL;
    const long long total = static_cast<long long>(rows) * n;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_cfg(dim3(static_cast<unsigned>((total + 255) / 256)), dim3(256), st, attr);
    return cudaLaunchKernelEx(&cfg, b200q_swiglu_rows_kernel, gu, out, rows, n) == cudaSuccess ? B200Q_OK
                                                                                             : B200Q_ECUDA;
}

int launch_unshard_rows(const float* in, float* out, int shards, int rows, int cols, cudaStream_t st) {
    if (!in || !out || shards <= 0 || rows <= 0 || cols <= 0) return B200Q_EINVAL;
    const long long total = static_cast<long long>(shards) * rows * cols;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_cfg(dim3(static_cast<unsigned>((total + 255) / 256)), dim3(256), st, attr);
    return cudaLaunchKernelEx(&cfg, b200q_unshard_rows_kernel, in, out, shards, rows, cols) == cudaSuccess ? B200Q_OK
                                                                                                  : B200Q_ECUDA;
}

}  // namespace b200q
