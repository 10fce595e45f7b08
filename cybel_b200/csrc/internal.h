// Internal host-side interfaces shared by the .cu files of libb200q.so.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/b200q.h"

namespace b200q {

struct FmtInfo {
    int elems;            // elements per block
    int bytes;            // bytes per block
    int lanes_per_block;  // GEMV lanes sharing one block
    int blocks_per_slice; // blocks one GEMV warp covers
    int group;            // elements per integer-sum group
    bool r4;              // 4-row block-major layout
};

bool fmt_info(int qtype, FmtInfo& f);
long long row_bytes_of(int qtype, int k);

// Per-device runtime state owned by the library.
struct Device {
    int id = -1;
    int num_sms = 0;
    volatile int* status_host = nullptr;  // host view of the mapped status word
    volatile int* status = nullptr;       // device view (kernels write STATUS_* values)
};
Device* device_state(int dev, int* err);
int current_device_state(Device** out);

// Launch the decode GEMV for m activation rows (looping over row chunks).
// All pointers are device pointers. Returns a B200Q_* status.
int launch_gemv(int qtype, int act_mode, const void* w, const float* x, float* y, int m, int k, int n,
                long long x_stride, long long y_stride, int32_t* isums, Device* dev, cudaStream_t st, bool pdl,
                int flags = 0);

// Quantize m activation rows (act mode x8/x16) into scratch slot `slot`;
// returns the codes and their row pitch.
int quantize_activations(int act_mode, const float* x, long long x_stride, int m, int k, Device* dev, cudaStream_t st,
                         bool pdl, int slot, const uint8_t** xq, long long* xq_row);
// y = alpha * (W xq) + beta * y for quantized activation rows.
int gemv_from_xq(int qtype, int act_mode, const void* w, const uint8_t* xq, long long xq_row, float* y, int m, int k,
                 int n, long long y_stride, float alpha, float beta, int32_t* isums, Device* dev, cudaStream_t st,
                 bool pdl, int flags);
// The same from fp32 activation rows (x_stride floats apart, 16-byte
// aligned), quantized inside the GEMV: one launch per chunk of rows.
int gemv_from_f32(int qtype, int act_mode, const void* w, const float* x, long long x_stride, float* y, int m, int k,
                  int n, long long y_stride, float alpha, float beta, int32_t* isums, Device* dev, cudaStream_t st,
                  bool pdl, int flags);
// y = alpha * (W rmsnorm(x) * gamma) + beta * y for one fp32 row x of k, the
// RMSNorm computed inside the GEMV (B200Q_ESHAPE when the row is too long to
// stage in one pass).
int gemv_norm_f32(int qtype, int act_mode, const void* w, const float* x, const float* gamma, float eps, float* y,
                  int k, int n, float alpha, float beta, Device* dev, cudaStream_t st, bool pdl, int flags);
// y = alpha * (W (silu(gate) * up)) + beta * y for one row: the SwiGLU step
// inside the down projection's GEMV (gate and up staged and combined in
// shared memory before quantizing).
int gemv_swiglu_f32(int qtype, int act_mode, const void* w, const float* gate, const float* up, float* y, int k, int n,
                    float alpha, float beta, Device* dev, cudaStream_t st, bool pdl, int flags);
int gemv_check_shape(int qtype, int act_mode, int k, int n, Device* dev);
// The GEMV launch plan for (qtype, act_mode, k, n, mr activation rows per
// launch, fq: quantizes fp32 x itself) on num_sms SMs, as kPlanInfoFields
// values: threads, dynamic smem bytes, grid, S, WR, G, SW, R, NS,
// stage_stride, PD, x_off, staged-activation bytes, row bytes, rows per CTA.
constexpr int kPlanInfoFields = 15;
int gemv_plan_info(int qtype, int act_mode, int k, int n, int mr, bool fq, int num_sms, long long* out, int out_len);
// quantize_act kernel over `rows` contiguous rows of k into xq (row pitch xq_bytes_per_row).
int launch_quantize_rows(int act_mode, const float* x, int rows, int k, uint8_t* xq, cudaStream_t st, bool pdl);
// zero: a buffer (re)allocated by this call is zeroed in full on the stream
// (otherwise the contents of a new buffer are undefined).
int scratch_for(Device* dev, cudaStream_t st, int slot, size_t bytes, void** out, bool zero = false);
long long xq_bytes_per_row(int k, int act_mode);

int launch_repack(int dst_qtype, const void* src, void* dst, int k, int n, cudaStream_t st);
int launch_dequant_rows(int qtype, const void* w, const int* rows, int nrows, float* out, int k, int n,
                        bool tail_canonical, cudaStream_t st);
// y = W x for fp32 weights [rows][cols] (the graph's unquantized branch).
int launch_matvec_f32(const float* W, const float* x, float* y, int rows, int cols, cudaStream_t st);
int launch_swiglu_quantize(int act_mode, const float* g, const float* u, int hidden, uint8_t* xq, cudaStream_t st,
                           bool pdl);
int expert_swiglu(int act_mode, const float* x, int in_dim, const void* gate, int gq, int hidden, const void* up, int uq,
                  const void* down, int dq, int out_dim, float* out, float alpha, float beta, Device* dev,
                  cudaStream_t st, bool pdl, int flags);

// Scratch slots used by the tile path (0 = GEMV activations, 1-3 = fused FFN).
constexpr int kScratchTileX = 4;     // fp16 activation chunks
constexpr int kScratchTilePart = 5;  // split-K partial outputs
constexpr int kScratchTileB2 = 7;    // per-block sub-block sums

// Tile path (tcgen05 on fp16 operands: the exact products sc*q and the
// fp16 activations -- plus their rounding residues when `precise` --, fp32
// accumulators) for 1..tile_max_rows(precise) activation rows of a Q4_K
// matrix; x rows at stride x_stride, y rows at y_stride. Returns a B200Q_*
// status.
constexpr int kTileMaxM = 128;
int tile_max_rows(bool precise);
int launch_tile(int qtype, const void* w, const float* x, long long x_stride, float* y, int m, int k, int n,
                long long y_stride, Device* dev, cudaStream_t st, bool pdl, bool precise);
// Kernel launches one launch_tile call issues (3 or 4).
int tile_kernel_launches(int k, int n, long long y_stride, int num_sms);
// Whether launch_gemv hands (qtype, act_mode, m, flags) to the tile path:
// 0 no, 1 the fp16 variant, 2 the precise variant.
int uses_tile_path(int qtype, int act_mode, int m, int flags);

// Decode-step glue (decode.cu).
constexpr int kScratchAttn = 6;     // attention chunk partials
constexpr int kScratchAttnCnt = 8;  // fused attention arrival counters (zero between launches)
int launch_add_rmsnorm(float* res, const float* delta, const float* gamma, float* out, int n, int rows, float eps,
                       cudaStream_t st, void* xq = nullptr, int act_mode = 0);
int launch_rope_kv(float* q, float* k, const float* v, int batch, int n_heads, int n_kv, int hd, int pos, float theta,
                   void* kc, void* vc, int max_ctx, cudaStream_t st);
int launch_attention(const float* q, const void* kc, const void* vc, float* out, int batch, int n_heads, int n_kv,
                     int hd, int ctx, int max_ctx, Device* dev, cudaStream_t st, void* xq = nullptr,
                     int act_mode = 0);
// RoPE + KV append + attention + chunk merge in one launch (b200q_attn_decode_kernel)
// for n_tok consecutive tokens (positions pos .. pos + n_tok - 1) of each of
// `batch` sequences.
// q_stride / kv_stride: floats between consecutive q / k, v rows (0: packed).
int launch_rope_attention(const float* q, const float* k, const float* v, int batch, int n_tok, int n_heads, int n_kv,
                          int hd, int pos, float theta, void* kc, void* vc, int max_ctx, float* out, void* xq,
                          int act_mode, Device* dev, cudaStream_t st, long long q_stride = 0,
                          long long kv_stride = 0);
// The same over a paged cache (b200q_rope_attention_decode_paged).
int launch_rope_attention_paged(const float* q, const float* k, const float* v, int batch, int n_tok, int n_heads,
                                int n_kv, int hd, int pos, float theta, int kv_mode, void* k_pages, void* v_pages,
                                float* k_scales, float* v_scales, int n_slots, int page_size, const int* page_table,
                                int pages_per_seq, float* out, void* xq, int act_mode, Device* dev, cudaStream_t st,
                                long long q_stride = 0, long long kv_stride = 0);
int launch_swiglu(const float* g, const float* u, float* out, long long n, cudaStream_t st);
// SiLU(gate) * up for `rows` rows of [gate n | up n] (b200q_swiglu_rows).
int launch_swiglu_rows(const float* gu, float* out, int rows, int n, cudaStream_t st);
// dst[0..n) = src[0..n) from page-locked host memory mapped into the device
// (src_mapped: its device address), by a kernel that lets a PDL-launched
// GEMV behind it start streaming weights (ops.cu).
int launch_stage_host_rows(const float* src_mapped, float* dst, long long n, cudaStream_t st);
int launch_unshard_rows(const float* in, float* out, int shards, int rows, int cols, cudaStream_t st);

// Peer-memory all-gather (peer.cu).
int launch_allgather_peer(const float* local, int rows, int n_local, void* const* bases, long long data_offset,
                          long long flags_offset, int rank, int world, uint32_t* counters, int slot, Device* dev,
                          cudaStream_t st, void* xq = nullptr, int act_mode = 0);
int peer_counter_slots();
// Limit of the peer all-gather's wait for the other ranks' flags, in ns
// (ns <= 0 leaves it unchanged); returns the previous limit.
long long set_peer_wait_ns(long long ns);

// Device state if it exists already (never creates it).
Device* device_state_if_present(int dev);
// STATUS bits recorded by b200q_matvec_noalloc's kernels on `device` since
// the last read (0 when that entry point never ran there); cleared on read.
int noalloc_take_status(int device);

bool pdl_enabled();
void set_last_error(int status);

}  // namespace b200q
