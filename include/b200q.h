/*
 * b200q.h -- C ABI of libb200q.so, the B200 (sm_100a) GGUF dequant-matvec.
 *
 * Two groups of entry points:
 *
 * 1. Drop-in replacements, with the exact names, signatures, argument
 *    meaning and error behaviour of the reference engine's CPU kernels
 *    (Team-Ferrous/Cybel, JSBuild/src/verso/Anvil/core/native/
 *    quantized_matmul.cpp, "QM" below). Pointers are HOST pointers, as in
 *    the reference: x is copied in, y copied out, and the packed weights are
 *    uploaded to HBM on first use and kept resident (keyed by host address
 *    and size; see b200q_weight_cache_*). Invalid arguments return silently
 *    without writing y (void kernels) or return 0 (int kernels), like the
 *    reference; the reason is available from b200q_last_error().
 *
 * 2. Device-pointer entry points (prefix b200q_), for callers that own
 *    device buffers (the Python layer, graph-captured decode loops). They
 *    take a cudaStream_t (as void*), are asynchronous, and return a status
 *    code (B200Q_OK = 0, negative on error).
 *
 * Activation arithmetic ("act mode"):
 *   B200Q_ACT_X16 (default)  x is quantized per 32 elements to 16-bit codes
 *                            and dotted with dp4a in two byte planes; the
 *                            result is within 1e-5 of ||w_row||*||x|| of the
 *                            reference's fp32 result.
 *   B200Q_ACT_X8             x is quantized per 32 elements to int8 (one
 *                            dp4a plane): fastest, ~5e-4 normalised error.
 *                            For Q4_K with m >= 8 activation rows
 *                            (B200Q_TILE_MIN_M) the tile path below is used.
 *   B200Q_ACT_F16            (device entry points, Q4_K only) the tile path:
 *                            tcgen05 tensor cores on fp16 operands (the
 *                            reference's fp32 dequantized weight and x, each
 *                            rounded to fp16) with fp32 accumulation; W is
 *                            streamed once per 128 activation rows; about
 *                            3e-5 normalised error against the fp32 result.
 * The drop-in entry points use the mode set by b200q_set_act_mode() or the
 * B200Q_ACT environment variable ("x16" | "x8"); default x16.
 */
#ifndef B200Q_H
#define B200Q_H

#if defined(__GNUC__)
#define B200Q_API __attribute__((visibility("default")))
#else
#define B200Q_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* qtype ids: GGUF ids (QM:39-44) plus ggml's Q4_0. */
#define B200Q_Q4_0 2
#define B200Q_Q8_0 8
#define B200Q_Q4_K 12
#define B200Q_Q6_K 14
#define B200Q_Q4_K_R4 112
#define B200Q_Q6_K_R4 114
#define B200Q_Q6_K_LM 214

#define B200Q_ACT_X8 1
#define B200Q_ACT_X16 2
#define B200Q_ACT_F16 3

/* KV storage of b200q_rope_attention_decode_paged */
#define B200Q_KV_F16 0         /* fp16 pages */
#define B200Q_KV_Q8 1          /* int8 pages + one fp32 scale per (position, kv head) */

/* status codes */
#define B200Q_OK 0
#define B200Q_EINVAL (-1)      /* null pointer, non-positive size */
#define B200Q_EQTYPE (-2)      /* unknown or unsupported qtype */
#define B200Q_ESHAPE (-3)      /* k not a multiple of the block, shape too large */
#define B200Q_EALIGN (-4)      /* device pointer not 16-byte aligned */
#define B200Q_ECUDA (-5)       /* CUDA runtime error */
#define B200Q_ENOMEM (-6)      /* device allocation failed */
#define B200Q_ETIMEOUT (-7)    /* a kernel's bounded pipeline wait gave up */
#define B200Q_ENODEV (-8)      /* no usable sm_100 device */
#define B200Q_ECAPTURE (-9)    /* scratch must grow while the stream is being captured */
#define B200Q_ESCRATCH (-10)   /* request larger than b200q_matvec_noalloc's fixed scratch */
#define B200Q_EPAGE (-11)      /* a paged cache's table named no page, or one outside its pool */

/* ---------------------------------------------------------------------
 * 1. Drop-in entry points (host pointers), reference signatures.
 * ------------------------------------------------------------------- */

/* y[n] = W x. Replace QM:1536 simd_matvec_q4k, QM:1585 simd_matvec_q4k_r4,
 * QM:1647 simd_matvec_q6k, QM:1717 simd_matvec_q6k_r4, QM:1781
 * simd_matvec_q6k_lm, QM:1818 simd_matvec_q8_0. simd_matvec_q4_0 has no
 * reference counterpart (ggml Q4_0, same argument convention). */
B200Q_API void simd_matvec_q4k(const float* x, const void* a_quant, float* y, int k, int n);
B200Q_API void simd_matvec_q4k_r4(const float* x, const void* a_quant_r4, float* y, int k, int n);
B200Q_API void simd_matvec_q6k(const float* x, const void* a_quant, float* y, int k, int n);
B200Q_API void simd_matvec_q6k_r4(const float* x, const void* a_quant_r4, float* y, int k, int n);
B200Q_API void simd_matvec_q6k_lm(const float* x, const void* a_quant_lm, float* y, int k, int n);
B200Q_API void simd_matvec_q8_0(const float* x, const void* a_quant, float* y, int k, int n);
B200Q_API void simd_matvec_q4_0(const float* x, const void* a_quant, float* y, int k, int n);

/* Y[m][n] = X[m][k] W^T. Replace QM:1944 simd_matmul_q4k, QM:1975
 * simd_matmul_q4k_r4, QM:2034 simd_matmul_q6k, QM:2065 simd_matmul_q6k_r4,
 * QM:2125 simd_matmul_q8_0 (m == 1 behaves as the matvec, QM:1953-1956).
 * simd_matmul_q4_0 has no reference counterpart. */
B200Q_API void simd_matmul_q4k(const float* x, const void* a_quant, float* y, int m, int k, int n);
B200Q_API void simd_matmul_q4k_r4(const float* x, const void* a_quant_r4, float* y, int m, int k, int n);
B200Q_API void simd_matmul_q6k(const float* x, const void* a_quant, float* y, int m, int k, int n);
B200Q_API void simd_matmul_q6k_r4(const float* x, const void* a_quant_r4, float* y, int m, int k, int n);
B200Q_API void simd_matmul_q8_0(const float* x, const void* a_quant, float* y, int m, int k, int n);
B200Q_API void simd_matmul_q4_0(const float* x, const void* a_quant, float* y, int m, int k, int n);

/* Layout repacks: QM:1573 simd_repack_q4k_r4, QM:1577 simd_repack_q6k_r4,
 * QM:1581 simd_repack_q6k_lm (layouts QM:250-365). Host pointers; run on the
 * GPU. Return 1 on success, 0 on invalid arguments. */
B200Q_API int simd_repack_q4k_r4(const void* src_q4k, void* dst_q4k_r4, int k, int n);
B200Q_API int simd_repack_q6k_r4(const void* src_q6k, void* dst_q6k_r4, int k, int n);
B200Q_API int simd_repack_q6k_lm(const void* src_q6k, void* dst_q6k_lm, int k, int n);

/* One dequantized row (embedding lookup): QM:2179 simd_dequantize_row.
 * fp32 values bit-identical to the reference. Like the reference (which has
 * no row-count argument), R4 layouts are addressed as whole 4-row groups.
 * Returns 1 on success, 0 otherwise. */
B200Q_API int simd_dequantize_row(const void* quant_data, int qtype, int row, float* out, int k);

/* Three / four matvecs sharing x, x quantized once: QM:1855
 * simd_fused_qkv_matvec_quant, QM:1898 simd_fused_quad_matvec_quant.
 * Qtypes Q4_K, Q4_K_R4, Q6_K, Q6_K_R4 (as the reference). 1 / 0. */
B200Q_API int simd_fused_qkv_matvec_quant(const float* x, const void* q_data, int q_qtype, float* q_out, int q_rows,
                                          const void* k_data, int k_qtype, float* k_out, int k_rows,
                                          const void* v_data, int v_qtype, float* v_out, int v_rows, int cols);
B200Q_API int simd_fused_quad_matvec_quant(const float* x, const void* a_data, int a_qtype, float* a_out, int a_rows,
                                           const void* b_data, int b_qtype, float* b_out, int b_rows,
                                           const void* c_data, int c_qtype, float* c_out, int c_rows,
                                           const void* d_data, int d_qtype, float* d_out, int d_rows, int cols);

/* SwiGLU expert FFN out = down(silu(gate x) * (up x)): QM:2307
 * simd_fused_expert_swiglu. Top-k MoE FFN sum_e w_e * expert_e(x) with
 * write_mode 0 = overwrite / else accumulate: QM:2426 simd_fused_moe_ffn. */
B200Q_API void simd_fused_expert_swiglu(const float* x, int in_dim, const void* gate_data, int gate_qtype,
                                        int hidden_dim, const void* up_data, int up_qtype, const void* down_data,
                                        int down_qtype, int out_dim, float* output);
B200Q_API void simd_fused_moe_ffn(const float* x, int in_dim, const int* expert_indices, const float* expert_weights,
                                  int top_k, const void* const* gate_data_ptrs, int gate_qtype, int hidden_dim,
                                  const void* const* up_data_ptrs, int up_qtype, const void* const* down_data_ptrs,
                                  int down_qtype, int out_dim, float* output, int write_mode);

/* ---------------------------------------------------------------------
 * 2. Device-pointer entry points.
 * ------------------------------------------------------------------- */

/* Y[m][n] = X[m][k] W^T with X, W, Y device pointers (16-byte aligned,
 * row strides k and n), on `stream`. Any qtype above. Replaces the
 * computation of QM:1536-2154 for callers whose buffers live in HBM. */
B200Q_API int b200q_matmul(int qtype, int act_mode, const float* x, const void* w, float* y, int m, int k, int n,
                 void* stream);

/* b200q_matmul with flags. B200Q_WEIGHTS_STATIC declares that no kernel
 * still running or queued ahead of this call on `stream` writes `w`; with
 * programmatic dependent launch (default on, see b200q_set_pdl) the kernel
 * then starts streaming weights while the preceding kernel drains, and only
 * waits for it before reading x and writing y. */
#define B200Q_WEIGHTS_STATIC 1
/* B200Q_TILE_FROM_2: Q4_K batches of 2 to 7 rows also take the tile kernel
 * (by default only 8 rows and more do; below that each launch of the GEMV
 * carries at most 2 rows in x8 and 1 in x16, so the weights stream once per
 * 1-2 rows). The batched speculative verify sets it. */
#define B200Q_TILE_FROM_2 2
B200Q_API int b200q_matmul_ex(int qtype, int act_mode, const float* x, const void* w, float* y, int m, int k, int n,
                              int flags, void* stream);

/* Debug form of b200q_matmul for m == 1: additionally writes the exact
 * per-group integer dot sums  sum_i code_i * q_i  to isums[n][k / G]
 * (G = 16 for Q6_K-family types, else 32). No reference counterpart: the
 * reference dots are fp32; this exposes the integer stage for bit-exact
 * checks against the CPU restatement. */
B200Q_API int b200q_matvec_isums(int qtype, int act_mode, const float* x, const void* w, float* y, int* isums, int k, int n,
                       void* stream);

/* The decode graph's dispatch on device pointers, with its semantics
 * (model_graph.cpp:731-760, "MG"):
 * b200q_matvec_quant replaces MG:731-747 matvec_quant: y[rows] = W x for a
 *   quantized W of `rows` rows of `cols` (argument order of MG), in the
 *   drop-in act mode; a qtype without a kernel zero-fills y and returns
 *   B200Q_OK, as MG does.
 * b200q_matvec_dispatch replaces MG:749-760 matvec_dispatch: fp32 weights
 *   [rows][cols] when w_f32 is non-NULL (MG's matvec_f32, MG:700-727),
 *   else the quantized weights when w_quant is non-NULL and qtype > 0, else
 *   a zeroed y. */
B200Q_API int b200q_matvec_quant(const void* w_quant, int qtype, const float* x, float* y, int cols, int rows,
                                 void* stream);
B200Q_API int b200q_matvec_dispatch(const float* w_f32, const void* w_quant, int qtype, const float* x, float* y,
                                    int rows, int cols, void* stream);

/* Decode matvec (m = 1) that allocates nothing, for callers that cannot
 * allocate device memory during a call: engines whose memory pool owns HBM
 * after start-up, latency-bound decode loops that cannot absorb
 * cudaMalloc/cudaFree, embedders that budget device memory up front. No
 * counterpart in the reference (its CPU kernels need no device scratch).
 * Same arguments and results as b200q_matmul with m = 1 (device pointers,
 * act mode B200Q_ACT_X8 or B200Q_ACT_X16, any qtype of the GEMV).
 * Its scratch is a fixed array of B200Q_NOALLOC_SCRATCH_BYTES in the
 * library's device image, held by every GPU that loads the library until
 * exit. The quantized activation row (2.25 k bytes in x16, 1.25 k in x8,
 * rounded up to 16) must fit in that size minus 256 bytes: k <= 28992 (x16)
 * or k <= 52224 (x8), else B200Q_ESCRATCH. The first call
 * on a device resolves the array's address (make it before any stream
 * capture). All calls share the array: calls that overlap on the GPU race.
 * A kernel wait that gives up is recorded in a status word inside the same
 * array (the call itself returns before the GPU runs it): after the call's
 * stream has finished, b200q_device_status(device) reports it (bit 1), with
 * a plain copy out of the array and no allocation. */
#define B200Q_NOALLOC_SCRATCH_BYTES (64 * 1024)
B200Q_API int b200q_matvec_noalloc(int qtype, int act_mode, const float* x, const void* w, float* y, int k, int n,
                                   void* stream);

/* Repack device buffers into dst_qtype (B200Q_Q4_K_R4 / Q6_K_R4 from the
 * canonical type, B200Q_Q6_K_LM from Q6_K). Layouts of QM:250-365. */
B200Q_API int b200q_repack(int dst_qtype, const void* src, void* dst, int k, int n, void* stream);

/* out[i][k] = dequantized row rows[i] (device int array) of a matrix with n
 * rows; the R4 tail rows are addressed canonically (QM:2179-2296 values). */
B200Q_API int b200q_dequantize_rows(int qtype, const void* w, const int* rows, int nrows, float* out, int k, int n,
                                    void* stream);

/* count matvecs y[i] = W[i] x sharing one x (quantized once); w, qtypes, y,
 * rows are host arrays of device pointers / values (QM:1855-1942). */
B200Q_API int b200q_fused_matvec(int act_mode, const float* x, int cols, int count, const void* const* w,
                                 const int* qtypes, float* const* y, const int* rows, int flags, void* stream);

/* out = alpha * down(silu(gate x) * (up x)) + beta * out on device buffers
 * (QM:2307-2416); the SiLU * up product is re-quantized for the down GEMV. */
B200Q_API int b200q_expert_swiglu(int act_mode, const float* x, int in_dim, const void* gate, int gate_qtype,
                                  int hidden, const void* up, int up_qtype, const void* down, int down_qtype,
                                  int out_dim, float* out, float alpha, float beta, int flags, void* stream);

/* Top-k MoE FFN on device buffers (QM:2426-2525); expert_indices,
 * expert_weights and the pointer arrays are host arrays. */
B200Q_API int b200q_moe_ffn(int act_mode, const float* x, int in_dim, const int* expert_indices,
                            const float* expert_weights, int top_k, const void* const* gate_ptrs, int gate_qtype,
                            int hidden, const void* const* up_ptrs, int up_qtype, const void* const* down_ptrs,
                            int down_qtype, int out_dim, float* out, int write_mode, int flags, void* stream);

/* ---------------------------------------------------------------------
 * Decode-step glue on device buffers, so a whole layer stack runs on the
 * GPU around the quantized linears (one CUDA graph per token). These
 * restate the non-matvec stages of the reference decode graph
 * (model_graph.cpp "MG"); they are internal functions there, not exports.
 * ------------------------------------------------------------------- */

/* For each of `rows` rows of n elements: residual += delta (delta may be
 * NULL), out = residual / sqrt(mean(residual^2) + eps) * gamma: MG:674-697
 * rmsnorm_inplace / rmsnorm_copy with the residual add of the previous
 * sub-layer fused in. n % 4 == 0, all pointers 16-byte aligned. */
B200Q_API int b200q_add_rmsnorm(float* residual, const float* delta, const float* gamma, float* out, int n, int rows,
                                float eps, void* stream);

/* For each of `batch` sequences at the same position pos: RoPE on
 * q [n_heads][head_dim] and k [n_kv_heads][head_dim] in place (interleaved
 * pairs, theta^(-2p/head_dim): MG:1222-1323), then k and v appended to fp16
 * caches [batch][n_kv_heads][max_ctx][head_dim] at pos. */
B200Q_API int b200q_rope_kv(float* q, float* k, const float* v, int batch, int n_heads, int n_kv_heads, int head_dim,
                            int pos, float theta, void* k_cache, void* v_cache, int max_ctx, void* stream);

/* For each of `batch` sequences: out[h] = softmax(q[h] . K[0..ctx) /
 * sqrt(head_dim)) V for one query token, query head h reading kv head
 * h / (n_heads / n_kv_heads) (GQA), over the fp16 caches above; head_dim
 * 128, at most 8 query heads per kv head. */
B200Q_API int b200q_attention_decode(const float* q, const void* k_cache, const void* v_cache, float* out, int batch,
                                     int n_heads, int n_kv_heads, int head_dim, int ctx_len, int max_ctx, void* stream);

/* out[i] = silu(gate[i]) * up[i] for n elements (the SwiGLU product of
 * QM:2380-2412, for FFNs whose gate/up and down run on different GPUs). */
B200Q_API int b200q_swiglu(const float* gate, const float* up, float* out, long long n, void* stream);

/* Quantized-activation variants: the same steps also writing their output
 * rows as the GEMV's activation codes (act_mode B200Q_ACT_X8 / X16, row pitch
 * b200q_xq_row_bytes(n, act_mode), 16-byte aligned), so the projection that
 * follows starts from codes (b200q_matmul_xq) instead of quantizing first.
 * The fp32 output pointer may be NULL. add_rmsnorm_q needs n % 128 == 0;
 * swiglu_q quantizes one row of n. */
B200Q_API long long b200q_xq_row_bytes(int k, int act_mode);
B200Q_API int b200q_add_rmsnorm_q(float* residual, const float* delta, const float* gamma, float* out, void* xq,
                                  int act_mode, int n, int rows, float eps, void* stream);
B200Q_API int b200q_attention_decode_q(const float* q, const void* k_cache, const void* v_cache, float* out, void* xq,
                                       int act_mode, int batch, int n_heads, int n_kv_heads, int head_dim, int ctx_len,
                                       int max_ctx, void* stream);

/* RoPE + KV append + attention in one launch: for each of `batch` sequences
 * at position pos, rotates q [n_heads][head_dim] and k [n_kv_heads][head_dim]
 * (as b200q_rope_kv, without writing q and k back), appends k and v to the
 * caches at pos, and attends over positions 0..pos (as
 * b200q_attention_decode with ctx_len = pos + 1). out (may be NULL when xq
 * is given) receives [batch][n_heads][head_dim]; xq (may be NULL) the codes
 * of the same rows (act_mode B200Q_ACT_X8 / X16). head_dim == 128,
 * n_heads / n_kv_heads in {1, 2, 4, 8}; q, k, v, the caches, out and xq
 * 16-byte aligned. Replaces the MG:1222-1323 RoPE and the attention after it
 * in the decode step. */
B200Q_API int b200q_rope_attention_decode(const float* q, const float* k, const float* v, int batch, int n_heads,
                                          int n_kv_heads, int head_dim, int pos, float theta, void* k_cache,
                                          void* v_cache, int max_ctx, float* out, void* xq, int act_mode,
                                          void* stream);

/* The same for n_tokens consecutive tokens of each sequence: q, k, v and the
 * outputs hold batch x n_tokens rows (sequence-major), token t of a sequence
 * sits at position pos0 + t, is appended there, and attends causally over
 * positions 0 .. pos0 + t (the cache and the tokens before it in this call).
 * One launch for the rows a speculative verify feeds through the stack at
 * once, in place of n_tokens single-token steps (the sequential verify loop
 * of cpu_speculative_decode.py:740-769). k and v 16-byte aligned;
 * pos0 + n_tokens <= max_ctx. q_stride / kv_stride: floats between
 * consecutive q / k and v rows (0: packed, n_heads * 128 / n_kv_heads * 128);
 * rows of one q|k|v projection output pass its row length for both. */
B200Q_API int b200q_rope_attention_decode_tokens(const float* q, const float* k, const float* v, int batch,
                                                 int n_tokens, int n_heads, int n_kv_heads, int head_dim, int pos0,
                                                 float theta, void* k_cache, void* v_cache, int max_ctx, float* out,
                                                 void* xq, int act_mode, long long q_stride, long long kv_stride,
                                                 void* stream);

/* The same over a paged KV cache: the reference's PagedKVStore
 * (model_graph.cpp:1413-1576: pages of page_size positions, allocated per
 * (layer, page) when a position is first written) and its attention
 * (fused_gqa_attention_decode_paged, model_graph.cpp:1686-1930). One pool of
 * n_slots pages per cache: k_pages / v_pages [n_slots][n_kv_heads][page_size]
 * [head_dim] of fp16 (kv_mode B200Q_KV_F16) or int8 codes (B200Q_KV_Q8, the
 * reference's ANVIL_KV_QUANT=q8 mode, model_graph.cpp:507-513) with
 * k_scales / v_scales [n_slots][n_kv_heads][page_size] fp32 (NULL for fp16).
 * page_table [batch][pages_per_seq] int32 gives the slot of each page of
 * each sequence, -1 for a page not allocated: a position there scores -1e9
 * and adds no value, as in the reference. The caller assigns the slot of
 * pos's page before the call. A Q8 append stores, per kv head,
 * scale = amax / 127 (1 / 127 for an all-zero row) and
 * code = clamp(round(x * (1 / scale)), -127, 127); scores are
 * dot(q, codes) * scale and values enter as softmax weight * scale * codes,
 * as the reference computes them. A slot outside [0, n_slots) in the table,
 * or no page at pos, is recorded as device status bit 2 (value 2) and the
 * position is masked. pos + n_tokens <= pages_per_seq * page_size; pools 16-byte
 * aligned. n_tokens consecutive tokens per sequence as in
 * b200q_rope_attention_decode_tokens (1 for a decode step), with its row
 * strides; the pages of pos .. pos + n_tokens - 1 assigned before the call. */
B200Q_API int b200q_rope_attention_decode_paged(const float* q, const float* k, const float* v, int batch,
                                                int n_tokens, int n_heads, int n_kv_heads, int head_dim, int pos,
                                                float theta, int kv_mode, void* k_pages, void* v_pages,
                                                float* k_scales, float* v_scales, int n_slots, int page_size,
                                                const int* page_table, int pages_per_seq, float* out, void* xq,
                                                int act_mode, long long q_stride, long long kv_stride, void* stream);
B200Q_API int b200q_swiglu_q(const float* gate, const float* up, void* xq, int act_mode, int n, void* stream);
/* out[r][j] = silu(gate_up[r][j]) * gate_up[r][n + j] for `rows` rows of one
 * gate|up projection output ([gate n | up n] per row): the SwiGLU step of a
 * multi-token pass (QM:2380-2412). */
B200Q_API int b200q_swiglu_rows(const float* gate_up, float* out, int rows, int n, void* stream);

/* y = alpha * (W x) + beta * y for m activation rows given as codes written
 * by the *_q steps above (row pitch b200q_xq_row_bytes(k, act_mode)); y rows
 * of n floats. The computation of b200q_matmul_ex without its quantizer. */
B200Q_API int b200q_matmul_xq(int qtype, int act_mode, const void* xq, const void* w, float* y, int m, int k, int n,
                              float alpha, float beta, int flags, void* stream);

/* y = alpha * (W xn) + beta * y for one fp32 row x of k, where
 * xn = x * (1 / sqrt(sum(x^2) / k + eps)) * gamma: the RMSNorm of the decode
 * graph (model_graph.cpp:674-697) and the projection that follows it
 * (matvec_dispatch, model_graph.cpp:731-790) in one GEMV launch that
 * normalizes and quantizes x while its weights stream. x and gamma 16-byte
 * aligned; act_mode B200Q_ACT_X8 or X16; k / 32 <= 32 x the GEMV's consumer
 * warps (B200Q_ESHAPE otherwise; every hidden size of the decode stacks
 * fits). */
B200Q_API int b200q_matmul_norm(int qtype, int act_mode, const float* x, const float* gamma, float eps, const void* w,
                                float* y, int k, int n, float alpha, float beta, int flags, void* stream);

/* y = alpha * (W h) + beta * y with h = silu(gate) * up, element-wise, for
 * one row of k: the SiLU * up step of the decode layer (QM:2380-2412, as
 * b200q_swiglu_q forms it) inside the down projection's GEMV, which stages
 * gate and up (written by the preceding gate/up projection) and quantizes h
 * itself. gate and up 16-byte aligned; act_mode B200Q_ACT_X8 or X16. */
B200Q_API int b200q_matmul_swiglu(int qtype, int act_mode, const float* gate, const float* up, const void* w, float* y,
                                  int k, int n, float alpha, float beta, int flags, void* stream);

/* The decode GEMV's launch plan for a matrix of n rows of k elements, without
 * touching a device (no reference counterpart: a planning query for callers
 * sizing resources and for tests). rows_per_launch: activation rows one launch
 * carries (1-4); fused_quantize: 1 when the GEMV quantizes fp32 x itself (the
 * matvec entry points), 0 when it reads codes (b200q_matmul_xq). Fills out[0..14]
 * with threads per CTA, dynamic shared memory bytes, grid, k-slices, walkers
 * per slice, walker groups, walkers per group, rows per stage, ring stages,
 * stage stride, stages issued before the activation loads, ring offset and
 * size of the staged activations, bytes per row, rows per CTA. Returns
 * B200Q_OK, B200Q_ESHAPE when no plan fits, or B200Q_EINVAL. */
B200Q_API int b200q_gemv_plan(int qtype, int act_mode, int k, int n, int rows_per_launch, int fused_quantize,
                              int num_sms, long long* out, int out_len);

/* out[r][s * cols + j] = in[s][r][j]: rows of a row-sharded output from the
 * all-gather of per-shard [rows][cols] blocks (identity for rows == 1). */
B200Q_API int b200q_unshard_rows(const float* in, float* out, int shards, int rows, int cols, void* stream);

/* ---------------------------------------------------------------------
 * Multi-GPU (one process per GPU of a node): buffers shared through CUDA
 * IPC and a one-kernel all-gather over NVLink peer memory for the outputs
 * of row-sharded linears. No reference counterpart (the reference engine
 * runs on one host and has no collectives).
 * ------------------------------------------------------------------- */

/* Allocate `bytes` of zeroed device memory shareable with other processes;
 * *handle (64 bytes, B200Q_IPC_HANDLE_BYTES) is passed to their
 * b200q_ipc_open. b200q_ipc_close unmaps a peer's buffer, b200q_ipc_free
 * frees one's own (after every peer has closed it). */
#define B200Q_IPC_HANDLE_BYTES 64
B200Q_API int b200q_ipc_alloc(long long bytes, void** dptr, void* handle);
B200Q_API int b200q_ipc_open(const void* handle, void** dptr);
B200Q_API int b200q_ipc_close(void* dptr);
B200Q_API int b200q_ipc_free(void* dptr);

/* All-gather of row-sharded outputs: this rank's rows [rows][n_local] go to
 * columns [rank * n_local, (rank + 1) * n_local) of every rank's receive area
 * [rows][world * n_local] at byte offset data_offset of its shared buffer
 * (bases: host array of the world buffers as mapped here, this rank's own
 * at index rank); each writer then release-stores a sequence number into
 * the receiver's flag row (world uint32 at flags_offset) and the call
 * returns on the device once all ranks' rows have arrived here (bounded
 * wait: on timeout the device status records it, see b200q_device_status).
 * counters: zeroed device memory of 16 uint32 per slot, private to this
 * rank; slot: which gather (its receive area, flags and counters). Every
 * rank issues the same gathers in the same order, and the consumers of a
 * slot's data run before the rank's next gather. n_local % 4 == 0.
 * With xq non-NULL the gathered rows are also written there as activation
 * codes of act_mode (row pitch b200q_xq_row_bytes(world * n_local, act_mode);
 * world * n_local % 128 == 0). */
B200Q_API int b200q_allgather_peer(const float* local, int rows, int n_local, void* const* bases,
                                   long long data_offset, long long flags_offset, int rank, int world,
                                   void* counters, int slot, void* xq, int act_mode, void* stream);

/* Activation codes of act_mode for `rows` fp32 rows of k (the quantizer the
 * GEMV entry points run before their kernel), for b200q_matmul_xq. */
B200Q_API int b200q_quantize_rows(int act_mode, const float* x, int rows, int k, void* xq, void* stream);

/* ---------------------------------------------------------------------
 * Runtime controls.
 * ------------------------------------------------------------------- */
B200Q_API int b200q_set_act_mode(int act_mode);       /* drop-in mode; returns previous */
B200Q_API int b200q_get_act_mode(void);
B200Q_API int b200q_last_error(void);                 /* last status of this host thread */
B200Q_API const char* b200q_status_string(int status);
/* STATUS bits recorded on a device since the last read, cleared on read:
 * bit 1 (value 1) = a kernel's bounded wait gave up (the call's results are
 * incomplete; B200Q_ETIMEOUT in the Python layer).
 * bit 2 (value 2) = a paged attention call met a page-table entry outside
 * its pool, or no page at the appended position (those positions were
 * masked). Covers the regular entry
 * points and b200q_matvec_noalloc; read it after the work's stream has
 * finished. Allocates nothing. */
B200Q_API int b200q_device_status(int device);
/* Longest time, in ns, that b200q_allgather_peer waits for the other ranks'
 * rows before it records a timeout and returns (default 2 s; ns <= 0 only
 * queries). Library-wide, read at each launch. Returns the previous limit. */
B200Q_API long long b200q_set_peer_wait_ns(long long ns);
B200Q_API void b200q_weight_cache_clear(void);        /* free all resident weight copies */
B200Q_API int b200q_weight_cache_evict(const void* host_ptr); /* 1 if an entry was freed */
B200Q_API long long b200q_weight_cache_bytes(void);   /* bytes resident */
B200Q_API int b200q_set_pdl(int enable);              /* programmatic dependent launch on/off; returns previous */
B200Q_API const char* b200q_version(void);

#ifdef __cplusplus
}
#endif

#endif /* B200Q_H */
