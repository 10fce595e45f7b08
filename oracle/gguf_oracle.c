/*
 * gguf_oracle.c -- TEST INFRASTRUCTURE ONLY (the checker, never the product).
 *
 * A plain-C CPU restatement of the GGUF block-quantized dequant-matvec that
 * Team-Ferrous/Cybel's native engine runs for every linear layer, plus a
 * restatement of this repository's integer-activation dot product, so the
 * CUDA kernels in cybel_b200/csrc can be checked bit-exactly (integer sums)
 * and within tolerance (fp32 outputs).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * this library. The product path (libb200q.so) never links or calls it.
 *
 * Reference citations are relative to the reference project root, with
 *   QM = JSBuild/src/verso/Anvil/core/native/quantized_matmul.cpp
 *
 * Parity pins: this restatement is checked in tests/ against
 *   (1) gguf-py 0.19.0 `dequantize` (the reference's own test ground truth,
 *       A/tests/test_quantized_matmul.py:179-206), bit-exactly;
 *   (2) the reference op compiled from its sources (oracle/_ref), on the
 *       golden fixtures in tests/golden/ produced by tests/golden/make_golden.py.
 *
 * Compile with -ffp-contract=off: the activation quantizer must round exactly
 * like the GPU (IEEE division, one rounded multiply, round-half-even).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#define Q4_0 2
#define Q8_0 8
#define Q4_K 12
#define Q6_K 14
#define Q4_K_R4 112
#define Q6_K_R4 114
#define Q6_K_LM 214

/* fp16 -> fp32, exact (QM:46-78). */
float orc_fp16_to_fp32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t mant = (uint32_t)h & 0x03FFu;
    int exp = (int)((h >> 10) & 0x1Fu);
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            int e = -14;
            while ((mant & 0x0400u) == 0) { mant <<= 1; --e; }
            mant &= 0x03FFu;
            bits = sign | ((uint32_t)(e + 127) << 23) | (mant << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (mant << 13);
    } else {
        bits = sign | ((uint32_t)(exp - 15 + 127) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static uint16_t rd16(const uint8_t* p) { uint16_t v; memcpy(&v, p, 2); return v; }

/* Block specs (QW:35-42 for 8/12/14 and the R4/LM repacks; Q4_0 is ggml's). */
int orc_block_spec(int qtype, int* elems, int* bytes) {
    switch (qtype) {
        case Q4_0: *elems = 32; *bytes = 18; return 1;
        case Q8_0: *elems = 32; *bytes = 34; return 1;
        case Q4_K: case Q4_K_R4: *elems = 256; *bytes = 144; return 1;
        case Q6_K: case Q6_K_R4: *elems = 256; *bytes = 210; return 1;
        case Q6_K_LM: *elems = 256; *bytes = 276; return 1;
        default: return 0;
    }
}

/* Byte offset of (row, block) in the packed matrix. Canonical layouts are
 * row-major [n][nb][B]; the R4 layouts are [n/4][nb][4][B] with the n%4 tail
 * rows stored canonically after the full groups (QM:250-300, QM:1405-1420). */
size_t orc_block_offset(int qtype, int k, int n, int row, int blk) {
    int E, B;
    orc_block_spec(qtype, &E, &B);
    size_t nb = (size_t)(k / E);
    size_t rb = nb * (size_t)B;
    if (qtype == Q4_K_R4 || qtype == Q6_K_R4) {
        int full = n / 4;
        if (row < full * 4) {
            size_t g = (size_t)(row / 4), r = (size_t)(row % 4);
            return g * 4 * rb + ((size_t)blk * 4 + r) * (size_t)B;
        }
        return (size_t)full * 4 * rb + (size_t)(row - full * 4) * rb + (size_t)blk * B;
    }
    return (size_t)row * rb + (size_t)blk * B;
}

/* Q4_K sub-block scale/min decode (QM:423-437). */
static void q4k_scale_min(const uint8_t* s, int j, int* sc, int* mn) {
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 2) & 0x30);
        *mn = (s[j + 4] >> 4) | ((s[j] >> 2) & 0x30);
    }
}

/* Integer weight code of element e (0..E-1) in a block and the fp32 scale
 * factors that turn it into the dequantized value. For every qtype the
 * dequantized weight is  w = a * code - b  with a, b fp32 (b = 0 except Q4_K),
 * computed exactly like the reference: a = d*sc, w = a*code - dmn. */
static void block_element(int qtype, const uint8_t* blk, int e, int* code, float* a, float* b) {
    switch (qtype) {
        case Q4_0: {
            float d = orc_fp16_to_fp32(rd16(blk));
            const uint8_t* qs = blk + 2;
            int q = (e < 16) ? (qs[e] & 0x0F) : (qs[e - 16] >> 4);
            *code = q - 8; *a = d; *b = 0.0f; return;
        }
        case Q8_0: {  /* QM:1041-1081 */
            float d = orc_fp16_to_fp32(rd16(blk));
            *code = (int8_t)blk[2 + e]; *a = d; *b = 0.0f; return;
        }
        case Q4_K: case Q4_K_R4: {  /* QM:411-515 */
            float d = orc_fp16_to_fp32(rd16(blk));
            float dmin = orc_fp16_to_fp32(rd16(blk + 2));
            int j = e / 32, i = e % 32, sc, mn;
            q4k_scale_min(blk + 4, j, &sc, &mn);
            uint8_t byte = blk[16 + (j / 2) * 32 + i];
            *code = (j & 1) ? (byte >> 4) : (byte & 0x0F);
            *a = d * (float)sc; *b = dmin * (float)mn; return;
        }
        case Q6_K: case Q6_K_R4: {  /* QM:683-775 */
            int g = e / 32, i = e % 32;
            int ql_shift = ((g % 4) >= 2) ? 4 : 0;
            uint8_t qlb = blk[(g / 4) * 64 + (g % 2) * 32 + i];
            uint8_t qhb = blk[128 + (g / 4) * 32 + i];
            int q = ((qlb >> ql_shift) & 0x0F) | (((qhb >> ((g % 4) * 2)) & 0x03) << 4);
            int sidx = g * 2 + i / 16;
            float d = orc_fp16_to_fp32(rd16(blk + 208));
            *code = q - 32; *a = d * (float)(int8_t)blk[192 + sidx]; *b = 0.0f; return;
        }
        case Q6_K_LM: {  /* QM:1083-1154 */
            float d; memcpy(&d, blk + 272, 4);
            *code = (int8_t)blk[e]; *a = d * (float)(int8_t)blk[256 + e / 16]; *b = 0.0f; return;
        }
    }
    *code = 0; *a = 0.0f; *b = 0.0f;
}

/* Dequantize rows [row0, row0+count) to fp32, exactly as the reference
 * (simd_dequantize_row, QM:2179-2296): w = (a*code) - b in fp32. */
int orc_dequant_rows(const uint8_t* W, int qtype, int k, int n, int row0, int count, float* out) {
    int E, B;
    if (!orc_block_spec(qtype, &E, &B) || k <= 0 || k % E) return 0;
    int nb = k / E;
    for (int r = 0; r < count; ++r) {
        int row = row0 + r;
        for (int b = 0; b < nb; ++b) {
            const uint8_t* blk = W + orc_block_offset(qtype, k, n, row, b);
            for (int e = 0; e < E; ++e) {
                int code; float a, bb;
                block_element(qtype, blk, e, &code, &a, &bb);
                float prod = a * (float)code;
                out[(size_t)r * k + (size_t)b * E + e] = prod - bb;
            }
        }
    }
    return 1;
}

/* y[m][n] = sum_k dequant(W)[n][k] * x[m][k] accumulated in double: the
 * mathematically exact product of the reference's fp32 weights and x. */
int orc_matvec_f64(const uint8_t* W, int qtype, const float* x, int m, int k, int n, double* y) {
    int E, B;
    if (!orc_block_spec(qtype, &E, &B) || k <= 0 || k % E) return 0;
    #pragma omp parallel
    {
        float wrow[65536 + 256];
        float* wr = (k <= 65536) ? wrow : NULL;
        #pragma omp for schedule(static)
        for (int row = 0; row < n; ++row) {
            if (!wr) continue;
            orc_dequant_rows(W, qtype, k, n, row, 1, wr);
            for (int i = 0; i < m; ++i) {
                const float* xi = x + (size_t)i * k;
                double acc = 0.0;
                for (int c = 0; c < k; ++c) acc += (double)wr[c] * (double)xi[c];
                y[(size_t)i * n + row] = acc;
            }
        }
    }
    return k <= 65536;
}

/* Row norms ||w_row||_2 (double) of the dequantized weights: the tolerance
 * normaliser  |dy| / (||w_row|| * ||x||). */
int orc_row_norms(const uint8_t* W, int qtype, int k, int n, double* norms) {
    int E, B;
    if (!orc_block_spec(qtype, &E, &B) || k <= 0 || k % E || k > 65536) return 0;
    #pragma omp parallel
    {
        float wr[65536];
        #pragma omp for schedule(static)
        for (int row = 0; row < n; ++row) {
            orc_dequant_rows(W, qtype, k, n, row, 1, wr);
            double s = 0.0;
            for (int c = 0; c < k; ++c) s += (double)wr[c] * (double)wr[c];
            norms[row] = sqrt(s);
        }
    }
    return 1;
}

/* ------------------------------------------------------------------------
 * Integer-activation restatement (this repository's definition; the
 * reference has no activation quantizer, its dot products are fp32).
 *
 * Activations are quantized per 32-element group g of each row:
 *   amax  = max |x_i|
 *   QMAX  = 127 (digits = 1, "x8")  or  32767 (digits = 2, "x16")
 *   iscale = QMAX / amax           (IEEE fp32 division)
 *   q_i   = rint(x_i * iscale)     (one rounded fp32 multiply, half-even)
 *   d_g   = amax / QMAX            (IEEE fp32 division)
 *   amax == 0  ->  q = 0, d = 0.
 * q is stored as a signed high byte and an unsigned low byte
 * (q = 256*hi + lo for x16; q = hi, lo = 0 for x8), which is the operand form
 * the GPU feeds to dp4a. xsum_g = sum_i q_i.
 * ---------------------------------------------------------------------- */
int orc_quantize_act(const float* x, int k, int digits, int8_t* xhi, uint8_t* xlo, float* xd, int32_t* xsum) {
    if (k <= 0 || k % 32 || (digits != 1 && digits != 2)) return 0;
    const float qmax = (digits == 1) ? 127.0f : 32767.0f;
    for (int g = 0; g < k / 32; ++g) {
        const float* xs = x + g * 32;
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) { float a = fabsf(xs[i]); if (a > amax) amax = a; }
        int32_t s = 0;
        if (amax == 0.0f) {
            for (int i = 0; i < 32; ++i) { xhi[g * 32 + i] = 0; xlo[g * 32 + i] = 0; }
            xd[g] = 0.0f;
        } else {
            volatile float iscale = qmax / amax;
            for (int i = 0; i < 32; ++i) {
                volatile float prod = xs[i] * iscale;
                int q = (int)rintf(prod);
                s += q;
                if (digits == 1) { xhi[g * 32 + i] = (int8_t)q; xlo[g * 32 + i] = 0; }
                else { xhi[g * 32 + i] = (int8_t)(q >> 8); xlo[g * 32 + i] = (uint8_t)(q & 0xFF); }
            }
            xd[g] = amax / qmax;
        }
        xsum[g] = s;
    }
    return 1;
}

static inline int32_t xint(const int8_t* xhi, const uint8_t* xlo, int digits, size_t i) {
    return digits == 1 ? (int32_t)xhi[i] : (int32_t)xhi[i] * 256 + (int32_t)xlo[i];
}

/* Group size of the integer sums: the span of one weight scale. */
int orc_isum_group(int qtype) {
    return (qtype == Q6_K || qtype == Q6_K_R4 || qtype == Q6_K_LM) ? 16 : 32;
}

/* Per-group integer dot sums  isum[row][grp] = sum_i code_i * q_i  over the
 * group's elements, with code the signed weight integer of block_element()
 * (Q4_K: nibble 0..15, its min enters separately through xsum; Q4_0: nibble-8;
 * Q8_0: int8; Q6_K: 6-bit - 32; Q6_K_LM: int8). These must match the GPU
 * bit for bit. */
int orc_isums(const uint8_t* W, int qtype, int k, int n, const int8_t* xhi, const uint8_t* xlo,
              int digits, int32_t* isums) {
    int E, B;
    if (!orc_block_spec(qtype, &E, &B) || k <= 0 || k % E) return 0;
    const int G = orc_isum_group(qtype);
    const int ng = k / G, nb = k / E;
    #pragma omp parallel for schedule(static)
    for (int row = 0; row < n; ++row) {
        for (int b = 0; b < nb; ++b) {
            const uint8_t* blk = W + orc_block_offset(qtype, k, n, row, b);
            for (int e0 = 0; e0 < E; e0 += G) {
                int32_t s = 0;
                for (int e = e0; e < e0 + G; ++e) {
                    int code; float a, bb;
                    block_element(qtype, blk, e, &code, &a, &bb);
                    s += code * xint(xhi, xlo, digits, (size_t)b * E + e);
                }
                isums[(size_t)row * ng + (b * E + e0) / G] = s;
            }
        }
    }
    return 1;
}

/* y = sum over groups of  d_x * (a * isum - b * xsum)  in double, from the
 * exact integer sums: the value the GPU's fp32 combine approximates. */
int orc_matvec_q(const uint8_t* W, int qtype, int k, int n, const float* x, int digits, double* y) {
    int E, B;
    if (!orc_block_spec(qtype, &E, &B) || k <= 0 || k % E || k > 65536) return 0;
    int8_t xhi[65536]; uint8_t xlo[65536]; float xd[2048]; int32_t xs[2048];
    orc_quantize_act(x, k, digits, xhi, xlo, xd, xs);
    const int G = orc_isum_group(qtype), nb = k / E;
    #pragma omp parallel for schedule(static)
    for (int row = 0; row < n; ++row) {
        double acc = 0.0;
        for (int b = 0; b < nb; ++b) {
            const uint8_t* blk = W + orc_block_offset(qtype, k, n, row, b);
            for (int e0 = 0; e0 < E; e0 += G) {
                int32_t s = 0;
                int code; float a = 0.0f, bb = 0.0f;
                for (int e = e0; e < e0 + G; ++e) {
                    block_element(qtype, blk, e, &code, &a, &bb);
                    s += code * xint(xhi, xlo, digits, (size_t)b * E + e);
                }
                int g32 = (b * E + e0) / 32;
                double term = (double)a * (double)s;
                if (bb != 0.0f && (e0 % 32) == 0) term -= (double)bb * (double)xs[g32];
                acc += (double)xd[g32] * term;
            }
        }
        y[row] = acc;
    }
    return 1;
}

/* ------------------------------------------------------------------------
 * Layout repacks (QM:250-365), restated for bit-exact checks of the GPU
 * repack kernels.
 * ---------------------------------------------------------------------- */
int orc_repack_r4(const uint8_t* src, uint8_t* dst, int k, int n, int block_bytes) {
    if (!src || !dst || k <= 0 || n <= 0 || k % 256) return 0;
    size_t nb = (size_t)(k / 256), rb = nb * (size_t)block_bytes, off = 0;
    int row = 0;
    for (; row + 4 <= n; row += 4)
        for (size_t b = 0; b < nb; ++b)
            for (int r = 0; r < 4; ++r) {
                memcpy(dst + off, src + (size_t)(row + r) * rb + b * block_bytes, (size_t)block_bytes);
                off += (size_t)block_bytes;
            }
    if (row < n) memcpy(dst + off, src + (size_t)row * rb, (size_t)(n - row) * rb);
    return 1;
}

int orc_repack_q6k_lm(const uint8_t* src, uint8_t* dst, int k, int n) {
    if (!src || !dst || k <= 0 || n <= 0 || k % 256) return 0;
    int nb = k / 256;
    for (int row = 0; row < n; ++row)
        for (int b = 0; b < nb; ++b) {
            const uint8_t* blk = src + ((size_t)row * nb + b) * 210;
            uint8_t* o = dst + ((size_t)row * nb + b) * 276;
            for (int e = 0; e < 256; ++e) {
                int code; float a, bb;
                block_element(Q6_K, blk, e, &code, &a, &bb);
                o[e] = (uint8_t)(int8_t)code;
            }
            memcpy(o + 256, blk + 192, 16);
            float d = orc_fp16_to_fp32(rd16(blk + 208));
            memcpy(o + 272, &d, 4);
        }
    return 1;
}

/* SwiGLU expert FFN (QM:2307-2416) in double: out = Wd (silu(Wg x) * (Wu x)). */
int orc_fused_expert_swiglu_f64(const float* x, int in_dim, const uint8_t* gate, int gq, int hidden,
                                const uint8_t* up, int uq, const uint8_t* down, int dq, int out_dim,
                                double* out) {
    if (hidden > 65536 || in_dim > 65536) return 0;
    static double g[65536], u[65536];
    static float h[65536];
    if (!orc_matvec_f64(gate, gq, x, 1, in_dim, hidden, g)) return 0;
    if (!orc_matvec_f64(up, uq, x, 1, in_dim, hidden, u)) return 0;
    for (int i = 0; i < hidden; ++i) h[i] = (float)((g[i] / (1.0 + exp(-g[i]))) * u[i]);
    return orc_matvec_f64(down, dq, h, 1, hidden, out_dim, out);
}
