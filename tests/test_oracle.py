"""Pin the CPU oracle before trusting it (no GPU needed).

* against gguf-py 0.19.0 ``dequantize``, the ground truth of the reference's
  own tests (A/tests/test_quantized_matmul.py:179-206), bit for bit;
* against the reference op's golden vectors (tests/golden/reference_ops.npz,
  produced by the compiled reference through tests/golden/make_golden.py);
* on the reference's synthetic-Q6_K scenario (7 x 512 matrix of random
  6-bit codes, int8 scales and fp16 d; A/tests/test_quantized_matmul.py:
  94-124, 303-310), restated with this repository's own packer.
"""

from __future__ import annotations

import gguf
import numpy as np
import pytest

from cybel_b200 import quantize as Q

GGT = gguf.GGMLQuantizationType
BASE = {2: GGT.Q4_0, 8: GGT.Q8_0, 12: GGT.Q4_K, 14: GGT.Q6_K}


@pytest.mark.parametrize("qt", [2, 8, 12, 14])
@pytest.mark.parametrize("shape", [(8, 256), (33, 1024), (5, 2304)])
def test_dequant_matches_gguf_bitexact(oracle_mod, qt, shape):
    O = oracle_mod
    n, k = shape
    rng = np.random.default_rng(1000 + qt + n)
    w = rng.normal(0, 0.02, size=(n, k)).astype(np.float32)
    W = Q.quantize(w, qt)
    ref = gguf.dequantize(W, BASE[qt]).reshape(n, k)
    got = O.dequant(W, qt, k, n)
    assert np.array_equal(ref.view(np.uint32), got.view(np.uint32))


@pytest.mark.parametrize("qt", [2, 8])
def test_packers_match_gguf_quantize(qt):
    rng = np.random.default_rng(7 + qt)
    w = rng.normal(0, 0.02, size=(16, 1024)).astype(np.float32)
    w[3, :32] = 0.0  # an all-zero block
    assert np.array_equal(Q.quantize(w, qt), gguf.quantize(w, BASE[qt]))


@pytest.mark.parametrize("qt", [12, 14])
def test_k_quant_packers_roundtrip(qt):
    rng = np.random.default_rng(3 + qt)
    w = rng.normal(0, 0.02, size=(16, 2048)).astype(np.float32)
    W = Q.quantize(w, qt)
    dq = gguf.dequantize(W, BASE[qt]).reshape(w.shape)
    # 4-bit asymmetric / 6-bit symmetric codes: error well under one step.
    step = {12: 0.02 * 8 / 15, 14: 0.02 * 5 / 31}[qt]
    assert np.max(np.abs(dq - w)) < step


def test_oracle_matches_reference_golden(oracle_mod, golden):
    O = oracle_mod
    for name in ("q4k", "q6k", "q8_0", "q4k_r4", "q6k_r4", "q6k_lm"):
        qt, n, k = (int(v) for v in golden[f"{name}/meta"])
        W, x, y = golden[f"{name}/W"], golden[f"{name}/x"], golden[f"{name}/y"]
        exact = O.matvec_f64(W, qt, x, k, n)
        wn = O.row_norms(W, qt, k, n)
        assert O.normalized_error(y, exact, wn, x) < 1e-6, name
        rows = golden[f"{name}/deq_rows"]
        deq = golden[f"{name}/deq"]
        full = O.dequant(W, qt, k, n)
        for i, r in enumerate(rows):
            if qt in (O.Q4_K_R4, O.Q6_K_R4) and r >= (n // 4) * 4:
                # simd_dequantize_row has no `n` argument, so for an R4 tail
                # row (stored canonically, quantized_matmul.cpp:290-297) it
                # still applies the 4-row group addressing
                # (quantized_matmul.cpp:2214-2229) and returns other bytes.
                assert not np.array_equal(full[r], deq[i]), name
                continue
            assert np.array_equal(full[r].view(np.uint32), deq[i].view(np.uint32)), name
        if f"{name}/X" in golden.files:
            X, Y = golden[f"{name}/X"], golden[f"{name}/Y"]
            EX = O.matvec_f64(W, qt, X, k, n)
            assert O.normalized_error(Y, EX, wn, X) < 1e-6, name


def test_oracle_repacks_match_reference_golden(oracle_mod, golden):
    O = oracle_mod
    # The golden R4 / LM weights were produced by the reference's own
    # simd_repack_*; the canonical source bytes are re-derived from the packer.
    from cybel_b200 import quantize as Qz

    for name, base_name, seed in (("q4k_r4", "q4k", 14), ("q6k_r4", "q6k", 15), ("q6k_lm", "q6k", 16)):
        qt, n, k = (int(v) for v in golden[f"{name}/meta"])
        rng = np.random.default_rng(seed)
        w = rng.normal(0.0, 0.02, size=(n, k)).astype(np.float32)
        src = Qz.quantize(w, O.Q4_K if base_name == "q4k" else O.Q6_K)
        if qt == O.Q6_K_LM:
            got = O.repack_q6k_lm(src, k, n)
        else:
            got = O.repack_r4(src, k, n, 144 if qt == O.Q4_K_R4 else 210)
        assert np.array_equal(got, golden[f"{name}/W"]), name


def _pack_q6k_from_codes(codes: np.ndarray, scales: np.ndarray, d: np.float16) -> np.ndarray:
    """One Q6_K block from 256 codes in [-32, 31] (element order), 16 int8
    scales and fp16 d; layout of quantized_matmul.cpp:683-775."""
    u = (codes.astype(np.int16) + 32).astype(np.uint8).reshape(2, 4, 32)
    ql = np.zeros((2, 64), np.uint8)
    qh = np.zeros((2, 32), np.uint8)
    for gm in range(4):
        ql[:, (gm % 2) * 32:(gm % 2) * 32 + 32] |= (u[:, gm] & 0x0F) << (4 if gm >= 2 else 0)
        qh |= ((u[:, gm] >> 4) & 0x03) << (2 * gm)
    return np.concatenate([ql.reshape(-1), qh.reshape(-1), scales.astype(np.int8).view(np.uint8),
                           np.array([d], dtype=np.float16).view(np.uint8)])


def test_reference_synthetic_q6k_scenario(oracle_mod):
    O = oracle_mod
    n, k = 7, 512
    rng = np.random.default_rng(127)
    W = np.zeros((n, (k // 256) * 210), np.uint8)
    for r in range(n):
        for b in range(k // 256):
            codes = rng.integers(-32, 32, size=256).astype(np.int8)
            scales = rng.integers(-32, 32, size=16).astype(np.int8)
            d = np.float16(rng.uniform(0.02, 0.5))
            W[r, b * 210:(b + 1) * 210] = _pack_q6k_from_codes(codes, scales, d)
    x = np.random.default_rng(131).standard_normal(k).astype(np.float32)
    dense = gguf.dequantize(W, GGT.Q6_K).reshape(n, k)
    assert np.array_equal(dense.view(np.uint32), O.dequant(W, O.Q6_K, k, n).view(np.uint32))
    np.testing.assert_allclose(O.matvec_f64(W, O.Q6_K, x, k, n), dense.astype(np.float64) @ x, rtol=1e-9, atol=1e-9)


@pytest.mark.parametrize("digits", [1, 2])
def test_activation_quantizer_properties(oracle_mod, digits):
    O = oracle_mod
    rng = np.random.default_rng(5)
    x = rng.standard_normal(4096).astype(np.float32)
    x[64:96] = 0.0  # an all-zero group
    hi, lo, d, s = O.quantize_act(x, digits)
    q = hi.astype(np.int64) * (256 if digits == 2 else 1) + (lo.astype(np.int64) if digits == 2 else 0)
    qmax = 127 if digits == 1 else 32767
    assert np.all(np.abs(q) <= qmax)
    g = q.reshape(-1, 32)
    assert np.array_equal(g.sum(axis=1), s)
    assert d[2] == 0.0 and np.all(g[2] == 0)
    amax = np.abs(x.reshape(-1, 32)).max(axis=1)
    nz = amax > 0
    assert np.all(np.abs(g[nz]).max(axis=1) == qmax)
    err = np.abs(g * d[:, None] - x.reshape(-1, 32))
    assert np.all(err <= (d[:, None] * 0.5 + 1e-7 * amax[:, None]))


@pytest.mark.parametrize("qt", [2, 8, 12, 14, 112, 114, 214])
def test_integer_sums_recombine_to_q_result(oracle_mod, qt):
    """isums + scales reproduce orc_matvec_q (the two oracle paths agree)."""
    O = oracle_mod
    n, k = 9, 512
    rng = np.random.default_rng(40 + qt)
    w = rng.normal(0, 0.02, size=(n, k)).astype(np.float32)
    base = {112: 12, 114: 14, 214: 14}.get(qt, qt)
    W = Q.quantize(w, base)
    if qt in (112, 114):
        W = O.repack_r4(W, k, n, 144 if qt == 112 else 210)
    elif qt == 214:
        W = O.repack_q6k_lm(W, k, n)
    x = rng.standard_normal(k).astype(np.float32)
    for digits in (1, 2):
        yq = O.matvec_q(W, qt, x, k, n, digits)
        exact = O.matvec_f64(W, qt, x, k, n)
        wn = O.row_norms(W, qt, k, n)
        bound = 5e-3 if digits == 1 else 1e-5
        assert O.normalized_error(yq, exact, wn, x) < bound
        isums = O.isums(W, qt, x, k, n, digits)
        assert isums.shape == (n, k // O.isum_group(qt))
