"""Parity of the tcgen05 tile path (8-128 activation rows, Q4_K).

The tile kernel multiplies the exact products sc*q (fp16) by the activations
in fp16 on the tensor cores, accumulates each 256-element block in tensor
memory, and applies the block's d and dmin (the mins through a second MMA on
the sub-block sums) in fp32: the reference's weights, against fp16(x) -- or,
in the precise variant (x16 batches), fp16(x) + fp16(x - fp16(x)). Checks:

* against the oracle's restatement of exactly those activations
  (oracle.tile_matmul, fp64 accumulation of the reference's fp32 weights):
  max |dy| / (||w_row|| * ||x||) <= 1e-5 and ||dy||_inf / ||y||_inf <= 1e-3;
* against the exact product of the reference's fp32 weights and x
  (orc_matvec_f64 and the reference op's golden outputs): the fp16 rounding
  of x alone (unit roundoff 2^-11) bounds the fp16 variant's normalised error
  by TILE_VS_FP32 = 1e-4 at k >= 512 (measured 1e-5 .. 3e-5); the precise
  variant stays within 1e-5, max rel 1e-3;
* ragged n (rows past n are TMA zero-fill), m from 1 to 128 (columns padded
  to 16/32/64/128), split-K with the deterministic reduction, the full
  config shapes 14336x4096 and 4096x14336 at m = 8, 32, 128 (sampled rows
  against the oracle, all rows against the x16 GEMV), routing of x8 / x16
  batches and invalid arguments.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

NORM_TOL = 1e-5
REL_TOL = 1e-3
TILE_VS_FP32 = 1e-4

ACT_X8, ACT_X16, ACT_F16 = 1, 2, 3


def _q4k(n: int, k: int, seed: int) -> np.ndarray:
    from cybel_b200 import quantize as Q

    rng = np.random.default_rng(seed)
    return Q.quantize_q4_k(rng.normal(0.0, 0.02, size=(n, k)).astype(np.float32))


def _run(W, X, k, n, act_mode=ACT_F16):
    import torch
    from cybel_b200.quantized_matmul import DeviceMatrix, matmul_device

    dm = DeviceMatrix(12, k, n, W)
    Y = matmul_device(torch.from_numpy(X).cuda(), dm, act_mode=act_mode)
    torch.cuda.synchronize()
    return Y.cpu().numpy()


SHAPES = [
    # (n, k, m)
    (128, 256, 16),
    (130, 512, 8),
    (66, 1024, 1),
    (300, 2048, 5),
    (257, 768, 17),
    (1000, 1536, 33),
    (512, 4096, 64),
    (384, 2304, 100),
    (129, 1024, 128),
    (4096, 1024, 12),
]


@pytest.mark.parametrize("n,k,m", SHAPES)
def test_tile_matches_oracle(oracle_mod, n, k, m):
    O = oracle_mod
    W = _q4k(n, k, seed=n * 7 + k + m)
    X = np.random.default_rng(m + 3 * n).standard_normal((m, k)).astype(np.float32)
    Y = _run(W, X, k, n)
    assert Y.shape == (m, n) and np.all(np.isfinite(Y))
    wn = O.row_norms(W, 12, k, n)
    ref16 = O.tile_matmul(W, 12, X, k, n)
    assert O.normalized_error(Y, ref16, wn, X) <= NORM_TOL
    assert O.max_rel_error(Y, ref16) <= REL_TOL
    exact = O.matvec_f64(W, 12, X, k, n)
    if k >= 512:
        assert O.normalized_error(Y, exact, wn, X) <= TILE_VS_FP32
    assert O.max_rel_error(Y, exact) <= REL_TOL


@pytest.mark.parametrize("m", [8, 32, 128])
@pytest.mark.parametrize("n,k", [(14336, 4096), (4096, 14336)])
def test_tile_speculative_verify_shapes(oracle_mod, n, k, m):
    """The batched-matmul shapes: sampled row ranges against the oracle,
    every row against the x16 GEMV (an independent kernel)."""
    import torch
    from cybel_b200.quantized_matmul import DeviceMatrix, matmul_device

    O = oracle_mod
    W = _q4k(n, k, seed=n + k)
    X = np.random.default_rng(m).standard_normal((m, k)).astype(np.float32)
    dm = DeviceMatrix(12, k, n, W)
    xt = torch.from_numpy(X).cuda()
    Y = matmul_device(xt, dm, act_mode=ACT_F16).cpu().numpy()
    Y2 = matmul_device(xt, dm, act_mode=ACT_F16).cpu().numpy()
    assert np.array_equal(Y, Y2)  # deterministic (fixed split-K order)
    wn = O.row_norms(W, 12, k, n)
    for r0, r1 in ((0, 192), (n // 2 - 64, n // 2 + 64), (n - 192, n)):
        ref16 = O.tile_matmul(W, 12, X, k, n, r0, r1)
        assert O.normalized_error(Y[:, r0:r1], ref16, wn[r0:r1], X) <= NORM_TOL
        assert O.max_rel_error(Y[:, r0:r1], ref16) <= REL_TOL
    G = matmul_device(xt, dm, act_mode=ACT_X16).cpu().numpy()
    assert O.normalized_error(Y, G, wn, X) <= TILE_VS_FP32
    assert O.max_rel_error(Y, G) <= REL_TOL


def test_tile_against_reference_golden(oracle_mod, golden):
    """The reference op's own simd_matmul_q4k outputs (fp32)."""
    O = oracle_mod
    qt, n, k = (int(v) for v in golden["q4k/meta"])
    W, X, Yref = np.ascontiguousarray(golden["q4k/W"]), np.ascontiguousarray(golden["q4k/X"]), golden["q4k/Y"]
    Y = _run(W, X, k, n)
    wn = O.row_norms(W, qt, k, n)
    assert O.normalized_error(Y, Yref, wn, X) <= TILE_VS_FP32
    assert O.max_rel_error(Y, Yref) <= REL_TOL
    assert O.normalized_error(Y, O.tile_matmul(W, qt, X, k, n), wn, X) <= NORM_TOL


def test_x8_batches_route_to_tile():
    """x8 mode hands Q4_K batches of >= 8 rows to the tile kernel: identical
    bits to the explicit fp16 mode, and a strided y/x slice of 128 + rest."""
    k, n = 1024, 200
    W = _q4k(n, k, seed=5)
    X = np.random.default_rng(9).standard_normal((8, k)).astype(np.float32)
    assert np.array_equal(_run(W, X, k, n, ACT_X8), _run(W, X, k, n, ACT_F16))
    X2 = np.random.default_rng(10).standard_normal((130, k)).astype(np.float32)
    Y2 = _run(W, X2, k, n, ACT_F16)
    assert np.array_equal(Y2[128:], _run(W, X2[128:], k, n, ACT_F16))
    assert np.array_equal(Y2[:128], _run(W, X2[:128], k, n, ACT_F16))


def test_tile_invalid_arguments():
    import torch
    from cybel_b200 import _native

    L = _native.lib()
    st = torch.cuda.current_stream().cuda_stream
    w = torch.zeros(144 * 4 * 64 + 64, dtype=torch.uint8, device="cuda")
    x = torch.zeros(16 * 1024 + 8, dtype=torch.float32, device="cuda")
    y = torch.zeros(16 * 64, dtype=torch.float32, device="cuda")
    assert L.b200q_matmul(14, ACT_F16, x.data_ptr(), w.data_ptr(), y.data_ptr(), 8, 1024, 64, st) == -2
    assert L.b200q_matmul(12, ACT_F16, x.data_ptr(), w.data_ptr() + 8, y.data_ptr(), 8, 1024, 64, st) == -4
    assert L.b200q_matmul(12, ACT_F16, x.data_ptr(), w.data_ptr(), y.data_ptr(), 8, 1000, 64, st) == -3
    assert L.b200q_matmul(12, ACT_F16, x.data_ptr(), w.data_ptr(), y.data_ptr(), 0, 1024, 64, st) == -1
    torch.cuda.synchronize()
    assert L.b200q_device_status(torch.cuda.current_device()) == 0


@pytest.mark.parametrize("n,k,m", [(130, 512, 8), (300, 2048, 9), (1000, 1536, 33), (512, 4096, 64), (129, 1024, 100),
                                   (4096, 1024, 12)])
def test_precise_tile_for_x16_batches(oracle_mod, n, k, m):
    """x16 batches of >= 8 rows run the precise variant: within the x16
    accuracy of the exact fp32 product (1e-5 normalised)."""
    O = oracle_mod
    W = _q4k(n, k, seed=n + 3 * k + m)
    X = np.random.default_rng(2 * m + n).standard_normal((m, k)).astype(np.float32)
    Y = _run(W, X, k, n, ACT_X16)
    wn = O.row_norms(W, 12, k, n)
    assert O.normalized_error(Y, O.tile_matmul(W, 12, X, k, n, precise=True), wn, X) <= NORM_TOL
    exact = O.matvec_f64(W, 12, X, k, n)
    assert O.normalized_error(Y, exact, wn, X) <= NORM_TOL
    assert O.max_rel_error(Y, exact) <= REL_TOL


@pytest.mark.parametrize("act", [ACT_X16, ACT_X8])
@pytest.mark.parametrize("n,k,m", [(300, 2048, 2), (1000, 1536, 3), (4096, 1024, 5), (130, 512, 7)])
def test_tile_from_two_rows(oracle_mod, n, k, m, act):
    """B200Q_TILE_FROM_2 sends Q4_K batches of 2-7 rows to the tile kernel
    (precise variant in x16, fp16 variant in x8), as the batched speculative
    verify does: the same bounds as the >= 8-row batches."""
    import torch

    from cybel_b200 import _native

    O = oracle_mod
    W = _q4k(n, k, seed=n + k + m)
    X = np.random.default_rng(5 * m + n).standard_normal((m, k)).astype(np.float32)
    w = torch.from_numpy(W).cuda()
    x = torch.from_numpy(X).cuda()
    y = torch.empty((m, n), device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    _native.check(_native.lib().b200q_matmul_ex(12, act, x.data_ptr(), w.data_ptr(), y.data_ptr(), m, k, n,
                                                _native.TILE_FROM_2, st), "matmul_ex")
    torch.cuda.synchronize()
    Y = y.cpu().numpy()
    wn = O.row_norms(W, 12, k, n)
    precise = act == ACT_X16
    assert O.normalized_error(Y, O.tile_matmul(W, 12, X, k, n, precise=precise), wn, X) <= NORM_TOL
    exact = O.matvec_f64(W, 12, X, k, n)
    assert O.normalized_error(Y, exact, wn, X) <= (NORM_TOL if precise else TILE_VS_FP32)
    assert O.max_rel_error(Y, exact) <= REL_TOL
