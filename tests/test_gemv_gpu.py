"""Parity of the sm_100a decode GEMV with the CPU oracle and the reference op.

* integer group sums: bit-exact against the oracle's restatement
  (orc_isums) for every qtype and both activation modes;
* fp32 outputs: max |dy| / (||w_row|| * ||x||) <= 1e-5 and
  ||dy||_inf / ||y||_inf <= 1e-3 against the oracle's exact combine of the
  same integer sums (orc_matvec_q);
* x16 mode additionally against the exact fp32-activation product
  (orc_matvec_f64) and the reference op's golden outputs, same bounds;
* edge cases: ragged n (R4 tails), rows whose byte size is not a multiple of
  16, n = 1, invalid arguments (silent return like the reference).
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

NORM_TOL = 1e-5
REL_TOL = 1e-3


def _weights(O, qt: int, n: int, k: int, seed: int) -> np.ndarray:
    from cybel_b200 import quantize as Q

    rng = np.random.default_rng(seed)
    w = rng.normal(0.0, 0.02, size=(n, k)).astype(np.float32)
    base = {O.Q4_K_R4: O.Q4_K, O.Q6_K_R4: O.Q6_K, O.Q6_K_LM: O.Q6_K}.get(qt, qt)
    W = Q.quantize(w, base)
    if qt in (O.Q4_K_R4, O.Q6_K_R4):
        W = O.repack_r4(W, k, n, 144 if qt == O.Q4_K_R4 else 210)
    elif qt == O.Q6_K_LM:
        W = O.repack_q6k_lm(W, k, n)
    return W


def _check(O, W, qt, x, k, n, y, digits):
    yq = O.matvec_q(W, qt, x, k, n, digits)
    wn = O.row_norms(W, qt, k, n)
    assert O.normalized_error(y, yq, wn, x) <= NORM_TOL
    assert O.max_rel_error(y, yq) <= REL_TOL
    if digits == 2:
        exact = O.matvec_f64(W, qt, x, k, n)
        assert O.normalized_error(y, exact, wn, x) <= NORM_TOL
        assert O.max_rel_error(y, exact) <= REL_TOL


SMALL = [
    (2, 7, 256), (2, 66, 160), (2, 33, 4096),
    (8, 7, 256), (8, 45, 96), (8, 66, 1024),
    (12, 1, 256), (12, 66, 512), (12, 130, 2304),
    (14, 7, 512), (14, 37, 768), (14, 66, 2048),
    (112, 66, 512), (112, 9, 1024),
    (114, 37, 512), (114, 10, 768),
    (214, 37, 512), (214, 5, 1024),
]


@pytest.mark.parametrize("digits", [1, 2])
@pytest.mark.parametrize("qt,n,k", SMALL)
def test_gemv_isums_bitexact_and_outputs(oracle_mod, qt, n, k, digits):
    import torch
    from cybel_b200.quantized_matmul import DeviceMatrix, matmul_device, matvec_isums_device

    O = oracle_mod
    W = _weights(O, qt, n, k, seed=qt * 1000 + n + k)
    x = np.random.default_rng(n + 7 * k).standard_normal(k).astype(np.float32)
    dm = DeviceMatrix(qt, k, n, W)
    xt = torch.from_numpy(x).cuda()
    y, isums = matvec_isums_device(xt, dm, act_mode=digits)
    y2 = matmul_device(xt, dm, act_mode=digits)
    torch.cuda.synchronize()
    ref_isums = O.isums(W, qt, x, k, n, digits)
    assert np.array_equal(isums.cpu().numpy(), ref_isums)
    y = y.cpu().numpy()
    assert np.array_equal(y, y2.cpu().numpy())  # debug and production paths agree bit for bit
    _check(O, W, qt, x, k, n, y, digits)


LLAMA8B = [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336)]


@pytest.mark.parametrize("digits", [1, 2])
@pytest.mark.parametrize("qt", [12, 8])
@pytest.mark.parametrize("n,k", LLAMA8B)
def test_gemv_llama8b_shapes(oracle_mod, qt, n, k, digits):
    """The Q8_0 / Q4_K sweep shapes at full size."""
    import torch
    from cybel_b200.quantized_matmul import DeviceMatrix, matvec_isums_device

    O = oracle_mod
    W = _weights(O, qt, n, k, seed=n + k + qt)
    x = np.random.default_rng(100 + LLAMA8B.index((n, k))).standard_normal(k).astype(np.float32)
    dm = DeviceMatrix(qt, k, n, W)
    y, isums = matvec_isums_device(torch.from_numpy(x).cuda(), dm, act_mode=digits)
    torch.cuda.synchronize()
    assert np.array_equal(isums.cpu().numpy(), O.isums(W, qt, x, k, n, digits))
    _check(O, W, qt, x, k, n, y.cpu().numpy(), digits)


@pytest.mark.parametrize("digits", [1, 2])
@pytest.mark.parametrize("m", [2, 3, 5, 8])
@pytest.mark.parametrize("qt,n,k", [(12, 66, 1024), (14, 37, 512), (8, 45, 512), (2, 40, 256), (112, 66, 512), (214, 9, 512)])
def test_small_batch_matmul(oracle_mod, qt, n, k, m, digits):
    import torch
    from cybel_b200.quantized_matmul import DeviceMatrix, matmul_device

    O = oracle_mod
    W = _weights(O, qt, n, k, seed=qt + n + k + m)
    X = np.random.default_rng(m).standard_normal((m, k)).astype(np.float32)
    Y = matmul_device(torch.from_numpy(X).cuda(), DeviceMatrix(qt, k, n, W), act_mode=digits).cpu().numpy()
    if qt == 12 and digits == 1 and m >= 8:
        # x8 batches of Q4_K take the tile path (fp16 activations; tests/test_tile_gpu.py)
        ref = O.tile_matmul(W, qt, X, k, n)
        assert O.normalized_error(Y, ref, O.row_norms(W, qt, k, n), X) <= NORM_TOL
        return
    for i in range(m):
        _check(O, W, qt, X[i], k, n, Y[i], digits)


def test_dropins_match_reference_golden(oracle_mod, golden):
    """Host-pointer C drop-ins (x16 default) against the reference op's outputs."""
    from cybel_b200 import _native
    from cybel_b200 import quantized_matmul as qm

    O = oracle_mod
    L = _native.lib()
    fp = ctypes.POINTER(ctypes.c_float)
    assert qm.set_act_mode("x16") in (1, 2)
    for name in ("q4k", "q6k", "q8_0", "q4k_r4", "q6k_r4", "q6k_lm"):
        qt, n, k = (int(v) for v in golden[f"{name}/meta"])
        W, x, yref = np.ascontiguousarray(golden[f"{name}/W"]), golden[f"{name}/x"], golden[f"{name}/y"]
        y = np.zeros(n, np.float32)
        getattr(L, f"simd_matvec_{name}")(x.ctypes.data_as(fp), W.ctypes.data, y.ctypes.data_as(fp), k, n)
        assert L.b200q_last_error() == 0
        wn = O.row_norms(W, qt, k, n)
        assert O.normalized_error(y, yref, wn, x) <= NORM_TOL, name
        assert O.max_rel_error(y, yref) <= REL_TOL, name
        if f"{name}/X" in golden.files:
            X, Yref = np.ascontiguousarray(golden[f"{name}/X"]), golden[f"{name}/Y"]
            Y = np.zeros((X.shape[0], n), np.float32)
            getattr(L, f"simd_matmul_{name}")(X.ctypes.data_as(fp), W.ctypes.data, Y.ctypes.data_as(fp), X.shape[0], k, n)
            assert L.b200q_last_error() == 0
            assert O.normalized_error(Y, Yref, wn, X) <= NORM_TOL, name
        # the Python mirror (device API) agrees with the C drop-in bit for bit
        mat = qm.QuantizedMatrix(name=name, qtype=qt, shape=(k, n), data=W)
        assert np.array_equal(qm.matvec(x, mat), y), name


@pytest.mark.parametrize("m", [1, 3, 8])
@pytest.mark.parametrize("act", ["x16", "x8"])
def test_dropin_pinned_buffers_equal_pageable(oracle_mod, m, act):
    """Page-locked x and y take the zero-copy route (a staging kernel reads x
    from host memory, the GEMV stores y there; m = 8 keeps y on the DMA copy,
    the tile path): the same results, bit for bit, as pageable buffers
    through DMA copies, and (x16) within 1e-5 of the exact product."""
    import torch

    from cybel_b200 import _native
    from cybel_b200 import quantize as Q
    from cybel_b200 import quantized_matmul as qm

    O = oracle_mod
    L = _native.lib()
    fp = ctypes.POINTER(ctypes.c_float)
    n, k = 300, 2048
    W = Q.quantize(np.random.default_rng(m).normal(0.0, 0.02, size=(n, k)).astype(np.float32), 12)
    X = np.random.default_rng(10 + m).standard_normal((m, k)).astype(np.float32)
    prev = qm.set_act_mode(act)
    try:
        Yp = np.zeros((m, n), np.float32)
        xh = torch.from_numpy(X.copy()).pin_memory()
        yh = torch.zeros((m, n)).pin_memory()
        if m == 1:
            L.simd_matvec_q4k(X.ctypes.data_as(fp), W.ctypes.data, Yp.ctypes.data_as(fp), k, n)
            assert L.b200q_last_error() == 0
            L.simd_matvec_q4k(ctypes.cast(xh.data_ptr(), fp), W.ctypes.data, ctypes.cast(yh.data_ptr(), fp), k, n)
        else:
            L.simd_matmul_q4k(X.ctypes.data_as(fp), W.ctypes.data, Yp.ctypes.data_as(fp), m, k, n)
            assert L.b200q_last_error() == 0
            L.simd_matmul_q4k(ctypes.cast(xh.data_ptr(), fp), W.ctypes.data, ctypes.cast(yh.data_ptr(), fp), m, k, n)
        assert L.b200q_last_error() == 0
    finally:
        qm.set_act_mode(prev)
    assert np.array_equal(yh.numpy(), Yp)
    if act == "x16":  # (x8 is bounded against its own restatement by the tests above)
        wn = O.row_norms(W, 12, k, n)
        assert O.normalized_error(Yp, O.matvec_f64(W, 12, X, k, n), wn, X) <= NORM_TOL


def test_dropin_invalid_arguments_leave_y_untouched():
    from cybel_b200 import _native

    L = _native.lib()
    fp = ctypes.POINTER(ctypes.c_float)
    x = np.ones(300, dtype=np.float32)
    W = np.zeros(10 * 144, dtype=np.uint8)
    y = np.full(10, 7.0, dtype=np.float32)
    L.simd_matvec_q4k(x.ctypes.data_as(fp), W.ctypes.data, y.ctypes.data_as(fp), 300, 10)  # k % 256 != 0
    assert np.all(y == 7.0) and L.b200q_last_error() == -3
    L.simd_matvec_q4k(None, W.ctypes.data, y.ctypes.data_as(fp), 256, 10)
    assert np.all(y == 7.0) and L.b200q_last_error() == -1
    L.simd_matvec_q4k(x.ctypes.data_as(fp), W.ctypes.data, y.ctypes.data_as(fp), 256, 0)
    assert np.all(y == 7.0) and L.b200q_last_error() == -1


def test_device_api_rejects_misaligned_pointer():
    import torch
    from cybel_b200 import _native

    L = _native.lib()
    buf = torch.zeros(4096 + 64, dtype=torch.uint8, device="cuda")
    x = torch.zeros(256 + 4, dtype=torch.float32, device="cuda")
    y = torch.zeros(16, dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    rc = L.b200q_matmul(12, 2, x.data_ptr(), buf.data_ptr() + 4, y.data_ptr(), 1, 256, 16, st)
    assert rc == -4
    rc = L.b200q_matmul(12, 2, x.data_ptr() + 4, buf.data_ptr(), y.data_ptr(), 1, 256, 16, st)
    assert rc == -4
    rc = L.b200q_matmul(99, 2, x.data_ptr(), buf.data_ptr(), y.data_ptr(), 1, 256, 16, st)
    assert rc == -2
    assert L.b200q_device_status(torch.cuda.current_device()) == 0


def test_weight_cache_residency(oracle_mod):
    from cybel_b200 import _native

    O = oracle_mod
    L = _native.lib()
    fp = ctypes.POINTER(ctypes.c_float)
    L.b200q_weight_cache_clear()
    W = _weights(O, 12, 64, 512, seed=3)
    x = np.ones(512, dtype=np.float32)
    y1, y2, y3 = (np.zeros(64, np.float32) for _ in range(3))
    L.simd_matvec_q4k(x.ctypes.data_as(fp), W.ctypes.data, y1.ctypes.data_as(fp), 512, 64)
    assert L.b200q_weight_cache_bytes() == W.nbytes
    L.simd_matvec_q4k(x.ctypes.data_as(fp), W.ctypes.data, y2.ctypes.data_as(fp), 512, 64)
    assert np.array_equal(y1, y2) and L.b200q_weight_cache_bytes() == W.nbytes
    # Same address, different bytes (a reused buffer): re-uploaded, not stale.
    W2 = _weights(O, 12, 64, 512, seed=4)
    W[...] = W2
    L.simd_matvec_q4k(x.ctypes.data_as(fp), W.ctypes.data, y3.ctypes.data_as(fp), 512, 64)
    exact = O.matvec_f64(W2, 12, x, 512, 64)
    assert O.normalized_error(y3, exact, O.row_norms(W2, 12, 512, 64), x) <= NORM_TOL
    assert L.b200q_weight_cache_evict(W.ctypes.data) == 1
    assert L.b200q_weight_cache_bytes() == 0
