"""Parity of the repack, row-dequantization and fused-op entry points with the
reference op's golden outputs and the CPU oracle (GPU required).

* repacks (R4 / LM): bit-exact against the reference's own simd_repack_*;
* simd_dequantize_row: bit-exact fp32 against the reference and gguf-py;
* fused QKV / quad matvec: bit-identical to the separate matvecs and within
  the matvec tolerances of the reference outputs;
* fused SwiGLU expert and MoE FFN: within tolerance of the reference
  outputs and of the double-precision oracle.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

FP = ctypes.POINTER(ctypes.c_float)


def _fp(a):
    return a.ctypes.data_as(FP)


@pytest.mark.parametrize("name,src_qt,fn,block", [
    ("q4k_r4", 12, "simd_repack_q4k_r4", 144),
    ("q6k_r4", 14, "simd_repack_q6k_r4", 210),
    ("q6k_lm", 14, "simd_repack_q6k_lm", 276),
])
def test_repack_matches_reference(oracle_mod, golden, name, src_qt, fn, block):
    from cybel_b200 import _native
    from cybel_b200 import quantize as Q

    O = oracle_mod
    qt, n, k = (int(v) for v in golden[f"{name}/meta"])
    seed = {"q4k_r4": 14, "q6k_r4": 15, "q6k_lm": 16}[name]
    rng = np.random.default_rng(seed)
    src = Q.quantize(rng.normal(0.0, 0.02, size=(n, k)).astype(np.float32), src_qt)
    dst = np.zeros((n, (k // 256) * block), dtype=np.uint8)
    assert getattr(_native.lib(), fn)(src.ctypes.data, dst.ctypes.data, k, n) == 1
    assert np.array_equal(dst, golden[f"{name}/W"])
    # invalid shape: returns 0 like the reference
    assert getattr(_native.lib(), fn)(src.ctypes.data, dst.ctypes.data, k + 1, n) == 0


def test_device_repack_ragged_rows(oracle_mod):
    import torch
    from cybel_b200 import _native
    from cybel_b200 import quantize as Q

    O = oracle_mod
    for n in (1, 3, 4, 5, 130):
        k = 512
        src = Q.quantize_q4_k(np.random.default_rng(n).normal(0, 0.02, size=(n, k)).astype(np.float32))
        s_dev = torch.from_numpy(src).cuda()
        d_dev = torch.empty_like(s_dev)
        rc = _native.lib().b200q_repack(112, s_dev.data_ptr(), d_dev.data_ptr(), k, n,
                                        torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        assert np.array_equal(d_dev.cpu().numpy(), O.repack_r4(src, k, n, 144))


def test_dequantize_row_matches_reference(oracle_mod, golden):
    from cybel_b200 import _native

    O = oracle_mod
    L = _native.lib()
    for name in ("q4k", "q6k", "q8_0", "q4k_r4", "q6k_r4", "q6k_lm"):
        qt, n, k = (int(v) for v in golden[f"{name}/meta"])
        W = np.ascontiguousarray(golden[f"{name}/W"])
        for i, r in enumerate(golden[f"{name}/deq_rows"]):
            if qt in (112, 114) and r >= (n // 4) * 4:
                continue  # the reference reads past the matrix for R4 tail rows
            out = np.zeros(k, dtype=np.float32)
            assert L.simd_dequantize_row(W.ctypes.data, qt, int(r), _fp(out), k) == 1
            assert np.array_equal(out.view(np.uint32), golden[f"{name}/deq"][i].view(np.uint32)), name
    out = np.zeros(16, dtype=np.float32)
    assert L.simd_dequantize_row(None, 12, 0, _fp(out), 256) == 0
    assert L.simd_dequantize_row(W.ctypes.data, 99, 0, _fp(out), 256) == 0


@pytest.mark.parametrize("qt", [2, 8, 12, 14, 112, 114, 214])
def test_device_dequantize_rows_bitexact(oracle_mod, qt):
    import torch
    from cybel_b200 import _native
    from cybel_b200.quantized_matmul import DeviceMatrix
    from test_gemv_gpu import _weights

    O = oracle_mod
    n, k = 66, 512
    W = _weights(O, qt, n, k, seed=qt)
    dm = DeviceMatrix(qt, k, n, W)
    rows = np.array([0, 1, 31, 63, 64, 65], dtype=np.int32)
    rd = torch.from_numpy(rows).cuda()
    out = torch.empty((rows.size, k), dtype=torch.float32, device="cuda")
    rc = _native.lib().b200q_dequantize_rows(qt, dm.ptr, rd.data_ptr(), rows.size, out.data_ptr(), k, n,
                                             torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    ref = O.dequant(W, qt, k, n)[rows]
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))


def test_python_dequantize_rows_and_full(oracle_mod):
    import gguf
    from cybel_b200 import quantize as Q
    from cybel_b200.quantized_matmul import QuantizedMatrix, dequantize_full, dequantize_rows

    n, k = 7, 512
    W = Q.quantize_q6_k(np.random.default_rng(3).normal(0, 0.02, size=(n, k)).astype(np.float32))
    m = QuantizedMatrix(name="w", qtype=14, shape=(k, n), data=W)
    ref = gguf.dequantize(W, gguf.GGMLQuantizationType.Q6_K).reshape(n, k)
    assert np.array_equal(dequantize_rows(m, [0, 6, 3]), ref[[0, 6, 3]])
    assert np.array_equal(dequantize_full(m), ref)
    assert dequantize_rows(m, []).shape == (0, k)


def test_fused_qkv_matches_separate_and_reference(oracle_mod, golden):
    from cybel_b200 import _native
    from cybel_b200 import quantized_matmul as qm

    O = oracle_mod
    L = _native.lib()
    qm.set_act_mode("x16")
    x = golden["qkv/x"]
    Ws = {nm: np.ascontiguousarray(golden[f"qkv/{nm}/W"]) for nm in "qkv"}
    rows = {nm: Ws[nm].shape[0] for nm in "qkv"}
    outs = {nm: np.zeros(rows[nm], np.float32) for nm in "qkv"}
    ok = L.simd_fused_qkv_matvec_quant(
        _fp(x), Ws["q"].ctypes.data, 12, _fp(outs["q"]), rows["q"],
        Ws["k"].ctypes.data, 12, _fp(outs["k"]), rows["k"],
        Ws["v"].ctypes.data, 12, _fp(outs["v"]), rows["v"], x.size)
    assert ok == 1
    for nm in "qkv":
        sep = qm.matvec(x, qm.QuantizedMatrix(name=nm, qtype=12, shape=(x.size, rows[nm]), data=Ws[nm]))
        assert np.array_equal(sep, outs[nm])
        wn = O.row_norms(Ws[nm], 12, x.size, rows[nm])
        assert O.normalized_error(outs[nm], golden[f"qkv/{nm}/y"], wn, x) <= 1e-5
    # Q8_0 is not a fused-projection type in the reference: 0, outputs untouched
    keep = outs["q"].copy()
    ok = L.simd_fused_qkv_matvec_quant(
        _fp(x), Ws["q"].ctypes.data, 8, _fp(outs["q"]), rows["q"],
        Ws["k"].ctypes.data, 12, _fp(outs["k"]), rows["k"],
        Ws["v"].ctypes.data, 12, _fp(outs["v"]), rows["v"], x.size)
    assert ok == 0 and np.array_equal(keep, outs["q"])


def test_fused_quad_matches_separate_and_oracle(oracle_mod):
    from cybel_b200 import _native
    from cybel_b200 import quantized_matmul as qm
    from test_gemv_gpu import _weights

    O = oracle_mod
    qm.set_act_mode("x16")
    k = 512
    mats = [(_weights(O, qt, r, k, seed=r), qt, r) for qt, r in ((12, 40), (14, 24), (112, 16), (114, 12))]
    x = np.random.default_rng(9).standard_normal(k).astype(np.float32)
    outs = [np.zeros(r, np.float32) for _, _, r in mats]
    args = []
    for (W, qt, r), o in zip(mats, outs):
        args += [W.ctypes.data, qt, _fp(o), r]
    assert _native.lib().simd_fused_quad_matvec_quant(_fp(x), *args, k) == 1
    for (W, qt, r), o in zip(mats, outs):
        assert np.array_equal(o, qm.matvec(x, qm.QuantizedMatrix(name="m", qtype=qt, shape=(k, r), data=W)))
        # against the restatement of the x16 product and the exact fp32-activation product
        wn = O.row_norms(W, qt, k, r)
        for want in (O.matvec_q(W, qt, x, k, r, 2), O.matvec_f64(W, qt, x, k, r)):
            assert O.normalized_error(o, want, wn, x) <= 1e-5
            assert O.max_rel_error(o, want) <= 1e-3


def _expert_exact(O, x, g, gq, u, uq, d, dq):
    """Exact expert output and the 1e-5 bound's normaliser per output row:
    ||w_down_row|| * ||h|| with h = silu(gate x) * (up x) in float64."""
    k, hidden, out_dim = x.size, g.shape[0], d.shape[0]
    gx = O.matvec_f64(g, gq, x, k, hidden)
    ux = O.matvec_f64(u, uq, x, k, hidden)
    h = gx / (1.0 + np.exp(-gx)) * ux
    y = O.matvec_f64(d, dq, h.astype(np.float32), hidden, out_dim)
    return y, O.row_norms(d, dq, hidden, out_dim) * np.linalg.norm(h)


def _rel(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - b)) / max(np.max(np.abs(b)), 1e-30))


def test_fused_expert_swiglu_matches_reference(oracle_mod, golden):
    from cybel_b200 import quantized_matmul as qm

    O = oracle_mod
    qm.set_act_mode("x16")
    x = golden["ffn/x"]
    g, u, d = (np.ascontiguousarray(golden[f"ffn/e0/{p}"]) for p in ("gate", "up", "down"))
    hidden, out_dim = g.shape[0], d.shape[0]
    mats = (qm.QuantizedMatrix(name="g", qtype=12, shape=(x.size, hidden), data=g),
            qm.QuantizedMatrix(name="u", qtype=12, shape=(x.size, hidden), data=u),
            qm.QuantizedMatrix(name="d", qtype=14, shape=(hidden, out_dim), data=d))
    y = qm.fused_expert_swiglu(x, *mats)
    assert _rel(y, golden["ffn/expert0_y"].astype(np.float64)) <= 1e-3
    exact = np.empty(out_dim, np.float64)
    assert O.lib().orc_fused_expert_swiglu_f64(x.ctypes.data, x.size, g.ctypes.data, 12, hidden, u.ctypes.data, 12,
                                               d.ctypes.data, 14, out_dim, exact.ctypes.data) == 1
    assert _rel(y, exact) <= 1e-3
    ex, scale = _expert_exact(O, x, g, 12, u, 12, d, 14)
    assert np.max(np.abs(y - ex) / scale) <= 1e-5


def test_fused_moe_matches_reference_and_expert_sum(oracle_mod, golden):
    from cybel_b200 import quantized_matmul as qm

    qm.set_act_mode("x16")
    x = golden["ffn/x"]
    experts = []
    for e in range(2):
        g, u, d = (np.ascontiguousarray(golden[f"ffn/e{e}/{p}"]) for p in ("gate", "up", "down"))
        experts.append((qm.QuantizedMatrix(name=f"g{e}", qtype=12, shape=(x.size, g.shape[0]), data=g),
                        qm.QuantizedMatrix(name=f"u{e}", qtype=12, shape=(x.size, g.shape[0]), data=u),
                        qm.QuantizedMatrix(name=f"d{e}", qtype=14, shape=(g.shape[0], d.shape[0]), data=d)))
    w = golden["ffn/moe_w"]
    y = qm.fused_moe_ffn(x, w, [e[0] for e in experts], [e[1] for e in experts], [e[2] for e in experts])
    assert _rel(y, golden["ffn/moe_y"].astype(np.float64)) <= 1e-3
    O = oracle_mod
    exact = [_expert_exact(O, x, np.ascontiguousarray(golden[f"ffn/e{e}/gate"]), 12,
                           np.ascontiguousarray(golden[f"ffn/e{e}/up"]), 12,
                           np.ascontiguousarray(golden[f"ffn/e{e}/down"]), 14) for e in range(2)]
    want = sum(float(wi) * ex for wi, (ex, _) in zip(w, exact) if wi > 0)
    scale = sum(abs(float(wi)) * sc for wi, (_, sc) in zip(w, exact) if wi > 0)
    assert np.max(np.abs(y - want) / scale) <= 1e-5
    expected = sum(float(wi) * qm.fused_expert_swiglu(x, *e).astype(np.float64) for wi, e in zip(w, experts))
    assert _rel(y, expected) <= 1e-5
    # non-positive weights are skipped; all skipped -> zeros (write_mode 0)
    y0 = qm.fused_moe_ffn(x, [0.0, -1.0], [e[0] for e in experts], [e[1] for e in experts], [e[2] for e in experts])
    assert np.all(y0 == 0.0)


def test_moe_write_mode_accumulates(oracle_mod, golden):
    from cybel_b200 import _native
    from cybel_b200 import quantized_matmul as qm

    qm.set_act_mode("x16")
    x = golden["ffn/x"]
    g, u, d = (np.ascontiguousarray(golden[f"ffn/e0/{p}"]) for p in ("gate", "up", "down"))
    hidden, out_dim = g.shape[0], d.shape[0]
    base = np.linspace(-1, 1, out_dim).astype(np.float32)
    out = base.copy()
    idx = np.array([0], np.int32)
    w = np.array([0.5], np.float32)
    vp = ctypes.c_void_p
    _native.lib().simd_fused_moe_ffn(
        _fp(x), x.size, idx.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), _fp(w), 1,
        (vp * 1)(g.ctypes.data), 12, hidden, (vp * 1)(u.ctypes.data), 12, (vp * 1)(d.ctypes.data), 14, out_dim,
        _fp(out), 1)
    assert _native.lib().b200q_last_error() == 0
    single = qm.fused_expert_swiglu(x, qm.QuantizedMatrix(name="g", qtype=12, shape=(x.size, hidden), data=g),
                                    qm.QuantizedMatrix(name="u", qtype=12, shape=(x.size, hidden), data=u),
                                    qm.QuantizedMatrix(name="d", qtype=14, shape=(hidden, out_dim), data=d))
    assert _rel(out, base.astype(np.float64) + 0.5 * single) <= 1e-5


def test_interleaved_strict_mode(monkeypatch, golden):
    from cybel_b200 import quantized_matmul as qm

    x = golden["ffn/x"]
    g, u, d = (np.ascontiguousarray(golden[f"ffn/e0/{p}"]) for p in ("gate", "up", "down"))
    hidden, out_dim = g.shape[0], d.shape[0]
    gm = qm.QuantizedMatrix(name="g", qtype=12, shape=(x.size, hidden), data=g)
    um = qm.QuantizedMatrix(name="u", qtype=12, shape=(x.size, hidden), data=u)
    dm = qm.QuantizedMatrix(name="d", qtype=14, shape=(hidden, out_dim), data=d)
    gi = qm.interleave_quantized_rows(gm, 4)
    monkeypatch.setenv("ANVIL_STRICT_NATIVE_QSG", "1")
    with pytest.raises(RuntimeError, match="Strict native QSG"):
        qm.fused_expert_swiglu(x, gi, um, dm)
    monkeypatch.setenv("ANVIL_STRICT_NATIVE_QSG", "0")
    assert np.array_equal(qm.fused_expert_swiglu(x, gi, um, dm), qm.fused_expert_swiglu(x, gm, um, dm))


@pytest.mark.parametrize("qt,n,k", [(12, 300, 4096), (14, 200, 4096), (12, 128, 8192), (8, 96, 2048)])
@pytest.mark.parametrize("act,tol", [(2, 1e-5), (1, 1e-3)])
def test_matmul_norm_matches_exact(oracle_mod, qt, n, k, act, tol):
    """b200q_matmul_norm: RMSNorm(x) * gamma computed inside the GEMV, against
    the double-precision product of the oracle's dequantized rows with the
    norm restated in float64: x16 within the 1e-5 matvec bound; x8 within its
    int8 activation quantization error (1e-3 of ||w_row|| * ||xn|| for these
    inputs) and within 3e-5 of the separate GEMV given the same normalized x."""
    import torch

    from cybel_b200 import _native
    from cybel_b200 import quantize as Q
    from cybel_b200.quantized_matmul import DeviceMatrix

    O = oracle_mod
    rng = np.random.default_rng(qt + n + k + act)
    W = Q.quantize(rng.normal(0.0, 0.02, size=(n, k)).astype(np.float32), qt)
    x = (rng.standard_normal(k) * 3.0).astype(np.float32)
    gamma = rng.uniform(0.5, 1.5, size=k).astype(np.float32)
    eps = 1e-5
    xd = x.astype(np.float64)
    xn = (xd / np.sqrt(np.mean(xd * xd) + eps) * gamma).astype(np.float32)
    exact = O.matvec_f64(W, qt, xn, k, n)
    dm = DeviceMatrix(qt, k, n, W)
    xt, gt = torch.from_numpy(x).cuda(), torch.from_numpy(gamma).cuda()
    L = _native.lib()
    st = torch.cuda.current_stream().cuda_stream
    y = torch.full((n,), 0.5, dtype=torch.float32, device="cuda")
    _native.check(L.b200q_matmul_norm(qt, act, xt.data_ptr(), gt.data_ptr(), eps, dm.ptr, y.data_ptr(), k, n, 1.0, 0.0,
                                      _native.WEIGHTS_STATIC, st), "matmul_norm")
    yy = y.cpu().numpy()
    wn = O.row_norms(W, qt, k, n)
    assert O.normalized_error(yy, exact, wn, xn) <= tol
    if act == 1:
        from cybel_b200.quantized_matmul import matmul_device

        y_sep = matmul_device(torch.from_numpy(xn).cuda(), dm, act_mode=act).cpu().numpy()
        assert O.normalized_error(yy, y_sep, wn, xn) <= 3e-5
    # beta = 1 accumulates onto y (the residual form of the decode step)
    y2 = torch.full((n,), 0.5, dtype=torch.float32, device="cuda")
    _native.check(L.b200q_matmul_norm(qt, act, xt.data_ptr(), gt.data_ptr(), eps, dm.ptr, y2.data_ptr(), k, n, 1.0,
                                      1.0, _native.WEIGHTS_STATIC, st), "matmul_norm beta")
    assert O.normalized_error(y2.cpu().numpy() - 0.5, exact, wn, xn) <= tol


def test_matmul_norm_rejects_long_rows(oracle_mod):
    """A row too long to stage in one pass is refused (B200Q_ESHAPE), not computed."""
    import torch

    from cybel_b200 import _native
    from cybel_b200 import quantize as Q
    from cybel_b200.quantized_matmul import DeviceMatrix

    k, n = 28672, 8
    W = Q.quantize(np.random.default_rng(3).normal(0.0, 0.02, size=(n, k)).astype(np.float32), 12)
    dm = DeviceMatrix(12, k, n, W)
    x = torch.ones(k, device="cuda")
    y = torch.zeros(n, device="cuda")
    rc = _native.lib().b200q_matmul_norm(12, 1, x.data_ptr(), x.data_ptr(), 1e-5, dm.ptr, y.data_ptr(), k, n, 1.0, 0.0,
                                         _native.WEIGHTS_STATIC, torch.cuda.current_stream().cuda_stream)
    assert rc == -3


@pytest.mark.parametrize("qt,n,k", [(12, 4096, 14336), (12, 300, 768), (14, 256, 2048), (8, 96, 4096)])
@pytest.mark.parametrize("act", [2, 1])
def test_matmul_swiglu_equals_swiglu_then_gemv(oracle_mod, qt, n, k, act):
    """b200q_matmul_swiglu (SiLU(gate) * up formed and quantized inside the
    down projection's GEMV) against the two-launch form it replaces,
    b200q_swiglu_q + b200q_matmul_xq: the same codes, so the same outputs bit
    for bit, with and without the residual (beta = 1); and (x16) within 1e-5
    of the exact product with the float64 SwiGLU vector."""
    import torch

    from cybel_b200 import _native
    from cybel_b200 import quantize as Q
    from cybel_b200.quantized_matmul import DeviceMatrix

    O = oracle_mod
    rng = np.random.default_rng(qt + n + k + act)
    W = Q.quantize(rng.normal(0.0, 0.02, size=(n, k)).astype(np.float32), qt)
    g = (rng.standard_normal(k) * 2.0).astype(np.float32)
    u = rng.standard_normal(k).astype(np.float32)
    dm = DeviceMatrix(qt, k, n, W)
    gt, ut = torch.from_numpy(g).cuda(), torch.from_numpy(u).cuda()
    L = _native.lib()
    st = torch.cuda.current_stream().cuda_stream
    W_ = _native.WEIGHTS_STATIC
    for beta in (0.0, 1.0):
        y1 = torch.full((n,), 0.25, dtype=torch.float32, device="cuda")
        y2 = y1.clone()
        _native.check(L.b200q_matmul_swiglu(qt, act, gt.data_ptr(), ut.data_ptr(), dm.ptr, y1.data_ptr(), k, n, 1.0,
                                            beta, W_, st), "matmul_swiglu")
        xq = torch.zeros(int(L.b200q_xq_row_bytes(k, act)), dtype=torch.uint8, device="cuda")
        _native.check(L.b200q_swiglu_q(gt.data_ptr(), ut.data_ptr(), xq.data_ptr(), act, k, st), "swiglu_q")
        _native.check(L.b200q_matmul_xq(qt, act, xq.data_ptr(), dm.ptr, y2.data_ptr(), 1, k, n, 1.0, beta, W_, st),
                      "matmul_xq")
        torch.cuda.synchronize()
        assert np.array_equal(y1.cpu().numpy(), y2.cpu().numpy()), beta
    if act == 2:
        gd = g.astype(np.float64)
        h = (gd / (1.0 + np.exp(-gd)) * u).astype(np.float32)
        wn = O.row_norms(W, qt, k, n)
        assert O.normalized_error(y1.cpu().numpy() - 0.25, O.matvec_f64(W, qt, h, k, n), wn, h) <= 1e-5
