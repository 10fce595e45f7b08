"""The decode graph's matvec dispatch on the device (model_graph.cpp:731-760).

b200q_matvec_quant / b200q_matvec_dispatch keep the graph's semantics:
a quantized W goes to the GEMV of its qtype (drop-in act mode, x16 by
default: within 1e-5 of ||w_row|| * ||x|| of the oracle's x16
restatement); a qtype without a kernel zero-fills y and succeeds; fp32
weights take the fp32 matvec (compared with a float64 product, relative
1e-5); with neither weight y is zeroed.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _st():
    import torch

    return torch.cuda.current_stream().cuda_stream


def test_unknown_qtype_zero_fills(oracle_mod):
    import torch

    from cybel_b200 import _native

    L = _native.lib()
    rows, cols = 77, 512
    x = torch.randn(cols, device="cuda")
    w = torch.zeros(rows * cols, dtype=torch.uint8, device="cuda")
    for qt in (13, 99, 3):  # Q5_K, an unknown id, Q4_1: no kernel -> y = 0
        y = torch.full((rows,), float("nan"), device="cuda")
        assert L.b200q_matvec_quant(w.data_ptr(), qt, x.data_ptr(), y.data_ptr(), cols, rows, _st()) == 0
        torch.cuda.synchronize()
        assert torch.all(y == 0.0)
    y = torch.full((rows,), 5.0, device="cuda")
    assert L.b200q_matvec_dispatch(None, None, 12, x.data_ptr(), y.data_ptr(), rows, cols, _st()) == 0
    torch.cuda.synchronize()
    assert torch.all(y == 0.0)
    y.fill_(5.0)
    assert L.b200q_matvec_dispatch(None, w.data_ptr(), 0, x.data_ptr(), y.data_ptr(), rows, cols, _st()) == 0
    torch.cuda.synchronize()
    assert torch.all(y == 0.0)


@pytest.mark.parametrize("rows,cols", [(300, 4096), (129, 1001), (1, 8)])
def test_f32_branch(rows, cols):
    import torch

    from cybel_b200 import _native

    L = _native.lib()
    rng = np.random.default_rng(rows + cols)
    W = rng.standard_normal((rows, cols)).astype(np.float32)
    x = rng.standard_normal(cols).astype(np.float32)
    dW, dx = torch.from_numpy(W).cuda(), torch.from_numpy(x).cuda()
    y = torch.full((rows,), float("nan"), device="cuda")
    assert L.b200q_matvec_dispatch(dW.data_ptr(), None, 12, dx.data_ptr(), y.data_ptr(), rows, cols, _st()) == 0
    torch.cuda.synchronize()
    want = W.astype(np.float64) @ x.astype(np.float64)
    got = y.cpu().numpy()
    scale = np.abs(W).astype(np.float64) @ np.abs(x).astype(np.float64)
    assert np.max(np.abs(got - want) / scale) <= 1e-5


@pytest.mark.parametrize("qt", [12, 14, 8, 2])
def test_quant_branch_matches_oracle(oracle_mod, qt):
    import torch

    from cybel_b200 import _native
    from cybel_b200 import quantize as Q

    O = oracle_mod
    L = _native.lib()
    rows, cols = 260, 2048
    rng = np.random.default_rng(qt)
    W = Q.quantize(rng.normal(0.0, 0.02, size=(rows, cols)).astype(np.float32), qt)
    x = rng.standard_normal(cols).astype(np.float32)
    dW, dx = torch.from_numpy(W.reshape(-1)).cuda(), torch.from_numpy(x).cuda()
    prev = L.b200q_set_act_mode(2)
    try:
        for fn in ("quant", "dispatch"):
            y = torch.full((rows,), float("nan"), device="cuda")
            if fn == "quant":
                rc = L.b200q_matvec_quant(dW.data_ptr(), qt, dx.data_ptr(), y.data_ptr(), cols, rows, _st())
            else:
                rc = L.b200q_matvec_dispatch(None, dW.data_ptr(), qt, dx.data_ptr(), y.data_ptr(), rows, cols, _st())
            assert rc == 0
            torch.cuda.synchronize()
            got = y.cpu().numpy()
            want = O.matvec_q(W, qt, x, cols, rows, 2)
            assert O.normalized_error(got, want, O.row_norms(W, qt, cols, rows), x) <= 1e-5
    finally:
        L.b200q_set_act_mode(prev)
