"""b200q_matvec_noalloc: the matvec whose only scratch is a fixed device array.

Called through the C ABI twice in a row with different inputs (the shared
array keeps the first call's contents) and compared with b200q_matmul, the
regular device entry point, on the same inputs, and with the oracle's
restatement of the same activation mode: the same fp32 tolerances as the
GEMV tests (max |dy| / (||w_row|| * ||x||) <= 1e-5, ||dy||_inf /
||y||_inf <= 1e-3). The device status word inside the fixed array reads 0
afterwards (b200q_device_status). Oversized requests are refused with
B200Q_ESCRATCH and leave y untouched. The file runs last so that it also passes after the
other tests have used the library on the same device.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

NORM_TOL = 1e-5
REL_TOL = 1e-3
ESCRATCH = -10


def _weights(qt: int, n: int, k: int, seed: int) -> np.ndarray:
    from cybel_b200 import quantize as Q

    rng = np.random.default_rng(seed)
    return Q.quantize(rng.normal(0.0, 0.02, size=(n, k)).astype(np.float32), qt)


@pytest.mark.parametrize("qt,act,n,k", [(12, 2, 4096, 4096), (8, 1, 1024, 4096), (14, 2, 300, 2048), (12, 1, 66, 14336)])
def test_noalloc_matches_matmul_two_calls(oracle_mod, qt, act, n, k):
    import torch
    from cybel_b200 import _native

    O = oracle_mod
    L = _native.lib()
    W = _weights(qt, n, k, seed=qt + n + k)
    dw = torch.from_numpy(W.reshape(-1)).cuda()
    st = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(k + act)
    xs = [torch.from_numpy(rng.standard_normal(k).astype(np.float32)).cuda() for _ in range(2)]
    ys = [torch.full((n,), np.nan, dtype=torch.float32, device="cuda") for _ in range(2)]
    for x, y in zip(xs, ys):  # two calls in a row on the shared scratch
        assert L.b200q_matvec_noalloc(qt, act, x.data_ptr(), dw.data_ptr(), y.data_ptr(), k, n, st) == 0
    torch.cuda.synchronize()
    assert L.b200q_device_status(torch.cuda.current_device()) == 0
    wn = O.row_norms(W, qt, k, n)
    for x, y in zip(xs, ys):
        ref = torch.empty(n, dtype=torch.float32, device="cuda")
        assert L.b200q_matmul(qt, act, x.data_ptr(), dw.data_ptr(), ref.data_ptr(), 1, k, n, st) == 0
        torch.cuda.synchronize()
        yv, rv, xv = y.cpu().numpy(), ref.cpu().numpy(), x.cpu().numpy()
        assert np.all(np.isfinite(yv))
        assert O.normalized_error(yv, rv, wn, xv) <= NORM_TOL
        assert O.max_rel_error(yv, rv) <= REL_TOL
        want = O.matvec_q(W, qt, xv, k, n, act)  # the oracle in the same activation mode
        assert O.normalized_error(yv, want, wn, xv) <= NORM_TOL
        assert O.max_rel_error(yv, want) <= REL_TOL


def test_noalloc_rejects_oversized_request():
    import torch
    from cybel_b200 import _native

    L = _native.lib()
    k, n = 32768, 4  # 2.25 k = 73728 bytes of x16 codes exceed the 64 KiB scratch; 1.25 k fits
    st = torch.cuda.current_stream().cuda_stream
    w = torch.zeros((k // 256) * 144 * n, dtype=torch.uint8, device="cuda")
    x = torch.zeros(k, dtype=torch.float32, device="cuda")
    y = torch.full((n,), 7.0, dtype=torch.float32, device="cuda")
    assert L.b200q_matvec_noalloc(12, 2, x.data_ptr(), w.data_ptr(), y.data_ptr(), k, n, st) == ESCRATCH
    assert L.b200q_last_error() == ESCRATCH
    torch.cuda.synchronize()
    assert torch.all(y == 7.0)
    # the same request fits in x8 (1.25 k bytes)
    assert L.b200q_matvec_noalloc(12, 1, x.data_ptr(), w.data_ptr(), y.data_ptr(), k, n, st) == 0
    torch.cuda.synchronize()
    assert torch.all(y == 0.0)
