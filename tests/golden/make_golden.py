"""Generate the golden fixtures of the reference's own CPU op.

    make -C oracle ref            # compiles the reference op into oracle/_ref
    python tests/golden/make_golden.py

Runs the reference engine's compiled kernels
(JSBuild/src/verso/Anvil/core/native/quantized_matmul.cpp, built from its
sources by oracle/Makefile) on seeded synthetic inputs and stores inputs and
outputs in ``tests/golden/reference_ops.npz``. The tests then pin both the
oracle restatement and the CUDA kernels against these vectors without needing
the reference tree.

Inputs: weights N(0, 0.02) packed with cybel_b200.quantize (Q4_K / Q6_K /
Q8_0), repacked by the reference's own simd_repack_* for the R4 / LM types;
activations N(0, 1). Seeds are fixed below.
"""

from __future__ import annotations

import ctypes
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from cybel_b200 import quantize as Q  # noqa: E402
from oracle import oracle as O  # noqa: E402

OUT = Path(__file__).resolve().parent / "reference_ops.npz"

CASES = [
    # (name, qtype, n, k, seed)
    ("q4k", O.Q4_K, 66, 512, 11),
    ("q6k", O.Q6_K, 37, 512, 12),
    ("q8_0", O.Q8_0, 45, 512, 13),
    ("q4k_r4", O.Q4_K_R4, 66, 512, 14),
    ("q6k_r4", O.Q6_K_R4, 37, 512, 15),
    ("q6k_lm", O.Q6_K_LM, 37, 512, 16),
]


def main() -> None:
    if not O.ref_available():
        O.build(ref=True)
    os.environ.setdefault("ANVIL_NUM_THREADS", "4")
    ref = O.ref()
    fp = ctypes.POINTER(ctypes.c_float)
    out: dict[str, np.ndarray] = {}
    for name, qt, n, k, seed in CASES:
        rng = np.random.default_rng(seed)
        w = rng.normal(0.0, 0.02, size=(n, k)).astype(np.float32)
        base = {O.Q4_K: O.Q4_K, O.Q4_K_R4: O.Q4_K, O.Q6_K: O.Q6_K, O.Q6_K_R4: O.Q6_K, O.Q6_K_LM: O.Q6_K, O.Q8_0: O.Q8_0}[qt]
        W = Q.quantize(w, base)
        if qt == O.Q4_K_R4:
            dst = np.empty_like(W)
            assert ref.simd_repack_q4k_r4(W.ctypes.data, dst.ctypes.data, k, n) == 1
            W = dst
        elif qt == O.Q6_K_R4:
            dst = np.empty_like(W)
            assert ref.simd_repack_q6k_r4(W.ctypes.data, dst.ctypes.data, k, n) == 1
            W = dst
        elif qt == O.Q6_K_LM:
            dst = np.empty((n, (k // 256) * 276), dtype=np.uint8)
            assert ref.simd_repack_q6k_lm(W.ctypes.data, dst.ctypes.data, k, n) == 1
            W = dst
        x = rng.standard_normal(k).astype(np.float32)
        y = O.ref_matvec(qt, W, x, k, n)
        out[f"{name}/W"] = W
        out[f"{name}/x"] = x
        out[f"{name}/y"] = y
        out[f"{name}/meta"] = np.array([qt, n, k], dtype=np.int64)
        if qt != O.Q6_K_LM:
            X = rng.standard_normal((3, k)).astype(np.float32)
            out[f"{name}/X"] = X
            out[f"{name}/Y"] = O.ref_matmul(qt, W, X, k, n)
        rows = [0, n // 2, n - 1]
        deq = np.zeros((len(rows), k), dtype=np.float32)
        for i, r in enumerate(rows):
            assert ref.simd_dequantize_row(W.ctypes.data, qt, r, deq[i].ctypes.data_as(fp), k) == 1
        out[f"{name}/deq_rows"] = np.array(rows, dtype=np.int64)
        out[f"{name}/deq"] = deq
    # Fused ops of the reference (quantized_matmul.cpp:1855-1896, 2307-2525).
    rng = np.random.default_rng(21)
    cols = 512
    qkv = {}
    for nm, rows in (("q", 64), ("k", 32), ("v", 32)):
        qkv[nm] = Q.quantize_q4_k(rng.normal(0.0, 0.02, size=(rows, cols)).astype(np.float32))
    x = rng.standard_normal(cols).astype(np.float32)
    outs = {nm: np.zeros(qkv[nm].shape[0], np.float32) for nm in qkv}
    ok = ref.simd_fused_qkv_matvec_quant(
        x.ctypes.data_as(fp),
        qkv["q"].ctypes.data, O.Q4_K, outs["q"].ctypes.data_as(fp), 64,
        qkv["k"].ctypes.data, O.Q4_K, outs["k"].ctypes.data_as(fp), 32,
        qkv["v"].ctypes.data, O.Q4_K, outs["v"].ctypes.data_as(fp), 32,
        cols)
    assert ok == 1
    for nm in qkv:
        out[f"qkv/{nm}/W"] = qkv[nm]
        out[f"qkv/{nm}/y"] = outs[nm]
    out["qkv/x"] = x

    in_dim, hidden, out_dim = 512, 512, 256
    experts = []
    for e in range(2):
        g = Q.quantize_q4_k(rng.normal(0.0, 0.02, size=(hidden, in_dim)).astype(np.float32))
        u = Q.quantize_q4_k(rng.normal(0.0, 0.02, size=(hidden, in_dim)).astype(np.float32))
        d = Q.quantize_q6_k(rng.normal(0.0, 0.02, size=(out_dim, hidden)).astype(np.float32))
        experts.append((g, u, d))
        out[f"ffn/e{e}/gate"], out[f"ffn/e{e}/up"], out[f"ffn/e{e}/down"] = g, u, d
    xf = rng.standard_normal(in_dim).astype(np.float32) * 4.0
    out["ffn/x"] = xf
    y0 = np.zeros(out_dim, np.float32)
    ref.simd_fused_expert_swiglu(xf.ctypes.data_as(fp), in_dim, experts[0][0].ctypes.data, O.Q4_K, hidden,
                                 experts[0][1].ctypes.data, O.Q4_K, experts[0][2].ctypes.data, O.Q6_K, out_dim,
                                 y0.ctypes.data_as(fp))
    out["ffn/expert0_y"] = y0
    idx = np.array([0, 1], dtype=np.int32)
    wts = np.array([0.625, 0.375], dtype=np.float32)
    vp = ctypes.c_void_p
    gp = (vp * 2)(experts[0][0].ctypes.data, experts[1][0].ctypes.data)
    upp = (vp * 2)(experts[0][1].ctypes.data, experts[1][1].ctypes.data)
    dp = (vp * 2)(experts[0][2].ctypes.data, experts[1][2].ctypes.data)
    ymoe = np.zeros(out_dim, np.float32)
    ref.simd_fused_moe_ffn(xf.ctypes.data_as(fp), ctypes.c_int(in_dim), idx.ctypes.data_as(ctypes.POINTER(ctypes.c_int)),
                           wts.ctypes.data_as(fp), ctypes.c_int(2), gp, ctypes.c_int(O.Q4_K), ctypes.c_int(hidden),
                           upp, ctypes.c_int(O.Q4_K), dp, ctypes.c_int(O.Q6_K), ctypes.c_int(out_dim),
                           ymoe.ctypes.data_as(fp), ctypes.c_int(0))
    out["ffn/moe_idx"], out["ffn/moe_w"], out["ffn/moe_y"] = idx, wts, ymoe
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
