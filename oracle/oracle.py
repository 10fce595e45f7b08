"""ctypes front end of the CPU checkers -- TEST INFRASTRUCTURE ONLY.

Loads two libraries built by ``oracle/Makefile``:

* ``_build/liboracle.so`` -- this repository's C restatement of the GGUF
  dequant-matvec (``gguf_oracle.c``) and of the integer-activation dot
  product the CUDA kernels implement;
* ``_ref/libref_qm.so`` -- the reference's own CPU op
  (JSBuild/src/verso/Anvil/core/native/quantized_matmul.cpp), compiled from
  its sources. Optional: it exists only where it was built.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` import this module, as the checker. The product
(``cybel_b200``) never does.

Parity pin: the restatement is checked against gguf-py ``dequantize``
(bit-exact) and against ``libref_qm.so`` through the committed golden
fixtures in ``tests/golden/``.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "liboracle.so"
REF_SO = HERE / "_ref" / "libref_qm.so"

Q4_0, Q8_0, Q4_K, Q6_K = 2, 8, 12, 14
Q4_K_R4, Q6_K_R4, Q6_K_LM = 112, 114, 214

BLOCK_SPECS = {
    Q4_0: (32, 18),
    Q8_0: (32, 34),
    Q4_K: (256, 144),
    Q6_K: (256, 210),
    Q4_K_R4: (256, 144),
    Q6_K_R4: (256, 210),
    Q6_K_LM: (256, 276),
}

_lib = None
_ref = None

_vp = ctypes.c_void_p
_i = ctypes.c_int


def reference_root() -> Path | None:
    """The reference checkout the recipe compiles from: $CYBEL_REF_ROOT, else a
    ``reference`` directory beside this repository; None when neither exists."""
    env = os.environ.get("CYBEL_REF_ROOT")
    cand = Path(env) if env else HERE.parent.parent / "reference"
    return cand if (cand / "JSBuild").is_dir() else None


def build(ref: bool = False) -> None:
    """Compile the restatement (and, when asked and the reference tree is
    present, the reference op from its sources)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    root = reference_root() if ref else None
    if root is not None:
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REF_ROOT={root}"], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not ORACLE_SO.exists():
            build()
        L = ctypes.CDLL(str(ORACLE_SO))
        L.orc_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        L.orc_fp16_to_fp32.restype = ctypes.c_float
        for name, args in {
            "orc_dequant_rows": [_vp, _i, _i, _i, _i, _i, _vp],
            "orc_matvec_f64": [_vp, _i, _vp, _i, _i, _i, _vp],
            "orc_row_norms": [_vp, _i, _i, _i, _vp],
            "orc_quantize_act": [_vp, _i, _i, _vp, _vp, _vp, _vp],
            "orc_isums": [_vp, _i, _i, _i, _vp, _vp, _i, _vp],
            "orc_matvec_q": [_vp, _i, _i, _i, _vp, _i, _vp],
            "orc_repack_r4": [_vp, _vp, _i, _i, _i],
            "orc_repack_q6k_lm": [_vp, _vp, _i, _i],
            "orc_isum_group": [_i],
            "orc_fused_expert_swiglu_f64": [_vp, _i, _vp, _i, _i, _vp, _i, _vp, _i, _i, _vp],
        }.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = _i
        _lib = L
    return _lib


def ref_available() -> bool:
    return REF_SO.exists()


def ref() -> ctypes.CDLL:
    """The reference's compiled CPU op (raises if it was not built here)."""
    global _ref
    if _ref is None:
        if not REF_SO.exists():
            raise FileNotFoundError(f"reference op not built: {REF_SO}")
        L = ctypes.CDLL(str(REF_SO))
        fp = ctypes.POINTER(ctypes.c_float)
        for q in ("q4k", "q4k_r4", "q6k", "q6k_r4", "q6k_lm", "q8_0"):
            fn = getattr(L, f"simd_matvec_{q}")
            fn.argtypes = [fp, _vp, fp, _i, _i]
            fn.restype = None
        for q in ("q4k", "q4k_r4", "q6k", "q6k_r4", "q8_0"):
            fn = getattr(L, f"simd_matmul_{q}")
            fn.argtypes = [fp, _vp, fp, _i, _i, _i]
            fn.restype = None
        for q in ("q4k_r4", "q6k_r4", "q6k_lm"):
            fn = getattr(L, f"simd_repack_{q}")
            fn.argtypes = [_vp, _vp, _i, _i]
            fn.restype = _i
        L.simd_dequantize_row.argtypes = [_vp, _i, _i, fp, _i]
        L.simd_dequantize_row.restype = _i
        L.simd_fused_expert_swiglu.argtypes = [fp, _i, _vp, _i, _i, _vp, _i, _vp, _i, _i, fp]
        L.simd_fused_expert_swiglu.restype = None
        L.simd_fused_qkv_matvec_quant.argtypes = [fp, _vp, _i, fp, _i, _vp, _i, fp, _i, _vp, _i, fp, _i, _i]
        L.simd_fused_qkv_matvec_quant.restype = _i
        vpp = ctypes.POINTER(ctypes.c_void_p)
        L.simd_fused_moe_ffn.argtypes = [fp, _i, ctypes.POINTER(ctypes.c_int), fp, _i, vpp, _i, _i, vpp, _i, vpp, _i,
                                         _i, fp, _i]
        L.simd_fused_moe_ffn.restype = None
        _ref = L
    return _ref


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def row_bytes(qtype: int, k: int) -> int:
    e, b = BLOCK_SPECS[qtype]
    return (k // e) * b


def dequant(W: np.ndarray, qtype: int, k: int, n: int) -> np.ndarray:
    W = np.ascontiguousarray(W, dtype=np.uint8)
    out = np.empty((n, k), dtype=np.float32)
    assert lib().orc_dequant_rows(_p(W), qtype, k, n, 0, n, _p(out)) == 1
    return out


def matvec_f64(W: np.ndarray, qtype: int, x: np.ndarray, k: int, n: int) -> np.ndarray:
    """Exact (double-accumulated) y = X @ dequant(W).T, X of shape [m, k] or [k]."""
    W = np.ascontiguousarray(W, dtype=np.uint8)
    xx = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    m = xx.shape[0]
    y = np.empty((m, n), dtype=np.float64)
    assert lib().orc_matvec_f64(_p(W), qtype, _p(xx), m, k, n, _p(y)) == 1
    return y if np.ndim(x) == 2 else y[0]


def row_norms(W: np.ndarray, qtype: int, k: int, n: int) -> np.ndarray:
    W = np.ascontiguousarray(W, dtype=np.uint8)
    out = np.empty((n,), dtype=np.float64)
    assert lib().orc_row_norms(_p(W), qtype, k, n, _p(out)) == 1
    return out


def quantize_act(x: np.ndarray, digits: int):
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    k = x.shape[0]
    hi = np.empty(k, dtype=np.int8)
    lo = np.empty(k, dtype=np.uint8)
    d = np.empty(k // 32, dtype=np.float32)
    s = np.empty(k // 32, dtype=np.int32)
    assert lib().orc_quantize_act(_p(x), k, digits, _p(hi), _p(lo), _p(d), _p(s)) == 1
    return hi, lo, d, s


def isum_group(qtype: int) -> int:
    return int(lib().orc_isum_group(qtype))


def isums(W: np.ndarray, qtype: int, x: np.ndarray, k: int, n: int, digits: int) -> np.ndarray:
    hi, lo, _, _ = quantize_act(x, digits)
    W = np.ascontiguousarray(W, dtype=np.uint8)
    g = isum_group(qtype)
    out = np.empty((n, k // g), dtype=np.int32)
    assert lib().orc_isums(_p(W), qtype, k, n, _p(hi), _p(lo), digits, _p(out)) == 1
    return out


def matvec_q(W: np.ndarray, qtype: int, x: np.ndarray, k: int, n: int, digits: int) -> np.ndarray:
    W = np.ascontiguousarray(W, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    y = np.empty((n,), dtype=np.float64)
    assert lib().orc_matvec_q(_p(W), qtype, k, n, _p(x), digits, _p(y)) == 1
    return y


def repack_r4(W: np.ndarray, k: int, n: int, block_bytes: int) -> np.ndarray:
    W = np.ascontiguousarray(W, dtype=np.uint8)
    dst = np.empty_like(W)
    assert lib().orc_repack_r4(_p(W), _p(dst), k, n, block_bytes) == 1
    return dst


def repack_q6k_lm(W: np.ndarray, k: int, n: int) -> np.ndarray:
    W = np.ascontiguousarray(W, dtype=np.uint8)
    dst = np.empty((n, (k // 256) * 276), dtype=np.uint8)
    assert lib().orc_repack_q6k_lm(_p(W), _p(dst), k, n) == 1
    return dst


def tile_matmul(W: np.ndarray, qtype: int, X: np.ndarray, k: int, n: int, r0: int = 0, r1: int | None = None,
                precise: bool = False):
    """Restatement of the tile path: Y[m][r] for weight rows [r0, r1) =
    sum_i w[r][i] * xe[m][i], accumulated exactly (fp64), where w is the
    reference's fp32 dequantized weight (orc_dequant_rows, which follows
    quantized_matmul.cpp:1323-1375 bit for bit) and xe the activations the
    tensor cores see: fp16(x) (IEEE binary16, round to nearest even, as
    numpy's float32 -> float16 conversion), plus fp16(x - fp16(x)) when
    `precise`. (The kernel multiplies the exact products sc*q and applies
    d, dmin per block in fp32, which equals w within fp32 rounding.)"""
    r1 = n if r1 is None else r1
    W = np.ascontiguousarray(W, dtype=np.uint8)
    wd = np.empty((r1 - r0, k), dtype=np.float32)
    assert lib().orc_dequant_rows(_p(W), qtype, k, n, r0, r1 - r0, _p(wd)) == 1
    x = np.atleast_2d(np.asarray(X, dtype=np.float32))
    hi = x.astype(np.float16)
    xe = hi.astype(np.float64)
    if precise:
        xe = xe + (x - hi.astype(np.float32)).astype(np.float16).astype(np.float64)
    return xe @ wd.astype(np.float64).T


def normalized_error(y: np.ndarray, y_ref: np.ndarray, wnorm: np.ndarray, x: np.ndarray) -> float:
    """max |y - y_ref| / (||w_row|| * ||x||), per activation row."""
    xx = np.atleast_2d(np.asarray(x, dtype=np.float64))
    yy = np.atleast_2d(np.asarray(y, dtype=np.float64))
    rr = np.atleast_2d(np.asarray(y_ref, dtype=np.float64))
    xn = np.linalg.norm(xx, axis=1)[:, None]
    denom = np.maximum(wnorm[None, :] * xn, 1e-30)
    return float(np.max(np.abs(yy - rr) / denom))


def max_rel_error(y: np.ndarray, y_ref: np.ndarray) -> float:
    """||y - y_ref||_inf / ||y_ref||_inf (per-element relative error is
    ill-posed on outputs near zero)."""
    yy = np.asarray(y, dtype=np.float64)
    rr = np.asarray(y_ref, dtype=np.float64)
    return float(np.max(np.abs(yy - rr)) / max(np.max(np.abs(rr)), 1e-30))


def ref_matvec(qtype: int, W: np.ndarray, x: np.ndarray, k: int, n: int, threads: int | None = None) -> np.ndarray:
    """Run the reference's simd_matvec_* on (W, x) and return y (fp32)."""
    if threads is not None:
        os.environ["ANVIL_NUM_THREADS"] = str(threads)
    name = {Q4_K: "q4k", Q4_K_R4: "q4k_r4", Q6_K: "q6k", Q6_K_R4: "q6k_r4", Q6_K_LM: "q6k_lm", Q8_0: "q8_0"}[qtype]
    W = np.ascontiguousarray(W, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    y = np.zeros((n,), dtype=np.float32)
    fp = ctypes.POINTER(ctypes.c_float)
    getattr(ref(), f"simd_matvec_{name}")(x.ctypes.data_as(fp), _p(W), y.ctypes.data_as(fp), k, n)
    return y


def ref_matmul(qtype: int, W: np.ndarray, X: np.ndarray, k: int, n: int) -> np.ndarray:
    name = {Q4_K: "q4k", Q4_K_R4: "q4k_r4", Q6_K: "q6k", Q6_K_R4: "q6k_r4", Q8_0: "q8_0"}[qtype]
    W = np.ascontiguousarray(W, dtype=np.uint8)
    X = np.ascontiguousarray(X, dtype=np.float32)
    m = X.shape[0]
    Y = np.zeros((m, n), dtype=np.float32)
    fp = ctypes.POINTER(ctypes.c_float)
    getattr(ref(), f"simd_matmul_{name}")(X.ctypes.data_as(fp), _p(W), Y.ctypes.data_as(fp), m, k, n)
    return Y
