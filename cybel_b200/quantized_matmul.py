"""Host-side mirror of the engine's quantized-matmul operator module.

Same names, argument meaning and error behaviour as
JSBuild/src/verso/Anvil/core/native/quantized_matmul_wrapper.py ("QW"):
``QuantizedMatrix`` holds packed GGUF rows ``[output_dim, row_bytes]`` with
``shape = (input_dim, output_dim)``; ``matvec`` / ``matmul`` / the fused FFN
compute on the B200 through the device entry points of libb200q.so, with
each matrix's packed bytes uploaded once to a torch-owned HBM buffer attached
to the object. Layout validation happens once per matrix and invalid layouts
raise ``ValueError`` (QW:457-467, 507-517). C callers use the host-pointer
drop-ins (``simd_matvec_*`` ...) declared in include/b200q.h instead.

For callers that keep activations on the GPU, ``DeviceMatrix`` +
``matmul_device`` take torch CUDA tensors (torch owns the device buffers)
and call the asynchronous ``b200q_matmul`` on the current stream.
"""

from __future__ import annotations

import ctypes
import warnings
from dataclasses import dataclass, field
from typing import Iterable, Optional

import numpy as np

from . import _native
from .formats import (
    BLOCK_SPECS,
    Q4_0,
    Q4_K,
    Q4_K_R4,
    Q6_K,
    Q6_K_LM,
    Q6_K_R4,
    Q8_0,
    QTYPE_NAMES,
)

QTYPE_Q4_0 = Q4_0
QTYPE_Q8_0 = Q8_0
QTYPE_Q4_K = Q4_K
QTYPE_Q6_K = Q6_K
QTYPE_Q4_K_R4 = Q4_K_R4
QTYPE_Q6_K_R4 = Q6_K_R4
QTYPE_Q6_K_LM = Q6_K_LM

_BLOCK_SPECS = BLOCK_SPECS

_MATVEC_NAMES = {q: f"simd_matvec_{QTYPE_NAMES[q]}" for q in (Q4_K, Q4_K_R4, Q6_K, Q6_K_R4, Q6_K_LM, Q8_0, Q4_0)}
_MATMUL_NAMES = {q: f"simd_matmul_{QTYPE_NAMES[q]}" for q in (Q4_K, Q4_K_R4, Q6_K, Q6_K_R4, Q8_0, Q4_0)}


@dataclass
class QuantizedMatrix:
    """GGUF-backed quantized matrix stored in row-wise packed blocks (QW:45-98)."""

    name: str
    qtype: int
    shape: tuple[int, int]  # (input_dim, output_dim)
    data: np.ndarray  # uint8 packed rows, shape [output_dim, bytes_per_row]
    interleave_factor: int = 1

    _validated: bool = field(default=False, init=False, repr=False)
    _packed: np.ndarray | None = field(default=None, init=False, repr=False)
    _data_ptr: int = field(default=0, init=False, repr=False)
    _inverse_row_permutation: np.ndarray | None = field(default=None, init=False, repr=False)

    @property
    def input_dim(self) -> int:
        return int(self.shape[0])

    @property
    def output_dim(self) -> int:
        return int(self.shape[1])

    def ensure_packed(self) -> np.ndarray:
        if self._packed is not None:
            return self._packed
        arr = self.data
        if arr.dtype != np.uint8:
            arr = np.asarray(arr, dtype=np.uint8)
        if arr.ndim == 1:
            arr = arr.reshape(1, -1)
        if not arr.flags["C_CONTIGUOUS"]:
            arr = np.ascontiguousarray(arr)
        spec = _BLOCK_SPECS.get(self.qtype)
        if spec is not None:
            block_elems, block_bytes = spec
            if self.input_dim % block_elems == 0:
                expected = (self.input_dim // block_elems) * block_bytes
                if arr.shape == (self.output_dim, expected):
                    self._validated = True
        self._packed = arr
        self._data_ptr = arr.ctypes.data
        return arr


def is_quantized_matrix(value: object) -> bool:
    return isinstance(value, QuantizedMatrix)


def _ensure_f32_vec(x: np.ndarray, target_dim: int) -> np.ndarray:
    """Contiguous float32 vector of exactly target_dim (pads / truncates, QW:425-441)."""
    if x.dtype == np.float32 and x.ndim == 1 and x.shape[0] == target_dim and x.flags["C_CONTIGUOUS"]:
        return x
    vec = np.asarray(x, dtype=np.float32).reshape(-1)
    if vec.shape[0] == target_dim:
        return np.ascontiguousarray(vec)
    if vec.shape[0] > target_dim:
        return np.ascontiguousarray(vec[:target_dim])
    out = np.zeros((target_dim,), dtype=np.float32)
    out[: vec.shape[0]] = vec
    return out


def _fp(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _raise_if_failed(what: str) -> None:
    st = _native.lib().b200q_last_error()
    if st != 0:
        raise _native.NativeError(st, what)


def _device(matrix: "QuantizedMatrix") -> "DeviceMatrix":
    """The matrix's HBM-resident copy, uploaded on first use and owned by the
    QuantizedMatrix object (the packed data is immutable from then on, as in
    QW's own _packed cache)."""
    dm = getattr(matrix, "_device_copy", None)
    if dm is None:
        dm = DeviceMatrix.from_host(matrix)
        matrix._device_copy = dm
    return dm


def _act_mode() -> int:
    return int(_native.lib().b200q_get_act_mode())


def _checked(matrix: QuantizedMatrix, names: dict) -> None:
    packed = matrix.ensure_packed()
    if not matrix._validated:
        raise ValueError(f"Invalid quantized layout for '{matrix.name}': qtype={matrix.qtype} shape={packed.shape}")
    if matrix.qtype not in names:
        raise ValueError(f"Unsupported quantization type for '{matrix.name}': qtype={matrix.qtype}")


def matvec(x: np.ndarray, matrix: QuantizedMatrix) -> np.ndarray:
    """y = x @ W for W quantized [in, out] (QW:449-479), on the B200."""
    import torch

    x_f = _ensure_f32_vec(x, matrix.input_dim)
    _checked(matrix, _MATVEC_NAMES)
    y = matmul_device(torch.from_numpy(x_f).cuda(), _device(matrix), act_mode=_act_mode())
    out = y.cpu().numpy()
    if matrix._inverse_row_permutation is not None:
        out = out[matrix._inverse_row_permutation]
    return out


def matmul(x: np.ndarray, matrix: QuantizedMatrix) -> np.ndarray:
    """Y = X @ W for X [batch, in] (QW:482-530), on the B200."""
    import torch

    x_f = np.asarray(x, dtype=np.float32)
    if x_f.ndim == 1:
        return matvec(x_f, matrix)
    if x_f.ndim != 2:
        raise ValueError(f"matmul expects 2D input, got shape={x_f.shape}")
    if x_f.shape[1] != matrix.input_dim:
        if x_f.shape[1] > matrix.input_dim:
            x_f = x_f[:, : matrix.input_dim]
        else:
            padded = np.zeros((x_f.shape[0], matrix.input_dim), dtype=np.float32)
            padded[:, : x_f.shape[1]] = x_f
            x_f = padded
    x_f = np.ascontiguousarray(x_f)
    if x_f.shape[0] == 1:
        return matvec(x_f[0], matrix).reshape(1, matrix.output_dim)
    names = dict(_MATMUL_NAMES)
    names[QTYPE_Q6_K_LM] = "b200q_matmul"  # the device API also takes the LM layout
    _checked(matrix, names)
    y = matmul_device(torch.from_numpy(x_f).cuda(), _device(matrix), act_mode=_act_mode())
    out = y.cpu().numpy()
    if matrix._inverse_row_permutation is not None:
        out = out[:, matrix._inverse_row_permutation]
    return out


def set_act_mode(mode: str | int) -> int:
    """Select the activation arithmetic of the drop-ins: "x16" (default) or "x8"."""
    m = {"x8": _native.ACT_X8, "x16": _native.ACT_X16}.get(mode, mode) if isinstance(mode, str) else int(mode)
    return int(_native.lib().b200q_set_act_mode(int(m)))


# ---------------------------------------------------------------------------
# Device-resident path (torch owns the buffers).
# ---------------------------------------------------------------------------
class DeviceMatrix:
    """Packed GGUF rows resident in HBM as a torch uint8 CUDA tensor."""

    def __init__(self, qtype: int, input_dim: int, output_dim: int, data, name: str = ""):
        import torch

        if not isinstance(data, torch.Tensor):
            arr = np.ascontiguousarray(data, dtype=np.uint8)
            with warnings.catch_warnings():
                # A read-only array (a memory-mapped GGUF file) is only read here:
                # it is copied to the device just below.
                warnings.simplefilter("ignore", UserWarning)
                data = torch.from_numpy(arr)
        if data.device.type != "cuda":
            data = data.cuda()
        e, b = BLOCK_SPECS[qtype]
        if input_dim % e:
            raise ValueError(f"input_dim {input_dim} not a multiple of the qtype {qtype} block ({e})")
        rb = (input_dim // e) * b
        flat = data.reshape(-1)
        if flat.numel() != rb * output_dim:
            raise ValueError(f"packed size {flat.numel()} != {output_dim} x {rb}")
        # +16 bytes: kernels copy 16-byte-aligned windows around rows.
        buf = torch.empty(flat.numel() + 16, dtype=torch.uint8, device=flat.device)
        buf[: flat.numel()].copy_(flat)
        # Weights are immutable from here on: once the upload has completed,
        # kernels may stream them ahead of their grid dependency.
        torch.cuda.synchronize(flat.device)
        self.buffer = buf
        self.qtype = int(qtype)
        self.input_dim = int(input_dim)
        self.output_dim = int(output_dim)
        self.name = name

    @classmethod
    def from_host(cls, m: QuantizedMatrix) -> "DeviceMatrix":
        return cls(m.qtype, m.input_dim, m.output_dim, m.ensure_packed(), name=m.name)

    @property
    def ptr(self) -> int:
        return int(self.buffer.data_ptr())

    def clone(self) -> "DeviceMatrix":
        """A second resident copy of the same rows (device-to-device)."""
        return DeviceMatrix(self.qtype, self.input_dim, self.output_dim, self.buffer[: self.buffer.numel() - 16],
                            name=self.name)


def matmul_device(x, matrix: DeviceMatrix, out=None, act_mode: int = _native.ACT_X16):
    """Y = X @ W on the current CUDA stream; X float32 CUDA [m, in] or [in]."""
    import torch

    if x.device.type != "cuda" or x.dtype != torch.float32:
        raise ValueError("matmul_device expects a float32 CUDA tensor")
    squeeze = x.dim() == 1
    xx = x.reshape(1, -1) if squeeze else x
    xx = xx.contiguous()
    if xx.shape[1] != matrix.input_dim:
        raise ValueError(f"x has {xx.shape[1]} features, matrix expects {matrix.input_dim}")
    m = xx.shape[0]
    if out is None:
        out = torch.empty((m, matrix.output_dim), dtype=torch.float32, device=xx.device)
    st = torch.cuda.current_stream(xx.device).cuda_stream
    rc = _native.lib().b200q_matmul_ex(
        matrix.qtype, int(act_mode), xx.data_ptr(), matrix.ptr, out.data_ptr(), m, matrix.input_dim, matrix.output_dim,
        _native.WEIGHTS_STATIC, st,
    )
    _native.check(rc, "b200q_matmul_ex")
    return out.reshape(-1) if squeeze else out


def matvec_isums_device(x, matrix: DeviceMatrix, act_mode: int = _native.ACT_X16):
    """(y, isums): the matvec plus its exact per-group integer sums."""
    import torch

    g = 16 if matrix.qtype in (Q6_K, Q6_K_R4, Q6_K_LM) else 32
    y = torch.empty((matrix.output_dim,), dtype=torch.float32, device=x.device)
    isums = torch.empty((matrix.output_dim, matrix.input_dim // g), dtype=torch.int32, device=x.device)
    st = torch.cuda.current_stream(x.device).cuda_stream
    rc = _native.lib().b200q_matvec_isums(
        matrix.qtype, int(act_mode), x.contiguous().data_ptr(), matrix.ptr, y.data_ptr(), isums.data_ptr(),
        matrix.input_dim, matrix.output_dim, st,
    )
    _native.check(rc, "b200q_matvec_isums")
    return y, isums


# ---------------------------------------------------------------------------
# Layout repacks (QW:270-415), row interleave (QW:232-268), dequantization
# (QW:533-566) and the fused expert / MoE FFN (QW:569-765).
# ---------------------------------------------------------------------------
def interleave_quantized_rows(matrix: QuantizedMatrix, factor: int) -> QuantizedMatrix:
    """Row-interleaved copy with inverse permutation metadata (storage only)."""
    interleave = int(max(1, factor))
    if interleave <= 1:
        return matrix
    packed = matrix.ensure_packed()
    rows = int(packed.shape[0])
    if rows <= 1:
        return matrix
    order = np.concatenate([np.arange(off, rows, interleave, dtype=np.int64) for off in range(interleave)])
    if order.shape[0] != rows or np.array_equal(order, np.arange(rows, dtype=np.int64)):
        return matrix
    result = QuantizedMatrix(name=matrix.name, qtype=matrix.qtype, shape=matrix.shape,
                             data=np.ascontiguousarray(packed[order]), interleave_factor=interleave)
    result._validated = bool(matrix._validated)
    result._inverse_row_permutation = np.argsort(order)
    return result


def _requires_output_deinterleave(matrix: QuantizedMatrix) -> bool:
    perm = matrix._inverse_row_permutation
    return isinstance(perm, np.ndarray) and perm.size > 0


def has_q4k_r4_support() -> bool:
    return hasattr(_native.lib(), "simd_repack_q4k_r4")


def has_q6k_r4_support() -> bool:
    return hasattr(_native.lib(), "simd_repack_q6k_r4")


def has_q6k_lm_support() -> bool:
    return hasattr(_native.lib(), "simd_repack_q6k_lm")


def _repack(matrix: QuantizedMatrix, src_qtype: int, dst_qtype: int, fn_name: str, dst_block: int, suffix: str):
    if matrix.qtype == dst_qtype or matrix.qtype != src_qtype:
        return matrix
    packed = matrix.ensure_packed()
    if not matrix._validated or _requires_output_deinterleave(matrix):
        return matrix
    cache_attr = f"_repacked_{suffix}"
    cached = getattr(matrix, cache_attr, None)
    if isinstance(cached, QuantizedMatrix):
        return cached
    dst = np.empty((matrix.output_dim, (matrix.input_dim // 256) * dst_block), dtype=np.uint8)
    ok = getattr(_native.lib(), fn_name)(packed.ctypes.data, dst.ctypes.data, matrix.input_dim, matrix.output_dim)
    if int(ok) != 1:
        return matrix
    out = QuantizedMatrix(name=f"{matrix.name}::{suffix}", qtype=dst_qtype, shape=matrix.shape, data=dst)
    out.ensure_packed()
    out._validated = True
    setattr(matrix, cache_attr, out)
    return out


def repack_q4k_r4(matrix: QuantizedMatrix) -> QuantizedMatrix:
    """Canonical Q4_K -> 4-row block-major Q4_K_R4 (QW:270-312), on the GPU."""
    return _repack(matrix, QTYPE_Q4_K, QTYPE_Q4_K_R4, "simd_repack_q4k_r4", 144, "q4k_r4")


def repack_q6k_r4(matrix: QuantizedMatrix) -> QuantizedMatrix:
    """Canonical Q6_K -> 4-row block-major Q6_K_R4 (QW:315-357), on the GPU."""
    return _repack(matrix, QTYPE_Q6_K, QTYPE_Q6_K_R4, "simd_repack_q6k_r4", 210, "q6k_r4")


def repack_q6k_lm(matrix: QuantizedMatrix) -> QuantizedMatrix:
    """Q6_K -> expanded LM-head layout Q6_K_LM (QW:360-401), on the GPU."""
    return _repack(matrix, QTYPE_Q6_K, QTYPE_Q6_K_LM, "simd_repack_q6k_lm", 276, "q6k_lm")


def dequantize_rows(matrix: QuantizedMatrix, row_ids: Iterable[int]) -> np.ndarray:
    """Dequantize selected rows (embedding lookups), on the GPU (QW:533-546)."""
    idx = np.asarray(list(row_ids), dtype=np.int64).reshape(-1)
    if idx.size == 0:
        return np.zeros((0, matrix.input_dim), dtype=np.float32)
    clipped = np.clip(idx, 0, matrix.output_dim - 1)
    if matrix._inverse_row_permutation is not None:
        clipped = matrix._inverse_row_permutation[clipped]
    packed = matrix.ensure_packed()
    if matrix.qtype not in _BLOCK_SPECS or not matrix._validated:
        raise ValueError(f"Unsupported GGUF quantization type: {matrix.qtype}")
    out = np.empty((idx.size, matrix.input_dim), dtype=np.float32)
    if matrix.qtype in (QTYPE_Q4_K_R4, QTYPE_Q6_K_R4):
        # The 4-row groups need the whole matrix (and n for the tail rows).
        import torch

        dm = getattr(matrix, "_device_copy", None)
        if dm is None:
            dm = DeviceMatrix.from_host(matrix)
            matrix._device_copy = dm
        rows_dev = torch.from_numpy(clipped.astype(np.int32)).cuda()
        out_dev = torch.empty((idx.size, matrix.input_dim), dtype=torch.float32, device="cuda")
        rc = _native.lib().b200q_dequantize_rows(matrix.qtype, dm.ptr, rows_dev.data_ptr(), int(idx.size),
                                                 out_dev.data_ptr(), matrix.input_dim, matrix.output_dim,
                                                 torch.cuda.current_stream().cuda_stream)
        _native.check(rc, "b200q_dequantize_rows")
        return out_dev.cpu().numpy()
    lib = _native.lib()
    for i, r in enumerate(clipped.tolist()):
        ok = lib.simd_dequantize_row(packed.ctypes.data, matrix.qtype, int(r), _fp(out[i]), matrix.input_dim)
        if int(ok) != 1:
            raise _native.NativeError(lib.b200q_last_error(), "simd_dequantize_row")
    return out


def dequantize_full(matrix: QuantizedMatrix) -> np.ndarray:
    """The whole matrix as dense fp32 [output_dim, input_dim] (QW:549-566)."""
    return dequantize_rows(matrix, range(matrix.output_dim)) if matrix._inverse_row_permutation is None else \
        dequantize_rows(matrix, np.argsort(matrix._inverse_row_permutation))


def _strict_native_qsg_enabled() -> bool:
    import os

    raw = os.getenv("ANVIL_STRICT_NATIVE_QSG")
    if raw is not None:
        return str(raw).strip().lower() not in {"0", "false", "no", "off"}
    return False


def _canonical(matrix: QuantizedMatrix) -> QuantizedMatrix:
    """The matrix with its row interleave undone (data movement only)."""
    if not _requires_output_deinterleave(matrix):
        return matrix
    packed = matrix.ensure_packed()
    out = QuantizedMatrix(name=matrix.name, qtype=matrix.qtype, shape=matrix.shape,
                          data=np.ascontiguousarray(packed[matrix._inverse_row_permutation]))
    out.ensure_packed()
    return out


def fused_expert_swiglu(x: np.ndarray, gate_matrix: QuantizedMatrix, up_matrix: QuantizedMatrix,
                        down_matrix: QuantizedMatrix) -> np.ndarray:
    """down(silu(gate x) * (up x)) in one native call on the B200 (QW:569-633)."""
    lib = _native.lib()
    x_f = _ensure_f32_vec(x, gate_matrix.input_dim)
    for m in (gate_matrix, up_matrix, down_matrix):
        m.ensure_packed()
    if not (gate_matrix._validated and up_matrix._validated and down_matrix._validated):
        if _strict_native_qsg_enabled():
            raise RuntimeError("Strict native QSG requires validated fused expert matrices; fallback is disabled.")
        raise ValueError("Invalid quantized layout for fused expert matrices")
    if _requires_output_deinterleave(gate_matrix) or _requires_output_deinterleave(up_matrix):
        if _strict_native_qsg_enabled():
            raise RuntimeError("Strict native QSG requires fused expert kernels without row-deinterleave fallback.")
        gate_matrix, up_matrix = _canonical(gate_matrix), _canonical(up_matrix)
    import torch

    for m, nm in ((gate_matrix, "gate"), (up_matrix, "up"), (down_matrix, "down")):
        if m.qtype not in _FFN_QTYPES:
            raise ValueError(f"unsupported {nm} qtype {m.qtype}")
    xt = torch.from_numpy(x_f).cuda()
    out = torch.empty((down_matrix.output_dim,), dtype=torch.float32, device="cuda")
    g, u, d = _device(gate_matrix), _device(up_matrix), _device(down_matrix)
    rc = lib.b200q_expert_swiglu(
        _act_mode(), xt.data_ptr(), gate_matrix.input_dim, g.ptr, gate_matrix.qtype, gate_matrix.output_dim, u.ptr,
        up_matrix.qtype, d.ptr, down_matrix.qtype, down_matrix.output_dim, out.data_ptr(), 1.0, 0.0,
        _native.WEIGHTS_STATIC, torch.cuda.current_stream().cuda_stream,
    )
    _native.check(rc, "b200q_expert_swiglu")
    res = out.cpu().numpy()
    if _requires_output_deinterleave(down_matrix):
        res = res[down_matrix._inverse_row_permutation]
    return res


_FFN_QTYPES = {QTYPE_Q4_K, QTYPE_Q4_K_R4, QTYPE_Q6_K, QTYPE_Q6_K_R4, QTYPE_Q6_K_LM, QTYPE_Q8_0}


def fused_moe_ffn(x: np.ndarray, expert_weights, gate_matrices, up_matrices, down_matrices) -> np.ndarray:
    """sum_e w_e * expert_e(x) for quantized SwiGLU experts (QW:636-765)."""
    k = len(expert_weights)
    if k == 0 or len(gate_matrices) != k or len(up_matrices) != k or len(down_matrices) != k:
        raise ValueError("fused_moe_ffn expects non-empty, equal-length expert lists")
    if not all(isinstance(m, QuantizedMatrix) for m in (*gate_matrices, *up_matrices, *down_matrices)):
        raise ValueError("fused_moe_ffn only supports QuantizedMatrix expert weights")
    gq, uq, dq = gate_matrices[0].qtype, up_matrices[0].qtype, down_matrices[0].qtype
    allowed = {QTYPE_Q8_0, QTYPE_Q4_K, QTYPE_Q4_K_R4, QTYPE_Q6_K}
    if gq not in allowed or uq not in allowed or dq not in allowed:
        raise ValueError("fused_moe_ffn only supports Q8_0/Q4_K/Q4_K_R4/Q6_K experts")
    in_dim, hidden, out_dim = gate_matrices[0].input_dim, gate_matrices[0].output_dim, down_matrices[0].output_dim
    for g, u, d in zip(gate_matrices, up_matrices, down_matrices):
        if g.qtype != gq or u.qtype != uq or d.qtype != dq:
            raise ValueError("fused_moe_ffn requires uniform qtype per projection kind")
        if g.input_dim != in_dim or u.input_dim != in_dim:
            raise ValueError("fused_moe_ffn requires consistent input dims across experts")
        if g.output_dim != hidden or u.output_dim != hidden:
            raise ValueError("fused_moe_ffn requires consistent hidden dims across experts")
        if d.input_dim != hidden or d.output_dim != out_dim:
            raise ValueError("fused_moe_ffn requires down projection dims matching hidden/out dims")
    x_f = _ensure_f32_vec(x, in_dim)
    w = np.ascontiguousarray(np.asarray(expert_weights, dtype=np.float32).reshape(-1))
    for m in (*gate_matrices, *up_matrices, *down_matrices):
        m.ensure_packed()
        if not m._validated:
            raise ValueError(f"Invalid quantized layout for '{m.name}'")
    if any(_requires_output_deinterleave(m) for m in (*gate_matrices, *up_matrices, *down_matrices)):
        if _strict_native_qsg_enabled():
            raise RuntimeError("Strict native QSG requires fused MoE kernels without row-deinterleave fallback.")
        gate_matrices = [_canonical(m) for m in gate_matrices]
        up_matrices = [_canonical(m) for m in up_matrices]
        down_matrices = [_canonical(m) for m in down_matrices]
    import torch

    idx = np.arange(k, dtype=np.int32)
    gp = (ctypes.c_void_p * k)(*[_device(m).ptr for m in gate_matrices])
    up = (ctypes.c_void_p * k)(*[_device(m).ptr for m in up_matrices])
    dp = (ctypes.c_void_p * k)(*[_device(m).ptr for m in down_matrices])
    xt = torch.from_numpy(x_f).cuda()
    out = torch.empty((out_dim,), dtype=torch.float32, device="cuda")
    rc = _native.lib().b200q_moe_ffn(
        _act_mode(), xt.data_ptr(), in_dim, idx.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), _fp(w), k, gp, gq,
        hidden, up, uq, dp, dq, out_dim, out.data_ptr(), 0, _native.WEIGHTS_STATIC,
        torch.cuda.current_stream().cuda_stream,
    )
    _native.check(rc, "b200q_moe_ffn")
    return out.cpu().numpy()
