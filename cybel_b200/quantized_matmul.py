"""Host-side mirror of the engine's quantized-matmul operator module.

Same names, argument meaning and error behaviour as
JSBuild/src/verso/Anvil/core/native/quantized_matmul_wrapper.py ("QW"):
``QuantizedMatrix`` holds packed GGUF rows ``[output_dim, row_bytes]`` with
``shape = (input_dim, output_dim)``; ``matvec`` / ``matmul`` compute
``x @ W`` through the drop-in C entry points of libb200q.so, which run on the
B200 (weights resident in HBM after first use). Layout validation happens
once per matrix and invalid layouts raise ``ValueError`` (QW:457-467,
507-517).

For callers that keep activations on the GPU, ``DeviceMatrix`` +
``matmul_device`` take torch CUDA tensors (torch owns the device buffers)
and call the asynchronous ``b200q_matmul`` on the current stream.
"""

from __future__ import annotations

import ctypes
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


def matvec(x: np.ndarray, matrix: QuantizedMatrix) -> np.ndarray:
    """y = x @ W for W quantized [in, out] (QW:449-479)."""
    lib = _native.lib()
    x_f = _ensure_f32_vec(x, matrix.input_dim)
    packed = matrix.ensure_packed()
    if not matrix._validated:
        raise ValueError(f"Invalid quantized layout for '{matrix.name}': qtype={matrix.qtype} shape={packed.shape}")
    name = _MATVEC_NAMES.get(matrix.qtype)
    if name is None:
        raise ValueError(f"Unsupported quantization type for '{matrix.name}': qtype={matrix.qtype}")
    out = np.empty((matrix.output_dim,), dtype=np.float32)
    getattr(lib, name)(_fp(x_f), ctypes.c_void_p(matrix._data_ptr), _fp(out), matrix.input_dim, matrix.output_dim)
    _raise_if_failed(name)
    if matrix._inverse_row_permutation is not None:
        out = out[matrix._inverse_row_permutation]
    return out


def matmul(x: np.ndarray, matrix: QuantizedMatrix) -> np.ndarray:
    """Y = X @ W for X [batch, in] (QW:482-530)."""
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
    if not x_f.flags["C_CONTIGUOUS"]:
        x_f = np.ascontiguousarray(x_f)
    if x_f.shape[0] == 1:
        return matvec(x_f[0], matrix).reshape(1, matrix.output_dim)
    lib = _native.lib()
    packed = matrix.ensure_packed()
    if not matrix._validated:
        raise ValueError(f"Invalid quantized layout for '{matrix.name}': qtype={matrix.qtype} shape={packed.shape}")
    name = _MATMUL_NAMES.get(matrix.qtype)
    if name is None:
        raise ValueError(f"Unsupported quantization type for '{matrix.name}': qtype={matrix.qtype}")
    out = np.empty((x_f.shape[0], matrix.output_dim), dtype=np.float32)
    getattr(lib, name)(
        _fp(x_f), ctypes.c_void_p(matrix._data_ptr), _fp(out), x_f.shape[0], matrix.input_dim, matrix.output_dim
    )
    _raise_if_failed(name)
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
            data = torch.from_numpy(np.ascontiguousarray(data, dtype=np.uint8))
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
