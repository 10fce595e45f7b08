"""GGUF model files: the on-disk container of the quantized weights.

The reference engine reads its models through gguf-py's ``GGUFReader``
(JSBuild/src/verso/Anvil/core/model/gguf_loader.py:178) and turns each 2-D
tensor of a supported quantized type into a ``QuantizedMatrix`` whose bytes
are the file's own rows (core/native/weight_store.py:86-114). This module
reads the same container directly -- header, typed metadata, tensor table and
aligned data section (GGUF version 2 and 3, little endian) -- and hands out
memory-mapped views of the tensors, so a matrix goes from the file to HBM in
one copy with its block layout untouched:

    f = GGUFFile("model.gguf")
    f.metadata["llama.block_count"]
    wq = f.quantized("blk.0.attn_q.weight")        # QuantizedMatrix, shape (k, n)
    dm = f.device_matrix("blk.0.attn_q.weight")    # resident DeviceMatrix

``load_llama_stack`` maps a llama-architecture file onto the decode stacks
(``DecodeStack.from_gguf``). Only this file's parser is used; gguf-py is a
test dependency (it writes the fixtures the tests read back).
"""

from __future__ import annotations

import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from .formats import Q4_0, Q4_K, Q6_K, Q8_0

GGUF_MAGIC = b"GGUF"
DEFAULT_ALIGNMENT = 32

# Metadata value types of the format and their little-endian struct codes.
_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}
_STRING, _ARRAY = 8, 9

# ggml tensor types this module sizes: (elements per block, bytes per block).
GGML_F32, GGML_F16, GGML_BF16 = 0, 1, 30
_BLOCKS = {GGML_F32: (1, 4), GGML_F16: (1, 2), GGML_BF16: (1, 2), Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144),
           Q6_K: (256, 210)}
# Types the matvec kernels consume as they lie in the file.
QUANTIZED_TYPES = (Q4_0, Q8_0, Q4_K, Q6_K)


class GGUFError(ValueError):
    """The file is not a GGUF file this reader understands."""


@dataclass(frozen=True)
class TensorInfo:
    name: str
    dims: tuple[int, ...]  # ne0 (elements per row, contiguous) first
    ggml_type: int
    offset: int            # absolute byte offset of the data in the file
    nbytes: int            # -1 for a type this reader cannot size

    @property
    def row_elems(self) -> int:
        return self.dims[0]

    @property
    def rows(self) -> int:
        r = 1
        for d in self.dims[1:]:
            r *= d
        return r


class _Cursor:
    def __init__(self, buf: memoryview):
        self.buf, self.pos = buf, 0

    def take(self, n: int) -> memoryview:
        if self.pos + n > len(self.buf):
            raise GGUFError("truncated GGUF file")
        v = self.buf[self.pos:self.pos + n]
        self.pos += n
        return v

    def scalar(self, code: str):
        return struct.unpack(code, self.take(struct.calcsize(code)))[0]

    def string(self) -> str:
        n = self.scalar("<Q")
        return bytes(self.take(n)).decode("utf-8", errors="replace")

    def value(self, vtype: int):
        if vtype in _SCALAR:
            return self.scalar(_SCALAR[vtype])
        if vtype == _STRING:
            return self.string()
        if vtype == _ARRAY:
            etype, count = self.scalar("<I"), self.scalar("<Q")
            if etype in _SCALAR and etype != 7:
                code = _SCALAR[etype]
                raw = self.take(count * struct.calcsize(code))
                return np.frombuffer(raw, dtype=np.dtype(code)).tolist()
            return [self.value(etype) for _ in range(count)]
        raise GGUFError(f"unknown metadata value type {vtype}")


def _tensor_nbytes(ggml_type: int, dims: tuple[int, ...]) -> int:
    blk = _BLOCKS.get(ggml_type)
    if blk is None:
        return -1
    elems, nbytes = blk
    if dims[0] % elems:
        raise GGUFError(f"row of {dims[0]} elements is not a whole number of type-{ggml_type} blocks")
    n = dims[0] // elems * nbytes
    for d in dims[1:]:
        n *= d
    return n


class GGUFFile:
    """A GGUF file opened read-only and memory-mapped."""

    def __init__(self, path: str | Path):
        self.path = Path(path)
        self._map = np.memmap(self.path, dtype=np.uint8, mode="r")
        cur = _Cursor(memoryview(self._map))
        if bytes(cur.take(4)) != GGUF_MAGIC:
            raise GGUFError(f"{self.path}: not a GGUF file")
        self.version = cur.scalar("<I")
        if self.version not in (2, 3):
            raise GGUFError(f"{self.path}: GGUF version {self.version} is not supported")
        n_tensors, n_kv = cur.scalar("<Q"), cur.scalar("<Q")
        self.metadata: dict[str, object] = {}
        for _ in range(n_kv):
            key = cur.string()
            self.metadata[key] = cur.value(cur.scalar("<I"))
        infos = []
        for _ in range(n_tensors):
            name = cur.string()
            nd = cur.scalar("<I")
            dims = tuple(int(cur.scalar("<Q")) for _ in range(nd))
            infos.append((name, dims, cur.scalar("<I"), cur.scalar("<Q")))
        align = int(self.metadata.get("general.alignment", DEFAULT_ALIGNMENT))
        if align <= 0 or align & (align - 1):
            raise GGUFError(f"alignment {align} is not a power of two")
        self.alignment = align
        self.data_offset = (cur.pos + align - 1) // align * align
        self.tensors: dict[str, TensorInfo] = {}
        for name, dims, gtype, off in infos:
            if off % align:
                raise GGUFError(f"tensor {name} is not aligned to {align} bytes")
            nbytes = _tensor_nbytes(gtype, dims)
            start = self.data_offset + off
            if nbytes >= 0 and start + nbytes > len(self._map):
                raise GGUFError(f"tensor {name} runs past the end of the file")
            self.tensors[name] = TensorInfo(name, dims, gtype, start, nbytes)

    def __contains__(self, name: str) -> bool:
        return name in self.tensors

    def raw(self, name: str) -> np.ndarray:
        """The tensor's bytes as a read-only [rows][row_bytes] uint8 view."""
        t = self.tensors[name]
        if t.nbytes < 0:
            raise GGUFError(f"tensor {name}: ggml type {t.ggml_type} is not supported")
        return self._map[t.offset:t.offset + t.nbytes].reshape(t.rows, t.nbytes // t.rows)

    def array(self, name: str) -> np.ndarray:
        """A float tensor (F32, F16 or BF16) as float32, shape [rows][ne0]
        (1-D tensors as [ne0])."""
        t = self.tensors[name]
        raw = self.raw(name).reshape(-1)
        if t.ggml_type == GGML_F32:
            a = raw.view("<f4").astype(np.float32)
        elif t.ggml_type == GGML_F16:
            a = raw.view("<f2").astype(np.float32)
        elif t.ggml_type == GGML_BF16:
            a = (raw.view("<u2").astype(np.uint32) << 16).view(np.float32)
        else:
            raise GGUFError(f"tensor {name} is quantized (ggml type {t.ggml_type}), not a float tensor")
        return a if len(t.dims) == 1 else a.reshape(t.rows, t.row_elems)

    def quantized(self, name: str):
        """A 2-D tensor of a quantized type as a QuantizedMatrix (shape (k, n):
        k elements per row, n rows), its data the file's own rows (copied once
        into host memory)."""
        from .quantized_matmul import QuantizedMatrix

        t = self.tensors[name]
        if len(t.dims) != 2 or t.ggml_type not in QUANTIZED_TYPES:
            raise GGUFError(f"tensor {name}: a 2-D Q4_0 / Q8_0 / Q4_K / Q6_K tensor is required")
        return QuantizedMatrix(name=name, qtype=t.ggml_type, shape=(t.dims[0], t.dims[1]),
                               data=np.ascontiguousarray(self.raw(name)))

    def device_matrix(self, name: str):
        """The quantized tensor resident on the current CUDA device."""
        from .quantized_matmul import DeviceMatrix

        t = self.tensors[name]
        if len(t.dims) != 2 or t.ggml_type not in QUANTIZED_TYPES:
            raise GGUFError(f"tensor {name}: a 2-D Q4_0 / Q8_0 / Q4_K / Q6_K tensor is required")
        return DeviceMatrix(t.ggml_type, t.dims[0], t.dims[1], np.ascontiguousarray(self.raw(name)), name=name)


def load_llama_stack(path: str | Path):
    """(StackShape, layers, embed, head, out_norm) of a llama-architecture GGUF
    file, in the form DecodeStack and ShardedDecode take: per layer the packed
    rows of wq / wk / wv / wo / w_gate / w_up / w_down and fp32 RMSNorm gains.
    Every linear must share one quantized type (q/k/v and gate/up are joined
    into one matrix each); the embedding and head may have their own. A file
    without ``output.weight`` ties the head to the embedding."""
    from .decode import StackShape

    f = GGUFFile(path)
    arch = str(f.metadata.get("general.architecture", "llama"))

    def meta(key, default=None):
        v = f.metadata.get(f"{arch}.{key}", default)
        if v is None:
            raise GGUFError(f"metadata {arch}.{key} is missing")
        return v

    n_layers = int(meta("block_count"))
    hidden = int(meta("embedding_length"))
    heads = int(meta("attention.head_count"))
    kv_heads = int(meta("attention.head_count_kv", heads))
    ffn = int(meta("feed_forward_length"))
    eps = float(meta("attention.layer_norm_rms_epsilon", 1e-5))
    theta = float(meta("rope.freq_base", 10000.0))
    embed_t = f.tensors["token_embd.weight"]
    vocab = embed_t.dims[1]
    head_name = "output.weight" if "output.weight" in f else "token_embd.weight"
    names = {"wq": "attn_q", "wk": "attn_k", "wv": "attn_v", "wo": "attn_output", "w_gate": "ffn_gate",
             "w_up": "ffn_up", "w_down": "ffn_down"}
    qtypes = {f.tensors[f"blk.{i}.{n}.weight"].ggml_type for i in range(n_layers) for n in names.values()}
    if len(qtypes) != 1 or next(iter(qtypes)) not in QUANTIZED_TYPES:
        raise GGUFError(f"the linears use quantized types {sorted(qtypes)}; one of {QUANTIZED_TYPES} is required")
    shape = StackShape(layers=n_layers, hidden=hidden, heads=heads, kv_heads=kv_heads, ffn=ffn, vocab=vocab,
                       rope_theta=theta, eps=eps, linear_qtype=next(iter(qtypes)),
                       head_qtype=f.tensors[head_name].ggml_type, embed_qtype=embed_t.ggml_type)
    layers = []
    for i in range(n_layers):
        lay = {key: np.ascontiguousarray(f.raw(f"blk.{i}.{n}.weight")) for key, n in names.items()}
        lay["attn_norm"] = f.array(f"blk.{i}.attn_norm.weight")
        lay["ffn_norm"] = f.array(f"blk.{i}.ffn_norm.weight")
        layers.append(lay)
    return (shape, layers, np.ascontiguousarray(f.raw("token_embd.weight")), np.ascontiguousarray(f.raw(head_name)),
            f.array("output_norm.weight"))
