"""Host-side GGUF block packers for synthetic and user weights.

The engine only ever *loads* pre-quantized GGUF tensors
(core/native/weight_store.py:86-114); gguf-py 0.19.0 can quantize Q4_0 and
Q8_0 but raises ``NotImplementedError`` for Q4_K and Q6_K. These packers
produce the exact on-disk block layouts the kernels consume:

* ``quantize_q8_0`` / ``quantize_q4_0`` follow ggml's reference quantizers
  (the same arithmetic as gguf-py's ``Q8_0.quantize_blocks`` /
  ``Q4_0.quantize_blocks``), so their bytes equal ``gguf.quantize``'s.
* ``quantize_q4_k`` / ``quantize_q6_k`` use a simple min/max (Q4_K) and
  abs-max (Q6_K) scheme of this package's own. Any valid scale choice is a
  valid block; the layouts are those decoded by quantized_matmul.cpp:411-455
  (Q4_K) and :683-775 (Q6_K), and the tests round-trip them through
  ``gguf.dequantize``.

All functions take a float array of shape [n, k] (rows = output channels) and
return uint8 [n, row_bytes].
"""

from __future__ import annotations

import numpy as np

QK = 256


def _f16(a: np.ndarray) -> np.ndarray:
    return np.asarray(a, dtype=np.float32).astype(np.float16)


def _roundf(a: np.ndarray) -> np.ndarray:
    """C ``roundf``: half away from zero."""
    return np.sign(a) * np.floor(np.abs(a) + np.float32(0.5))


def quantize_q8_0(w: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    assert k % 32 == 0
    blocks = w.reshape(-1, 32)
    d = np.abs(blocks).max(axis=1, keepdims=True) / np.float32(127)
    with np.errstate(divide="ignore"):
        inv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
    qs = _roundf(blocks * inv).astype(np.int8)
    out = np.concatenate([_f16(d).view(np.uint8), qs.view(np.uint8)], axis=1)
    return out.reshape(n, (k // 32) * 34)


def quantize_q4_0(w: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    assert k % 32 == 0
    blocks = w.reshape(-1, 32)
    imax = np.abs(blocks).argmax(axis=-1)[:, None]
    mx = np.take_along_axis(blocks, imax, axis=-1)
    d = (mx / np.float32(-8)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
    q = np.trunc(blocks * inv + np.float32(8.5)).astype(np.float32)
    q = np.clip(q, 0, 15).astype(np.uint8)
    qs = q[:, :16] | (q[:, 16:] << np.uint8(4))
    out = np.concatenate([_f16(d).view(np.uint8), qs], axis=1)
    return out.reshape(n, (k // 32) * 18)


def quantize_q4_k(w: np.ndarray) -> np.ndarray:
    """Q4_K: per 32-element sub-block an asymmetric 4-bit range, sub-block
    scales and mins quantized to 6 bits against fp16 super-scales d / dmin."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    assert k % QK == 0
    sb = w.reshape(-1, 8, 32)                       # [nblk, 8, 32]
    mn = np.minimum(sb.min(axis=2), 0.0)            # <= 0
    mx = sb.max(axis=2)
    scale = (mx - mn) / np.float32(15)              # >= 0
    neg_min = -mn                                   # >= 0
    d = _f16(scale.max(axis=1) / np.float32(63))
    dmin = _f16(neg_min.max(axis=1) / np.float32(63))
    d32 = d.astype(np.float32)[:, None]
    dmin32 = dmin.astype(np.float32)[:, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d32 > 0, np.rint(scale / d32), 0)
        m6 = np.where(dmin32 > 0, np.rint(neg_min / dmin32), 0)
    sc = np.clip(sc, 0, 63).astype(np.uint8)
    m6 = np.clip(m6, 0, 63).astype(np.uint8)
    step = d32 * sc.astype(np.float32)              # [nblk, 8]
    off = dmin32 * m6.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(step[..., None] > 0, np.rint((sb + off[..., None]) / step[..., None]), 0)
    q = np.clip(q, 0, 15).astype(np.uint8)          # [nblk, 8, 32]

    nblk = sb.shape[0]
    scales = np.zeros((nblk, 12), dtype=np.uint8)
    lo_sc, hi_sc = sc[:, :4], sc[:, 4:]
    lo_mn, hi_mn = m6[:, :4], m6[:, 4:]
    scales[:, 0:4] = (lo_sc & 63) | ((hi_sc >> 4) << 6)
    scales[:, 4:8] = (lo_mn & 63) | ((hi_mn >> 4) << 6)
    scales[:, 8:12] = (hi_sc & 15) | ((hi_mn & 15) << 4)
    qs = (q[:, 0::2, :] | (q[:, 1::2, :] << np.uint8(4))).reshape(nblk, 128)
    out = np.concatenate([d.view(np.uint8).reshape(nblk, 2), dmin.view(np.uint8).reshape(nblk, 2), scales, qs], axis=1)
    return out.reshape(n, (k // QK) * 144)


def quantize_q6_k(w: np.ndarray) -> np.ndarray:
    """Q6_K: symmetric 6-bit codes per 16-element group, int8 group scales
    against one fp16 super-scale d."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    assert k % QK == 0
    g = w.reshape(-1, 16, 16)                       # [nblk, 16 groups, 16]
    amax = np.abs(g).max(axis=2)
    s = amax / np.float32(31)
    d = _f16(s.max(axis=1) / np.float32(127))
    d32 = d.astype(np.float32)[:, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d32 > 0, np.rint(s / d32), 0)
    sc = np.clip(sc, -128, 127).astype(np.int8)
    step = d32 * sc.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(step[..., None] != 0, np.rint(g / step[..., None]), 0)
    q = (np.clip(q, -32, 31).astype(np.int16) + 32).astype(np.uint8)   # [nblk, 16, 16] in 0..63
    nblk = g.shape[0]
    q = q.reshape(nblk, 2, 4, 32)                  # [blk, half h, group-in-half gm, 32]
    ql = np.zeros((nblk, 2, 64), dtype=np.uint8)
    qh = np.zeros((nblk, 2, 32), dtype=np.uint8)
    for gm in range(4):
        lo = q[:, :, gm, :] & 0x0F
        hi = (q[:, :, gm, :] >> 4) & 0x03
        start = (gm % 2) * 32
        shift = 4 if gm >= 2 else 0
        ql[:, :, start:start + 32] |= (lo << shift).astype(np.uint8)
        qh[:, :, :] |= (hi << (2 * gm)).astype(np.uint8)
    out = np.concatenate([ql.reshape(nblk, 128), qh.reshape(nblk, 64), sc.view(np.uint8), d.view(np.uint8).reshape(nblk, 2)], axis=1)
    return out.reshape(n, (k // QK) * 210)


def quantize(w: np.ndarray, qtype: int) -> np.ndarray:
    from .formats import Q4_0, Q4_K, Q6_K, Q8_0

    fn = {Q4_0: quantize_q4_0, Q8_0: quantize_q8_0, Q4_K: quantize_q4_k, Q6_K: quantize_q6_k}.get(int(qtype))
    if fn is None:
        raise ValueError(f"no packer for qtype {qtype}")
    return fn(w)
