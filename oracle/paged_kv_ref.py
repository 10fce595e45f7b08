"""CPU restatement of the reference's paged KV store and its decode attention
-- TEST INFRASTRUCTURE ONLY (imported by tests; never by the product).

Follows JSBuild/src/verso/Anvil/core/native/model_graph.cpp:
* PagedKVStore (1413-1576): pages of `page_size` positions per layer,
  allocated when a position is first written; in Q8 mode each
  (position, kv head) row is stored as int8 codes with one fp32 scale:
  amax = max |x|, scale = amax / 127 (1 / 127 when amax is 0),
  inv = 1 / scale, code = clamp(round(x * inv), -127, 127) with std::round
  (half away from zero) -- all in fp32 (1545-1573);
* fused_gqa_attention_decode_paged (1686-1930): query head h reads kv head
  h / (heads / kv_heads); score = dot(q, k) * scale, or in Q8 mode
  (dot(q, codes) * k_scale) * scale (1790-1812); a position whose page does
  not exist scores -1e9 and adds no value (1793-1795, 1896-1897); the
  output is sum_j p_j v_j / sum_j p_j with p_j = exp(score_j - max), the
  value term p_j * v_scale * codes_j in Q8 mode (1894-1915).
Arithmetic of the attention is float64 (the reference's fast_exp and its
tile-wise online softmax agree with the exact softmax to rounding); the Q8
quantizer is fp32 like the reference's.

The quantizer is pinned by known answers in tests/test_paged_kv_oracle.py
(round-half-away cases, the all-zero row, clamping); the attention has no
reference vectors to pin against (parity of the restatement rests on the
formulas cited above).
"""

from __future__ import annotations

import numpy as np

MASKED_SCORE = -1e9


def q8_row(x: np.ndarray):
    """(codes int8 [d], scale fp32) of one row, as PagedKVStore::write
    computes them (model_graph.cpp:1552-1572)."""
    x = np.asarray(x, dtype=np.float32)
    amax = np.float32(np.max(np.abs(x))) if x.size else np.float32(0)
    scale = np.float32(amax / np.float32(127.0)) if amax > 0 else np.float32(np.float32(1.0) / np.float32(127.0))
    inv = np.float32(np.float32(1.0) / scale)
    prod = (x * inv).astype(np.float32)
    # std::round: half away from zero (float64 holds |prod| + 0.5 exactly)
    r = np.sign(prod).astype(np.float64) * np.floor(np.abs(prod).astype(np.float64) + 0.5)
    return np.clip(r, -127, 127).astype(np.int8), scale


def q8_rows(x: np.ndarray):
    """q8_row over the last axis: (codes [..., d] int8, scales [...] fp32)."""
    x = np.asarray(x, dtype=np.float32)
    flat = x.reshape(-1, x.shape[-1])
    out = [q8_row(r) for r in flat]
    codes = np.stack([c for c, _ in out]).reshape(x.shape)
    scales = np.asarray([s for _, s in out], dtype=np.float32).reshape(x.shape[:-1])
    return codes, scales


def rope(v: np.ndarray, pos: int, theta: float) -> np.ndarray:
    """apply_rope_with_dim (model_graph.cpp:1222-1323): interleaved pairs
    (2p, 2p + 1) of each head's last axis rotated by pos * theta^(-2p / d);
    float64."""
    v = np.asarray(v, dtype=np.float64).copy()
    d = v.shape[-1]
    p = np.arange(d // 2)
    ang = pos * theta ** (-2.0 * p / d)
    c, s = np.cos(ang), np.sin(ang)
    x0, x1 = v[..., 0::2].copy(), v[..., 1::2].copy()
    v[..., 0::2] = x0 * c - x1 * s
    v[..., 1::2] = x0 * s + x1 * c
    return v


class PagedKVStoreRef:
    """One sequence's PagedKVStore for `layers` layers.

    Float mode stores rows as `store_dtype` (the reference: float32; pass
    float16 to model a cache of that precision)."""

    def __init__(self, layers: int, kv_heads: int, head_dim: int, max_seq: int, page_size: int, q8: bool,
                 store_dtype=np.float32):
        self.layers, self.kv_heads, self.hd = layers, kv_heads, head_dim
        self.page_size, self.q8 = page_size, q8
        self.total_pages = (max_seq + page_size - 1) // page_size
        self.store_dtype = store_dtype
        self.pages: dict[tuple[int, int], dict] = {}  # (layer, page) -> arrays, lazily

    def ensure_page(self, layer: int, page: int) -> dict:
        key = (layer, page)
        if key not in self.pages:
            P, H, D = self.page_size, self.kv_heads, self.hd
            if self.q8:
                self.pages[key] = {"k": np.zeros((P, H, D), np.int8), "v": np.zeros((P, H, D), np.int8),
                                   "ks": np.ones((P, H), np.float32), "vs": np.ones((P, H), np.float32)}
            else:
                self.pages[key] = {"k": np.zeros((P, H, D), self.store_dtype),
                                   "v": np.zeros((P, H, D), self.store_dtype)}
        return self.pages[key]

    def drop_page(self, layer: int, page: int) -> None:
        self.pages.pop((layer, page), None)

    def write(self, layer: int, pos: int, k: np.ndarray, v: np.ndarray) -> None:
        """k, v: [kv_heads][head_dim] (k already rotated)."""
        pg = self.ensure_page(layer, pos // self.page_size)
        o = pos % self.page_size
        if self.q8:
            pg["k"][o], pg["ks"][o] = q8_rows(k)
            pg["v"][o], pg["vs"][o] = q8_rows(v)
        else:
            pg["k"][o] = np.asarray(k, np.float32).astype(self.store_dtype)
            pg["v"][o] = np.asarray(v, np.float32).astype(self.store_dtype)

    def set_row(self, layer: int, pos: int, k, v, ks=None, vs=None) -> None:
        """Store rows as given (codes and scales in Q8 mode)."""
        pg = self.ensure_page(layer, pos // self.page_size)
        o = pos % self.page_size
        pg["k"][o], pg["v"][o] = k, v
        if self.q8:
            pg["ks"][o], pg["vs"][o] = ks, vs

    def gather(self, layer: int, kv_len: int):
        """Rows of positions 0..kv_len-1 as float64 arrays: keys, values
        [kv_len][kv_heads][head_dim], key / value scales [kv_len][kv_heads]
        (ones in float mode), and which positions have a page."""
        H, D, P = self.kv_heads, self.hd, self.page_size
        K = np.zeros((kv_len, H, D))
        V = np.zeros((kv_len, H, D))
        KS = np.ones((kv_len, H))
        VS = np.ones((kv_len, H))
        present = np.zeros(kv_len, bool)
        for pg in range((kv_len + P - 1) // P):
            page = self.pages.get((layer, pg))
            if page is None:
                continue
            j0, j1 = pg * P, min(kv_len, (pg + 1) * P)
            n = j1 - j0
            K[j0:j1] = page["k"][:n]
            V[j0:j1] = page["v"][:n]
            if self.q8:
                KS[j0:j1] = page["ks"][:n]
                VS[j0:j1] = page["vs"][:n]
            present[j0:j1] = True
        return K, V, KS, VS, present

    def attention(self, layer: int, q: np.ndarray, kv_len: int) -> np.ndarray:
        """q: [heads][head_dim] (rotated). Returns [heads][head_dim] float64."""
        Hq, D = q.shape
        G = Hq // self.kv_heads
        K, V, KS, VS, present = self.gather(layer, kv_len)
        out = np.zeros((Hq, D))
        for h in range(Hq):
            kvh = min(self.kv_heads - 1, h // G)
            sc = (K[:, kvh] @ q[h].astype(np.float64)) * KS[:, kvh] / np.sqrt(D)
            sc[~present] = MASKED_SCORE
            p = np.exp(sc - sc.max())
            w = np.where(present, p * VS[:, kvh], 0.0)
            out[h] = (w @ V[:, kvh]) / p.sum()
        return out
