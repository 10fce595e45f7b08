"""CPU restatement of one single-token decode step -- TEST INFRASTRUCTURE ONLY.

Follows the reference decode graph (JSBuild/src/verso/Anvil/core/native/
model_graph.cpp): rmsnorm_inplace (674-693: x / sqrt(mean(x^2) + eps) *
gamma), the q/k/v projections, apply_rope_with_dim (1222-1323: interleaved
pairs (2p, 2p+1) rotated by pos * theta^(-2p / head_dim)), GQA attention of
the token over the cache (softmax(q . k / sqrt(head_dim)) v, query head h on
kv head h / (heads / kv_heads)), the o projection and residual add, RMSNorm,
the SwiGLU FFN (silu(gate) * up, down) and residual add, the final norm and
the LM head. Weights are the reference's fp32 dequantized values
(orc_dequant_rows); arithmetic is float64, except that cached k and v are
rounded to fp16 as the device cache stores them, or (DecodeRef with kv_q8)
stored as the reference's Q8 KV rows (PagedKVStore::write,
model_graph.cpp:1545-1573).

Only the tests import this module.
"""

from __future__ import annotations

import numpy as np

from . import oracle as O


def _stored(rows, q8: bool) -> np.ndarray:
    """KV rows as the cache holds them: fp16 values, or Q8 codes * scale."""
    if not q8:
        return rows.astype(np.float16).astype(np.float64)
    from .paged_kv_ref import q8_rows

    codes, scales = q8_rows(rows.astype(np.float32))
    return codes.astype(np.float64) * scales[..., None].astype(np.float64)


class DecodeRef:
    def __init__(self, shape, layers, embed, head, out_norm, max_ctx: int, kv_q8: bool = False):
        """kv_q8: the cache holds the reference's Q8 rows (codes * scale, the
        quantizer of oracle/paged_kv_ref.py) instead of fp16 values."""
        self.s = shape
        self.max_ctx = max_ctx
        self.kv_q8 = kv_q8
        h, kv, f = shape.hidden, shape.kv_dim, shape.ffn
        q = shape.linear_qtype
        dims = {"wq": (h, h), "wk": (kv, h), "wv": (kv, h), "wo": (h, h), "w_gate": (f, h), "w_up": (f, h),
                "w_down": (h, f)}
        self.layers = []
        for i in range(shape.layers):
            src = layers[i % len(layers)]
            lay = {name: O.dequant(src[name], q, k, n).astype(np.float64) for name, (n, k) in dims.items()}
            lay["attn_norm"] = src["attn_norm"].astype(np.float64)
            lay["ffn_norm"] = src["ffn_norm"].astype(np.float64)
            self.layers.append(lay)
        self.embed = O.dequant(embed, shape.embedding_qtype, h, shape.vocab).astype(np.float64)
        self.head = O.dequant(head, shape.head_qtype, h, shape.vocab).astype(np.float64)
        self.out_norm = out_norm.astype(np.float64)
        hd = shape.head_dim
        self.kc = np.zeros((shape.layers, shape.kv_heads, max_ctx, hd))
        self.vc = np.zeros((shape.layers, shape.kv_heads, max_ctx, hd))

    def _rms(self, x, g):
        return x / np.sqrt(np.mean(x * x) + self.s.eps) * g

    def _rope(self, v, heads, pos):
        hd = self.s.head_dim
        p = np.arange(hd // 2)
        ang = pos * self.s.rope_theta ** (-2.0 * p / hd)
        c, s = np.cos(ang), np.sin(ang)
        v = v.reshape(heads, hd).copy()
        x0, x1 = v[:, 0::2].copy(), v[:, 1::2].copy()
        v[:, 0::2] = x0 * c - x1 * s
        v[:, 1::2] = x0 * s + x1 * c
        return v

    def step(self, token: int, pos: int) -> np.ndarray:
        s = self.s
        hd, G = s.head_dim, s.heads // s.kv_heads
        x = self.embed[token].copy()
        for li, L in enumerate(self.layers):
            hn = self._rms(x, L["attn_norm"])
            q = self._rope(L["wq"] @ hn, s.heads, pos)
            k = self._rope(L["wk"] @ hn, s.kv_heads, pos)
            v = (L["wv"] @ hn).reshape(s.kv_heads, hd)
            self.kc[li, :, pos] = _stored(k, self.kv_q8)
            self.vc[li, :, pos] = _stored(v, self.kv_q8)
            att = np.zeros((s.heads, hd))
            for hh in range(s.heads):
                kvh = hh // G
                sc = self.kc[li, kvh, : pos + 1] @ q[hh] / np.sqrt(hd)
                e = np.exp(sc - sc.max())
                att[hh] = (e / e.sum()) @ self.vc[li, kvh, : pos + 1]
            x = x + L["wo"] @ att.reshape(-1)
            hn = self._rms(x, L["ffn_norm"])
            g, u = L["w_gate"] @ hn, L["w_up"] @ hn
            x = x + L["w_down"] @ (g / (1.0 + np.exp(-g)) * u)
        return self.head @ self._rms(x, self.out_norm)


class DecodeRefPacked:
    """The same decode step for `batch` sequences at one position, with the
    linears computed straight from the packed weights (orc_matvec_f64: the
    reference's fp32 dequantized values, double accumulation, activations
    rounded to fp32 at each linear's input) instead of dequantized copies, so
    full-width layers (hidden 8192, FFN 28672) fit in host memory. k/v caches
    are [batch][layer][kv_head][max_ctx][head_dim] float64 holding fp16 values;
    ``load_cache`` fills them from the device caches' values."""

    def __init__(self, shape, layers, embed, head, out_norm, max_ctx: int, batch: int = 1):
        self.s = shape
        self.max_ctx = max_ctx
        self.batch = batch
        self.layers = [layers[i % len(layers)] for i in range(shape.layers)]
        self.embed, self.head, self.out_norm = embed, head, out_norm.astype(np.float64)
        hd = shape.head_dim
        self.kc = np.zeros((batch, shape.layers, shape.kv_heads, max_ctx, hd))
        self.vc = np.zeros_like(self.kc)

    def load_cache(self, k_cache, v_cache) -> None:
        """k_cache / v_cache: arrays [batch][layer][kv_head][ctx][hd] (any float type)."""
        c = np.asarray(k_cache).shape[3]
        self.kc[:, :, :, :c] = np.asarray(k_cache, dtype=np.float64)
        self.vc[:, :, :, :c] = np.asarray(v_cache, dtype=np.float64)

    def _lin(self, W, qt, X, k, n):
        return O.matvec_f64(W, qt, np.ascontiguousarray(X, dtype=np.float32), k, n)

    def _rms(self, X, g):
        return X / np.sqrt(np.mean(X * X, axis=1, keepdims=True) + self.s.eps) * g.astype(np.float64)

    def _rope(self, v, heads, pos):
        hd = self.s.head_dim
        p = np.arange(hd // 2)
        ang = pos * self.s.rope_theta ** (-2.0 * p / hd)
        c, s = np.cos(ang), np.sin(ang)
        v = v.reshape(-1, heads, hd).copy()
        x0, x1 = v[..., 0::2].copy(), v[..., 1::2].copy()
        v[..., 0::2] = x0 * c - x1 * s
        v[..., 1::2] = x0 * s + x1 * c
        return v

    def step(self, tokens, pos: int) -> np.ndarray:
        """Logits [batch][vocab] after appending tokens[b] at position pos."""
        s, B = self.s, self.batch
        h, kv, f, hd, G = s.hidden, s.kv_dim, s.ffn, s.head_dim, s.heads // s.kv_heads
        q_t = s.linear_qtype
        X = O.dequant(self.embed, s.embedding_qtype, h, s.vocab)[np.asarray(tokens)].astype(np.float64)
        for li, L in enumerate(self.layers):
            hn = self._rms(X, L["attn_norm"])
            q = self._rope(self._lin(L["wq"], q_t, hn, h, h), s.heads, pos)
            k = self._rope(self._lin(L["wk"], q_t, hn, h, kv), s.kv_heads, pos)
            v = self._lin(L["wv"], q_t, hn, h, kv).reshape(B, s.kv_heads, hd)
            self.kc[:, li, :, pos] = k.astype(np.float16).astype(np.float64)
            self.vc[:, li, :, pos] = v.astype(np.float16).astype(np.float64)
            att = np.zeros((B, s.heads, hd))
            for b in range(B):
                for hh in range(s.heads):
                    kvh = hh // G
                    sc = self.kc[b, li, kvh, : pos + 1] @ q[b, hh] / np.sqrt(hd)
                    e = np.exp(sc - sc.max())
                    att[b, hh] = (e / e.sum()) @ self.vc[b, li, kvh, : pos + 1]
            X = X + self._lin(L["wo"], q_t, att.reshape(B, -1), h, h)
            hn = self._rms(X, L["ffn_norm"])
            g, u = self._lin(L["w_gate"], q_t, hn, h, f), self._lin(L["w_up"], q_t, hn, h, f)
            X = X + self._lin(L["w_down"], q_t, g / (1.0 + np.exp(-g)) * u, f, h)
        return self._lin(self.head, s.head_qtype, self._rms(X, self.out_norm), h, s.vocab)
