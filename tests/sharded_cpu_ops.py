"""CPU (float64 numpy) arithmetic for ShardedDecode -- test helper only.

Same method set as cybel_b200.sharded.GpuOps, restating each step the way
oracle/decode_ref.py does (the reference's fp32 dequantized weights, fp16
cache rounding), with the all-gathers done by torch.distributed over gloo.
It lets the sharding orchestration (row slices, head ownership, gather
layout for batch > 1) run as several CPU ranks and be compared with the
unsharded restatement.
"""

from __future__ import annotations

import numpy as np

from oracle import oracle as O


class NumpyOps:
    def __init__(self, world: int = 1, group=None):
        self.world = world
        self.group = group

    def zeros(self, n):
        return np.zeros(n)

    def gather_target(self, name, n):
        return np.zeros(n)

    def vector(self, a):
        return np.asarray(a, dtype=np.float64).copy()

    def matrix(self, qtype, k, n_rows, packed):
        return O.dequant(packed, qtype, k, n_rows).astype(np.float64)

    def cache(self, layers, batch, kv_heads, max_ctx, hd):
        shape = (layers, batch, kv_heads, max_ctx, hd)
        return np.zeros(shape), np.zeros(shape)

    def cache_layer(self, cache, li):
        return cache[li]

    def tokens(self, batch):
        return np.zeros(batch, dtype=np.int64)

    def embed(self, m, tokens, out, batch, hidden, vocab):
        for b in range(batch):
            out[b * hidden:(b + 1) * hidden] = m[int(tokens[b])]

    def codes(self, rows, k):
        # the restatement keeps activations in float64 (no quantization)
        return np.zeros(rows * k)

    def quantize(self, x, xq, rows, k):
        xq[: rows * k] = x[: rows * k]

    def linear_codes(self, m, xq, out, batch, k, n_rows):
        out[: batch * n_rows] = (xq[: batch * k].reshape(batch, k) @ m.T).reshape(-1)

    def linear_norm(self, m, x, gamma, out, k, n_rows, eps):
        xn = x[:k] / np.sqrt(np.mean(x[:k] * x[:k]) + eps) * gamma
        out[:n_rows] = m @ xn

    def linear_codes_add(self, m, xq, out, k, n_rows):
        out[:n_rows] += m @ xq[:k]

    def norm_codes(self, res, delta, gamma, xq, n, rows, eps):
        for r in range(rows):
            sl = slice(r * n, (r + 1) * n)
            if delta is not None:
                res[sl] += delta[sl]
            x = res[sl]
            xq[sl] = x / np.sqrt(np.mean(x * x) + eps) * gamma

    def norm_f32(self, res, delta, gamma, out, n, rows, eps):
        self.norm_codes(res, delta, gamma, out, n, rows, eps)

    def linear_f32(self, m, x, out, batch, k, n_rows):
        self.linear_codes(m, x, out, batch, k, n_rows)

    def rope_kv(self, q, k, v, batch, heads, kv_heads, hd, pos, theta, kc, vc, max_ctx):
        p = np.arange(hd // 2)
        ang = pos * theta ** (-2.0 * p / hd)
        c, s = np.cos(ang), np.sin(ang)

        def rot(vec, nh):
            a = vec.reshape(nh, hd)
            x0, x1 = a[:, 0::2].copy(), a[:, 1::2].copy()
            a[:, 0::2] = x0 * c - x1 * s
            a[:, 1::2] = x0 * s + x1 * c

        for b in range(batch):
            qb = q[b * heads * hd:(b + 1) * heads * hd]
            kb = k[b * kv_heads * hd:(b + 1) * kv_heads * hd]
            vb = v[b * kv_heads * hd:(b + 1) * kv_heads * hd]
            rot(qb, heads)
            rot(kb, kv_heads)
            kc[b, :, pos] = kb.reshape(kv_heads, hd).astype(np.float16).astype(np.float64)
            vc[b, :, pos] = vb.reshape(kv_heads, hd).astype(np.float16).astype(np.float64)

    def attention(self, q, kc, vc, out, batch, heads, kv_heads, hd, ctx, max_ctx):
        G = heads // kv_heads
        for b in range(batch):
            for h in range(heads):
                qh = q[(b * heads + h) * hd:(b * heads + h + 1) * hd]
                sc = kc[b, h // G, :ctx] @ qh / np.sqrt(hd)
                e = np.exp(sc - sc.max())
                out[(b * heads + h) * hd:(b * heads + h + 1) * hd] = (e / e.sum()) @ vc[b, h // G, :ctx]

    def rope_attention(self, q, k, v, batch, heads, kv_heads, hd, pos, theta, kc, vc, max_ctx, out, xq):
        q, k = q.copy(), k.copy()  # the fused kernel rotates without writing q and k back
        self.rope_kv(q, k, v, batch, heads, kv_heads, hd, pos, theta, kc, vc, max_ctx)
        o = out if out is not None else np.zeros(batch * heads * hd)
        self.attention(q, kc, vc, o, batch, heads, kv_heads, hd, pos + 1, max_ctx)
        if xq is not None:
            self.quantize(o, xq, batch, heads * hd)

    def swiglu_codes(self, g, u, xq, n):
        f = np.zeros(n)
        self.swiglu(g, u, f, n)
        self.quantize(f, xq, 1, n)

    def swiglu(self, g, u, out, n):
        out[:n] = g[:n] / (1.0 + np.exp(-g[:n])) * u[:n]

    def all_gather(self, full, local, gbuf, batch, n_local, codes=None):
        import torch
        import torch.distributed as dist

        parts = [torch.zeros(batch * n_local, dtype=torch.float64) for _ in range(self.world)]
        dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(local[: batch * n_local])), group=self.group)
        n = self.world * n_local
        for g, t in enumerate(parts):
            blk = t.numpy().reshape(batch, n_local)
            for b in range(batch):
                full[b * n + g * n_local:b * n + (g + 1) * n_local] = blk[b]
        if codes is not None:
            codes[: batch * n] = full[: batch * n]
