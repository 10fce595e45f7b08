"""Paged KV cache on the device: the reference's PagedKVStore, B200-side.

The reference keeps each layer's keys and values in pages of KV_PAGE_SIZE
(4096) positions, allocated when a position of the page is first written
(JSBuild/src/verso/Anvil/core/native/model_graph.cpp:317, 1413-1576), in
fp32 or -- with ANVIL_KV_QUANT set (model_graph.cpp:507-513) -- as int8 codes
with one fp32 scale per (position, kv head). It resets (graph_reset,
model_graph.cpp:5191-5193) and snapshots / restores its pages with a graph
execution checkpoint (model_graph.cpp:4725-4776).

Here every page lives in one preallocated pool per cache (keys, values and,
in Q8 mode, their scales), and a page table ``[layer][sequence][page]`` of
int32 slots (-1: no page) tells the attention kernel
(b200q_rope_attention_decode_paged) where each position is. Pages of a
sequence are assigned from a free list when ``ensure(pos)`` first meets them,
so the pool can be smaller than layers x sequences x max_seq positions. fp16
replaces the reference's fp32 pages (the contiguous decode cache stores fp16
too); Q8 pages hold the reference's codes and scales exactly.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Mapping

import numpy as np

from . import _native

KV_PAGE_SIZE = 4096  # positions per page (model_graph.cpp:317)
HEAD_DIM = 128       # the attention kernels' head size


def q8_from_env(env: Mapping[str, str] | None = None) -> bool:
    """The reference's use_q8_kv_cache (model_graph.cpp:468-513): on for
    ANVIL_KV_QUANT=q8 or any non-empty value other than 0 / false / off."""
    env = os.environ if env is None else env
    v = env.get("ANVIL_KV_QUANT")
    if v is None or v == "":
        return False
    return v == "q8" or v not in ("0", "false", "off")


@dataclass
class KVSnapshot:
    """A copy of a cache's pages and page table (graph_create_execution_checkpoint)."""

    k: object
    v: object
    ks: object
    vs: object
    table: np.ndarray
    free: list


class PagedKVCache:
    """Pools of ``n_slots`` pages for ``layers`` layers of ``batch`` sequences.

    Pool layout (device): keys / values ``[n_slots][kv_heads][page_size]
    [head_dim]`` fp16, or int8 codes with fp32 scales ``[n_slots][kv_heads]
    [page_size]`` when ``q8``. ``table`` (device, int32) is
    ``[layers][batch][pages_per_seq]``; ``table_host`` mirrors it.
    """

    def __init__(self, layers: int, kv_heads: int, max_seq: int, batch: int = 1, page_size: int = KV_PAGE_SIZE,
                 q8: bool | None = None, n_slots: int | None = None, device: int | str = 0,
                 head_dim: int = HEAD_DIM):
        """``device``: a CUDA ordinal, or a torch device string ("cpu" holds
        the pools on the host: page bookkeeping only, no attention calls)."""
        import torch

        if head_dim != HEAD_DIM:
            raise ValueError("the attention kernels are built for head_dim 128")
        if min(layers, kv_heads, max_seq, batch, page_size) <= 0:
            raise ValueError("layers, kv_heads, max_seq, batch and page_size must be positive")
        self.layers, self.kv_heads, self.batch = layers, kv_heads, batch
        self.max_seq, self.page_size, self.head_dim = max_seq, page_size, head_dim
        self.q8 = q8_from_env() if q8 is None else bool(q8)
        self.pages_per_seq = (max_seq + page_size - 1) // page_size
        full = layers * batch * self.pages_per_seq
        self.n_slots = full if n_slots is None else int(n_slots)
        if self.n_slots <= 0:
            raise ValueError("n_slots must be positive")
        self.dev = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        shape = (self.n_slots, kv_heads, page_size, head_dim)
        dt = torch.int8 if self.q8 else torch.float16
        self.k = torch.zeros(shape, dtype=dt, device=self.dev)
        self.v = torch.zeros(shape, dtype=dt, device=self.dev)
        if self.q8:  # fresh pages hold scale 1 (model_graph.cpp:1500-1501)
            self.ks = torch.ones(shape[:3], dtype=torch.float32, device=self.dev)
            self.vs = torch.ones(shape[:3], dtype=torch.float32, device=self.dev)
        else:
            self.ks = self.vs = None
        self.table_host = np.full((layers, batch, self.pages_per_seq), -1, dtype=np.int32)
        self.table = torch.from_numpy(self.table_host).to(self.dev)
        self._free = list(range(self.n_slots - 1, -1, -1))  # pop() hands out slot 0 first

    # -- page assignment -------------------------------------------------------
    @property
    def kv_mode(self) -> int:
        return _native.KV_Q8 if self.q8 else _native.KV_F16

    @property
    def pages_in_use(self) -> int:
        return self.n_slots - len(self._free)

    @property
    def page_bytes(self) -> int:
        per = self.kv_heads * self.page_size
        return 2 * per * (self.head_dim + 4 if self.q8 else 2 * self.head_dim)

    def ensure(self, pos: int, last: int | None = None) -> None:
        """Give every layer and sequence a page for positions pos .. last
        (default pos), as ensure_page does when the reference writes a
        position (model_graph.cpp:1473-1522); copies the table to the device
        on the current stream when it changed. Raises MemoryError when the
        pool has no free page."""
        import torch

        last = pos if last is None else last
        if not 0 <= pos <= last < self.max_seq:
            raise ValueError("position outside the cache")
        pages = slice(pos // self.page_size, last // self.page_size + 1)
        need = int((self.table_host[:, :, pages] < 0).sum())
        if need == 0:
            return
        if need > len(self._free):  # nothing is assigned then
            raise MemoryError(f"KV page pool exhausted ({self.n_slots} pages, {len(self._free)} free, {need} needed)")
        for p in range(pages.start, pages.stop):
            for li, b in np.argwhere(self.table_host[:, :, p] < 0):
                self.table_host[li, b, p] = self._free.pop()
        self.table.copy_(torch.from_numpy(self.table_host))

    def assign(self, layer: int, seq: int, page: int, slot: int) -> None:
        """Place page `page` of sequence `seq` in layer `layer` at pool slot
        `slot` (for callers that choose placement themselves, e.g. pages
        shared between sequences); the table reaches the device with
        ``sync_table``."""
        if not 0 <= slot < self.n_slots:
            raise ValueError("slot outside the pool")
        if slot in self._free:
            self._free.remove(slot)
        old = int(self.table_host[layer, seq, page])
        self.table_host[layer, seq, page] = slot
        if old >= 0 and old != slot and not (self.table_host == old).any():
            self._free.append(old)  # the page it replaced is referenced nowhere else

    def sync_table(self) -> None:
        """Copy the host page table to the device (current stream)."""
        import torch

        self.table.copy_(torch.from_numpy(self.table_host))

    def reset(self) -> None:
        """Drop every page (graph_reset, model_graph.cpp:5191-5193)."""
        import torch

        self.table_host.fill(-1)
        self._free = list(range(self.n_slots - 1, -1, -1))
        self.table.copy_(torch.from_numpy(self.table_host))

    def snapshot(self) -> KVSnapshot:
        """Device copies of the pools and a copy of the table."""
        c = (lambda t: None if t is None else t.clone())
        return KVSnapshot(c(self.k), c(self.v), c(self.ks), c(self.vs), self.table_host.copy(), list(self._free))

    def restore(self, snap: KVSnapshot) -> None:
        import torch

        self.k.copy_(snap.k)
        self.v.copy_(snap.v)
        if self.q8:
            self.ks.copy_(snap.ks)
            self.vs.copy_(snap.vs)
        self.table_host[...] = snap.table
        self._free = list(snap.free)
        self.table.copy_(torch.from_numpy(self.table_host))

    # -- kernel arguments ------------------------------------------------------
    def table_ptr(self, layer: int) -> int:
        return self.table.data_ptr() + 4 * layer * self.batch * self.pages_per_seq

    def attention(self, layer: int, q: int, k: int, v: int, pos: int, n_heads: int, theta: float, out: int | None,
                  xq: int | None, act_mode: int, stream: int, n_tokens: int = 1, q_stride: int = 0,
                  kv_stride: int = 0) -> None:
        """RoPE + append + attention of layer `layer` for n_tokens
        consecutive tokens of every sequence, token t at pos + t attending
        over 0..pos + t (device pointers; q [batch][n_tokens][n_heads][128], k
        and v [batch][n_tokens][kv_heads][128], or rows q_stride / kv_stride
        floats apart); the pages of those positions must have been ensured."""
        if self.dev.type != "cuda":
            raise RuntimeError("the paged attention runs on a CUDA device")
        L = _native.lib()
        ks = self.ks.data_ptr() if self.q8 else None
        vs = self.vs.data_ptr() if self.q8 else None
        _native.check(L.b200q_rope_attention_decode_paged(
            q, k, v, self.batch, n_tokens, n_heads, self.kv_heads, self.head_dim, pos, theta, self.kv_mode, self.k.data_ptr(),
            self.v.data_ptr(), ks, vs, self.n_slots, self.page_size, self.table_ptr(layer), self.pages_per_seq, out,
            xq, act_mode, q_stride, kv_stride, stream), "paged attention")

    def rows(self, layer: int, seq: int, kv_head: int, p0: int, p1: int):
        """Stored (codes or fp16 values, scales or None) of positions p0..p1-1
        (host arrays; for tests and inspection)."""
        import torch

        pos = np.arange(p0, p1)
        slots = self.table_host[layer, seq, pos // self.page_size]
        if (slots < 0).any():
            raise ValueError("a position without a page")
        si = torch.from_numpy(slots.astype(np.int64)).to(self.dev)
        oi = torch.from_numpy(pos % self.page_size).to(self.dev)
        kc, vc = self.k[si, kv_head, oi].cpu().numpy(), self.v[si, kv_head, oi].cpu().numpy()
        if not self.q8:
            return kc, vc, None, None
        return kc, vc, self.ks[si, kv_head, oi].cpu().numpy(), self.vs[si, kv_head, oi].cpu().numpy()
