"""Output-row-sharded decode across the GPUs of one node (one process per GPU).

Every linear of the stack is split by output rows: rank g of G holds rows
[g * n / G, (g + 1) * n / G) of each matrix, resident in its own HBM, and the
partial outputs are all-gathered (NCCL over NVLink / NVSwitch) before the
next consumer that needs the full vector. The q/k/v row slices are whole
heads (q heads g * H/G.., kv heads g * KV/G..; G divides KV), so RoPE, the
KV cache and attention stay local to the rank that owns the heads. Per layer
the gathers are: the attention output (input of the o projection), the o
projection (the residual), the SwiGLU hidden vector (input of the down
projection) and the down projection (the residual); one more gathers the
logits. Norms and the residual stream are replicated on every rank.

``ShardedDecode`` holds that orchestration once; the arithmetic comes from
an ops object: ``GpuOps`` (libb200q kernels + torch.distributed NCCL) on the
device, or a CPU restatement in the tests, which checks the same
orchestration with gloo ranks.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import _native
from .decode import StackShape, layer_matrix_shapes


@dataclass(frozen=True)
class ShardPlan:
    shape: StackShape
    world: int
    rank: int

    def __post_init__(self):
        s, G = self.shape, self.world
        if G < 1 or not 0 <= self.rank < G:
            raise ValueError("bad rank / world size")
        for what, v in (("heads", s.heads), ("kv_heads", s.kv_heads), ("hidden", s.hidden), ("ffn", s.ffn),
                        ("vocab", s.vocab)):
            if v % G:
                raise ValueError(f"{what} = {v} is not divisible by {G} ranks")

    @property
    def heads(self) -> int:
        return self.shape.heads // self.world

    @property
    def kv_heads(self) -> int:
        return self.shape.kv_heads // self.world

    def local_rows(self, name: str) -> int:
        n = layer_matrix_shapes(self.shape)[name][0] if name != "head" else self.shape.vocab
        return n // self.world

    def row_range(self, name: str) -> tuple[int, int]:
        """Rows of matrix `name` ("head" for the LM head) this rank owns."""
        n_l = self.local_rows(name)
        return self.rank * n_l, (self.rank + 1) * n_l


def shard_rows(packed: np.ndarray, plan: ShardPlan, name: str) -> np.ndarray:
    """This rank's rows of a packed row-major matrix (canonical layouts: a
    row's blocks are contiguous, so a row range is a byte range)."""
    r0, r1 = plan.row_range(name)
    return np.ascontiguousarray(packed[r0:r1])


def shard_layer(layer: dict[str, np.ndarray], plan: ShardPlan) -> dict[str, np.ndarray]:
    out = {name: shard_rows(layer[name], plan, name) for name in layer_matrix_shapes(plan.shape)}
    out["attn_norm"] = layer["attn_norm"]
    out["ffn_norm"] = layer["ffn_norm"]
    return out


class ShardedDecode:
    """One rank's part of a row-sharded single-token decode of ``batch``
    sequences (all at the same position).

    layers: this rank's shards (``shard_layer``) of one weight dict per layer;
    a shorter list is cycled (each layer still gets its own copy); embed: the
    full packed embedding (replicated); head: this rank's rows of the LM head.
    With batch 1 a layer's local q/k/v rows are one matrix and its local
    gate/up rows another (one GEMV each). Norms write the GEMVs' activation
    codes, and the gathers of the attention output and of the SwiGLU vector
    deliver codes of the gathered rows, so no projection quantizes by itself.
    From ``TILE_MIN_BATCH`` sequences on (``tile``), the activations stay
    fp32 and every Q4_K linear runs on the tile path (tcgen05, the weights
    streamed once for the whole batch; other qtypes take the GEMV).
    """

    TILE_MIN_BATCH = 8

    def __init__(self, plan: ShardPlan, max_ctx: int, batch: int, layers, embed, head, out_norm, ops,
                 fuse_norm: bool | None = None, tile: bool | None = None):
        s = plan.shape
        self.plan, self.shape, self.ops = plan, s, ops
        self.max_ctx, self.batch = max_ctx, batch
        B, G, hd = batch, plan.world, s.head_dim
        self.fused = batch == 1
        if tile is None:
            tile = batch >= self.TILE_MIN_BATCH
        self.tile = bool(tile) and batch > 1 and hasattr(ops, "linear_f32")
        h, h_l, f_l = s.hidden, s.hidden // G, s.ffn // G
        q_l, kv_l = plan.heads * hd, plan.kv_heads * hd
        self.q_l, self.kv_l, self.f_l = q_l, kv_l, f_l
        qt = s.linear_qtype
        self.layers = []
        for li in range(s.layers):
            src = layers[li % len(layers)]
            if li >= len(layers) and hasattr(ops, "clone_matrix"):
                base = self.layers[li % len(layers)]
                lay = {k: (ops.clone_matrix(v) if k not in ("attn_norm", "ffn_norm") else v) for k, v in base.items()}
                self.layers.append(lay)
                continue
            lay = {"wo": ops.matrix(qt, h, h_l, src["wo"]), "w_down": ops.matrix(qt, s.ffn, h_l, src["w_down"]),
                   "attn_norm": ops.vector(src["attn_norm"]), "ffn_norm": ops.vector(src["ffn_norm"])}
            if self.fused:
                lay["wqkv"] = ops.matrix(qt, h, q_l + 2 * kv_l, np.concatenate([src["wq"], src["wk"], src["wv"]]))
                lay["w_gu"] = ops.matrix(qt, h, 2 * f_l, np.concatenate([src["w_gate"], src["w_up"]]))
            else:
                for name, n in (("wq", q_l), ("wk", kv_l), ("wv", kv_l), ("w_gate", f_l), ("w_up", f_l)):
                    lay[name] = ops.matrix(qt, h, n, src[name])
            self.layers.append(lay)
        self.embed = ops.matrix(s.embedding_qtype, h, s.vocab, embed)
        self.head = ops.matrix(s.head_qtype, h, plan.local_rows("head"), head)
        self.out_norm = ops.vector(out_norm)
        self.k_cache, self.v_cache = ops.cache(s.layers, B, plan.kv_heads, max_ctx, hd)
        z = ops.zeros
        # Batch 1: each RMSNorm runs inside the projection after it
        # (ops.linear_norm), and the o / down projections add their rows into
        # this rank's slice of the residual (beta = 1), whose slices are then
        # all-gathered back into the full residual on every rank.
        # fuse_norm (default on) applies at batch 1; with several ranks the
        # residual gather runs in place (each rank's slice is its own input).
        if fuse_norm is None:
            fuse_norm = True
        self.norm_fused = bool(fuse_norm) and batch == 1 and hasattr(ops, "linear_norm")
        self.x = ops.gather_target("x", h) if (self.norm_fused and G > 1) else z(B * h)
        self.x_l = self.x[plan.rank * h_l:(plan.rank + 1) * h_l] if self.norm_fused else None
        self.xq_h = ops.codes(B, h)        # codes of a hidden vector (normed, or the gathered attention)
        self.xq_f = ops.codes(B, s.ffn)    # codes of the gathered SwiGLU vector
        if self.fused:
            self.qkv, self.gu = z(q_l + 2 * kv_l), z(2 * f_l)
            self.q, self.k, self.v = self.qkv[:q_l], self.qkv[q_l:q_l + kv_l], self.qkv[q_l + kv_l:]
            self.g_l, self.u_l = self.gu[:f_l], self.gu[f_l:]
        else:
            self.q, self.k, self.v = z(B * q_l), z(B * kv_l), z(B * kv_l)
            self.g_l, self.u_l = z(B * f_l), z(B * f_l)
        self.a_l, self.o_l, self.f_l_buf, self.d_l = z(B * q_l), z(B * h_l), z(B * f_l), z(B * h_l)
        self.logits_l = z(B * plan.local_rows("head"))
        if G > 1:
            t = ops.gather_target
            self.a, self.o, self.f, self.d = t("a", B * h), t("o", B * h), t("f", B * s.ffn), t("d", B * h)
            self.logits = t("logits", B * s.vocab)
        else:  # one rank: the local vectors are the whole vectors
            self.a, self.o, self.f, self.d, self.logits = self.a_l, self.o_l, self.f_l_buf, self.d_l, self.logits_l
        # with B > 1 and NCCL, an all-gather lands in [G][B][n/G] first
        self.gbuf = z(B * max(s.ffn, s.vocab)) if (B > 1 and G > 1) else None
        self.xn = z(B * h) if self.tile else None  # normalized rows, fp32 (tile mode)
        self.tokens = ops.tokens(B)

    def _gather(self, full, local, n_local, codes=None, k=None):
        if self.plan.world > 1:
            self.ops.all_gather(full, local, self.gbuf, self.batch, n_local, codes)
        elif codes is not None:
            self.ops.quantize(local, codes, self.batch, k)

    def step(self, pos: int) -> None:
        """Decode the tokens in ``self.tokens`` at position ``pos``; the full
        logits of every sequence land in ``self.logits`` ([batch][vocab])."""
        if self.norm_fused:
            self._step_norm_fused(pos)
            return
        if self.tile:
            self._step_tile(pos)
            return
        s, p, ops, B = self.shape, self.plan, self.ops, self.batch
        if not 0 <= pos < self.max_ctx:
            raise ValueError("position outside the KV cache")
        h, hd, G = s.hidden, s.head_dim, p.world
        ops.embed(self.embed, self.tokens, self.x, B, h, s.vocab)
        delta = None
        for li, lay in enumerate(self.layers):
            ops.norm_codes(self.x, delta, lay["attn_norm"], self.xq_h, h, B, s.eps)
            if self.fused:
                ops.linear_codes(lay["wqkv"], self.xq_h, self.qkv, 1, h, self.q_l + 2 * self.kv_l)
            else:
                for name, out, n in (("wq", self.q, self.q_l), ("wk", self.k, self.kv_l), ("wv", self.v, self.kv_l)):
                    ops.linear_codes(lay[name], self.xq_h, out, B, h, n)
            kc, vc = ops.cache_layer(self.k_cache, li), ops.cache_layer(self.v_cache, li)
            if G > 1:  # local heads' outputs, gathered (as codes) for the o projection
                ops.rope_attention(self.q, self.k, self.v, B, p.heads, p.kv_heads, hd, pos, s.rope_theta, kc, vc,
                                   self.max_ctx, self.a_l, None)
                self._gather(self.a, self.a_l, h // G, self.xq_h, h)
            else:  # one rank: the attention writes the o projection's codes itself
                ops.rope_attention(self.q, self.k, self.v, B, p.heads, p.kv_heads, hd, pos, s.rope_theta, kc, vc,
                                   self.max_ctx, None, self.xq_h)
            ops.linear_codes(lay["wo"], self.xq_h, self.o_l, B, h, h // G)
            self._gather(self.o, self.o_l, h // G)
            ops.norm_codes(self.x, self.o, lay["ffn_norm"], self.xq_h, h, B, s.eps)
            if self.fused:
                ops.linear_codes(lay["w_gu"], self.xq_h, self.gu, 1, h, 2 * self.f_l)
            else:
                ops.linear_codes(lay["w_gate"], self.xq_h, self.g_l, B, h, self.f_l)
                ops.linear_codes(lay["w_up"], self.xq_h, self.u_l, B, h, self.f_l)
            if G == 1 and B == 1:  # one rank: SwiGLU writes the down projection's codes itself
                ops.swiglu_codes(self.g_l, self.u_l, self.xq_f, self.f_l)
            else:
                ops.swiglu(self.g_l, self.u_l, self.f_l_buf, B * self.f_l)
                self._gather(self.f, self.f_l_buf, self.f_l, self.xq_f, s.ffn)
            ops.linear_codes(lay["w_down"], self.xq_f, self.d_l, B, s.ffn, h // G)
            self._gather(self.d, self.d_l, h // G)
            delta = self.d
        ops.norm_codes(self.x, delta, self.out_norm, self.xq_h, h, B, s.eps)
        ops.linear_codes(self.head, self.xq_h, self.logits_l, B, h, p.local_rows("head"))
        self._gather(self.logits, self.logits_l, p.local_rows("head"))


    def _step_tile(self, pos: int) -> None:
        """Batched step on fp32 activations: each norm writes fp32 rows, every
        linear takes all ``batch`` rows at once (the tile path for Q4_K), the
        attention writes fp32 outputs and the gathers move fp32 rows."""
        s, p, ops, B = self.shape, self.plan, self.ops, self.batch
        if not 0 <= pos < self.max_ctx:
            raise ValueError("position outside the KV cache")
        h, hd, G = s.hidden, s.head_dim, p.world
        h_l = h // G
        ops.embed(self.embed, self.tokens, self.x, B, h, s.vocab)
        delta = None
        for li, lay in enumerate(self.layers):
            ops.norm_f32(self.x, delta, lay["attn_norm"], self.xn, h, B, s.eps)
            for name, out, n in (("wq", self.q, self.q_l), ("wk", self.k, self.kv_l), ("wv", self.v, self.kv_l)):
                ops.linear_f32(lay[name], self.xn, out, B, h, n)
            kc, vc = ops.cache_layer(self.k_cache, li), ops.cache_layer(self.v_cache, li)
            ops.rope_attention(self.q, self.k, self.v, B, p.heads, p.kv_heads, hd, pos, s.rope_theta, kc, vc,
                               self.max_ctx, self.a_l, None)
            self._gather(self.a, self.a_l, h_l)
            ops.linear_f32(lay["wo"], self.a, self.o_l, B, h, h_l)
            self._gather(self.o, self.o_l, h_l)
            ops.norm_f32(self.x, self.o, lay["ffn_norm"], self.xn, h, B, s.eps)
            ops.linear_f32(lay["w_gate"], self.xn, self.g_l, B, h, self.f_l)
            ops.linear_f32(lay["w_up"], self.xn, self.u_l, B, h, self.f_l)
            ops.swiglu(self.g_l, self.u_l, self.f_l_buf, B * self.f_l)
            self._gather(self.f, self.f_l_buf, self.f_l)
            ops.linear_f32(lay["w_down"], self.f, self.d_l, B, s.ffn, h_l)
            self._gather(self.d, self.d_l, h_l)
            delta = self.d
        ops.norm_f32(self.x, delta, self.out_norm, self.xn, h, B, s.eps)
        ops.linear_f32(self.head, self.xn, self.logits_l, B, h, p.local_rows("head"))
        self._gather(self.logits, self.logits_l, p.local_rows("head"))

    def _step_norm_fused(self, pos: int) -> None:
        """Batch-1 step: per layer the q/k/v projection with the attention
        RMSNorm inside, attention, the o projection added into this rank's
        residual slice, the residual gathered, the gate/up projection with the
        FFN RMSNorm inside, SwiGLU, the down projection added into the slice,
        the residual gathered."""
        s, p, ops = self.shape, self.plan, self.ops
        if not 0 <= pos < self.max_ctx:
            raise ValueError("position outside the KV cache")
        h, hd, G = s.hidden, s.head_dim, p.world
        h_l = h // G
        ops.embed(self.embed, self.tokens, self.x, 1, h, s.vocab)
        for li, lay in enumerate(self.layers):
            ops.linear_norm(lay["wqkv"], self.x, lay["attn_norm"], self.qkv, h, self.q_l + 2 * self.kv_l, s.eps)
            kc, vc = ops.cache_layer(self.k_cache, li), ops.cache_layer(self.v_cache, li)
            if G > 1:
                ops.rope_attention(self.q, self.k, self.v, 1, p.heads, p.kv_heads, hd, pos, s.rope_theta, kc, vc,
                                   self.max_ctx, self.a_l, None)
                self._gather(self.a, self.a_l, h_l, self.xq_h, h)
            else:
                ops.rope_attention(self.q, self.k, self.v, 1, p.heads, p.kv_heads, hd, pos, s.rope_theta, kc, vc,
                                   self.max_ctx, None, self.xq_h)
            ops.linear_codes_add(lay["wo"], self.xq_h, self.x_l, h, h_l)
            if G > 1:
                self._gather(self.x, self.x_l, h_l)
            ops.linear_norm(lay["w_gu"], self.x, lay["ffn_norm"], self.gu, h, 2 * self.f_l, s.eps)
            if G == 1:
                ops.swiglu_codes(self.g_l, self.u_l, self.xq_f, self.f_l)
            else:
                ops.swiglu(self.g_l, self.u_l, self.f_l_buf, self.f_l)
                self._gather(self.f, self.f_l_buf, self.f_l, self.xq_f, s.ffn)
            ops.linear_codes_add(lay["w_down"], self.xq_f, self.x_l, s.ffn, h_l)
            if G > 1:
                self._gather(self.x, self.x_l, h_l)
        ops.linear_norm(self.head, self.x, self.out_norm, self.logits_l, h, p.local_rows("head"), s.eps)
        self._gather(self.logits, self.logits_l, p.local_rows("head"))


class _CudaView:
    """Minimal __cuda_array_interface__ exporter, to view device memory the
    library allocated as a torch tensor."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3}


class _PeerTarget:
    """A gather slot's receive area [rows][world * n_local] in this rank's
    IPC-shared buffer, plus the peers' mappings of their own buffers."""

    def __init__(self, slot: int, own: int, bases, data_bytes: int):
        self.slot, self.own, self.bases, self.flags_offset = slot, own, bases, data_bytes


class PeerGather:
    """One IPC-shared buffer per gather slot on every rank (data + a flag
    row), opened by all peers; gathers run as b200q_allgather_peer."""

    MAX_SLOTS = 16

    def __init__(self, rank: int, world: int, group=None):
        import torch

        self.torch, self.rank, self.world, self.group = torch, rank, world, group
        self.lib = _native.lib()
        self.targets: list[_PeerTarget] = []
        self._by_ptr: dict[int, _PeerTarget] = {}
        self._own: list[int] = []
        self._opened: list[int] = []
        self.counters = torch.zeros(self.MAX_SLOTS * 16, dtype=torch.int32, device="cuda")

    def target(self, n_floats: int):
        """A new gather slot; returns its receive area as a float32 tensor
        (a view of library-owned memory, valid until close())."""
        import ctypes

        import torch.distributed as dist

        slot = len(self.targets)
        if slot >= self.MAX_SLOTS:
            raise ValueError("too many gather slots")
        data = (4 * n_floats + 255) // 256 * 256
        ptr, handle = ctypes.c_void_p(), (ctypes.c_ubyte * 64)()
        _native.check(self.lib.b200q_ipc_alloc(data + 4 * 64, ctypes.byref(ptr), handle), "ipc alloc")
        self._own.append(ptr.value)
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=self.group)
        bases = []
        for r, h in enumerate(handles):
            if r == self.rank:
                bases.append(ptr.value)
                continue
            peer = ctypes.c_void_p()
            buf = (ctypes.c_ubyte * 64).from_buffer_copy(h)
            _native.check(self.lib.b200q_ipc_open(buf, ctypes.byref(peer)), "ipc open")
            self._opened.append(peer.value)
            bases.append(peer.value)
        t = _PeerTarget(slot, ptr.value, (ctypes.c_void_p * self.world)(*bases), data)
        self.targets.append(t)
        view = self.torch.as_tensor(_CudaView(ptr.value, n_floats), device="cuda")
        self._by_ptr[view.data_ptr()] = t
        return view

    def gather(self, full, local, rows: int, n_local: int, codes=None, act_mode: int = 0) -> None:
        target = self._by_ptr[full.data_ptr()]
        st = self.torch.cuda.current_stream().cuda_stream
        _native.check(self.lib.b200q_allgather_peer(local.data_ptr(), rows, n_local, target.bases, 0,
                                                    target.flags_offset, self.rank, self.world,
                                                    self.counters.data_ptr(), target.slot,
                                                    None if codes is None else codes.data_ptr(), act_mode, st),
                      "peer all-gather")

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (call on every rank,
        with no gather in flight)."""
        import torch.distributed as dist

        self.torch.cuda.synchronize()
        for p in self._opened:
            self.lib.b200q_ipc_close(p)
        dist.barrier(group=self.group)
        for p in self._own:
            self.lib.b200q_ipc_free(p)
        self._opened, self._own = [], []


class GpuOps:
    """ShardedDecode arithmetic on one GPU: libb200q kernels on the current
    stream, all-gathers on the same stream through torch.distributed (NCCL,
    collective="nccl") or through b200q_allgather_peer over NVLink peer
    memory (collective="peer"). With world 1 no collective runs."""

    def __init__(self, device: int = 0, act_mode: int = _native.ACT_X16, group=None, world: int = 1,
                 collective: str = "nccl", rank: int = 0):
        import torch

        self.torch = torch
        self.dev = torch.device("cuda", device)
        self.lib = _native.lib()
        self.act = act_mode
        self.group = group
        self.world = world
        self.peer = PeerGather(rank, world, group) if (collective == "peer" and world > 1) else None
        self._keep = []  # ctypes arrays referenced by captured calls

    def gather_target(self, name: str, n: int):
        return self.peer.target(n) if self.peer else self.zeros(n)

    def close(self) -> None:
        if self.peer:
            self.peer.close()

    # -- storage -------------------------------------------------------------------
    def zeros(self, n: int):
        return self.torch.zeros(n, dtype=self.torch.float32, device=self.dev)

    def vector(self, a: np.ndarray):
        return self.torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(self.dev)

    def matrix(self, qtype: int, k: int, n_rows: int, packed: np.ndarray):
        from .quantized_matmul import DeviceMatrix

        return DeviceMatrix(qtype, k, n_rows, packed)

    def clone_matrix(self, m):
        return m.clone()

    def cache(self, layers: int, batch: int, kv_heads: int, max_ctx: int, hd: int):
        shape = (layers, batch, kv_heads, max_ctx, hd)
        t = self.torch
        return t.zeros(shape, dtype=t.float16, device=self.dev), t.zeros(shape, dtype=t.float16, device=self.dev)

    def cache_layer(self, cache, li: int):
        return cache[li]

    def tokens(self, batch: int):
        return self.torch.zeros(batch, dtype=self.torch.int32, device=self.dev)

    # -- arithmetic ----------------------------------------------------------------
    def _st(self):
        return self.torch.cuda.current_stream(self.dev).cuda_stream

    def _ok(self, rc, what):
        _native.check(rc, what)

    def codes(self, rows: int, k: int):
        """Buffer for `rows` rows of activation codes of length k."""
        n = int(self.lib.b200q_xq_row_bytes(k, self.act))
        return self.torch.zeros(rows * n, dtype=self.torch.uint8, device=self.dev)

    def embed(self, m, tokens, out, batch, hidden, vocab):
        self._ok(self.lib.b200q_dequantize_rows(m.qtype, m.ptr, tokens.data_ptr(), batch, out.data_ptr(), hidden,
                                                vocab, self._st()), "embedding")

    def norm_codes(self, res, delta, gamma, xq, n, rows, eps):
        self._ok(self.lib.b200q_add_rmsnorm_q(res.data_ptr(), None if delta is None else delta.data_ptr(),
                                              gamma.data_ptr(), None, xq.data_ptr(), self.act, n, rows, eps,
                                              self._st()), "rmsnorm")

    def linear_codes(self, m, xq, out, batch, k, n_rows):
        self._ok(self.lib.b200q_matmul_xq(m.qtype, self.act, xq.data_ptr(), m.ptr, out.data_ptr(), batch, k, n_rows,
                                          1.0, 0.0, _native.WEIGHTS_STATIC, self._st()), "linear")

    def norm_f32(self, res, delta, gamma, out, n, rows, eps):
        """res += delta (when given); out = RMSNorm(res) * gamma, fp32 rows."""
        self._ok(self.lib.b200q_add_rmsnorm(res.data_ptr(), None if delta is None else delta.data_ptr(),
                                            gamma.data_ptr(), out.data_ptr(), n, rows, eps, self._st()), "rmsnorm")

    def linear_f32(self, m, x, out, batch, k, n_rows):
        """out [batch][n_rows] = x [batch][k] m^T from fp32 rows: Q4_K on the
        tile path (fp16 activations), other qtypes on the GEMV (x16)."""
        from .formats import Q4_K

        act = _native.ACT_F16 if m.qtype == Q4_K else _native.ACT_X16
        self._ok(self.lib.b200q_matmul_ex(m.qtype, act, x.data_ptr(), m.ptr, out.data_ptr(), batch, k, n_rows,
                                          _native.WEIGHTS_STATIC, self._st()), "linear (fp32 rows)")

    def linear_norm(self, m, x, gamma, out, k, n_rows, eps):
        """out = m (RMSNorm(x) * gamma) for one row, the norm inside the GEMV."""
        self._ok(self.lib.b200q_matmul_norm(m.qtype, self.act, x.data_ptr(), gamma.data_ptr(), eps, m.ptr,
                                            out.data_ptr(), k, n_rows, 1.0, 0.0, _native.WEIGHTS_STATIC, self._st()),
                 "linear+norm")

    def linear_codes_add(self, m, xq, out, k, n_rows):
        """out += m xq for one row of codes (the residual add in the epilogue)."""
        self._ok(self.lib.b200q_matmul_xq(m.qtype, self.act, xq.data_ptr(), m.ptr, out.data_ptr(), 1, k, n_rows, 1.0,
                                          1.0, _native.WEIGHTS_STATIC, self._st()), "linear+add")

    def quantize(self, x, xq, rows, k):
        self._ok(self.lib.b200q_quantize_rows(self.act, x.data_ptr(), rows, k, xq.data_ptr(), self._st()), "quantize")

    def rope_kv(self, q, k, v, batch, heads, kv_heads, hd, pos, theta, kc, vc, max_ctx):
        self._ok(self.lib.b200q_rope_kv(q.data_ptr(), k.data_ptr(), v.data_ptr(), batch, heads, kv_heads, hd, pos,
                                        theta, kc.data_ptr(), vc.data_ptr(), max_ctx, self._st()), "rope_kv")

    def rope_attention(self, q, k, v, batch, heads, kv_heads, hd, pos, theta, kc, vc, max_ctx, out, xq):
        self._ok(self.lib.b200q_rope_attention_decode(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), batch, heads, kv_heads, hd, pos, theta, kc.data_ptr(),
            vc.data_ptr(), max_ctx, None if out is None else out.data_ptr(), None if xq is None else xq.data_ptr(),
            self.act, self._st()), "rope_attention")

    def attention(self, q, kc, vc, out, batch, heads, kv_heads, hd, ctx, max_ctx):
        self._ok(self.lib.b200q_attention_decode(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), batch,
                                                 heads, kv_heads, hd, ctx, max_ctx, self._st()), "attention")

    def swiglu_codes(self, g, u, xq, n):
        self._ok(self.lib.b200q_swiglu_q(g.data_ptr(), u.data_ptr(), xq.data_ptr(), self.act, n, self._st()),
                 "swiglu_q")

    def swiglu(self, g, u, out, n):
        self._ok(self.lib.b200q_swiglu(g.data_ptr(), u.data_ptr(), out.data_ptr(), n, self._st()), "swiglu")

    def all_gather(self, full, local, gbuf, batch, n_local, codes=None):
        """full [batch][world * n_local] = every rank's local [batch][n_local];
        with `codes`, also the activation codes of the gathered rows."""
        if self.peer:
            self.peer.gather(full, local, batch, n_local, codes, self.act)
            return
        import torch.distributed as dist

        n = self.world * batch * n_local
        if batch == 1:
            dist.all_gather_into_tensor(full[:n], local[:n_local], group=self.group)
        else:
            dist.all_gather_into_tensor(gbuf[:n], local[: batch * n_local], group=self.group)
            self._ok(self.lib.b200q_unshard_rows(gbuf.data_ptr(), full.data_ptr(), self.world, batch, n_local,
                                                 self._st()), "unshard")
        if codes is not None:
            self.quantize(full, codes, batch, self.world * n_local)
