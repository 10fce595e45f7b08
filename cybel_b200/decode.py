"""Single-token decode of a Llama-style layer stack on one B200.

The caller of the quantized linears in the reference is its C++ decode graph
(JSBuild/src/verso/Anvil/core/native/model_graph.cpp): per layer RMSNorm,
the q/k/v projections, RoPE and the KV-cache append, GQA attention over the
cache, the o projection with the residual add, RMSNorm, and the SwiGLU FFN
with its residual add; then the final norm and the LM head. ``DecodeStack``
runs that step entirely on the device through libb200q's entry points:

* ``b200q_matmul_norm`` -- each projection that follows an RMSNorm (q/k/v
  as one matrix, gate/up as one matrix, the LM head), the norm computed by
  the GEMV itself from the fp32 residual stream (``fused_norm=False`` runs
  ``b200q_add_rmsnorm_q`` then ``b200q_matmul_xq`` instead);
* ``b200q_matmul_xq`` -- the o projection fed by the attention's codes, with
  the residual add in its epilogue (beta = 1);
* ``b200q_rope_attention_decode`` -- RoPE, the KV append and attention in
  one launch, which also writes the o projection's codes;
* ``b200q_swiglu_q`` -- SiLU(gate) * up, written as the down projection's
  codes, and ``b200q_matmul_xq`` -- the down projection with the residual
  add (``fused_swiglu=True`` runs both inside one GEMV,
  ``b200q_matmul_swiglu``);

all on one stream, so one token's step is one CUDA graph. The KV cache is
fp16, [layer][kv_head][max_ctx][head_dim], or the reference's paged store
(kv_cache.PagedKVCache: fp16 or Q8 pages, ``b200q_rope_attention_decode_paged``).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import _native
from .formats import Q4_K, Q6_K, row_bytes
from .quantized_matmul import DeviceMatrix


@dataclass(frozen=True)
class StackShape:
    layers: int
    hidden: int
    heads: int
    kv_heads: int
    ffn: int
    vocab: int
    rope_theta: float = 500000.0
    eps: float = 1e-5
    linear_qtype: int = Q4_K
    head_qtype: int = Q6_K
    embed_qtype: int | None = None  # token embedding rows; None: the linears' type

    @property
    def embedding_qtype(self) -> int:
        return self.linear_qtype if self.embed_qtype is None else self.embed_qtype

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim

    def layer_weight_bytes(self) -> int:
        from .formats import row_bytes

        h, kv, f, q = self.hidden, self.kv_dim, self.ffn, self.linear_qtype
        return (2 * h + 2 * kv + 2 * f) * row_bytes(q, h) + h * row_bytes(q, f)

    def token_weight_bytes(self) -> int:
        """Packed weight bytes one decode step streams (layers + LM head)."""
        from .formats import row_bytes

        return self.layers * self.layer_weight_bytes() + self.vocab * row_bytes(self.head_qtype, self.hidden)


# Llama-3-8B and Llama-3-70B shapes.
LLAMA3_8B = StackShape(layers=32, hidden=4096, heads=32, kv_heads=8, ffn=14336, vocab=128256)
LLAMA3_70B = StackShape(layers=80, hidden=8192, heads=64, kv_heads=8, ffn=28672, vocab=128256, head_qtype=Q4_K)

LAYER_MATRICES = ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down")


def layer_matrix_shapes(shape: StackShape) -> dict[str, tuple[int, int]]:
    """(n_rows, k) of each linear of a layer."""
    h, kv, f = shape.hidden, shape.kv_dim, shape.ffn
    return {"wq": (h, h), "wk": (kv, h), "wv": (kv, h), "wo": (h, h), "w_gate": (f, h), "w_up": (f, h),
            "w_down": (h, f)}


def random_layer(shape: StackShape, rng: np.random.Generator, std: float = 0.02,
                 block_rows: int | None = None) -> dict[str, np.ndarray]:
    """One layer's weights: N(0, std) linears packed to the linear qtype, and
    RMSNorm gains near 1 (fp32). With block_rows, each linear repeats one
    quantized block of that many rows (see random_rows)."""
    out: dict[str, np.ndarray] = {}
    for name, (n, k) in layer_matrix_shapes(shape).items():
        out[name] = random_rows(shape.linear_qtype, n, k, rng, block_rows=block_rows, std=std)
    out["attn_norm"] = (1.0 + 0.1 * rng.standard_normal(shape.hidden)).astype(np.float32)
    out["ffn_norm"] = (1.0 + 0.1 * rng.standard_normal(shape.hidden)).astype(np.float32)
    return out


def random_rows(qtype: int, n: int, k: int, rng: np.random.Generator, block_rows: int | None = None,
                std: float = 0.02) -> np.ndarray:
    """A packed [n][k] matrix of N(0, std) weights. With block_rows, one block
    of that many rows is quantized and repeated to n rows (the bytes every
    row streams are the same size; used for the 128K-row embedding and head
    at benchmark scale)."""
    from . import quantize as Q

    if block_rows is None or block_rows >= n:
        return Q.quantize(rng.normal(0.0, std, size=(n, k)).astype(np.float32), qtype)
    blk = Q.quantize(rng.normal(0.0, std, size=(block_rows, k)).astype(np.float32), qtype)
    reps = (n + block_rows - 1) // block_rows
    return np.ascontiguousarray(np.tile(blk, (reps, 1))[:n])


@dataclass
class _Layer:
    wqkv: DeviceMatrix      # q, k and v rows, one after the other
    wo: DeviceMatrix
    w_gu: DeviceMatrix      # gate rows, then up rows
    w_down: DeviceMatrix
    attn_norm: object
    ffn_norm: object


class DecodeStack:
    """Device-resident Llama-style stack; ``step(pos)`` issues one token.

    ``layers`` holds one weight dict per layer (``random_layer`` layout); a
    shorter list is cycled, each layer still getting its own device copy.
    On the device the q/k/v rows of a layer are stored as one matrix, and so
    are the gate/up rows, so each is one GEMV. A layer is six launches: qkv
    (RMSNorm inside), RoPE + KV append + attention (writing the o
    projection's codes), o (+ residual), gate/up (RMSNorm inside), SwiGLU
    (writing the down projection's codes), down (+ residual); five with
    ``fused_swiglu``, eight with ``fused_norm=False``.
    """

    def __init__(self, shape: StackShape, max_ctx: int, layers: list[dict[str, np.ndarray]], embed: np.ndarray,
                 head: np.ndarray, out_norm: np.ndarray, act_mode: int = _native.ACT_X16, device: int = 0,
                 fused_norm: bool = True, repack: "RepackPolicy | None" = None, architecture: str = "llama",
                 kv: str | None = None, page_size: int | None = None, fused_swiglu: bool = False):
        """``repack`` picks each weight's decode layout as the reference does
        when it registers a graph's weights (repack_policy.RepackPolicy; by
        default from the ANVIL_* environment switches for `architecture`).

        ``kv`` picks the KV cache: "contiguous" (fp16 [layer][kv_head][max_ctx]
        [head_dim]), "paged" (fp16 pages) or "q8" (the reference's Q8 pages);
        by default "q8" when ANVIL_KV_QUANT asks for it (kv_cache.q8_from_env),
        else "contiguous". Pages hold ``page_size`` positions (default
        kv_cache.KV_PAGE_SIZE).

        ``fused_swiglu`` forms SiLU(gate) * up inside the down projection's
        GEMV (``b200q_matmul_swiglu``, one launch fewer per layer) instead of
        ``b200q_swiglu_q`` + ``b200q_matmul_xq``; off by default, because
        staging the two fp32 rows in every CTA of the down GEMV costs more
        than the launch it saves on the Llama-3-8B shape."""
        import torch

        from .kv_cache import KV_PAGE_SIZE, PagedKVCache, q8_from_env
        from .repack_policy import RepackPolicy, apply

        if kv is None:
            kv = "q8" if q8_from_env() else "contiguous"
        if kv not in ("contiguous", "paged", "q8"):
            raise ValueError(f"unknown KV cache kind {kv!r}")
        self.kv = kv

        policy = RepackPolicy.from_env(architecture) if repack is None else repack
        if shape.head_dim != 128:
            raise ValueError("the attention kernels are built for head_dim 128")
        if act_mode not in (_native.ACT_X8, _native.ACT_X16):
            raise ValueError("DecodeStack runs the GEMV activation modes (x8 / x16)")
        self.shape = shape
        self.max_ctx = max_ctx
        self.act_mode = act_mode
        self.fused_norm = fused_norm
        self.fused_swiglu = fused_swiglu
        self._vbufs: dict = {}  # verify-pass buffers per row count
        self.dev = torch.device("cuda", device)
        self.lib = _native.lib()
        f32 = dict(dtype=torch.float32, device=self.dev)
        h, kv, f, q = shape.hidden, shape.kv_dim, shape.ffn, shape.linear_qtype
        self.layers: list[_Layer] = []
        first: list[_Layer] = []
        for i in range(shape.layers):
            if i < len(layers):
                src = layers[i]
                lay = _Layer(
                    apply(policy, DeviceMatrix(q, h, h + 2 * kv, np.concatenate([src["wq"], src["wk"], src["wv"]]))),
                    apply(policy, DeviceMatrix(q, h, h, src["wo"])),
                    apply(policy, DeviceMatrix(q, h, 2 * f, np.concatenate([src["w_gate"], src["w_up"]]))),
                    apply(policy, DeviceMatrix(q, f, h, src["w_down"])),
                    torch.from_numpy(src["attn_norm"]).to(self.dev),
                    torch.from_numpy(src["ffn_norm"]).to(self.dev))
                first.append(lay)
            else:  # its own device copy of a cycled layer
                b = first[i % len(layers)]
                lay = _Layer(b.wqkv.clone(), b.wo.clone(), b.w_gu.clone(), b.w_down.clone(), b.attn_norm, b.ffn_norm)
            self.layers.append(lay)
        self.embed = DeviceMatrix(shape.embedding_qtype, h, shape.vocab, embed)
        self.head = apply(policy, DeviceMatrix(shape.head_qtype, h, shape.vocab, head), lm_head=True)
        self.out_norm = torch.from_numpy(out_norm).to(self.dev)
        if self.kv == "contiguous":
            cache_shape = (shape.layers, shape.kv_heads, max_ctx, shape.head_dim)
            self.k_cache = torch.zeros(cache_shape, dtype=torch.float16, device=self.dev)
            self.v_cache = torch.zeros(cache_shape, dtype=torch.float16, device=self.dev)
            self.kv_cache = None
        else:
            self.k_cache = self.v_cache = None
            self.kv_cache = PagedKVCache(shape.layers, shape.kv_heads, max_ctx, batch=1,
                                         page_size=page_size or KV_PAGE_SIZE, q8=self.kv == "q8", device=device)
        self.x = torch.zeros(h, **f32)             # residual stream
        self.qkv = torch.zeros(h + 2 * kv, **f32)  # q | k | v
        self.gu = torch.zeros(2 * f, **f32)        # gate | up
        self.logits = torch.zeros(shape.vocab, **f32)
        self.token = torch.zeros(1, dtype=torch.int32, device=self.dev)
        xb = self.lib.b200q_xq_row_bytes
        self.xq_h = torch.zeros(int(xb(h, act_mode)), dtype=torch.uint8, device=self.dev)  # codes of a hidden vector
        self.xq_f = torch.zeros(int(xb(f, act_mode)), dtype=torch.uint8, device=self.dev)  # codes of the FFN vector
        torch.cuda.synchronize(self.dev)

    # -- one token ----------------------------------------------------------------
    def _check(self, rc, what):
        _native.check(rc, what)

    def step(self, pos: int, linears_only: bool = False) -> None:
        """Append the token in ``self.token`` at position ``pos`` and leave the
        next-token logits in ``self.logits`` (stream: the current one).

        ``linears_only`` issues just the quantized linears of the step, on
        the same buffers, for timing the matvec share of a token."""
        import torch

        if not 0 <= pos < self.max_ctx:
            raise ValueError("position outside the KV cache")
        if self.kv_cache is not None and not linears_only:
            self.kv_cache.ensure(pos)  # the page of pos (a table copy only when it is new)
        s, L, st = self.shape, self.lib, torch.cuda.current_stream(self.dev).cuda_stream
        W = _native.WEIGHTS_STATIC
        act = self.act_mode
        h, kv, hd, f = s.hidden, s.kv_dim, s.head_dim, s.ffn
        x, xq_h, xq_f = self.x.data_ptr(), self.xq_h.data_ptr(), self.xq_f.data_ptr()
        qp = self.qkv.data_ptr()
        kp, vp = qp + 4 * h, qp + 4 * (h + kv)
        gp = self.gu.data_ptr()
        up = gp + 4 * f
        resid = 0.0 if linears_only else 1.0
        if not linears_only:
            self._check(L.b200q_dequantize_rows(s.embedding_qtype, self.embed.ptr, self.token.data_ptr(), 1, x, h,
                                                s.vocab, st),
                        "embedding")
        for li, lay in enumerate(self.layers):
            # RMSNorm inside the q/k/v GEMV (it normalizes and quantizes x while its weights stream)
            self._norm_matmul(lay.wqkv.qtype, x, lay.attn_norm, xq_h, lay.wqkv.ptr, qp, h, h + 2 * kv, "qkv", st,
                              linears_only)
            if not linears_only and self.kv_cache is not None:
                self.kv_cache.attention(li, qp, kp, vp, pos, s.heads, s.rope_theta, None, xq_h, act, st)
            elif not linears_only:
                kc = self.k_cache[li].data_ptr()
                vc = self.v_cache[li].data_ptr()
                self._check(L.b200q_rope_attention_decode(qp, kp, vp, 1, s.heads, s.kv_heads, hd, pos,
                                                          s.rope_theta, kc, vc, self.max_ctx, None, xq_h, act, st),
                            "rope_attention")
            # o projection with the residual add in its epilogue: x = Wo a + x
            self._check(L.b200q_matmul_xq(lay.wo.qtype, act, xq_h, lay.wo.ptr, x, 1, h, h, 1.0, resid, W, st), "o_proj")
            self._norm_matmul(lay.w_gu.qtype, x, lay.ffn_norm, xq_h, lay.w_gu.ptr, gp, h, 2 * f, "gate_up", st,
                              linears_only)
            if self.fused_swiglu and not linears_only:
                # SiLU(gate) * up formed and quantized inside the down GEMV, with the residual add
                self._check(L.b200q_matmul_swiglu(lay.w_down.qtype, act, gp, up, lay.w_down.ptr, x, f, h, 1.0, resid,
                                                  W, st), "swiglu+down")
            else:
                if not linears_only:
                    self._check(L.b200q_swiglu_q(gp, up, xq_f, act, f, st), "swiglu")
                self._check(L.b200q_matmul_xq(lay.w_down.qtype, act, xq_f, lay.w_down.ptr, x, 1, f, h, 1.0, resid, W,
                                              st), "down")
        self._norm_matmul(self.head.qtype, x, self.out_norm, xq_h, self.head.ptr, self.logits.data_ptr(), h, s.vocab,
                          "lm_head", st, linears_only)

    def _norm_matmul(self, qt, x, gamma, xq, w, y, k, n, what, st, linears_only) -> None:
        """y = W (RMSNorm(x) * gamma): one GEMV that normalizes x itself
        (b200q_matmul_norm), or, with fused_norm off, b200q_add_rmsnorm_q writing
        the codes and b200q_matmul_xq reading them (linears_only keeps only the
        GEMV of that pair)."""
        L, s, W = self.lib, self.shape, _native.WEIGHTS_STATIC
        if self.fused_norm:
            self._check(L.b200q_matmul_norm(qt, self.act_mode, x, gamma.data_ptr(), s.eps, w, y, k, n, 1.0, 0.0, W, st),
                        what)
            return
        if not linears_only:
            self._check(L.b200q_add_rmsnorm_q(x, None, gamma.data_ptr(), None, xq, self.act_mode, k, 1, s.eps, st),
                        what + " norm")
        self._check(L.b200q_matmul_xq(qt, self.act_mode, xq, w, y, 1, k, n, 1.0, 0.0, W, st), what)

    @classmethod
    def from_gguf(cls, path, max_ctx: int, act_mode: int = _native.ACT_X16, device: int = 0,
                  fused_norm: bool = True) -> "DecodeStack":
        """A stack whose weights are the tensors of a llama-architecture GGUF
        file (gguf_file.load_llama_stack), uploaded as the file stores them
        and then given the decode layouts the repack policy picks for the
        file's architecture (repack_policy.RepackPolicy.from_env)."""
        from .gguf_file import GGUFFile, load_llama_stack

        shape, layers, embed, head, out_norm = load_llama_stack(path)
        arch = str(GGUFFile(path).metadata.get("general.architecture", "llama"))
        return cls(shape, max_ctx, layers, embed, head, out_norm, act_mode=act_mode, device=device,
                   fused_norm=fused_norm, architecture=arch)

    def set_token(self, token: int) -> None:
        self.token.fill_(int(token))

    # -- several tokens in one pass ---------------------------------------------
    def _verify_buffers(self, m: int) -> dict:
        import torch

        bufs = self._vbufs.get(m)
        if bufs is None:
            s = self.shape
            h, kv, f = s.hidden, s.kv_dim, s.ffn
            z = (lambda *shape: torch.zeros(shape, dtype=torch.float32, device=self.dev))
            bufs = dict(x=z(m, h), hn=z(m, h), qkv=z(m, h + 2 * kv), att=z(m, h), o=z(m, h), gu=z(m, 2 * f),
                        sw=z(m, f), d=z(m, h), logits=z(m, s.vocab),
                        tok=torch.zeros(m, dtype=torch.int32, device=self.dev))
            self._vbufs[m] = bufs
        return bufs

    def verify(self, tokens, pos0: int):
        """Feed len(tokens) tokens at positions pos0, pos0 + 1, ... through
        the stack in ONE pass and return their next-token logits, a device
        tensor [m][vocab] (row j: the logits after tokens[j]).

        This is the batched form of the reference's speculative verify, which
        asks the engine for the logits of each drafted prefix in turn
        (cpu_speculative_decode.py:740-769): every quantized linear runs once
        over the m rows (b200q_matmul_ex with B200Q_TILE_FROM_2: the tcgen05
        tile kernel for Q4_K from 2 rows, the GEMV for the other qtypes; q, k
        and v as one linear, gate and up as one), and one attention launch per
        layer, reading q, k and v straight from the rows of the q|k|v output,
        appends the m keys/values and attends causally
        (b200q_rope_attention_decode_tokens / the paged form). The cache then
        holds all m tokens; positions past the accepted prefix are simply
        written again by the next step before anything reads them."""
        import torch

        m = len(tokens)
        if m <= 0:
            raise ValueError("no tokens to verify")
        if pos0 < 0 or pos0 + m > self.max_ctx:
            raise ValueError("positions outside the KV cache")
        s, L = self.shape, self.lib
        st = torch.cuda.current_stream(self.dev).cuda_stream
        act, W = self.act_mode, _native.WEIGHTS_STATIC | _native.TILE_FROM_2
        h, kv, hd, f = s.hidden, s.kv_dim, s.head_dim, s.ffn
        B = self._verify_buffers(m)
        if isinstance(tokens, torch.Tensor) and tokens.is_cuda:  # already on the device (graph capture)
            B["tok"].copy_(tokens.to(torch.int32))
        else:
            B["tok"].copy_(torch.tensor([int(t) for t in tokens], dtype=torch.int32))
        if self.kv_cache is not None:
            self.kv_cache.ensure(pos0, pos0 + m - 1)
        P = {name: t.data_ptr() for name, t in B.items()}

        def lin(mat, row0, n, x, y, k):
            ptr = mat.ptr + row0 * row_bytes(mat.qtype, k)
            self._check(L.b200q_matmul_ex(mat.qtype, act, x, ptr, y, m, k, n, W, st), "verify linear")

        self._check(L.b200q_dequantize_rows(s.embedding_qtype, self.embed.ptr, P["tok"], m, P["x"], h, s.vocab, st),
                    "embedding")
        delta = None
        for li, lay in enumerate(self.layers):
            self._check(L.b200q_add_rmsnorm(P["x"], delta, lay.attn_norm.data_ptr(), P["hn"], h, m, s.eps, st),
                        "attn norm")
            lin(lay.wqkv, 0, h + 2 * kv, P["hn"], P["qkv"], h)
            qp, kp, vp = P["qkv"], P["qkv"] + 4 * h, P["qkv"] + 4 * (h + kv)
            row = h + 2 * kv  # floats between consecutive tokens' q (and k, v) rows
            if self.kv_cache is not None:
                self.kv_cache.attention(li, qp, kp, vp, pos0, s.heads, s.rope_theta, P["att"], None, 0, st,
                                        n_tokens=m, q_stride=row, kv_stride=row)
            else:
                self._check(L.b200q_rope_attention_decode_tokens(
                    qp, kp, vp, 1, m, s.heads, s.kv_heads, hd, pos0, s.rope_theta, self.k_cache[li].data_ptr(),
                    self.v_cache[li].data_ptr(), self.max_ctx, P["att"], None, 0, row, row, st), "verify attention")
            lin(lay.wo, 0, h, P["att"], P["o"], h)
            self._check(L.b200q_add_rmsnorm(P["x"], P["o"], lay.ffn_norm.data_ptr(), P["hn"], h, m, s.eps, st),
                        "ffn norm")
            lin(lay.w_gu, 0, 2 * f, P["hn"], P["gu"], h)
            self._check(L.b200q_swiglu_rows(P["gu"], P["sw"], m, f, st), "swiglu")
            lin(lay.w_down, 0, h, P["sw"], P["d"], f)
            delta = P["d"]
        self._check(L.b200q_add_rmsnorm(P["x"], delta, self.out_norm.data_ptr(), P["hn"], h, m, s.eps, st),
                    "output norm")
        lin(self.head, 0, s.vocab, P["hn"], P["logits"], h)
        return B["logits"]
