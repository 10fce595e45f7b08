"""Decode-step glue and a small layer stack against CPU restatements.

* b200q_add_rmsnorm / b200q_rope_kv / b200q_attention_decode against float64
  numpy restatements of the reference's rmsnorm_inplace, apply_rope_with_dim
  and GQA attention (model_graph.cpp:674-693, 1222-1323), with the fp16 cache
  rounding mirrored: max |d| / max |ref| <= 1e-5 (norm), <= 1e-4 (rope:
  fp32 angles pos * theta^(-2p/hd) up to pos ~ 1e3, as the reference forms
  them; attention: fp32 softmax and accumulation over up to 2048 positions).
* DecodeStack (2 layers, hidden 512, 4 query / 2 kv heads, FFN 768, vocab 512)
  for 12 consecutive tokens against oracle/decode_ref.py: logits within
  ||d||_inf / ||ref||_inf <= 2e-3 (x16 activations, fp16 KV cache) and the
  same argmax wherever the top logit leads the runner-up clearly.
* CPU-only: the per-token weight bytes of the Llama-3-8B / 70B shapes.
"""

from __future__ import annotations

import numpy as np
import pytest


def test_token_weight_bytes_match_the_layer_inventory():
    from cybel_b200.decode import LLAMA3_70B, LLAMA3_8B

    assert LLAMA3_8B.layer_weight_bytes() == 122_683_392
    assert LLAMA3_8B.token_weight_bytes() == 4_356_808_704
    assert LLAMA3_70B.layer_weight_bytes() == 481_296_384
    assert LLAMA3_70B.token_weight_bytes() == 39_094_714_368


def _rel(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - b)) / max(np.max(np.abs(b)), 1e-30))


@pytest.mark.gpu
@pytest.mark.parametrize("with_delta", [False, True])
def test_add_rmsnorm(with_delta):
    import torch
    from cybel_b200 import _native

    rng = np.random.default_rng(1)
    n = 4096
    res = rng.standard_normal(n).astype(np.float32)
    delta = rng.standard_normal(n).astype(np.float32)
    gamma = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    r, d, g = (torch.from_numpy(a).cuda() for a in (res, delta, gamma))
    out = torch.empty(n, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    rc = _native.lib().b200q_add_rmsnorm(r.data_ptr(), d.data_ptr() if with_delta else None, g.data_ptr(),
                                         out.data_ptr(), n, 1, 1e-5, st)
    assert rc == 0
    x = res.astype(np.float64) + (delta if with_delta else 0.0)
    ref = x / np.sqrt(np.mean(x * x) + 1e-5) * gamma
    assert _rel(out.cpu().numpy(), ref) <= 1e-5
    assert _rel(r.cpu().numpy(), x) <= 1e-6


@pytest.mark.gpu
def test_rope_kv_append():
    import torch
    from cybel_b200 import _native

    rng = np.random.default_rng(2)
    H, KV, hd, pos, max_ctx, theta = 32, 8, 128, 777, 1024, 500000.0
    q = rng.standard_normal(H * hd).astype(np.float32)
    k = rng.standard_normal(KV * hd).astype(np.float32)
    v = rng.standard_normal(KV * hd).astype(np.float32)
    qt, kt, vt = (torch.from_numpy(a).cuda() for a in (q, k, v))
    kc = torch.zeros((KV, max_ctx, hd), dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    st = torch.cuda.current_stream().cuda_stream
    assert _native.lib().b200q_rope_kv(qt.data_ptr(), kt.data_ptr(), vt.data_ptr(), 1, H, KV, hd, pos, theta,
                                       kc.data_ptr(), vc.data_ptr(), max_ctx, st) == 0

    def rope(a, heads):
        p = np.arange(hd // 2)
        ang = pos * theta ** (-2.0 * p / hd)
        a = a.reshape(heads, hd).astype(np.float64)
        out = a.copy()
        out[:, 0::2] = a[:, 0::2] * np.cos(ang) - a[:, 1::2] * np.sin(ang)
        out[:, 1::2] = a[:, 0::2] * np.sin(ang) + a[:, 1::2] * np.cos(ang)
        return out

    qr, kr = rope(q, H), rope(k, KV)
    # fp32 angles pos * theta^(-2p/hd), as the reference computes them
    assert _rel(qt.cpu().numpy().reshape(H, hd), qr) <= 1e-4
    assert _rel(kt.cpu().numpy().reshape(KV, hd), kr) <= 1e-4
    kcn, vcn = kc.float().cpu().numpy(), vc.float().cpu().numpy()
    assert _rel(kcn[:, pos], kr.astype(np.float16).astype(np.float64)) <= 1e-3
    assert np.array_equal(vcn[:, pos], v.reshape(KV, hd).astype(np.float16).astype(np.float32))
    assert not kcn[:, :pos].any() and not kcn[:, pos + 1:].any()


@pytest.mark.gpu
@pytest.mark.parametrize("H,KV,ctx", [(32, 8, 1), (32, 8, 5), (32, 8, 128), (32, 8, 300), (32, 8, 2048), (4, 2, 129),
                                      (64, 8, 1000)])
def test_attention_decode(H, KV, ctx):
    import torch
    from cybel_b200 import _native

    rng = np.random.default_rng(H + ctx)
    hd, max_ctx = 128, max(ctx, 64) + 3
    q = rng.standard_normal(H * hd).astype(np.float32)
    kc = rng.standard_normal((KV, max_ctx, hd)).astype(np.float16)
    vc = rng.standard_normal((KV, max_ctx, hd)).astype(np.float16)
    qt = torch.from_numpy(q).cuda()
    kct, vct = torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda()
    out = torch.empty(H * hd, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert _native.lib().b200q_attention_decode(qt.data_ptr(), kct.data_ptr(), vct.data_ptr(), out.data_ptr(), 1, H,
                                                KV, hd, ctx, max_ctx, st) == 0
    ref = np.zeros((H, hd))
    G = H // KV
    for h in range(H):
        K = kc[h // G, :ctx].astype(np.float64)
        V = vc[h // G, :ctx].astype(np.float64)
        s = K @ q[h * hd:(h + 1) * hd].astype(np.float64) / np.sqrt(hd)
        e = np.exp(s - s.max())
        ref[h] = (e / e.sum()) @ V
    assert _rel(out.cpu().numpy().reshape(H, hd), ref) <= 1e-4


LAYOUTS = {
    "canonical": {"ANVIL_LM_HEAD_PACKED": "0"},
    "default": {},  # the reference's defaults for llama: the Q6_K head as Q6_K_R4
    "r4_lm": {"ANVIL_Q4K_R4": "1", "ANVIL_LM_HEAD_Q6K_LM": "1"},  # Q4_K_R4 linears, Q6_K_LM head
}


@pytest.mark.gpu
@pytest.mark.parametrize("layout", sorted(LAYOUTS))
@pytest.mark.parametrize("fused_norm,fused_swiglu", [(True, False), (False, False), (True, True)])
def test_decode_stack_matches_restatement(fused_norm, fused_swiglu, layout):
    """Logits of 12 tokens against the float64 restatement, with the weights
    in each decode layout the registration policy can pick."""
    from cybel_b200.decode import DecodeStack, StackShape, random_layer, random_rows
    from cybel_b200.formats import Q4_K, Q4_K_R4, Q6_K, Q6_K_LM, Q6_K_R4
    from cybel_b200.repack_policy import RepackPolicy
    from oracle.decode_ref import DecodeRef

    shape = StackShape(layers=2, hidden=512, heads=4, kv_heads=2, ffn=768, vocab=512)
    rng = np.random.default_rng(7)
    layers = [random_layer(shape, rng) for _ in range(shape.layers)]
    embed = random_rows(Q4_K, shape.vocab, shape.hidden, rng, std=1.0)
    head = random_rows(Q6_K, shape.vocab, shape.hidden, rng)
    out_norm = (1 + 0.1 * rng.standard_normal(shape.hidden)).astype(np.float32)
    max_ctx = 64
    policy = RepackPolicy.from_env("llama", env=LAYOUTS[layout])
    dev = DecodeStack(shape, max_ctx, layers, embed, head, out_norm, fused_norm=fused_norm, repack=policy,
                      kv="contiguous", fused_swiglu=fused_swiglu)
    assert dev.kv_cache is None and dev.k_cache is not None
    want_q = {"canonical": (Q4_K, Q6_K), "default": (Q4_K, Q6_K_R4), "r4_lm": (Q4_K_R4, Q6_K_LM)}[layout]
    assert (dev.layers[0].wqkv.qtype, dev.head.qtype) == want_q
    ref = DecodeRef(shape, layers, embed, head, out_norm, max_ctx)
    tokens = [3, 17, 5, 100, 511, 0, 42, 42, 7, 300, 64, 1]
    for pos, tok in enumerate(tokens):
        dev.set_token(tok)
        dev.step(pos)
        got = dev.logits.cpu().numpy()
        want = ref.step(tok, pos)
        assert _rel(got, want) <= 2e-3, pos
        top2 = np.sort(want)[-2:]
        if top2[1] - top2[0] > 5e-3 * np.max(np.abs(want)):  # a clear winner
            assert int(np.argmax(got)) == int(np.argmax(want)), pos


@pytest.mark.gpu
@pytest.mark.parametrize("kv", ["paged", "q8"])
def test_decode_stack_paged_cache(kv):
    """The stack over the paged caches (8-position pages, so the 12 tokens
    cross a page boundary) against the restatement with the same cache
    storage: fp16 rows, or the reference's Q8 rows (ANVIL_KV_QUANT)."""
    from cybel_b200.decode import DecodeStack, StackShape, random_layer, random_rows
    from cybel_b200.formats import Q4_K, Q6_K
    from cybel_b200.repack_policy import RepackPolicy
    from oracle.decode_ref import DecodeRef

    shape = StackShape(layers=2, hidden=512, heads=4, kv_heads=2, ffn=768, vocab=512)
    rng = np.random.default_rng(8)
    layers = [random_layer(shape, rng) for _ in range(shape.layers)]
    embed = random_rows(Q4_K, shape.vocab, shape.hidden, rng, std=1.0)
    head = random_rows(Q6_K, shape.vocab, shape.hidden, rng)
    out_norm = (1 + 0.1 * rng.standard_normal(shape.hidden)).astype(np.float32)
    dev = DecodeStack(shape, 64, layers, embed, head, out_norm, repack=RepackPolicy.canonical(), kv=kv, page_size=8)
    ref = DecodeRef(shape, layers, embed, head, out_norm, 64, kv_q8=kv == "q8")
    tokens = [3, 17, 5, 100, 511, 0, 42, 42, 7, 300, 64, 1]
    for pos, tok in enumerate(tokens):
        dev.set_token(tok)
        dev.step(pos)
        got = dev.logits.cpu().numpy()
        assert _rel(got, ref.step(tok, pos)) <= 2e-3, pos
    assert dev.k_cache is None and dev.kv_cache.q8 == (kv == "q8")
    assert dev.kv_cache.pages_in_use == shape.layers * 2


@pytest.mark.gpu
def test_unshard_rows():
    import torch
    from cybel_b200 import _native

    G, B, c = 4, 3, 40
    src = torch.arange(G * B * c, dtype=torch.float32, device="cuda")
    out = torch.empty_like(src)
    st = torch.cuda.current_stream().cuda_stream
    assert _native.lib().b200q_unshard_rows(src.data_ptr(), out.data_ptr(), G, B, c, st) == 0
    want = src.cpu().numpy().reshape(G, B, c).transpose(1, 0, 2).reshape(-1)
    assert np.array_equal(out.cpu().numpy(), want)


@pytest.mark.gpu
@pytest.mark.parametrize("batch", [1, 3])
def test_sharded_decode_one_rank_matches_restatement(batch):
    """ShardedDecode on one GPU (world 1) with the device kernels, batched
    glue included, against the unsharded restatement."""
    from cybel_b200.decode import StackShape, random_layer, random_rows
    from cybel_b200.formats import Q4_K, Q6_K
    from cybel_b200.sharded import GpuOps, ShardedDecode, ShardPlan
    from oracle.decode_ref import DecodeRef

    shape = StackShape(layers=2, hidden=512, heads=4, kv_heads=2, ffn=768, vocab=512)
    rng = np.random.default_rng(5)
    layers = [random_layer(shape, rng) for _ in range(shape.layers)]
    embed = random_rows(Q4_K, shape.vocab, shape.hidden, rng, std=1.0)
    head = random_rows(Q6_K, shape.vocab, shape.hidden, rng)
    out_norm = (1 + 0.1 * rng.standard_normal(shape.hidden)).astype(np.float32)
    model = ShardedDecode(ShardPlan(shape, 1, 0), 32, batch, layers, embed, head, out_norm, GpuOps())
    tokens = [[3, 17, 5, 100, 7, 8], [9, 0, 511, 42, 42, 1], [1, 2, 3, 4, 5, 6]]
    refs = [DecodeRef(shape, layers, embed, head, out_norm, 32) for _ in range(batch)]
    for pos in range(len(tokens[0])):
        model.tokens.copy_(torch_tokens([tokens[b][pos] for b in range(batch)]))
        model.step(pos)
        got = model.logits.cpu().numpy().reshape(batch, shape.vocab)
        for b in range(batch):
            assert _rel(got[b], refs[b].step(tokens[b][pos], pos)) <= 2e-3, (b, pos)


def torch_tokens(vals):
    import torch

    return torch.tensor(vals, dtype=torch.int32)


def _parse_xq(raw: np.ndarray, k: int, digits: int):
    """hi codes, lo codes (x16), group scales and group sums of a quantized row."""
    hi = raw[:k].view(np.int8)
    lo = raw[k:2 * k] if digits == 2 else None
    off = k * digits
    d = raw[off:off + 4 * (k // 32)].view(np.float32)
    s = raw[off + 4 * (k // 32):off + 8 * (k // 32)].view(np.int32)
    return hi, lo, d, s


def _check_codes(raw, x, digits):
    from oracle import oracle as O

    k = x.shape[0]
    hi, lo, d, s = _parse_xq(raw, k, digits)
    rh, rl, rd, rs = O.quantize_act(x, digits)
    assert np.array_equal(hi, rh) and np.array_equal(d, rd) and np.array_equal(s, rs)
    if digits == 2:
        assert np.array_equal(lo, rl)


@pytest.mark.gpu
@pytest.mark.parametrize("digits", [1, 2])
def test_quantized_outputs_of_norm_attention_swiglu(digits):
    """The *_q glue writes exactly the codes the activation quantizer would
    write for its fp32 output (the oracle's orc_quantize_act, bit for bit)."""
    import torch
    from cybel_b200 import _native

    L = _native.lib()
    st = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(digits)
    n = 4096
    rb = int(L.b200q_xq_row_bytes(n, digits))
    res = torch.from_numpy(rng.standard_normal(n).astype(np.float32)).cuda()
    gam = torch.from_numpy((1 + 0.1 * rng.standard_normal(n)).astype(np.float32)).cuda()
    out = torch.empty(n, device="cuda")
    xq = torch.zeros(rb, dtype=torch.uint8, device="cuda")
    assert L.b200q_add_rmsnorm_q(res.data_ptr(), None, gam.data_ptr(), out.data_ptr(), xq.data_ptr(), digits, n, 1,
                                 1e-5, st) == 0
    torch.cuda.synchronize()
    _check_codes(xq.cpu().numpy(), out.cpu().numpy(), digits)

    H, KV, hd, ctx, max_ctx = 32, 8, 128, 300, 320
    q = torch.from_numpy(rng.standard_normal(H * hd).astype(np.float32)).cuda()
    kc = torch.from_numpy(rng.standard_normal((KV, max_ctx, hd)).astype(np.float16)).cuda()
    vc = torch.from_numpy(rng.standard_normal((KV, max_ctx, hd)).astype(np.float16)).cuda()
    att = torch.empty(H * hd, device="cuda")
    assert L.b200q_attention_decode_q(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), att.data_ptr(), xq.data_ptr(),
                                      digits, 1, H, KV, hd, ctx, max_ctx, st) == 0
    torch.cuda.synchronize()
    _check_codes(xq.cpu().numpy(), att.cpu().numpy(), digits)

    f = 14336
    g = torch.from_numpy(rng.standard_normal(f).astype(np.float32)).cuda()
    u = torch.from_numpy(rng.standard_normal(f).astype(np.float32)).cuda()
    hf = torch.empty(f, device="cuda")
    xqf = torch.zeros(int(L.b200q_xq_row_bytes(f, digits)), dtype=torch.uint8, device="cuda")
    assert L.b200q_swiglu(g.data_ptr(), u.data_ptr(), hf.data_ptr(), f, st) == 0
    assert L.b200q_swiglu_q(g.data_ptr(), u.data_ptr(), xqf.data_ptr(), digits, f, st) == 0
    torch.cuda.synchronize()
    _check_codes(xqf.cpu().numpy(), hf.cpu().numpy(), digits)


@pytest.mark.gpu
@pytest.mark.parametrize("batch,H,KV,pos", [(1, 32, 8, 2047), (1, 64, 8, 300), (2, 8, 8, 63), (3, 16, 8, 64),
                                            (1, 8, 4, 0), (2, 4, 2, 129)])
def test_rope_attention_fused_matches_two_step_path(batch, H, KV, pos):
    """b200q_rope_attention_decode (one launch) against b200q_rope_kv +
    b200q_attention_decode on copies of the same inputs: same caches (the
    appended value row bit for bit), outputs within 1e-5 relative (fp32 merge
    order differs), the o projection's codes those of its own output; two
    launches in a row (the arrival counters reset themselves)."""
    import torch
    from cybel_b200 import _native

    L = _native.lib()
    st = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(batch * 1000 + H + pos)
    hd, max_ctx = 128, pos + 70
    q = torch.from_numpy(rng.standard_normal(batch * H * hd).astype(np.float32)).cuda()
    k = torch.from_numpy(rng.standard_normal(batch * KV * hd).astype(np.float32)).cuda()
    v = torch.from_numpy(rng.standard_normal(batch * KV * hd).astype(np.float32)).cuda()
    kc = torch.from_numpy(rng.standard_normal((batch, KV, max_ctx, hd)).astype(np.float16)).cuda()
    vc = torch.from_numpy(rng.standard_normal((batch, KV, max_ctx, hd)).astype(np.float16)).cuda()
    kc2, vc2, q2, k2 = kc.clone(), vc.clone(), q.clone(), k.clone()
    out = torch.empty(batch * H * hd, device="cuda")
    ref = torch.empty(batch * H * hd, device="cuda")
    xq = torch.zeros(batch * int(L.b200q_xq_row_bytes(H * hd, 2)), dtype=torch.uint8, device="cuda")
    for _ in range(2):
        assert L.b200q_rope_attention_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), batch, H, KV, hd, pos, 5e5,
                                             kc.data_ptr(), vc.data_ptr(), max_ctx, out.data_ptr(), xq.data_ptr(), 2,
                                             st) == 0
    assert L.b200q_rope_kv(q2.data_ptr(), k2.data_ptr(), v.data_ptr(), batch, H, KV, hd, pos, 5e5, kc2.data_ptr(),
                           vc2.data_ptr(), max_ctx, st) == 0
    assert L.b200q_attention_decode(q2.data_ptr(), kc2.data_ptr(), vc2.data_ptr(), ref.data_ptr(), batch, H, KV, hd,
                                    pos + 1, max_ctx, st) == 0
    torch.cuda.synchronize()
    assert L.b200q_device_status(torch.cuda.current_device()) == 0
    assert torch.equal(vc, vc2)
    # the rotated key: the same fp32 formula in both kernels, so at most an
    # fp16 rounding step apart if the compiler contracts them differently
    assert torch.allclose(kc.float(), kc2.float(), rtol=1e-3, atol=1e-3)
    got, want = out.cpu().numpy(), ref.cpu().numpy()
    assert _rel(got, want) <= 1e-5
    rb = int(L.b200q_xq_row_bytes(H * hd, 2))
    codes = xq.cpu().numpy()
    for b in range(batch):
        _check_codes(codes[b * rb:(b + 1) * rb], got[b * H * hd:(b + 1) * H * hd], 2)


@pytest.mark.gpu
def test_rope_attention_rejects_bad_shapes():
    import torch
    from cybel_b200 import _native

    L = _native.lib()
    st = torch.cuda.current_stream().cuda_stream
    buf = torch.zeros(1 << 20, device="cuda")
    p = buf.data_ptr()
    assert L.b200q_rope_attention_decode(p, p, p, 1, 12, 4, 128, 5, 1e4, p, p, 64, p, None, 0, st) == -3  # G = 3
    assert L.b200q_rope_attention_decode(p, p, p, 1, 8, 8, 64, 5, 1e4, p, p, 64, p, None, 0, st) == -3  # head_dim
    assert L.b200q_rope_attention_decode(p, p, p, 1, 8, 8, 128, 64, 1e4, p, p, 64, p, None, 0, st) == -3  # pos
    assert L.b200q_rope_attention_decode(p, p, p, 1, 8, 8, 128, 5, 1e4, p, p, 64, None, None, 0, st) == -1
    torch.cuda.synchronize()
    assert L.b200q_device_status(torch.cuda.current_device()) == 0
