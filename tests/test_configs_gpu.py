"""Parity at the five benchmark configurations, against the reference op where
one exists.

1. Q4_0 4096 x 4096: W ~ N(0, 0.02) from default_rng(0), packed by gguf-py's
   ``quantize`` (the reference quantizer for Q4_0; this repository's packer
   gives the same bytes), x ~ N(0, 1) from default_rng(1). Integer group sums
   bit-exact against the restatement (orc_isums) in both activation modes;
   fp32 outputs within 1e-5 of ||w_row|| * ||x|| and 1e-3 relative of the
   restatement of the same mode, and (x16) of gguf ``dequantize(W) @ x`` in
   float64. The reference has no Q4_0 kernel.
2. Q4_K and Q8_0 at the four Llama-3-8B shapes (W seed = shape index,
   x seed = 100 + index), x16: device entry point and host drop-in against
   the compiled reference op simd_matvec_* (quantized_matmul.cpp:1536-1571,
   1818) run on the same bytes and x, same bounds; isums bit-exact.
3. Q4_K 14336 x 4096 and 4096 x 14336 at m = 8, 32, 128 (all rows): the
   tile path against the compiled reference simd_matmul_q4k
   (quantized_matmul.cpp:1944-1973): fp16 activations within 1e-4, the
   precise (x16) variant within 1e-5 normalised; 1e-3 relative.
4. One full-width Llama-3-8B layer (hidden 4096, 32 / 8 heads, FFN 14336)
   at context 2048 (KV cache prefilled), batch 1, x16: logits against the
   float64 restatement (oracle/decode_ref.py), ||d||_inf / ||ref||_inf
   <= 2e-3.
5. One full-width Llama-3-70B layer (hidden 8192, 64 / 8 heads, FFN 28672)
   at context 2048 through the row-sharded decode on one rank, batch 1
   (x16) and batch 8 (x8), same bound.
"""

from __future__ import annotations

import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

NORM_TOL = 1e-5
REL_TOL = 1e-3
TILE_F16_TOL = 1e-4
LOGIT_TOL = 2e-3
LLAMA8B = [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336)]


@pytest.fixture(scope="module")
def ref_op(oracle_mod):
    O = oracle_mod
    if not O.ref_available():
        pytest.skip("the reference op (oracle/_ref) was not built")
    os.environ["ANVIL_NUM_THREADS"] = str(len(os.sched_getaffinity(0)))
    return O


def _st():
    import torch

    return torch.cuda.current_stream().cuda_stream


# --------------------------------------------------------------------------- 1
@pytest.fixture(scope="module")
def config1():
    import gguf

    from cybel_b200 import quantize as Q

    w = np.random.default_rng(0).normal(0.0, 0.02, size=(4096, 4096)).astype(np.float32)
    W = np.ascontiguousarray(gguf.quantize(w, gguf.GGMLQuantizationType.Q4_0))
    assert np.array_equal(W, Q.quantize(w, 2))
    x = np.random.default_rng(1).standard_normal(4096).astype(np.float32)
    exact = gguf.dequantize(W, gguf.GGMLQuantizationType.Q4_0).astype(np.float64) @ x.astype(np.float64)
    return W, x, exact


@pytest.mark.parametrize("digits", [1, 2])
def test_config1_q4_0(oracle_mod, config1, digits):
    import torch

    from cybel_b200.quantized_matmul import DeviceMatrix, matvec_isums_device

    O = oracle_mod
    W, x, exact = config1
    k = n = 4096
    dm = DeviceMatrix(2, k, n, W)
    y, isums = matvec_isums_device(torch.from_numpy(x).cuda(), dm, act_mode=digits)
    torch.cuda.synchronize()
    assert np.array_equal(isums.cpu().numpy(), O.isums(W, 2, x, k, n, digits))
    y = y.cpu().numpy()
    wn = O.row_norms(W, 2, k, n)
    yq = O.matvec_q(W, 2, x, k, n, digits)
    assert O.normalized_error(y, yq, wn, x) <= NORM_TOL
    assert O.max_rel_error(y, yq) <= REL_TOL
    if digits == 2:
        assert O.normalized_error(y, exact, wn, x) <= NORM_TOL
        assert O.max_rel_error(y, exact) <= REL_TOL


def test_config1_q4_0_dropin(oracle_mod, config1):
    from cybel_b200 import quantized_matmul as qm

    O = oracle_mod
    W, x, exact = config1
    mat = qm.QuantizedMatrix(name="c1", qtype=2, shape=(4096, 4096), data=W.copy())
    y = qm.matvec(x, mat)  # simd_matvec_q4_0, host buffers, x16
    wn = O.row_norms(W, 2, 4096, 4096)
    assert O.normalized_error(y, exact, wn, x) <= NORM_TOL
    assert O.max_rel_error(y, exact) <= REL_TOL


# --------------------------------------------------------------------------- 2
@pytest.mark.parametrize("qt", [12, 8])
@pytest.mark.parametrize("idx", range(len(LLAMA8B)))
def test_config2_against_reference_op(ref_op, qt, idx):
    import torch

    from cybel_b200 import quantize as Q
    from cybel_b200 import quantized_matmul as qm
    from cybel_b200.quantized_matmul import DeviceMatrix, matvec_isums_device

    O = ref_op
    n, k = LLAMA8B[idx]
    W = Q.quantize(np.random.default_rng(idx).normal(0.0, 0.02, size=(n, k)).astype(np.float32), qt)
    x = np.random.default_rng(100 + idx).standard_normal(k).astype(np.float32)
    ref = O.ref_matvec(qt, W, x, k, n)
    wn = O.row_norms(W, qt, k, n)
    y, isums = matvec_isums_device(torch.from_numpy(x).cuda(), DeviceMatrix(qt, k, n, W), act_mode=2)
    torch.cuda.synchronize()
    assert np.array_equal(isums.cpu().numpy(), O.isums(W, qt, x, k, n, 2))
    mat = qm.QuantizedMatrix(name=f"c2_{qt}_{idx}", qtype=qt, shape=(k, n), data=W.copy())
    for got in (y.cpu().numpy(), qm.matvec(x, mat)):
        assert O.normalized_error(got, ref, wn, x) <= NORM_TOL
        assert O.max_rel_error(got, ref) <= REL_TOL


# --------------------------------------------------------------------------- 3
@pytest.fixture(scope="module")
def config3_weights():
    from cybel_b200 import quantize as Q

    return {(n, k): Q.quantize(np.random.default_rng(n + k).normal(0.0, 0.02, size=(n, k)).astype(np.float32), 12)
            for n, k in [(14336, 4096), (4096, 14336)]}


@pytest.mark.parametrize("act", [3, 2])
@pytest.mark.parametrize("m", [8, 32, 128])
@pytest.mark.parametrize("n,k", [(14336, 4096), (4096, 14336)])
def test_config3_tile_against_reference_op(ref_op, config3_weights, n, k, m, act):
    import torch

    from cybel_b200.quantized_matmul import DeviceMatrix, matmul_device

    O = ref_op
    W = config3_weights[(n, k)]
    X = np.random.default_rng(m).standard_normal((m, k)).astype(np.float32)
    ref = O.ref_matmul(12, W, X, k, n)
    Y = matmul_device(torch.from_numpy(X).cuda(), DeviceMatrix(12, k, n, W), act_mode=act).cpu().numpy()
    wn = O.row_norms(W, 12, k, n)
    assert O.normalized_error(Y, ref, wn, X) <= (TILE_F16_TOL if act == 3 else NORM_TOL)
    assert O.max_rel_error(Y, ref) <= REL_TOL


# ------------------------------------------------------------------------- 4, 5
def _layer_case(shape_name: str):
    from cybel_b200 import decode as D
    from cybel_b200.formats import Q4_K, Q6_K

    base = {"llama3_8b": D.LLAMA3_8B, "llama3_70b": D.LLAMA3_70B}[shape_name]
    # one full-width layer; a short vocabulary (the LM head GEMV is covered by
    # the Q6_K / Q4_K GEMV tests), head type as in the full model
    shape = D.StackShape(layers=1, hidden=base.hidden, heads=base.heads, kv_heads=base.kv_heads, ffn=base.ffn,
                         vocab=2048, head_qtype=base.head_qtype)
    rng = np.random.default_rng(11)
    layer = D.random_layer(shape, rng, block_rows=2048)
    embed = D.random_rows(Q4_K, shape.vocab, shape.hidden, rng, std=1.0)
    head = D.random_rows(shape.head_qtype, shape.vocab, shape.hidden, rng)
    out_norm = (1 + 0.1 * rng.standard_normal(shape.hidden)).astype(np.float32)
    assert shape.head_qtype in (Q4_K, Q6_K)
    return shape, layer, embed, head, out_norm


def _logit_err(got, want):
    return float(np.max(np.abs(got - want)) / np.max(np.abs(want)))


CTX = 2048


def test_config4_llama8b_layer():
    import torch

    from cybel_b200 import decode as D
    from oracle.decode_ref import DecodeRefPacked

    shape, layer, embed, head, out_norm = _layer_case("llama3_8b")
    stack = D.DecodeStack(shape, CTX, [layer], embed, head, out_norm, act_mode=2)
    g = torch.Generator(device="cuda").manual_seed(3)
    stack.k_cache.normal_(generator=g)
    stack.v_cache.normal_(generator=g)
    ref = DecodeRefPacked(shape, [layer], embed, head, out_norm, CTX)
    ref.load_cache(stack.k_cache.float().cpu().numpy()[None], stack.v_cache.float().cpu().numpy()[None])
    pos, token = CTX - 1, 1234
    stack.set_token(token)
    stack.step(pos)
    torch.cuda.synchronize()
    want = ref.step([token], pos)[0]
    assert _logit_err(stack.logits.cpu().numpy(), want) <= LOGIT_TOL


@pytest.mark.parametrize("batch", [1, 8])
def test_config5_llama70b_layer_rowsharded(batch):
    import torch

    from cybel_b200 import _native
    from cybel_b200.sharded import GpuOps, ShardedDecode, ShardPlan, shard_layer, shard_rows
    from oracle.decode_ref import DecodeRefPacked

    shape, layer, embed, head, out_norm = _layer_case("llama3_70b")
    plan = ShardPlan(shape, 1, 0)
    act = _native.ACT_X16 if batch < 8 else _native.ACT_X8
    ops = GpuOps(torch.cuda.current_device(), act_mode=act, world=1, rank=0)
    model = ShardedDecode(plan, CTX, batch, [shard_layer(layer, plan)], embed, shard_rows(head, plan, "head"),
                          out_norm, ops)
    g = torch.Generator(device="cuda").manual_seed(5)
    model.k_cache.normal_(generator=g)
    model.v_cache.normal_(generator=g)
    ref = DecodeRefPacked(shape, [layer], embed, head, out_norm, CTX, batch=batch)
    # device caches are [layer][batch][kv_head][ctx][hd]
    ref.load_cache(model.k_cache.float().cpu().numpy().transpose(1, 0, 2, 3, 4),
                   model.v_cache.float().cpu().numpy().transpose(1, 0, 2, 3, 4))
    pos = CTX - 1
    tokens = [(37 * b + 5) % shape.vocab for b in range(batch)]
    model.tokens.copy_(torch.tensor(tokens, dtype=torch.int32))
    model.step(pos)
    torch.cuda.synchronize()
    got = model.logits.cpu().numpy().reshape(batch, shape.vocab)
    want = ref.step(tokens, pos)
    for b in range(batch):
        assert _logit_err(got[b], want[b]) <= LOGIT_TOL, b
    ops.close()
