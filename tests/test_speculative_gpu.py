"""Batched speculative verify on the device: ``DecodeStack.verify`` (m draft
tokens in one pass: m-row linears -- the tcgen05 tile kernel for Q4_K from 2
rows, the GEMV for the Q6_K head -- and one causal multi-token attention launch per layer)
against the float64 restatement stepping the same tokens one at a time
(oracle/decode_ref.py): every row's logits within max |d| / max |ref| <=
2e-3, for the contiguous fp16 cache and the Q8 paged cache, and a decode
step after a partial acceptance continuing from the right cache state.
``BatchedVerifier`` reaches the acceptance decisions of the reference's
sequential loop (oracle/speculative_ref.py) driven by the restatement.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - b)) / max(np.max(np.abs(b)), 1e-30))


def _model(seed=4):
    from cybel_b200.decode import StackShape, random_layer, random_rows
    from cybel_b200.formats import Q4_K, Q6_K

    shape = StackShape(layers=2, hidden=512, heads=4, kv_heads=2, ffn=768, vocab=512)
    rng = np.random.default_rng(seed)
    layers = [random_layer(shape, rng) for _ in range(shape.layers)]
    embed = random_rows(Q4_K, shape.vocab, shape.hidden, rng, std=1.0)
    head = random_rows(Q6_K, shape.vocab, shape.hidden, rng)
    out_norm = (1 + 0.1 * rng.standard_normal(shape.hidden)).astype(np.float32)
    return shape, layers, embed, head, out_norm


PROMPT = [3, 17, 5, 100, 511]


@pytest.mark.parametrize("kv", ["contiguous", "q8"])
@pytest.mark.parametrize("m", [4, 8, 12])
def test_verify_rows_match_sequential_steps(m, kv):
    from cybel_b200.decode import DecodeStack
    from cybel_b200.repack_policy import RepackPolicy
    from oracle.decode_ref import DecodeRef

    shape, layers, embed, head, out_norm = _model()
    dev = DecodeStack(shape, 64, layers, embed, head, out_norm, repack=RepackPolicy.canonical(), kv=kv, page_size=8)
    ref = DecodeRef(shape, layers, embed, head, out_norm, 64, kv_q8=kv == "q8")
    for pos, tok in enumerate(PROMPT):
        dev.set_token(tok)
        dev.step(pos)
        ref.step(tok, pos)
    draft = [int(t) for t in np.random.default_rng(m).integers(0, shape.vocab, m)]
    rows = dev.verify(draft, len(PROMPT)).cpu().numpy()
    for j, tok in enumerate(draft):
        want = ref.step(tok, len(PROMPT) + j)
        assert _rel(rows[j], want) <= 2e-3, j
    # accept two drafts, then decode the next token at position len(PROMPT) + 2
    nxt = 42
    dev.set_token(nxt)
    dev.step(len(PROMPT) + 2)
    ref2 = DecodeRef(shape, layers, embed, head, out_norm, 64, kv_q8=kv == "q8")
    for pos, tok in enumerate(PROMPT + draft[:2] + [nxt]):
        want = ref2.step(tok, pos)
    assert _rel(dev.logits.cpu().numpy(), want) <= 2e-3


def test_batched_verifier_matches_the_sequential_loop():
    from cybel_b200.decode import DecodeStack
    from cybel_b200.repack_policy import RepackPolicy
    from cybel_b200.speculative import BatchedVerifier
    from oracle.decode_ref import DecodeRef
    from oracle.speculative_ref import sequential_verify, softmax64

    shape, layers, embed, head, out_norm = _model(seed=6)
    dev = DecodeStack(shape, 64, layers, embed, head, out_norm, repack=RepackPolicy.canonical(), kv="contiguous")
    for pos, tok in enumerate(PROMPT):
        dev.set_token(tok)
        dev.step(pos)
    draft = [7, 300, 64, 1]
    T = 1.0

    def engine(ctx):  # the reference's engine call: a fresh pass over the whole context
        r = DecodeRef(shape, layers, embed, head, out_norm, 64)
        for pos, tok in enumerate(ctx):
            out = r.step(tok, pos)
        return out

    # draft probabilities: the target's own for the first two drafts (ratio 1), twice it for the third (ratio 0.5)
    probs = []
    for i in range(len(draft)):
        p = float(softmax64(engine(PROMPT + draft[:i]), T)[draft[i]])
        probs.append(p if i < 2 else 2.0 * p)
    want = sequential_verify(engine, PROMPT, draft, probs, T, 0.7)
    ver = BatchedVerifier(dev, max_draft_length=4, acceptance_threshold=0.7)
    got = ver.verify(PROMPT, draft, probs, T)
    assert want[0] == 2 and got[0] == want[0]
    assert np.allclose(got[1], want[1], rtol=2e-2)
    assert _rel(ver.bonus_logits, engine(PROMPT + draft[:2])) <= 2e-3
