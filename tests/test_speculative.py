"""Batched speculative verify, host side: the restated softmax guards
(cpu_speculative_decode.py:33-83) on known answers, and the acceptance loop
fed by one batched pass equal to the reference's sequential loop
(oracle/speculative_ref.py) on the same logits, with and without a logits
processor and draft probabilities."""

from __future__ import annotations

import numpy as np
import pytest

from cybel_b200.speculative import BatchedVerifier, accept_prefix, sanitize_logits, stable_softmax
from oracle.speculative_ref import sequential_verify


def test_softmax_guards():
    assert np.allclose(stable_softmax(np.array([-np.inf, -np.inf, np.nan], np.float32)), 1 / 3)
    p = stable_softmax(np.array([0.0, -100.0], np.float32))  # shifted logits clipped at -80
    assert np.isclose(p[1], np.exp(np.float32(-80.0)), rtol=1e-5)
    p = stable_softmax(np.array([np.nan, 1.0, np.inf], np.float32))  # nan / inf floored to min - 1e4
    assert p[0] == p[2] and np.isclose(p[1], 1.0)
    assert np.array_equal(sanitize_logits(np.array([np.inf, 2.0], np.float32)), np.array([2.0 - 1e4, 2.0], np.float32))
    x = np.random.default_rng(0).standard_normal(50).astype(np.float32)
    e = np.exp((x - x.max()) / 0.5)
    assert np.allclose(stable_softmax(x, 0.5), e / e.sum(), rtol=1e-5)


def _ban(token):
    def proc(tokens, logits):
        out = logits.copy()
        out[token] = -np.inf
        return out
    return proc


@pytest.mark.parametrize("use_probs", [False, True])
@pytest.mark.parametrize("proc", [None, "ban"])
def test_accept_prefix_equals_sequential_loop(use_probs, proc):
    rng = np.random.default_rng(1)
    V, m = 64, 6
    prompt = [5, 9, 2]
    draft = [int(t) for t in rng.integers(0, V, m)]
    table = {len(prompt) + i: (3.0 * rng.standard_normal(V)).astype(np.float32) for i in range(m)}
    for i, t in enumerate(draft):  # make most drafts likely, one not
        table[len(prompt) + i][t] += 6.0 if i != 4 else -6.0
    probs = [0.5] * m if use_probs else None
    processor = _ban(draft[2]) if proc else None
    engine = (lambda ctx: table[len(ctx)])
    want = sequential_verify(engine, prompt, draft, probs, 0.8, 0.7, processor)
    got = accept_prefix([table[len(prompt) + i] for i in range(m)], prompt, draft, probs, 0.8, 0.7, processor)
    assert got[0] == want[0]
    assert np.allclose(got[1], want[1], rtol=1e-5)


class _FakeStack:
    """Rows of a batched pass looked up from a table (host only)."""

    def __init__(self, table, n_prompt):
        import torch

        self.table, self.n_prompt = table, n_prompt
        self.logits = torch.from_numpy(table[n_prompt])
        self.calls = []

    def verify(self, tokens, pos0):
        import torch

        self.calls.append((list(tokens), pos0))
        return torch.from_numpy(np.stack([self.table[pos0 + 1 + j] for j in range(len(tokens))]))


def test_batched_verifier_wiring():
    rng = np.random.default_rng(2)
    V, prompt = 32, [1, 2, 3, 4]
    draft = [7, 8, 9, 10]
    table = {len(prompt) + i: rng.standard_normal(V).astype(np.float32) for i in range(len(draft) + 1)}
    for i, t in enumerate(draft):
        table[len(prompt) + i][t] += 8.0 if i < 3 else -8.0
    st = _FakeStack(table, len(prompt))
    ver = BatchedVerifier(st, max_draft_length=4, acceptance_threshold=0.7)
    got = ver.verify(prompt, draft, None, 1.0)
    want = sequential_verify(lambda ctx: table[len(ctx)], prompt, draft, None, 1.0, 0.7)
    assert st.calls == [(draft, len(prompt))]  # one pass, the drafts at positions 4..7
    assert got[0] == want[0] == 3 and np.allclose(got[1], want[1], rtol=1e-5)
    assert np.array_equal(ver.bonus_logits, table[len(prompt) + 3])  # logits after the 3rd accepted draft
