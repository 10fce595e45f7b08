"""Batched speculative verify over the device decode stack.

The reference's self-speculative decoder (JSBuild/src/verso/Anvil/core/
native/cpu_speculative_decode.py:671-769, SSMSelfSpeculativeDecoder) checks
drafted tokens one at a time: for draft i it asks the engine for the logits
of prompt + drafts[:i], takes p = softmax(logits / T)[draft_i], and accepts
while min(1, p / q_i) >= acceptance_threshold (q_i: the draft's own
probability). Each of those logits is a full pass over the weights.

``BatchedVerifier`` gets the same logits from ONE pass: the drafted tokens
run through ``DecodeStack.verify`` as m rows at consecutive positions, so
every quantized linear streams its weights once for all of them (the tile
kernel from 8 rows), and row j of the result is the logits after draft j --
the context logits of draft j + 1. The acceptance rule, the NaN-safe softmax
(cpu_speculative_decode.py:53-83) and the logits-processor hook
(cpu_speculative_decode.py:683-699) are restated here on the host.
"""

from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

import numpy as np


def sanitize_logits(logits) -> np.ndarray:
    """Non-finite entries replaced by (finite min - 1e4); all-non-finite ->
    zeros (cpu_speculative_decode.py:33-41)."""
    x = np.asarray(logits, dtype=np.float32)
    if x.size <= 0:
        return x
    finite = np.isfinite(x)
    if not np.any(finite):
        return np.zeros_like(x, dtype=np.float32)
    floor = float(np.min(x[finite])) - 1.0e4
    return np.where(finite, x, floor).astype(np.float32, copy=False)


def stable_softmax(logits, temperature: float = 1.0) -> np.ndarray:
    """fp32 softmax of logits / T with the reference's guards
    (cpu_speculative_decode.py:53-83): non-finite entries floored, shifted
    logits clipped to [-80, 0], a uniform distribution over the finite
    entries when the sum is not usable."""
    x = np.asarray(logits, dtype=np.float32)
    if x.size <= 0:
        return x
    finite = np.isfinite(x)
    n_finite = int(np.sum(finite))
    if n_finite <= 0:
        return np.full(x.shape, 1.0 / float(x.size), dtype=np.float32)
    floor = float(np.min(x[finite])) - 1.0e4
    x = np.where(finite, x, floor)
    x = x / max(float(temperature), 1e-8)
    x = x - float(np.max(x))
    x = np.clip(x, -80.0, 0.0)
    e = np.exp(x).astype(np.float32, copy=False)
    total = float(np.sum(e))
    if total <= 0.0 or not np.isfinite(total):
        out = np.zeros_like(e)
        out[finite] = 1.0 / float(n_finite)
        return out
    probs = e / total
    if not np.all(np.isfinite(probs)) or np.any(probs < 0):
        out = np.zeros_like(probs)
        out[finite] = 1.0 / float(n_finite)
        return out
    return probs


def apply_logits_processor(tokens: List[int], logits, processor) -> np.ndarray:
    """The reference's hook (cpu_speculative_decode.py:683-699): a callable
    or a list of callables (tokens, logits) -> logits or None (None keeps
    the current logits); every result sanitized."""
    out = sanitize_logits(logits)
    if processor is None:
        return out
    for p in (processor if isinstance(processor, list) else [processor]):
        nxt = p(tokens, out)
        if nxt is not None:
            out = sanitize_logits(nxt)
    return out


def accept_prefix(context_logits: Sequence, prompt_tokens: Sequence[int], draft_tokens: Sequence[int],
                  draft_probs: Optional[Sequence[float]], temperature: float, threshold: float,
                  logits_processor: Optional[Callable] = None) -> Tuple[int, List[float]]:
    """The acceptance loop of verify() (cpu_speculative_decode.py:740-769)
    given context_logits[i] = logits of prompt + drafts[:i]."""
    accepted, ratios = 0, []
    context = [int(t) for t in prompt_tokens]
    for i, token in enumerate(draft_tokens):
        logits = apply_logits_processor(context, context_logits[i], logits_processor)
        probs = stable_softmax(logits, temperature=max(temperature, 1e-8))
        target = float(probs[int(token)])
        proposal = float(draft_probs[i]) if draft_probs is not None and i < len(draft_probs) else 1.0
        ratio = min(1.0, target / max(proposal, 1e-8))
        ratios.append(ratio)
        if ratio < threshold:
            break
        accepted += 1
        context.append(int(token))
    return accepted, ratios


class BatchedVerifier:
    """Speculative verify over a ``DecodeStack`` whose cache holds the prompt.

    ``verify(prompt_tokens, draft_tokens, draft_probs, temperature,
    logits_processor, last_logits)`` has the reference's arguments and result
    (accepted prefix length, ratios) plus ``last_logits``: the logits after
    the last prompt token (the stack's ``logits`` after its last step).
    ``bonus_logits`` afterwards holds the logits after the last accepted
    token, for sampling the next one."""

    def __init__(self, stack, max_draft_length: int = 4, acceptance_threshold: float = 0.7):
        self.stack = stack
        self.max_draft_length = int(max(1, max_draft_length))
        self.acceptance_threshold = float(np.clip(acceptance_threshold, 0.0, 1.0))
        self.bonus_logits: Optional[np.ndarray] = None

    def verify(self, prompt_tokens: Sequence[int], draft_tokens: Sequence[int],
               draft_probs: Optional[Sequence[float]] = None, temperature: float = 0.8,
               logits_processor: Optional[Callable] = None, last_logits=None) -> Tuple[int, List[float]]:
        import torch

        draft = [int(t) for t in draft_tokens][: self.max_draft_length]
        if last_logits is None:
            last_logits = self.stack.logits
        last = last_logits.cpu().numpy() if isinstance(last_logits, torch.Tensor) else np.asarray(last_logits)
        if not draft:
            self.bonus_logits = last
            return 0, []
        rows = self.stack.verify(draft, len(prompt_tokens)).cpu().numpy()
        contexts = [last] + [rows[j] for j in range(len(draft) - 1)]
        accepted, ratios = accept_prefix(contexts, prompt_tokens, draft, draft_probs, temperature,
                                         self.acceptance_threshold, logits_processor)
        self.bonus_logits = last if accepted == 0 else rows[accepted - 1]
        return accepted, ratios
