"""CPU restatement of the reference's sequential speculative verify --
TEST INFRASTRUCTURE ONLY (imported by tests; never by the product).

Follows SSMSelfSpeculativeDecoder.verify (JSBuild/src/verso/Anvil/core/
native/cpu_speculative_decode.py:740-769): for each drafted token i, the
engine's logits for prompt + drafts[:i] (one engine call per prefix), the
logits processor applied, probabilities softmax(logits / T), the ratio
min(1, p[draft_i] / max(q_i, 1e-8)) (q_i = 1 without draft probabilities),
stop at the first ratio below the threshold. The softmax here is the plain
float64 formula; the reference's guards (cpu_speculative_decode.py:53-83)
only act on non-finite or underflowing logits, which these tests avoid.
"""

from __future__ import annotations

import numpy as np


def softmax64(logits, temperature: float) -> np.ndarray:
    x = np.asarray(logits, dtype=np.float64) / max(float(temperature), 1e-8)
    e = np.exp(x - x.max())
    return e / e.sum()


def sequential_verify(engine_logits, prompt_tokens, draft_tokens, draft_probs, temperature, threshold,
                      logits_processor=None):
    """engine_logits(context tokens) -> logits; returns (accepted, ratios)."""
    accepted, ratios = 0, []
    context = [int(t) for t in prompt_tokens]
    for i, token in enumerate(draft_tokens):
        logits = np.asarray(engine_logits(list(context)), dtype=np.float32)
        if logits_processor is not None:
            out = logits_processor(list(context), logits)
            logits = logits if out is None else np.asarray(out, dtype=np.float32)
        p = float(softmax64(logits, max(temperature, 1e-8))[int(token)])
        q = float(draft_probs[i]) if draft_probs is not None and i < len(draft_probs) else 1.0
        ratio = min(1.0, p / max(q, 1e-8))
        ratios.append(ratio)
        if ratio < threshold:
            break
        accepted += 1
        context.append(int(token))
    return accepted, ratios
