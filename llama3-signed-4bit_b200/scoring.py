"""Log-likelihood scoring over the engine, for evaluation harnesses.

The reference's lm-eval adapter (tests/lm_eval_adapter.py:111-229) scores a continuation by
calling forward_token with logits for every token, copying the vocab_size logits to the host and
forming (l - max l) - log(sum exp(l - max l)) with numpy.  The functions here give the same sums
through ``LlamaEngine.score_tokens``: the token run goes through the batched path in chunks, and
the log-softmax, the gather of the target's log-probability and the greedy test run on the device,
so only one float and one flag per token cross to the host.
"""
from __future__ import annotations

import numpy as np


def loglikelihood(engine, ctx_tokens: list[int], cont_tokens: list[int],
                  max_length: int | None = None) -> tuple[float, bool]:
    """log P(cont | ctx) and whether every continuation token is the greedy id, as in
    tests/lm_eval_adapter.py:111-190: the context is left-truncated so that context plus
    continuation fit in ``max_length`` (at least one context token kept), prefilled up to its
    last token, and the continuation is scored from the position of that last token.
    An empty continuation scores (0.0, True).  The caller substitutes a prefix token for an
    empty context, as the adapter does (:123-128)."""
    cont = [int(t) for t in cont_tokens]
    if not cont:
        return 0.0, True
    ctx = [int(t) for t in ctx_tokens]
    if not ctx:
        raise ValueError("loglikelihood: empty context (pass the prefix token)")
    if max_length is not None and len(ctx) + len(cont) > max_length:
        ctx = ctx[-max(1, max_length - len(cont)):]
    engine.reset()
    if len(ctx) > 1:
        engine.prefill(ctx[:-1], 0, False)
    lp, greedy = engine.score_tokens([ctx[-1]] + cont, len(ctx) - 1)
    return float(np.sum(lp, dtype=np.float64)), bool(greedy.all())


def loglikelihood_rolling(engine, tokens: list[int], prefix_token_id: int, max_length: int) -> float:
    """Sum of log P(token | earlier tokens) over a text split into windows of ``max_length``
    tokens that overlap by one, each window scored from position 0 after a reset
    (tests/lm_eval_adapter.py:192-229).  The prefix token is prepended; an empty text scores
    0.0."""
    if not tokens:
        return 0.0
    if max_length < 2:
        raise ValueError("loglikelihood_rolling: max_length must be at least 2")
    seq = [int(prefix_token_id)] + [int(t) for t in tokens]
    total = 0.0
    for start in range(0, len(seq) - 1, max_length - 1):
        window = seq[start:start + max_length]
        if len(window) <= 1:
            break
        engine.reset()
        lp, _ = engine.score_tokens(window, 0)
        total += float(np.sum(lp, dtype=np.float64))
    return total
