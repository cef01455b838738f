"""Host logic of the scoring helpers (context truncation, window split, sums) over a fake engine
that records its calls; no GPU."""
from __future__ import annotations

import numpy as np
import pytest


class FakeEngine:
    """score_tokens returns log P = -(token id) / 1000 and greedy = (id even)."""

    def __init__(self):
        self.calls = []

    def reset(self):
        self.calls.append(("reset",))

    def prefill(self, tokens, start_pos, compute_last_logits=False):
        self.calls.append(("prefill", list(tokens), start_pos, compute_last_logits))

    def score_tokens(self, tokens, start_pos=0):
        self.calls.append(("score", list(tokens), start_pos))
        t = np.array(tokens[1:], dtype=np.float32)
        return -t / 1000.0, (np.array(tokens[1:]) % 2 == 0)


def test_loglikelihood_calls_and_sum(pkg):
    e = FakeEngine()
    total, greedy = pkg.scoring.loglikelihood(e, [5, 6, 7], [8, 10])
    assert e.calls == [("reset",), ("prefill", [5, 6], 0, False), ("score", [7, 8, 10], 2)]
    assert total == pytest.approx(-(8 + 10) / 1000.0)
    assert greedy
    assert pkg.scoring.loglikelihood(e, [5], [9])[1] is False


def test_loglikelihood_single_context_token_skips_prefill(pkg):
    e = FakeEngine()
    pkg.scoring.loglikelihood(e, [5], [8])
    assert e.calls == [("reset",), ("score", [5, 8], 0)]


def test_loglikelihood_truncates_context_like_the_adapter(pkg):
    e = FakeEngine()
    # 6 context + 3 continuation > 7: keep the last 4 context tokens
    pkg.scoring.loglikelihood(e, [1, 2, 3, 4, 5, 6], [7, 8, 9], max_length=7)
    assert e.calls[1] == ("prefill", [3, 4, 5], 0, False)
    assert e.calls[2] == ("score", [6, 7, 8, 9], 3)
    # continuation alone over the limit: one context token survives
    e = FakeEngine()
    pkg.scoring.loglikelihood(e, [1, 2, 3], [7, 8, 9, 10], max_length=3)
    assert e.calls[1] == ("score", [3, 7, 8, 9, 10], 0)


def test_loglikelihood_empty_cases(pkg):
    e = FakeEngine()
    assert pkg.scoring.loglikelihood(e, [1], []) == (0.0, True)
    assert e.calls == []
    with pytest.raises(ValueError):
        pkg.scoring.loglikelihood(e, [], [1])


def test_rolling_windows_overlap_by_one(pkg):
    e = FakeEngine()
    toks = list(range(10, 20))  # 10 tokens + prefix = 11
    total = pkg.scoring.loglikelihood_rolling(e, toks, prefix_token_id=1, max_length=4)
    scores = [c for c in e.calls if c[0] == "score"]
    assert [c[1] for c in scores] == [[1, 10, 11, 12], [12, 13, 14, 15], [15, 16, 17, 18], [18, 19]]
    assert all(c[2] == 0 for c in scores)
    # every token after the prefix is scored exactly once
    assert total == pytest.approx(-sum(toks) / 1000.0, rel=1e-6)
    assert pkg.scoring.loglikelihood_rolling(FakeEngine(), [], 1, 4) == 0.0
