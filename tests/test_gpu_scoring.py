"""GPU parity of llama_engine_score_tokens (device log-softmax + gather) against the oracle engine
with the lm-eval adapter's host formula (tests/lm_eval_adapter.py:175-181 of the reference).

Tolerance: each logit is within 1e-3 * max|l_ref| of the oracle's, so a log-probability
(l[t] - logsumexp(l)) is within twice that; greedy flags must match exactly.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import fptr

pytestmark = pytest.mark.gpu

LOGIT_RTOL = 1e-3


@pytest.fixture(scope="module")
def bindings(pkg, gpu_available):
    return pkg.LlamaEngineBindings()


def _oracle_logits(oracle_lib, o, vocab):
    return np.ctypeslib.as_array(oracle_lib.orc_get_logits(o), shape=(vocab,)).copy()


def _adapter_logprob(logits, target):
    """The reference adapter's numpy expression, in float32 as there."""
    max_l = np.max(logits)
    log_probs = (logits - max_l) - np.log(np.sum(np.exp(logits - max_l)))
    return float(log_probs[target]), int(np.argmax(logits)) == int(target)


def _oracle_walk(oracle_lib, o, vocab, n, rng):
    """n tokens through the oracle from position 0: every third next token is the oracle's greedy
    id (so the greedy flag is exercised both ways), the rest random.  Returns the ids and the
    adapter's log-probability and greedy flag for each next token."""
    ids = [int(rng.integers(0, vocab))]
    lps, greedy, scale = [], [], 0.0
    for i in range(n - 1):
        oracle_lib.orc_forward_token(o, ids[i], i, 1)
        lg = _oracle_logits(oracle_lib, o, vocab)
        scale = max(scale, float(np.abs(lg).max()))
        nxt = int(np.argmax(lg)) if i % 3 == 0 else int(rng.integers(0, vocab))
        lp, g = _adapter_logprob(lg, nxt)
        ids.append(nxt)
        lps.append(lp)
        greedy.append(g)
    return ids, np.array(lps), np.array(greedy), scale


@pytest.mark.parametrize("batched", [True, False])
def test_score_tokens_vs_oracle(pkg, bindings, small_model, oracle_lib, monkeypatch, batched):
    """300 tokens (two chunks of the batched path: 256 + 44 rows) or 24 tokens token by token;
    every position's log-probability and greedy flag against the oracle."""
    if not batched:
        monkeypatch.setenv("LLAMA_B200_BATCHED", "0")
    eng = pkg.LlamaEngine(str(small_model), bindings)
    o = oracle_lib.orc_create(str(small_model).encode())
    try:
        assert eng.batch_path == ("tensor-core" if batched else "token-loop")
        vocab = eng.vocab_size
        n = 300 if batched else 24
        ids, ref_lp, ref_g, scale = _oracle_walk(oracle_lib, o, vocab, n, np.random.default_rng(404 + n))
        assert ref_g.any() and not ref_g.all()
        lp, g = eng.score_tokens(ids, 0)
        assert lp.shape == (n - 1,)
        assert np.abs(lp - ref_lp).max() <= 2 * LOGIT_RTOL * scale
        assert (g == ref_g).all()
        # the current logits are those of the last token
        oracle_lib.orc_forward_token(o, int(ids[-1]), n - 1, 1)
        ref = _oracle_logits(oracle_lib, o, vocab)
        assert np.abs(eng.get_logits() - ref).max() <= LOGIT_RTOL * np.abs(ref).max()
        assert eng.sample(0.0, 0.9) == int(np.argmax(ref))
    finally:
        oracle_lib.orc_free(o)
        eng.close()


def test_loglikelihood_matches_adapter_loop(pkg, bindings, small_model, oracle_lib):
    """scoring.loglikelihood (prefill of the context, then one score_tokens call from the last
    context position) against the adapter's forward_token loop replayed on the oracle, with a
    greedy continuation so that the all-greedy flag is True."""
    eng = pkg.LlamaEngine(str(small_model), bindings)
    o = oracle_lib.orc_create(str(small_model).encode())
    try:
        vocab = eng.vocab_size
        rng = np.random.default_rng(9)
        ctx = [int(t) for t in rng.integers(0, vocab, 37)]
        # oracle: prefill ctx[:-1], forward ctx[-1]; continuation = 5 greedy tokens + 1 random
        oracle_lib.orc_prefill(o, fptr(np.array(ctx, np.int32)), len(ctx) - 1, 0, 0)
        pos = len(ctx) - 1
        tok = ctx[-1]
        cont, ref_sum, scale = [], 0.0, 0.0
        for i in range(6):
            oracle_lib.orc_forward_token(o, tok, pos, 1)
            lg = _oracle_logits(oracle_lib, o, vocab)
            scale = max(scale, float(np.abs(lg).max()))
            nxt = int(np.argmax(lg)) if i < 5 else int((np.argmax(lg) + 1) % vocab)
            ref_sum += _adapter_logprob(lg, nxt)[0]
            cont.append(nxt)
            tok, pos = nxt, pos + 1
        total, greedy = pkg.scoring.loglikelihood(eng, ctx, cont[:5])
        assert greedy
        total6, greedy6 = pkg.scoring.loglikelihood(eng, ctx, cont)
        assert not greedy6
        assert abs(total6 - ref_sum) <= 6 * 2 * LOGIT_RTOL * scale
        assert total6 < total
    finally:
        oracle_lib.orc_free(o)
        eng.close()


def test_score_tokens_rejects_bad_args(pkg, bindings, small_model):
    eng = pkg.LlamaEngine(str(small_model), bindings)
    try:
        lib = bindings.lib
        one = (ctypes.c_int32 * 2)(1, 2)
        out = (ctypes.c_float * 2)()
        assert lib.llama_engine_score_tokens(eng.handle, one, 1, 0, out, None) == -1  # n < 2
        assert lib.llama_engine_score_tokens(eng.handle, None, 2, 0, out, None) == -1
        assert lib.llama_engine_score_tokens(eng.handle, one, 2, 0, None, None) == -1
        assert lib.llama_engine_score_tokens(eng.handle, one, 2, eng.max_seq_len - 1, out, None) == -1
        assert lib.llama_engine_score_tokens(None, one, 2, 0, out, None) == -1
        # the last two positions are still valid
        assert lib.llama_engine_score_tokens(eng.handle, one, 2, eng.max_seq_len - 2, out, None) == 0
    finally:
        eng.close()
