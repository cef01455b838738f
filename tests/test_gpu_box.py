"""Box-scale decode at full size: 256 sequences on one engine with KV for 4096 positions each
(LLaMA-3.2-1B shape, 68.7 GB of KV), 1024-id prompts, greedy decode, and two sequences carried
on to position 4095.

At this size the oracle needs hours, so parity rests on properties that do not depend on the
size, each path being pinned to the oracle at small sizes by the other test files:

* batch invariance: the logits of sampled sequences (slots 0, 85, 170 and 255, the last one at
  byte offsets past 2^32 elements into the cache) equal those of a one-sequence engine that
  prefills the same ids (query-tiled causal attention instead of per-row decode attention);
* full length: slots 0 and 255 decoded alone (two rows per step, so decode attention is split
  over position ranges and merged) up to position 4095, checked the same way at positions 2047
  and 4095.

Tolerance: max|l - l_ref| <= 1e-3 * max|l_ref| per compared step, greedy ids identical.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_RTOL = 1e-3
B, P, MAXS = 256, 1024, 4096
CHECK = (0, 85, 170, 255)


def rel_max_err(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.fixture(scope="module")
def bindings(pkg, gpu_available):
    return pkg.LlamaEngineBindings()


def _single_logits(single, ids):
    """Last-position logits of a one-sequence engine after prefilling ids from position 0."""
    single.prefill([int(t) for t in ids], 0, True)
    return single.get_logits()


def test_box_scale_decode(pkg, bindings, full_model):
    eng = pkg.LlamaEngine(str(full_model), bindings, device=0, max_batch=B, max_seq_len=MAXS)
    single = pkg.LlamaEngine(str(full_model), bindings, device=0, max_batch=1, max_seq_len=MAXS)
    try:
        assert eng.batch_path == "tensor-core"
        vocab = eng.vocab_size
        prompts = np.random.default_rng(256).integers(0, vocab, (B, P)).astype(np.int32)
        # prompts: 4 positions of every sequence per call, sequence-major rows
        for p0 in range(0, P - 1, 4):
            ps = list(range(p0, min(P - 1, p0 + 4)))
            eng.forward_batch([int(prompts[s, p]) for s in range(B) for p in ps], [p for s in range(B) for p in ps],
                              [s for s in range(B) for p in ps], False)
        seqs = [list(map(int, prompts[s])) for s in range(B)]
        toks = [int(prompts[s, -1]) for s in range(B)]
        kept = {}
        for step in range(64):
            eng.forward_batch(toks, [P - 1 + step] * B, list(range(B)), True)
            toks = eng.argmax_batch(B)
            if step in (0, 63):
                kept[step] = {s: eng.get_logits_batch(s) for s in CHECK}
            for s in range(B):
                seqs[s].append(int(toks[s]))
        for step, rows in kept.items():
            for s in CHECK:
                ref = _single_logits(single, seqs[s][:P + step])
                assert rel_max_err(rows[s], ref) <= LOGIT_RTOL, (step, s)
                assert int(np.argmax(rows[s])) == seqs[s][P + step] == int(np.argmax(ref)), (step, s)

        # slots 0 and 255 alone to position 4095
        pair = [0, B - 1]
        t2 = [seqs[s][-1] for s in pair]
        at = {}
        for pos in range(P - 1 + 64, MAXS):
            eng.forward_batch(t2, [pos, pos], pair, True)
            t2 = eng.argmax_batch(2)
            if pos in (2047, MAXS - 1):
                at[pos] = [eng.get_logits_batch(0), eng.get_logits_batch(1)]
            for i, s in enumerate(pair):
                seqs[s].append(int(t2[i]))
        for pos, rows in at.items():
            for i, s in enumerate(pair):
                ref = _single_logits(single, seqs[s][:pos + 1])
                assert rel_max_err(rows[i], ref) <= LOGIT_RTOL, (pos, s)
                assert int(np.argmax(rows[i])) == int(np.argmax(ref)), (pos, s)
    finally:
        single.close()
        eng.close()
