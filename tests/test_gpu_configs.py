"""Parity at the benchmark configurations' own shapes, on the LLaMA-3.2-1B model, against golden
fixtures that the reference engine itself produced (tests/golden/make_golden.py):

* config 3 — prefill of 8 prompts of 2048 ids on the batched tensor-core path; the last
  position's logits (all 128,256) within 1e-3 of the reference's, greedy id identical;
* config 2 — 64 sequences (512-id prompts) fed through forward_batch, then 32 batched greedy
  decode steps of all 64 rows; each step's ids come from the reference run (teacher forcing, so a
  near-tie cannot derail the comparison), and every row's greedy id, top-16 logits and 128 sampled
  logits are checked against it.  A greedy id may differ only where the reference's own top-2
  margin is below 1e-4 and the engine chose the reference's runner-up (reported as a tie).

Tolerance: max |l - l_ref| <= 1e-3 * max |l_ref| per row ("1e-3 relative").
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

LOGIT_RTOL = 1e-3
TIE_MARGIN = 1e-4  # a reference top-2 margin below this counts as a tie for the greedy id


@pytest.fixture(scope="module")
def bindings(pkg, gpu_available):
    return pkg.LlamaEngineBindings()


def _fixture(name):
    p = GOLDEN / name
    if not p.exists():
        pytest.skip(f"{name} not generated")
    return np.load(p)


def test_config3_prefill_2048_vs_reference(pkg, bindings, full_model):
    g = _fixture("config3_prefill.npz")
    assert pkg.model_file.file_sha256(full_model) == str(g["model_sha256"]), "generator output differs"
    eng = pkg.LlamaEngine(str(full_model), bindings)
    try:
        assert eng.batch_path == "tensor-core", bindings.last_error(eng.handle)
        errs = []
        for i, prompt in enumerate(g["prompts"]):
            eng.prefill([int(t) for t in prompt], 0, True)
            lg = eng.get_logits()
            ref = g["logits"][i]
            err = float(np.abs(lg - ref).max() / np.abs(ref).max())
            errs.append(err)
            assert err <= LOGIT_RTOL, f"prompt {i}: rel err {err:.3e}"
            tok = eng.sample(0.0, 0.9)
            assert tok == int(g["tokens"][i]), f"prompt {i}: greedy id (top-2 margin {float(g['margins'][i]):.3g})"
        print(f"config 3: max rel err over 8 prompts {max(errs):.3e}")
    finally:
        eng.close()


def test_config2_batched_decode_vs_reference(pkg, bindings, full_model):
    g = _fixture("config2_decode.npz")
    assert pkg.model_file.file_sha256(full_model) == str(g["model_sha256"]), "generator output differs"
    prompts, ref_tok = g["prompts"], g["tokens"]
    B, P = prompts.shape
    steps = ref_tok.shape[1]
    idx = g["sample_idx"]
    eng = pkg.LlamaEngine(str(full_model), bindings, device=0, max_batch=B, max_seq_len=P + steps + 8)
    try:
        assert eng.batch_path == "tensor-core", bindings.last_error(eng.handle)
        per = 1024 // B
        slots = list(range(B))
        for p0 in range(0, P - 1, per):
            ps = list(range(p0, min(P - 1, p0 + per)))
            eng.forward_batch([int(prompts[s, p]) for p in ps for s in slots], [p for p in ps for s in slots],
                              [s for p in ps for s in slots], False)
        toks = [int(prompts[s, P - 1]) for s in slots]
        worst = 0.0
        ties = []
        for step in range(steps):
            pos = P - 1 + step
            eng.forward_batch(toks, [pos] * B, slots, True)
            am = eng.argmax_batch(B)
            for s in slots:
                lg = eng.get_logits_batch(s)
                scale = max(float(np.abs(g["top_vals"][s, step]).max()), float(np.abs(g["sampled"][s, step]).max()))
                e1 = float(np.abs(lg[idx] - g["sampled"][s, step]).max()) / scale
                e2 = float(np.abs(lg[g["top_ids"][s, step]] - g["top_vals"][s, step]).max()) / scale
                worst = max(worst, e1, e2)
                assert e1 <= LOGIT_RTOL and e2 <= LOGIT_RTOL, f"step {step} seq {s}: {e1:.3e} {e2:.3e}"
                if am[s] != int(ref_tok[s, step]):
                    # a tie within the rounding of a different summation order: the reference's own
                    # top-2 margin is below 1e-4 and the engine picked its runner-up
                    margin = float(g["margins"][s, step])
                    assert margin < TIE_MARGIN and am[s] == int(g["top_ids"][s, step, 1]), \
                        f"step {step} seq {s}: greedy id {am[s]} vs {int(ref_tok[s, step])} (top-2 margin {margin:.3g})"
                    ties.append((step, s, margin))
            toks = [int(t) for t in ref_tok[:, step]]
        print(f"config 2: worst rel err over {B} x {steps} rows {worst:.3e}; near-ties taken the other way: {ties}")
    finally:
        eng.close()
