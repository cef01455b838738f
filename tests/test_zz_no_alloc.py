"""The allocation-free greedy argmax (llama_b128_argmax_noalloc) against the engine's own greedy
sampler.

Callers that cannot allocate device memory while running (a memory budget fixed at start-up, or a
decode loop that cannot afford the device synchronisation a cudaMalloc may cause) use this entry
point; its scratch is a fixed device array inside the library.  This file is collected last so
that a run stopping at the first failure has already run every other test.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_argmax_noalloc_matches_engine_greedy(pkg, small_model, gpu_available):
    import torch

    bindings = pkg.LlamaEngineBindings()
    lib = bindings.lib
    eng = pkg.LlamaEngine(str(small_model), bindings)
    out = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    try:
        # two calls in a row, each on fresh logits, against llama_engine_sample(temperature 0)
        for pos, tok in enumerate([17, 523]):
            eng.forward_token(tok, pos, True)
            logits = torch.from_numpy(eng.get_logits()).cuda()
            assert lib.llama_b128_argmax_noalloc(logits.data_ptr(), logits.numel(), out.data_ptr(), None) == 0
            torch.cuda.synchronize()
            assert int(out.item()) == eng.sample(0.0, 0.9)
        # after a temperature draw the engine's greedy path re-reduces its rewritten logits with
        # the same kernels and engine-owned scratch; both must agree again, twice
        for _ in range(2):
            eng.sample(0.9, 0.9)
            probs = torch.from_numpy(eng.get_logits()).cuda()
            assert lib.llama_b128_argmax_noalloc(probs.data_ptr(), probs.numel(), out.data_ptr(), None) == 0
            torch.cuda.synchronize()
            assert int(out.item()) == eng.sample(0.0, 0.9)
        # ties resolve to the first index, as in the reference
        tied = np.zeros(100_000, np.float32)
        tied[[40_000, 7, 99_999]] = 3.5
        t = torch.from_numpy(tied).cuda()
        assert lib.llama_b128_argmax_noalloc(t.data_ptr(), t.numel(), out.data_ptr(), None) == 0
        torch.cuda.synchronize()
        assert int(out.item()) == 7
        # sizes beyond the scratch array's reach are rejected
        assert lib.llama_b128_argmax_noalloc(t.data_ptr(), 16_777_217, out.data_ptr(), None) == -2
    finally:
        eng.close()
