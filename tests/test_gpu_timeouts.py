"""The error path of the bounded device waits, exercised without a fault.

Every wait in the persistent token-step kernel, the tensor-core GEMM and the prefill attention is
bounded in time; on timeout the launch records an error word, drains its own copies and returns.
These tests shorten the bound to a millisecond and make one launch wait on a device word that
nothing writes (``llama_engine_debug_waits``), then check that

* the launch returns (no hang) and the next waiting call reports the timeout,
* after the hook is turned off and the error cleared, the same engine again matches the oracle.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import fptr

pytestmark = pytest.mark.gpu

LOGIT_RTOL = 1e-3
WAIT_NS = 1_000_000  # 1 ms


def rel_max_err(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.fixture(scope="module")
def bindings(pkg, gpu_available):
    return pkg.LlamaEngineBindings()


def _oracle_run(oracle_lib, model, ids, n_steps):
    """Greedy run on the oracle: prefill ids[:-1], then n_steps greedy steps; ids and logits."""
    o = oracle_lib.orc_create(str(model).encode())
    try:
        vocab = oracle_lib.orc_get_vocab(o)
        pre = np.ascontiguousarray(ids[:-1], dtype=np.int32)
        oracle_lib.orc_prefill(o, fptr(pre), len(pre), 0, 0)
        tok, pos = int(ids[-1]), len(ids) - 1
        toks, logits = [], []
        for _ in range(n_steps):
            oracle_lib.orc_forward_token(o, tok, pos, 1)
            logits.append(np.ctypeslib.as_array(oracle_lib.orc_get_logits(o), shape=(vocab,)).copy())
            tok = oracle_lib.orc_sample_engine(o, ctypes.c_float(0.0), ctypes.c_float(0.9))
            toks.append(tok)
            pos += 1
        return toks, logits
    finally:
        oracle_lib.orc_free(o)


def test_persistent_kernel_wait_expires_and_engine_recovers(pkg, bindings, small_model, oracle_lib):
    eng = pkg.LlamaEngine(str(small_model), bindings)
    try:
        assert eng.decode_path == "persistent", bindings.last_error(eng.handle)
        lib = bindings.lib
        ids = np.random.default_rng(21).integers(0, eng.vocab_size, 12).astype(np.int32)
        eng.prefill([int(t) for t in ids[:-1]], 0, False)
        assert lib.llama_engine_debug_waits(eng.handle, WAIT_NS, 9999) == 0
        out = (ctypes.c_int32 * 4)()
        rc = lib.llama_engine_generate_greedy(eng.handle, int(ids[-1]), len(ids) - 1, 4, out)
        assert rc == -1
        msg = bindings.last_error(eng.handle)
        assert "timed out" in msg, msg
        # the error stays reported until it is cleared
        assert lib.llama_engine_generate_greedy(eng.handle, int(ids[-1]), len(ids) - 1, 1, out) == -1
        assert lib.llama_engine_debug_waits(eng.handle, 0, 0) == 0
        # the engine works again: redo the steps (the failed ones left garbage in the KV cache)
        ref_toks, ref_logits = _oracle_run(oracle_lib, small_model, ids, 4)
        eng.prefill([int(t) for t in ids[:-1]], 0, False)
        tok, pos = int(ids[-1]), len(ids) - 1
        for s in range(4):
            eng.forward_token(tok, pos, True)
            assert rel_max_err(eng.get_logits(), ref_logits[s]) <= LOGIT_RTOL
            tok = eng.sample(0.0, 0.9)
            assert tok == ref_toks[s]
            pos += 1
    finally:
        eng.close()


def test_tensor_core_gemm_wait_expires_and_engine_recovers(pkg, bindings, small_model, oracle_lib):
    eng = pkg.LlamaEngine(str(small_model), bindings, max_batch=4)
    try:
        if eng.batch_path != "tensor-core":
            pytest.skip("batched path not on the tensor cores: " + bindings.last_error(eng.handle))
        lib = bindings.lib
        ids = np.random.default_rng(22).integers(0, eng.vocab_size, 10).astype(np.int32)
        assert lib.llama_engine_debug_waits(eng.handle, WAIT_NS, 1) == 0
        eng.forward_batch([int(ids[0])] * 4, [0, 0, 0, 0], [0, 1, 2, 3], True)
        out = (ctypes.c_int32 * 4)()
        assert lib.llama_engine_argmax_batch(eng.handle, out, 4) == -1
        msg = bindings.last_error(eng.handle)
        assert "timed out" in msg, msg
        assert lib.llama_engine_debug_waits(eng.handle, 0, 0) == 0
        # recovered: slot-0 prefill on the batched path, then greedy decode, against the oracle
        ref_toks, ref_logits = _oracle_run(oracle_lib, small_model, ids, 3)
        eng.prefill([int(t) for t in ids[:-1]], 0, False)
        tok, pos = int(ids[-1]), len(ids) - 1
        for s in range(3):
            eng.forward_batch([tok], [pos], [0], True)
            got = eng.argmax_batch(1)[0]
            assert rel_max_err(eng.get_logits_batch(0), ref_logits[s]) <= LOGIT_RTOL
            assert got == ref_toks[s]
            tok, pos = got, pos + 1
    finally:
        eng.close()


def test_prefill_attention_wait_expires_and_engine_recovers(pkg, bindings, small_model, oracle_lib):
    """Expire code 20 makes only the prefill attention kernel's issuing thread wait on a barrier
    phase that nothing completes (after its first K / V tile copies are issued): the kernel drains
    its copies, the next waiting call reports the attention timeout, and after clearing it the
    same engine's prefill matches the oracle again."""
    eng = pkg.LlamaEngine(str(small_model), bindings)
    try:
        if eng.batch_path != "tensor-core":
            pytest.skip("batched path not on the tensor cores: " + bindings.last_error(eng.handle))
        lib = bindings.lib
        ids = np.random.default_rng(23).integers(0, eng.vocab_size, 70).astype(np.int32)
        assert lib.llama_engine_debug_waits(eng.handle, WAIT_NS, 20) == 0
        eng.prefill([int(t) for t in ids], 0, True)  # queued; the failure shows at the next wait
        assert lib.llama_engine_sample(eng.handle, ctypes.c_float(0.0), ctypes.c_float(0.9)) == 0
        msg = bindings.last_error(eng.handle)
        assert "prefill attention" in msg and "timed out" in msg, msg
        assert lib.llama_engine_debug_waits(eng.handle, 0, 0) == 0
        o = oracle_lib.orc_create(str(small_model).encode())
        try:
            oracle_lib.orc_prefill(o, fptr(ids), len(ids), 0, 1)
            ref = np.ctypeslib.as_array(oracle_lib.orc_get_logits(o), shape=(eng.vocab_size,)).copy()
            eng.prefill([int(t) for t in ids], 0, True)
            assert rel_max_err(eng.get_logits(), ref) <= LOGIT_RTOL
            assert eng.sample(0.0, 0.9) == oracle_lib.orc_sample_engine(o, ctypes.c_float(0.0), ctypes.c_float(0.9))
        finally:
            oracle_lib.orc_free(o)
    finally:
        eng.close()
