"""RoPE tables (host code, no GPU): the default table is bit-identical to the reference's
(src/llama_engine.cpp:908-917, through the oracle that is pinned to it), and the opt-in llama3
scaling (models/config.json:26-32 of the reference) matches the Hugging Face llama3 rotary
frequencies (transformers' llama3 rope-init function)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

N_POS = 8192


def _table(lib, factor, low=1.0, high=4.0, orig=8192, n=N_POS):
    c = np.zeros((n, 32), np.float32)
    s = np.zeros((n, 32), np.float32)
    fp = ctypes.POINTER(ctypes.c_float)
    rc = lib.llama_engine_rope_table(factor, low, high, orig, n, c.ctypes.data_as(fp), s.ctypes.data_as(fp))
    assert rc == 0
    return c, s


@pytest.fixture(scope="module")
def lib(pkg):
    return pkg.LlamaEngineBindings().lib


def test_default_table_is_the_references(lib, oracle_lib, small_model):
    c, s = _table(lib, 0.0)
    o = oracle_lib.orc_create(str(small_model).encode())
    try:
        oc = np.ctypeslib.as_array(oracle_lib.orc_get_rope(o, 0), shape=(N_POS * 32,)).reshape(N_POS, 32)
        osn = np.ctypeslib.as_array(oracle_lib.orc_get_rope(o, 1), shape=(N_POS * 32,)).reshape(N_POS, 32)
        assert np.array_equal(c.view(np.uint32), oc.view(np.uint32))
        assert np.array_equal(s.view(np.uint32), osn.view(np.uint32))
    finally:
        oracle_lib.orc_free(o)


def _hf_llama3_inv_freq():
    from transformers import LlamaConfig
    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS
    cfg = LlamaConfig(hidden_size=2048, num_attention_heads=32, num_key_value_heads=8, head_dim=64,
                      max_position_embeddings=131072,
                      rope_parameters={"rope_type": "llama3", "rope_theta": 500000.0, "factor": 32.0,
                                       "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                                       "original_max_position_embeddings": 8192})
    inv, _ = ROPE_INIT_FUNCTIONS["llama3"](cfg, "cpu")
    return inv.numpy().astype(np.float64)


def test_llama3_scaled_table_matches_hugging_face(lib):
    pytest.importorskip("transformers")
    c, s = _table(lib, 32.0)
    theta = np.arctan2(s[1].astype(np.float64), c[1].astype(np.float64))  # pos 1: the frequencies
    hf = _hf_llama3_inv_freq()
    assert np.allclose(theta, hf, rtol=3e-7, atol=0), np.abs(theta / hf - 1).max()
    # the scaling actually bites: low frequencies stretched by 32, high ones kept
    base = 500000.0 ** (-np.arange(32) * 2 / 64)
    assert np.isclose(theta[-1], base[-1] / 32, rtol=1e-6) and np.isclose(theta[0], base[0], rtol=1e-7)
    # every entry is cos / sin of pos x theta: against float64 with the Hugging Face frequencies,
    # the error is bounded by the argument's float32 roundings (theta within a couple of ulps,
    # the product within one) plus one ulp of the result
    pos = np.arange(N_POS, dtype=np.float64)[:, None]
    arg = pos * hf[None, :]
    tol = np.abs(arg) * 2.0 ** -21 + 2e-7
    assert (np.abs(c - np.cos(arg)) <= tol).all()
    assert (np.abs(s - np.sin(arg)) <= tol).all()


def test_rope_table_rejects_bad_arguments(lib):
    c = np.zeros((4, 32), np.float32)
    fp = ctypes.POINTER(ctypes.c_float)
    p = c.ctypes.data_as(fp)
    assert lib.llama_engine_rope_table(32.0, 4.0, 1.0, 8192, 4, p, p) == -1   # high <= low
    assert lib.llama_engine_rope_table(0.0, 1.0, 4.0, 8192, 0, p, p) == -1    # n_pos < 1
    assert lib.llama_engine_rope_table(0.0, 1.0, 4.0, 8192, 8193, p, p) == -1
    assert lib.llama_engine_rope_table(0.0, 1.0, 4.0, 8192, 4, None, p) == -1
