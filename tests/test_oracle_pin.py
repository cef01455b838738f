"""Pins the oracle: the C restatement (oracle/oracle.c) must reproduce the reference itself,
compiled from its own source (oracle/_ref), bit for bit — kernels on isolated inputs and the
whole token loop on a seeded model.  CPU only."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import fptr


def _mat(pkg, N, K, seed, uniform=True):
    return pkg.model_file.gen_matrix(N, K, seed=seed, tensor=1, uniform_codes=uniform)


@pytest.mark.parametrize("N,K,uniform", [(512, 2048, True), (256, 8192, True), (1024, 2048, False), (4, 128, True)])
def test_gemv_bitexact(pkg, oracle_lib, ref_kernels, N, K, uniform):
    nib, step, mn = _mat(pkg, N, K, seed=N + K, uniform=uniform)
    x = np.random.default_rng(1).standard_normal(K).astype(np.float32)
    xs_o = np.zeros(K // 128, np.float32)
    xs_r = np.zeros(K // 128, np.float32)
    oracle_lib.orc_block_sums(fptr(x), K, fptr(xs_o))
    ref_kernels.ref_block_sums(fptr(x), K, fptr(xs_r))
    assert xs_o.tobytes() == xs_r.tobytes()
    y_o = np.zeros(N, np.float32)
    y_r = np.zeros(N, np.float32)
    oracle_lib.orc_gemv(fptr(nib), fptr(step), fptr(mn), N, K, fptr(x), fptr(xs_o), fptr(y_o))
    ref_kernels.ref_gemv(fptr(nib), fptr(step), fptr(mn), N, K, fptr(x), fptr(xs_r), fptr(y_r))
    assert y_o.tobytes() == y_r.tobytes()
    # and the restatement is the dense product to fp32 accuracy
    W = pkg.model_file.dequantize({"N": N, "K": K, "nib": nib, "step": step, "min": mn})
    dense = W.astype(np.float64) @ x.astype(np.float64)
    scale = np.abs(W).astype(np.float64) @ np.abs(x).astype(np.float64)
    assert np.all(np.abs(y_o - dense) <= 1e-5 * scale + 1e-30)


def test_swiglu_bitexact(pkg, oracle_lib, ref_kernels):
    N, K = 512, 2048
    g = _mat(pkg, N, K, seed=3, uniform=False)
    u = _mat(pkg, N, K, seed=4, uniform=False)
    x = np.random.default_rng(2).standard_normal(K).astype(np.float32)
    xs = np.zeros(K // 128, np.float32)
    oracle_lib.orc_block_sums(fptr(x), K, fptr(xs))
    a_o = np.zeros(N, np.float32)
    a_r = np.zeros(N, np.float32)
    args = [fptr(g[0]), fptr(g[1]), fptr(g[2]), fptr(u[0]), fptr(u[1]), fptr(u[2]), N, K, fptr(x), fptr(xs)]
    oracle_lib.orc_swiglu(*args, fptr(a_o))
    ref_kernels.ref_swiglu(*args, fptr(a_r))
    assert a_o.tobytes() == a_r.tobytes()


def test_norm_rope_dequant_bitexact(pkg, oracle_lib, ref_kernels):
    rng = np.random.default_rng(3)
    x = rng.standard_normal(2048).astype(np.float32)
    w = rng.uniform(0.5, 1.5, 2048).astype(np.float32)
    o1 = np.zeros(2048, np.float32)
    o2 = np.zeros(2048, np.float32)
    oracle_lib.orc_rms_norm(fptr(x), fptr(w), fptr(o1), 2048)
    ref_kernels.ref_rms_norm(fptr(x), fptr(w), fptr(o2), 2048)
    assert o1.tobytes() == o2.tobytes()

    cos = rng.uniform(-1, 1, 8192 * 32).astype(np.float32)
    sin = rng.uniform(-1, 1, 8192 * 32).astype(np.float32)
    v1 = rng.standard_normal(32 * 64).astype(np.float32)
    v2 = v1.copy()
    oracle_lib.orc_apply_rope(fptr(v1), 32, 64, 77, fptr(cos), fptr(sin))
    ref_kernels.ref_apply_rope(fptr(v2), 32, 64, 77, fptr(cos), fptr(sin))
    assert v1.tobytes() == v2.tobytes()

    nib, step, mn = _mat(pkg, 64, 2048, seed=5, uniform=False)
    e1 = np.zeros(2048, np.float32)
    e2 = np.zeros(2048, np.float32)
    oracle_lib.orc_dequant_row(fptr(nib), fptr(step), fptr(mn), 2048, 37, fptr(e1))
    ref_kernels.ref_dequant_row(fptr(nib), fptr(step), fptr(mn), 64, 2048, 37, fptr(e2))
    assert e1.tobytes() == e2.tobytes()


def test_sampler_bitexact(oracle_lib, ref_kernels):
    libc = ctypes.CDLL(None)
    rng = np.random.default_rng(4)
    for trial in range(6):
        logits = (rng.standard_normal(5000) * 3).astype(np.float32)
        if trial == 1:
            logits[100] = logits[200] = logits.max() + 1.0  # tie: first index wins
        for temp, top_p in [(0.0, 0.9), (0.7, 0.9), (1.3, 0.5), (0.005, 0.9)]:
            a, b = logits.copy(), logits.copy()
            libc.srand(1234 + trial)
            ia = oracle_lib.orc_sample(fptr(a), a.size, ctypes.c_float(temp), ctypes.c_float(top_p))
            libc.srand(1234 + trial)
            ib = ref_kernels.ref_sample(fptr(b), b.size, ctypes.c_float(temp), ctypes.c_float(top_p))
            assert ia == ib
            assert a.tobytes() == b.tobytes()  # in-place probability overwrite matches too


def test_token_loop_bitexact(pkg, oracle_lib, ref_engine, small_model):
    """The restated engine and the reference engine agree bit for bit on logits, greedy ids and
    KV-dependent state over prefill + decode on a seeded model (dim 2048, 32/8 heads)."""
    o = oracle_lib.orc_create(str(small_model).encode())
    r = ref_engine.llama_engine_create(str(small_model).encode())
    assert o and r
    try:
        vocab = ref_engine.llama_engine_get_vocab_size(r)
        prompt = np.random.default_rng(11).integers(0, vocab, 9).astype(np.int32)
        oracle_lib.orc_prefill(o, fptr(prompt), 8, 0, 0)
        ref_engine.llama_engine_prefill(r, prompt.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), 8, 0, 0)
        tok = int(prompt[8])
        for pos in range(8, 14):
            oracle_lib.orc_forward_token(o, tok, pos, 1)
            ref_engine.llama_engine_forward_token(r, tok, pos, 1)
            lo = np.ctypeslib.as_array(oracle_lib.orc_get_logits(o), shape=(vocab,)).copy()
            lr = np.ctypeslib.as_array(ref_engine.llama_engine_get_logits(r), shape=(vocab,)).copy()
            assert lo.tobytes() == lr.tobytes(), f"logits differ at pos {pos}"
            to = oracle_lib.orc_sample_engine(o, ctypes.c_float(0.0), ctypes.c_float(0.9))
            tr = ref_engine.llama_engine_sample(r, ctypes.c_float(0.0), ctypes.c_float(0.9))
            assert to == tr
            tok = to
        # the reference's silent no-op and token clamp
        oracle_lib.orc_forward_token(o, -5, 8192, 1)
        ref_engine.llama_engine_forward_token(r, -5, 8192, 1)
        oracle_lib.orc_forward_token(o, vocab + 10, 14, 1)
        ref_engine.llama_engine_forward_token(r, vocab + 10, 14, 1)
        lo = np.ctypeslib.as_array(oracle_lib.orc_get_logits(o), shape=(vocab,))
        lr = np.ctypeslib.as_array(ref_engine.llama_engine_get_logits(r), shape=(vocab,))
        assert lo.tobytes() == lr.tobytes()
    finally:
        oracle_lib.orc_free(o)
        ref_engine.llama_engine_free(r)
