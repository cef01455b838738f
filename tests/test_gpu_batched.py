"""GPU parity of the token-batched path (tensor-core GEMMs): the isolated GEMM against the oracle
GEMV, batched prefill and batched decode against the oracle engine.

Tolerances:
* GEMM: |y_gpu - y_ref| <= 3e-5 * sum_k |w_nk| |x_k| per output.  The activations enter the
  tensor cores as bf16 hi + lo parts, so each x carries a relative error of at most 2^-17
  (7.6e-6) before fp32 accumulation; the bound leaves room for the accumulation order.
* Logits: max|l_gpu - l_ref| <= 1e-3 * max|l_ref| per step; greedy ids identical.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import fptr

pytestmark = pytest.mark.gpu

LOGIT_RTOL = 1e-3
GEMM_TOL = 3e-5


def rel_max_err(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.fixture(scope="module")
def torch_cuda(gpu_available):
    import torch
    return torch


@pytest.fixture(scope="module")
def bindings(pkg, gpu_available):
    return pkg.LlamaEngineBindings()


def _gemv_ref(oracle_lib, nib, step, mn, N, K, X):
    out = []
    for x in X:
        xs = np.zeros(K // 128, np.float32)
        oracle_lib.orc_block_sums(fptr(x), K, fptr(xs))
        y = np.zeros(N, np.float32)
        oracle_lib.orc_gemv(fptr(nib), fptr(step), fptr(mn), N, K, fptr(x), fptr(xs), fptr(y))
        out.append(y)
    return np.stack(out)


def _dense_ref(pkg, nib, step, mn, N, K, X):
    """X @ W^T in float64 with W = min + q * step dequantised per block, in row chunks of W."""
    q = np.empty((N, K), np.uint8)
    q[:, 0::2] = (nib.reshape(N, K // 2) & 0x0F)
    q[:, 1::2] = (nib.reshape(N, K // 2) >> 4)
    st = pkg.model_file.bf16_to_f32(step).reshape(N, K // 128).astype(np.float64)
    mv = pkg.model_file.bf16_to_f32(mn).reshape(N, K // 128).astype(np.float64)
    X64 = X.astype(np.float64)
    out = np.empty((len(X), N), np.float64)
    for n0 in range(0, N, 4096):
        n1 = min(N, n0 + 4096)
        w = q[n0:n1].reshape(n1 - n0, K // 128, 128) * st[n0:n1, :, None] + mv[n0:n1, :, None]
        out[:, n0:n1] = X64 @ w.reshape(n1 - n0, K).T
    return out


def _abs_scale(pkg, step, mn, N, K, X):
    st = pkg.model_file.bf16_to_f32(step).reshape(N, K // 128).astype(np.float64)
    mv = pkg.model_file.bf16_to_f32(mn).reshape(N, K // 128).astype(np.float64)
    bound = np.abs(mv) + 15.0 * st
    ax = np.abs(X.astype(np.float64)).reshape(len(X), K // 128, 128).sum(axis=2)
    return ax @ bound.T  # [M, N]


@pytest.mark.parametrize("K,N,M", [(2048, 2048, 1), (2048, 2048, 64), (2048, 320, 17), (8192, 2048, 64),
                                   (2048, 512, 100), (8192, 384, 130), (2048, 128256, 64),
                                   (2048, 8192, 1024),  # a prefill chunk through the gate/up shape
                                   # two-tile units: an odd tile count (the last unit's second tile
                                   # repeats its first) and ragged rows over a long K
                                   (2048, 2048, 1050), (8192, 2048, 1100)])
def test_tc_gemm_vs_oracle(pkg, bindings, oracle_lib, torch_cuda, K, N, M):
    torch = torch_cuda
    nib, step, mn = pkg.model_file.gen_matrix(N, K, seed=300 + K + N, tensor=3, uniform_codes=True)
    X = np.random.default_rng(K + 3 * N + M).standard_normal((M, K)).astype(np.float32)
    d_nib = torch.from_numpy(nib).cuda()
    d_step = torch.from_numpy(step.view(np.int16)).cuda()
    d_min = torch.from_numpy(mn.view(np.int16)).cuda()
    d_x = torch.from_numpy(X).cuda()
    d_y = torch.full((M, N), float("nan"), device="cuda")
    # every row of every launch against a float64 dense product (the oracle itself on a few rows)
    dense = _dense_ref(pkg, nib, step, mn, N, K, X)
    scale = _abs_scale(pkg, step, mn, N, K, X)
    rows = np.arange(M) if M <= 8 else np.unique(np.r_[0, 1, 7, 8, M // 2, M - 2, M - 1])
    orc = _gemv_ref(oracle_lib, nib, step, mn, N, K, X[rows])
    first = None
    for launch in range(8):
        d_y.fill_(float("nan"))
        rc = bindings.lib.llama_b128_gemm(d_nib.data_ptr(), d_step.data_ptr(), d_min.data_ptr(), N, K,
                                          d_x.data_ptr(), M, d_y.data_ptr(), None)
        assert rc == 0
        y = d_y.cpu().numpy()
        assert np.isfinite(y).all(), f"launch {launch}"
        err = np.abs(y.astype(np.float64) - dense)
        bad = err > GEMM_TOL * scale
        assert not bad.any(), (f"launch {launch}: {int(bad.sum())} outputs off, rows {np.unique(np.nonzero(bad)[0])[:8]}, "
                               f"max err/scale {float((err / scale).max()):.3e}")
        assert (np.abs(y[rows].astype(np.float64) - orc) <= GEMM_TOL * scale[rows]).all()
        if first is None:
            first = y
        else:
            assert np.array_equal(y, first), f"launch {launch} differs from launch 0"


def test_tc_gemm_rejects_bad_args(bindings, torch_cuda):
    lib = bindings.lib
    assert lib.llama_b128_gemm(None, None, None, 8, 2048, None, 1, None, None) == -1
    buf = torch_cuda.zeros(1 << 20, dtype=torch_cuda.uint8, device="cuda")
    p = buf.data_ptr()
    assert lib.llama_b128_gemm(p, p, p, 8, 1024, p, 1, p, None) == -1    # K not a multiple of 2048
    assert lib.llama_b128_gemm(p, p, p, 8, 2048, p, 0, p, None) == -1    # M < 1
    assert lib.llama_b128_gemm(p, p, p, 8, 2048, p, 4097, p, None) == -1  # M > 4096
    assert lib.llama_b128_gemm(p + 4, p, p, 8, 2048, p, 1, p, None) == -1  # misaligned nibbles


def _oracle_logits(oracle_lib, o, vocab):
    return np.ctypeslib.as_array(oracle_lib.orc_get_logits(o), shape=(vocab,)).copy()


def test_batched_prefill_vs_oracle(pkg, bindings, small_model, oracle_lib, monkeypatch):
    """150 prompt tokens in chunks of 64 (two full chunks and a ragged one), then greedy decode
    on the KV cache the batched path wrote."""
    monkeypatch.setenv("LLAMA_B200_PREFILL_CHUNK", "64")
    eng = pkg.LlamaEngine(str(small_model), bindings)
    o = oracle_lib.orc_create(str(small_model).encode())
    try:
        assert eng.batch_path == "tensor-core"
        vocab = eng.vocab_size
        ids = np.random.default_rng(31).integers(0, vocab, 150).astype(np.int32)
        eng.prefill([int(t) for t in ids], 0, True)
        oracle_lib.orc_prefill(o, fptr(ids), len(ids), 0, 1)
        assert rel_max_err(eng.get_logits(), _oracle_logits(oracle_lib, o, vocab)) <= LOGIT_RTOL
        tok = eng.sample(0.0, 0.9)
        assert tok == oracle_lib.orc_sample_engine(o, ctypes.c_float(0.0), ctypes.c_float(0.9))
        for pos in range(150, 156):
            eng.forward_token(tok, pos, True)
            oracle_lib.orc_forward_token(o, tok, pos, 1)
            assert rel_max_err(eng.get_logits(), _oracle_logits(oracle_lib, o, vocab)) <= LOGIT_RTOL
            tok = eng.sample(0.0, 0.9)
            assert tok == oracle_lib.orc_sample_engine(o, ctypes.c_float(0.0), ctypes.c_float(0.9))
    finally:
        oracle_lib.orc_free(o)
        eng.close()


def test_prefill_without_logits_then_decode(pkg, bindings, small_model, oracle_lib):
    """compute_last_logits = 0, then a single forward_token reads the batched KV."""
    eng = pkg.LlamaEngine(str(small_model), bindings)
    o = oracle_lib.orc_create(str(small_model).encode())
    try:
        vocab = eng.vocab_size
        ids = np.random.default_rng(5).integers(0, vocab, 40).astype(np.int32)
        eng.prefill([int(t) for t in ids[:-1]], 0, False)
        oracle_lib.orc_prefill(o, fptr(ids), len(ids) - 1, 0, 0)
        eng.forward_token(int(ids[-1]), len(ids) - 1, True)
        oracle_lib.orc_forward_token(o, int(ids[-1]), len(ids) - 1, 1)
        assert rel_max_err(eng.get_logits(), _oracle_logits(oracle_lib, o, vocab)) <= LOGIT_RTOL
    finally:
        oracle_lib.orc_free(o)
        eng.close()


def test_batched_decode_40_rows(pkg, bindings, small_model, oracle_lib):
    """40 sequences with different prompt lengths decoded together (MMA N = 48 token columns);
    four of them replayed on the oracle."""
    n = 40
    eng = pkg.LlamaEngine(str(small_model), bindings, device=0, max_batch=n, max_seq_len=256)
    check = [0, 13, 27, 39]
    orcs = {i: oracle_lib.orc_create(str(small_model).encode()) for i in check}
    try:
        assert eng.batch_path == "tensor-core"
        vocab = eng.vocab_size
        rng = np.random.default_rng(77)
        lens = [int(x) for x in rng.integers(3, 30, n)]
        prompts = [rng.integers(0, vocab, L).astype(np.int32) for L in lens]
        slots = list(range(n))
        # all but the last prompt token: batched steps over the slots still in their prompt
        maxlen = max(lens)
        for t in range(maxlen - 1):
            rows = [i for i in range(n) if t < lens[i] - 1]
            eng.forward_batch([int(prompts[i][t]) for i in rows], [t] * len(rows), rows, False)
        for i in check:
            oracle_lib.orc_prefill(orcs[i], fptr(prompts[i]), lens[i] - 1, 0, 0)
        toks = [int(prompts[i][-1]) for i in range(n)]
        pos = [lens[i] - 1 for i in range(n)]
        for step in range(4):
            eng.forward_batch(toks, pos, slots, True)
            am = eng.argmax_batch(n)
            for i in check:
                oracle_lib.orc_forward_token(orcs[i], toks[i], pos[i], 1)
                ref = _oracle_logits(oracle_lib, orcs[i], vocab)
                assert rel_max_err(eng.get_logits_batch(i), ref) <= LOGIT_RTOL, (step, i)
                assert am[i] == int(np.argmax(ref)), (step, i)
            toks = am
            pos = [p + 1 for p in pos]
    finally:
        for o in orcs.values():
            oracle_lib.orc_free(o)
        eng.close()


def test_prefill_chunk_edges(pkg, bindings, small_model, oracle_lib):
    """One sequence prefilled as consecutive chunks whose starts and lengths sit on and off the
    prefill attention's 32-query and 64-key tile edges (single-query chunks, a chunk that ends a
    key tile exactly, chunks starting mid-tile); after every chunk the last position's logits and
    greedy id against the oracle fed the same chunks.  One-token chunks go through forward_token
    (the batch-1 path), so the two paths also read each other's KV rows."""
    eng = pkg.LlamaEngine(str(small_model), bindings)
    o = oracle_lib.orc_create(str(small_model).encode())
    try:
        vocab = eng.vocab_size
        lens = [1, 31, 32, 2, 33, 63, 65, 1, 128]  # starts 0, 1, 32, 64, 66, 99, 162, 227, 228
        ids = np.random.default_rng(61).integers(0, vocab, sum(lens)).astype(np.int32)
        start = 0
        for n in lens:
            chunk = ids[start:start + n]
            eng.prefill([int(t) for t in chunk], start, True)
            oracle_lib.orc_prefill(o, fptr(chunk), n, start, 1)
            ref = _oracle_logits(oracle_lib, o, vocab)
            err = rel_max_err(eng.get_logits(), ref)
            assert err <= LOGIT_RTOL, (start, n, err)
            assert int(np.argmax(eng.get_logits())) == int(np.argmax(ref)), (start, n)
            start += n
    finally:
        oracle_lib.orc_free(o)
        eng.close()


def test_max_context_three_attention_paths(pkg, bindings, small_model):
    """The whole context (8192 positions = max_seq_len): the last position's logits computed by
    three independent attention implementations over the same cache contents.  (a) prefill of
    all 8192 ids in 2048-token chunks (tcgen05 prefill attention, up to 128 key tiles per CTA);
    (b) prefill of the first 8191, then id 8191 through forward_token (the persistent batch-1
    kernel's attention); (c) the same, through forward_batch (batched decode attention split
    over position ranges).  The oracle needs minutes per thousand positions at this length, so
    the paths are checked against each other: logits within 1e-3, same greedy id."""
    eng = pkg.LlamaEngine(str(small_model), bindings)
    try:
        assert eng.batch_path == "tensor-core" and eng.decode_path == "persistent"
        n = 8192
        ids = np.random.default_rng(8192).integers(0, eng.vocab_size, n).astype(np.int32)
        eng.prefill([int(t) for t in ids], 0, True)
        la = eng.get_logits()
        eng.prefill([int(t) for t in ids[:-1]], 0, False)
        eng.forward_token(int(ids[-1]), n - 1, True)
        lb = eng.get_logits()
        eng.forward_batch([int(ids[-1])], [n - 1], [0], True)
        lc = eng.get_logits_batch(0)
        assert rel_max_err(lb, la) <= LOGIT_RTOL, rel_max_err(lb, la)
        assert rel_max_err(lc, la) <= LOGIT_RTOL, rel_max_err(lc, la)
        assert int(np.argmax(la)) == int(np.argmax(lb)) == int(np.argmax(lc))
    finally:
        eng.close()


def test_long_prefill_and_split_attention(pkg, bindings, small_model, oracle_lib, monkeypatch):
    """1040 prompt tokens in two chunks of at most 1024 (query-tiled causal attention, the second
    chunk over 33 key tiles), then two batched decode rows at positions 1040 and 1041: their
    attention is split over position ranges and merged (k_attn_combine)."""
    monkeypatch.setenv("LLAMA_B200_PREFILL_CHUNK", "1024")
    eng = pkg.LlamaEngine(str(small_model), bindings)
    o = oracle_lib.orc_create(str(small_model).encode())
    try:
        vocab = eng.vocab_size
        ids = np.random.default_rng(52).integers(0, vocab, 1040).astype(np.int32)
        eng.prefill([int(t) for t in ids], 0, True)
        oracle_lib.orc_prefill(o, fptr(ids), len(ids), 0, 1)
        assert rel_max_err(eng.get_logits(), _oracle_logits(oracle_lib, o, vocab)) <= LOGIT_RTOL
        tok = eng.sample(0.0, 0.9)
        assert tok == oracle_lib.orc_sample_engine(o, ctypes.c_float(0.0), ctypes.c_float(0.9))
        for pos in (1040, 1041):
            eng.forward_batch([tok], [pos], [0], True)
            oracle_lib.orc_forward_token(o, tok, pos, 1)
            ref = _oracle_logits(oracle_lib, o, vocab)
            assert rel_max_err(eng.get_logits_batch(0), ref) <= LOGIT_RTOL
            tok = eng.argmax_batch(1)[0]
            assert tok == int(np.argmax(ref))
    finally:
        oracle_lib.orc_free(o)
        eng.close()


def test_forward_batch_several_positions_per_slot(pkg, bindings, small_model, oracle_lib):
    """Calls that carry 8 consecutive positions of each of 8 slots (64 rows; later rows read the
    k / v that earlier rows of the same call append), then decode steps with one row per slot
    (k / v appended by the attention kernel itself); two slots replayed on the oracle."""
    n, L, per = 8, 40, 8
    eng = pkg.LlamaEngine(str(small_model), bindings, device=0, max_batch=n, max_seq_len=256)
    check = (0, 5)
    orcs = {i: oracle_lib.orc_create(str(small_model).encode()) for i in check}
    try:
        assert eng.batch_path == "tensor-core"
        vocab = eng.vocab_size
        prompts = np.random.default_rng(123).integers(0, vocab, (n, L)).astype(np.int32)
        for p0 in range(0, L - 1, per):
            ps = list(range(p0, min(L - 1, p0 + per)))
            eng.forward_batch([int(prompts[s, p]) for p in ps for s in range(n)], [p for p in ps for s in range(n)],
                              [s for p in ps for s in range(n)], False)
        for i in check:
            oracle_lib.orc_prefill(orcs[i], fptr(prompts[i]), L - 1, 0, 0)
        toks = [int(t) for t in prompts[:, -1]]
        for step in range(3):
            pos = L - 1 + step
            eng.forward_batch(toks, [pos] * n, list(range(n)), True)
            am = eng.argmax_batch(n)
            for i in check:
                oracle_lib.orc_forward_token(orcs[i], toks[i], pos, 1)
                ref = _oracle_logits(oracle_lib, orcs[i], vocab)
                assert rel_max_err(eng.get_logits_batch(i), ref) <= LOGIT_RTOL, (step, i)
                assert am[i] == int(np.argmax(ref)), (step, i)
            toks = am
    finally:
        for o in orcs.values():
            oracle_lib.orc_free(o)
        eng.close()


def test_forward_batch_rejects_duplicate_rows(pkg, bindings, small_model):
    """Two rows for the same (slot, position) would both append that position's k / v."""
    eng = pkg.LlamaEngine(str(small_model), bindings, device=0, max_batch=4, max_seq_len=64)
    try:
        lib = bindings.lib
        t = (ctypes.c_int32 * 3)(1, 2, 3)
        p = (ctypes.c_int32 * 3)(0, 1, 0)
        sl = (ctypes.c_int32 * 3)(2, 2, 2)
        assert lib.llama_engine_forward_batch(eng.handle, t, p, sl, 3, 0) == -1
        assert "same (slot, position)" in bindings.last_error(eng.handle)
        p2 = (ctypes.c_int32 * 3)(0, 1, 2)
        assert lib.llama_engine_forward_batch(eng.handle, t, p2, sl, 3, 0) == 0
    finally:
        eng.close()
