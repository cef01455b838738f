"""GPU parity: the CUDA engine (through its C ABI) against the oracle and the reference's golden
fixtures.

Tolerances (fp32 accumulate in a different order than the reference's sequential loops):
* GEMV: |y_gpu - y_ref| <= 2e-6 * sum_k |w_nk| |x_k| per output (the sum of absolute products
  bounds the rounding of any summation order).
* Logits: max|l_gpu - l_ref| <= 1e-3 * max|l_ref| per step ("1e-3 relative").
* Greedy ids: identical at every step.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import GOLDEN, fptr

pytestmark = pytest.mark.gpu

LOGIT_RTOL = 1e-3
GEMV_TOL = 2e-6


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


def _abs_scale(pkg, step, mn, N, K, X):
    st = pkg.model_file.bf16_to_f32(step).reshape(N, K // 128).astype(np.float64)
    mv = pkg.model_file.bf16_to_f32(mn).reshape(N, K // 128).astype(np.float64)
    bound = np.abs(mv) + 15.0 * st
    ax = np.abs(X.astype(np.float64)).reshape(len(X), K // 128, 128).sum(axis=2)
    return ax @ bound.T  # [M, N]


@pytest.mark.parametrize("K,N", [(2048, 2048), (2048, 512), (2048, 8192), (8192, 2048), (2048, 128256)])
@pytest.mark.parametrize("M", [1, 4])
def test_gemv_sweep(pkg, bindings, oracle_lib, torch_cuda, K, N, M):
    torch = torch_cuda
    nib, step, mn = pkg.model_file.gen_matrix(N, K, seed=100 + K + N, tensor=3, uniform_codes=True)
    X = np.random.default_rng(K * 7 + N + M).standard_normal((M, K)).astype(np.float32)
    d_nib = torch.from_numpy(nib).cuda()
    d_step = torch.from_numpy(step.view(np.int16)).cuda()
    d_min = torch.from_numpy(mn.view(np.int16)).cuda()
    d_x = torch.from_numpy(X).cuda()
    d_y = torch.full((M, N), float("nan"), device="cuda")
    rc = bindings.lib.llama_b128_gemv(d_nib.data_ptr(), d_step.data_ptr(), d_min.data_ptr(), N, K,
                                      d_x.data_ptr(), M, d_y.data_ptr(), None)
    assert rc == 0
    torch.cuda.synchronize()
    y = d_y.cpu().numpy()
    ref = _gemv_ref(oracle_lib, nib, step, mn, N, K, X)
    scale = _abs_scale(pkg, step, mn, N, K, X)
    err = np.abs(y.astype(np.float64) - ref)
    assert np.isfinite(y).all()
    assert (err <= GEMV_TOL * scale).all(), f"max err/scale {float((err / scale).max()):.3e}"


@pytest.mark.parametrize("K,N,M", [(384, 40, 3), (2048, 1000, 5), (8192, 24, 8), (128, 16, 1), (6144, 2056, 2),
                                   (2048, 4100, 1)])
def test_gemv_ragged(pkg, bindings, oracle_lib, torch_cuda, K, N, M):
    """Shapes off the model's grid: N not a multiple of 16 (the last tile overlaps the previous
    one and stores only its own rows), K blocks that do not divide evenly over the warps of the
    split-K form, one K block, and M > 4 (two launches)."""
    torch = torch_cuda
    nib, step, mn = pkg.model_file.gen_matrix(N, K, seed=7 + K + N, tensor=3, uniform_codes=True)
    X = np.random.default_rng(K + 3 * N + M).standard_normal((M, K)).astype(np.float32)
    d_nib = torch.from_numpy(nib).cuda()
    d_step = torch.from_numpy(step.view(np.int16)).cuda()
    d_min = torch.from_numpy(mn.view(np.int16)).cuda()
    d_x = torch.from_numpy(X).cuda()
    d_y = torch.full((M, N), float("nan"), device="cuda")
    rc = bindings.lib.llama_b128_gemv(d_nib.data_ptr(), d_step.data_ptr(), d_min.data_ptr(), N, K,
                                      d_x.data_ptr(), M, d_y.data_ptr(), None)
    assert rc == 0
    torch.cuda.synchronize()
    y = d_y.cpu().numpy()
    ref = _gemv_ref(oracle_lib, nib, step, mn, N, K, X)
    scale = _abs_scale(pkg, step, mn, N, K, X)
    assert np.isfinite(y).all()
    assert (np.abs(y.astype(np.float64) - ref) <= GEMV_TOL * scale).all()


def test_gemv_rejects_bad_args(bindings, torch_cuda):
    lib = bindings.lib
    assert lib.llama_b128_gemv(None, None, None, 8, 2048, None, 1, None, None) == -1
    buf = torch_cuda.zeros(1 << 20, dtype=torch_cuda.uint8, device="cuda")
    p = buf.data_ptr()
    assert lib.llama_b128_gemv(p, p, p, 8, 100, p, 1, p, None) == -1   # K not a multiple of 128
    assert lib.llama_b128_gemv(p, p, p, 8, 2048, p, 0, p, None) == -1   # M < 1
    assert lib.llama_b128_gemv(p, p, p, 8, 2048, p, 9, p, None) == -1   # M > 8


# ---------------------------------------------------------------------------------------------
# Whole token loop on the small seeded model (live oracle)
# ---------------------------------------------------------------------------------------------

@pytest.fixture(scope="module")
def small_engine(pkg, bindings, small_model):
    eng = pkg.LlamaEngine(str(small_model), bindings)
    yield eng
    eng.close()


def _oracle_logits(oracle_lib, o, vocab):
    return np.ctypeslib.as_array(oracle_lib.orc_get_logits(o), shape=(vocab,)).copy()


def test_small_model_golden(small_engine):
    g = np.load(GOLDEN / "small_greedy.npz")
    eng = small_engine
    assert eng.decode_path == "persistent", eng.bindings.last_error(eng.handle)
    prompt = [int(t) for t in g["prompt"]]
    eng.reset()
    eng.prefill(prompt[:-1], 0, False)
    tok, pos = prompt[-1], len(prompt) - 1
    for s in range(len(g["tokens"])):
        eng.forward_token(tok, pos, True)
        lg = eng.get_logits()
        assert rel_max_err(lg, g["full_logits"][s]) <= LOGIT_RTOL, f"step {s}"
        nx = eng.sample(0.0, 0.9)
        assert nx == int(g["tokens"][s]), f"greedy id differs at step {s} (margin {g['margins'][s]:.3g})"
        tok, pos = nx, pos + 1


def test_small_model_vs_oracle_long(pkg, small_engine, oracle_lib, small_model):
    """Prefill 300 positions then decode: exercises attention over a longer KV prefix."""
    eng = small_engine
    o = oracle_lib.orc_create(str(small_model).encode())
    try:
        vocab = eng.vocab_size
        ids = np.random.default_rng(5).integers(0, vocab, 300).astype(np.int32)
        eng.prefill([int(t) for t in ids], 0, True)
        oracle_lib.orc_prefill(o, fptr(ids), len(ids), 0, 1)
        assert rel_max_err(eng.get_logits(), _oracle_logits(oracle_lib, o, vocab)) <= LOGIT_RTOL
        tok = eng.sample(0.0, 0.9)
        assert tok == oracle_lib.orc_sample_engine(o, ctypes.c_float(0.0), ctypes.c_float(0.9))
        for pos in range(300, 306):
            eng.forward_token(tok, pos, True)
            oracle_lib.orc_forward_token(o, tok, pos, 1)
            assert rel_max_err(eng.get_logits(), _oracle_logits(oracle_lib, o, vocab)) <= LOGIT_RTOL
            tok = eng.sample(0.0, 0.9)
            assert tok == oracle_lib.orc_sample_engine(o, ctypes.c_float(0.0), ctypes.c_float(0.9))
    finally:
        oracle_lib.orc_free(o)


def test_semantics_edge_cases(pkg, small_engine, oracle_lib, small_model):
    eng = small_engine
    o = oracle_lib.orc_create(str(small_model).encode())
    try:
        vocab = eng.vocab_size
        eng.forward_token(5, 0, True)
        oracle_lib.orc_forward_token(o, 5, 0, 1)
        before = eng.get_logits()
        # pos >= 8192: silent no-op (src/llama_engine.cpp:936)
        eng.forward_token(7, 8192, True)
        assert np.array_equal(eng.get_logits(), before)
        # compute_logits = 0 leaves the logits untouched
        eng.forward_token(7, 1, False)
        oracle_lib.orc_forward_token(o, 7, 1, 0)
        assert np.array_equal(eng.get_logits(), before)
        # out-of-range ids are replaced by 0 (:937)
        eng.forward_token(-3, 2, True)
        oracle_lib.orc_forward_token(o, 0, 2, 1)
        assert rel_max_err(eng.get_logits(), _oracle_logits(oracle_lib, o, vocab)) <= LOGIT_RTOL
        eng.forward_token(vocab + 100, 3, True)
        oracle_lib.orc_forward_token(o, 0, 3, 1)
        ref = _oracle_logits(oracle_lib, o, vocab)
        assert rel_max_err(eng.get_logits(), ref) <= LOGIT_RTOL
        # embedding dequantisation is bit-exact
        e_gpu = eng.dequantize_embedding(1234)
        mf = pkg.model_file.ModelFile(small_model)
        e_ref = np.zeros(eng.dim, np.float32)
        lm = mf.lm_head
        oracle_lib.orc_dequant_row(fptr(np.ascontiguousarray(lm["nib"])), fptr(np.ascontiguousarray(lm["step"])),
                                   fptr(np.ascontiguousarray(lm["min"])), lm["K"], 1234, fptr(e_ref))
        assert e_gpu.tobytes() == e_ref.tobytes()
        # temperature sampling rewrites the logits with probabilities, like the reference
        libc = ctypes.CDLL(None)
        libc.srand(99)
        sid = eng.sample(0.8, 0.9)
        probs = eng.get_logits()
        ref_p = ref.copy()
        libc.srand(99)
        rid = oracle_lib.orc_sample(fptr(ref_p), vocab, ctypes.c_float(0.8), ctypes.c_float(0.9))
        assert abs(float(probs.sum()) - 1.0) < 1e-4
        assert np.abs(probs - ref_p).max() <= 1e-3 * ref_p.max()
        assert sid == rid
        # greedy after the in-place rewrite picks the argmax of the probabilities
        assert eng.sample(0.0, 0.9) == int(np.argmax(ref_p))
    finally:
        oracle_lib.orc_free(o)


def test_generate_greedy_equals_loop(pkg, bindings, small_model):
    eng = pkg.LlamaEngine(str(small_model), bindings)
    try:
        prompt = [3, 17, 400, 9, 2000]
        eng.prefill(prompt[:-1], 0, False)
        dev = eng.generate_greedy(prompt[-1], len(prompt) - 1, 16)
        eng.prefill(prompt[:-1], 0, False)
        tok, pos, loop = prompt[-1], len(prompt) - 1, []
        for _ in range(16):
            eng.forward_token(tok, pos, True)
            tok = eng.sample(0.0, 0.9)
            loop.append(tok)
            pos += 1
        assert dev == loop
    finally:
        eng.close()


def test_forward_batch_matches_single(pkg, bindings, small_model, oracle_lib):
    n = 3
    eng = pkg.LlamaEngine(str(small_model), bindings, device=0, max_batch=n, max_seq_len=512)
    orcs = [oracle_lib.orc_create(str(small_model).encode()) for _ in range(n)]
    try:
        vocab = eng.vocab_size
        rng = np.random.default_rng(21)
        lens = [5, 9, 2]
        prompts = [rng.integers(0, vocab, L).astype(np.int32) for L in lens]
        # ragged prefill through the batch API, one row per live sequence
        for t in range(max(lens)):
            rows = [i for i in range(n) if t < lens[i]]
            eng.forward_batch([int(prompts[i][t]) for i in rows], [t] * len(rows), rows, True)
            am = eng.argmax_batch(len(rows))
            for j, i in enumerate(rows):
                oracle_lib.orc_forward_token(orcs[i], int(prompts[i][t]), t, 1)
                ref = _oracle_logits(oracle_lib, orcs[i], vocab)
                assert rel_max_err(eng.get_logits_batch(j), ref) <= LOGIT_RTOL
                assert am[j] == int(np.argmax(ref))
    finally:
        for o in orcs:
            oracle_lib.orc_free(o)
        eng.close()


# ---------------------------------------------------------------------------------------------
# Full LLaMA-3.2-1B shape against the reference's own greedy run
# ---------------------------------------------------------------------------------------------

def test_config0_golden(pkg, bindings, full_model):
    g = np.load(GOLDEN / "config0_greedy.npz")
    assert pkg.model_file.file_sha256(full_model) == str(g["model_sha256"]), "generator output differs"
    eng = pkg.LlamaEngine(str(full_model), bindings)
    assert eng.decode_path == "persistent"
    try:
        prompt = [int(t) for t in g["prompt"]]
        eng.prefill(prompt[:-1], 0, False)
        tok, pos = prompt[-1], len(prompt) - 1
        idx = g["sample_idx"]
        full = {int(s): k for k, s in enumerate(g["full_steps"])}
        mismatches = []
        for s in range(len(g["tokens"])):
            eng.forward_token(tok, pos, True)
            lg = eng.get_logits()
            ref_sampled = g["sampled"][s]
            scale = float(np.abs(g["top_vals"][s]).max())
            assert np.abs(lg[idx] - ref_sampled).max() <= LOGIT_RTOL * scale, f"step {s}"
            assert np.abs(lg[g["top_ids"][s]] - g["top_vals"][s]).max() <= LOGIT_RTOL * scale, f"step {s}"
            if s in full:
                assert rel_max_err(lg, g["full_logits"][full[s]]) <= LOGIT_RTOL, f"step {s}"
            nx = eng.sample(0.0, 0.9)
            if nx != int(g["tokens"][s]):
                mismatches.append((s, float(g["margins"][s])))
                break
            tok, pos = nx, pos + 1
        assert not mismatches, f"greedy id mismatch at (step, top-2 margin) {mismatches}"
    finally:
        eng.close()


def test_kernel_chain_path_vs_oracle(pkg, bindings, chain_model, oracle_lib):
    """Geometries outside the persistent kernel's (here ffn 1024) run the per-phase kernel chain."""
    eng = pkg.LlamaEngine(str(chain_model), bindings)
    o = oracle_lib.orc_create(str(chain_model).encode())
    try:
        assert eng.decode_path == "kernel-chain"
        vocab = eng.vocab_size
        ids = np.random.default_rng(8).integers(0, vocab, 20).astype(np.int32)
        eng.prefill([int(t) for t in ids], 0, True)
        oracle_lib.orc_prefill(o, fptr(ids), len(ids), 0, 1)
        assert rel_max_err(eng.get_logits(), _oracle_logits(oracle_lib, o, vocab)) <= LOGIT_RTOL
        tok = eng.sample(0.0, 0.9)
        assert tok == oracle_lib.orc_sample_engine(o, ctypes.c_float(0.0), ctypes.c_float(0.9))
        for pos in range(20, 24):
            eng.forward_token(tok, pos, True)
            oracle_lib.orc_forward_token(o, tok, pos, 1)
            assert rel_max_err(eng.get_logits(), _oracle_logits(oracle_lib, o, vocab)) <= LOGIT_RTOL
            tok = eng.sample(0.0, 0.9)
            assert tok == oracle_lib.orc_sample_engine(o, ctypes.c_float(0.0), ctypes.c_float(0.9))
    finally:
        oracle_lib.orc_free(o)
        eng.close()


def test_persistent_matches_kernel_chain(pkg, bindings, small_model, monkeypatch):
    """Same model, both decode paths: logits agree within the parity tolerance, ids identical."""
    a = pkg.LlamaEngine(str(small_model), bindings)
    monkeypatch.setenv("LLAMA_B200_PERSISTENT", "0")
    b = pkg.LlamaEngine(str(small_model), bindings)
    try:
        assert a.decode_path == "persistent" and b.decode_path == "kernel-chain"
        prompt = [5, 77, 1000, 4095, 12, 0, 9]
        a.prefill(prompt, 0, True)
        b.prefill(prompt, 0, True)
        assert rel_max_err(a.get_logits(), b.get_logits()) <= LOGIT_RTOL
        ga = a.generate_greedy(a.sample(0.0, 0.9), len(prompt), 12)
        gb = b.generate_greedy(b.sample(0.0, 0.9), len(prompt), 12)
        assert ga == gb
    finally:
        a.close()
        b.close()


def _reference_walk(p, top_p, r_int):
    """sample_top_p's candidate walk and draw (src/llama_engine.cpp:808-838) in float32 over the
    probabilities p, with the libc rand() value r_int."""
    k = min(64, len(p))
    pl = [float(v) for v in p]  # float32 values compare the same as doubles
    vals = pl[:k]
    ids = list(range(k))
    for i in range(k, len(pl)):
        v = pl[i]
        if v > vals[k - 1]:
            q = k - 1
            while q > 0 and v > vals[q - 1]:
                vals[q], ids[q] = vals[q - 1], ids[q - 1]
                q -= 1
            vals[q], ids[q] = v, i
    cum = np.float32(0.0)
    last = 0
    for i in range(k):
        cum = np.float32(cum + np.float32(vals[i]))
        last = i
        if cum >= np.float32(top_p):
            break
    r = np.float32(np.float32(r_int) / np.float32(2147483647)) * cum
    run = np.float32(0.0)
    for i in range(last + 1):
        run = np.float32(run + np.float32(vals[i]))
        if run >= r:
            return ids[i]
    return ids[0]


def test_temperature_sampling_matches_walk(small_engine):
    """The 64 candidates are built on the device and the draw runs on the host: for several
    temperatures, top_p values and rand() seeds the sampled id equals the reference's walk and
    draw restated over the same probabilities (the ones get_logits returns after sampling)."""
    eng = small_engine
    libc = ctypes.CDLL(None)
    libc.rand.restype = ctypes.c_int
    cases = [(0.8, 0.9), (1.3, 0.95), (0.3, 0.5), (2.0, 1.0), (1.0, 0.2)]
    for j, (temp, top_p) in enumerate(cases):
        for seed in (1, 7, 12345):
            eng.forward_token(100 + j, 5, True)
            libc.srand(seed)
            sid = eng.sample(temp, top_p)
            probs = eng.get_logits()
            libc.srand(seed)
            assert sid == _reference_walk(probs, top_p, libc.rand()), (temp, top_p, seed)


def test_temperature_sampling_full_vocab(pkg, bindings, full_model):
    """The device candidate walk over the 1B model's 128,256 probabilities (32 staged tiles)."""
    eng = pkg.LlamaEngine(str(full_model), bindings)
    try:
        libc = ctypes.CDLL(None)
        libc.rand.restype = ctypes.c_int
        for temp, top_p, seed in [(0.8, 0.9, 3), (1.5, 0.99, 11), (0.6, 0.7, 29)]:
            eng.forward_token(1000, 0, True)
            libc.srand(seed)
            sid = eng.sample(temp, top_p)
            probs = eng.get_logits()
            libc.srand(seed)
            assert sid == _reference_walk(probs, top_p, libc.rand()), (temp, top_p, seed)
    finally:
        eng.close()


def test_llama3_rope_scaling_changes_only_the_table(pkg, bindings, small_model, oracle_lib):
    """The opt-in llama3 RoPE scaling replaces the table and nothing else: at position 0 (cos 1,
    sin 0 in both tables) the logits are bit-identical; later positions differ; restoring the
    reference's table gives the oracle's logits again."""
    eng = pkg.LlamaEngine(str(small_model), bindings)
    o = oracle_lib.orc_create(str(small_model).encode())
    try:
        vocab = eng.vocab_size
        ids = [17, 99, 5, 4000, 23]
        eng.forward_token(ids[0], 0, True)
        l0 = eng.get_logits()
        eng.set_rope_scaling(32.0, 1.0, 4.0, 8192)
        eng.forward_token(ids[0], 0, True)
        assert np.array_equal(eng.get_logits(), l0)
        for p, t in enumerate(ids[1:], start=1):
            eng.forward_token(t, p, True)
        scaled = eng.get_logits()
        eng.set_rope_scaling(0.0, 1.0, 4.0, 8192)
        for p, t in enumerate(ids):
            eng.forward_token(t, p, True)
            oracle_lib.orc_forward_token(o, t, p, 1)
        ref = _oracle_logits(oracle_lib, o, vocab)
        assert rel_max_err(eng.get_logits(), ref) <= LOGIT_RTOL
        assert rel_max_err(scaled, ref) > 1e-4  # the scaled table does change the result
        assert eng.bindings.lib.llama_engine_set_rope_scaling(eng.handle, 32.0, 4.0, 1.0, 8192) == -1
    finally:
        oracle_lib.orc_free(o)
        eng.close()
