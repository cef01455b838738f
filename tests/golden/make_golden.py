"""Generates the golden fixtures in this directory by running the REFERENCE engine itself
(compiled from its own source by oracle/Makefile) on seeded model files.

    python tests/golden/make_golden.py            # both fixtures
    python tests/golden/make_golden.py small      # only the small-model fixture
    python tests/golden/make_golden.py config3 config2 --procs 8   # the large-config fixtures

Fixtures:
* ``small_greedy.npz`` — 2-layer model (dim 2048, 32/8 heads, ffn 2048, vocab 4096, seed 7,
  random norm weights), 9-token prompt, prefill 8 + 24 greedy steps: ids, top-2 margins and full
  logits of every step.
* ``config0_greedy.npz`` — the LLaMA-3.2-1B shape (16 layers, dim 2048, ffn 8192, vocab 128256),
  weights N(0, 0.02) seed 0, norms 1.0; prompt = 32 ids from numpy default_rng(0) in [0, 128256);
  prefill(ids[:31]) then 128 x (forward_token(prev, pos, 1) + greedy sample) at pos 31..158.
  Stores the 128 ids, the top-2 margin per step, full logits of step 0 and of the last step,
  the top-16 (id, value) per step and the logits at 256 fixed indices per step.

* ``config3_prefill.npz`` — prefill on the 1B shape (same model file as config0): 8 prompts of
  2048 ids from numpy default_rng(3) in [0, 128256); the reference runs
  ``prefill(ids, 2048, 0, 1)`` (a loop of forward_token, src/llama_engine.cpp:1118-1127).  Stores
  the full last-position logits, the greedy id and the top-2 margin of each prompt.
* ``config2_decode.npz`` — batched decode on the 1B shape: 64 prompts of 512 ids from numpy
  default_rng(2); per sequence ``prefill(ids[:511], 0, 0)`` then 32 x (forward_token(prev, pos, 1)
  + greedy sample) at pos 511..542.  Stores the 32 ids per sequence (a GPU test feeds these ids
  back, so a near-tie cannot derail the comparison), the top-2 margins, the top-16 (id, value) per
  step and the logits at 128 fixed indices per step.

``config3`` and ``config2`` take ~30 and ~60 minutes on 8 host cores (one reference process per
core; ``--procs N`` to change).

Each fixture records the sha256 of the model file it was made from, so a test can tell a
generator difference from an engine difference.
"""
from __future__ import annotations

import ctypes
import importlib.util
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402


def _pkg():
    name = "llama3_signed_4bit_b200"
    if name in sys.modules:
        return sys.modules[name]
    d = ROOT / "llama3-signed-4bit_b200"
    spec = importlib.util.spec_from_file_location(name, d / "__init__.py", submodule_search_locations=[str(d)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def run_reference(model_path: Path, prompt: np.ndarray, n_gen: int, full_logit_steps, sample_idx):
    lib = oracle.load_ref_engine()
    h = lib.llama_engine_create(str(model_path).encode())
    assert h, "reference failed to load the model"
    vocab = lib.llama_engine_get_vocab_size(h)
    ids = prompt.astype(np.int32)
    i32p = ctypes.POINTER(ctypes.c_int32)
    lib.llama_engine_prefill(h, ids.ctypes.data_as(i32p), len(ids) - 1, 0, 0)
    tok, pos = int(ids[-1]), len(ids) - 1
    tokens, margins, top_ids, top_vals, sampled, full = [], [], [], [], [], {}
    for s in range(n_gen):
        lib.llama_engine_forward_token(h, tok, pos, 1)
        lg = np.ctypeslib.as_array(lib.llama_engine_get_logits(h), shape=(vocab,)).copy()
        nx = lib.llama_engine_sample(h, ctypes.c_float(0.0), ctypes.c_float(0.9))
        order = np.argsort(-lg, kind="stable")
        margins.append(float(lg[order[0]] - lg[order[1]]))
        top_ids.append(order[:16].astype(np.int32))
        top_vals.append(lg[order[:16]])
        sampled.append(lg[sample_idx])
        if s in full_logit_steps:
            full[s] = lg
        tokens.append(nx)
        tok, pos = nx, pos + 1
    lib.llama_engine_free(h)
    return dict(tokens=np.array(tokens, np.int32), margins=np.array(margins, np.float32),
                top_ids=np.stack(top_ids), top_vals=np.stack(top_vals), sampled=np.stack(sampled),
                full_steps=np.array(sorted(full), np.int32),
                full_logits=(np.stack([full[k] for k in sorted(full)]) if full
                             else np.zeros((0, vocab), np.float32)))


def make_small(cache: Path):
    pkg = _pkg()
    shape = pkg.model_file.ModelShape(layers=2, dim=2048, ffn=2048, vocab=4096, heads=32, kv_heads=8)
    model = pkg.model_file.cached_model(cache, shape, seed=7, sigma=0.02, random_norms=True)
    prompt = np.random.default_rng(11).integers(0, shape.vocab, 9).astype(np.int32)
    n_gen = 24
    idx = np.arange(0, shape.vocab, 16, dtype=np.int64)
    r = run_reference(model, prompt, n_gen, set(range(n_gen)), idx)
    np.savez_compressed(HERE / "small_greedy.npz", prompt=prompt, sample_idx=idx,
                        model_sha256=pkg.model_file.file_sha256(model), **r)


def make_config0(cache: Path):
    pkg = _pkg()
    shape = pkg.model_file.LLAMA_3_2_1B
    model = pkg.model_file.cached_model(cache, shape, seed=0, sigma=0.02)
    prompt = np.random.default_rng(0).integers(0, shape.vocab, 32).astype(np.int32)
    n_gen = 128
    idx = np.random.default_rng(1).choice(shape.vocab, 256, replace=False).astype(np.int64)
    t0 = time.time()
    r = run_reference(model, prompt, n_gen, {0, n_gen - 1}, idx)
    print(f"config0 reference run: {time.time() - t0:.1f} s", flush=True)
    np.savez_compressed(HERE / "config0_greedy.npz", prompt=prompt, sample_idx=idx,
                        model_sha256=pkg.model_file.file_sha256(model), **r)


def _config3_worker(args):
    model_path, prompt = args
    lib = oracle.load_ref_engine()
    h = lib.llama_engine_create(str(model_path).encode())
    assert h, "reference failed to load the model"
    vocab = lib.llama_engine_get_vocab_size(h)
    ids = prompt.astype(np.int32)
    i32p = ctypes.POINTER(ctypes.c_int32)
    rc = lib.llama_engine_prefill(h, ids.ctypes.data_as(i32p), len(ids), 0, 1)
    assert rc == 0
    lg = np.ctypeslib.as_array(lib.llama_engine_get_logits(h), shape=(vocab,)).copy()
    nx = lib.llama_engine_sample(h, ctypes.c_float(0.0), ctypes.c_float(0.9))
    lib.llama_engine_free(h)
    order = np.argsort(-lg, kind="stable")
    return lg, int(nx), float(lg[order[0]] - lg[order[1]])


def _config2_worker(args):
    model_path, prompt, n_gen, idx = args
    return run_reference(model_path, prompt, n_gen, set(), idx)


def _pool(procs):
    import multiprocessing as mp
    return mp.get_context("spawn").Pool(procs)


def make_config3(cache: Path, procs: int):
    pkg = _pkg()
    shape = pkg.model_file.LLAMA_3_2_1B
    model = pkg.model_file.cached_model(cache, shape, seed=0, sigma=0.02)
    prompts = np.random.default_rng(3).integers(0, shape.vocab, (8, 2048)).astype(np.int32)
    t0 = time.time()
    with _pool(procs) as pool:
        res = pool.map(_config3_worker, [(model, p) for p in prompts], chunksize=1)
    print(f"config3 reference run: {time.time() - t0:.1f} s", flush=True)
    np.savez_compressed(HERE / "config3_prefill.npz", prompts=prompts,
                        logits=np.stack([r[0] for r in res]).astype(np.float32),
                        tokens=np.array([r[1] for r in res], np.int32),
                        margins=np.array([r[2] for r in res], np.float32),
                        model_sha256=pkg.model_file.file_sha256(model))


def make_config2(cache: Path, procs: int):
    pkg = _pkg()
    shape = pkg.model_file.LLAMA_3_2_1B
    model = pkg.model_file.cached_model(cache, shape, seed=0, sigma=0.02)
    prompts = np.random.default_rng(2).integers(0, shape.vocab, (64, 512)).astype(np.int32)
    idx = np.random.default_rng(4).choice(shape.vocab, 128, replace=False).astype(np.int64)
    n_gen = 32
    t0 = time.time()
    with _pool(procs) as pool:
        res = pool.map(_config2_worker, [(model, p, n_gen, idx) for p in prompts], chunksize=1)
    print(f"config2 reference run: {time.time() - t0:.1f} s", flush=True)
    np.savez_compressed(HERE / "config2_decode.npz", prompts=prompts, sample_idx=idx,
                        tokens=np.stack([r["tokens"] for r in res]),
                        margins=np.stack([r["margins"] for r in res]),
                        top_ids=np.stack([r["top_ids"] for r in res]),
                        top_vals=np.stack([r["top_vals"] for r in res]),
                        sampled=np.stack([r["sampled"] for r in res]),
                        model_sha256=pkg.model_file.file_sha256(model))


if __name__ == "__main__":
    oracle.build()
    assert oracle.have_reference(), "the reference build is needed to make golden fixtures"
    cache = Path(tempfile.gettempdir()) / "llama3_b200_cache"
    args = sys.argv[1:]
    procs = 8
    if "--procs" in args:
        i = args.index("--procs")
        procs = int(args[i + 1])
        del args[i:i + 2]
    which = args or ["small", "config0"]
    if "small" in which:
        make_small(cache)
    if "config0" in which:
        make_config0(cache)
    if "config3" in which:
        make_config3(cache, procs)
    if "config2" in which:
        make_config2(cache, procs)
