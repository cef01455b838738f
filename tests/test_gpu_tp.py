"""2-way tensor-parallel batch-1 engine (llama_engine_create_tp) on two GPUs, against the oracle.

Two child processes (one per GPU) share an NCCL unique id made by the parent; both make the same
calls: a token-by-token prefill, decode steps with logits (gathered on both ranks), greedy
samples, and a device-resident greedy generation.  Rank 0's logits are compared with the
oracle's within 1e-3 relative, and the greedy ids of both ranks must equal the oracle's.
Skipped when fewer than two GPUs are visible.
"""
from __future__ import annotations

import ctypes
import multiprocessing as mp

import numpy as np
import pytest

from conftest import ROOT, fptr, load_package

pytestmark = pytest.mark.gpu

LOGIT_RTOL = 1e-3


def _child(rank, uid, model, ids, n_gen, q):
    try:
        import sys
        sys.path.insert(0, str(ROOT / "tests"))
        pkg = load_package()
        b = pkg.LlamaEngineBindings()
        eng = pkg.LlamaEngine(str(model), b, device=rank, tp_rank=rank, tp_world=2, tp_unique_id=uid)
        out = {"path": eng.decode_path, "logits": [], "greedy": []}
        eng.prefill([int(t) for t in ids[:-1]], 0, False)
        tok, pos = int(ids[-1]), len(ids) - 1
        for _ in range(n_gen):
            eng.forward_token(tok, pos, True)
            out["logits"].append(eng.get_logits())
            tok = eng.sample(0.0, 0.9)
            out["greedy"].append(tok)
            pos += 1
        # the device-resident loop from the same start
        eng.prefill([int(t) for t in ids[:-1]], 0, False)
        out["gen"] = eng.generate_greedy(int(ids[-1]), len(ids) - 1, n_gen)
        eng.close()
        q.put((rank, out if rank == 0 else {k: v for k, v in out.items() if k != "logits"}))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, {"error": repr(e)}))


def test_tensor_parallel_2_matches_oracle(pkg, small_model, oracle_lib, gpu_available):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    b = pkg.LlamaEngineBindings()
    uid = pkg.tp_unique_id(b)
    vocab = 4096
    ids = np.random.default_rng(31).integers(0, vocab, 12).astype(np.int32)
    n_gen = 6
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_child, args=(r, uid, str(small_model), ids, n_gen, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            r, out = q.get(timeout=600)
            res[r] = out
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in (0, 1):
        assert "error" not in res[r], res[r]
        assert res[r]["path"] == "tensor-parallel"
    # the oracle's greedy run
    o = oracle_lib.orc_create(str(small_model).encode())
    try:
        pre = np.ascontiguousarray(ids[:-1])
        oracle_lib.orc_prefill(o, fptr(pre), len(pre), 0, 0)
        tok, pos = int(ids[-1]), len(ids) - 1
        for s in range(n_gen):
            oracle_lib.orc_forward_token(o, tok, pos, 1)
            ref = np.ctypeslib.as_array(oracle_lib.orc_get_logits(o), shape=(vocab,)).copy()
            err = float(np.abs(res[0]["logits"][s] - ref).max() / np.abs(ref).max())
            assert err <= LOGIT_RTOL, f"step {s}: {err:.3e}"
            tok = oracle_lib.orc_sample_engine(o, ctypes.c_float(0.0), ctypes.c_float(0.9))
            assert res[0]["greedy"][s] == tok and res[1]["greedy"][s] == tok, f"step {s}"
            pos += 1
    finally:
        oracle_lib.orc_free(o)
    assert res[0]["gen"] == res[0]["greedy"] == res[1]["gen"]
