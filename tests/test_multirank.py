"""Multi-rank plumbing of bench.py on CPU: two gloo ranks, as torchrun launches one process per GPU.

With N GPUs every rank decodes its own sequences (data-parallel replicas, no collective on the
data path).  The only collectives are the timing barrier and the max over ranks, which every
rank calls at the same points; these tests run those helpers on world size 2.
"""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, queue):
    import datetime

    import numpy as np
    import torch.distributed as dist

    sys.path.insert(0, str(ROOT))
    import bench

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        # rank r's "timings": the reduced values are the slowest rank's
        got = bench.max_over_ranks([1.0 + rank, 10.0 - rank, 5.0], world, device="cpu")
        dist.barrier()
        seed = bench.rank_seed(1000, rank)
        prompt = np.random.default_rng(seed).integers(0, 128256, bench.PROMPT_LEN).tolist()
        queue.put((rank, got, seed, prompt))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_and_rank_sequences_gloo():
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in procs:
            rank, got, seed, prompt = queue.get(timeout=120)
            out[rank] = (got, seed, prompt)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    assert out[0][0] == out[1][0] == [2.0, 10.0, 5.0]  # element-wise max over the two ranks
    assert out[0][1] != out[1][1]  # each rank has its own sequences
    assert out[0][2] != out[1][2]


def test_single_rank_needs_no_process_group():
    sys.path.insert(0, str(ROOT))
    import bench

    assert bench.max_over_ranks([3, 4.5], 1) == [3.0, 4.5]
    assert bench.rank_seed(4000, 0) == 4000

