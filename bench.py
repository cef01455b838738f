#!/usr/bin/env python3
"""Benchmark of the block-128 4-bit LLaMA token loop on B200.

Workload (one "step" = one greedy decode token of one sequence per GPU): the LLaMA-3.2-1B shape
(16 layers, dim 2048, ffn 8192, vocab 128256, 32/8 heads) with seeded random-init weights
quantised to the LLM4S128 block-128 4-bit format; a 32-token prompt is prefilled, then the
128-token greedy generation at positions 31..158 is repeated until K steps are timed.  Every
step streams all 657 MB of weights, far more than the 126 MB L2, so no flush is needed between
steps.  With N GPUs every rank decodes its own sequence (independent replicas, weak scaling).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

The same line carries ``batch64`` (64 sequences decoded from position 511, and 8 x 2048-id
prefills; rank 0 of a 1-GPU run) and ``box256`` (256 sequences per GPU with KV for 4096 positions,
greedy steps timed near position 1023 and near 4095; every rank, weak scaling) and
``gemv_sweep`` (the isolated block-128 GEMV at the model's five K x N shapes, M = 1 and 4).

Prints one JSON line on rank 0.  ``value`` is device-resident throughput (CUDA events around K
graph steps fed by the on-device argmax), ``e2e`` is the same loop through the reference C ABI
(forward_token + sample per step from the host).  ``--impl reference`` times the reference
engine itself (compiled from its own source) on the host cores.
"""
from __future__ import annotations

import argparse
import ctypes
import importlib.util
import json
import math
import multiprocessing as mp
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG_DIR = ROOT / "llama3-signed-4bit_b200"
METRIC = "decode tok/s (1B, 4-bit b128) at batch 1 and 64; GEMV HBM GB/s vs peak"
PROMPT_LEN = 32
GEN_LEN = 128
FALLBACK_HBM_GBS = 6650.0


def load_package():
    name = "llama3_signed_4bit_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def cache_dir() -> Path:
    d = Path(os.environ.get("LLAMA_B200_CACHE", Path(tempfile.gettempdir()) / "llama3_b200_cache"))
    d.mkdir(parents=True, exist_ok=True)
    return d


def hbm_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        v = float(json.loads(p.read_text())["hbm_gbs"])
        return v, "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


# ---------------------------------------------------------------------------------------------
# algorithmic bytes (weights + activations + KV actually required by the math)
# ---------------------------------------------------------------------------------------------
def phase_bytes(shape, pos: int) -> dict:
    d, f, kv, v = shape.dim, shape.ffn, shape.kv_dim, shape.vocab
    mat = lambda n, k: n * (k // 128) * 68  # noqa: E731
    return {
        "qkv": mat(d + 2 * kv, d) + 4 * (3 * d + d + 2 * kv),          # W, x + norm, out
        "attn": 2 * 4 * kv * (pos + 1) + 4 * (d + 2 * kv + d),          # K/V rows, q/k/v in, out
        "oproj": mat(d, d) + 4 * (d + 2 * d),                           # W, attn in, x rw
        "gateup": 2 * mat(f, d) + 4 * (2 * d + f),                       # Wg+Wu, x + norm, act
        "down": mat(d, f) + 4 * (f + 2 * d),                            # W, act, x rw
        "lmhead": mat(v, d) + 4 * (2 * d + v),                           # W, x + norm, logits
    }


# ---------------------------------------------------------------------------------------------
# multi-GPU plumbing: one process per GPU, independent sequences (no collective on the data path)
# ---------------------------------------------------------------------------------------------
def max_over_ranks(values, world: int, device="cuda"):
    """Element-wise max of a list of timings over the ranks: every multi-GPU number is timed as
    the slowest rank's.  Every rank must call it at the same point."""
    vals = [float(v) for v in values]
    if world <= 1:
        return vals
    import torch
    import torch.distributed as dist

    t = torch.tensor(vals, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t.tolist()]


def rank_seed(base: int, rank: int) -> int:
    """Seed of a rank's synthetic sequences: each rank decodes its own (weak scaling)."""
    return base + rank


def bytes_per_tok_ref(shape, start: int) -> float:
    """Mean algorithmic bytes per token of a GEN_LEN-token launch from `start` (the launch that
    profiles/traffic_per_launch.txt scales its DRAM capture to)."""
    return sum(token_bytes(shape, p) for p in range(start, start + GEN_LEN)) / GEN_LEN


def token_bytes(shape, pos: int) -> int:
    """Weights + norms + KV read (pos+1 rows incl. the new one) + KV write, per token."""
    kv_row = shape.layers * shape.kv_dim * 4 * 2
    return shape.weight_bytes() + kv_row * (pos + 1) + kv_row


# ---------------------------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = set(gpus)
        self.proc = None
        self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "50"], stdout=self.out, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        # wait (up to 5 s) until the sampler has written its first row, so that a short timed
        # region is still covered
        t0 = time.time()
        while self.proc is not None and time.time() - t0 < 5.0:
            self.out.flush()
            if Path(self.out.name).stat().st_size > 0:
                break
            time.sleep(0.02)
        return self

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.12)  # at least one more sample after the timed region
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        self.out.flush()
        rows = []
        for line in Path(self.out.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                if int(parts[0]) in self.gpus:
                    rows.append(parts)
            except ValueError:
                pass
        os.unlink(self.out.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------------------------
# reference / oracle on the host (CPU baseline)
# ---------------------------------------------------------------------------------------------
def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------------
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    pkg = load_package()
    shape = pkg.model_file.ModelShape(layers=args.layers)
    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", init_method="env://", timeout=__import__("datetime").timedelta(seconds=300))
    if rank == 0:
        pkg.build.build_all()
        model = pkg.model_file.cached_model(cache_dir(), shape, seed=0, sigma=0.02)
    if world > 1:
        dist.barrier()
    if rank != 0:
        model = pkg.model_file.cached_model(cache_dir(), shape, seed=0, sigma=0.02)
    import numpy as np

    bindings = pkg.LlamaEngineBindings()
    eng = pkg.LlamaEngine(str(model), bindings, device=local_rank, max_batch=1, max_seq_len=0)
    lib = bindings.lib
    stream = torch.cuda.ExternalStream(lib.llama_engine_get_stream(eng.handle))
    prompt = np.random.default_rng(rank_seed(1000, rank)).integers(0, shape.vocab, PROMPT_LEN).astype(np.int32)
    eng.prefill([int(t) for t in prompt[:-1]], 0, False)
    first, start = int(prompt[-1]), PROMPT_LEN - 1

    def device_steps(n):
        """n greedy steps in chunks of the 128-token generation (positions 31..158)."""
        done = 0
        while done < n:
            c = min(GEN_LEN, n - done)
            eng.generate_greedy(first, start, c)
            done += c

    # clocks: rank 0 samples every GPU of the job (nvidia-smi indices) from the warm-up through
    # the timed region (the sampler starts before the warm-up, so a short region is covered)
    import contextlib
    clk = ClockSampler(range(world) if world > 1 else [local_rank]) if rank == 0 else None
    with (clk if clk is not None else contextlib.nullcontext()):
        device_steps(args.warmup)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        ev0.record(stream)
        device_steps(args.steps)
        ev1.record(stream)
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    clocks = clk.summary() if clk is not None else None
    ms = max_over_ranks([ms], world)[0]
    value = world * args.steps / (ms / 1e3)

    # e2e through the reference ABI: forward_token + sample(0) per step, from the host
    def host_steps(n):
        done = 0
        while done < n:
            tok, pos = first, start
            for _ in range(min(GEN_LEN, n - done)):
                lib.llama_engine_forward_token(eng.handle, tok, pos, 1)
                tok = lib.llama_engine_sample(eng.handle, ctypes.c_float(0.0), ctypes.c_float(0.9))
                pos += 1
                done += 1

    host_steps(min(args.warmup, GEN_LEN))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    w0 = time.perf_counter()
    host_steps(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - w0
    e2e_ms = e0.elapsed_time(e1)
    e2e_ms, wall_ms = max_over_ranks([e2e_ms, wall * 1e3], world)
    wall = wall_ms / 1e3
    e2e_value = world * args.steps / max(e2e_ms / 1e3, wall)

    # roofline of the dominant kernel, over the positions actually timed: device_steps runs
    # generations of up to GEN_LEN tokens, each from position `start`
    peak, peak_kind = hbm_peak()
    chunks = [min(GEN_LEN, args.steps - d) for d in range(0, args.steps, GEN_LEN)]
    timed_bytes = sum(token_bytes(shape, start + i) for c in chunks for i in range(c))
    bytes_tok = timed_bytes / args.steps
    avg_pos = start + sum(c * (c - 1) / 2.0 for c in chunks) / args.steps
    persistent = eng.decode_path == "persistent"
    pb = phase_bytes(shape, int(avg_pos))
    launches = {"qkv": shape.layers, "attn": shape.layers, "oproj": shape.layers, "gateup": shape.layers,
                "down": shape.layers, "lmhead": 1}
    phase_ms = {}
    for ph in launches:
        out = ctypes.c_float(0.0)
        iters = 64 if ph != "lmhead" else 16
        lib.llama_engine_profile_phase(eng.handle, ph.encode(), 4, ctypes.byref(out))
        rc = lib.llama_engine_profile_phase(eng.handle, ph.encode(), iters, ctypes.byref(out))
        phase_ms[ph] = float(out.value) if rc == 0 else float("nan")
    share = {ph: phase_ms[ph] * launches[ph] for ph in launches}
    if persistent:
        # one launch = one greedy generation of up to GEN_LEN tokens from position 31; achieved =
        # the timed launches' algorithmic bytes over their summed duration
        launch_ms = ms / len(chunks)
        launch_bytes = timed_bytes / len(chunks)
        achieved = timed_bytes / (ms / 1e3) / 1e9
        traffic = read_traffic("k_decode_persistent")
        roofline = {"bound": "hbm", "kernel": "k_decode_persistent", "achieved": round(achieved, 1), "peak": peak,
                    "unit": "GB/s", "frac": round(achieved / peak, 4),
                    "traffic": int(traffic * launch_bytes / (GEN_LEN * bytes_per_tok_ref(shape, start)))
                    if traffic else None,
                    "peak_source": peak_kind, "algorithmic_bytes_per_launch": int(launch_bytes),
                    "launch_ms": round(launch_ms, 5), "tokens_per_launch": round(args.steps / len(chunks), 2),
                    "timed_positions": f"{start}..{start + max(chunks) - 1}",
                    "kernel_chain_phase_ms": {k: round(v, 5) for k, v in phase_ms.items()}}
    else:
        dom = max(share, key=share.get)
        achieved = pb[dom] / (phase_ms[dom] / 1e3) / 1e9
        roofline = {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                    "frac": round(achieved / peak, 4), "traffic": read_traffic(dom), "peak_source": peak_kind,
                    "algorithmic_bytes_per_launch": pb[dom], "launch_ms": round(phase_ms[dom], 5),
                    "phase_ms": {k: round(v, 5) for k, v in phase_ms.items()},
                    "phase_share": {k: round(v / sum(share.values()), 4) for k, v in share.items()}}
    step_gbs = bytes_tok * (value / world) / 1e9
    step_roofline = {"bound": "hbm", "achieved": round(step_gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(step_gbs / peak, 4), "bytes_per_token": int(bytes_tok),
                     "ideal_tok_s_per_gpu": round(peak * 1e9 / bytes_tok, 1)}

    batched = None
    if rank == 0 and world == 1 and args.b64_steps > 0:
        eng_b1 = eng
        batched = run_batched(args, model, shape, local_rank)
        eng = eng_b1
    gemv = run_gemv_sweep(local_rank) if (rank == 0 and world == 1 and args.gemv_sweep) else None
    box = None
    if args.box_steps > 0:  # every rank: its own 256 sequences
        box = run_box(args, model, shape, local_rank, world)
    tp2 = run_tp2(args, model, prompt, local_rank, rank, world) if (world == 2 and args.tp2) else None
    trace = None
    if persistent and rank == 0 and args.trace:
        tr = load_package().trace
        trace = tr.capture(eng, first, start, args.trace_raw)
    result = None
    if rank == 0:
        kernels_per_token = 1 + 5 * shape.layers + 2
        launches_timed = (args.steps + GEN_LEN - 1) // GEN_LEN if persistent else kernels_per_token * args.steps
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            with mp.get_context("spawn").Pool(1) as pool:
                secs, use_ref = pool.map(_ref_decode_worker, [(str(model), prompt, 1, args.cpu_tokens, True)])[0]
            cpu = {"value": round(args.cpu_tokens / secs, 4), "unit": "tok/s", "cores": 1,
                   "kind": "reference" if use_ref else "port",
                   "sample": f"one process, 1 thread: prefill of the 31-id prompt (untimed), 1 warm-up + "
                             f"{args.cpu_tokens} timed greedy decode tokens (forward_token + sample) from position 32"}
        if world == 1 and not args.no_cpu_baseline and (batched or box):
            # configs with many sequences: one reference process per host core, one sequence each
            # (the reference's prefill is the same token loop, so this also bounds its prefill rate)
            n_proc = max(1, min(host_cores(), 32))
            agg_steps = 6
            with mp.get_context("spawn").Pool(n_proc) as pool:
                times = pool.map(_ref_decode_worker, [(str(model), prompt, 1, agg_steps, False)] * n_proc)
            cpu_all = {"value": round(n_proc * agg_steps / max(t for t, _ in times), 4), "unit": "tok/s",
                       "cores": n_proc, "kind": "reference" if all(u for _, u in times) else "port",
                       "sample": f"{n_proc} concurrent processes (1 thread each), one sequence each from position "
                                 f"0, 1 warm-up + {agg_steps} timed greedy tokens each; aggregate tok/s"}
            for obj in (batched, box):
                if obj:
                    obj["cpu_baseline"] = cpu_all
        result = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": ("decode-b1: LLaMA-3.2-1B shape" if args.layers == 16 else
                                    f"decode-b1 profiling model: LLaMA-3.2-1B widths, {args.layers} layers")
                                   + ", LLM4S128 block-128 4-bit, seeded random-init N(0,0.02) weights, batch 1 per "
                                   f"GPU, greedy; 32-id prompt, then {args.steps} timed greedy tokens as generations "
                                   f"of up to {GEN_LEN} tokens from position {start} "
                                   f"(positions {start}..{start + max(chunks) - 1})",
                       "global_batch": world, "seq_len": start + GEN_LEN, "parallelism": f"dp{world} (replicas)",
                       "l2": "no flush: 657 MB of weights streamed per step > 126 MB L2"},
            "roofline": roofline, "step_roofline": step_roofline, "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 2), "unit": "tok/s", "h2d_bytes_per_step": 16, "d2h_bytes_per_step": 4,
                    "api": "llama_engine_forward_token + llama_engine_sample per step (C ABI via ctypes)",
                    "wall_s": round(wall, 4)},
            "gpu_launches": launches_timed, "decode_path": eng.decode_path, "clocks": clocks,
            **({"batch64": batched} if batched else {}),
            **({"box256": box} if box else {}),
            **({"tp2": tp2} if tp2 else {}),
            **({"gemv_sweep": gemv} if gemv else {}),
            **({"phase_trace": trace} if trace else {}),
        }
    eng.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


# ---------------------------------------------------------------------------------------------
# batched decode (64 sequences) and prefill (8 x 2048 tokens) on the tensor-core batched path
# ---------------------------------------------------------------------------------------------
def run_batched(args, model, shape, local_rank):
    """Batch-64 greedy decode: 64 prompts of 512 ids (fed through forward_batch, 1024 rows per
    call), then the greedy steps from position 512 on (b64_steps of them; 1536 reaches 2048).
    Prefill: 8 prompts of 2048 ids through llama_engine_prefill (last-position logits)."""
    import numpy as np
    import torch

    pkg = load_package()
    B, P = 64, 512
    bindings = pkg.LlamaEngineBindings()
    eng = pkg.LlamaEngine(str(model), bindings, device=local_rank, max_batch=B, max_seq_len=2048)
    lib = bindings.lib
    out = {"batch_path": eng.batch_path}
    if eng.batch_path != "tensor-core":
        eng.close()
        return out
    stream = torch.cuda.ExternalStream(lib.llama_engine_get_stream(eng.handle))
    rng = np.random.default_rng(2000 + local_rank)
    prompts = rng.integers(0, shape.vocab, (B, P)).astype(np.int32)
    per = 1024 // B
    for p0 in range(0, P - 1, per):
        ps = list(range(p0, min(P - 1, p0 + per)))
        eng.forward_batch([int(prompts[s, p]) for p in ps for s in range(B)], [p for p in ps for s in range(B)],
                          [s for p in ps for s in range(B)], False)
    slots = list(range(B))
    toks = [int(prompts[s, P - 1]) for s in range(B)]
    pos0 = P - 1
    steps = max(1, min(args.b64_steps, 2048 - P))
    # the timed steps start at position 511; warm-up steps run first at the same positions
    for w in range(3):
        eng.forward_batch(toks, [pos0 + w] * B, slots, True)
        eng.argmax_batch(B)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("decode64")  # profiling filter (ncu --nvtx-include "decode64/")
    ev0.record(stream)
    w0 = time.perf_counter()
    t = toks
    for i in range(steps):
        eng.forward_batch(t, [pos0 + i] * B, slots, True)
        t = eng.argmax_batch(B)
    ev1.record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - w0
    torch.cuda.nvtx.range_pop()
    ms = ev0.elapsed_time(ev1)
    peak, peak_kind = hbm_peak()
    kv_row = shape.layers * shape.kv_dim * 4 * 2
    step_bytes = [shape.weight_bytes() + B * kv_row * (pos0 + i + 2) for i in range(steps)]
    gbs = sum(step_bytes) / (ms / 1e3) / 1e9
    out.update({
        "value": round(B * steps / (ms / 1e3), 1), "unit": "tok/s", "ms_per_step": round(ms / steps, 4),
        "workload": f"decode-b64: {B} sequences, prompts of {P} ids, greedy steps at positions {pos0}..{pos0 + steps - 1}",
        "e2e": {"value": round(B * steps / wall, 1), "unit": "tok/s", "h2d_bytes_per_step": B * 12,
                "d2h_bytes_per_step": B * 4, "api": "llama_engine_forward_batch + llama_engine_argmax_batch per step"},
        "step_roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                          "frac": round(gbs / peak, 4), "peak_source": peak_kind,
                          "bytes_per_step": int(sum(step_bytes) / steps)},
    })
    # prefill: 8 prompts of 2048 ids, last-position logits
    n_seq, L = max(1, args.prefill_seqs), 2048
    pre = rng.integers(0, shape.vocab, (n_seq, L)).astype(np.int32)
    eng.prefill([int(x) for x in pre[0]], 0, True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("prefill")
    e0.record(stream)
    w0 = time.perf_counter()
    for sq in range(n_seq):
        eng.prefill([int(x) for x in pre[sq]], 0, True)
        eng.sample(0.0, 0.9)
    e1.record(stream)
    torch.cuda.synchronize()
    pwall = time.perf_counter() - w0
    torch.cuda.nvtx.range_pop()
    pms = e0.elapsed_time(e1)
    flops = n_seq * (2 * shape.layer_matrix_params() * L + shape.layers * 4 * shape.heads * 64 * L * (L + 1) // 2
                     + 2 * shape.vocab * shape.dim)
    out["prefill"] = {"value": round(n_seq * L / (pms / 1e3), 1), "unit": "tok/s", "ms_per_seq": round(pms / n_seq, 3),
                      "workload": f"prefill: {n_seq} sequences of {L} ids, last-position logits + greedy id",
                      "tflops": round(flops / (pms / 1e3) / 1e12, 2),
                      "e2e": {"value": round(n_seq * L / pwall, 1), "unit": "tok/s"}}
    eng.close()
    return out


def run_box(args, model, shape, local_rank, world):
    """Box-scale decode, one engine per rank: 256 sequences per GPU (KV for 4096 positions each,
    68.7 GB), 1024-id prompts fed through forward_batch (4 positions x 256 sequences per call),
    then greedy steps of all 256 sequences through forward_batch + argmax_batch.  Two windows of
    box_steps steps are timed: one from position 1023 and one ending at position 4094, after the
    KV of every sequence has been filled up to it by the same batched forward (random ids).  A
    step's bytes are affine in the position (weights + 256 * 64 KiB per position), so the mean of
    the two windows is the mean step of the whole 1024 -> 4096 decode.  Every rank runs the same
    collective steps; times are the max over ranks."""
    import numpy as np
    import torch
    import torch.distributed as dist

    pkg = load_package()
    B, P, MAXS = 256, 1024, 4096
    S = max(1, min(args.box_steps, 256))
    bindings = pkg.LlamaEngineBindings()
    eng = pkg.LlamaEngine(str(model), bindings, device=local_rank, max_batch=B, max_seq_len=MAXS)
    out = {"batch_path": eng.batch_path}
    if eng.batch_path != "tensor-core":
        eng.close()
        return out
    lib = bindings.lib
    stream = torch.cuda.ExternalStream(lib.llama_engine_get_stream(eng.handle))
    rank = dist.get_rank() if world > 1 else 0
    rng = np.random.default_rng(rank_seed(4000, rank))
    slots = list(range(B))
    per = 1024 // B

    def fill(p_begin, p_end, ids):
        """KV of positions [p_begin, p_end) of every sequence, ids[s, p] at (s, p).  Rows are
        sequence-major, so the rows of one sequence read its K / V rows as neighbouring CTAs."""
        for p0 in range(p_begin, p_end, per):
            ps = list(range(p0, min(p_end, p0 + per)))
            eng.forward_batch([int(ids[s, p]) for s in range(B) for p in ps], [p for s in range(B) for p in ps],
                              [s for s in range(B) for p in ps], False)

    def window(pos0, toks):
        """3 warm-up steps, then S timed greedy steps from pos0; returns (ms, next ids)."""
        for w in range(3):
            eng.forward_batch(toks, [pos0 + w] * B, slots, True)
            eng.argmax_batch(B)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        w0 = time.perf_counter()
        t = toks
        for i in range(S):
            eng.forward_batch(t, [pos0 + i] * B, slots, True)
            t = eng.argmax_batch(B)
        e1.record(stream)
        torch.cuda.synchronize()
        times = max_over_ranks([e0.elapsed_time(e1), (time.perf_counter() - w0) * 1e3], world)
        return times, t

    ids = rng.integers(0, shape.vocab, (B, MAXS)).astype(np.int32)
    f0 = time.perf_counter()
    fill(0, P - 1, ids)
    torch.cuda.synchronize()
    fill_s = time.perf_counter() - f0
    early_pos = P - 1
    (ms_a, wall_a), _ = window(early_pos, [int(x) for x in ids[:, P - 1]])
    late_pos = MAXS - 1 - S
    f0 = time.perf_counter()
    fill(early_pos + S, late_pos, ids)
    torch.cuda.synchronize()
    fill_s += time.perf_counter() - f0
    (ms_b, wall_b), _ = window(late_pos, [int(x) for x in ids[:, late_pos]])
    eng.close()
    peak, peak_kind = hbm_peak()
    kv_row = shape.layers * shape.kv_dim * 4 * 2

    def step_bytes(p):
        return shape.weight_bytes() + B * kv_row * (p + 2)

    bytes_a = sum(step_bytes(early_pos + i) for i in range(S))
    bytes_b = sum(step_bytes(late_pos + i) for i in range(S))
    mean_ms = (ms_a + ms_b) / (2 * S)
    mean_wall = (wall_a + wall_b) / (2 * S)
    gbs = (bytes_a + bytes_b) / ((ms_a + ms_b) / 1e3) / 1e9
    out.update({
        "value": round(world * B / (mean_ms / 1e3), 1), "unit": "tok/s", "n_gpus": world, "scaling": "weak",
        "ms_per_step": round(mean_ms, 4),
        "workload": (f"decode-b256 box scale: {B} sequences per GPU, 1024-id prompts, KV for {MAXS} positions; "
                     f"greedy steps at positions {early_pos}..{early_pos + S - 1} and {late_pos}..{late_pos + S - 1} "
                     f"(mean = mean step of the 1024 -> 4096 decode)"),
        "windows_ms_per_step": {str(early_pos): round(ms_a / S, 4), str(late_pos): round(ms_b / S, 4)},
        "e2e": {"value": round(world * B / (mean_wall / 1e3), 1), "unit": "tok/s", "h2d_bytes_per_step": B * 12,
                "d2h_bytes_per_step": B * 4, "api": "llama_engine_forward_batch + llama_engine_argmax_batch per step"},
        "step_roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                          "frac": round(gbs / peak, 4), "peak_source": peak_kind,
                          "bytes_per_step": int((bytes_a + bytes_b) / (2 * S))},
        "fill_s": round(fill_s, 2),
    })
    return out


def run_tp2(args, model, prompt, local_rank, rank, world):
    """Batch-1 latency on two GPUs with the 2-way tensor-parallel engine: one sequence, its layers
    split over the two ranks with two NCCL all-reduces per layer.  Same greedy generations from
    position 31 as the headline line; device time of each rank, max over the two."""
    import torch
    import torch.distributed as dist

    pkg = load_package()
    b = pkg.LlamaEngineBindings()
    obj = [pkg.tp_unique_id(b) if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    eng = pkg.LlamaEngine(str(model), b, device=local_rank, tp_rank=rank, tp_world=world, tp_unique_id=obj[0])
    stream = torch.cuda.ExternalStream(b.lib.llama_engine_get_stream(eng.handle))
    eng.prefill([int(t) for t in prompt[:-1]], 0, False)
    first, start = int(prompt[-1]), PROMPT_LEN - 1
    steps = min(args.steps, 512)

    def gen(n):
        done = 0
        while done < n:
            c = min(GEN_LEN, n - done)
            eng.generate_greedy(first, start, c)
            done += c

    gen(min(args.warmup, GEN_LEN))
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    gen(steps)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks([e0.elapsed_time(e1)], world)[0]
    eng.close()
    return {"value": round(steps / (ms / 1e3), 2), "unit": "tok/s", "n_gpus": 2, "steps": steps,
            "ms_per_token": round(ms / steps, 5),
            "workload": "decode-b1 latency, one sequence split over 2 GPUs (tensor parallel: q/kv heads, "
                        "W_o / W_down column halves, gate/up and lm_head row halves; 2 NCCL all-reduces per "
                        "layer), per-phase kernels in one CUDA graph per token",
            "api": "llama_engine_create_tp + llama_engine_generate_greedy"}


def run_gemv_sweep(local_rank, reps=200):
    """Isolated block-128 GEMV (llama_b128_gemv) at the model's five K x N shapes, M = 1 and 4:
    nibbles uniform 0..15, step ~U(1e-3, 2e-2) and min = -8 step U(0.8, 1.2) as bf16, x ~N(0, 1).
    Each shape cycles through enough copies of its matrix to pass 256 MB, so every call streams
    its weights from HBM rather than L2; algorithmic bytes N*K/128*68 + M*K*4 + M*N*4 per call."""
    import torch

    pkg = load_package()
    lib = pkg.LlamaEngineBindings().lib
    dev = torch.device("cuda", local_rank)
    g = torch.Generator(device=dev).manual_seed(11)
    peak, peak_kind = hbm_peak()
    stream = torch.cuda.current_stream(dev)
    rows = []
    for K, N in ((2048, 2048), (2048, 512), (2048, 8192), (8192, 2048), (2048, 128256)):
        mat = N * K // 128 * 68
        copies = max(1, -(-256 * 2**20 // mat))
        mats = []
        for _ in range(copies):
            nib = torch.randint(0, 256, (N * K // 2,), dtype=torch.uint8, device=dev, generator=g)
            step = torch.empty(N * K // 128, device=dev).uniform_(1e-3, 2e-2, generator=g)
            mn = -8.0 * step * torch.empty_like(step).uniform_(0.8, 1.2, generator=g)
            mats.append((nib, step.to(torch.bfloat16).view(torch.int16), mn.to(torch.bfloat16).view(torch.int16)))
        for M in (1, 4):
            x = torch.randn(M, K, device=dev, generator=g)
            y = torch.empty(M, N, device=dev)

            def call(i, st_handle):
                nib, st, mi = mats[i % copies]
                rc = lib.llama_b128_gemv(ctypes.c_void_p(nib.data_ptr()), ctypes.c_void_p(st.data_ptr()),
                                         ctypes.c_void_p(mi.data_ptr()), N, K, ctypes.c_void_p(x.data_ptr()), M,
                                         ctypes.c_void_p(y.data_ptr()), ctypes.c_void_p(st_handle))
                if rc != 0:
                    raise RuntimeError(f"llama_b128_gemv failed at K={K} N={N} M={M}")

            for i in range(min(2 * copies, 64)):
                call(i, stream.cuda_stream)
            torch.cuda.synchronize()
            # the launches are captured into a graph, so the timing is the kernels' back-to-back
            # device time and not the host's per-call cost
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                cap = torch.cuda.current_stream().cuda_stream
                for i in range(reps):
                    call(i, cap)
            graph.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(3):
                graph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (3 * reps)
            del graph
            gbs = (mat + M * K * 4 + M * N * 4) / (us * 1e-6) / 1e9
            rows.append({"K": K, "N": N, "M": M, "us": round(us, 2), "gbs": round(gbs, 1),
                         "frac": round(gbs / peak, 4)})
        del mats
    torch.cuda.empty_cache()
    return {"kernel": "k_gemv_mma (llama_b128_gemv)", "unit": "GB/s", "peak": peak, "peak_source": peak_kind,
            "timing": f"CUDA graph of {reps} launches per shape, replayed 3 times, CUDA events",
            "l2": "matrix copies cycled past 256 MB per shape", "shapes": rows}


def read_traffic(kernel_phase: str):
    """DRAM bytes per launch of the dominant kernel, from the committed ncu summary."""
    p = ROOT / "profiles" / "traffic_per_launch.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 2 and parts[0] == kernel_phase:
            try:
                return int(float(parts[1]))
            except ValueError:
                return None
    return None


def _write_model_subprocess() -> Path:
    """The config-0 model file, written (once, cached) by a child process, so that the reference
    arm's own process maps no library of this repository (the writer is one)."""
    out = subprocess.run([sys.executable, str(Path(__file__).resolve()), "--write-model"], capture_output=True,
                         text=True, check=True)
    return Path(out.stdout.strip().splitlines()[-1])


def _ref_decode_worker(args):
    """One reference process: prefill the 31-id prompt (untimed), `warm` greedy steps, then
    `steps` timed greedy steps (forward_token + sample), as in src/main.py:339-370."""
    model_path, prompt, warm, steps, with_prefill = args
    sys.path.insert(0, str(ROOT))
    import oracle
    use_ref = oracle.have_reference()
    lib = oracle.load_ref_engine() if use_ref else oracle.load_oracle()
    if use_ref:
        h = lib.llama_engine_create(str(model_path).encode())
        fwd = lambda t, p: lib.llama_engine_forward_token(h, t, p, 1)  # noqa: E731
        smp = lambda: lib.llama_engine_sample(h, ctypes.c_float(0.0), ctypes.c_float(0.9))  # noqa: E731
        pre = lambda ids: lib.llama_engine_prefill(h, (ctypes.c_int32 * len(ids))(*ids), len(ids), 0, 0)  # noqa: E731
    else:
        h = lib.orc_create(str(model_path).encode())
        fwd = lambda t, p: lib.orc_forward_token(h, t, p, 1)  # noqa: E731
        smp = lambda: lib.orc_sample_engine(h, ctypes.c_float(0.0), ctypes.c_float(0.9))  # noqa: E731
        pre = lambda ids: lib.orc_prefill(h, (ctypes.c_int32 * len(ids))(*ids), len(ids), 0, 0)  # noqa: E731
    pos = 0
    if with_prefill:
        pre([int(t) for t in prompt[:-1]])
        pos = len(prompt) - 1
    tok = int(prompt[-1])
    for _ in range(warm):
        fwd(tok, pos)
        tok = smp()
        pos += 1
    t0 = time.perf_counter()
    for _ in range(steps):
        fwd(tok, pos)
        tok = smp()
        pos += 1
    return time.perf_counter() - t0, use_ref


def run_reference(args, rank):
    """The reference engine itself (oracle/_ref, compiled from its own source; the C port of it
    only when that build is absent, and then labelled "port") on the host cores, on our arm's
    workload: one sequence, batch 1, the 32-id config-0 prompt prefilled, then greedy decode
    tokens from position 31.  The reference runs one sequence on one thread on Linux
    (src/llama_engine.cpp:79-80), so one process is all the threads it can use for this
    workload.  The all-cores aggregate (one sequence per process) is reported beside it."""
    if rank != 0:
        return None
    import numpy as np

    model = _write_model_subprocess()
    prompt = np.random.default_rng(rank_seed(1000, 0)).integers(0, 128256, PROMPT_LEN).astype(np.int32)
    steps = max(1, min(args.steps, args.ref_max_steps))
    warm = max(1, min(args.warmup, 2))
    ctx = mp.get_context("spawn")
    with ctx.Pool(1) as pool:
        secs, use_ref = pool.map(_ref_decode_worker, [(str(model), prompt, warm, steps, True)])[0]
    kind = "reference" if use_ref else "port"
    rate = steps / secs
    n_proc = max(1, min(host_cores(), 32))
    agg_steps = max(1, min(steps, 6))
    with ctx.Pool(n_proc) as pool:
        times = pool.map(_ref_decode_worker, [(str(model), prompt, 1, agg_steps, False)] * n_proc)
    agg = n_proc * agg_steps / max(t for t, _ in times)
    sample = (f"one process, 1 thread: prefill of the 31-id prompt (untimed), {warm} warm-up + {steps} timed "
              f"greedy decode tokens (forward_token + sample) at positions {PROMPT_LEN - 1 + warm}.."
              f"{PROMPT_LEN - 1 + warm + steps - 1}")
    return {"impl": "reference", "metric": METRIC, "value": round(rate, 4), "unit": "tok/s", "n_gpus": 0,
            "steps": steps, "warmup": warm, "ms_per_step": round(1e3 * secs / steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "decode-b1: LLaMA-3.2-1B shape, LLM4S128 block-128 4-bit, seeded random-init "
                                   "N(0,0.02) weights, batch 1, greedy; 32-id prompt, decode from position 31",
                       "global_batch": 1, "seq_len": PROMPT_LEN + warm + steps, "parallelism": "none (host CPU)"},
            "cpu_baseline": {"value": round(rate, 4), "unit": "tok/s", "cores": 1, "kind": kind, "sample": sample},
            "e2e": {"value": round(rate, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "all_cores_aggregate": {"value": round(agg, 4), "unit": "tok/s", "cores": n_proc, "kind": kind,
                                    "sample": f"{n_proc} concurrent processes, one sequence each from position 0, "
                                              f"1 warm-up + {agg_steps} timed greedy tokens each"}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3840)
    ap.add_argument("--warmup", type=int, default=256)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-tokens", type=int, default=12)
    ap.add_argument("--ref-max-steps", type=int, default=12)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--b64-steps", type=int, default=1536,
                    help="timed batch-64 decode steps from position 511 (0 = skip the batched measurements)")
    ap.add_argument("--no-gemv-sweep", dest="gemv_sweep", action="store_false",
                    help="skip the isolated GEMV sweep (five K x N shapes, M = 1 and 4)")
    ap.add_argument("--box-steps", type=int, default=32,
                    help="box-scale decode (256 sequences per GPU, 1024 -> 4096): timed steps per window (0 = skip)")
    ap.add_argument("--prefill-seqs", type=int, default=8, help="prefill measurement: sequences of 2048 ids")
    ap.add_argument("--trace", action="store_true", help="add the persistent kernel's phase timeline")
    ap.add_argument("--trace-raw", default=None, help="with --trace: save the raw trace array (.npy) here")
    ap.add_argument("--layers", type=int, default=16,
                    help="layers of the synthetic model (16 = LLaMA-3.2-1B; fewer only for profiling runs)")
    ap.add_argument("--no-tp2", dest="tp2", action="store_false",
                    help="skip the 2-way tensor-parallel batch-1 measurement of a 2-GPU run")
    ap.add_argument("--gemm-trace", default=None, metavar="M,N,K",
                    help="only trace CTA 0's pipeline of one isolated tcgen05 GEMM launch and print it")
    ap.add_argument("--write-model", action="store_true", help=argparse.SUPPRESS)
    args = ap.parse_args()
    if args.write_model:  # child of the reference arm: write the config-0 model, print its path
        pkg = load_package()
        print(pkg.model_file.cached_model(cache_dir(), pkg.model_file.LLAMA_3_2_1B, seed=0, sigma=0.02))
        return
    if args.gemm_trace:  # diagnostics of the batched path's GEMM, not a benchmark line
        M, N, K = (int(v) for v in args.gemm_trace.split(","))
        pkg = load_package()
        print(json.dumps(pkg.trace.capture_gemm(pkg.LlamaEngineBindings().lib, M, N, K)), flush=True)
        return
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    # libraries (NCCL's version banner, for one) may write to stdout; keep it for the JSON line
    sys.stdout.flush()
    saved_stdout = os.dup(1)
    os.dup2(2, 1)
    try:
        if args.impl == "reference":
            res = run_reference(args, rank)
        else:
            res = run_ours(args, rank, world, local_rank)
    finally:
        sys.stdout.flush()
        os.dup2(saved_stdout, 1)
        os.close(saved_stdout)
    if rank == 0 and res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
