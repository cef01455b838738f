"""Phase timeline of the persistent token-step kernel (llama_engine_trace).

For one token it reports, per phase kind, the mean over CTAs and layers of
* ``wait_us``  — from the phase's start to its dependency being satisfied,
* ``stage_us`` — staging the input vector into MMA digit fragments,
* ``work_us``  — the CTA's records / attention heads of the phase,
and ``end_us``, the time (from the token's start) at which the last CTA finished the phase,
per layer, which is the critical path through the token.
"""
from __future__ import annotations

import ctypes
from collections import defaultdict

import numpy as np

KINDS = {0: "qkv", 1: "attn", 2: "oproj", 3: "gateup", 4: "down", 5: "lmhead"}
CAP = 1024


def capture(engine, token: int, pos: int, raw_path: str | None = None) -> dict:
    """Runs one traced forward_token (with logits) and returns the phase breakdown; with
    ``raw_path`` the raw [cta][entry][(time, word)] array is also saved there (numpy .npy)."""
    lib = engine.bindings.lib
    h = engine.handle
    if lib.llama_engine_trace(h, 1, None, 0) != 0:
        raise RuntimeError("trace needs the persistent decode path")
    engine.forward_token(token, pos, True)
    engine.sample(0.0, 0.9)
    n_max = 4096 * CAP
    buf = np.zeros(n_max * 2, dtype=np.uint64)
    n = lib.llama_engine_trace(h, 2, buf.ctypes.data_as(ctypes.c_void_p), n_max)
    lib.llama_engine_trace(h, 0, None, 0)
    if n <= 0:
        raise RuntimeError("trace read failed")
    tr = buf[: 2 * n].reshape(-1, CAP, 2)
    if raw_path:
        np.save(raw_path, tr)
    out = analyse(tr)
    out["fine_cycles"] = analyse_fine(tr)
    return out


# events: 1 segment start, 2 after the CTA barrier, 3 input staged, 4 end, 5 ring-wait cycles,
# 6 residual loaded, 7 record data ready, 8 record reduced, 9 partials accumulated (layers 1-2);
# attention (layers 1-2): 10 q/k/v loaded, 11 scores, 12 softmax, 13 PV partials
EVENT_NAMES = {1: "start", 2: "barrier", 3: "staged", 4: "end", 6: "residual", 7: "rec_ready", 8: "rec_reduced",
               9: "rec_accumulated", 10: "qkv_loaded", 11: "scores", 12: "softmax", 13: "pv"}


def analyse_fine(tr: np.ndarray) -> dict:
    """SM-clock intervals between consecutive events of one CTA inside the segments of layers 1
    and 2: mean cycles per occurrence of each (kind, from -> to) transition, and its count."""
    acc = defaultdict(list)
    for c in range(tr.shape[0]):
        prev = None
        for time_ns, word in tr[c]:
            time_ns, word = int(time_ns), int(word)
            if time_ns == 0:
                break
            tag, clk = word & 0xFFFFFFFF, word >> 32
            if tag == 0xFFFF0000:
                prev = None
                continue
            ev, kind, layer = tag >> 16, (tag >> 8) & 0xFF, tag & 0xFF
            if ev == 5:
                continue
            if layer in (1, 2) and prev is not None and prev[0] == (kind, layer):
                acc[(KINDS.get(kind, str(kind)), EVENT_NAMES.get(prev[1], str(prev[1])),
                     EVENT_NAMES.get(ev, str(ev)))].append((clk - prev[2]) & 0xFFFFFFFF)
            prev = ((kind, layer), ev, clk)
    return {f"{k} {a}->{b}": {"mean_cyc": round(float(np.mean(v)), 1), "max_cyc": int(np.max(v)), "n": len(v)}
            for (k, a, b), v in sorted(acc.items())}


def analyse(tr: np.ndarray) -> dict:
    """tr: [cta][CAP][(time_ns, tag | clock << 32)]"""
    t0 = None
    per_seg = defaultdict(dict)  # (kind, layer, cta) -> {event: t}
    for c in range(tr.shape[0]):
        for time_ns, tag in tr[c]:
            time_ns, tag = int(time_ns), int(tag) & 0xFFFFFFFF
            if time_ns == 0:
                break
            if tag == 0xFFFF0000:
                t0 = time_ns if t0 is None else min(t0, time_ns)
                continue
            ev, kind, layer = tag >> 16, (tag >> 8) & 0xFF, tag & 0xFF
            per_seg[(kind, layer, c)][ev] = time_ns  # event 5 holds SM cycles spent waiting on ring data
    agg = defaultdict(lambda: defaultdict(list))
    ends = defaultdict(lambda: defaultdict(int))
    layer_work = defaultdict(lambda: defaultdict(list))  # kind -> layer -> work of each CTA
    for (kind, layer, c), ev in per_seg.items():
        if all(e in ev for e in (1, 2, 3, 4)):
            k = KINDS.get(kind, str(kind))
            agg[k]["wait_us"].append((ev[2] - ev[1]) / 1e3)
            agg[k]["stage_us"].append((ev[3] - ev[2]) / 1e3)
            agg[k]["work_us"].append((ev[4] - ev[3]) / 1e3)
            layer_work[k][layer].append((ev[4] - ev[3]) / 1e3)
            if 5 in ev:
                agg[k]["ring_wait_kcyc"].append(ev[5] / 1e3)
            ends[k][layer] = max(ends[k][layer], ev[4])
    out = {}
    for k, d in agg.items():
        out[k] = {m: round(float(np.mean(v)), 3) for m, v in d.items()}
        # slowest single (CTA, layer) sample, and the slowest CTA of each layer averaged over the
        # layers (the one that holds up the next phase): max-over-CTAs / mean-over-CTAs per layer
        out[k]["max_work_us"] = round(float(np.max(d["work_us"])), 3)
        lw = layer_work[k].values()
        out[k]["layer_max_work_us"] = round(float(np.mean([max(v) for v in lw])), 3)
        out[k]["layer_max_over_mean"] = round(float(np.mean([max(v) / max(np.mean(v), 1e-9) for v in lw])), 3)
        out[k]["n"] = len(d["work_us"])
    if t0 is not None:
        out["critical_path_end_us"] = {k: {int(l): round((t - t0) / 1e3, 2) for l, t in sorted(v.items())}
                                       for k, v in ends.items()}
    return out


# ---------------------------------------------------------------------------------------------
# tcgen05 GEMM pipeline trace: CTA 0's globaltimer stamps per K block (kTraceEvents x
# kTraceBlocks, written by llama_b128_gemm when $LLAMA_B128_GEMM_TRACE names a file).
# ---------------------------------------------------------------------------------------------
GEMM_EVENTS = 10
GEMM_BLOCKS = 256
# 0 copies issued, 1 MMA inputs ready, 2 dequantiser sees the stage, 3 A codes written,
# 4 epilogue sees the accumulator, 5 epilogue done, 6 MMAs issued, 7 commit issued,
# 8 MMA loop top, 9 issuer past its barrier tests
GEMM_INTERVALS = {
    "issuer: barrier tests (8 -> 9)": (8, 9, 0),
    "issuer: tests -> inputs ready (9 -> 1)": (9, 1, 0),
    "issuer: the block's MMAs issued (1 -> 6)": (1, 6, 0),  # 8 (64-token units) or 16 (128-token)
    "issuer: commit (6 -> 7)": (6, 7, 0),
    "issuer: to next block (7 -> 8 of g+1)": (7, 8, 1),
    "issuer: block period (8 -> 8 of g+1)": (8, 8, 1),
    "slack: copies issued -> inputs ready (0 -> 1)": (0, 1, 0),
    "dequantiser: stage seen -> A codes written (2 -> 3)": (2, 3, 0),
    "slack: A codes written -> inputs ready (3 -> 1)": (3, 1, 0),
    "commit -> epilogue sees the accumulator (7 -> 4)": (7, 4, 0),
    "epilogue per block (4 -> 5)": (4, 5, 0),
    "slack: epilogue done -> inputs of g+2 ready (5 -> 1 of g+2)": (5, 1, 2),
}


def gemm_pipeline(path) -> dict:
    """Median ns of each pipeline interval over CTA 0's blocks (the first 8 and the last are
    left out: pipeline fill and drain)."""
    t = np.fromfile(path, dtype=np.uint64).astype(np.int64).reshape(GEMM_EVENTS, GEMM_BLOCKS)
    nb = int((t[7] > 0).sum())
    sl = slice(8, max(9, min(nb - 2, GEMM_BLOCKS - 2)))
    out = {"blocks": nb}
    for name, (a, b, shift) in GEMM_INTERVALS.items():
        out[name] = float(np.median(np.roll(t[b], -shift)[sl] - t[a][sl]))
    return out


def capture_gemm(lib, M: int, N: int, K: int, seed: int = 3, path: str | None = None) -> dict:
    """Runs the isolated tcgen05 GEMM (llama_b128_gemm) on seeded synthetic weights at M x N x K
    twice untraced and once traced, and returns gemm_pipeline() of the traced launch."""
    import os
    import tempfile

    import torch

    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(seed)
    nib = torch.randint(0, 256, (N * K // 2,), dtype=torch.uint8, device=dev, generator=g)
    step = torch.empty(N * K // 128, device=dev).uniform_(1e-3, 2e-2, generator=g)
    mn = -8.0 * step * torch.empty_like(step).uniform_(0.8, 1.2, generator=g)
    step16 = step.to(torch.bfloat16).view(torch.int16)
    mn16 = mn.to(torch.bfloat16).view(torch.int16)
    x = torch.randn(M, K, device=dev, generator=g)
    y = torch.empty(M, N, device=dev)
    path = path or os.path.join(tempfile.gettempdir(), f"gemm_trace_{M}x{N}x{K}.bin")
    stream = torch.cuda.current_stream(dev).cuda_stream
    for rep in range(3):
        if rep == 2:
            os.environ["LLAMA_B128_GEMM_TRACE"] = path
        try:
            rc = lib.llama_b128_gemm(ctypes.c_void_p(nib.data_ptr()), ctypes.c_void_p(step16.data_ptr()),
                                     ctypes.c_void_p(mn16.data_ptr()), N, K, ctypes.c_void_p(x.data_ptr()), M,
                                     ctypes.c_void_p(y.data_ptr()), ctypes.c_void_p(stream))
        finally:
            os.environ.pop("LLAMA_B128_GEMM_TRACE", None)
        if rc != 0:
            raise RuntimeError(f"llama_b128_gemm failed at {M} x {N} x {K}")
    return {"M": M, "N": N, "K": K, **gemm_pipeline(path)}
