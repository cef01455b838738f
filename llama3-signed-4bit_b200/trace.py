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


def capture(engine, token: int, pos: int) -> dict:
    """Runs one traced forward_token (with logits) and returns the phase breakdown."""
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
    return analyse(buf[: 2 * n].reshape(-1, CAP, 2))


def analyse(tr: np.ndarray) -> dict:
    """tr: [cta][CAP][(time_ns, tag)]"""
    t0 = None
    per_seg = defaultdict(dict)  # (kind, layer, cta) -> {event: t}
    for c in range(tr.shape[0]):
        for time_ns, tag in tr[c]:
            time_ns, tag = int(time_ns), int(tag)
            if time_ns == 0:
                break
            if tag == 0xFFFF0000:
                t0 = time_ns if t0 is None else min(t0, time_ns)
                continue
            ev, kind, layer = tag >> 16, (tag >> 8) & 0xFF, tag & 0xFF
            per_seg[(kind, layer, c)][ev] = time_ns  # event 5 holds SM cycles spent waiting on ring data
    agg = defaultdict(lambda: defaultdict(list))
    ends = defaultdict(lambda: defaultdict(int))
    for (kind, layer, c), ev in per_seg.items():
        if all(e in ev for e in (1, 2, 3, 4)):
            k = KINDS.get(kind, str(kind))
            agg[k]["wait_us"].append((ev[2] - ev[1]) / 1e3)
            agg[k]["stage_us"].append((ev[3] - ev[2]) / 1e3)
            agg[k]["work_us"].append((ev[4] - ev[3]) / 1e3)
            if 5 in ev:
                agg[k]["ring_wait_kcyc"].append(ev[5] / 1e3)
            ends[k][layer] = max(ends[k][layer], ev[4])
    out = {}
    for k, d in agg.items():
        out[k] = {m: round(float(np.mean(v)), 3) for m, v in d.items()}
        out[k]["max_work_us"] = round(float(np.max(d["work_us"])), 3)
        out[k]["n"] = len(d["work_us"])
    if t0 is not None:
        out["critical_path_end_us"] = {k: {int(l): round((t - t0) / 1e3, 2) for l, t in sorted(v.items())}
                                       for k, v in ends.items()}
    return out
