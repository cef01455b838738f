"""Phase-trace decoder of the persistent kernel (host logic only, on a synthetic trace array)."""
from __future__ import annotations

import numpy as np


def _entry(ev, kind, layer):
    return (ev << 16) | (kind << 8) | layer


def test_analyse_phase_breakdown(pkg):
    tr_mod = pkg.trace
    # 3 CTAs, one qkv segment (kind 0) in layers 0 and 1; times in ns after a token start at 1000
    tr = np.zeros((3, 16, 2), dtype=np.int64)
    work = {0: [1000, 2000, 3000], 1: [1000, 1000, 4000]}  # ns of work per CTA and layer
    for c in range(3):
        rows = [(1000, 0xFFFF0000)]
        t = 2000
        for layer in (0, 1):
            rows += [(t, _entry(1, 0, layer)), (t + 100, _entry(2, 0, layer)), (t + 300, _entry(3, 0, layer)),
                     (t + 300 + work[layer][c], _entry(4, 0, layer))]
            t += 10000
        for i, (a, b) in enumerate(rows):
            tr[c, i] = (a, b)
    out = tr_mod.analyse(tr)
    q = out["qkv"]
    assert q["n"] == 6
    assert abs(q["wait_us"] - 0.1) < 1e-9 and abs(q["stage_us"] - 0.2) < 1e-9
    assert abs(q["work_us"] - np.mean(work[0] + work[1]) / 1e3) < 1e-9
    assert q["max_work_us"] == 4.0
    assert abs(q["layer_max_work_us"] - (3.0 + 4.0) / 2) < 1e-9
    assert abs(q["layer_max_over_mean"] - round((3.0 / 2.0 + 4.0 / 2.0) / 2, 3)) < 1e-9
    # the last CTA to finish each layer, from the token's start
    assert out["critical_path_end_us"]["qkv"] == {0: 4.3, 1: 15.3}


def test_gemm_pipeline_intervals(pkg, tmp_path):
    tr_mod = pkg.trace
    E, B = tr_mod.GEMM_EVENTS, tr_mod.GEMM_BLOCKS
    nb = 40
    t = np.zeros((E, B), dtype=np.uint64)
    for g in range(nb):  # a steady pipeline: one block every 700 ns
        base = 10_000 + 700 * g
        t[8, g], t[9, g], t[1, g], t[6, g], t[7, g] = base, base + 60, base + 200, base + 520, base + 580
        t[0, g], t[2, g], t[3, g] = base - 3000, base - 2500, base - 2000
        t[4, g], t[5, g] = base + 800, base + 1150
    p = tmp_path / "trace.bin"
    t.tofile(p)
    out = tr_mod.gemm_pipeline(p)
    assert out["blocks"] == nb
    assert out["issuer: block period (8 -> 8 of g+1)"] == 700
    assert out["issuer: barrier tests (8 -> 9)"] == 60
    assert out["issuer: the block's MMAs issued (1 -> 6)"] == 320
    assert out["epilogue per block (4 -> 5)"] == 350
    assert out["slack: epilogue done -> inputs of g+2 ready (5 -> 1 of g+2)"] == 200 + 1400 - 1150
