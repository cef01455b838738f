"""C-ABI checks that need no GPU: the library loads, exports every declared symbol, and the
host-side error paths behave like the reference (NULL handle, bad files)."""
from __future__ import annotations

import ctypes
import re

import numpy as np
import pytest

from conftest import ROOT


def declared_symbols():
    text = (ROOT / "include" / "llama_engine.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b((?:llama_engine|llama_tokenizer|llama_b128)_[a-z0-9_]+)\s*\(", text)))


REFERENCE_SYMBOLS = [
    "llama_engine_create", "llama_engine_free", "llama_engine_reset", "llama_engine_get_num_layers",
    "llama_engine_get_dim", "llama_engine_get_ffn_dim", "llama_engine_get_vocab_size",
    "llama_engine_get_num_heads", "llama_engine_get_num_kv_heads", "llama_engine_get_head_dim",
    "llama_engine_get_max_seq_len", "llama_engine_forward_token", "llama_engine_prefill",
    "llama_engine_sample", "llama_engine_get_logits", "llama_engine_dequantize_embedding",
    "llama_tokenizer_create", "llama_tokenizer_free", "llama_tokenizer_encode", "llama_tokenizer_decode",
]


@pytest.fixture(scope="module")
def bindings(pkg):
    return pkg.LlamaEngineBindings()


def test_header_declares_reference_abi():
    decl = declared_symbols()
    for s in REFERENCE_SYMBOLS:
        assert s in decl


def test_library_exports_every_declared_symbol(bindings):
    for s in declared_symbols():
        assert hasattr(bindings.lib, s), s


def test_reference_exports_same_abi(ref_engine):
    for s in REFERENCE_SYMBOLS:
        assert hasattr(ref_engine, s)


def test_null_handle_behaviour(bindings):
    lib = bindings.lib
    for name in ("num_layers", "dim", "ffn_dim", "vocab_size", "num_heads", "num_kv_heads", "head_dim"):
        assert getattr(lib, "llama_engine_get_" + name)(None) == 0
    assert lib.llama_engine_get_max_seq_len(None) == 8192
    assert lib.llama_engine_forward_token(None, 1, 0, 1) == -1
    assert lib.llama_engine_prefill(None, None, 0, 0, 0) == -1
    assert lib.llama_engine_sample(None, 0.0, 0.9) == 0
    assert not lib.llama_engine_get_logits(None)
    lib.llama_engine_free(None)
    lib.llama_engine_reset(None)
    lib.llama_engine_dequantize_embedding(None, 0, None)
    assert lib.llama_engine_generate_greedy(None, 0, 0, 1, None) == -1
    assert lib.llama_engine_forward_batch(None, None, None, None, 1, 1) == -1
    assert not lib.llama_engine_create(None)


def test_create_rejects_bad_files(bindings, tmp_path, small_model):
    lib = bindings.lib
    assert not lib.llama_engine_create(str(tmp_path / "missing.bin").encode())
    bad = tmp_path / "bad.bin"
    bad.write_bytes(b"NOTLLM4S" + bytes(64))
    assert not lib.llama_engine_create(str(bad).encode())
    assert b"magic" in lib.llama_engine_last_error(None)
    data = small_model.read_bytes()
    trunc = tmp_path / "trunc.bin"
    trunc.write_bytes(data[: len(data) - 1000])
    assert not lib.llama_engine_create(str(trunc).encode())
    assert b"truncated" in lib.llama_engine_last_error(None)
    # a matrix record whose num_blocks disagrees with its shape
    mangled = bytearray(data)
    off = 36 + 2048 * 4 + 2 * 2048 * 4 + 8  # first matrix header: num_blocks field
    mangled[off:off + 4] = (12345).to_bytes(4, "little")
    mm = tmp_path / "mangled.bin"
    mm.write_bytes(bytes(mangled))
    assert not lib.llama_engine_create(str(mm).encode())


def test_geometry_checks(bindings, pkg, tmp_path):
    shape = pkg.model_file.ModelShape(layers=1, dim=1024, ffn=1024, vocab=256, heads=8, kv_heads=2)
    p = pkg.model_file.write_model(tmp_path / "hd128.bin", shape, seed=1)  # head_dim 128
    assert not bindings.lib.llama_engine_create(str(p).encode())
    assert b"head_dim" in bindings.lib.llama_engine_last_error(None)


@pytest.mark.parametrize("geometry", [
    (16, 2048, 8192, 128256, 32, 8),   # LLaMA-3.2-1B
    (2, 2048, 2048, 4096, 32, 8),      # the small test model
    (2, 2048, 4096, 4096, 32, 8),
])
@pytest.mark.parametrize("grid", [148, 160])
def test_persistent_schedule_is_complete(bindings, geometry, grid):
    """The persistent kernel's schedule, read the way the kernel reads it: every tile of every
    phase on exactly one CTA with its own records, records in stream order, heads once a layer."""
    err = ctypes.create_string_buffer(256)
    rc = bindings.lib.llama_engine_check_schedule(*geometry, grid, err, 256)
    assert rc == 0, err.value.decode()


def test_persistent_schedule_rejects_bad_geometry(bindings):
    err = ctypes.create_string_buffer(256)
    assert bindings.lib.llama_engine_check_schedule(16, 4096, 8192, 128256, 32, 8, 148, err, 256) == -1
    assert err.value
    assert bindings.lib.llama_engine_check_schedule(16, 2048, 8192, 128256, 32, 8, 0, None, 0) == -1


def _plan(bindings, sms, tiles, kb, img_tiles, splits_req):
    out = (ctypes.c_int32 * 4)()
    assert bindings.lib.llama_b128_gemm_plan(sms, tiles, kb, img_tiles, splits_req, out) == 0
    return tuple(out)


# LLaMA-3.2-1B batched-path matrices: (128-row tiles, K blocks, fixed splits or -1)
_MATS = {"qkv": (24, 16, -1), "o": (16, 16, -1), "gate_up": (128, 16, 1), "down": (16, 64, -1),
         "lm_head": (1002, 16, 1)}


@pytest.mark.parametrize("rows", [1, 64, 128, 192, 256, 512, 1024, 2048])
@pytest.mark.parametrize("mat", sorted(_MATS))
def test_gemm_plan_covers_the_work(bindings, rows, mat):
    """Whatever form the planner picks, its units cover every token tile and every K block once."""
    tiles, kb, req = _MATS[mat]
    img = (rows + 63) // 64
    p, groups, splits, kbs = _plan(bindings, 148, tiles, kb, img, req)
    assert p in (1, 2) and (p == 1 or img >= 2)
    assert groups == (img + p - 1) // p
    assert splits * kbs >= kb and (splits - 1) * kbs < kb
    if req > 0:
        assert splits == req


def test_gemm_plan_choices(bindings):
    """The forms the engine's steps take: one image tile cannot pair (batch-64 decode); prefill
    chunks and box-scale steps pair tiles; 192 rows keep one-tile q|k|v units (the estimate is
    slightly shorter)."""
    P = lambda mat, rows: _plan(bindings, 148, *_MATS[mat][:2], (rows + 63) // 64, _MATS[mat][2])
    for mat in _MATS:
        assert P(mat, 64)[0] == 1
        assert P(mat, 2048) == (2, 16, 1, _MATS[mat][1])
    assert P("qkv", 64) == (1, 1, 6, 3)
    assert P("qkv", 256) == (2, 2, 3, 6)
    assert P("down", 256) == (2, 2, 4, 16)
    assert P("qkv", 192)[0] == 1
    # the isolated GEMM's test shapes (splits fixed at 1)
    assert _plan(bindings, 148, 64, 16, 16, 1)[0] == 2    # 1024 x 8192 x 2048
    assert _plan(bindings, 148, 16, 16, 17, 1)[:2] == (2, 9)  # 1050 rows: odd tile count
    assert _plan(bindings, 148, 16, 64, 18, 1)[0] == 2    # 1100 x 2048 x 8192
    assert _plan(bindings, 148, 3, 64, 3, 1)[0] == 1      # 130 x 384 x 8192


def test_gemm_plan_rejects_bad_args(bindings):
    out = (ctypes.c_int32 * 4)()
    lib = bindings.lib
    assert lib.llama_b128_gemm_plan(0, 16, 16, 1, -1, out) == -1
    assert lib.llama_b128_gemm_plan(148, 0, 16, 1, -1, out) == -1
    assert lib.llama_b128_gemm_plan(148, 16, 16, 0, -1, out) == -1
    assert lib.llama_b128_gemm_plan(148, 16, 16, 1, 17, out) == -1
    assert lib.llama_b128_gemm_plan(148, 16, 16, 1, -1, None) == -1
