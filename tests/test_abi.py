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
