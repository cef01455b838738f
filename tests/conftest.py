"""Shared fixtures.

* ``gpu`` marks tests that need a CUDA device (run on the B200 box); everything else runs on CPU.
* The product package lives in ``llama3-signed-4bit_b200/`` (not an identifier) and is imported
  here as ``llama3_signed_4bit_b200``.
* Model files are generated (seeded, deterministic) into a cache directory outside the repo:
  $LLAMA_B200_CACHE, default <tmpdir>/llama3_b200_cache.
"""
from __future__ import annotations

import importlib.util
import os
import sys
import tempfile
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG_DIR = ROOT / "llama3-signed-4bit_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"

if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


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


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")
    config.addinivalue_line("markers", "slow: long-running (full 1B model on the oracle)")


@pytest.fixture(scope="session")
def pkg():
    return load_package()


@pytest.fixture(scope="session")
def cache_dir() -> Path:
    d = Path(os.environ.get("LLAMA_B200_CACHE", Path(tempfile.gettempdir()) / "llama3_b200_cache"))
    d.mkdir(parents=True, exist_ok=True)
    return d


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle
    oracle.build()
    return oracle.load_oracle()


@pytest.fixture(scope="session")
def ref_kernels():
    import oracle
    oracle.build()
    if not oracle.have_reference():
        pytest.skip("reference build (oracle/_ref) not available")
    return oracle.load_ref_kernels()


@pytest.fixture(scope="session")
def ref_engine():
    import oracle
    oracle.build()
    if not oracle.have_reference():
        pytest.skip("reference build (oracle/_ref) not available")
    return oracle.load_ref_engine()


# Small model with the reference's fixed attention geometry (32 heads of 64, 8 kv heads: the
# reference hard-codes 4 head groups of 8 and kv_h = h/4, src/llama_engine.cpp:960-966).
SMALL_SHAPE = dict(layers=2, dim=2048, ffn=2048, vocab=4096, heads=32, kv_heads=8)
# ffn not a multiple of 2048: served by the per-phase kernel chain
CHAIN_SHAPE = dict(layers=2, dim=2048, ffn=1024, vocab=4096, heads=32, kv_heads=8)


@pytest.fixture(scope="session")
def small_model(pkg, cache_dir):
    shape = pkg.model_file.ModelShape(**SMALL_SHAPE)
    return pkg.model_file.cached_model(cache_dir, shape, seed=7, sigma=0.02, random_norms=True)


@pytest.fixture(scope="session")
def chain_model(pkg, cache_dir):
    shape = pkg.model_file.ModelShape(**CHAIN_SHAPE)
    return pkg.model_file.cached_model(cache_dir, shape, seed=9, sigma=0.02, random_norms=True)


@pytest.fixture(scope="session")
def full_model(pkg, cache_dir):
    return pkg.model_file.cached_model(cache_dir, pkg.model_file.LLAMA_3_2_1B, seed=0, sigma=0.02)


def fptr(a: np.ndarray):
    return a.ctypes.data


@pytest.fixture(scope="session")
def gpu_available():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return True
