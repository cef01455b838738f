"""ORACLE — test infrastructure only.

ctypes loaders for (a) the C restatement of the reference token loop (``oracle.c``) and (b) the
reference itself compiled from its own source (``_ref/``).  Only the test suite,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` import this package, and only
to check or time the reference algorithm; the product library never touches it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

ORACLE_DIR = Path(__file__).resolve().parent
ORACLE_LIB = ORACLE_DIR / "_build" / "liboracle.so"
REF_ENGINE_LIB = ORACLE_DIR / "_ref" / "libllama_engine_ref.so"
REF_KERNELS_LIB = ORACLE_DIR / "_ref" / "libref_kernels.so"

_P = ctypes.c_void_p
_F = ctypes.POINTER(ctypes.c_float)


def _default_ref_dir() -> str | None:
    """The reference tree: $LLAMA_REF_DIR, else the building machine's copy if present."""
    env = os.environ.get("LLAMA_REF_DIR")
    if env:
        return env
    cand = Path("/root/reference")
    return str(cand) if (cand / "src" / "llama_engine.cpp").exists() else None


def build(ref_dir: str | None = None) -> None:
    """Runs oracle/Makefile (restatement always; the reference builds when its source is given)."""
    cmd = ["make", "-s", "-C", str(ORACLE_DIR)]
    ref_dir = ref_dir or _default_ref_dir()
    if ref_dir:
        cmd.append(f"REF_DIR={ref_dir}")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{res.stdout}\n{res.stderr}")


def _kernel_sigs(lib, prefix: str) -> None:
    u8p, u16p, fp = ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p
    getattr(lib, prefix + "gemv").argtypes = [u8p, u16p, u16p, ctypes.c_uint32, ctypes.c_uint32, fp, fp, fp]
    getattr(lib, prefix + "gemv").restype = None
    getattr(lib, prefix + "swiglu").argtypes = [u8p, u16p, u16p, u8p, u16p, u16p, ctypes.c_uint32,
                                                ctypes.c_uint32, fp, fp, fp]
    getattr(lib, prefix + "swiglu").restype = None
    getattr(lib, prefix + "block_sums").argtypes = [fp, ctypes.c_size_t, fp]
    getattr(lib, prefix + "rms_norm").argtypes = [fp, fp, fp, ctypes.c_size_t]
    getattr(lib, prefix + "apply_rope").argtypes = [fp, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t, fp, fp]
    getattr(lib, prefix + "sample").argtypes = [fp, ctypes.c_size_t, ctypes.c_float, ctypes.c_float]
    getattr(lib, prefix + "sample").restype = ctypes.c_int32


def load_oracle():
    """The C restatement (``orc_*`` functions)."""
    if not ORACLE_LIB.exists():
        build()
    lib = ctypes.CDLL(str(ORACLE_LIB))
    _kernel_sigs(lib, "orc_")
    lib.orc_dequant_row.argtypes = [_P, _P, _P, ctypes.c_uint32, ctypes.c_size_t, _P]
    lib.orc_create.argtypes = [ctypes.c_char_p]
    lib.orc_create.restype = _P
    lib.orc_free.argtypes = [_P]
    lib.orc_forward_token.argtypes = [_P, ctypes.c_int32, ctypes.c_size_t, ctypes.c_int]
    lib.orc_prefill.argtypes = [_P, _P, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_int]
    lib.orc_prefill.restype = ctypes.c_int
    lib.orc_sample_engine.argtypes = [_P, ctypes.c_float, ctypes.c_float]
    lib.orc_sample_engine.restype = ctypes.c_int32
    lib.orc_get_logits.argtypes = [_P]
    lib.orc_get_logits.restype = _F
    lib.orc_get_kv.argtypes = [_P, ctypes.c_int, ctypes.c_int]
    lib.orc_get_kv.restype = _F
    lib.orc_get_x.argtypes = [_P]
    lib.orc_get_x.restype = _F
    lib.orc_get_rope.argtypes = [_P, ctypes.c_int]
    lib.orc_get_rope.restype = _F
    lib.orc_get_vocab.argtypes = [_P]
    lib.orc_get_vocab.restype = ctypes.c_uint32
    lib.orc_greedy_run.argtypes = [_P, _P, ctypes.c_size_t, ctypes.c_size_t, _P, _P]
    lib.orc_greedy_run.restype = ctypes.c_int
    return lib


def have_reference() -> bool:
    return REF_ENGINE_LIB.exists() and REF_KERNELS_LIB.exists()


def load_ref_kernels():
    """The reference's own kernels (``ref_*``), compiled from the reference source."""
    lib = ctypes.CDLL(str(REF_KERNELS_LIB))
    _kernel_sigs(lib, "ref_")
    lib.ref_dequant_row.argtypes = [_P, _P, _P, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_size_t, _P]
    return lib


def load_ref_engine():
    """The reference engine (``llama_engine_*``), with the argtypes of src/main.py:57-140."""
    lib = ctypes.CDLL(str(REF_ENGINE_LIB))
    lib.llama_engine_create.argtypes = [ctypes.c_char_p]
    lib.llama_engine_create.restype = _P
    lib.llama_engine_free.argtypes = [_P]
    lib.llama_engine_forward_token.argtypes = [_P, ctypes.c_int32, ctypes.c_size_t, ctypes.c_int]
    lib.llama_engine_forward_token.restype = ctypes.c_int
    lib.llama_engine_prefill.argtypes = [_P, ctypes.POINTER(ctypes.c_int32), ctypes.c_size_t,
                                         ctypes.c_size_t, ctypes.c_int]
    lib.llama_engine_prefill.restype = ctypes.c_int
    lib.llama_engine_sample.argtypes = [_P, ctypes.c_float, ctypes.c_float]
    lib.llama_engine_sample.restype = ctypes.c_int32
    lib.llama_engine_get_logits.argtypes = [_P]
    lib.llama_engine_get_logits.restype = _F
    for name in ("num_layers", "dim", "ffn_dim", "vocab_size", "num_heads", "num_kv_heads",
                 "head_dim", "max_seq_len"):
        f = getattr(lib, "llama_engine_get_" + name)
        f.argtypes = [_P]
        f.restype = ctypes.c_int32
    return lib
