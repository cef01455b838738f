"""The ``LLM4S128`` block-128 4-bit weight file: seeded writer and a numpy reader.

Format (read by the reference at src/llama_engine.cpp:865-906 and 164-180)::

    "LLM4S128" | u32 layers, dim, ffn, vocab, heads, kv_heads, block(=128)
    f32 final_norm[dim]
    layers x ( f32 in_norm[dim] | f32 post_norm[dim] | Wq Wk Wv Wo Wgate Wup Wdown )
    lm_head (tied token embedding)
    matrix = u32 out_dim, in_dim, num_blocks | u8 nibbles[num_blocks*64]
             | u16 step[num_blocks] | u16 min[num_blocks]          (bf16 bit patterns)

The 16-bit step and min fields are bf16 (the reference decodes them as ``bits << 16``,
src/llama_engine.cpp:28-33).
"""
from __future__ import annotations

import ctypes
import hashlib
import os
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from . import build as _build

MAGIC = b"LLM4S128"
MATRIX_NAMES = ("wq", "wk", "wv", "wo", "wg", "wu", "wd")


@dataclass(frozen=True)
class ModelShape:
    layers: int = 16
    dim: int = 2048
    ffn: int = 8192
    vocab: int = 128256
    heads: int = 32
    kv_heads: int = 8

    @property
    def head_dim(self) -> int:
        return self.dim // self.heads

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim

    def matrix_shapes(self) -> list[tuple[int, int]]:
        d, f, kv = self.dim, self.ffn, self.kv_dim
        return [(d, d), (kv, d), (kv, d), (d, d), (f, d), (f, d), (d, f)]

    def file_size(self) -> int:
        def mat(n, k):
            return 12 + n * (k // 128) * 68
        per_layer = 2 * self.dim * 4 + sum(mat(n, k) for n, k in self.matrix_shapes())
        return 8 + 28 + self.dim * 4 + self.layers * per_layer + mat(self.vocab, self.dim)

    def layer_matrix_params(self) -> int:
        """Weights of all layers' matrices (the per-token GEMM work of a forward is 2 flops each)."""
        return sum(n * k for n, k in self.matrix_shapes()) * self.layers

    def weight_bytes(self) -> int:
        """Bytes of all matrices (nibbles + step + min) and norms: streamed once per decode step."""
        mats = sum(n * (k // 128) * 68 for n, k in self.matrix_shapes()) * self.layers
        mats += self.vocab * (self.dim // 128) * 68
        norms = (2 * self.layers + 1) * self.dim * 4
        return mats + norms


LLAMA_3_2_1B = ModelShape()

_lib = None


def _gen_lib():
    global _lib
    if _lib is None:
        path = _build.build_generator()
        lib = ctypes.CDLL(str(path))
        lib.llm4s128_write_model.argtypes = [ctypes.c_char_p] + [ctypes.c_uint32] * 6 + [
            ctypes.c_uint64, ctypes.c_double, ctypes.c_int]
        lib.llm4s128_write_model.restype = ctypes.c_int
        lib.llm4s128_gen_matrix.argtypes = [ctypes.c_int, ctypes.c_double, ctypes.c_uint64,
                                            ctypes.c_uint64, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        lib.llm4s128_gen_matrix.restype = ctypes.c_int
        lib.llm4s128_quantize.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                          ctypes.c_void_p, ctypes.c_void_p]
        lib.llm4s128_quantize.restype = ctypes.c_int
        _lib = lib
    return _lib


def write_model(path: str | os.PathLike, shape: ModelShape = LLAMA_3_2_1B, seed: int = 0,
                sigma: float = 0.02, random_norms: bool = False) -> Path:
    """Writes a seeded random-init model: weights ~ N(0, sigma), affine block-128 quantised."""
    path = Path(path)
    rc = _gen_lib().llm4s128_write_model(str(path).encode(), shape.layers, shape.dim, shape.ffn,
                                         shape.vocab, shape.heads, shape.kv_heads, seed, sigma,
                                         1 if random_norms else 0)
    if rc != 0:
        raise RuntimeError(f"llm4s128_write_model failed ({rc}) for {path}")
    return path


def cached_model(directory: str | os.PathLike, shape: ModelShape = LLAMA_3_2_1B, seed: int = 0,
                 sigma: float = 0.02, random_norms: bool = False) -> Path:
    """Returns a model file under ``directory``, generating it once per (shape, seed, options)."""
    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    tag = (f"L{shape.layers}_d{shape.dim}_f{shape.ffn}_v{shape.vocab}_h{shape.heads}"
           f"_kv{shape.kv_heads}_s{seed}_sg{sigma:g}_n{int(random_norms)}")
    path = d / f"llm4s128_{tag}.bin"
    if not path.exists() or path.stat().st_size != shape.file_size():
        tmp = path.with_suffix(f".tmp{os.getpid()}")
        write_model(tmp, shape, seed, sigma, random_norms)
        tmp.replace(path)  # atomic: concurrent writers produce identical bytes
    return path


def gen_matrix(N: int, K: int, seed: int, tensor: int = 0, uniform_codes: bool = True,
               sigma: float = 0.02):
    """One quantised matrix.  uniform_codes: nibbles U{0..15}, step ~ U(1e-3, 2e-2),
    min = -8*step*U(0.8, 1.2) (the GEMV sweep distribution); else N(0, sigma) quantised."""
    nb = N * (K // 128)
    nib = np.empty(nb * 64, dtype=np.uint8)
    step = np.empty(nb, dtype=np.uint16)
    mn = np.empty(nb, dtype=np.uint16)
    rc = _gen_lib().llm4s128_gen_matrix(1 if uniform_codes else 0, sigma, seed, tensor, N, K,
                                        nib.ctypes.data, step.ctypes.data, mn.ctypes.data)
    if rc != 0:
        raise RuntimeError("llm4s128_gen_matrix failed")
    return nib, step, mn


def quantize(w: np.ndarray) -> dict:
    """Affine block-128 quantisation of an N x K fp32 matrix (K % 128 == 0): per block of 128
    weights of a row, min = block minimum and step = (max - min)/15, both rounded to bf16 (nearest
    even), q = clamp(rint((w - min)/step), 0, 15).  Returns the matrix record of the file
    ({"N", "K", "nib", "step", "min"})."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    if w.ndim != 2 or w.shape[1] % 128 != 0 or w.shape[0] == 0:
        raise ValueError(f"quantize: need an N x K matrix with K % 128 == 0, got {w.shape}")
    if not np.isfinite(w).all():
        raise ValueError("quantize: non-finite weights")
    N, K = w.shape
    nb = N * (K // 128)
    nib = np.empty(nb * 64, dtype=np.uint8)
    step = np.empty(nb, dtype=np.uint16)
    mn = np.empty(nb, dtype=np.uint16)
    if _gen_lib().llm4s128_quantize(w.ctypes.data, N, K, nib.ctypes.data, step.ctypes.data, mn.ctypes.data) != 0:
        raise RuntimeError("llm4s128_quantize failed")
    return {"N": N, "K": K, "nib": nib, "step": step, "min": mn}


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


class ModelFile:
    """Zero-copy numpy view of an ``LLM4S128`` file (for tests and tooling)."""

    def __init__(self, path: str | os.PathLike):
        self.path = Path(path)
        self.buf = np.memmap(self.path, dtype=np.uint8, mode="r")
        if bytes(self.buf[:8]) != MAGIC:
            raise ValueError("bad magic")
        h = self.buf[8:36].view(np.uint32)
        self.shape = ModelShape(int(h[0]), int(h[1]), int(h[2]), int(h[3]), int(h[4]), int(h[5]))
        self.block = int(h[6])
        off = 36
        d = self.shape.dim
        self.final_norm = self.buf[off:off + 4 * d].view(np.float32); off += 4 * d
        self.layers = []
        for _ in range(self.shape.layers):
            layer = {}
            layer["in_norm"] = self.buf[off:off + 4 * d].view(np.float32); off += 4 * d
            layer["post_norm"] = self.buf[off:off + 4 * d].view(np.float32); off += 4 * d
            for name in MATRIX_NAMES:
                layer[name], off = self._matrix(off)
            self.layers.append(layer)
        self.lm_head, off = self._matrix(off)
        self.end = off

    def _matrix(self, off):
        n, k, nb = (int(v) for v in self.buf[off:off + 12].view(np.uint32))
        off += 12
        nib = self.buf[off:off + nb * 64]; off += nb * 64
        step = self.buf[off:off + nb * 2].view(np.uint16); off += nb * 2
        mn = self.buf[off:off + nb * 2].view(np.uint16); off += nb * 2
        return {"N": n, "K": k, "nib": nib, "step": step, "min": mn}, off


def dequantize(m: dict) -> np.ndarray:
    """Dense fp32 copy of a quantised matrix (w = min + q*step), for small test shapes."""
    n, k = m["N"], m["K"]
    nib = np.asarray(m["nib"]).reshape(n, k // 2)
    q = np.empty((n, k), dtype=np.float32)
    q[:, 0::2] = nib & 0x0F
    q[:, 1::2] = nib >> 4
    st = np.repeat(bf16_to_f32(np.asarray(m["step"])).reshape(n, k // 128), 128, axis=1)
    mn = np.repeat(bf16_to_f32(np.asarray(m["min"])).reshape(n, k // 128), 128, axis=1)
    return mn + q * st


def file_sha256(path: str | os.PathLike) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            chunk = f.read(1 << 24)
            if not chunk:
                break
            h.update(chunk)
    return h.hexdigest()
