"""Producer and validator of the ``LLM4S128`` weight file.

The reference ships no converter (its README downloads a ready ``.bin``); this module closes the
loop from a Hugging Face Llama checkpoint (``*.safetensors`` + ``config.json``) to the file read
by ``llama_engine_create`` (layout: src/llama_engine.cpp:865-906 and 164-180 of the reference).

* ``read_safetensors`` — a dependency-free reader of the safetensors container (8-byte header
  length, JSON header of dtype / shape / data_offsets, raw little-endian data), memory-mapped;
  F32, F16 and BF16 tensors.
* ``convert`` — streams the tensors in file order, quantising each matrix with
  ``model_file.quantize`` (affine block-128, bf16 step and min).  Q and K projections are written
  as stored: the reference's RoPE rotates the pairs (i, i + head_dim/2) of each head
  (src/llama_engine.cpp:120-150), which is the layout of Hugging Face's q_proj / k_proj.  The
  lm_head slot holds the token embedding (the file ties them); an untied checkpoint is refused.
* ``validate`` — structural checks of a file (magic, geometry, every matrix header, exact size,
  finite scales and norms).

Command line::

    python llama3-signed-4bit_b200/convert.py convert <checkpoint dir> <out.bin>
    python llama3-signed-4bit_b200/convert.py validate <file.bin>
"""
from __future__ import annotations

import json
import os
import struct
import sys
import warnings
from pathlib import Path

import numpy as np

if __package__:
    from . import model_file as _mf
else:  # run as a script: load the package through the repository's entry module
    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
    import __graft_entry__

    _mf = __graft_entry__.load_package().model_file

# numerics fixed by the engines that read the file (src/llama_engine.cpp:909-916 and the RMSNorm eps)
ENGINE_ROPE_THETA = 500000.0
ENGINE_RMS_EPS = 1e-5

_DTYPES = {"F32": np.dtype("<f4"), "F16": np.dtype("<f2"), "BF16": np.dtype("<u2")}


class SafeTensors:
    """Tensors of one or more safetensors files, memory-mapped; ``get`` returns fp32."""

    def __init__(self, files: list[Path]):
        self._where: dict[str, tuple[np.memmap, dict, int]] = {}
        for f in files:
            raw = np.memmap(f, dtype=np.uint8, mode="r")
            if raw.size < 8:
                raise ValueError(f"{f}: not a safetensors file")
            (hlen,) = struct.unpack("<Q", bytes(raw[:8]))
            if 8 + hlen > raw.size:
                raise ValueError(f"{f}: header length {hlen} beyond the file")
            header = json.loads(bytes(raw[8:8 + hlen]).decode("utf-8"))
            for name, meta in header.items():
                if name == "__metadata__":
                    continue
                self._where[name] = (raw, meta, 8 + hlen)

    def names(self) -> list[str]:
        return sorted(self._where)

    def __contains__(self, name: str) -> bool:
        return name in self._where

    def shape(self, name: str) -> tuple[int, ...]:
        return tuple(int(d) for d in self._where[name][1]["shape"])

    def get(self, name: str) -> np.ndarray:
        raw, meta, base = self._where[name]
        dt = meta["dtype"]
        if dt not in _DTYPES:
            raise ValueError(f"{name}: unsupported dtype {dt}")
        b0, b1 = (int(v) for v in meta["data_offsets"])
        shape = tuple(int(d) for d in meta["shape"])
        count = int(np.prod(shape)) if shape else 1
        if b1 - b0 != count * _DTYPES[dt].itemsize or base + b1 > raw.size:
            raise ValueError(f"{name}: data_offsets do not match dtype and shape")
        a = raw[base + b0:base + b1].view(_DTYPES[dt]).reshape(shape)
        if dt == "BF16":
            return _mf.bf16_to_f32(a)
        return a.astype(np.float32)


def read_safetensors(path: str | os.PathLike) -> SafeTensors:
    """A checkpoint directory (all ``*.safetensors`` in it) or a single file."""
    p = Path(path)
    files = sorted(p.glob("*.safetensors")) if p.is_dir() else [p]
    if not files:
        raise FileNotFoundError(f"no .safetensors under {p}")
    return SafeTensors(files)


def _shape_from(st: SafeTensors, config: dict | None) -> "_mf.ModelShape":
    layers = 0
    while f"model.layers.{layers}.self_attn.q_proj.weight" in st:
        layers += 1
    vocab, dim = st.shape("model.embed_tokens.weight")
    ffn = st.shape("model.layers.0.mlp.gate_proj.weight")[0]
    q_rows = st.shape("model.layers.0.self_attn.q_proj.weight")[0]
    kv_rows = st.shape("model.layers.0.self_attn.k_proj.weight")[0]
    if config:
        heads = int(config["num_attention_heads"])
        kv_heads = int(config.get("num_key_value_heads", heads))
    else:  # head_dim 64, the only head size of the engines
        heads, kv_heads = q_rows // 64, kv_rows // 64
    if q_rows != dim or dim % heads or kv_rows != kv_heads * (dim // heads):
        raise ValueError(f"unsupported attention geometry: q rows {q_rows}, kv rows {kv_rows}, dim {dim}, "
                         f"heads {heads}/{kv_heads}")
    return _mf.ModelShape(layers=layers, dim=dim, ffn=ffn, vocab=vocab, heads=heads, kv_heads=kv_heads)


def _check_config(config: dict) -> list[str]:
    notes = []
    theta = float(config.get("rope_theta", ENGINE_ROPE_THETA))
    if theta != ENGINE_ROPE_THETA:
        notes.append(f"rope_theta {theta:g}: the engines use {ENGINE_ROPE_THETA:g}")
    eps = float(config.get("rms_norm_eps", ENGINE_RMS_EPS))
    if eps != ENGINE_RMS_EPS:
        notes.append(f"rms_norm_eps {eps:g}: the engines use {ENGINE_RMS_EPS:g}")
    if config.get("rope_scaling"):
        notes.append("rope_scaling is not applied by the engines (plain RoPE at every position)")
    hd = config.get("head_dim")
    if hd is not None and int(hd) != int(config["hidden_size"]) // int(config["num_attention_heads"]):
        notes.append(f"head_dim {hd} differs from hidden_size / num_attention_heads")
    return notes


def _write_norm(f, v: np.ndarray, dim: int, name: str) -> None:
    v = np.ascontiguousarray(v, dtype="<f4")
    if v.shape != (dim,) or not np.isfinite(v).all():
        raise ValueError(f"{name}: expected {dim} finite values")
    f.write(v.tobytes())


def _write_matrix(f, w: np.ndarray, n: int, k: int, name: str) -> None:
    if w.shape != (n, k):
        raise ValueError(f"{name}: shape {w.shape}, expected {(n, k)}")
    m = _mf.quantize(w)
    nb = n * (k // 128)
    f.write(struct.pack("<3I", n, k, nb))
    f.write(m["nib"].tobytes())
    f.write(m["step"].astype("<u2").tobytes())
    f.write(m["min"].astype("<u2").tobytes())


def convert(src: str | os.PathLike, out: str | os.PathLike, log=None) -> "_mf.ModelShape":
    """Writes ``out`` from a Hugging Face Llama checkpoint directory (or one safetensors file).
    Returns the geometry written.  Warnings list the config values the engines do not follow."""
    src = Path(src)
    st = read_safetensors(src)
    cfg_path = (src if src.is_dir() else src.parent) / "config.json"
    config = json.loads(cfg_path.read_text()) if cfg_path.exists() else None
    if config:
        for note in _check_config(config):
            warnings.warn(note)
    if "lm_head.weight" in st:
        emb, head = st.get("model.embed_tokens.weight"), st.get("lm_head.weight")
        if emb.shape != head.shape or not np.array_equal(emb, head):
            raise ValueError("untied lm_head: the LLM4S128 file holds one matrix for embedding and lm_head")
    shape = _shape_from(st, config)
    if (shape.heads, shape.kv_heads, shape.dim // shape.heads) != (32, 8, 64):
        warnings.warn(f"{shape.heads} query heads over {shape.kv_heads} kv heads: the reference engine's "
                      "attention is written for 32 over 8 heads of 64")
    d, F, kvd = shape.dim, shape.ffn, shape.kv_dim
    if d % 128 or F % 128:
        raise ValueError("dim and ffn must be multiples of 128")
    out = Path(out)
    tmp = out.with_name(out.name + f".tmp{os.getpid()}")
    try:
        with open(tmp, "wb") as f:
            f.write(_mf.MAGIC)
            f.write(struct.pack("<7I", shape.layers, d, F, shape.vocab, shape.heads, shape.kv_heads, 128))
            _write_norm(f, st.get("model.norm.weight"), d, "model.norm.weight")
            for layer in range(shape.layers):
                pre = f"model.layers.{layer}."
                _write_norm(f, st.get(pre + "input_layernorm.weight"), d, pre + "input_layernorm.weight")
                _write_norm(f, st.get(pre + "post_attention_layernorm.weight"), d,
                            pre + "post_attention_layernorm.weight")
                for suffix, n, k in (("self_attn.q_proj", d, d), ("self_attn.k_proj", kvd, d),
                                     ("self_attn.v_proj", kvd, d), ("self_attn.o_proj", d, d),
                                     ("mlp.gate_proj", F, d), ("mlp.up_proj", F, d), ("mlp.down_proj", d, F)):
                    _write_matrix(f, st.get(pre + suffix + ".weight"), n, k, pre + suffix)
                if log:
                    log(f"layer {layer + 1}/{shape.layers}")
            _write_matrix(f, st.get("model.embed_tokens.weight"), shape.vocab, d, "model.embed_tokens")
    except BaseException:
        tmp.unlink(missing_ok=True)
        raise
    tmp.replace(out)
    validate(out)
    return shape


def validate(path: str | os.PathLike) -> dict:
    """Structural check of an LLM4S128 file; raises ValueError naming the first problem.
    Returns {"shape", "bytes", "matrices", "max_step"}."""
    path = Path(path)
    size = path.stat().st_size
    if size < 36:
        raise ValueError("file shorter than its header")
    buf = np.memmap(path, dtype=np.uint8, mode="r")
    if bytes(buf[:8]) != _mf.MAGIC:
        raise ValueError("bad magic (expected LLM4S128)")
    L, d, F, V, H, KV, block = struct.unpack("<7I", bytes(buf[8:36]))
    if block != 128:
        raise ValueError(f"block size {block}, expected 128")
    if min(L, d, F, V, H, KV) == 0 or d % H or H % KV or d % 128 or F % 128:
        raise ValueError(f"inconsistent geometry L={L} dim={d} ffn={F} vocab={V} heads={H} kv_heads={KV}")
    shape = _mf.ModelShape(L, d, F, V, H, KV)
    if size != shape.file_size():
        raise ValueError(f"file has {size} bytes, the geometry needs {shape.file_size()}")
    off = 36
    max_step = 0.0

    def norm(name):
        nonlocal off
        v = buf[off:off + 4 * d].view("<f4")
        if not np.isfinite(v).all():
            raise ValueError(f"{name}: non-finite norm weights")
        off += 4 * d

    def matrix(name, n, k):
        nonlocal off, max_step
        hn, hk, nb = struct.unpack("<3I", bytes(buf[off:off + 12]))
        if (hn, hk, nb) != (n, k, n * (k // 128)):
            raise ValueError(f"{name}: header ({hn}, {hk}, {nb}), expected ({n}, {k}, {n * (k // 128)})")
        off += 12 + nb * 64
        st = _mf.bf16_to_f32(buf[off:off + 2 * nb].view("<u2")); off += 2 * nb
        mn = _mf.bf16_to_f32(buf[off:off + 2 * nb].view("<u2")); off += 2 * nb
        if not (np.isfinite(st).all() and np.isfinite(mn).all()):
            raise ValueError(f"{name}: non-finite step or min")
        if (st < 0).any():
            raise ValueError(f"{name}: negative step")
        max_step = max(max_step, float(st.max()))

    norm("final_norm")
    kvd = KV * (d // H)
    count = 0
    for layer in range(L):
        norm(f"layer {layer} in_norm")
        norm(f"layer {layer} post_norm")
        for nm, n, k in (("Wq", d, d), ("Wk", kvd, d), ("Wv", kvd, d), ("Wo", d, d), ("Wgate", F, d),
                         ("Wup", F, d), ("Wdown", d, F)):
            matrix(f"layer {layer} {nm}", n, k)
            count += 1
    matrix("lm_head", V, d)
    count += 1
    assert off == size
    return {"shape": shape, "bytes": size, "matrices": count, "max_step": max_step}


def main(argv: list[str] | None = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if len(argv) == 3 and argv[0] == "convert":
        shape = convert(argv[1], argv[2], log=lambda m: print(m, file=sys.stderr))
        print(f"wrote {argv[2]}: {shape}")
        return 0
    if len(argv) == 2 and argv[0] == "validate":
        rep = validate(argv[1])
        print(f"ok: {rep['shape']}, {rep['bytes']} bytes, {rep['matrices']} matrices, max step {rep['max_step']:g}")
        return 0
    print("usage:\n" + __doc__.split("Command line::")[1].rstrip(), file=sys.stderr)
    return 2


if __name__ == "__main__":
    sys.exit(main())
