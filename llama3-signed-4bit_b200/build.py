"""In-tree build of the native libraries of this package.

* ``libllama_engine.so``  — the drop-in engine: C++ host code plus hand-written sm_100a CUDA
  kernels behind the ``llama_engine.h`` C ABI (``include/llama_engine.h``).
* ``libllm4s128.so``      — host-only seeded writer of ``LLM4S128`` weight files.

Both land next to this file so that they travel with the source tree.  Rebuilds happen only when
a source is newer than its output.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
ROOT = PKG_DIR.parent
INCLUDE = ROOT / "include"

ENGINE_LIB = PKG_DIR / "libllama_engine.so"
GEN_LIB = PKG_DIR / "libllm4s128.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA engine cannot be built")


def _stale(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")


def engine_sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("engine_*.cpp")) + sorted(CSRC.glob("tokenizer.cpp"))


def engine_deps() -> list[Path]:
    return engine_sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def build_engine(force: bool = False, verbose: bool = False) -> Path:
    deps = engine_deps()
    if not force and not _stale(ENGINE_LIB, deps + [Path(__file__)]):
        return ENGINE_LIB
    nvcc = _nvcc()
    objdir = PKG_DIR / "_build"
    objdir.mkdir(exist_ok=True)
    objs = []
    for src in engine_sources():
        obj = objdir / (src.name + ".o")
        if src.suffix == ".cu":
            cmd = [nvcc, *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
                   "-Xcompiler", "-fvisibility=hidden", f"-I{INCLUDE}", f"-I{CSRC}",
                   "--expt-relaxed-constexpr", "-c", str(src), "-o", str(obj)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
        else:
            cmd = ["g++", "-O3", "-std=c++17", "-fPIC", "-fvisibility=hidden", f"-I{INCLUDE}",
                   f"-I{CSRC}", "-I/usr/local/cuda/include", "-c", str(src), "-o", str(obj)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"build failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
        if verbose and res.stderr:
            sys.stderr.write(res.stderr)
        objs.append(str(obj))
    tmp = ENGINE_LIB.with_suffix(".so.tmp")
    _run([nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *objs, "-lcudart_static", "-lpthread",
          "-ldl", "-lrt"])
    tmp.replace(ENGINE_LIB)
    return ENGINE_LIB


def build_generator(force: bool = False) -> Path:
    src = CSRC / "llm4s128_gen.c"
    if force or _stale(GEN_LIB, [src]):
        tmp = GEN_LIB.with_suffix(".so.tmp")
        _run(["gcc", "-O2", "-std=c11", "-shared", "-fPIC", str(src), "-o", str(tmp), "-lpthread", "-lm"])
        tmp.replace(GEN_LIB)
    return GEN_LIB


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_generator(force)
    build_engine(force, verbose)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(ENGINE_LIB)
