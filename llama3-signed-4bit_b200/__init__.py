"""B200-native (sm_100a) drop-in for the llama3-signed-4bit token loop.

The product is ``libllama_engine.so``: C++ host code and hand-written CUDA kernels behind the
reference's ``llama_engine.h`` C ABI (declared in ``include/llama_engine.h``).  This Python
package mirrors the reference's ctypes shell (src/main.py) on top of that library and holds the
build and weight-file tooling.

The directory name is not a Python identifier; import it as ``llama3_signed_4bit_b200`` through
``load_package()`` in ``__graft_entry__.py`` or the test suite's conftest.
"""
from . import build, convert, model_file, scoring, trace  # noqa: F401
from .engine import (  # noqa: F401
    LlamaEngine,
    LlamaEngineBindings,
    TokenizerWrapper,
    ensure_library_built,
    tp_unique_id,
)
