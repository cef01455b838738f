"""ctypes shell over ``libllama_engine.so``, mirroring the reference's src/main.py:27-228.

``LlamaEngineBindings``, ``TokenizerWrapper`` and ``LlamaEngine`` keep the reference's names,
argument meaning and error behaviour (RuntimeError when create returns NULL); the batched and
device-resident extensions of the B200 build are added as extra methods.  The library is the
CUDA build: there is no CPU path, and loading fails loudly if the library is missing or cannot
be built.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

from . import build as _build

LIB_PATH = _build.ENGINE_LIB

_P = ctypes.c_void_p
_I32P = ctypes.POINTER(ctypes.c_int32)
_FP = ctypes.POINTER(ctypes.c_float)


def ensure_library_built() -> Path:
    """Counterpart of ensure_dylib_built (src/main.py:27-46): builds the sm_100a library in-tree
    when a source is newer than it."""
    return _build.build_engine()


class LlamaEngineBindings:
    """Argtypes of src/main.py:57-140, plus the extensions declared in include/llama_engine.h."""

    def __init__(self, lib_path: Path | str | None = None):
        path = Path(lib_path) if lib_path else ensure_library_built()
        self.lib = lib = ctypes.CDLL(str(path))

        lib.llama_engine_create.argtypes = [ctypes.c_char_p]
        lib.llama_engine_create.restype = _P
        lib.llama_engine_free.argtypes = [_P]
        lib.llama_engine_free.restype = None
        lib.llama_engine_reset.argtypes = [_P]
        lib.llama_engine_reset.restype = None
        for name in ("num_layers", "dim", "ffn_dim", "vocab_size", "num_heads", "num_kv_heads",
                     "head_dim", "max_seq_len"):
            f = getattr(lib, "llama_engine_get_" + name)
            f.argtypes = [_P]
            f.restype = ctypes.c_int32
        lib.llama_engine_forward_token.argtypes = [_P, ctypes.c_int32, ctypes.c_size_t, ctypes.c_int]
        lib.llama_engine_forward_token.restype = ctypes.c_int
        lib.llama_engine_prefill.argtypes = [_P, _I32P, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_int]
        lib.llama_engine_prefill.restype = ctypes.c_int
        lib.llama_engine_sample.argtypes = [_P, ctypes.c_float, ctypes.c_float]
        lib.llama_engine_sample.restype = ctypes.c_int32
        lib.llama_engine_get_logits.argtypes = [_P]
        lib.llama_engine_get_logits.restype = _FP
        lib.llama_engine_dequantize_embedding.argtypes = [_P, ctypes.c_size_t, _FP]
        lib.llama_engine_dequantize_embedding.restype = None

        lib.llama_tokenizer_create.argtypes = [ctypes.c_char_p]
        lib.llama_tokenizer_create.restype = _P
        lib.llama_tokenizer_free.argtypes = [_P]
        lib.llama_tokenizer_free.restype = None
        lib.llama_tokenizer_encode.argtypes = [_P, ctypes.c_char_p, _I32P, ctypes.c_int]
        lib.llama_tokenizer_encode.restype = ctypes.c_int
        lib.llama_tokenizer_decode.argtypes = [_P, ctypes.c_int32]
        lib.llama_tokenizer_decode.restype = ctypes.c_char_p

        # extensions
        lib.llama_engine_create_ex.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        lib.llama_engine_create_ex.restype = _P
        lib.llama_engine_decode_path.argtypes = [_P]
        lib.llama_engine_decode_path.restype = ctypes.c_int
        lib.llama_engine_batch_path.argtypes = [_P]
        lib.llama_engine_batch_path.restype = ctypes.c_int
        lib.llama_engine_trace.argtypes = [_P, ctypes.c_int, ctypes.c_void_p, ctypes.c_int]
        lib.llama_engine_trace.restype = ctypes.c_int
        lib.llama_engine_get_stream.argtypes = [_P]
        lib.llama_engine_get_stream.restype = _P
        lib.llama_engine_profile_phase.argtypes = [_P, ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(ctypes.c_float)]
        lib.llama_engine_profile_phase.restype = ctypes.c_int
        lib.llama_engine_last_error.argtypes = [_P]
        lib.llama_engine_last_error.restype = ctypes.c_char_p
        lib.llama_engine_generate_greedy.argtypes = [_P, ctypes.c_int32, ctypes.c_size_t, ctypes.c_int32, _I32P]
        lib.llama_engine_generate_greedy.restype = ctypes.c_int
        lib.llama_engine_forward_batch.argtypes = [_P, _I32P, _I32P, _I32P, ctypes.c_int, ctypes.c_int]
        lib.llama_engine_forward_batch.restype = ctypes.c_int
        lib.llama_engine_argmax_batch.argtypes = [_P, _I32P, ctypes.c_int]
        lib.llama_engine_argmax_batch.restype = ctypes.c_int
        lib.llama_engine_get_logits_batch.argtypes = [_P, ctypes.c_int]
        lib.llama_engine_get_logits_batch.restype = _FP
        lib.llama_engine_score_tokens.argtypes = [_P, _I32P, ctypes.c_size_t, ctypes.c_size_t, _FP, _I32P]
        lib.llama_engine_score_tokens.restype = ctypes.c_int
        lib.llama_b128_gemv.argtypes = [_P, _P, _P, ctypes.c_int, ctypes.c_int, _P, ctypes.c_int, _P, _P]
        lib.llama_b128_gemv.restype = ctypes.c_int
        lib.llama_b128_gemm.argtypes = [_P, _P, _P, ctypes.c_int, ctypes.c_int, _P, ctypes.c_int, _P, _P]
        lib.llama_b128_gemm.restype = ctypes.c_int
        lib.llama_b128_gemm_plan.argtypes = [ctypes.c_int] * 5 + [_I32P]
        lib.llama_b128_gemm_plan.restype = ctypes.c_int
        lib.llama_b128_argmax_noalloc.argtypes = [_P, ctypes.c_int, _P, _P]
        lib.llama_b128_argmax_noalloc.restype = ctypes.c_int
        lib.llama_engine_set_rope_scaling.argtypes = [_P, ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_int]
        lib.llama_engine_set_rope_scaling.restype = ctypes.c_int
        lib.llama_engine_rope_table.argtypes = [ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_int,
                                                ctypes.c_int, _FP, _FP]
        lib.llama_engine_rope_table.restype = ctypes.c_int
        lib.llama_engine_tp_unique_id.argtypes = [_P, ctypes.c_int]
        lib.llama_engine_tp_unique_id.restype = ctypes.c_int
        lib.llama_engine_create_tp.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P,
                                               ctypes.c_int]
        lib.llama_engine_create_tp.restype = _P
        lib.llama_engine_check_schedule.argtypes = [ctypes.c_int] * 7 + [ctypes.c_char_p, ctypes.c_int]
        lib.llama_engine_check_schedule.restype = ctypes.c_int
        lib.llama_engine_debug_waits.argtypes = [_P, ctypes.c_ulonglong, ctypes.c_int]
        lib.llama_engine_debug_waits.restype = ctypes.c_int

    def last_error(self, handle=None) -> str:
        return self.lib.llama_engine_last_error(handle).decode(errors="replace")


def tp_unique_id(bindings: LlamaEngineBindings) -> bytes:
    """The NCCL unique id that rank 0 of a tensor-parallel pair makes and shares."""
    buf = ctypes.create_string_buffer(128)
    if bindings.lib.llama_engine_tp_unique_id(buf, 128) != 0:
        raise RuntimeError("NCCL unique id: NCCL could not be loaded")
    return buf.raw


class TokenizerWrapper:
    """Tokenizer: HF ``tokenizers`` when importable, else the library's BPE (src/main.py:143-185)."""

    def __init__(self, tokenizer_path: str, bindings: LlamaEngineBindings):
        self._hf_tok = None
        self._c_tok = None
        self._bindings = bindings
        try:
            from tokenizers import Tokenizer
            self._hf_tok = Tokenizer.from_file(tokenizer_path)
        except Exception:
            self._hf_tok = None
        if self._hf_tok is None:
            self._c_tok = bindings.lib.llama_tokenizer_create(tokenizer_path.encode("utf-8"))
            if not self._c_tok:
                raise RuntimeError(f"Failed to load tokenizer from {tokenizer_path}")

    def encode(self, text: str) -> list[int]:
        if self._hf_tok is not None:
            return self._hf_tok.encode(text, add_special_tokens=False).ids
        buf = (ctypes.c_int32 * 4096)()
        n = self._bindings.lib.llama_tokenizer_encode(self._c_tok, text.encode("utf-8"), buf, 4096)
        return [buf[i] for i in range(n)]

    def decode(self, token_id: int) -> str:
        if self._hf_tok is not None:
            return self._hf_tok.decode([token_id], skip_special_tokens=False)
        res = self._bindings.lib.llama_tokenizer_decode(self._c_tok, token_id)
        return res.decode("utf-8", errors="replace") if res else ""

    def __del__(self):
        if getattr(self, "_c_tok", None):
            self._bindings.lib.llama_tokenizer_free(self._c_tok)
            self._c_tok = None


class LlamaEngine:
    """Same surface as the reference's LlamaEngine (src/main.py:188-228), on the GPU.

    Extra keyword arguments select the device and the number of independent sequence slots
    (batched decode); the defaults reproduce ``llama_engine_create``.
    """

    def __init__(self, model_path: str, bindings: LlamaEngineBindings, device: int | None = None,
                 max_batch: int = 1, max_seq_len: int = 0, tp_rank: int | None = None, tp_world: int = 1,
                 tp_unique_id: bytes | None = None):
        self.bindings = bindings
        lib = bindings.lib
        if tp_rank is not None:  # 2-way tensor-parallel engine (llama_engine_create_tp)
            uid = ctypes.create_string_buffer(tp_unique_id, 128)
            self.handle = lib.llama_engine_create_tp(model_path.encode("utf-8"), device or 0, tp_rank, tp_world,
                                                     uid, max_seq_len)
        elif device is None and max_batch == 1 and max_seq_len == 0:
            self.handle = lib.llama_engine_create(model_path.encode("utf-8"))
        else:
            self.handle = lib.llama_engine_create_ex(model_path.encode("utf-8"), device or 0, max_batch,
                                                     max_seq_len)
        if not self.handle:
            raise RuntimeError(f"Failed to load model from {model_path}: {bindings.last_error(None)}")
        self.num_layers = lib.llama_engine_get_num_layers(self.handle)
        self.dim = lib.llama_engine_get_dim(self.handle)
        self.ffn_dim = lib.llama_engine_get_ffn_dim(self.handle)
        self.vocab_size = lib.llama_engine_get_vocab_size(self.handle)
        self.num_heads = lib.llama_engine_get_num_heads(self.handle)
        self.num_kv_heads = lib.llama_engine_get_num_kv_heads(self.handle)
        self.head_dim = lib.llama_engine_get_head_dim(self.handle)
        self.max_seq_len = lib.llama_engine_get_max_seq_len(self.handle)
        self.max_batch = max_batch

    def _check(self, rc: int, what: str) -> None:
        if rc != 0:
            raise RuntimeError(f"{what} failed: {self.bindings.last_error(self.handle)}")

    def reset(self):
        self.bindings.lib.llama_engine_reset(self.handle)

    def forward_token(self, token_id: int, pos: int, compute_logits: bool = True):
        self._check(self.bindings.lib.llama_engine_forward_token(self.handle, token_id, pos,
                                                                  1 if compute_logits else 0),
                    "forward_token")

    def prefill(self, tokens: list[int], start_pos: int, compute_last_logits: bool = False):
        if not tokens:
            return
        arr = (ctypes.c_int32 * len(tokens))(*tokens)
        self._check(self.bindings.lib.llama_engine_prefill(self.handle, arr, len(tokens), start_pos,
                                                           1 if compute_last_logits else 0),
                    "prefill")

    def sample(self, temperature: float = 0.0, top_p: float = 0.9) -> int:
        return self.bindings.lib.llama_engine_sample(self.handle, temperature, top_p)

    # ---- conveniences and extensions ----
    def get_logits(self) -> np.ndarray:
        ptr = self.bindings.lib.llama_engine_get_logits(self.handle)
        if not ptr:
            raise RuntimeError("get_logits failed")
        return np.ctypeslib.as_array(ptr, shape=(self.vocab_size,)).copy()

    def dequantize_embedding(self, token_id: int) -> np.ndarray:
        out = np.zeros(self.dim, dtype=np.float32)
        self.bindings.lib.llama_engine_dequantize_embedding(self.handle, token_id,
                                                            out.ctypes.data_as(_FP))
        return out

    def generate_greedy(self, first_token: int, start_pos: int, n_steps: int) -> list[int]:
        out = (ctypes.c_int32 * max(n_steps, 1))()
        self._check(self.bindings.lib.llama_engine_generate_greedy(self.handle, first_token, start_pos,
                                                                   n_steps, out), "generate_greedy")
        return list(out[:n_steps])

    def forward_batch(self, tokens, positions, slots, compute_logits: bool = True):
        n = len(tokens)
        t = (ctypes.c_int32 * n)(*tokens)
        p = (ctypes.c_int32 * n)(*positions)
        s = (ctypes.c_int32 * n)(*slots)
        self._check(self.bindings.lib.llama_engine_forward_batch(self.handle, t, p, s, n,
                                                                  1 if compute_logits else 0),
                    "forward_batch")

    def argmax_batch(self, n: int) -> list[int]:
        out = (ctypes.c_int32 * n)()
        self._check(self.bindings.lib.llama_engine_argmax_batch(self.handle, out, n), "argmax_batch")
        return list(out)

    def get_logits_batch(self, row: int) -> np.ndarray:
        ptr = self.bindings.lib.llama_engine_get_logits_batch(self.handle, row)
        if not ptr:
            raise RuntimeError("get_logits_batch failed")
        return np.ctypeslib.as_array(ptr, shape=(self.vocab_size,)).copy()

    def score_tokens(self, tokens, start_pos: int = 0) -> tuple[np.ndarray, np.ndarray]:
        """Log P(tokens[i+1] | tokens[..i]) for i < len(tokens)-1 and the per-position greedy
        flags, computed on the device (the scoring loop of the reference's
        tests/lm_eval_adapter.py:160-190 without a logits copy per token)."""
        n = len(tokens)
        t = (ctypes.c_int32 * n)(*tokens)
        lp = np.zeros(max(n - 1, 1), dtype=np.float32)
        gr = np.zeros(max(n - 1, 1), dtype=np.int32)
        self._check(self.bindings.lib.llama_engine_score_tokens(self.handle, t, n, start_pos,
                                                                lp.ctypes.data_as(_FP),
                                                                gr.ctypes.data_as(_I32P)),
                    "score_tokens")
        return lp[:n - 1], gr[:n - 1].astype(bool)

    def set_rope_scaling(self, factor: float = 32.0, low_freq_factor: float = 1.0, high_freq_factor: float = 4.0,
                         original_max_position: int = 8192) -> None:
        """Opt-in llama3 RoPE scaling (factor <= 0 restores the reference's unscaled table)."""
        self._check(self.bindings.lib.llama_engine_set_rope_scaling(self.handle, factor, low_freq_factor,
                                                                     high_freq_factor, original_max_position),
                    "set_rope_scaling")

    @property
    def decode_path(self) -> str:
        return {1: "persistent", 0: "kernel-chain", 2: "tensor-parallel"}.get(
            self.bindings.lib.llama_engine_decode_path(self.handle), "?")

    @property
    def batch_path(self) -> str:
        """Implementation of prefill and forward_batch: "tensor-core" or "token-loop"."""
        return {1: "tensor-core", 0: "token-loop"}.get(self.bindings.lib.llama_engine_batch_path(self.handle), "?")

    def close(self):
        if getattr(self, "handle", None):
            self.bindings.lib.llama_engine_free(self.handle)
            self.handle = None

    def __del__(self):
        self.close()
