"""Tokenizer parity (host code, no GPU): llama_tokenizer_* of this library against the reference's
own build (oracle/_ref, compiled from src/llama_engine.cpp), byte for byte, on a synthetic
tokenizer.json.

The file exercises the reference's reading rules (src/llama_engine.cpp:571-650): vocabulary
pieces with escaped quotes and backslashes (undone), \\u escapes and other backslash sequences
(kept as written), multi-byte UTF-8 pieces, merges that contain escaped characters (kept
verbatim), merges without a space (skipped), repeated merges (last rank wins).  The texts mix
runs of spaces, quotes, backslashes and 2-, 3- and 4-byte UTF-8 characters.
"""
from __future__ import annotations

import ctypes
import json

import numpy as np
import pytest


def _byte_table():
    printable = list(range(ord("!"), ord("~") + 1)) + list(range(161, 173)) + list(range(174, 256))
    table, extra = {}, 0
    for b in range(256):
        if b in printable:
            table[b] = chr(b)
        else:
            table[b] = chr(256 + extra)
            extra += 1
    return table


def _esc(s: str) -> str:
    return s.replace("\\", "\\\\").replace('"', '\\"')


def make_tokenizer_json(path, seed: int = 0, n_merges: int = 600) -> None:
    rng = np.random.default_rng(seed)
    table = _byte_table()
    vocab = {}
    for b in range(256):
        vocab.setdefault(table[b], len(vocab))
    words = ["hello", "world", "the", 'say"hi"', "back\\slash", "café", "中文", "naïve",
             "\U0001F600ok", "a\\nb", "x\\u00e9y", "quote\"s", "été"]
    pieces = [[table[b] for b in w.encode("utf-8")] for w in words]
    merges = []
    for _ in range(n_merges):
        w = pieces[rng.integers(len(pieces))]
        if len(w) < 2:
            continue
        i = int(rng.integers(len(w) - 1))
        a, b = w[i], w[i + 1]
        merges.append((a, b))
        w[i:i + 2] = [a + b]
        vocab.setdefault(a + b, len(vocab))
        if all(len(p) <= 1 for p in pieces):
            break
    # random pairs of base symbols too
    syms = [table[b] for b in range(256)]
    for _ in range(200):
        a, b = syms[rng.integers(256)], syms[rng.integers(256)]
        merges.append((a, b))
        vocab.setdefault(a + b, len(vocab))
    merges.append(merges[3])  # a repeated pair keeps its last rank
    lines = ['{', '  "version": "1.0",', '  "added_tokens": [{"id": 9, "content": "<|x|>"}],',
             '  "model": {', '    "type": "BPE",', '    "vocab": {']
    items = list(vocab.items())
    body = []
    for k, (piece, idx) in enumerate(items):
        if k % 37 == 5 and all(ord(c) < 0x100 for c in piece) and any(ord(c) >= 0x80 for c in piece):
            enc = "".join(f"\\u{ord(c):04x}" if ord(c) >= 0x80 else _esc(c) for c in piece)  # kept as written
        else:
            enc = _esc(piece)
        body.append(f'      "{enc}": {idx}')
    body.append(f'      "tab\\there": {len(vocab)}')      # \t kept as the two characters
    body.append(f'      "\\\\\\"": {len(vocab) + 1}')     # \\\" -> backslash, quote
    lines.append(",\n".join(body))
    lines.append('    },')
    lines.append('    "merges": [')
    mer = [f'      "{_esc(a)} {_esc(b)}"' for a, b in merges]
    mer.insert(5, '      "nospace"')
    mer.insert(9, '      "a \\" b"')
    lines.append(",\n".join(mer))
    lines.append('    ]')
    lines.append('  }')
    lines.append('}')
    path.write_text("\n".join(lines), encoding="utf-8")


def _texts(seed: int, n: int):
    rng = np.random.default_rng(seed)
    alphabet = (list("abcdehilnorstwxy") + [" ", " ", "  ", '"', "\\", "é", "ï", "中", "文",
                                            "\U0001F600", "\n", "\t", "hello", "world", "café", 'say"hi"',
                                            "back\\slash", "x\\u00e9y"])
    out = ["", " ", "   ", "hello world", 'say"hi" back\\slash', "café  中文 \U0001F600ok"]
    for _ in range(n):
        k = int(rng.integers(1, 24))
        out.append("".join(alphabet[int(i)] for i in rng.integers(len(alphabet), size=k)))
    return out


def _lib_tok(lib):
    lib.llama_tokenizer_create.argtypes = [ctypes.c_char_p]
    lib.llama_tokenizer_create.restype = ctypes.c_void_p
    lib.llama_tokenizer_free.argtypes = [ctypes.c_void_p]
    lib.llama_tokenizer_encode.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int32),
                                           ctypes.c_int]
    lib.llama_tokenizer_encode.restype = ctypes.c_int
    lib.llama_tokenizer_decode.argtypes = [ctypes.c_void_p, ctypes.c_int32]
    lib.llama_tokenizer_decode.restype = ctypes.c_char_p
    return lib


@pytest.fixture(scope="module")
def tok_json(tmp_path_factory):
    p = tmp_path_factory.mktemp("tok") / "tokenizer.json"
    make_tokenizer_json(p)
    json.loads(p.read_text(encoding="utf-8"))  # the synthetic file is valid JSON
    return p


def _encode(lib, h, text: str):
    buf = (ctypes.c_int32 * 4096)()
    n = lib.llama_tokenizer_encode(h, text.encode("utf-8"), buf, 4096)
    return list(buf[:n])


def test_tokenizer_matches_reference(pkg, ref_engine, tok_json):
    ours = _lib_tok(pkg.LlamaEngineBindings().lib)
    ref = _lib_tok(ref_engine)
    h_o = ours.llama_tokenizer_create(str(tok_json).encode())
    h_r = ref.llama_tokenizer_create(str(tok_json).encode())
    assert h_o and h_r
    try:
        n_merged = 0
        for text in _texts(1, 400):
            a, b = _encode(ours, h_o, text), _encode(ref, h_r, text)
            assert a == b, repr(text)
            n_merged += sum(1 for t in a if t >= 256)
        assert n_merged > 100  # the merges are exercised
        for i in list(range(0, 1200)) + [-1, 10 ** 6]:
            assert ours.llama_tokenizer_decode(h_o, i) == ref.llama_tokenizer_decode(h_r, i), i
        # max_tokens truncation and bad arguments behave the same
        buf = (ctypes.c_int32 * 3)()
        assert ours.llama_tokenizer_encode(h_o, b"hello world again", buf, 3) == \
            ref.llama_tokenizer_encode(h_r, b"hello world again", buf, 3)
        assert ours.llama_tokenizer_encode(h_o, None, buf, 3) == 0
        assert ours.llama_tokenizer_encode(h_o, b"x", buf, 0) == 0
        assert ours.llama_tokenizer_decode(None, 5) == b""
    finally:
        ours.llama_tokenizer_free(h_o)
        ref.llama_tokenizer_free(h_r)


def test_tokenizer_missing_file_and_sections(pkg, ref_engine, tmp_path):
    ours = _lib_tok(pkg.LlamaEngineBindings().lib)
    ref = _lib_tok(ref_engine)
    assert not ours.llama_tokenizer_create(str(tmp_path / "absent.json").encode())
    assert not ref.llama_tokenizer_create(str(tmp_path / "absent.json").encode())
    # compact JSON ("vocab":{ without the space): the reference reads no vocabulary and encodes
    # nothing; so does this library
    p = tmp_path / "compact.json"
    p.write_text(json.dumps({"model": {"vocab": {"a": 0, "b": 1}, "merges": ["a b"]}}, separators=(",", ":")))
    h_o = ours.llama_tokenizer_create(str(p).encode())
    h_r = ref.llama_tokenizer_create(str(p).encode())
    assert h_o and h_r
    assert _encode(ours, h_o, "ab a") == _encode(ref, h_r, "ab a") == []
    ours.llama_tokenizer_free(h_o)
    ref.llama_tokenizer_free(h_r)
