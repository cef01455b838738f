"""The LLM4S128 producer: block quantiser against a numpy restatement (bit-exact), a tiny
Hugging Face style checkpoint converted, validated, read back and run through the oracle engine
against a float64 numpy Llama forward of the dequantised weights; validator failure cases."""
from __future__ import annotations

import ctypes
import json
import struct

import numpy as np
import pytest

from conftest import fptr

# 32 query heads over 8 kv heads of 64: the attention geometry the reference engine is written for
# (src/llama_engine.cpp:958-1021); small ffn and vocab keep the checkpoint near 50 MB.
TINY = dict(layers=2, dim=2048, ffn=256, vocab=512, heads=32, kv_heads=8)


def _bf16_rne(x: np.ndarray) -> np.ndarray:
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def _quantize_np(w: np.ndarray):
    """Restatement of the block rule: min = block min, step = (max-min)/15 (fp32), both bf16
    round-to-nearest-even; q = clamp(rint((w - min)/step), 0, 15); step 0 gives q = 0."""
    N, K = w.shape
    b = w.reshape(N, K // 128, 128)
    lo, hi = b.min(axis=2), b.max(axis=2)
    st = _bf16_rne((hi - lo) / np.float32(15.0))
    mn = _bf16_rne(lo)
    s = (st.astype(np.uint32) << 16).view(np.float32)[..., None]
    m = (mn.astype(np.uint32) << 16).view(np.float32)[..., None]
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(s > 0, np.clip(np.rint((b - m) / np.where(s > 0, s, 1)), 0, 15), 0).astype(np.uint8)
    q = q.reshape(N, K)
    nib = (q[:, 0::2] | (q[:, 1::2] << 4)).reshape(-1)
    return nib, st.reshape(-1), mn.reshape(-1)


def test_quantize_bit_exact_vs_numpy(pkg):
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((37, 512)) * 0.05).astype(np.float32)
    w[0, :128] = 0.25            # constant block: step 0
    w[1, 128:256] *= 1e4         # wide range
    w[2, 256:384] = -np.abs(w[2, 256:384])
    m = pkg.model_file.quantize(w)
    nib, st, mn = _quantize_np(w)
    assert np.array_equal(m["nib"], nib)
    assert np.array_equal(m["step"], st)
    assert np.array_equal(m["min"], mn)
    deq = pkg.model_file.dequantize(m)
    assert np.all(deq[0, :128] == np.float32(0.25))
    with pytest.raises(ValueError):
        pkg.model_file.quantize(np.zeros((4, 100), np.float32))
    bad = w.copy()
    bad[5, 7] = np.nan
    with pytest.raises(ValueError):
        pkg.model_file.quantize(bad)


def _write_safetensors(path, tensors: dict[str, np.ndarray]):
    header, blobs, off = {}, [], 0
    for name, a in tensors.items():
        raw = _bf16_rne(a).tobytes()
        header[name] = {"dtype": "BF16", "shape": list(a.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def _tiny_checkpoint(directory, seed=1, tied=True):
    s = TINY
    d, F, V, hd = s["dim"], s["ffn"], s["vocab"], s["dim"] // s["heads"]
    kvd = s["kv_heads"] * hd
    rng = np.random.default_rng(seed)
    t = {"model.embed_tokens.weight": rng.standard_normal((V, d)) * 0.5,
         "model.norm.weight": rng.uniform(0.8, 1.2, d)}
    for layer in range(s["layers"]):
        p = f"model.layers.{layer}."
        t[p + "input_layernorm.weight"] = rng.uniform(0.8, 1.2, d)
        t[p + "post_attention_layernorm.weight"] = rng.uniform(0.8, 1.2, d)
        for nm, n, k in (("self_attn.q_proj", d, d), ("self_attn.k_proj", kvd, d), ("self_attn.v_proj", kvd, d),
                         ("self_attn.o_proj", d, d), ("mlp.gate_proj", F, d), ("mlp.up_proj", F, d),
                         ("mlp.down_proj", d, F)):
            t[p + nm + ".weight"] = rng.standard_normal((n, k)) * 0.08
    if not tied:
        t["lm_head.weight"] = rng.standard_normal((V, d)) * 0.5
    t = {k: v.astype(np.float32) for k, v in t.items()}
    directory.mkdir(parents=True, exist_ok=True)
    _write_safetensors(directory / "model.safetensors", t)
    (directory / "config.json").write_text(json.dumps({
        "num_hidden_layers": s["layers"], "hidden_size": d, "intermediate_size": F, "vocab_size": V,
        "num_attention_heads": s["heads"], "num_key_value_heads": s["kv_heads"], "rope_theta": 500000.0,
        "rms_norm_eps": 1e-5, "tie_word_embeddings": tied}))
    return {k: (_bf16_rne(v).astype(np.uint32) << 16).view(np.float32) for k, v in t.items()}


def _llama_forward(mf, tokens):
    """float64 Llama forward over the dequantised weights (Hugging Face conventions: RMSNorm
    eps 1e-5, RoPE theta 500000 rotating (i, i + hd/2), GQA, SiLU MLP, tied lm_head)."""
    from_q = lambda m: mf_deq(m).astype(np.float64)  # noqa: E731
    s = mf.shape
    d, hd = s.dim, s.dim // s.heads
    group = s.heads // s.kv_heads
    emb = from_q(mf.lm_head)
    inv = 500000.0 ** (-np.arange(0, hd, 2) / hd)
    rms = lambda x, w: x / np.sqrt(np.mean(x * x) + 1e-5) * w  # noqa: E731

    def rope(v, pos):
        v = v.reshape(-1, hd)
        c, si = np.cos(pos * inv), np.sin(pos * inv)
        a, b = v[:, :hd // 2], v[:, hd // 2:]
        return np.concatenate([a * c - b * si, a * si + b * c], axis=1).reshape(-1)

    Ws = [{k: (from_q(v) if isinstance(v, dict) else np.asarray(v, np.float64)) for k, v in L.items()}
          for L in mf.layers]
    ks = [[] for _ in Ws]
    vs = [[] for _ in Ws]
    out = []
    for pos, tok in enumerate(tokens):
        x = emb[tok].copy()
        for li, W in enumerate(Ws):
            h = rms(x, W["in_norm"])
            q, k, v = rope(W["wq"] @ h, pos), rope(W["wk"] @ h, pos), W["wv"] @ h
            ks[li].append(k.reshape(s.kv_heads, hd))
            vs[li].append(v.reshape(s.kv_heads, hd))
            K, Vv = np.stack(ks[li]), np.stack(vs[li])
            att = np.empty(d)
            for hh in range(s.heads):
                sc = K[:, hh // group] @ q[hh * hd:(hh + 1) * hd] / np.sqrt(hd)
                p = np.exp(sc - sc.max())
                p /= p.sum()
                att[hh * hd:(hh + 1) * hd] = p @ Vv[:, hh // group]
            x = x + W["wo"] @ att
            h = rms(x, W["post_norm"])
            g, u = W["wg"] @ h, W["wu"] @ h
            x = x + W["wd"] @ (g / (1 + np.exp(-g)) * u)
        out.append(emb @ rms(x, np.asarray(mf.final_norm, np.float64)))
    return out


mf_deq = None


def test_convert_validate_and_run_on_oracle(pkg, tmp_path, oracle_lib):
    global mf_deq
    mf_deq = pkg.model_file.dequantize
    src = _tiny_checkpoint(tmp_path / "ckpt")
    out = tmp_path / "tiny.bin"
    shape = pkg.convert.convert(tmp_path / "ckpt", out)
    assert shape == pkg.model_file.ModelShape(**TINY)
    rep = pkg.convert.validate(out)
    assert rep["matrices"] == 7 * TINY["layers"] + 1 and rep["bytes"] == shape.file_size()

    mf = pkg.model_file.ModelFile(out)
    assert np.array_equal(mf.final_norm, src["model.norm.weight"])
    names = dict(wq="self_attn.q_proj", wk="self_attn.k_proj", wv="self_attn.v_proj", wo="self_attn.o_proj",
                 wg="mlp.gate_proj", wu="mlp.up_proj", wd="mlp.down_proj")
    for li, L in enumerate(mf.layers):
        p = f"model.layers.{li}."
        assert np.array_equal(L["in_norm"], src[p + "input_layernorm.weight"])
        assert np.array_equal(L["post_norm"], src[p + "post_attention_layernorm.weight"])
        for key, nm in names.items():
            w = src[p + nm + ".weight"]
            deq = pkg.model_file.dequantize(L[key])
            st = np.repeat(pkg.model_file.bf16_to_f32(np.asarray(L[key]["step"])).reshape(w.shape[0], -1), 128, 1)
            # half a step, plus the bf16 rounding of min and step (at most 16 steps' worth of 2^-8)
            assert np.all(np.abs(deq - w) <= 0.5 * st + 2.0 ** -8 * (np.abs(w).max() + 16 * st)), (li, key)
    emb = pkg.model_file.dequantize(mf.lm_head)
    assert np.abs(emb - src["model.embed_tokens.weight"]).max() < 0.2

    tokens = [5, 77, 300, 2]
    ref = _llama_forward(mf, tokens)
    o = oracle_lib.orc_create(str(out).encode())
    assert o
    try:
        for pos, tok in enumerate(tokens):
            oracle_lib.orc_forward_token(o, tok, pos, 1)
            lg = np.ctypeslib.as_array(oracle_lib.orc_get_logits(o), shape=(TINY["vocab"],))
            err = np.abs(lg - ref[pos]).max() / np.abs(ref[pos]).max()
            assert err < 1e-4, (pos, err)
    finally:
        oracle_lib.orc_free(o)


def test_convert_refuses_untied_head(pkg, tmp_path):
    _tiny_checkpoint(tmp_path / "ckpt", tied=False)
    with pytest.raises(ValueError, match="untied"):
        pkg.convert.convert(tmp_path / "ckpt", tmp_path / "x.bin")
    assert not (tmp_path / "x.bin").exists()


def test_convert_warns_on_config_the_engines_ignore(pkg, tmp_path):
    _tiny_checkpoint(tmp_path / "ckpt")
    cfg = json.loads((tmp_path / "ckpt" / "config.json").read_text())
    cfg["rope_scaling"] = {"rope_type": "llama3", "factor": 32.0}
    cfg["rope_theta"] = 10000.0
    (tmp_path / "ckpt" / "config.json").write_text(json.dumps(cfg))
    with pytest.warns(UserWarning) as rec:
        pkg.convert.convert(tmp_path / "ckpt", tmp_path / "x.bin")
    msgs = " ".join(str(r.message) for r in rec)
    assert "rope_scaling" in msgs and "rope_theta" in msgs


def test_validate_rejects_damaged_files(pkg, small_model, tmp_path):
    good = small_model.read_bytes()
    assert pkg.convert.validate(small_model)["shape"] == pkg.model_file.ModelFile(small_model).shape
    cases = {
        "magic": b"LLM4S129" + good[8:],
        "size": good[:-1],
        "block": good[:32] + struct.pack("<I", 64) + good[36:],
    }
    # first matrix header (Wq of layer 0) claims one row fewer
    d = struct.unpack("<I", good[12:16])[0]
    off = 36 + 4 * d * 3
    cases["header"] = good[:off] + struct.pack("<I", d - 1) + good[off + 4:]
    for why, blob in cases.items():
        p = tmp_path / f"{why}.bin"
        p.write_bytes(blob)
        with pytest.raises(ValueError):
            pkg.convert.validate(p)


def test_cli(pkg, tmp_path, capsys):
    _tiny_checkpoint(tmp_path / "ckpt")
    assert pkg.convert.main(["convert", str(tmp_path / "ckpt"), str(tmp_path / "m.bin")]) == 0
    assert pkg.convert.main(["validate", str(tmp_path / "m.bin")]) == 0
    assert "ok:" in capsys.readouterr().out
    assert pkg.convert.main(["bogus"]) == 2
