"""GGUF on the host: the parser (vvli_b200.gguf, src/gguf.zig), Config.fromGguf,
the host loader (loadGgufIntoOwnedModel), and the oracle's interleaved RoPE
pinned against the transformers golden fixtures."""

import dataclasses
import os
import struct
import sys

import numpy as np
import pytest

from vvli_b200 import config as C
from vvli_b200 import gguf as G
from vvli_b200 import weights as Wt
from vvli_b200.errors import VvliError

from gguf_writer import gguf_bytes, gguf_cfg, interleave_qk, model_metadata, model_tensors, string, write_model

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))


def test_parses_gguf_metadata_and_tensor_table():
    # The reference's own parser test (src/gguf.zig:357-409), byte for byte.
    b = bytearray(b"GGUF" + struct.pack("<IQQ", 3, 1, 4))
    b += string("general.architecture") + struct.pack("<I", G.STRING) + string("llama")
    b += string("llama.block_count") + struct.pack("<II", G.UINT32, 16)
    b += string("general.alignment") + struct.pack("<II", G.UINT32, 32)
    b += string("tokenizer.ggml.tokens") + struct.pack("<IIQ", G.ARRAY, G.STRING, 2) + string("hello") + string("world")
    b += string("token_embd.weight") + struct.pack("<IQQIQ", 2, 4, 8, G.F32, 0)
    b += b"\0" * ((32 - len(b) % 32) % 32)
    f = G.parse(bytes(b))
    assert f.version == 3
    assert f.string("general.architecture") == "llama"
    assert f.usize_value("llama.block_count") == 16
    assert f.data_start % 32 == 0
    t = f.tensor("token_embd.weight")
    assert t.tensor_type == G.F32 and t.element_count() == 32
    assert f.string_array("tokenizer.ggml.tokens") == ["hello", "world"]


def _expect(data, name):
    with pytest.raises(VvliError) as e:
        G.parse(data)
    assert e.value.name == name


def test_parse_errors():
    good = gguf_bytes([("a", G.UINT32, 1)], [("t", (4,), G.F32, b"\0" * 16)])
    G.parse(good)
    _expect(b"GGUX" + good[4:], "InvalidGguf")
    _expect(good[:4] + struct.pack("<I", 1) + good[8:], "UnsupportedGgufVersion")
    _expect(good[:4] + struct.pack("<I", 4) + good[8:], "UnsupportedGgufVersion")
    _expect(good[:30], "InvalidGguf")  # cut short
    _expect(gguf_bytes([("a", G.UINT32, 1)], []).replace(struct.pack("<I", G.UINT32), struct.pack("<I", 13), 1),
            "UnsupportedMetadataType")
    _expect(b"GGUF" + struct.pack("<IQQ", 3, 1, 0) + string("t") + struct.pack("<I", 0), "InvalidGguf")  # 0 dims
    _expect(b"GGUF" + struct.pack("<IQQ", 3, 1, 0) + string("t") + struct.pack("<IQI", 1, 4, 5) + b"\0" * 8,
            "UnsupportedMetadataType")  # tensor type 5 is not a gguf.TensorType
    _expect(gguf_bytes([("general.alignment", G.UINT32, 0)], []), "InvalidGguf")
    _expect(b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + string("s") + struct.pack("<IQ", G.STRING, 1 << 40),
            "InvalidGguf")  # string longer than the file
    # metadata lookups: first entry wins; negative integers are no usize; f32 of integers
    f = G.parse(gguf_bytes([("k", G.INT32, -3), ("k", G.UINT32, 9), ("x", G.UINT16, 7), ("y", G.FLOAT64, 0.1)], []))
    assert f.usize_value("k") is None and f.f32_value("k") == -3.0
    assert f.f32_value("x") == 7.0 and f.f32_value("y") == np.float32(0.1)
    arr = G.parse(gguf_bytes([("v", G.ARRAY, (G.INT16, [1, -2, 3]))], []))
    assert arr.f32_array("v") == [1.0, -2.0, 3.0]


@pytest.mark.parametrize("tied", [True, False])
def test_config_from_gguf(tmp_path, tied):
    cfg = gguf_cfg(C.tiny_qwen())
    cfg.tie_word_embeddings = tied
    cfg.architecture = C.ARCH_LLAMA
    blob = np.random.default_rng(0).integers(0, 1 << 16, cfg.storage_element_count(), dtype=np.uint16)
    p = tmp_path / "m.gguf"
    write_model(str(p), cfg, blob)
    back = C.Config.from_gguf(G.parse(p.read_bytes()))
    assert back == cfg
    # optional keys fall back like Config.fromGguf: head_count_kv -> heads, theta 1e4, eps 1e-6
    md = [m for m in model_metadata(cfg) if not m[0].endswith(("head_count_kv", "freq_base", "rms_epsilon"))]
    f = G.parse(gguf_bytes(md, []))
    c2 = C.Config.from_gguf(f)
    assert c2.num_key_value_heads == cfg.num_attention_heads and c2.rope_theta == 10000.0
    assert c2.rms_norm_eps == C._f32(1e-6) and c2.tie_word_embeddings
    with pytest.raises(VvliError) as e:
        C.Config.from_gguf(G.parse(gguf_bytes([m for m in md if m[0] != "llama.block_count"], [])))
    assert e.value.name == "MissingJsonField"
    with pytest.raises(VvliError) as e:
        C.Config.from_gguf(G.parse(gguf_bytes([("general.architecture", G.STRING, "gpt2")] + md[1:], [])))
    assert e.value.name == "UnsupportedModelArchitecture"


def test_load_gguf_bf16_round_trip(tmp_path):
    cfg = gguf_cfg(C.tiny_qwen())
    blob = np.random.default_rng(1).integers(0, 1 << 16, cfg.storage_element_count(), dtype=np.uint16)
    p = str(tmp_path / "m.gguf")
    write_model(p, cfg, blob)
    cfg2, back = Wt.load_gguf(p)
    assert cfg2 == cfg
    for name, off, shape, _ in Wt.tensor_entries(cfg):
        n = int(np.prod(shape))
        assert np.array_equal(back[off:off + n], blob[off:off + n]), name


@pytest.mark.parametrize("ttype", [G.F32, G.F16])
def test_load_gguf_rounds_f32_and_f16(tmp_path, ttype):
    cfg = gguf_cfg(C.tiny_qwen())
    rng = np.random.default_rng(2)
    vals, want = {}, {}
    for name, off, shape, _ in Wt.tensor_entries(cfg):
        v = (rng.standard_normal(int(np.prod(shape))) * 0.05).astype(np.float32)
        v[:3] = [0.05 * (1 + 2.0 ** -8), -0.0, 6e-8]  # a bf16 tie, a signed zero, an f16 subnormal
        if ttype == G.F16:
            v = v.astype(np.float16).astype(np.float32)  # what the file holds, widened exactly
        vals[name] = v
        want[name] = Wt.f32_to_bf16(v)
    p = str(tmp_path / "m.gguf")
    write_model(p, cfg, None, ttype, vals)
    _, back = Wt.load_gguf(p)
    for name, off, shape, _ in Wt.tensor_entries(cfg):
        n = int(np.prod(shape))
        assert np.array_equal(back[off:off + n], want[name]), name


def test_load_gguf_errors(tmp_path):
    cfg = gguf_cfg(C.tiny_qwen())
    blob = np.zeros(cfg.storage_element_count(), np.uint16)
    md, ts = model_metadata(cfg), model_tensors(cfg, blob)

    def expect(md, ts, err):
        p = tmp_path / "bad.gguf"
        p.write_bytes(gguf_bytes(md, ts))
        with pytest.raises(VvliError) as e:
            Wt.load_gguf(str(p))
        assert e.value.name == err

    expect(md, [t for t in ts if t[0] != "blk.1.ffn_up.weight"], "MissingSafetensorsTensor")
    q8 = [(n, d, 8 if n == "blk.0.attn_k.weight" else t, r) for n, d, t, r in ts]
    expect(md, q8, "UnsupportedDType")
    short = [(n, (d[0] - 1,) + d[1:] if n == "output_norm.weight" else d, t, r) for n, d, t, r in ts]
    expect(md, short, "InvalidWeight")
    cut = gguf_bytes(md, ts)
    p = tmp_path / "cut.gguf"
    p.write_bytes(cut[:-2])  # the last tensor runs past the end of the file
    with pytest.raises(VvliError) as e:
        Wt.load_gguf(str(p))
    assert e.value.name == "InvalidWeight"
    olmoe = [("general.architecture", G.STRING, "olmoe")] + [(k.replace("qwen2.", "olmoe."), t, v) for k, t, v in md[1:]]
    expect(olmoe, ts, "UnsupportedModelArchitecture")


@pytest.mark.parametrize("name", ["qwen2_tiny", "llama3_tiny_rs"])
def test_oracle_interleaved_rope_matches_transformers(oracle, name):
    # GGUF files hold q/k rows in interleaved rotary order; interleaved RoPE on
    # those rows must reproduce the split-half (transformers) golden forward.
    from make_golden import fixture_configs
    cfg, seed = fixture_configs()[name]
    fx = np.load(os.path.join(HERE, "golden", f"{name}.npz"))
    blob = interleave_qk(cfg, oracle.synthetic_blob(cfg, seed=int(fx["seed"])))
    icfg = dataclasses.replace(cfg, rope_layout=C.ROPE_INTERLEAVED)
    r = oracle.RefRunner(icfg, blob=blob, max_seq=64, threads=2)
    for pos, tok in enumerate(fx["tokens"]):
        logits = r.forward_token(int(tok), pos)
        assert np.max(np.abs(logits - fx["logits"][pos])) < 2e-5, pos
    # and the split-half rule on the same rows does not
    r2 = oracle.RefRunner(cfg, blob=blob, max_seq=64, threads=2)
    worst = max(float(np.max(np.abs(r2.forward_token(int(t), p) - fx["logits"][p])))
                for p, t in enumerate(fx["tokens"][:6]))
    assert worst > 1e-4
