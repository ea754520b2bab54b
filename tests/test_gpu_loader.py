"""vvli_cuda_load_safetensors / vvli_cuda_load_gguf: weights from a file straight to the device.

A file written from the synthetic blob (BF16, the reference's own dtype) must
load bit-identically to vvli_cuda_load_weights of that blob; an F32 (or, for
GGUF, F16) file must give the blob of the reference's f32ToBf16
(src/llm.zig:795-803) of its values; the errors follow copyTensorIntoWeight
(src/llm.zig:1149-1183) and copyGgufTensorIntoWeight / gguf.parse
(src/llm.zig:1081-1138, src/gguf.zig:234-287).  GGUF models run interleaved
RoPE (Config.fromGguf, src/llm.zig:182) and are checked against the oracle.
"""

import dataclasses
import json
import os
import struct
import sys

import numpy as np
import pytest

from vvli_b200 import config as C
from vvli_b200 import gguf as G
from vvli_b200 import weights as Wt
from vvli_b200.errors import VvliError

from gguf_writer import gguf_bytes, gguf_cfg, model_metadata, model_tensors, write_model

pytestmark = pytest.mark.gpu

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))


@pytest.fixture(scope="module")
def vv():
    import vvli_b200
    return vvli_b200


def write_file(path, tensors):
    """tensors: name -> (dtype string, shape, raw bytes)."""
    header, chunks, cur = {}, [], 0
    for name, (dt, shape, raw) in tensors.items():
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [cur, cur + len(raw)]}
        chunks.append(raw)
        cur += len(raw)
    header["__metadata__"] = {"format": "pt"}
    hb = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for c in chunks:
            f.write(c)


def bf16_tensors(cfg, blob):
    out = {}
    for name, off, shape, _ in Wt.tensor_entries(cfg):
        n = int(np.prod(shape))
        out[name] = ("BF16", shape, np.ascontiguousarray(blob[off: off + n], dtype="<u2").tobytes())
    return out


def logits_of(gpu, toks):
    return np.stack([gpu.forward_token(t, p) for p, t in enumerate(toks)])


@pytest.mark.parametrize("name", ["qwen2_tiny", "llama3_tiny_rs"])
def test_bf16_file_equals_blob_load(oracle, vv, tmp_path, name):
    from make_golden import fixture_configs
    cfg, seed = fixture_configs()[name]
    blob = oracle.synthetic_blob(cfg, seed=seed)
    path = str(tmp_path / "model.safetensors")
    write_file(path, bf16_tensors(cfg, blob))
    a = vv.Runner(cfg, max_seq=32)
    a.load_weights(blob)
    b = vv.Runner(cfg, max_seq=32)
    b.load_safetensors(path)
    toks = [3, 44, 101, 7]
    assert np.array_equal(logits_of(a, toks), logits_of(b, toks))


def test_f32_file_rounds_like_the_reference(oracle, vv, tmp_path):
    from make_golden import fixture_configs
    cfg, seed = fixture_configs()["llama3_tiny_rs"]
    rng = np.random.default_rng(3)
    blob = np.zeros(cfg.storage_element_count(), dtype=np.uint16)
    tensors = {}
    for name, off, shape, _ in Wt.tensor_entries(cfg):
        n = int(np.prod(shape))
        v = (rng.standard_normal(n) * 0.05).astype(np.float32)  # most values are not bf16: they get rounded
        # round-to-even ties (down and up), a signed zero and a subnormal
        v[: min(n, 4)] = np.array([0.05 * (1.0 + 2.0 ** -8), 0.05 * (1.0 + 3 * 2.0 ** -8), -0.0, 1e-40],
                                  np.float32)[: min(n, 4)]
        blob[off: off + n] = Wt.f32_to_bf16(v)
        tensors[name] = ("F32", shape, v.astype("<f4").tobytes())
    path = str(tmp_path / "model_f32.safetensors")
    write_file(path, tensors)
    a = vv.Runner(cfg, max_seq=32)
    a.load_weights(blob)
    b = vv.Runner(cfg, max_seq=32)
    b.load_safetensors(path)
    toks = [5, 9, 200]
    assert np.array_equal(logits_of(a, toks), logits_of(b, toks))


def test_loader_errors(oracle, vv, tmp_path):
    from make_golden import fixture_configs
    cfg, seed = fixture_configs()["qwen2_tiny"]
    blob = oracle.synthetic_blob(cfg, seed=seed)
    gpu = vv.Runner(cfg, max_seq=8)
    good = bf16_tensors(cfg, blob)

    def expect(tensors, err, fname):
        p = str(tmp_path / fname)
        write_file(p, tensors)
        with pytest.raises(VvliError) as e:
            gpu.load_safetensors(p)
        assert e.value.name == err, e.value

    missing = dict(good)
    missing.pop("model.layers.1.mlp.down_proj.weight")
    expect(missing, "MissingSafetensorsTensor", "missing.safetensors")
    f16 = dict(good)
    dt, shape, raw = f16["model.norm.weight"]
    f16["model.norm.weight"] = ("F16", shape, raw)
    expect(f16, "UnsupportedDType", "f16.safetensors")
    bad = dict(good)
    dt, shape, raw = bad["model.layers.0.self_attn.k_proj.weight"]
    bad["model.layers.0.self_attn.k_proj.weight"] = (dt, [shape[0] - 1, shape[1]], raw[: (shape[0] - 1) * shape[1] * 2])
    expect(bad, "InvalidWeight", "shape.safetensors")
    with pytest.raises(VvliError) as e:
        gpu.load_safetensors(str(tmp_path / "does_not_exist.safetensors"))
    assert e.value.name == "InvalidArgument"
    # still usable: a good file loads afterwards
    p = str(tmp_path / "good.safetensors")
    write_file(p, good)
    gpu.load_safetensors(p)
    assert gpu.forward_token(1, 0).shape == (cfg.vocab_size,)


LOGIT_MAX_ABS = 2e-2
TIGHT = 1e-4          # fp32 vs fp32, different summation order


@pytest.mark.parametrize("name", ["qwen2_tiny", "llama3_tiny_rs"])
def test_gguf_file_matches_blob_load_and_oracle(oracle, vv, tmp_path, name):
    from make_golden import fixture_configs
    cfg0, seed = fixture_configs()[name]
    cfg = gguf_cfg(cfg0)
    blob = oracle.synthetic_blob(cfg, seed=seed)
    path = str(tmp_path / "model.gguf")
    write_model(path, cfg, blob)
    with open(path, "rb") as f:
        fcfg = C.Config.from_gguf(G.parse(f.read()))
    assert fcfg == cfg
    g = vv.Runner(fcfg, max_seq=64)
    g.load_gguf(path)
    a = vv.Runner(cfg, max_seq=64)
    a.load_weights(blob)
    ref = oracle.RefRunner(cfg, blob=blob, max_seq=64, threads=2)
    toks = [3, 44, 101, 7, 200, 9]
    lg = logits_of(g, toks)
    assert np.array_equal(lg, logits_of(a, toks))
    for pos, t in enumerate(toks):
        lr = ref.forward_token(t, pos)
        assert np.max(np.abs(lg[pos] - lr)) < LOGIT_MAX_ABS, pos
        assert np.linalg.norm(lg[pos] - lr) < TIGHT * np.linalg.norm(lr), pos
    # identical greedy streams over 32 tokens
    g.reset()
    ref.reset()
    assert g.generate_greedy([5, 17, 99], 32)[0] == ref.generate_greedy([5, 17, 99], 32)


@pytest.mark.parametrize("ttype", [G.F32, G.F16])
def test_gguf_float_files_round_like_the_reference(vv, tmp_path, ttype):
    cfg = gguf_cfg(C.tiny_qwen())
    rng = np.random.default_rng(4)
    vals = {}
    for name, off, shape, _ in Wt.tensor_entries(cfg):
        v = (rng.standard_normal(int(np.prod(shape))) * 0.05).astype(np.float32)
        v[:3] = [0.05 * (1 + 2.0 ** -8), -0.0, 6e-8]
        vals[name] = v
    path = str(tmp_path / "model.gguf")
    write_model(path, cfg, None, ttype, vals)
    _, blob = Wt.load_gguf(path)  # the host restatement of copyGgufTensorIntoWeight
    a = vv.Runner(cfg, max_seq=16)
    a.load_weights(blob)
    b = vv.Runner(cfg, max_seq=16)
    b.load_gguf(path)
    toks = [5, 9, 20, 3]
    assert np.array_equal(logits_of(a, toks), logits_of(b, toks))


def test_interleaved_rope_tensor_core_prefill_and_decode(oracle, vv):
    # A GGUF-style config large enough for the tensor-core prefill (d = 64, GQA 4:1).
    cfg = C.Config(vocab_size=2048, hidden_size=512, intermediate_size=1536, num_hidden_layers=2,
                   num_attention_heads=8, num_key_value_heads=2, max_position_embeddings=1024,
                   rope_theta=10000.0, rms_norm_eps=C._f32(1e-5), tie_word_embeddings=False,
                   architecture=C.ARCH_LLAMA, qkv_bias=False, rope_layout=C.ROPE_INTERLEAVED)
    prompt = np.random.default_rng(6).integers(0, cfg.vocab_size, size=200).tolist()
    ref = oracle.RefRunner(cfg, synthetic_seed=0, max_seq=256, threads=2)
    gpu = vv.Runner(cfg, max_seq=256)
    gpu.fill_synthetic(0)
    assert gpu.query("tc_prefill") == 1
    for pos, t in enumerate(prompt):
        lr = ref.forward_token(t, pos)
    lg = gpu.prefill(prompt, 0)
    assert np.max(np.abs(lg - lr)) < LOGIT_MAX_ABS
    ref_tokens, tok = [], oracle.argmax(lr)
    assert gpu.last_argmax == tok
    for pos in range(len(prompt), len(prompt) + 16):
        ref_tokens.append(tok)
        tok = oracle.argmax(ref.forward_token(tok, pos))
    got, _ = gpu.decode(16)
    assert got[:15] == ref_tokens[1:16]


def test_gguf_errors(oracle, vv, tmp_path):
    cfg = gguf_cfg(C.tiny_qwen())
    blob = oracle.synthetic_blob(cfg, seed=1)
    md, ts = model_metadata(cfg), model_tensors(cfg, blob)
    gpu = vv.Runner(cfg, max_seq=8)

    def expect(data, err, runner=gpu):
        p = tmp_path / "bad.gguf"
        p.write_bytes(data)
        with pytest.raises(VvliError) as e:
            runner.load_gguf(str(p))
        assert e.value.name == err, e.value

    good = gguf_bytes(md, ts)
    expect(b"GGUX" + good[4:], "InvalidGguf")
    expect(good[:4] + struct.pack("<I", 1) + good[8:], "UnsupportedGgufVersion")
    expect(good[:200], "InvalidGguf")
    expect(gguf_bytes(md, [t for t in ts if t[0] != "blk.1.ffn_down.weight"]), "MissingSafetensorsTensor")
    expect(gguf_bytes(md, [(n, d, 12 if n == "blk.0.attn_q.weight" else t, r) for n, d, t, r in ts]),
           "UnsupportedDType")
    expect(gguf_bytes(md, [(n, (d[0] - 1,) if n == "output_norm.weight" else d, t, r) for n, d, t, r in ts]),
           "InvalidWeight")
    expect(good[:-2], "InvalidWeight")
    split = vv.Runner(dataclasses.replace(cfg, rope_layout=C.ROPE_SPLIT_HALF), max_seq=8)
    expect(good, "InvalidConfig", split)
    biased = vv.Runner(dataclasses.replace(cfg, qkv_bias=True), max_seq=8)
    expect(good, "UnsupportedModelArchitecture", biased)
    with pytest.raises(VvliError) as e:
        gpu.load_gguf(str(tmp_path / "does_not_exist.gguf"))
    assert e.value.name == "InvalidArgument"
    p = tmp_path / "good.gguf"
    p.write_bytes(good)
    gpu.load_gguf(str(p))
    assert gpu.forward_token(1, 0).shape == (cfg.vocab_size,)
