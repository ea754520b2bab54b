"""vvli_cuda_load_safetensors: weights from a safetensors file straight to the device.

A file written from the synthetic blob (BF16, the reference's own dtype) must
load bit-identically to vvli_cuda_load_weights of that blob; an F32 file must
give the blob of the reference's f32ToBf16 (src/llm.zig:799-803) of its
values; the errors follow copyTensorIntoWeight (src/llm.zig:1149-1183).
"""

import json
import os
import struct
import sys

import numpy as np
import pytest

from vvli_b200 import weights as Wt
from vvli_b200.errors import VvliError

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
