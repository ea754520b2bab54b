"""Host safetensors reader/writer (vvli_b200.weights): round trip, F32 rounding, errors."""

import json
import struct

import numpy as np
import pytest

from vvli_b200 import config as C
from vvli_b200 import weights as Wt
from vvli_b200.errors import VvliError


def ranges(cfg):
    return [(name, off, int(np.prod(shape))) for name, off, shape, _ in Wt.tensor_entries(cfg)]


def test_round_trip(tmp_path):
    cfg = C.tiny_qwen()
    blob = np.random.default_rng(0).integers(0, 65535, size=cfg.storage_element_count(), dtype=np.uint16)
    p = str(tmp_path / "m.safetensors")
    Wt.save_safetensors(p, cfg, blob)
    back = Wt.load_safetensors(p, cfg)
    for name, off, n in ranges(cfg):
        assert np.array_equal(blob[off:off + n], back[off:off + n]), name


def test_f32_tensors_round_to_nearest_even(tmp_path):
    cfg = C.tiny_qwen()
    header, chunks, cur, want = {}, [], 0, {}
    rng = np.random.default_rng(1)
    for name, off, n in ranges(cfg):
        v = rng.standard_normal(n).astype(np.float32)
        raw = v.astype("<f4").tobytes()
        header[name] = {"dtype": "F32", "shape": [n], "data_offsets": [cur, cur + len(raw)]}
        chunks.append(raw)
        cur += len(raw)
        want[name] = Wt.f32_to_bf16(v)
    hb = json.dumps(header).encode()
    p = tmp_path / "f32.safetensors"
    p.write_bytes(struct.pack("<Q", len(hb)) + hb + b"".join(chunks))
    back = Wt.load_safetensors(str(p), cfg)
    for name, off, n in ranges(cfg):
        assert np.array_equal(back[off:off + n], want[name]), name
    # f32ToBf16 ties go to even: 1 + 2^-8 -> 1.0, 1 + 3 * 2^-8 -> 1 + 2^-6
    assert Wt.f32_to_bf16(np.array([1.0 + 2.0 ** -8], np.float32))[0] == 0x3F80
    assert Wt.f32_to_bf16(np.array([1.0 + 3 * 2.0 ** -8], np.float32))[0] == 0x3F82


def test_missing_tensor(tmp_path):
    cfg = C.tiny_qwen()
    hb = json.dumps({"model.embed_tokens.weight": {"dtype": "BF16", "shape": [1], "data_offsets": [0, 2]}}).encode()
    p = tmp_path / "bad.safetensors"
    p.write_bytes(struct.pack("<Q", len(hb)) + hb + b"\0\0")
    with pytest.raises(VvliError) as e:
        Wt.load_safetensors(str(p), cfg)
    assert e.value.name in ("MissingSafetensorsTensor", "InvalidWeight")
