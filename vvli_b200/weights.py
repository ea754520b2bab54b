"""Host-side weight blob utilities.

The bf16 blob layout is llm.OwnedModel's (src/llm.zig:415-537): the token
embedding, then per layer [input_norm, q, q_bias?, k, k_bias?, v, v_bias?, o,
post_attention_norm, gate, up, down], then the final norm and the untied LM
head, every tensor at a 64-byte aligned element offset.  ``load_safetensors``
follows loadSafetensorsIntoOwnedModel / copyTensorIntoWeight
(src/llm.zig:923-1006, 1149-1218): tensor names, BF16 copied as is, F32
rounded with f32ToBf16 (round to nearest even), any other dtype rejected.
``load_gguf`` does the same for a GGUF file (src/llm.zig:885-921,
1008-1138): GGUF tensor names, F32 / F16 / BF16 accepted.
"""

from __future__ import annotations

import json
import mmap
import struct

import numpy as np

from .config import Config
from .errors import VvliError

ALIGN = 32  # bf16 elements per 64-byte line


def tensor_entries(cfg: Config):
    """[(hf_name, element_offset, shape, kind)] in blob order; kind is 'mat', 'bias' or 'norm'."""
    h, kv, inter, V = cfg.hidden_size, cfg.kv_dim(), cfg.intermediate_size, cfg.vocab_size
    out = []
    cur = 0

    def take(name, shape, kind):
        nonlocal cur
        cur = (cur + ALIGN - 1) // ALIGN * ALIGN
        out.append((name, cur, shape, kind))
        cur += int(np.prod(shape))

    take("model.embed_tokens.weight", (V, h), "mat")
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        take(p + "input_layernorm.weight", (h,), "norm")
        take(p + "self_attn.q_proj.weight", (h, h), "mat")
        if cfg.qkv_bias:
            take(p + "self_attn.q_proj.bias", (h,), "bias")
        take(p + "self_attn.k_proj.weight", (kv, h), "mat")
        if cfg.qkv_bias:
            take(p + "self_attn.k_proj.bias", (kv,), "bias")
        take(p + "self_attn.v_proj.weight", (kv, h), "mat")
        if cfg.qkv_bias:
            take(p + "self_attn.v_proj.bias", (kv,), "bias")
        take(p + "self_attn.o_proj.weight", (h, h), "mat")
        take(p + "post_attention_layernorm.weight", (h,), "norm")
        take(p + "mlp.gate_proj.weight", (inter, h), "mat")
        take(p + "mlp.up_proj.weight", (inter, h), "mat")
        take(p + "mlp.down_proj.weight", (h, inter), "mat")
    take("model.norm.weight", (h,), "norm")
    if not cfg.tie_word_embeddings:
        take("lm_head.weight", (V, h), "mat")
    return out


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    """f32ToBf16 (src/llm.zig:799-803), vectorised: round to nearest even on the bits."""
    bits = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFFFFFF
    return (rounded >> 16).astype(np.uint16)


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(a, np.uint16).astype(np.uint32) << 16).view(np.float32)


def tensor_view(cfg: Config, blob: np.ndarray, name: str) -> np.ndarray:
    for n, off, shape, _ in tensor_entries(cfg):
        if n == name:
            return blob[off: off + int(np.prod(shape))].reshape(shape)
    raise KeyError(name)


def state_dict_f32(cfg: Config, blob: np.ndarray) -> dict:
    return {n: bf16_to_f32(blob[off: off + int(np.prod(s))]).reshape(s)
            for n, off, s, _ in tensor_entries(cfg)}


def _read_header(buf):
    if len(buf) < 8:
        raise VvliError("InvalidWeight")
    (hlen,) = struct.unpack("<Q", buf[:8])
    if 8 + hlen > len(buf):
        raise VvliError("InvalidWeight")
    header = json.loads(bytes(buf[8: 8 + hlen]))
    if not isinstance(header, dict):
        raise VvliError("InvalidWeight")
    return header, 8 + hlen


def _copy_tensor(blob: np.ndarray, off: int, shape, name: str, meta, data: memoryview) -> None:
    """copyTensorIntoWeight (src/llm.zig:1149-1183) into blob[off:]; views die with this frame."""
    if meta is None:
        raise VvliError("MissingSafetensorsTensor", -1, name)
    dtype = meta.get("dtype")
    if dtype not in ("BF16", "F32"):
        raise VvliError("UnsupportedDType", None, name)
    count = int(np.prod(meta.get("shape", [])))
    start, end = meta["data_offsets"]
    if count != int(np.prod(shape)) or end > len(data) or end < start:
        raise VvliError("InvalidWeight", None, name)
    raw = data[start:end]
    try:
        if dtype == "BF16":
            if len(raw) != count * 2:
                raise VvliError("InvalidWeight", None, name)
            blob[off: off + count] = np.frombuffer(raw, dtype="<u2")
        else:
            if len(raw) != count * 4:
                raise VvliError("InvalidWeight", None, name)
            blob[off: off + count] = f32_to_bf16(np.frombuffer(raw, dtype="<f4"))
    finally:
        raw.release()


def load_safetensors(path: str, cfg: Config) -> np.ndarray:
    """Reads model.safetensors into a new bf16 blob (loadSafetensorsIntoOwnedModel)."""
    blob = np.zeros(cfg.storage_element_count(), dtype=np.uint16)
    with open(path, "rb") as f:
        mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        try:
            header, data_start = _read_header(mm)
            data = memoryview(mm)[data_start:]
            try:
                for name, off, shape, _ in tensor_entries(cfg):
                    _copy_tensor(blob, off, shape, name, header.get(name), data)
            finally:
                data.release()
        finally:
            mm.close()
    return blob


_GGUF_LAYER_NAMES = {
    "input_layernorm.weight": "attn_norm.weight",
    "self_attn.q_proj.weight": "attn_q.weight",
    "self_attn.k_proj.weight": "attn_k.weight",
    "self_attn.v_proj.weight": "attn_v.weight",
    "self_attn.o_proj.weight": "attn_output.weight",
    "post_attention_layernorm.weight": "ffn_norm.weight",
    "mlp.gate_proj.weight": "ffn_gate.weight",
    "mlp.up_proj.weight": "ffn_up.weight",
    "mlp.down_proj.weight": "ffn_down.weight",
}


def gguf_tensor_name(hf_name: str) -> str:
    """The GGUF name loadGgufIntoOwnedModel (src/llm.zig:1008-1065) reads for a blob tensor."""
    if hf_name == "model.embed_tokens.weight":
        return "token_embd.weight"
    if hf_name == "model.norm.weight":
        return "output_norm.weight"
    if hf_name == "lm_head.weight":
        return "output.weight"
    _, _, layer, rest = hf_name.split(".", 3)
    return f"blk.{layer}.{_GGUF_LAYER_NAMES[rest]}"


def _copy_gguf_tensor(blob: np.ndarray, off: int, shape, name: str, file, data) -> None:
    """copyGgufTensorIntoWeight (src/llm.zig:1081-1138) into blob[off:]."""
    from . import gguf as G

    info = file.tensor(name)
    if info is None:
        raise VvliError("MissingSafetensorsTensor", -1, name)
    if info.tensor_type not in G.NATIVE_FLOAT:
        raise VvliError("UnsupportedDType", None, name)
    count = int(np.prod(shape))
    if info.element_count() != count:
        raise VvliError("InvalidWeight", None, name)
    esz = 4 if info.tensor_type == G.F32 else 2
    start = file.data_start + info.offset
    end = start + count * esz
    if end > len(data):
        raise VvliError("InvalidWeight", None, name)
    raw = data[start:end]
    try:
        if info.tensor_type == G.BF16:
            blob[off: off + count] = np.frombuffer(raw, dtype="<u2")
        elif info.tensor_type == G.F16:  # f32ToBf16(f16ToF32(bits)); the widening is exact
            blob[off: off + count] = f32_to_bf16(np.frombuffer(raw, dtype="<f2").astype(np.float32))
        else:
            blob[off: off + count] = f32_to_bf16(np.frombuffer(raw, dtype="<f4"))
    finally:
        raw.release()


def load_gguf(path: str):
    """(config, bf16 blob) of a GGUF file: loadOwnedFromGgufFile (src/llm.zig:885-921) with
    Config.fromGguf and loadGgufIntoOwnedModel (:153-193, 1008-1065)."""
    from . import gguf as G

    with open(path, "rb") as f:
        mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        try:
            data = memoryview(mm)
            try:
                file = G.parse(data)
                cfg = Config.from_gguf(file)
                if not cfg.supports_dense_runner() or cfg.qkv_bias:
                    raise VvliError("UnsupportedModelArchitecture")
                blob = np.zeros(cfg.storage_element_count(), dtype=np.uint16)
                for name, off, shape, _ in tensor_entries(cfg):
                    _copy_gguf_tensor(blob, off, shape, gguf_tensor_name(name), file, data)
                file.data = None
            finally:
                data.release()
        finally:
            mm.close()
    return cfg, blob


def save_safetensors(path: str, cfg: Config, blob: np.ndarray) -> None:
    """Writes the blob's tensors as a BF16 model.safetensors."""
    header, chunks, cur = {}, [], 0
    for name, off, shape, _ in tensor_entries(cfg):
        n = int(np.prod(shape))
        raw = np.ascontiguousarray(blob[off: off + n], dtype="<u2").tobytes()
        header[name] = {"dtype": "BF16", "shape": list(shape), "data_offsets": [cur, cur + len(raw)]}
        chunks.append(raw)
        cur += len(raw)
    hb = json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for c in chunks:
            f.write(c)
