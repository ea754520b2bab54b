"""Writes GGUF files for the tests (the reference builds its parse fixture the
same way, src/gguf.zig:357-422: little-endian ints, u64-length strings)."""

import dataclasses
import struct

import numpy as np

from vvli_b200 import config as C
from vvli_b200 import gguf as G
from vvli_b200 import weights as Wt
from vvli_b200.config import ARCH_NAMES

_FMT = {G.UINT8: "<B", G.INT8: "<b", G.UINT16: "<H", G.INT16: "<h", G.UINT32: "<I", G.INT32: "<i",
        G.FLOAT32: "<f", G.BOOL: "<B", G.UINT64: "<Q", G.INT64: "<q", G.FLOAT64: "<d"}


def string(s) -> bytes:
    b = s.encode() if isinstance(s, str) else s
    return struct.pack("<Q", len(b)) + b


def value(t: int, v) -> bytes:
    if t == G.STRING:
        return string(v)
    if t == G.ARRAY:
        item_type, items = v
        return struct.pack("<IQ", item_type, len(items)) + b"".join(value(item_type, x) for x in items)
    return struct.pack(_FMT[t], v)


def gguf_bytes(metadata, tensors, version=3, alignment=32) -> bytes:
    """metadata: [(key, type, value)]; tensors: [(name, dims, type, raw bytes)], laid out in order
    at `alignment`-aligned offsets of the data section."""
    out = bytearray(b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(metadata)))
    for k, t, v in metadata:
        out += string(k) + struct.pack("<I", t) + value(t, v)
    offsets, cur = [], 0
    for _, _, _, raw in tensors:
        cur = (cur + alignment - 1) // alignment * alignment
        offsets.append(cur)
        cur += len(raw)
    for (name, dims, t, _), off in zip(tensors, offsets):
        out += string(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", t, off)
    out += b"\0" * ((alignment - len(out) % alignment) % alignment)
    base = len(out)
    for (_, _, _, raw), off in zip(tensors, offsets):
        out += b"\0" * (base + off - len(out)) + raw
    return bytes(out)


def model_metadata(cfg, vocab_tokens=None):
    """The keys Config.fromGguf reads (src/llm.zig:153-193) for `cfg`."""
    arch = {v: k for k, v in ARCH_NAMES.items()}[cfg.architecture]
    tokens = vocab_tokens if vocab_tokens is not None else [f"t{i}" for i in range(cfg.vocab_size)]
    return [
        ("general.architecture", G.STRING, arch),
        (f"{arch}.block_count", G.UINT32, cfg.num_hidden_layers),
        (f"{arch}.context_length", G.UINT32, cfg.max_position_embeddings),
        (f"{arch}.embedding_length", G.UINT32, cfg.hidden_size),
        (f"{arch}.feed_forward_length", G.UINT32, cfg.intermediate_size),
        (f"{arch}.attention.head_count", G.UINT32, cfg.num_attention_heads),
        (f"{arch}.attention.head_count_kv", G.UINT32, cfg.num_key_value_heads),
        (f"{arch}.rope.freq_base", G.FLOAT32, cfg.rope_theta),
        (f"{arch}.attention.layer_norm_rms_epsilon", G.FLOAT32, cfg.rms_norm_eps),
        ("general.alignment", G.UINT32, 32),
        ("tokenizer.ggml.tokens", G.ARRAY, (G.STRING, tokens)),
        ("tokenizer.ggml.eos_token_id", G.UINT32, cfg.eos_token_id),
        ("tokenizer.ggml.padding_token_id", G.UINT32, cfg.pad_token_id),
    ]


def model_tensors(cfg, blob, tensor_type=G.BF16, values_f32=None):
    """The model's tensors under their GGUF names, dims innermost first.  BF16 takes the blob's
    bits; F32 / F16 take values_f32[name] (float32 arrays) when given, else the blob's values."""
    out = []
    for name, off, shape, _ in Wt.tensor_entries(cfg):
        n = int(np.prod(shape))
        if tensor_type == G.BF16:
            raw = np.ascontiguousarray(blob[off: off + n], dtype="<u2").tobytes()
        else:
            v = values_f32[name] if values_f32 is not None else Wt.bf16_to_f32(blob[off: off + n])
            raw = np.asarray(v, "<f4" if tensor_type == G.F32 else "<f2").tobytes()
        out.append((Wt.gguf_tensor_name(name), tuple(reversed(shape)), tensor_type, raw))
    return out


def write_model(path, cfg, blob, tensor_type=G.BF16, values_f32=None):
    with open(path, "wb") as f:
        f.write(gguf_bytes(model_metadata(cfg), model_tensors(cfg, blob, tensor_type, values_f32)))


def interleave_qk(cfg, blob):
    """A copy of the blob with each q/k head's rows (and bias entries) moved from split-half
    rotary order to interleaved order: row i -> 2i, row i + d/2 -> 2i + 1.  This is how GGUF
    files hold q/k, so interleaved RoPE on the result equals split-half RoPE on the input."""
    out = blob.copy()
    d = cfg.head_dim()
    order = np.empty(d, np.int64)
    order[0::2] = np.arange(d // 2)
    order[1::2] = np.arange(d // 2) + d // 2
    for name, off, shape, kind in Wt.tensor_entries(cfg):
        if ".q_proj." not in name and ".k_proj." not in name:
            continue
        rows = shape[0]
        cols = shape[1] if len(shape) == 2 else 1
        m = blob[off: off + rows * cols].reshape(rows // d, d, cols)
        out[off: off + rows * cols] = m[:, order, :].reshape(-1)
    return out


def gguf_cfg(cfg):
    """The config a GGUF file of `cfg` gives back: interleaved RoPE, no biases, no rope scaling."""
    return dataclasses.replace(cfg, rope_layout=C.ROPE_INTERLEAVED, qkv_bias=False,
                               rope_scaling_type=C.ROPE_SCALING_NONE, rope_scaling_factor=1.0,
                               rope_low_freq_factor=1.0, rope_high_freq_factor=1.0, rope_original_max_position=0)


# ---------------------------------------------------------------- GGML block quantisation (Q8_0, Q4_0)
# The published GGML block formats that GGUF files carry for tensor types 8 and 2
# (src/gguf.zig:35, 39 names them; ggml / llama.cpp define them): blocks of 32
# consecutive weights along a row (the innermost GGUF dimension).
#   Q8_0: {fp16 d; int8 q[32]}, 34 bytes, weight = d * q;  d = amax / 127,
#         q = roundf(x * (1 / d)) (halves away from zero).
#   Q4_0: {fp16 d; uint8 qs[16]}, 18 bytes, weight = d * (n - 8) where
#         qs[j] holds n of weight j in its low nibble and of weight j + 16 in
#         its high nibble;  d = m / -8 with m the weight of largest magnitude,
#         n = min(15, trunc(x * (1 / d) + 8.5)).
# The steps are single fp32 operations, as the device quantiser
# (vvli_cuda_fill_synthetic_quantized) performs them, so both give the same blocks.
# Each returns the raw block bytes and the dequantised float32 values (exact:
# an fp16 scale times a small integer fits a float32).

def quantize_q8_0(values):
    x = np.ascontiguousarray(values, np.float32).reshape(-1, 32)
    amax = np.abs(x).max(axis=1)
    d = (amax / 127.0).astype(np.float32)
    inv = np.where(d != 0, 1.0 / np.where(d != 0, d, 1), 0).astype(np.float32)
    t = x * inv[:, None]
    r = np.trunc(t)
    r = r + np.sign(t) * (np.abs(t - r) >= 0.5)  # roundf: halves away from zero
    q = np.clip(r, -127, 127).astype(np.int8)
    d16 = d.astype(np.float16)
    raw = np.zeros((x.shape[0], 34), np.uint8)
    raw[:, :2] = d16.view(np.uint8).reshape(-1, 2)
    raw[:, 2:] = q.view(np.uint8)
    deq = d16.astype(np.float32)[:, None] * q.astype(np.float32)
    return raw.tobytes(), deq.reshape(-1)


def quantize_q4_0(values):
    x = np.ascontiguousarray(values, np.float32).reshape(-1, 32)
    idx = np.abs(x).argmax(axis=1)
    m = x[np.arange(x.shape[0]), idx]
    d = (m / -8.0).astype(np.float32)
    inv = np.where(d != 0, 1.0 / np.where(d != 0, d, 1), 0).astype(np.float32)
    n = np.clip(np.minimum(15, np.trunc(x * inv[:, None] + 8.5)), 0, 15).astype(np.uint8)
    d16 = d.astype(np.float16)
    raw = np.zeros((x.shape[0], 18), np.uint8)
    raw[:, :2] = d16.view(np.uint8).reshape(-1, 2)
    raw[:, 2:] = n[:, :16] | (n[:, 16:] << 4)
    deq = d16.astype(np.float32)[:, None] * (n.astype(np.float32) - 8.0)
    return raw.tobytes(), deq.reshape(-1)


def quantized_model(cfg, blob, qtype, matrices=None):
    """GGUF tensors with every matrix (or those named in `matrices`) quantised to `qtype` and
    the rest in F32, plus the float32 blob (OwnedModel layout) of the values the file holds
    -- the oracle's weights for the quantised model."""
    out, f32 = [], Wt.bf16_to_f32(blob).copy()
    quant = quantize_q8_0 if qtype == G.Q8_0 else quantize_q4_0
    for name, off, shape, kind in Wt.tensor_entries(cfg):
        n = int(np.prod(shape))
        v = f32[off: off + n]
        if kind == "mat" and (matrices is None or name in matrices):
            raw, deq = quant(v)
            f32[off: off + n] = deq
            out.append((Wt.gguf_tensor_name(name), tuple(reversed(shape)), qtype, raw))
        else:
            out.append((Wt.gguf_tensor_name(name), tuple(reversed(shape)), G.F32, np.asarray(v, "<f4").tobytes()))
    return out, f32


def write_quantized_model(path, cfg, blob, qtype, matrices=None):
    """Writes the quantised model; returns its float32 blob for the oracle."""
    tensors, f32 = quantized_model(cfg, blob, qtype, matrices)
    with open(path, "wb") as f:
        f.write(gguf_bytes(model_metadata(cfg), tensors))
    return f32
