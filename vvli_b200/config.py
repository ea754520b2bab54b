"""Model configuration: the host-side mirror of llm.Config.

Follows src/llm.zig:77-276 (Config, fromJson, fromGguf, validate, headDim, kvDim,
kvGroupSize, layerParameterCount, parameterCount) and src/llm.zig:814-837
(storageElementCount for the bf16 weight blob).  The one extension is
``rope_scaling`` (llama3 type), which the reference never reads; pass
``rope_scaling=False`` to ``from_json`` to reproduce the reference exactly.
"""

from __future__ import annotations

import ctypes
import dataclasses
import json
import math

from .errors import VvliError, MISSING_JSON_FIELD

ARCH_LLAMA, ARCH_MISTRAL, ARCH_OLMOE, ARCH_QWEN2 = 0, 1, 2, 3
ARCH_NAMES = {"llama": ARCH_LLAMA, "mistral": ARCH_MISTRAL, "olmoe": ARCH_OLMOE, "qwen2": ARCH_QWEN2}
ROPE_INTERLEAVED, ROPE_SPLIT_HALF = 0, 1
ROPE_SCALING_NONE, ROPE_SCALING_LLAMA3 = 0, 1
ELEMS_PER_CACHE_LINE_BF16 = 32  # 64-byte tensor alignment, src/llm.zig:1499-1504


class CModelConfig(ctypes.Structure):
    """ctypes layout of ``vvli_model_config`` (include/vvli_cuda.h)."""

    _fields_ = [
        ("vocab_size", ctypes.c_uint64),
        ("hidden_size", ctypes.c_uint64),
        ("intermediate_size", ctypes.c_uint64),
        ("num_hidden_layers", ctypes.c_uint64),
        ("num_attention_heads", ctypes.c_uint64),
        ("num_key_value_heads", ctypes.c_uint64),
        ("max_position_embeddings", ctypes.c_uint64),
        ("num_experts", ctypes.c_uint64),
        ("num_experts_per_token", ctypes.c_uint64),
        ("architecture", ctypes.c_uint32),
        ("rope_layout", ctypes.c_uint32),
        ("rope_theta", ctypes.c_float),
        ("rms_norm_eps", ctypes.c_float),
        ("tie_word_embeddings", ctypes.c_uint32),
        ("qkv_bias", ctypes.c_uint32),
        ("qk_norm", ctypes.c_uint32),
        ("eos_token_id", ctypes.c_uint32),
        ("pad_token_id", ctypes.c_uint32),
        ("rope_scaling_type", ctypes.c_uint32),
        ("rope_scaling_factor", ctypes.c_float),
        ("rope_low_freq_factor", ctypes.c_float),
        ("rope_high_freq_factor", ctypes.c_float),
        ("_pad0", ctypes.c_uint32),
        ("rope_original_max_position", ctypes.c_uint64),
    ]


def _f32(x: float) -> float:
    """Rounds a Python float to float32, as Zig's @floatCast to f32 does."""
    return float(ctypes.c_float(x).value)


@dataclasses.dataclass
class Config:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    max_position_embeddings: int
    rope_theta: float
    rms_norm_eps: float
    tie_word_embeddings: bool
    architecture: int = ARCH_QWEN2
    num_experts: int = 0
    num_experts_per_token: int = 0
    qk_norm: bool = False
    rope_layout: int = ROPE_SPLIT_HALF
    qkv_bias: bool = True
    eos_token_id: int = 0
    pad_token_id: int = 0
    rope_scaling_type: int = ROPE_SCALING_NONE
    rope_scaling_factor: float = 1.0
    rope_low_freq_factor: float = 1.0
    rope_high_freq_factor: float = 1.0
    rope_original_max_position: int = 0

    # ------------------------------------------------------------ derived (src/llm.zig:229-275)
    @property
    def is_moe(self) -> bool:
        return self.num_experts != 0

    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    def kv_dim(self) -> int:
        return self.num_key_value_heads * self.head_dim()

    def kv_group_size(self) -> int:
        return self.num_attention_heads // self.num_key_value_heads

    def supports_dense_runner(self) -> bool:
        return (not self.is_moe) and self.architecture in (ARCH_LLAMA, ARCH_MISTRAL, ARCH_QWEN2)

    def validate(self) -> None:
        """Config.validate (src/llm.zig:195-216)."""
        if 0 in (self.vocab_size, self.hidden_size, self.intermediate_size, self.num_hidden_layers,
                 self.num_attention_heads, self.num_key_value_heads, self.max_position_embeddings):
            raise VvliError("InvalidConfig")
        if self.hidden_size % self.num_attention_heads != 0:
            raise VvliError("InvalidConfig")
        if self.num_attention_heads % self.num_key_value_heads != 0:
            raise VvliError("InvalidConfig")
        if self.head_dim() % 2 != 0:
            raise VvliError("InvalidConfig")
        if not self.is_moe:
            if self.num_experts_per_token != 0:
                raise VvliError("InvalidConfig")
        else:
            if self.num_experts_per_token == 0 or self.num_experts_per_token > self.num_experts:
                raise VvliError("InvalidConfig")

    def layer_parameter_count(self) -> int:
        h, kv, inter = self.hidden_size, self.kv_dim(), self.intermediate_size
        bias = h + kv + kv if self.qkv_bias else 0
        total = h + h * h + bias + kv * h + kv * h + h * h + h
        if self.qk_norm:
            total += self.head_dim() * 2
        if not self.is_moe:
            total += 3 * inter * h
        else:
            total += self.num_experts * h + self.num_experts * (inter * h * 2 + h * inter)
        return total

    def parameter_count(self) -> int:
        total = self.vocab_size * self.hidden_size + self.num_hidden_layers * self.layer_parameter_count()
        total += self.hidden_size
        if not self.tie_word_embeddings:
            total += self.vocab_size * self.hidden_size
        return total

    def matrix_parameter_count(self) -> int:
        """Parameters streamed by one decode token's GEMVs (layers + LM head)."""
        h, kv, inter = self.hidden_size, self.kv_dim(), self.intermediate_size
        per_layer = h * h + 2 * kv * h + h * h + 3 * inter * h
        return self.num_hidden_layers * per_layer + self.vocab_size * h

    def storage_element_count(self) -> int:
        """storageElementCount(config, .bf16) (src/llm.zig:814-837)."""
        a = ELEMS_PER_CACHE_LINE_BF16
        cur = 0

        def add(n):
            nonlocal cur
            cur = (cur + a - 1) // a * a + n

        h, kv, inter = self.hidden_size, self.kv_dim(), self.intermediate_size
        add(self.vocab_size * h)
        for _ in range(self.num_hidden_layers):
            add(h)
            add(h * h)
            if self.qkv_bias:
                add(h)
            add(kv * h)
            if self.qkv_bias:
                add(kv)
            add(kv * h)
            if self.qkv_bias:
                add(kv)
            add(h * h)
            add(h)
            add(inter * h)
            add(inter * h)
            add(h * inter)
        add(h)
        if not self.tie_word_embeddings:
            add(self.vocab_size * h)
        return cur

    def to_c(self) -> CModelConfig:
        c = CModelConfig()
        for f in dataclasses.fields(self):
            v = getattr(self, f.name)
            setattr(c, f.name, int(v) if isinstance(v, bool) else v)
        return c

    # ------------------------------------------------------------ Config.fromJson (src/llm.zig:98-145)
    @classmethod
    def from_json(cls, text: str, rope_scaling: bool = True) -> "Config":
        root = json.loads(text, parse_float=str, parse_int=int)
        if not isinstance(root, dict):
            raise VvliError("InvalidConfig")
        model_type = root.get("model_type")
        if not isinstance(model_type, str):
            raise VvliError(MISSING_JSON_FIELD, -1, "model_type")
        if model_type not in ARCH_NAMES:
            raise VvliError("UnsupportedModelArchitecture")
        arch = ARCH_NAMES[model_type]

        def usize(v):  # jsonValueUsize (src/llm.zig:1571-1577)
            if isinstance(v, bool) or not isinstance(v, int):
                if isinstance(v, str):  # number_string
                    try:
                        return int(v, 10)
                    except ValueError:
                        pass
                raise VvliError("InvalidConfig")
            if v < 0:
                raise VvliError("InvalidConfig")
            return v

        def required(key):
            if key not in root:
                raise VvliError(MISSING_JSON_FIELD, -1, key)
            return usize(root[key])

        def optional_usize(key):
            if key not in root:
                return None
            try:
                return usize(root[key])
            except VvliError:
                return None

        def optional_f32(key):
            v = root.get(key)
            if v is None or isinstance(v, bool):
                return None
            if isinstance(v, int):
                return _f32(float(v))
            if isinstance(v, str):  # floats arrive as strings (parse_float=str)
                try:
                    return _f32(float(v))
                except ValueError:
                    return None
            return None

        def optional_bool(key):
            v = root.get(key)
            return v if isinstance(v, bool) else None

        def optional_token(key):  # getOptionalTokenId (src/llm.zig:1536-1543)
            if key not in root:
                return None
            v = root[key]
            if v is None:
                return None
            if isinstance(v, list):
                if not v:
                    return None
                v = v[0]
            try:
                return usize(v)
            except VvliError:
                return None

        heads = required("num_attention_heads")
        num_experts = optional_usize("num_experts") or 0
        cfg = cls(
            architecture=arch,
            vocab_size=required("vocab_size"),
            hidden_size=required("hidden_size"),
            intermediate_size=required("intermediate_size"),
            num_hidden_layers=required("num_hidden_layers"),
            num_attention_heads=heads,
            num_key_value_heads=optional_usize("num_key_value_heads") or heads,
            num_experts=num_experts,
            num_experts_per_token=optional_usize("num_experts_per_tok") or 0,
            qk_norm=arch == ARCH_OLMOE,
            rope_layout=ROPE_SPLIT_HALF,
            max_position_embeddings=required("max_position_embeddings"),
            rope_theta=_v(optional_f32("rope_theta"), 10000.0),
            rms_norm_eps=_v(optional_f32("rms_norm_eps"), _f32(1e-6)),
            tie_word_embeddings=_v(optional_bool("tie_word_embeddings"), False),
            qkv_bias=_v(optional_bool("attention_bias"), arch == ARCH_QWEN2),
            eos_token_id=_v(optional_token("eos_token_id"), 0),
            pad_token_id=_v(optional_token("pad_token_id"), 0),
        )
        if rope_scaling:
            rs = root.get("rope_scaling")
            if isinstance(rs, dict) and rs.get("rope_type", rs.get("type")) == "llama3":
                cfg.rope_scaling_type = ROPE_SCALING_LLAMA3
                cfg.rope_scaling_factor = _f32(float(rs.get("factor", 8.0)))
                cfg.rope_low_freq_factor = _f32(float(rs.get("low_freq_factor", 1.0)))
                cfg.rope_high_freq_factor = _f32(float(rs.get("high_freq_factor", 4.0)))
                cfg.rope_original_max_position = int(rs.get("original_max_position_embeddings", 8192))
        cfg.validate()
        return cfg

    # ------------------------------------------------------------ Config.fromGguf (src/llm.zig:153-193)
    @classmethod
    def from_gguf(cls, file) -> "Config":
        """The config of a parsed GGUF file (``vvli_b200.gguf.parse``): interleaved RoPE, no q/k/v biases."""
        from . import gguf as G

        arch_text = file.string("general.architecture")
        if arch_text is None:
            raise VvliError(MISSING_JSON_FIELD, -1, "general.architecture")
        if arch_text not in ARCH_NAMES:
            raise VvliError("UnsupportedModelArchitecture")
        arch = ARCH_NAMES[arch_text]
        prefix = arch_text  # Architecture.ggufPrefix (src/llm.zig:35-42)
        vocab = file.metadata_value("tokenizer.ggml.tokens")
        if vocab is None:
            raise VvliError(MISSING_JSON_FIELD, -1, "tokenizer.ggml.tokens")
        if vocab[0] != G.ARRAY:
            raise VvliError("InvalidConfig")

        def required(suffix):
            v = file.usize_value(f"{prefix}.{suffix}")
            if v is None:
                raise VvliError(MISSING_JSON_FIELD, -1, f"{prefix}.{suffix}")
            return v

        heads = required("attention.head_count")
        cfg = cls(
            architecture=arch,
            vocab_size=vocab[1].len,
            hidden_size=required("embedding_length"),
            intermediate_size=required("feed_forward_length"),
            num_hidden_layers=required("block_count"),
            num_attention_heads=heads,
            num_key_value_heads=_v(file.usize_value(f"{prefix}.attention.head_count_kv"), heads),
            rope_layout=ROPE_INTERLEAVED,
            max_position_embeddings=required("context_length"),
            rope_theta=_v(file.f32_value(f"{prefix}.rope.freq_base"), 10000.0),
            rms_norm_eps=_v(file.f32_value(f"{prefix}.attention.layer_norm_rms_epsilon"), _f32(1e-6)),
            tie_word_embeddings=file.tensor("output.weight") is None,
            qkv_bias=False,
            eos_token_id=_v(file.usize_value("tokenizer.ggml.eos_token_id"), 0),
            pad_token_id=_v(file.usize_value("tokenizer.ggml.padding_token_id"), 0),
        )
        cfg.validate()
        return cfg

    def to_hf_json(self) -> dict:
        """A config.json for this architecture (used to build transformers fixtures)."""
        d = {
            "model_type": {v: k for k, v in ARCH_NAMES.items()}[self.architecture],
            "vocab_size": self.vocab_size,
            "hidden_size": self.hidden_size,
            "intermediate_size": self.intermediate_size,
            "num_hidden_layers": self.num_hidden_layers,
            "num_attention_heads": self.num_attention_heads,
            "num_key_value_heads": self.num_key_value_heads,
            "max_position_embeddings": self.max_position_embeddings,
            "rope_theta": self.rope_theta,
            "rms_norm_eps": self.rms_norm_eps,
            "tie_word_embeddings": self.tie_word_embeddings,
            "attention_bias": self.qkv_bias,
            "eos_token_id": self.eos_token_id,
            "pad_token_id": self.pad_token_id,
            "hidden_act": "silu",
        }
        if self.rope_scaling_type == ROPE_SCALING_LLAMA3:
            d["rope_scaling"] = {
                "rope_type": "llama3",
                "factor": self.rope_scaling_factor,
                "low_freq_factor": self.rope_low_freq_factor,
                "high_freq_factor": self.rope_high_freq_factor,
                "original_max_position_embeddings": self.rope_original_max_position,
            }
        return d


def _v(value, default):
    return default if value is None else value


# ---------------------------------------------------------------- benchmark architectures
def qwen2_5_0_5b() -> Config:
    """Qwen2.5-0.5B architecture (hidden 896, 24 layers, 14/2 heads, tied, q/k/v bias)."""
    return Config(vocab_size=151936, hidden_size=896, intermediate_size=4864, num_hidden_layers=24,
                  num_attention_heads=14, num_key_value_heads=2, max_position_embeddings=32768,
                  rope_theta=1e6, rms_norm_eps=_f32(1e-6), tie_word_embeddings=True, architecture=ARCH_QWEN2,
                  qkv_bias=True, eos_token_id=151645, pad_token_id=151643)


def llama3_2_1b() -> Config:
    """Llama-3.2-1B architecture with llama3 rope scaling (factor 32, low 1, high 4, orig 8192)."""
    return Config(vocab_size=128256, hidden_size=2048, intermediate_size=8192, num_hidden_layers=16,
                  num_attention_heads=32, num_key_value_heads=8, max_position_embeddings=131072,
                  rope_theta=500000.0, rms_norm_eps=_f32(1e-5), tie_word_embeddings=True,
                  architecture=ARCH_LLAMA, qkv_bias=False, eos_token_id=128009, pad_token_id=128004,
                  rope_scaling_type=ROPE_SCALING_LLAMA3, rope_scaling_factor=32.0, rope_low_freq_factor=1.0,
                  rope_high_freq_factor=4.0, rope_original_max_position=8192)


def llama3_8b() -> Config:
    """Llama-3-8B architecture (hidden 4096, 32 layers, 32/8 heads, head_dim 128, untied)."""
    return Config(vocab_size=128256, hidden_size=4096, intermediate_size=14336, num_hidden_layers=32,
                  num_attention_heads=32, num_key_value_heads=8, max_position_embeddings=8192,
                  rope_theta=500000.0, rms_norm_eps=_f32(1e-5), tie_word_embeddings=False,
                  architecture=ARCH_LLAMA, qkv_bias=False, eos_token_id=128009, pad_token_id=128004)


def tiny_qwen() -> Config:
    """The reference's tiny runner test shape (src/llm.zig:1743-1758)."""
    return Config(vocab_size=24, hidden_size=16, intermediate_size=32, num_hidden_layers=2,
                  num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=16,
                  rope_theta=10000.0, rms_norm_eps=_f32(1e-6), tie_word_embeddings=True, eos_token_id=2,
                  pad_token_id=0)


PRESETS = {
    "qwen2.5-0.5b": qwen2_5_0_5b,
    "llama3.2-1b": llama3_2_1b,
    "llama3-8b": llama3_8b,
    "tiny": tiny_qwen,
}


def decode_bytes_per_token(cfg: Config, position: int, tp: int = 1, kv_bytes: int = 4) -> int:
    """Algorithmic HBM bytes of one decode token at `position` (whole job):
    every matrix once (bf16), norms and biases, the KV rows read (positions
    0..position) and the new row written."""
    h, kv = cfg.hidden_size, cfg.kv_dim()
    mats = cfg.matrix_parameter_count() * 2
    small = (cfg.num_hidden_layers * 2 * h + h) * 2
    if cfg.qkv_bias:
        small += cfg.num_hidden_layers * (h + 2 * kv) * 2
    kv_traffic = cfg.num_hidden_layers * (position + 1) * kv * 2 * kv_bytes
    return mats + small + kv_traffic
