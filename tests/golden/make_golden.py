"""Generates the transformers fp32 golden fixtures that pin the oracle.

Run from the repository root:  python tests/golden/make_golden.py
(needs `transformers` and the oracle library; the GPU is not used).

For each small architecture below, the seeded synthetic bf16 weight blob
(oracle generator) is upcast to fp32 and loaded into transformers'
Qwen2ForCausalLM / LlamaForCausalLM (eager attention, fp32).  A uniform
random prompt runs through one causal forward; the fixture stores the token
ids, every layer's output (the residual stream, which the reference keeps in
Scratch.x), the final logits at every position, and a SHA-256 of the blob so
a change of the generator is detected.  transformers uses split-half
(rotate_half) RoPE and 1/sqrt(head_dim) scaling like the reference's
safetensors path (src/llm.zig:134, 1351-1355, 1313); the llama fixture also
pins the llama3 rope_scaling extension against transformers' implementation.
"""

import hashlib
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle  # noqa: E402
from vvli_b200 import config as C  # noqa: E402
from vvli_b200.weights import state_dict_f32  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def fixture_configs():
    qwen = C.Config(vocab_size=256, hidden_size=64, intermediate_size=160, num_hidden_layers=2,
                    num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=1024,
                    rope_theta=1e6, rms_norm_eps=C._f32(1e-6), tie_word_embeddings=True,
                    architecture=C.ARCH_QWEN2, qkv_bias=True, eos_token_id=255, pad_token_id=0)
    llama = C.Config(vocab_size=256, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                     num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=1024,
                     rope_theta=500000.0, rms_norm_eps=C._f32(1e-5), tie_word_embeddings=False,
                     architecture=C.ARCH_LLAMA, qkv_bias=False, eos_token_id=255, pad_token_id=0,
                     rope_scaling_type=C.ROPE_SCALING_LLAMA3, rope_scaling_factor=32.0,
                     rope_low_freq_factor=1.0, rope_high_freq_factor=4.0, rope_original_max_position=64)
    return {"qwen2_tiny": (qwen, 7), "llama3_tiny_rs": (llama, 11)}


def hf_model(cfg):
    import transformers
    if cfg.architecture == C.ARCH_QWEN2:
        hc = transformers.Qwen2Config(
            vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size, intermediate_size=cfg.intermediate_size,
            num_hidden_layers=cfg.num_hidden_layers, num_attention_heads=cfg.num_attention_heads,
            num_key_value_heads=cfg.num_key_value_heads, max_position_embeddings=cfg.max_position_embeddings,
            rope_theta=cfg.rope_theta, rms_norm_eps=cfg.rms_norm_eps, tie_word_embeddings=cfg.tie_word_embeddings)
        cls = transformers.Qwen2ForCausalLM
    else:
        kw = {}
        if cfg.rope_scaling_type == C.ROPE_SCALING_LLAMA3:
            kw["rope_scaling"] = {"rope_type": "llama3", "factor": cfg.rope_scaling_factor,
                                  "low_freq_factor": cfg.rope_low_freq_factor,
                                  "high_freq_factor": cfg.rope_high_freq_factor,
                                  "original_max_position_embeddings": cfg.rope_original_max_position}
        hc = transformers.LlamaConfig(
            vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size, intermediate_size=cfg.intermediate_size,
            num_hidden_layers=cfg.num_hidden_layers, num_attention_heads=cfg.num_attention_heads,
            num_key_value_heads=cfg.num_key_value_heads, max_position_embeddings=cfg.max_position_embeddings,
            rope_theta=cfg.rope_theta, rms_norm_eps=cfg.rms_norm_eps, tie_word_embeddings=cfg.tie_word_embeddings,
            attention_bias=cfg.qkv_bias, **kw)
        cls = transformers.LlamaForCausalLM
    hc._attn_implementation = "eager"
    return cls(hc).float().eval()


def make(name, cfg, seed, n_tokens=16):
    blob = oracle.synthetic_blob(cfg, seed=seed)
    sd = {k: torch.from_numpy(v.copy()) for k, v in state_dict_f32(cfg, blob).items()}
    model = hf_model(cfg)
    missing, unexpected = model.load_state_dict(sd, strict=False)
    missing = [m for m in missing if not (cfg.tie_word_embeddings and m == "lm_head.weight")]
    assert not missing and not unexpected, (missing, unexpected)
    if cfg.tie_word_embeddings:
        model.tie_weights()
    rng = np.random.default_rng(1000 + seed)
    tokens = rng.integers(0, cfg.vocab_size, size=n_tokens, dtype=np.int64)
    layer_out = []
    hooks = [layer.register_forward_hook(lambda m, i, o: layer_out.append(
        (o[0] if isinstance(o, tuple) else o).detach()[0].numpy().copy())) for layer in model.model.layers]
    with torch.no_grad():
        logits = model(torch.from_numpy(tokens)[None], use_cache=False).logits[0].numpy()
    for h in hooks:
        h.remove()
    np.savez_compressed(
        os.path.join(HERE, f"{name}.npz"), tokens=tokens.astype(np.uint32), seed=np.uint64(seed),
        hidden=np.stack(layer_out).astype(np.float32), logits=logits.astype(np.float32),
        blob_sha256=np.frombuffer(hashlib.sha256(blob.tobytes()).digest(), dtype=np.uint8))
    print(name, "tokens", tokens[:8], "logit range", float(logits.min()), float(logits.max()))


if __name__ == "__main__":
    torch.manual_seed(0)
    for name, (cfg, seed) in fixture_configs().items():
        make(name, cfg, seed)
