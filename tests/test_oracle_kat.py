"""Pins the CPU oracle to the reference's own known-answer tests.

Each test restates one inline Zig test of VVLI (inputs and expected values)
and runs it against the oracle (oracle/vvli_ref_cpu.cpp) or the host-side
config mirror (vvli_b200/config.py).
"""

import math

import numpy as np
import pytest

from vvli_b200 import config as C
from vvli_b200.errors import VvliError


def test_bf16_conversion_and_expansion(oracle):
    # src/llm.zig:1690-1701
    for v in (1.0, -2.5, 0.25, 8.0):
        assert abs(oracle.bf16_to_f32(oracle.f32_to_bf16(v)) - v) <= 0.01


def test_f32_to_bf16_rounds_to_nearest_even(oracle):
    # f32ToBf16 (src/llm.zig:799-803): bits + 0x7fff + ((bits >> 16) & 1)
    import struct

    def bits(f):
        return struct.unpack("<I", struct.pack("<f", f))[0]

    for f in (1.0, 1.00390625, 1.01171875, -3.14159, 1e-30, 65504.0, 0.02):
        b = bits(f)
        expect = ((b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFFFFFF) >> 16
        assert oracle.f32_to_bf16(f) == expect


def test_rope_layouts_known_answer(oracle):
    # src/llm.zig:1703-1716: pos 1, theta 1e4, head_dim 4
    cfg = C.tiny_qwen()
    cfg.rope_theta = 10000.0
    cos0, sin0 = math.cos(1.0), math.sin(1.0)
    cfg.rope_layout = C.ROPE_SPLIT_HALF
    split = oracle.apply_rope([1.0, 2.0, 3.0, 4.0], 1, 4, 1, cfg)
    cfg.rope_layout = C.ROPE_INTERLEAVED
    inter = oracle.apply_rope([1.0, 2.0, 3.0, 4.0], 1, 4, 1, cfg)
    assert abs(split[0] - (1.0 * cos0 - 3.0 * sin0)) <= 1e-6
    assert abs(split[2] - (1.0 * sin0 + 3.0 * cos0)) <= 1e-6
    assert abs(inter[0] - (1.0 * cos0 - 2.0 * sin0)) <= 1e-6
    assert abs(inter[1] - (1.0 * sin0 + 2.0 * cos0)) <= 1e-6


def test_rms_norm_known_answer(oracle):
    # src/tensor.zig:866-878: [3, 4], weight 1, eps 0
    out = oracle.rms_norm([3.0, 4.0], [1.0, 1.0], 0.0)
    assert abs(out[0] - 0.84852815) <= 1e-6
    assert abs(out[1] - 1.1313708) <= 1e-6


def test_softmax_known_answer(oracle):
    # src/tensor.zig:848-864
    r0 = oracle.softmax([1.0, 2.0, 3.0])
    r1 = oracle.softmax([1.0, 1.0, 1.0])
    assert abs(r0.sum() - 1.0) <= 1e-6
    assert np.all(np.abs(r1 - 1.0 / 3.0) <= 1e-6)


def test_argmax_first_index_wins_ties(oracle):
    # src/llm.zig:778-789: strict >
    assert oracle.argmax([1.0, 3.0, 3.0, 2.0]) == 1
    assert oracle.argmax([5.0]) == 0
    assert oracle.argmax([-1.0, -1.0]) == 0


def test_repeat_penalty_moves_greedy_choice(oracle):
    # src/generator.zig:491-499
    assert oracle.greedy_with_penalties([10.0, 9.8, 1.0], [1, 0, 0], 2.0) == 1


def test_top_k_candidate_builder(oracle):
    # src/generator.zig:501-512
    cands = oracle.build_candidates([1.0, 4.0, 2.0, 3.0], [0, 0, 0, 0], top_k=2, repeat_penalty=1.0, capacity=2)
    assert len(cands) == 2
    assert cands[0]["id"] == 1 and cands[1]["id"] == 3


def test_qwen_config_numbers():
    # src/llm.zig:1579-1605
    cfg = C.Config.from_json("""{
      "model_type": "qwen2", "vocab_size": 151936, "hidden_size": 896, "intermediate_size": 4864,
      "num_hidden_layers": 24, "num_attention_heads": 14, "num_key_value_heads": 2,
      "max_position_embeddings": 32768, "rope_theta": 1000000.0, "rms_norm_eps": 1e-6,
      "tie_word_embeddings": true, "eos_token_id": 151645, "pad_token_id": 151654}""")
    assert cfg.head_dim() == 64 and cfg.kv_dim() == 128 and cfg.kv_group_size() == 7
    assert cfg.parameter_count() > 494_005_120
    assert cfg.storage_element_count() >= cfg.parameter_count()
    assert cfg.qkv_bias and cfg.rope_layout == C.ROPE_SPLIT_HALF


def test_llama_and_mistral_config():
    # src/llm.zig:1607-1658
    llama = C.Config.from_json("""{
      "model_type": "llama", "vocab_size": 128256, "hidden_size": 2048, "intermediate_size": 8192,
      "num_hidden_layers": 16, "num_attention_heads": 32, "num_key_value_heads": 8,
      "max_position_embeddings": 131072, "rope_theta": 500000.0, "rms_norm_eps": 1e-5,
      "tie_word_embeddings": true, "attention_bias": false, "eos_token_id": 128009, "pad_token_id": 128004}""")
    assert llama.architecture == C.ARCH_LLAMA and llama.supports_dense_runner() and llama.head_dim() == 64
    mistral = C.Config.from_json("""{
      "model_type": "mistral", "vocab_size": 32000, "hidden_size": 4096, "intermediate_size": 14336,
      "num_hidden_layers": 32, "num_attention_heads": 32, "num_key_value_heads": 8,
      "max_position_embeddings": 32768, "rope_theta": 10000.0, "rms_norm_eps": 1e-5,
      "tie_word_embeddings": false, "eos_token_id": 2, "pad_token_id": 2}""")
    assert mistral.rope_layout == C.ROPE_SPLIT_HALF and not mistral.qkv_bias and mistral.supports_dense_runner()


def test_olmoe_config_is_moe_and_rejected(oracle):
    # src/llm.zig:1660-1688
    cfg = C.Config.from_json("""{
      "model_type": "olmoe", "vocab_size": 50304, "hidden_size": 2048, "intermediate_size": 1024,
      "num_hidden_layers": 16, "num_attention_heads": 16, "num_key_value_heads": 16, "num_experts": 64,
      "num_experts_per_tok": 8, "max_position_embeddings": 4096, "rope_theta": 10000.0,
      "rms_norm_eps": 1e-5, "tie_word_embeddings": false, "attention_bias": false,
      "eos_token_id": 50279, "pad_token_id": 1}""")
    assert cfg.is_moe and not cfg.supports_dense_runner()
    with pytest.raises(VvliError) as e:
        oracle.RefRunner(cfg, synthetic_seed=0, max_seq=8)
    assert e.value.name == "UnsupportedModelArchitecture"


def test_config_missing_and_unsupported_fields():
    with pytest.raises(VvliError) as e:
        C.Config.from_json('{"model_type": "gpt2"}')
    assert e.value.name == "UnsupportedModelArchitecture"
    with pytest.raises(VvliError) as e:
        C.Config.from_json('{"model_type": "llama", "vocab_size": 10}')
    assert e.value.name == "MissingJsonField"
    with pytest.raises(VvliError) as e:
        C.Config.from_json("""{"model_type": "llama", "vocab_size": 10, "hidden_size": 6,
          "intermediate_size": 4, "num_hidden_layers": 1, "num_attention_heads": 4,
          "max_position_embeddings": 8}""")
    assert e.value.name == "InvalidConfig"  # hidden % heads != 0


def test_blob_layout_matches_storage_element_count(oracle):
    # src/llm.zig:1718-1741 + storageElementCount (src/llm.zig:814-837)
    for cfg in (C.tiny_qwen(), C.qwen2_5_0_5b(), C.llama3_2_1b(), C.llama3_8b()):
        n = oracle.storage_elements(cfg)
        assert n == cfg.storage_element_count()
        assert n * 2 >= cfg.parameter_count() * 2
        table = oracle.tensor_table(cfg)
        assert np.all(table[:, 0] % 32 == 0)  # 64-byte aligned offsets
        ends = table[:, 0] + table[:, 1]
        assert np.all(ends[:-1] <= table[1:, 0])
        assert int(ends[-1]) == n


def test_tiny_runner_token_step(oracle):
    # src/llm.zig:1743-1782 (threads 2, min rows 4; deterministic test weights)
    cfg = C.tiny_qwen()
    blob = oracle.deterministic_blob(cfg)
    r = oracle.RefRunner(cfg, blob=blob, max_seq=8, threads=2, min_rows_per_thread=4)
    logits = r.forward_token(3, 0)
    assert logits.shape == (cfg.vocab_size,) and np.all(np.isfinite(logits))
    assert oracle.argmax(logits) < cfg.vocab_size
    emb_logits = r.forward_embedding(np.full(16, 0.01, np.float32), 1)
    assert emb_logits.shape == (cfg.vocab_size,) and np.all(np.isfinite(emb_logits))


def test_runner_errors(oracle):
    cfg = C.tiny_qwen()
    r = oracle.RefRunner(cfg, synthetic_seed=0, max_seq=4)
    with pytest.raises(VvliError) as e:
        r.forward_token(cfg.vocab_size, 0)
    assert e.value.name == "InvalidToken"
    with pytest.raises(VvliError) as e:
        r.forward_token(1, 4)
    assert e.value.name == "ContextFull"
    with pytest.raises(VvliError) as e:
        r.generate_greedy([], 4)
    assert e.value.name == "EmptyPrompt"
    with pytest.raises(VvliError) as e:
        oracle.RefRunner(cfg, synthetic_seed=0, max_seq=cfg.max_position_embeddings + 1)
    assert e.value.name == "InvalidConfig"


def test_threading_does_not_change_results(oracle):
    # linearInto splits rows across threads; each row's dot is independent.
    cfg = C.tiny_qwen()
    cfg.vocab_size, cfg.hidden_size, cfg.intermediate_size = 300, 64, 192
    a = oracle.RefRunner(cfg, synthetic_seed=5, max_seq=8, threads=1)
    b = oracle.RefRunner(cfg, synthetic_seed=5, max_seq=8, threads=7, min_rows_per_thread=4)
    for pos, tok in enumerate([3, 17, 299, 0]):
        assert np.array_equal(a.forward_token(tok, pos), b.forward_token(tok, pos))


def test_synthetic_generator_statistics(oracle):
    cfg = C.tiny_qwen()
    cfg.vocab_size, cfg.hidden_size, cfg.intermediate_size = 4096, 64, 128
    blob = oracle.synthetic_blob(cfg, seed=0)
    again = oracle.synthetic_blob(cfg, seed=0, threads=3)
    other = oracle.synthetic_blob(cfg, seed=1)
    assert np.array_equal(blob, again) and not np.array_equal(blob, other)
    table = oracle.tensor_table(cfg)
    emb = blob[: cfg.vocab_size * cfg.hidden_size].astype(np.uint32) << 16
    vals = emb.view(np.float32)
    assert abs(vals.mean()) < 2e-4 and abs(vals.std() - 0.02) < 5e-4
    # input_norm of layer 0 is all ones
    off, n, tid = (int(v) for v in table[1])
    assert tid == 1 and np.all(blob[off: off + n] == 0x3F80)
