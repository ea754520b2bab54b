"""The oracle's checker conveniences give the reference loop's exact results.

Long-context GPU parity tests drive the oracle with attention heads split
over threads and with the LM head run only for the last prompt token.  Both
must leave every produced value bit-identical to plain forwardToken calls
(src/llm.zig:702-709) with the sequential computeAttentionInto
(src/llm.zig:1302-1335).
"""

import numpy as np

from vvli_b200 import config as C


def small_cfg():
    cfg = C.llama3_2_1b()
    cfg.hidden_size, cfg.intermediate_size, cfg.num_hidden_layers = 256, 512, 2
    cfg.num_attention_heads, cfg.num_key_value_heads, cfg.vocab_size = 4, 1, 1000
    return cfg


def test_parallel_attention_and_prefill_are_bit_identical(oracle):
    cfg = small_cfg()
    toks = np.random.default_rng(0).integers(0, cfg.vocab_size, size=150).tolist()
    a = oracle.RefRunner(cfg, synthetic_seed=3, max_seq=256)
    b = oracle.RefRunner(cfg, synthetic_seed=3, max_seq=256)
    b.set_attention_threads(3)
    for pos, t in enumerate(toks):
        la = a.forward_token(t, pos)
    lb = b.prefill(toks, 0)
    assert np.array_equal(la, lb)
    for layer in range(cfg.num_hidden_layers):
        assert np.array_equal(a.hidden(layer), b.hidden(layer))
    # decoding on from both caches stays identical
    for pos in range(len(toks), len(toks) + 5):
        t = oracle.argmax(la)
        la, lb = a.forward_token(t, pos), b.forward_token(t, pos)
        assert np.array_equal(la, lb)


def test_f32_weight_storage_matches_bf16_blob(oracle):
    # bf16 -> f32 is exact, and dotF32 has dotBf16's summation order, so the
    # f32-storage runner (used for dequantised GGUF tensors) must reproduce
    # the bf16 runner bit for bit.
    cfg = small_cfg()
    blob = oracle.synthetic_blob(cfg, seed=5)
    f32 = (blob.astype(np.uint32) << 16).view(np.float32)
    a = oracle.RefRunner(cfg, blob=blob, max_seq=64)
    b = oracle.RefRunner(cfg, blob_f32=f32, max_seq=64)
    for pos, t in enumerate([3, 999, 17, 250, 4]):
        la, lb = a.forward_token(t, pos), b.forward_token(t, pos)
        assert np.array_equal(la, lb)
        for layer in range(cfg.num_hidden_layers):
            assert np.array_equal(a.hidden(layer), b.hidden(layer))
