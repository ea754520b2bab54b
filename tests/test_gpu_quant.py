"""Block-quantised GGUF weights (Q8_0, Q4_0) through the decode megakernel.

The reference names these tensor types (src/gguf.zig:35, 39) but rejects
them when loading (src/llm.zig:1083: "quantized GGUF tensors still need
dequant kernels").  Here the loader keeps the 32-weight blocks on the device
and the megakernel dequantises them in registers while it streams them.  The
oracle runs the same model with the dequantised values as f32 weights (the
reference's .f32 Matrix path, dotF32), so the two agree to fp32 rounding:
per-layer hidden states and logits within 1e-4, identical greedy streams.
"""


import dataclasses

import numpy as np
import pytest

from vvli_b200 import config as C
from vvli_b200 import gguf as G
from vvli_b200.errors import VvliError

from gguf_writer import gguf_bytes, model_metadata, quantized_model, write_quantized_model

pytestmark = pytest.mark.gpu

TIGHT = 1e-4
LOGIT_MAX_ABS = 2e-2


@pytest.fixture(scope="module")
def vv():
    import vvli_b200
    return vvli_b200


def gguf_llama(hidden, heads, kv_heads, inter, layers, vocab, tied=False):
    return C.Config(vocab_size=vocab, hidden_size=hidden, intermediate_size=inter, num_hidden_layers=layers,
                    num_attention_heads=heads, num_key_value_heads=kv_heads, max_position_embeddings=4096,
                    rope_theta=500000.0, rms_norm_eps=C._f32(1e-5), tie_word_embeddings=tied,
                    architecture=C.ARCH_LLAMA, qkv_bias=False, rope_layout=C.ROPE_INTERLEAVED)


def rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def check_model(oracle, vv, tmp_path, cfg, qtype, prompt_len=6, n_new=32, seed=0):
    blob = oracle.synthetic_blob(cfg, seed=seed)
    path = str(tmp_path / "model.gguf")
    f32 = write_quantized_model(path, cfg, blob, qtype)
    with open(path, "rb") as f:
        assert C.Config.from_gguf(G.parse(f.read())) == cfg
    gpu = vv.Runner(cfg, max_seq=128)
    gpu.load_gguf(path)
    assert gpu.query("quantized") == 1 and gpu.query("megakernel") == 1
    ref = oracle.RefRunner(cfg, blob_f32=f32, max_seq=128, threads=4)
    prompt = np.random.default_rng(seed + 1).integers(0, cfg.vocab_size, size=prompt_len).tolist()
    gpu.set_debug(True)
    for pos, t in enumerate(prompt):
        lr = ref.forward_token(t, pos)
        lg = gpu.forward_token(t, pos)
        for layer in range(cfg.num_hidden_layers):
            assert rel(gpu.debug_hidden(layer), ref.hidden(layer)) < TIGHT, (pos, layer)
        assert np.max(np.abs(lg - lr)) < LOGIT_MAX_ABS and rel(lg, lr) < TIGHT, pos
        assert gpu.last_argmax == oracle.argmax(lr), pos
    gpu.set_debug(False)
    gpu.reset()
    ref.reset()
    got, stats = gpu.generate_greedy(prompt, n_new)
    want = ref.generate_greedy(prompt, n_new)
    assert got == want, next(i for i, (a, b) in enumerate(zip(got, want)) if a != b)
    assert stats.generated_tokens == n_new and len(set(want)) >= 8, want
    return gpu, blob


@pytest.mark.parametrize("qtype", [G.Q8_0, G.Q4_0], ids=["q8_0", "q4_0"])
def test_quantized_small_models_match_oracle(oracle, vv, tmp_path, qtype):
    # head_dim 64, GQA 4:1 (hidden 1024), untied, and tied at the Llama-3.2-1B width (the
    # quantised embedding is also the LM head)
    check_model(oracle, vv, tmp_path, gguf_llama(1024, 16, 4, 2816, 2, 4096), qtype, seed=1)
    check_model(oracle, vv, tmp_path, gguf_llama(2048, 32, 8, 8192, 2, 4096, tied=True), qtype, seed=3)


@pytest.mark.parametrize("qtype", [G.Q8_0, G.Q4_0], ids=["q8_0", "q4_0"])
def test_quantized_llama3_8b_layer_shapes(oracle, vv, tmp_path, qtype):
    # Llama-3-8B layer shapes (h 4096, 32/8 heads, d 128, I 14336): the widest
    # rows the plan splits over 16 warps; one layer, small vocabulary.
    check_model(oracle, vv, tmp_path, gguf_llama(4096, 32, 8, 14336, 1, 2048), qtype, n_new=16)


def test_bf16_load_after_quantized_load(oracle, vv, tmp_path):
    # A later bf16 load re-plans the megakernel for bf16 rows.
    cfg = gguf_llama(1024, 16, 4, 2816, 2, 4096)
    gpu, blob = check_model(oracle, vv, tmp_path, cfg, G.Q8_0, seed=1)
    gpu.load_weights(blob)
    assert gpu.query("quantized") == 0
    ref = oracle.RefRunner(cfg, blob=blob, max_seq=128, threads=4)
    for pos, t in enumerate([3, 77, 1000, 5]):
        lr = ref.forward_token(t, pos)
        assert rel(gpu.forward_token(t, pos), lr) < TIGHT


def test_quantized_errors(oracle, vv, tmp_path):
    cfg = gguf_llama(512, 8, 2, 1536, 1, 4096)
    blob = oracle.synthetic_blob(cfg, seed=2)
    md = model_metadata(cfg)

    def load(tensors, runner=None):
        p = tmp_path / "m.gguf"
        p.write_bytes(gguf_bytes(md, tensors))
        r = runner or vv.Runner(cfg, max_seq=16)
        r.load_gguf(str(p))
        return r

    # q quantised but k / v not: one fused q|k|v matrix has one format
    mixed, _ = quantized_model(cfg, blob, G.Q8_0, matrices={"model.layers.0.self_attn.q_proj.weight"})
    with pytest.raises(VvliError) as e:
        load(mixed)
    assert e.value.name == "UnsupportedDType"
    # a quantised norm weight
    ts, _ = quantized_model(cfg, blob, G.Q8_0)
    norm_q8 = bytes(cfg.hidden_size // 32 * 34)  # zero blocks
    bad = [(n, d, G.Q8_0, norm_q8) if n == "output_norm.weight" else (n, d, t, r) for n, d, t, r in ts]
    with pytest.raises(VvliError) as e:
        load(bad)
    assert e.value.name == "UnsupportedDType"
    # the quantised model runs; decode batches are bf16-only
    r = load(ts, vv.Runner(cfg, max_seq=16, max_batch=2))
    assert r.forward_token(1, 0).shape == (cfg.vocab_size,)
    with pytest.raises(VvliError) as e:
        r.forward_batch([1, 2], [1, 1])
    assert e.value.name == "Unimplemented"
    with pytest.raises(VvliError) as e:
        r.prefill_batch([[1, 2], [3]])
    assert e.value.name == "Unimplemented"


@pytest.mark.parametrize("qtype,fmt", [(G.Q8_0, "q8_0"), (G.Q4_0, "q4_0")], ids=["q8_0", "q4_0"])
def test_device_quantised_fill_equals_gguf_file(oracle, vv, tmp_path, qtype, fmt):
    # vvli_cuda_fill_synthetic_quantized quantises with the same fp32 steps as
    # the GGUF writer: the two models are the same blocks, bit for bit.
    cfg = gguf_llama(1024, 16, 4, 2816, 2, 4096)
    blob = oracle.synthetic_blob(cfg, seed=1)
    path = str(tmp_path / "model.gguf")
    write_quantized_model(path, cfg, blob, qtype)
    a = vv.Runner(cfg, max_seq=32)
    a.load_gguf(path)
    b = vv.Runner(cfg, max_seq=32)
    b.fill_synthetic_quantized(1, fmt)
    assert b.query("quantized") == 1
    for pos, t in enumerate([5, 4000, 17, 999]):
        assert np.array_equal(a.forward_token(t, pos), b.forward_token(t, pos)), pos


def test_device_quantised_llama3_8b_shapes_split_half_rope(oracle, vv):
    # The benchmarked architecture's layer (split-half RoPE, q/k rows re-paired
    # before quantisation) at Q8_0, against the oracle on the dequantised values.
    cfg = dataclasses.replace(C.llama3_8b(), num_hidden_layers=1, vocab_size=4096, eos_token_id=0, pad_token_id=0)
    blob = oracle.synthetic_blob(cfg, seed=0)
    _, f32 = quantized_model(cfg, blob, G.Q8_0)
    gpu = vv.Runner(cfg, max_seq=64)
    gpu.fill_synthetic_quantized(0, "q8_0")
    ref = oracle.RefRunner(cfg, blob_f32=f32, max_seq=64, threads=4)
    gpu.set_debug(True)
    prompt = [11, 3000, 7, 123]
    for pos, t in enumerate(prompt):
        lr = ref.forward_token(t, pos)
        lg = gpu.forward_token(t, pos)
        assert rel(gpu.debug_hidden(0), ref.hidden(0)) < TIGHT and rel(lg, lr) < TIGHT, pos
    gpu.set_debug(False)
    gpu.reset()
    ref.reset()
    got, _ = gpu.generate_greedy(prompt, 16)
    assert got == ref.generate_greedy(prompt, 16)
