"""Parity of the CUDA decoder (through the C ABI) against the CPU oracle.

Contract: per-layer hidden states within 1e-2
relative L2, logits within 2e-2 max-abs after the final norm, and identical
greedy token streams over the first 32 tokens.  The GPU path computes in fp32
like the reference, so tighter bounds are asserted too where they hold.
"""

import dataclasses
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

from make_golden import fixture_configs  # noqa: E402
from vvli_b200 import config as C  # noqa: E402
from vvli_b200.errors import VvliError  # noqa: E402

pytestmark = pytest.mark.gpu

HIDDEN_REL_L2 = 1e-2
LOGIT_MAX_ABS = 2e-2
TIGHT_REL_L2 = 1e-4    # fp32 vs fp32 (different summation order)


def rel_l2(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def vv():
    import vvli_b200
    return vvli_b200


def make_pair(oracle, vv, cfg, seed, max_seq, blob=None, synthetic_on_device=False):
    if blob is None:
        blob = oracle.synthetic_blob(cfg, seed=seed)
    ref = oracle.RefRunner(cfg, blob=blob, max_seq=max_seq)
    gpu = vv.Runner(cfg, max_seq=max_seq)
    if synthetic_on_device:
        gpu.fill_synthetic(seed)
    else:
        gpu.load_weights(blob)
    return ref, gpu, blob


def test_tiny_reference_shape(oracle, vv):
    # The reference's own tiny runner shape (src/llm.zig:1743-1782), test weights.
    cfg = C.tiny_qwen()
    blob = oracle.deterministic_blob(cfg)
    ref, gpu, _ = make_pair(oracle, vv, cfg, 0, 8, blob=blob)
    for pos, tok in enumerate([3, 1, 22, 7, 0, 5, 9, 23]):
        lr = ref.forward_token(tok, pos)
        lg = gpu.forward_token(tok, pos)
        assert np.all(np.isfinite(lg))
        assert np.max(np.abs(lg - lr)) < 1e-5, pos
        assert gpu.last_argmax == oracle.argmax(lr)
    e = np.full(16, 0.01, np.float32)
    ref.reset()
    gpu.reset()
    assert np.max(np.abs(gpu.forward_embedding(e, 0) - ref.forward_embedding(e, 0))) < 1e-5


@pytest.mark.parametrize("name", sorted(fixture_configs()))
def test_golden_configs_layer_by_layer(oracle, vv, name):
    cfg, seed = fixture_configs()[name]
    fx = np.load(os.path.join(HERE, "golden", f"{name}.npz"))
    ref, gpu, _ = make_pair(oracle, vv, cfg, seed, 64)
    gpu.set_debug(True)
    for pos, tok in enumerate(fx["tokens"]):
        lr = ref.forward_token(int(tok), pos)
        lg = gpu.forward_token(int(tok), pos)
        for layer in range(cfg.num_hidden_layers):
            assert rel_l2(gpu.debug_hidden(layer), ref.hidden(layer)) < TIGHT_REL_L2, (pos, layer)
            assert rel_l2(gpu.debug_hidden(layer), fx["hidden"][layer, pos]) < TIGHT_REL_L2, (pos, layer)
        assert np.max(np.abs(lg - lr)) < 1e-4
        assert np.max(np.abs(lg - fx["logits"][pos])) < 1e-4
        assert gpu.last_argmax == oracle.argmax(lr)


def test_device_synthetic_weights_match_host_blob(oracle, vv):
    cfg, seed = fixture_configs()["qwen2_tiny"]
    blob = oracle.synthetic_blob(cfg, seed=seed)
    a = vv.Runner(cfg, max_seq=16)
    a.load_weights(blob)
    b = vv.Runner(cfg, max_seq=16)
    b.fill_synthetic(seed)
    for pos, tok in enumerate([5, 9, 200, 31]):
        assert np.array_equal(a.forward_token(tok, pos), b.forward_token(tok, pos))


def check_layers(gpu, ref, cfg, where):
    """Per-layer residual stream of the last forward against the oracle."""
    worst = 0.0
    for layer in range(cfg.num_hidden_layers):
        err = rel_l2(gpu.debug_hidden(layer), ref.hidden(layer))
        assert err < HIDDEN_REL_L2, (where, layer, err)
        worst = max(worst, err)
    return worst


def divergence(gpu_tokens, ref_tokens, ref_logits_per_step=None):
    """Message for the first index where two greedy streams differ, with the
    oracle's top-2 logit gap at that step when its logits are known."""
    i = next((i for i, (a, b) in enumerate(zip(gpu_tokens, ref_tokens)) if a != b), None)
    if i is None:
        return f"streams differ in length: {len(gpu_tokens)} vs {len(ref_tokens)}"
    msg = f"first divergence at generated token {i}: gpu {gpu_tokens[i]} vs oracle {ref_tokens[i]}"
    if ref_logits_per_step is not None and i < len(ref_logits_per_step):
        top = np.sort(ref_logits_per_step[i])[-2:]
        msg += f"; oracle top-2 gap {float(top[1] - top[0]):.3e}"
    return msg


def stream_parity(oracle, vv, cfg, seed, n_prompt, n_new, max_seq, min_distinct=8):
    """The north-star contract on one architecture: every prompt and decode
    position's per-layer hidden states (1e-2 rel L2, and 1e-4) and logits
    (2e-2 max-abs, and 1e-4) against the oracle, an identical greedy stream
    of n_new tokens from the host loop and from the device loop, and a stream
    that is not degenerate (at least `min_distinct` distinct tokens)."""
    rng = np.random.default_rng(1)
    prompt = rng.integers(0, cfg.vocab_size, size=n_prompt).tolist()
    ref = oracle.RefRunner(cfg, synthetic_seed=seed, max_seq=max_seq)
    ref.set_attention_threads(os.cpu_count() or 1)
    gpu = vv.Runner(cfg, max_seq=max_seq)
    gpu.fill_synthetic(seed)
    gpu.set_debug(True)
    worst_h = worst_l = 0.0
    for pos, tok in enumerate(prompt):
        lr = ref.forward_token(tok, pos)
        lg = gpu.forward_token(tok, pos)
        worst_h = max(worst_h, check_layers(gpu, ref, cfg, ("prompt", pos)))
        worst_l = max(worst_l, float(np.max(np.abs(lg - lr))))
    # greedy decode, host loop: the oracle's argmax is fed to both
    ref_tokens, ref_logits = [], []
    for i in range(n_new):
        tok = oracle.argmax(lr)
        ref_tokens.append(tok)
        ref_logits.append(lr)
        assert gpu.last_argmax == tok, divergence(ref_tokens[:i] + [gpu.last_argmax], ref_tokens, ref_logits)
        if i + 1 == n_new:
            break
        pos = n_prompt + i
        lr = ref.forward_token(tok, pos)
        lg = gpu.forward_token(tok, pos)
        worst_h = max(worst_h, check_layers(gpu, ref, cfg, ("decode", pos)))
        worst_l = max(worst_l, float(np.max(np.abs(lg - lr))))
    assert worst_l < LOGIT_MAX_ABS, worst_l
    assert worst_h < TIGHT_REL_L2 and worst_l < 1e-4, (worst_h, worst_l)
    assert len(set(ref_tokens)) >= min_distinct, ref_tokens
    # the device loop (prefill + graph/megakernel replays) gives the same stream
    gpu.set_debug(False)
    gpu.reset()
    gpu_tokens, stats = gpu.generate_greedy(prompt, n_new)
    assert stats.generated_tokens == n_new
    assert gpu_tokens == ref_tokens, divergence(gpu_tokens, ref_tokens, ref_logits)


def test_qwen2_5_0_5b_architecture(oracle, vv):
    stream_parity(oracle, vv, C.qwen2_5_0_5b(), seed=0, n_prompt=8, n_new=32, max_seq=512)


def test_llama3_2_1b_architecture_with_rope_scaling(oracle, vv):
    stream_parity(oracle, vv, C.llama3_2_1b(), seed=0, n_prompt=8, n_new=32, max_seq=512)


def test_llama3_8b_architecture(oracle, vv):
    # The benchmarked configuration: 32-token prompt, 32 greedy tokens, every
    # layer at every position.
    stream_parity(oracle, vv, C.llama3_8b(), seed=0, n_prompt=32, n_new=32, max_seq=128)


def cut(cfg, layers=2, vocab=32000):
    """The same layer shapes with fewer layers and a smaller vocabulary, so the
    oracle can run thousands of positions in seconds."""
    return dataclasses.replace(cfg, num_hidden_layers=layers, vocab_size=vocab, eos_token_id=0, pad_token_id=0)


def long_context_parity(oracle, vv, cfg, n_prompt, n_new, seed=0):
    """Tensor-core prefill of a prompt longer than one 2,048-token chunk, then
    greedy decode at positions past 16 KV pages per split group (1,024
    positions), against the oracle: the last prompt token's per-layer hidden
    states and logits, every decode step's hidden states and logits (host
    loop), and the device decode loop's stream."""
    max_seq = n_prompt + n_new + 8
    prompt = np.random.default_rng(7).integers(0, cfg.vocab_size, size=n_prompt).tolist()
    ref = oracle.RefRunner(cfg, synthetic_seed=seed, max_seq=max_seq)
    ref.set_attention_threads(os.cpu_count() or 1)
    a = vv.Runner(cfg, max_seq=max_seq)
    a.fill_synthetic(seed)
    b = vv.Runner(cfg, max_seq=max_seq)
    b.fill_synthetic(seed)
    assert a.query("tc_prefill") == 1
    a.set_debug(True)
    lr = ref.prefill(prompt, 0)
    la = a.prefill(prompt, 0)
    lb = b.prefill(prompt, 0)
    assert np.array_equal(la, lb)
    check_layers(a, ref, cfg, ("prefill", n_prompt - 1))
    assert np.max(np.abs(la - lr)) < LOGIT_MAX_ABS
    ref_tokens, ref_logits = [], []
    for i in range(n_new):
        tok = oracle.argmax(lr)
        ref_tokens.append(tok)
        ref_logits.append(lr)
        assert a.last_argmax == tok, divergence(ref_tokens[:i] + [a.last_argmax], ref_tokens, ref_logits)
        if i + 1 == n_new:
            break
        pos = n_prompt + i
        lr = ref.forward_token(tok, pos)
        lg = a.forward_token(tok, pos)
        check_layers(a, ref, cfg, ("decode", pos))
        assert np.max(np.abs(lg - lr)) < LOGIT_MAX_ABS, pos
    assert len(set(ref_tokens)) >= 8, ref_tokens
    # device loop from b's prefilled cache: its first token is the prefill's argmax
    assert b.last_argmax == ref_tokens[0]
    got, _ = b.decode(n_new - 1)
    assert got == ref_tokens[1:], divergence(got, ref_tokens[1:], ref_logits[1:])


def test_llama3_8b_shapes_two_chunk_prefill_and_long_decode(oracle, vv):
    # head_dim 128, group 4: a 2,100-token prompt (chunks of 2,048 + 52), then
    # decode at positions 2,100-2,131 (34 pages over 16 split groups).
    long_context_parity(oracle, vv, cut(C.llama3_8b()), n_prompt=2100, n_new=32)


def test_llama3_2_1b_shapes_three_chunk_prefill_and_long_decode(oracle, vv):
    # head_dim 64, group 4, llama3 rope scaling: a 4,100-token prompt (chunks
    # of 2,048 + 2,048 + 4), then decode at positions 4,100-4,131.
    long_context_parity(oracle, vv, cut(C.llama3_2_1b()), n_prompt=4100, n_new=32)


def test_prefill_equals_sequential_forwards(oracle, vv):
    cfg, seed = fixture_configs()["llama3_tiny_rs"]
    blob = oracle.synthetic_blob(cfg, seed=seed)
    a = vv.Runner(cfg, max_seq=128)
    a.load_weights(blob)
    b = vv.Runner(cfg, max_seq=128)
    b.load_weights(blob)
    toks = np.random.default_rng(3).integers(0, cfg.vocab_size, size=40).tolist()
    for pos, t in enumerate(toks):
        la = a.forward_token(t, pos)
    lb = b.prefill(toks, 0)
    # prefill runs tensor-core GEMMs (bf16 hi+lo activations, fp32 accumulation)
    assert np.max(np.abs(la - lb)) < 2e-3 and a.last_argmax == b.last_argmax
    # decoding continues from the prefilled cache exactly like from the token-by-token one
    ta, _ = a.decode(8)
    tb, _ = b.decode(8)
    assert ta == tb


def test_tensor_core_prefill_long_prompt(oracle, vv):
    # Llama-3.2-1B architecture, 300-token prompt (ragged 128-row tiles), against the oracle.
    cfg = C.llama3_2_1b()
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, cfg.vocab_size, size=300).tolist()
    ref = oracle.RefRunner(cfg, synthetic_seed=0, max_seq=512)
    gpu = vv.Runner(cfg, max_seq=512)
    gpu.fill_synthetic(0)
    assert gpu.query("tc_prefill") == 1
    for pos, t in enumerate(prompt):
        lr = ref.forward_token(t, pos)
    lg = gpu.prefill(prompt, 0)
    assert np.max(np.abs(lg - lr)) < LOGIT_MAX_ABS
    assert gpu.last_argmax == oracle.argmax(lr)
    ref_tokens = []
    tok = oracle.argmax(lr)
    for pos in range(len(prompt), len(prompt) + 16):
        ref_tokens.append(tok)
        tok = oracle.argmax(ref.forward_token(tok, pos))
    got, _ = gpu.decode(15)
    assert got == ref_tokens[1:16], divergence(got, ref_tokens[1:16])


def test_generate_greedy_stops_at_eos(oracle, vv):
    cfg, seed = fixture_configs()["qwen2_tiny"]
    ref, gpu, _ = make_pair(oracle, vv, cfg, seed, 128)
    prompt = [1, 2, 3, 4]
    full = ref.generate_greedy(prompt, 40)
    eos = full[len(full) // 2]
    ref.reset()
    expect = ref.generate_greedy(prompt, 40, eos=eos)
    got, stats = gpu.generate_greedy(prompt, 40, eos_token_id=eos)
    assert got == expect and got[-1] == eos and stats.generated_tokens == len(expect)


def test_errors(oracle, vv):
    cfg = C.tiny_qwen()
    gpu = vv.Runner(cfg, max_seq=4)
    with pytest.raises(VvliError) as e:
        gpu.forward_token(1, 0)
    assert e.value.name == "WeightsNotLoaded"
    gpu.fill_synthetic(0)
    with pytest.raises(VvliError) as e:
        gpu.forward_token(cfg.vocab_size, 0)
    assert e.value.name == "InvalidToken"
    with pytest.raises(VvliError) as e:
        gpu.forward_token(1, 4)
    assert e.value.name == "ContextFull"
    with pytest.raises(VvliError) as e:
        gpu.generate_greedy([], 4)
    assert e.value.name == "EmptyPrompt"
    with pytest.raises(VvliError) as e:
        gpu.generate_greedy([1, 2], 8)  # needs positions up to 9 > max_seq 4
    assert e.value.name == "ContextFull"
    with pytest.raises(VvliError) as e:
        vv.Runner(cfg, max_seq=cfg.max_position_embeddings + 1)
    assert e.value.name == "InvalidConfig"
    # the context stays usable after errors
    gpu.reset()
    assert gpu.forward_token(1, 0).shape == (cfg.vocab_size,)


def test_fused_down_proj_plan_matches_oracle(oracle, vv, monkeypatch):
    # The opt-in megakernel plan that fuses down_proj into gate|up (transposed
    # down rows, fixed-point reduction) against the oracle, layer by layer.
    monkeypatch.setenv("VVLI_MEGA_FUSED_DOWN", "1")
    cfg, seed = fixture_configs()["llama3_tiny_rs"]
    ref, gpu, _ = make_pair(oracle, vv, cfg, seed, 64)
    assert gpu.query("megakernel") == 1
    gpu.set_debug(True)
    for pos, tok in enumerate([7, 3, 250, 19, 64, 1]):
        lr = ref.forward_token(tok, pos)
        lg = gpu.forward_token(tok, pos)
        for layer in range(cfg.num_hidden_layers):
            assert rel_l2(gpu.debug_hidden(layer), ref.hidden(layer)) < TIGHT_REL_L2, (pos, layer)
        assert np.max(np.abs(lg - lr)) < 1e-4
    gpu.set_debug(False)
    ref.reset()
    gpu.reset()
    prompt = [1, 2, 3, 4]
    assert gpu.generate_greedy(prompt, 24)[0] == ref.generate_greedy(prompt, 24)
