"""Parity of the CUDA decoder (through the C ABI) against the CPU oracle.

Contract: per-layer hidden states within 1e-2
relative L2, logits within 2e-2 max-abs after the final norm, and identical
greedy token streams over the first 32 tokens.  The GPU path computes in fp32
like the reference, so tighter bounds are asserted too where they hold.
"""

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


def greedy_parity(oracle, vv, cfg, seed, n_prompt, n_new, max_seq, check_layers=True):
    rng = np.random.default_rng(1)
    prompt = rng.integers(0, cfg.vocab_size, size=n_prompt).tolist()
    ref = oracle.RefRunner(cfg, synthetic_seed=seed, max_seq=max_seq)
    gpu = vv.Runner(cfg, max_seq=max_seq)
    gpu.fill_synthetic(seed)
    if check_layers:
        gpu.set_debug(True)
        worst_h = worst_l = 0.0
        for pos, tok in enumerate(prompt):
            lr = ref.forward_token(tok, pos)
            lg = gpu.forward_token(tok, pos)
            for layer in range(cfg.num_hidden_layers):
                worst_h = max(worst_h, rel_l2(gpu.debug_hidden(layer), ref.hidden(layer)))
            worst_l = max(worst_l, float(np.max(np.abs(lg - lr))))
        assert worst_h < HIDDEN_REL_L2 and worst_l < LOGIT_MAX_ABS, (worst_h, worst_l)
        assert worst_h < TIGHT_REL_L2, worst_h
        gpu.set_debug(False)
        ref.reset()
        gpu.reset()
    ref_tokens = ref.generate_greedy(prompt, n_new)
    gpu_tokens, stats = gpu.generate_greedy(prompt, n_new)
    assert stats.generated_tokens == n_new
    assert gpu_tokens == ref_tokens, next(i for i, (a, b) in enumerate(zip(gpu_tokens, ref_tokens)) if a != b)


def test_qwen2_5_0_5b_architecture(oracle, vv):
    greedy_parity(oracle, vv, C.qwen2_5_0_5b(), seed=0, n_prompt=8, n_new=32, max_seq=512)


def test_llama3_2_1b_architecture_with_rope_scaling(oracle, vv):
    greedy_parity(oracle, vv, C.llama3_2_1b(), seed=0, n_prompt=8, n_new=32, max_seq=512)


def test_llama3_8b_architecture(oracle, vv):
    greedy_parity(oracle, vv, C.llama3_8b(), seed=0, n_prompt=4, n_new=8, max_seq=64, check_layers=False)


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
    got, _ = gpu.decode(16)
    assert [gpu.last_argmax] and got[:15] == ref_tokens[1:16]


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
