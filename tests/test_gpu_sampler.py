"""Device Sampler.next (vvli_cuda_sample) against the oracle's restatement.

The oracle's ref_sampler_next (oracle/vvli_ref_cpu.cpp, following
src/generator.zig:97-126, 338-463) gets the uniform draw that random.float(f32)
produces from the same xoshiro256++ state, so the comparison is exact: the
token, and the state the device leaves behind (advanced only when the
reference draws).  Cases cover the greedy-with-penalties path, top-k in the
one-CTA path (k <= 4096) and the sorted-vocabulary path (top_k 0 or > 4096),
top-p cuts, repeat penalties, ties, NaN and infinities.
"""

import dataclasses
import os
import sys
import types

import numpy as np
import pytest

from vvli_b200 import config as C
from vvli_b200 import sampler as S
from vvli_b200.errors import VvliError

pytestmark = pytest.mark.gpu

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))


def opts(T, top_p, top_k, rp, last_n):
    return types.SimpleNamespace(temperature=T, top_p=top_p, top_k=top_k, repeat_penalty=rp, repeat_last_n=last_n,
                                 seed=None)


@pytest.fixture(scope="module")
def vv():
    import vvli_b200
    return vvli_b200


def runner_with_vocab(vv, V):
    cfg = dataclasses.replace(C.tiny_qwen(), vocab_size=V, tie_word_embeddings=False)
    r = vv.Runner(cfg, max_seq=8)
    r.fill_synthetic(0)
    return r


def expected(oracle, logits, prompt, generated, o, state):
    """(token, state after) of the reference for the given xoshiro state."""
    x = S.Xoshiro256(0)
    x.s = [int(v) for v in state]
    u = x.float32()
    tok = oracle.sampler_next(logits, prompt, generated, o, u)
    counts = S.repeat_counts(logits.size, prompt, generated, o)
    drawn = o.temperature > 0 and bool(np.isfinite(S.adjusted(logits, counts, o.repeat_penalty)).any())
    return tok, (np.array(x.s, dtype=np.uint64) if drawn else state.copy())


def logits_cases(V, rng):
    out = []
    for scale in (0.05, 1.0, 8.0):
        out.append((rng.standard_normal(V) * scale).astype(np.float32))
    q = (np.round(rng.standard_normal(V) * 3) / 4).astype(np.float32)  # many ties
    out.append(q)
    a = rng.standard_normal(V).astype(np.float32)
    a[rng.integers(0, V, V // 10)] = np.nan
    a[rng.integers(0, V, V // 10)] = -np.inf
    out.append(a)
    b = rng.standard_normal(V).astype(np.float32)
    b[0] = np.nan
    b[V // 3] = np.inf
    out.append(b)
    out.append(np.full(V, 0.25, np.float32))
    c = np.full(V, -np.inf, np.float32)
    c[[7, V - 2]] = [1.0, 1.0]
    out.append(c)
    out.append(np.full(V, np.nan, np.float32))  # no candidate: argmax of the raw logits
    return out


OPTION_GRID = [
    (0.0, 1.0, 40, 1.0, 64), (0.0, 1.0, 40, 1.3, 64), (0.8, 0.95, 40, 1.1, 64), (1.5, 1.0, 40, 1.0, 0),
    (0.8, 0.3, 1, 1.1, 64), (0.01, 0.95, 40, 1.1, 64), (1.0, 0.9, 4096, 1.1, 16), (1.0, 0.5, 4097, 1.1, 64),
    (0.7, 1.0, 0, 1.0, 64), (1.2, 0.95, 0, 2.0, 64),
]


@pytest.mark.parametrize("V", [5000, 150000])
def test_device_sampler_matches_oracle(oracle, vv, V):
    rng = np.random.default_rng(V)
    r = runner_with_vocab(vv, V)
    state = np.array(S.Xoshiro256(1234).s, dtype=np.uint64)
    prompt = rng.integers(0, V, 40).tolist()
    generated = rng.integers(0, V, 30).tolist() + [V + 5]  # out-of-vocab ids are ignored
    checked = 0
    for li, lg in enumerate(logits_cases(V, rng)):
        for T, top_p, top_k, rp, last_n in OPTION_GRID:
            o = opts(T, top_p, top_k, rp, last_n)
            want_tok, want_state = expected(oracle, lg, prompt, generated, o, state)
            recent = prompt + generated
            got = r.sample(o, recent[max(0, len(recent) - last_n):] if last_n else [], state, logits=lg)
            assert got == want_tok, (li, (T, top_p, top_k, rp, last_n))
            assert np.array_equal(state, want_state), (li, (T, top_p, top_k, rp, last_n))
            checked += 1
    assert checked == len(OPTION_GRID) * len(logits_cases(V, np.random.default_rng(0)))
    r.close()


@pytest.mark.parametrize("last_n", [256, 257, 4096, 5000])
def test_device_sampler_long_repeat_windows(oracle, vv, last_n):
    # The top-k step takes up to 256 recent tokens in its launch parameters,
    # up to 4096 through one copy, and more as per-token stamps.
    V = 150000
    rng = np.random.default_rng(last_n)
    r = runner_with_vocab(vv, V)
    state = np.array(S.Xoshiro256(99).s, dtype=np.uint64)
    recent = rng.integers(0, V, last_n + 10).tolist()
    for lg in logits_cases(V, rng)[:3]:
        lg = lg.copy()
        lg[recent[-5:]] += 20.0  # the penalised tokens would win without the penalty
        for top_k, rp in ((40, 1.3), (64, 4.0), (1, 1.1)):
            o = opts(0.9, 0.95, top_k, rp, last_n)
            want_tok, want_state = expected(oracle, lg, recent, [], o, state)
            got = r.sample(o, recent[len(recent) - last_n:], state, logits=lg)
            assert got == want_tok, (last_n, top_k, rp)
            assert np.array_equal(state, want_state), (last_n, top_k, rp)
    r.close()


def test_device_sampler_on_forward_logits(oracle, vv):
    # The logits of the last forward stay on the device; same result as passing them in.
    from make_golden import fixture_configs
    cfg, seed = fixture_configs()["qwen2_tiny"]
    r = vv.Runner(cfg, max_seq=64)
    r.fill_synthetic(seed)
    o = opts(0.9, 0.95, 40, 1.1, 64)
    smp = S.DeviceSampler(cfg.vocab_size, types.SimpleNamespace(seed=7))
    prompt = [3, 17, 99, 5]
    generated = []
    lg = r.prefill(prompt, 0)
    pos = len(prompt)
    for _ in range(24):
        state0 = smp.state.copy()
        want, want_state = expected(oracle, lg, prompt, generated, o, state0)
        got = smp.next(r, prompt, generated, o)
        assert got == want and np.array_equal(smp.state, want_state)
        generated.append(got)
        lg = r.forward_token(got, pos)
        pos += 1


def test_generate_measured_samples_on_device(oracle, vv):
    from make_golden import fixture_configs
    cfg, seed = fixture_configs()["llama3_tiny_rs"]
    r = vv.Runner(cfg, max_seq=128)
    r.fill_synthetic(seed)
    o = vv.Options(max_new_tokens=20, temperature=0.8, top_p=0.95, top_k=40, repeat_penalty=1.1, repeat_last_n=64,
                   seed=42)
    prompt = [1, 2, 3, 4, 5]
    res = vv.generate_greedy_measured(r, prompt, o)
    assert len(res.tokens) == 20
    # replay on the host: the same logits (GPU forwards), the oracle's sampler, the host PRNG
    r.reset()
    x = S.Xoshiro256(42)
    lg = r.prefill(prompt, 0)
    gen = []
    for pos in range(len(prompt), len(prompt) + 20):
        tok = oracle.sampler_next(lg, prompt, gen, o, x.float32())
        gen.append(tok)
        lg = r.forward_token(tok, pos)
    assert gen == res.tokens


def test_invalid_sampling_options(vv):
    r = runner_with_vocab(vv, 64)
    state = np.array(S.Xoshiro256(1).s, dtype=np.uint64)
    for bad in (opts(-1.0, 0.9, 40, 1.1, 64), opts(0.8, 0.0, 40, 1.1, 64), opts(0.8, 1.5, 40, 1.1, 64),
                opts(0.8, 0.9, 40, 0.5, 64), opts(float("nan"), 0.9, 40, 1.1, 64)):
        with pytest.raises(VvliError) as e:
            r.sample(bad, [], state, logits=np.zeros(64, np.float32))
        assert e.value.name == "InvalidSamplingOptions"
