"""The MoE oracle (oracle/moe_ref.py) against the fixtures that the OLMoE block of
`transformers` 5.5.0 produced (tests/golden/make_moe_golden.py).  No GPU."""

import os

import numpy as np
import pytest

from moe_ref import bf16_bits, bf16_float, make_inputs, moe_block

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "moe_olmoe.npz")


def cases():
    z = np.load(GOLDEN)
    names = sorted({k.split("__")[0] for k in z.files if "__" in k})
    return [(n, z) for n in names]


@pytest.mark.parametrize("name", [n for n, _ in cases()])
def test_oracle_matches_transformers_olmoe_block(name):
    z = np.load(GOLDEN)
    seed, T, h, inter, E, k, norm = (int(v) for v in z[f"{name}__params"])
    inp = make_inputs(seed, T, h, inter, E)
    out, idx, w = moe_block(inp["x"], inp["norm_w"], inp["router"], inp["gate_up"], inp["down"], k, bool(norm),
                            float(z["eps"][0]))
    # transformers runs in float32, the oracle in float64
    assert np.array_equal(idx, z[f"{name}__idx"])
    assert np.allclose(w, z[f"{name}__w"], rtol=2e-5, atol=1e-7)
    assert np.max(np.abs(out - z[f"{name}__out"])) < 2e-5 * max(1.0, float(np.max(np.abs(out))))


def test_bf16_round_trip_and_rounding():
    a = np.array([1.0, -2.5, 3.14159265, 1e-3, 65504.0], dtype=np.float32)
    assert np.array_equal(bf16_float(bf16_bits(a))[:2], a[:2])  # exact in bf16
    b = bf16_float(bf16_bits(a))
    assert np.all(np.abs(b - a) <= np.abs(a) * 2.0 ** -8)
    # ties go to even: 1 + 2^-8 lies halfway between 1 and 1 + 2^-7
    assert bf16_float(bf16_bits(np.float32(1.0 + 2.0 ** -8)))[()] == 1.0


def test_top_k_order_and_normalisation():
    inp = make_inputs(5, 4, 64, 32, 8)
    _, idx, w = moe_block(inp["x"], inp["norm_w"], inp["router"], inp["gate_up"], inp["down"], 3, True, 1e-5)
    assert np.allclose(w.sum(axis=1), 1.0)
    assert np.all(np.diff(w, axis=1) <= 0)  # larger probability first
    assert all(len(set(r)) == 3 for r in idx.tolist())


def test_top_k_equal_to_experts_uses_every_expert():
    inp = make_inputs(6, 2, 64, 32, 4)
    out_all, idx, w = moe_block(inp["x"], inp["norm_w"], inp["router"], inp["gate_up"], inp["down"], 4, False, 1e-5)
    assert sorted(idx[0].tolist()) == [0, 1, 2, 3]
    assert np.allclose(w.sum(axis=1), 1.0)  # the softmax over all experts sums to one
