"""vvli_cuda_moe_ffn (OLMoE sparse block) against oracle/moe_ref.py and the
fixtures of the transformers OLMoE block.  Needs a B200."""

import os

import numpy as np
import pytest

from moe_ref import make_inputs, moe_block

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "moe_olmoe.npz")
# fp32 on the GPU (other summation orders) against the float64 oracle
TOL = 3e-5


@pytest.fixture(scope="module")
def torch():
    import torch
    assert torch.cuda.is_available()
    return torch


def run_gpu(torch, inp, top_k, norm, eps=1e-5, tokens=None):
    from vvli_b200.moe import MoeFfn
    block = MoeFfn(inp["norm_w"], inp["router"], inp["gate_up"], inp["down"], top_k, norm, eps)
    x_host = inp["x"] if tokens is None else inp["x"][:tokens]
    x = torch.from_numpy(np.ascontiguousarray(x_host)).cuda()
    idx, w = block(x, routing=True)
    torch.cuda.synchronize()
    return x.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy(), block


def close(got, want):
    return float(np.max(np.abs(got - want))) / max(1.0, float(np.max(np.abs(want))))


@pytest.mark.parametrize("name", ["olmoe_like", "normed_topk", "ragged_dims"])
def test_matches_transformers_fixtures(torch, name):
    z = np.load(GOLDEN)
    seed, T, h, inter, E, k, norm = (int(v) for v in z[f"{name}__params"])
    inp = make_inputs(seed, T, h, inter, E)
    out, idx, w, _ = run_gpu(torch, inp, k, bool(norm), float(z["eps"][0]))
    assert np.array_equal(idx, z[f"{name}__idx"])
    assert np.allclose(w, z[f"{name}__w"], rtol=1e-5, atol=1e-7)
    assert close(out, z[f"{name}__out"]) < TOL


@pytest.fixture(scope="module")
def olmoe_inputs():
    # OLMoE-1B-7B block shape: h 2048, 64 experts of I 1024, 8 per token
    return make_inputs(21, 32, 2048, 1024, 64)


@pytest.mark.parametrize("T", [1, 5, 16, 32])
def test_olmoe_1b_7b_shape(torch, olmoe_inputs, T):
    inp = dict(olmoe_inputs, x=olmoe_inputs["x"][:T])
    want, widx, ww = moe_block(inp["x"], inp["norm_w"], inp["router"], inp["gate_up"], inp["down"], 8, False, 1e-5)
    out, idx, w, _ = run_gpu(torch, inp, 8, False)
    assert np.array_equal(idx, widx)
    assert np.allclose(w, ww, rtol=1e-5, atol=1e-7)
    assert close(out, want) < TOL


def test_many_tokens_per_expert_and_ties(torch):
    # a zero router gives every expert the same probability: every token takes
    # experts 0..k-1 (lower index first), so each of them serves all 37 tokens
    # (thirteen passes of at most three tokens over its weight tiles)
    inp = make_inputs(31, 37, 512, 256, 16)
    inp["router"] = np.zeros_like(inp["router"])
    want, widx, ww = moe_block(inp["x"], inp["norm_w"], inp["router"], inp["gate_up"], inp["down"], 6, True, 1e-5)
    out, idx, w, _ = run_gpu(torch, inp, 6, True)
    assert np.array_equal(idx, np.tile(np.arange(6, dtype=np.int32), (37, 1)))
    assert np.array_equal(idx, widx)
    assert np.allclose(w, 1.0 / 6, rtol=1e-6)
    assert close(out, want) < TOL


def test_top_k_all_experts_and_one_expert(torch):
    for E, k in ((4, 4), (1, 1)):
        inp = make_inputs(41 + E, 3, 128, 64, E)
        want, widx, _ = moe_block(inp["x"], inp["norm_w"], inp["router"], inp["gate_up"], inp["down"], k, False, 1e-6)
        out, idx, _, _ = run_gpu(torch, inp, k, False, 1e-6)
        assert np.array_equal(idx, widx)
        assert close(out, want) < TOL


def test_deterministic_and_workspace_reused(torch):
    inp = make_inputs(51, 9, 256, 128, 16)
    a, _, _, block = run_gpu(torch, inp, 4, False)
    x = torch.from_numpy(inp["x"]).cuda()
    block(x)
    torch.cuda.synchronize()
    assert np.array_equal(x.cpu().numpy(), a)  # bitwise: fixed summation orders


def test_errors_on_the_gpu_path(torch):
    from vvli_b200.errors import VvliError
    from vvli_b200.moe import MoeFfn
    inp = make_inputs(61, 2, 64, 32, 4)
    block = MoeFfn(inp["norm_w"], inp["router"], inp["gate_up"], inp["down"], 5, False)  # top_k > experts
    with pytest.raises(VvliError) as e:
        block(torch.from_numpy(inp["x"]).cuda())
    assert e.value.name == "InvalidArgument"
    block = MoeFfn(inp["norm_w"], inp["router"], inp["gate_up"], inp["down"], 2, False)
    buf = torch.zeros(2 * 64 + 1, dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError):
        block(buf[1:].view(2, 64)[:, :32])  # not contiguous
