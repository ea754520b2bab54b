"""Generates tests/golden/moe_olmoe.npz: outputs of the OLMoE block of the
`transformers` package (version 5.5.0, models/olmoe/modeling_olmoe.py) on the
seeded inputs of oracle/moe_ref.py's make_inputs().

Only the case parameters and the block's outputs are stored; the inputs are
regenerated from the seeds (numpy's PCG64 stream is stable across
platforms).  Each case runs OlmoeRMSNorm (the post-attention norm) and
OlmoeSparseMoeBlock in float32 with the eager experts loop, then adds the
residual, as OlmoeDecoderLayer does:
    x_out = x + moe(rmsnorm(x))
and records the router's top-k indices and weights.

Run from the repository root:  python tests/golden/make_moe_golden.py
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(HERE)), "oracle"))

from moe_ref import bf16_float, make_inputs  # noqa: E402

# (name, seed, tokens, hidden, inter, experts, top_k, norm_topk_prob)
CASES = [
    ("olmoe_like", 11, 5, 256, 128, 16, 4, False),
    ("normed_topk", 12, 3, 128, 64, 8, 2, True),
    ("ragged_dims", 13, 7, 264, 72, 12, 3, False),
]
EPS = 1e-5


def run_case(seed, tokens, hidden, inter, experts, top_k, norm_topk_prob):
    from transformers import OlmoeConfig
    from transformers.models.olmoe.modeling_olmoe import OlmoeRMSNorm, OlmoeSparseMoeBlock

    cfg = OlmoeConfig(hidden_size=hidden, intermediate_size=inter, num_experts=experts,
                      num_experts_per_tok=top_k, norm_topk_prob=norm_topk_prob, rms_norm_eps=EPS)
    cfg._experts_implementation = "eager"
    inp = make_inputs(seed, tokens, hidden, inter, experts)
    norm = OlmoeRMSNorm(hidden, eps=EPS)
    block = OlmoeSparseMoeBlock(cfg)
    with torch.no_grad():
        norm.weight.copy_(torch.from_numpy(bf16_float(inp["norm_w"])))
        block.gate.weight.copy_(torch.from_numpy(bf16_float(inp["router"])))
        block.experts.gate_up_proj.copy_(torch.from_numpy(bf16_float(inp["gate_up"])))
        block.experts.down_proj.copy_(torch.from_numpy(bf16_float(inp["down"])))
        x = torch.from_numpy(inp["x"]).reshape(1, tokens, hidden)
        xn = norm(x)
        _, w, idx = block.gate(xn.reshape(tokens, hidden))
        y = block(xn)
        out = (x + y).reshape(tokens, hidden)
    return out.numpy().astype(np.float32), idx.numpy().astype(np.int32), w.numpy().astype(np.float32)


def main():
    torch.manual_seed(0)
    arrays = {}
    for name, seed, T, h, inter, E, k, norm in CASES:
        out, idx, w = run_case(seed, T, h, inter, E, k, norm)
        arrays[f"{name}__params"] = np.array([seed, T, h, inter, E, k, int(norm)], dtype=np.int64)
        arrays[f"{name}__out"] = out
        arrays[f"{name}__idx"] = idx
        arrays[f"{name}__w"] = w
    arrays["eps"] = np.array([EPS], dtype=np.float64)
    path = os.path.join(HERE, "moe_olmoe.npz")
    np.savez_compressed(path, **arrays)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
