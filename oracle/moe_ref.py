"""CPU restatement of a mixture-of-experts feed-forward block (TEST INFRASTRUCTURE ONLY).

Imported only by tests/, tests/golden/make_moe_golden.py and bench.py's CPU
arm, as the checker -- never by the product package.

The reference parses OLMoE configs (num_experts, num_experts_per_tok:
src/llm.zig:45-48, 111-133, 210-214) and counts their parameters
(src/llm.zig:261-264), then rejects the model before any arithmetic
(src/main.zig:590-611).  It holds no MoE computation to restate.  The
arithmetic here follows the published OLMoE block of the third-party
`transformers` package, version 5.5.0 (models/olmoe/modeling_olmoe.py:
OlmoeTopKRouter, OlmoeExperts, OlmoeSparseMoeBlock), which is not part of
the reference.  tests/golden/make_moe_golden.py runs that block on the
seeded inputs of make_inputs() and commits its outputs; test_moe_oracle.py
pins this restatement to them.

For a token row x of the residual stream:
  xn = x / sqrt(mean(x^2) + eps) * norm_w      (rmsNormInto, src/llm.zig:1287-1300)
  p  = softmax(router . xn) over all experts
  the top_k experts by p (larger first; lower index on ties), weights
  w = p[top] (divided by their sum when norm_topk_prob)
  y  = sum over the chosen experts, in ascending expert index, of
       w_e * down_e . (silu(gate_e . xn) * (up_e . xn))
  x_out = x + y
Weight layouts: router [E][h], gate_up [E][2I][h] (the I gate rows, then the
I up rows), down [E][h][I]; all bf16 values.
"""

from __future__ import annotations

import numpy as np


def bf16_bits(a) -> np.ndarray:
    """float32 -> bf16 bit patterns, rounded to nearest even (finite inputs)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    return ((u + (((u >> 16) & 1) + 0x7FFF)) >> 16).astype(np.uint16)


def bf16_float(bits) -> np.ndarray:
    """bf16 bit patterns -> float32."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def make_inputs(seed: int, tokens: int, hidden: int, inter: int, experts: int) -> dict:
    """Seeded inputs: x ~ N(0, 1); weights scaled so router logits and the
    expert rows' dot products are O(1); every weight a bf16 value (uint16 bits)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((tokens, hidden), dtype=np.float32)
    norm_w = bf16_bits(1.0 + 0.1 * rng.standard_normal(hidden, dtype=np.float32))
    router = bf16_bits(rng.standard_normal((experts, hidden), dtype=np.float32) * np.float32(1.5 / np.sqrt(hidden)))
    gate_up = bf16_bits(rng.standard_normal((experts, 2 * inter, hidden), dtype=np.float32) * np.float32(1.0 / np.sqrt(hidden)))
    down = bf16_bits(rng.standard_normal((experts, hidden, inter), dtype=np.float32) * np.float32(1.0 / np.sqrt(inter)))
    return {"x": x, "norm_w": norm_w, "router": router, "gate_up": gate_up, "down": down}


def route(xn: np.ndarray, router_f: np.ndarray, top_k: int, norm_topk_prob: bool):
    """Router probabilities and the top-k choice of every row (float64)."""
    logits = xn @ router_f.T
    logits = logits - logits.max(axis=1, keepdims=True)
    p = np.exp(logits)
    p /= p.sum(axis=1, keepdims=True)
    idx = np.argsort(-p, axis=1, kind="stable")[:, :top_k]  # larger first, lower index on ties
    w = np.take_along_axis(p, idx, axis=1)
    if norm_topk_prob:
        w = w / w.sum(axis=1, keepdims=True)
    return p, idx.astype(np.int32), w


def moe_block(x, norm_w, router, gate_up, down, top_k: int, norm_topk_prob: bool, eps: float):
    """x_out, chosen experts [T][k] (larger probability first) and their weights.

    Weights are bf16 bit patterns (uint16); the arithmetic is float64."""
    x = np.asarray(x, dtype=np.float64)
    T, h = x.shape
    E, two_i, _ = gate_up.shape
    inter = two_i // 2
    nw = bf16_float(norm_w).astype(np.float64)
    xn = x / np.sqrt((x * x).mean(axis=1, keepdims=True) + eps) * nw
    _, idx, w = route(xn, bf16_float(router).astype(np.float64), top_k, norm_topk_prob)
    y = np.zeros_like(x)
    # experts in ascending index, each once; a token's contributions are
    # therefore added in ascending expert index
    for e in np.unique(idx):
        rows, slots = np.nonzero(idx == e)
        gu = bf16_float(gate_up[e]).astype(np.float64)
        dn = bf16_float(down[e]).astype(np.float64)
        a = xn[rows] @ gu.T
        g, u = a[:, :inter], a[:, inter:]
        f = g / (1.0 + np.exp(-g)) * u
        y[rows] += w[rows, slots][:, None] * (f @ dn.T)
    return x + y, idx, w
