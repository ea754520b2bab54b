"""Tensor-core prompt attention (tcgen05) against the SIMT flash kernel.

The SIMT kernel is the one the prefill parity tests pin to the oracle
(computeAttentionInto, src/llm.zig:1302-1335); here both run on the same
random q, K and V, over causal ranges that start at position 0 or later,
ragged tiles and a scrambled page table.  The end-to-end prefill tests in
test_gpu_parity.py cover the tensor-core kernel against the oracle.
"""

import ctypes

import pytest

pytestmark = pytest.mark.gpu

# fp32 vs fp32 through bf16 hi + lo operands (about 16 bits per operand).
REL_TOL = 2e-4


@pytest.mark.parametrize("d,group,tokens,pos0", [
    (128, 4, 512, 0),     # Llama-3-8B heads, one 512-token chunk
    (128, 4, 200, 777),   # a later chunk: keys before the chunk, ragged last tile
    (64, 4, 300, 0),      # Llama-3.2-1B heads
    (64, 7, 93, 5),       # Qwen2.5-0.5B grouping (7 q heads per kv head)
    (64, 8, 16, 64),      # a short chunk starting on a page boundary
    (128, 1, 130, 3),     # no grouping
])
def test_attention_tc_matches_simt(d, group, tokens, pos0):
    from vvli_b200 import _abi
    err = ctypes.c_float(-1.0)
    for seed in (1, 2):
        assert _abi.lib().vvli_cuda_attention_selftest(0, d, group, tokens, pos0, seed, ctypes.byref(err)) == 0
        assert 0.0 <= err.value < REL_TOL, (d, group, tokens, pos0, seed, err.value)
