"""The tcgen05 tensor-core GEMM (prefill) against a SIMT reference, through the C ABI."""

import ctypes

import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K,two_a", [
    (128, 256, 64, 0),      # one tile, one k-block
    (128, 256, 128, 1),     # hi + lo operands
    (256, 512, 1024, 1),    # several tiles, ring wrap-around
    (200, 1152, 896, 1),    # ragged M and N tails (Qwen q|k|v shape)
    (512, 4096, 4096, 1),   # Llama-3-8B hidden
    (32, 256, 14336, 1),    # long K (down_proj), few tokens
])
def test_gemm_matches_reference(M, N, K, two_a):
    from vvli_b200 import _abi
    err = ctypes.c_float(0)
    st = _abi.lib().vvli_cuda_gemm_selftest(0, M, N, K, two_a, 7, ctypes.byref(err))
    assert st == 0, _abi.lib().vvli_cuda_last_error()
    assert err.value < 1e-4, err.value  # fp32 accumulation over up to 14336 terms
