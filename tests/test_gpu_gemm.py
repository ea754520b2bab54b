"""The tcgen05 tensor-core GEMMs (prefill and decode batch) against a SIMT reference, through the C ABI."""

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
    (1536, 2048, 256, 1),   # enough tiles for the 256-wide residual tiles
])
def test_gemm_matches_reference(M, N, K, two_a):
    from vvli_b200 import _abi
    err = ctypes.c_float(0)
    st = _abi.lib().vvli_cuda_gemm_selftest(0, 0, M, N, K, two_a, 7, ctypes.byref(err))
    assert st == 0, _abi.lib().vvli_cuda_last_error()
    assert err.value < 1e-4, err.value  # fp32 accumulation over up to 14336 terms


@pytest.mark.parametrize("M,N,K", [
    (128, 256, 64),      # one tile, one k-block: a single CTA, nothing split
    (200, 1152, 896),    # 10 tiles x 14 k-blocks over 35 CTAs: tiles split 4-5 ways
    (512, 4096, 4096),   # 128 tiles: waves 86% full, whole tiles only
    (512, 6144, 4096),   # Llama-3-8B q|k|v on 512 tokens: 96 tiles in groups of 4 row tiles
    (256, 4096, 14336),  # down_proj: 64 tiles x 224 k-blocks
    (1536, 2048, 256),   # 96 tiles of 4 k-blocks over groups of 12: whole tiles, nothing split
    (512, 28672, 512),   # 448 tiles (3.03 waves): two waves of whole tiles, then 152 tiles shared
])
def test_streamk_gemm_matches_reference(M, N, K):
    # kernel 3: the stream-K schedule prefill uses; the self-test also runs it
    # a second time over the same flags (the next epoch) and requires the
    # same result bit for bit
    from vvli_b200 import _abi
    err = ctypes.c_float(0)
    st = _abi.lib().vvli_cuda_gemm_selftest(0, 3, M, N, K, 1, 5, ctypes.byref(err))
    assert st == 0, _abi.lib().vvli_cuda_last_error()
    assert err.value < 1e-4, err.value


@pytest.mark.parametrize("M,N,K", [
    (256, 256, 64),      # one CTA pair, one k-block
    (256, 256, 1024),    # ring wrap-around (16 k-blocks over 4 stages)
    (200, 512, 256),     # the second CTA's rows partly past M
    (384, 1152, 896),    # ragged M and N tails (Qwen q|k|v shape)
    (512, 6144, 4096),   # Llama-3-8B q|k|v on 512 tokens: 48 pair tiles
    (1024, 4096, 14336), # long K (down_proj)
    (4096, 512, 128),    # many row tiles, both accumulators in turn
])
def test_cta_pair_gemm_matches_reference(M, N, K):
    # kernel 2: 256-row tiles on CTA pairs (cta_group::2), each CTA loading its
    # own rows of A and half of the weight tile
    from vvli_b200 import _abi
    err = ctypes.c_float(0)
    st = _abi.lib().vvli_cuda_gemm_selftest(0, 2, M, N, K, 1, 13, ctypes.byref(err))
    assert st == 0, _abi.lib().vvli_cuda_last_error()
    assert err.value < 1e-4, err.value


@pytest.mark.parametrize("M,N,K", [
    (1, 256, 64),        # one row, one k-block, no split
    (5, 4096, 4096),     # 32 weight tiles: K split over clusters of 4
    (16, 6144, 4096),    # Llama-3-8B q|k|v, clusters of 3
    (17, 4096, 14336),   # 32-row MMA, long K (down_proj) split 4 ways
    (32, 28672, 4096),   # gate|up sized, 224 tiles, no split
    (8, 1152, 896),      # Qwen q|k|v: 9 tiles, clusters of 8 over 14 k-blocks
    (3, 130, 64),        # ragged weight tile
])
def test_decode_batch_gemm_matches_reference(M, N, K):
    from vvli_b200 import _abi
    err = ctypes.c_float(0)
    st = _abi.lib().vvli_cuda_gemm_selftest(0, 1, M, N, K, 1, 11, ctypes.byref(err))
    assert st == 0, _abi.lib().vvli_cuda_last_error()
    assert err.value < 1e-4, err.value
