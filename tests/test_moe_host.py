"""vvli_cuda_moe_workspace_bytes and the argument checks of vvli_cuda_moe_ffn
(both run before any CUDA call: no GPU needed)."""

import ctypes

from vvli_b200 import _abi
from vvli_b200.errors import CODE_OF

INVALID = CODE_OF["InvalidArgument"]


def test_args_struct_matches_c_layout():
    assert ctypes.sizeof(_abi.CMoeArgs) == 5 * 8 + 4 + 4 + 6 * 8 + 8 + 2 * 8 == 120
    assert _abi.CMoeArgs.x.offset == 48 and _abi.CMoeArgs.workspace_bytes.offset == 96


def test_workspace_bytes():
    lib = _abi.lib()
    T, h, inter, E, k = 16, 2048, 1024, 64, 8
    n = lib.vvli_cuda_moe_workspace_bytes(T, h, inter, E, k)
    # normed rows, router logits, the pairs' silu*up rows and down rows dominate
    assert n >= 4 * (T * h + T * k * inter + T * k * h) and n % 256 == 0
    assert n < 4 * (T * h + T * E + T * k * inter + T * k * h) + 16 * 256 + 4 * (3 * E + 4 * T * k)
    for bad in ((0, h, inter, E, k), (4097, h, inter, E, k), (T, 12, inter, E, k), (T, h, 8200, E, k),
                (T, h, inter, 0, k), (T, h, inter, 1025, k), (T, h, inter, 8, 9), (T, h, inter, 64, 33),
                (T, h, inter, E, 0)):
        assert lib.vvli_cuda_moe_workspace_bytes(*bad) == 0, bad


def test_ffn_rejects_bad_arguments_before_touching_the_device():
    lib = _abi.lib()
    assert lib.vvli_cuda_moe_ffn(0, None, None) == INVALID
    a = _abi.CMoeArgs()
    a.tokens, a.hidden, a.inter, a.experts, a.top_k = 2, 64, 32, 4, 5  # top_k > experts
    assert lib.vvli_cuda_moe_ffn(0, ctypes.byref(a), None) == INVALID
    assert b"top_k" in lib.vvli_cuda_last_error()
    a.top_k = 2
    assert lib.vvli_cuda_moe_ffn(0, ctypes.byref(a), None) == INVALID  # null pointers
    assert b"null" in lib.vvli_cuda_last_error()
    a.x, a.norm_w, a.router, a.gate_up, a.down, a.workspace = 16, 16, 16, 16, 8, 256
    assert lib.vvli_cuda_moe_ffn(0, ctypes.byref(a), None) == INVALID  # down misaligned
    assert b"aligned" in lib.vvli_cuda_last_error()
    a.down, a.workspace = 16, 16
    assert lib.vvli_cuda_moe_ffn(0, ctypes.byref(a), None) == INVALID  # workspace misaligned
    a.workspace, a.workspace_bytes = 256, 1
    assert lib.vvli_cuda_moe_ffn(0, ctypes.byref(a), None) == INVALID  # workspace too small
    assert b"workspace_bytes" in lib.vvli_cuda_last_error()
