"""The C-ABI library loads and exports every function include/vvli_cuda.h declares.

No compute calls: these run without a GPU.
"""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "vvli_cuda.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(vvli_cuda_\w+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for required in ("vvli_cuda_create", "vvli_cuda_load_weights", "vvli_cuda_forward_token",
                     "vvli_cuda_forward_embedding", "vvli_cuda_prefill", "vvli_cuda_generate_greedy",
                     "vvli_cuda_reset", "vvli_cuda_destroy", "vvli_cuda_strerror"):
        assert required in names


def test_library_exports_every_declared_symbol():
    from vvli_b200 import _abi
    lib = _abi.lib()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert set(declared_functions()) == set(_abi.SIGNATURES)


def test_strerror_and_storage_elements_without_gpu():
    from vvli_b200 import _abi
    from vvli_b200 import config as C
    assert _abi.strerror(0) == "ok"
    assert _abi.strerror(1) == "ContextFull"
    assert _abi.strerror(3) == "InvalidToken"
    for cfg in (C.tiny_qwen(), C.qwen2_5_0_5b(), C.llama3_8b()):
        c = cfg.to_c()
        n = ctypes.c_uint64(0)
        assert _abi.lib().vvli_cuda_storage_elements(ctypes.byref(c), ctypes.byref(n)) == 0
        assert n.value == cfg.storage_element_count()


def test_strerror_names_every_status():
    from vvli_b200 import _abi
    from vvli_b200.errors import CODES
    for code, name in CODES.items():
        assert _abi.strerror(code) == name, code


def test_config_struct_matches_c_layout():
    from vvli_b200.config import CModelConfig
    assert ctypes.sizeof(CModelConfig) == 9 * 8 + 14 * 4 + 8 == 136
