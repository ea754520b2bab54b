"""ctypes binding of libvvli_cuda.so (the C ABI declared in include/vvli_cuda.h).

The library is built in-tree by vvli_b200/csrc/Makefile.  There is no fallback:
if the shared library is missing or fails to load, ``lib()`` raises.
"""

from __future__ import annotations

import ctypes
import os

from .config import CModelConfig

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libvvli_cuda.so")
NCCL_ID_BYTES = 128

_f32p = ctypes.POINTER(ctypes.c_float)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_u64p = ctypes.POINTER(ctypes.c_uint64)
_cfgp = ctypes.POINTER(CModelConfig)
_ctx = ctypes.c_void_p


class CGenerateStats(ctypes.Structure):
    _fields_ = [
        ("prompt_tokens", ctypes.c_uint64),
        ("generated_tokens", ctypes.c_uint64),
        ("prefill_nanoseconds", ctypes.c_int64),
        ("decode_nanoseconds", ctypes.c_int64),
        ("total_nanoseconds", ctypes.c_int64),
    ]


class CSampleOptions(ctypes.Structure):
    _fields_ = [
        ("temperature", ctypes.c_float),
        ("top_p", ctypes.c_float),
        ("top_k", ctypes.c_uint64),
        ("repeat_penalty", ctypes.c_float),
        ("_pad0", ctypes.c_uint32),
        ("repeat_last_n", ctypes.c_uint64),
    ]


class CMoeArgs(ctypes.Structure):
    """vvli_moe_args (include/vvli_cuda.h)."""
    _fields_ = [
        ("tokens", ctypes.c_uint64),
        ("hidden", ctypes.c_uint64),
        ("inter", ctypes.c_uint64),
        ("experts", ctypes.c_uint64),
        ("top_k", ctypes.c_uint64),
        ("norm_topk_prob", ctypes.c_int32),
        ("rms_eps", ctypes.c_float),
        ("x", ctypes.c_void_p),
        ("norm_w", ctypes.c_void_p),
        ("router", ctypes.c_void_p),
        ("gate_up", ctypes.c_void_p),
        ("down", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_uint64),
        ("topk_index", ctypes.c_void_p),
        ("topk_weight", ctypes.c_void_p),
    ]


# name -> (restype, argtypes); every function declared in include/vvli_cuda.h.
SIGNATURES = {
    "vvli_cuda_strerror": (ctypes.c_char_p, [ctypes.c_int]),
    "vvli_cuda_last_error": (ctypes.c_char_p, []),
    "vvli_cuda_storage_elements": (ctypes.c_int, [_cfgp, _u64p]),
    "vvli_cuda_tp_plan": (ctypes.c_int, [_cfgp, ctypes.c_int, ctypes.c_int, _u64p, ctypes.c_uint64, _u64p]),
    "vvli_cuda_nccl_unique_id": (ctypes.c_int, [ctypes.c_void_p]),
    "vvli_cuda_create": (ctypes.c_int, [_cfgp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                        ctypes.c_uint64, ctypes.c_uint64, ctypes.POINTER(_ctx)]),
    "vvli_cuda_load_weights": (ctypes.c_int, [_ctx, _u16p, ctypes.c_uint64]),
    "vvli_cuda_fill_synthetic": (ctypes.c_int, [_ctx, ctypes.c_uint64]),
    "vvli_cuda_fill_synthetic_quantized": (ctypes.c_int, [_ctx, ctypes.c_uint64, ctypes.c_int]),
    "vvli_cuda_reset": (ctypes.c_int, [_ctx]),
    "vvli_cuda_forward_token": (ctypes.c_int, [_ctx, ctypes.c_uint32, ctypes.c_uint64, _f32p, _u32p]),
    "vvli_cuda_forward_embedding": (ctypes.c_int, [_ctx, _f32p, ctypes.c_uint64, _f32p, _u32p]),
    "vvli_cuda_prefill": (ctypes.c_int, [_ctx, _u32p, ctypes.c_uint64, ctypes.c_uint64, _f32p, _u32p]),
    "vvli_cuda_generate_greedy": (ctypes.c_int, [_ctx, _u32p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int64,
                                                 _u32p, _u64p, ctypes.POINTER(CGenerateStats)]),
    "vvli_cuda_decode": (ctypes.c_int, [_ctx, ctypes.c_uint64, _u32p, _f32p]),
    "vvli_cuda_time_kernel": (ctypes.c_int, [_ctx, ctypes.c_int, ctypes.c_int, _f32p,
                                             ctypes.POINTER(ctypes.c_double)]),
    "vvli_cuda_query": (ctypes.c_int, [_ctx, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double)]),
    "vvli_cuda_trace": (ctypes.c_int, [_ctx, _u64p, ctypes.c_uint64, _u64p]),
    "vvli_cuda_op_bench": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                          _f32p, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double),
                                          ctypes.POINTER(ctypes.c_int)]),
    "vvli_cuda_gemm_selftest": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                               ctypes.c_int, ctypes.c_uint64, _f32p]),
    "vvli_cuda_attention_selftest": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                    ctypes.c_int, ctypes.c_uint64, _f32p]),
    "vvli_cuda_forward_batch": (ctypes.c_int, [_ctx, _u32p, _u64p, ctypes.c_uint64, _f32p, _u32p]),
    "vvli_cuda_prefill_batch": (ctypes.c_int, [_ctx, _u32p, _u64p, ctypes.c_uint64, _f32p, _u32p]),
    "vvli_cuda_argmax_rows_static": (ctypes.c_int, [ctypes.c_int, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64,
                                                    ctypes.c_void_p, ctypes.c_void_p]),
    "vvli_cuda_sample": (ctypes.c_int, [_ctx, ctypes.c_void_p, _f32p, _u32p, ctypes.c_uint64, _u64p, _u32p]),
    "vvli_cuda_load_safetensors": (ctypes.c_int, [_ctx, ctypes.c_char_p]),
    "vvli_cuda_load_gguf": (ctypes.c_int, [_ctx, ctypes.c_char_p]),
    "vvli_cuda_set_debug": (ctypes.c_int, [_ctx, ctypes.c_int]),
    "vvli_cuda_debug_hidden": (ctypes.c_int, [_ctx, ctypes.c_int, _f32p]),
    "vvli_cuda_moe_workspace_bytes": (ctypes.c_uint64, [ctypes.c_uint64] * 5),
    "vvli_cuda_moe_ffn": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(CMoeArgs), ctypes.c_void_p]),
    "vvli_cuda_last_forward_ms": (ctypes.c_int, [_ctx, _f32p]),
    "vvli_cuda_destroy": (ctypes.c_int, [_ctx]),
}

_lib = None


def lib():
    """Loads libvvli_cuda.so once; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `make -C vvli_b200/csrc` "
                "(or __graft_entry__.build()); there is no CPU fallback")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def strerror(status: int) -> str:
    return lib().vvli_cuda_strerror(status).decode()
