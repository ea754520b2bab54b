"""ctypes wrapper of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Loads oracle/libvvli_ref_cpu.so, the C++ restatement of VVLI's CPU decoder
(src/llm.zig, src/generator.zig; see vvli_ref_cpu.cpp for the line map).
Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU arms, as
the checker and the CPU baseline -- never by the product package.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

from vvli_b200.config import Config
from vvli_b200.errors import check

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libvvli_ref_cpu.so")

_lib = None
_f32p = ctypes.POINTER(ctypes.c_float)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_u64p = ctypes.POINTER(ctypes.c_uint64)


def build():
    """Compiles the oracle with its Makefile (a few seconds)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        vp, cfgp = ctypes.c_void_p, ctypes.c_void_p
        sig = {
            "ref_f32_to_bf16": (ctypes.c_uint16, [ctypes.c_float]),
            "ref_bf16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
            "ref_host_simd_lanes": (ctypes.c_int, []),
            "ref_validate": (ctypes.c_int, [cfgp]),
            "ref_storage_elements": (ctypes.c_uint64, [cfgp]),
            "ref_tensor_table": (ctypes.c_uint64, [cfgp, _u64p, ctypes.c_uint64]),
            "ref_fill_synthetic": (None, [cfgp, ctypes.c_uint64, _u16p, ctypes.c_uint64, ctypes.c_uint64]),
            "ref_fill_deterministic": (None, [_u16p, ctypes.c_uint64]),
            "ref_rms_norm": (None, [_f32p, _f32p, _f32p, ctypes.c_uint64, ctypes.c_float, ctypes.c_int]),
            "ref_softmax": (None, [_f32p, ctypes.c_uint64]),
            "ref_argmax": (ctypes.c_uint64, [_f32p, ctypes.c_uint64]),
            "ref_apply_rope": (None, [_f32p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, cfgp]),
            "ref_linear": (None, [_f32p, _u16p, ctypes.c_uint64, ctypes.c_uint64, _f32p, _u16p,
                                  ctypes.c_uint64, ctypes.c_int]),
            "ref_runner_create": (vp, [cfgp, _u16p, ctypes.c_uint64, ctypes.c_int64, ctypes.c_uint64,
                                       ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int,
                                       ctypes.POINTER(ctypes.c_int)]),
            "ref_runner_create_f32": (vp, [cfgp, _f32p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64,
                                           ctypes.c_uint64, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
            "ref_runner_destroy": (None, [vp]),
            "ref_runner_blob": (_u16p, [vp]),
            "ref_runner_reset": (None, [vp]),
            "ref_runner_forward_token": (ctypes.c_int, [vp, ctypes.c_uint32, ctypes.c_uint64, _f32p]),
            "ref_runner_forward_embedding": (ctypes.c_int, [vp, _f32p, ctypes.c_uint64, _f32p]),
            "ref_runner_hidden": (None, [vp, ctypes.c_uint64, _f32p]),
            "ref_runner_set_attention_threads": (None, [vp, ctypes.c_uint64]),
            "ref_runner_prefill": (ctypes.c_int, [vp, _u32p, ctypes.c_uint64, ctypes.c_uint64, _f32p]),
            "ref_runner_logits": (None, [vp, _f32p]),
            "ref_generate_greedy": (ctypes.c_int, [vp, _u32p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int64,
                                                   _u32p, _u64p]),
            "ref_validate_sampling": (ctypes.c_int, [ctypes.c_float, ctypes.c_float, ctypes.c_float]),
            "ref_build_repeat_counts": (None, [_u16p, ctypes.c_uint64, _u32p, ctypes.c_uint64, _u32p,
                                               ctypes.c_uint64, ctypes.c_float, ctypes.c_uint64]),
            "ref_greedy_with_penalties": (ctypes.c_uint32, [_f32p, _u16p, ctypes.c_uint64, ctypes.c_float]),
            "ref_build_candidates": (ctypes.c_uint64, [vp, _f32p, _u16p, ctypes.c_uint64, ctypes.c_uint64,
                                                       ctypes.c_float]),
            "ref_prepare_probabilities": (ctypes.c_uint64, [vp, ctypes.c_uint64, ctypes.c_float, ctypes.c_float]),
            "ref_sample_candidate": (ctypes.c_uint32, [vp, ctypes.c_uint64, ctypes.c_float]),
            "ref_candidate_size": (ctypes.c_uint64, []),
            "ref_sampler_next": (ctypes.c_int, [_f32p, ctypes.c_uint64, _u32p, ctypes.c_uint64, _u32p,
                                                ctypes.c_uint64, vp, ctypes.c_float, _u32p]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def ptr(a, t):
    return a.ctypes.data_as(t) if a is not None else None


def f32(a):
    return ptr(a, _f32p)


def cfg_ref(cfg: Config):
    c = cfg.to_c()
    return c, ctypes.byref(c)


CANDIDATE_DTYPE = np.dtype([("id", np.uint32), ("logit", np.float32), ("probability", np.float32)])


# ---------------------------------------------------------------- weights
def storage_elements(cfg: Config) -> int:
    c, r = cfg_ref(cfg)
    return int(lib().ref_storage_elements(r))


def tensor_table(cfg: Config) -> np.ndarray:
    c, r = cfg_ref(cfg)
    cap = 16 + 12 * cfg.num_hidden_layers
    out = np.zeros((cap, 3), dtype=np.uint64)
    n = lib().ref_tensor_table(r, out.ctypes.data_as(_u64p), cap)
    return out[:n]


def synthetic_blob(cfg: Config, seed: int = 0, threads: int = 0) -> np.ndarray:
    n = storage_elements(cfg)
    blob = np.empty(n, dtype=np.uint16)
    c, r = cfg_ref(cfg)
    lib().ref_fill_synthetic(r, seed, ptr(blob, _u16p), n, threads)
    return blob


def deterministic_blob(cfg: Config) -> np.ndarray:
    n = storage_elements(cfg)
    blob = np.empty(n, dtype=np.uint16)
    lib().ref_fill_deterministic(ptr(blob, _u16p), n)
    return blob


# ---------------------------------------------------------------- kernels
def f32_to_bf16(x: float) -> int:
    return int(lib().ref_f32_to_bf16(x))


def bf16_to_f32(b: int) -> float:
    return float(lib().ref_bf16_to_f32(b))


def rms_norm(x, w, eps, lanes=16):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    lib().ref_rms_norm(f32(out), f32(x), f32(w), x.size, eps, lanes)
    return out


def softmax(v):
    v = np.array(v, dtype=np.float32)
    lib().ref_softmax(f32(v), v.size)
    return v


def argmax(v):
    v = np.ascontiguousarray(v, np.float32)
    return int(lib().ref_argmax(f32(v), v.size))


def apply_rope(values, heads, head_dim, position, cfg: Config):
    v = np.array(values, dtype=np.float32)
    c, r = cfg_ref(cfg)
    lib().ref_apply_rope(f32(v), heads, head_dim, position, r)
    return v


def linear(W_bf16, x, bias_bf16=None, threads=1, lanes=16):
    N, K = W_bf16.shape
    W = np.ascontiguousarray(W_bf16, np.uint16)
    x = np.ascontiguousarray(x, np.float32)
    b = None if bias_bf16 is None else np.ascontiguousarray(bias_bf16, np.uint16)
    out = np.empty(N, dtype=np.float32)
    lib().ref_linear(f32(out), ptr(W, _u16p), N, K, f32(x), ptr(b, _u16p), threads, lanes)
    return out


# ---------------------------------------------------------------- runner
class RefRunner:
    """The oracle's llm.Runner (src/llm.zig:688-776)."""

    def __init__(self, cfg: Config, blob=None, synthetic_seed=None, max_seq=None, threads=0,
                 min_rows_per_thread=64, lanes=0, blob_f32=None):
        """Weights: a bf16 blob (OwnedModel layout), a synthetic seed, or `blob_f32`:
        f32 weights in the same layout (the reference's .f32 Matrix storage, used for
        dequantised GGUF tensors)."""
        self.cfg = cfg
        self.max_seq = max_seq or min(cfg.max_position_embeddings, 512)
        self._blob = None if blob is None else np.ascontiguousarray(blob, np.uint16)
        self._c = cfg.to_c()
        st = ctypes.c_int(0)
        if blob_f32 is not None:
            self._blob = np.ascontiguousarray(blob_f32, np.float32)
            self.h = lib().ref_runner_create_f32(ctypes.byref(self._c), f32(self._blob), self._blob.size,
                                                 self.max_seq, threads, min_rows_per_thread, lanes,
                                                 ctypes.byref(st))
            check(st.value)
            return
        seed = -1 if synthetic_seed is None else int(synthetic_seed)
        self.h = lib().ref_runner_create(ctypes.byref(self._c), ptr(self._blob, _u16p),
                                         0 if self._blob is None else self._blob.size, seed, self.max_seq,
                                         threads, min_rows_per_thread, lanes, ctypes.byref(st))
        check(st.value)

    def close(self):
        if getattr(self, "h", None):
            lib().ref_runner_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def blob_view(self) -> np.ndarray:
        n = storage_elements(self.cfg)
        p = lib().ref_runner_blob(self.h)
        return np.ctypeslib.as_array(p, shape=(n,))

    def reset(self):
        lib().ref_runner_reset(self.h)

    def forward_token(self, token: int, position: int) -> np.ndarray:
        out = np.empty(self.cfg.vocab_size, dtype=np.float32)
        check(lib().ref_runner_forward_token(self.h, token, position, f32(out)))
        return out

    def forward_embedding(self, emb, position: int) -> np.ndarray:
        e = np.ascontiguousarray(emb, np.float32)
        out = np.empty(self.cfg.vocab_size, dtype=np.float32)
        check(lib().ref_runner_forward_embedding(self.h, f32(e), position, f32(out)))
        return out

    def set_attention_threads(self, threads: int):
        """Checker only: attention heads on `threads` threads (bit-identical)."""
        lib().ref_runner_set_attention_threads(self.h, threads)

    def prefill(self, tokens, start: int = 0) -> np.ndarray:
        """Checker only: forward_token over tokens at positions start.., the
        LM head run for the last token alone; returns its logits."""
        t = np.ascontiguousarray(tokens, np.uint32)
        out = np.empty(self.cfg.vocab_size, dtype=np.float32)
        check(lib().ref_runner_prefill(self.h, ptr(t, _u32p), t.size, start, f32(out)))
        return out

    def hidden(self, layer: int) -> np.ndarray:
        out = np.empty(self.cfg.hidden_size, dtype=np.float32)
        lib().ref_runner_hidden(self.h, layer, f32(out))
        return out

    def generate_greedy(self, prompt, max_new_tokens, eos=None):
        p = np.ascontiguousarray(prompt, np.uint32)
        out = np.zeros(max(1, max_new_tokens), dtype=np.uint32)
        n = ctypes.c_uint64(0)
        check(lib().ref_generate_greedy(self.h, ptr(p, _u32p), p.size, max_new_tokens,
                                        -1 if eos is None else eos, ptr(out, _u32p), ctypes.byref(n)))
        return out[: n.value].tolist()


# ---------------------------------------------------------------- sampler helpers
def greedy_with_penalties(logits, counts, repeat_penalty):
    lg = np.ascontiguousarray(logits, np.float32)
    ct = np.ascontiguousarray(counts, np.uint16)
    return int(lib().ref_greedy_with_penalties(f32(lg), ptr(ct, _u16p), lg.size, repeat_penalty))


def build_candidates(logits, counts, top_k, repeat_penalty, capacity=None):
    lg = np.ascontiguousarray(logits, np.float32)
    ct = np.ascontiguousarray(counts, np.uint16)
    cands = np.zeros(capacity or lg.size, dtype=CANDIDATE_DTYPE)
    n = lib().ref_build_candidates(cands.ctypes.data, f32(lg), ptr(ct, _u16p), lg.size, top_k, repeat_penalty)
    return cands[:n]


def prepare_probabilities(cands, temperature, top_p):
    n = lib().ref_prepare_probabilities(cands.ctypes.data, cands.size, temperature, top_p)
    return int(n)


def sample_candidate(cands, random_unit):
    return int(lib().ref_sample_candidate(cands.ctypes.data, cands.size, random_unit))


def build_repeat_counts(n, prompt, generated, repeat_penalty, repeat_last_n):
    counts = np.zeros(n, dtype=np.uint16)
    p = np.ascontiguousarray(prompt, np.uint32)
    g = np.ascontiguousarray(generated, np.uint32) if len(generated) else np.zeros(1, np.uint32)
    lib().ref_build_repeat_counts(ptr(counts, _u16p), n, ptr(p, _u32p), p.size, ptr(g, _u32p), len(generated),
                                  repeat_penalty, repeat_last_n)
    return counts


def sampler_next(logits, prompt, generated, options, random_unit):
    from vvli_b200._abi import CSampleOptions
    lg = np.ascontiguousarray(logits, np.float32)
    p = np.ascontiguousarray(prompt, np.uint32)
    g = np.ascontiguousarray(generated, np.uint32) if len(generated) else np.zeros(1, np.uint32)
    o = CSampleOptions(options.temperature, options.top_p, options.top_k, options.repeat_penalty, 0,
                       options.repeat_last_n)
    out = ctypes.c_uint32(0)
    check(lib().ref_sampler_next(f32(lg), lg.size, ptr(p, _u32p), p.size, ptr(g, _u32p), len(generated),
                                 ctypes.addressof(o), random_unit, ctypes.byref(out)))
    return int(out.value)
