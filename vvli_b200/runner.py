"""Runner: the host-side mirror of llm.Runner over the CUDA C ABI.

Same operations and error behaviour as the reference's Runner
(src/llm.zig:688-776): ``forward_token`` and ``forward_embedding`` return the
logits of one position and raise ``InvalidToken`` / ``ContextFull``; the KV
cache and scratch buffers live on the GPU inside the context.  Additions
for the GPU path are batched ``prefill`` and ``generate_greedy``, which run
the whole token loop on the device.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

from . import _abi
from .config import Config
from .errors import check

_f32p = ctypes.POINTER(ctypes.c_float)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_u32p = ctypes.POINTER(ctypes.c_uint32)


def nccl_unique_id() -> bytes:
    """A fresh NCCL unique id for vvli_cuda_create's tensor-parallel ranks."""
    buf = ctypes.create_string_buffer(_abi.NCCL_ID_BYTES)
    check(_abi.lib().vvli_cuda_nccl_unique_id(buf))
    return buf.raw


class Runner:
    def __init__(self, cfg: Config, max_seq: int, device: int = 0, tp_rank: int = 0, tp_size: int = 1,
                 nccl_id: bytes | None = None, max_batch: int = 1):
        self.cfg = cfg
        self.max_seq = max_seq
        self.tp_rank, self.tp_size = tp_rank, tp_size
        self._c = cfg.to_c()
        self._ctx = ctypes.c_void_p()
        idbuf = None if nccl_id is None else ctypes.create_string_buffer(nccl_id, _abi.NCCL_ID_BYTES)
        check(_abi.lib().vvli_cuda_create(ctypes.byref(self._c), device, tp_rank, tp_size, idbuf, max_seq, max_batch,
                                          ctypes.byref(self._ctx)))
        self.last_argmax = None

    # ------------------------------------------------------------ lifecycle
    def close(self):
        if self._ctx:
            check(_abi.lib().vvli_cuda_destroy(self._ctx))
            self._ctx = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def load_weights(self, blob: np.ndarray):
        """Uploads this rank's shard of an llm.OwnedModel-layout bf16 blob."""
        b = np.ascontiguousarray(blob, dtype=np.uint16)
        check(_abi.lib().vvli_cuda_load_weights(self._ctx, b.ctypes.data_as(_u16p), b.size))

    def load_safetensors(self, path: str):
        """This rank's weights straight from model.safetensors (loadOwnedFromSafetensorsFile)."""
        check(_abi.lib().vvli_cuda_load_safetensors(self._ctx, os.fsencode(path)))

    def load_gguf(self, path: str):
        """This rank's weights straight from a GGUF file (loadOwnedFromGgufFile); the
        Runner's config must come from ``Config.from_gguf`` of the same file."""
        check(_abi.lib().vvli_cuda_load_gguf(self._ctx, os.fsencode(path)))

    def fill_synthetic(self, seed: int = 0):
        check(_abi.lib().vvli_cuda_fill_synthetic(self._ctx, seed))

    def fill_synthetic_quantized(self, seed: int = 0, fmt: str = "q8_0"):
        """The synthetic model with every matrix quantised on the device (GGML Q8_0 or Q4_0)."""
        check(_abi.lib().vvli_cuda_fill_synthetic_quantized(self._ctx, seed, {"q8_0": 1, "q4_0": 2}[fmt]))

    def reset(self):
        """KVCache.clear (src/llm.zig:576-579)."""
        check(_abi.lib().vvli_cuda_reset(self._ctx))

    # ------------------------------------------------------------ forward
    def forward_token(self, token: int, position: int, logits: bool = True):
        """Runner.forwardToken (src/llm.zig:702-709): logits of `token` at `position`."""
        out = np.empty(self.cfg.vocab_size, dtype=np.float32) if logits else None
        am = ctypes.c_uint32(0)
        check(_abi.lib().vvli_cuda_forward_token(self._ctx, token, position,
                                                 None if out is None else out.ctypes.data_as(_f32p),
                                                 ctypes.byref(am)))
        self.last_argmax = int(am.value)
        return out

    def forward_embedding(self, embedding, position: int, logits: bool = True):
        """Runner.forwardEmbedding (src/llm.zig:711-718)."""
        e = np.ascontiguousarray(embedding, dtype=np.float32)
        if e.size != self.cfg.hidden_size:
            from .errors import VvliError
            raise VvliError("InvalidWeight")
        out = np.empty(self.cfg.vocab_size, dtype=np.float32) if logits else None
        am = ctypes.c_uint32(0)
        check(_abi.lib().vvli_cuda_forward_embedding(self._ctx, e.ctypes.data_as(_f32p), position,
                                                     None if out is None else out.ctypes.data_as(_f32p),
                                                     ctypes.byref(am)))
        self.last_argmax = int(am.value)
        return out

    def prefill(self, tokens, start: int = 0, logits: bool = True):
        """Runs tokens at positions start.. and returns the last token's logits."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.empty(self.cfg.vocab_size, dtype=np.float32) if logits else None
        am = ctypes.c_uint32(0)
        check(_abi.lib().vvli_cuda_prefill(self._ctx, t.ctypes.data_as(_u32p), t.size, start,
                                           None if out is None else out.ctypes.data_as(_f32p), ctypes.byref(am)))
        self.last_argmax = int(am.value)
        return out

    def forward_batch(self, tokens, positions, logits: bool = True):
        """One decode step of len(tokens) sequences: row b is sequence slot b at positions[b].

        Returns (logits [B, vocab] or None, argmax list).
        """
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        p = np.ascontiguousarray(positions, dtype=np.uint64)
        if t.size != p.size:
            raise ValueError("tokens and positions differ in length")
        out = np.empty((t.size, self.cfg.vocab_size), dtype=np.float32) if logits else None
        am = np.zeros(max(1, t.size), dtype=np.uint32)
        check(_abi.lib().vvli_cuda_forward_batch(self._ctx, t.ctypes.data_as(_u32p),
                                                 p.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)), t.size,
                                                 None if out is None else out.ctypes.data_as(_f32p),
                                                 am.ctypes.data_as(_u32p)))
        return out, am[: t.size].tolist()

    def prefill_batch(self, prompts, logits: bool = True):
        """Prefills independent sequences, prompts[b] into sequence slot b.

        Returns (last logits [B, vocab] or None, argmax list); decoding goes on
        with ``forward_batch`` (row b = slot b at position len(prompts[b]) ...).
        """
        lens = np.ascontiguousarray([len(p) for p in prompts], dtype=np.uint64)
        t = np.ascontiguousarray(np.concatenate([np.asarray(p, dtype=np.uint32) for p in prompts])
                                 if len(prompts) else np.zeros(0, np.uint32), dtype=np.uint32)
        B = len(prompts)
        out = np.empty((B, self.cfg.vocab_size), dtype=np.float32) if logits else None
        am = np.zeros(max(1, B), dtype=np.uint32)
        check(_abi.lib().vvli_cuda_prefill_batch(self._ctx, t.ctypes.data_as(_u32p),
                                                 lens.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)), B,
                                                 None if out is None else out.ctypes.data_as(_f32p),
                                                 am.ctypes.data_as(_u32p)))
        return out, am[:B].tolist()

    def generate_greedy(self, prompt, max_new_tokens: int, eos_token_id: int | None = None):
        """On-device greedy loop; returns (tokens, vvli_generate_stats)."""
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.zeros(max(1, max_new_tokens), dtype=np.uint32)
        n = ctypes.c_uint64(0)
        stats = _abi.CGenerateStats()
        check(_abi.lib().vvli_cuda_generate_greedy(self._ctx, p.ctypes.data_as(_u32p), p.size, max_new_tokens,
                                                   -1 if eos_token_id is None else int(eos_token_id),
                                                   out.ctypes.data_as(_u32p), ctypes.byref(n), ctypes.byref(stats)))
        return out[: n.value].tolist(), stats

    def decode(self, n_steps: int):
        """Continues greedy decoding on the device; returns (tokens, device_ms)."""
        out = np.zeros(max(1, n_steps), dtype=np.uint32)
        ms = ctypes.c_float(0)
        check(_abi.lib().vvli_cuda_decode(self._ctx, n_steps, out.ctypes.data_as(_u32p), ctypes.byref(ms)))
        return out[:n_steps].tolist(), float(ms.value)

    def sample(self, options, recent, rng_state: np.ndarray, logits=None) -> int:
        """Sampler.next on the device, over ``logits`` (host, uploaded) or the last forward's logits.

        ``recent``: prompt tokens followed by the generated ones (or their
        tail); ``rng_state``: uint64[4] xoshiro256++ state, advanced in place.
        """
        lg = None
        if logits is not None:
            lg = np.ascontiguousarray(logits, dtype=np.float32)
            if lg.size != self.cfg.vocab_size:
                from .errors import VvliError
                raise VvliError("OutputTooSmall")
        o = _abi.CSampleOptions(temperature=float(options.temperature), top_p=float(options.top_p),
                                top_k=int(options.top_k), repeat_penalty=float(options.repeat_penalty),
                                repeat_last_n=int(options.repeat_last_n))
        n_use = min(len(recent), int(options.repeat_last_n))
        tail = recent[len(recent) - n_use:] if n_use else recent[:0]  # a view for numpy arrays
        r = np.ascontiguousarray(tail, dtype=np.uint32)
        assert rng_state.dtype == np.uint64 and rng_state.size == 4 and rng_state.flags["C_CONTIGUOUS"]
        out = ctypes.c_uint32(0)
        check(_abi.lib().vvli_cuda_sample(self._ctx, ctypes.byref(o), None if lg is None else lg.ctypes.data_as(_f32p),
                                          r.ctypes.data_as(_u32p) if r.size else None,
                                          r.size, rng_state.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)),
                                          ctypes.byref(out)))
        return int(out.value)

    def time_kernel(self, kernel: int, reps: int):
        """(mean ms per launch, algorithmic bytes per launch) of one decode kernel alone."""
        ms = ctypes.c_float(0)
        b = ctypes.c_double(0)
        check(_abi.lib().vvli_cuda_time_kernel(self._ctx, kernel, reps, ctypes.byref(ms), ctypes.byref(b)))
        return float(ms.value), float(b.value)

    def query(self, key: str) -> float:
        """A numeric property of the context (vvli_cuda_query)."""
        v = ctypes.c_double(0)
        check(_abi.lib().vvli_cuda_query(self._ctx, key.encode(), ctypes.byref(v)))
        return float(v.value)

    # ------------------------------------------------------------ debug / timing
    def trace(self) -> np.ndarray:
        """Megakernel timeline of the last step (VVLI_TRACE=1 at creation), else an empty array."""
        n = ctypes.c_uint64(0)
        check(_abi.lib().vvli_cuda_trace(self._ctx, None, 0, ctypes.byref(n)))
        out = np.zeros(n.value, dtype=np.uint64)
        if n.value:
            check(_abi.lib().vvli_cuda_trace(self._ctx, out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)), n.value,
                                             ctypes.byref(n)))
        return out

    def set_debug(self, enabled: bool):
        check(_abi.lib().vvli_cuda_set_debug(self._ctx, int(enabled)))

    def debug_hidden(self, layer: int) -> np.ndarray:
        out = np.empty(self.cfg.hidden_size, dtype=np.float32)
        check(_abi.lib().vvli_cuda_debug_hidden(self._ctx, layer, out.ctypes.data_as(_f32p)))
        return out

    def last_forward_ms(self) -> float:
        v = ctypes.c_float(0)
        check(_abi.lib().vvli_cuda_last_forward_ms(self._ctx, ctypes.byref(v)))
        return float(v.value)
