"""Host side of the mixture-of-experts block (vvli_cuda_moe_ffn, include/vvli_cuda.h).

The reference detects OLMoE configs (src/llm.zig:45-48, 111-133, 210-214:
num_experts, num_experts_per_tok, qk_norm) and rejects them before any
arithmetic (src/main.zig:590-611).  MoeFfn runs that model's sparse
feed-forward block on the GPU: x += MoE(rmsnorm(x) * norm_w) for a batch of
token rows, with the routing of the OLMoE block of transformers 5.5.0.

Device memory is handled with torch tensors (plumbing only): the weights stay
resident, and the workspace is allocated once per token count.
"""

from __future__ import annotations

import ctypes

from . import _abi
from .errors import check


class MoeFfn:
    """One OLMoE sparse block: weights as bf16 bit patterns on one CUDA device.

    norm_w [h], router [E][h], gate_up [E][2I][h] (gate rows, then up rows),
    down [E][h][I]; torch tensors of dtype int16/uint16/bfloat16 (bit patterns
    are what count) or numpy uint16 arrays.
    """

    def __init__(self, norm_w, router, gate_up, down, top_k: int, norm_topk_prob: bool = False,
                 rms_eps: float = 1e-5, device: int = 0):
        import torch

        self.torch = torch
        self.device = torch.device("cuda", device)

        def put(a):
            t = a if isinstance(a, torch.Tensor) else torch.from_numpy(a.view("int16"))
            return t.view(torch.int16).contiguous().to(self.device)

        self.norm_w, self.router, self.gate_up, self.down = put(norm_w), put(router), put(gate_up), put(down)
        self.experts, two_i, self.hidden = self.gate_up.shape
        self.inter = two_i // 2
        if tuple(self.router.shape) != (self.experts, self.hidden) or tuple(self.down.shape) != (
                self.experts, self.hidden, self.inter) or tuple(self.norm_w.shape) != (self.hidden,):
            raise ValueError("MoeFfn: norm_w [h], router [E][h], gate_up [E][2I][h], down [E][h][I] expected")
        self.top_k = int(top_k)
        self.norm_topk_prob = bool(norm_topk_prob)
        self.rms_eps = float(rms_eps)
        self._ws = None

    def workspace_bytes(self, tokens: int) -> int:
        return int(_abi.lib().vvli_cuda_moe_workspace_bytes(tokens, self.hidden, self.inter, self.experts,
                                                              self.top_k))

    def __call__(self, x, stream=None, routing: bool = False):
        """x: [T][h] float32 CUDA tensor, updated in place (x += MoE(...)).

        With routing=True also returns the chosen experts [T][top_k] (int32,
        larger weight first) and their weights [T][top_k] (float32)."""
        torch = self.torch
        if x.dtype != torch.float32 or x.device != self.device or x.dim() != 2 or not x.is_contiguous():
            raise ValueError("MoeFfn: x must be a contiguous [T][h] float32 tensor on " + str(self.device))
        T = x.shape[0]
        need = self.workspace_bytes(T)
        if need and (self._ws is None or self._ws.numel() < need):
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        idx = torch.empty((T, self.top_k), dtype=torch.int32, device=self.device) if routing else None
        w = torch.empty((T, self.top_k), dtype=torch.float32, device=self.device) if routing else None
        a = _abi.CMoeArgs()
        a.tokens, a.hidden, a.inter, a.experts, a.top_k = T, self.hidden, self.inter, self.experts, self.top_k
        a.norm_topk_prob = int(self.norm_topk_prob)
        a.rms_eps = self.rms_eps
        a.x = x.data_ptr()
        a.norm_w, a.router = self.norm_w.data_ptr(), self.router.data_ptr()
        a.gate_up, a.down = self.gate_up.data_ptr(), self.down.data_ptr()
        a.workspace = self._ws.data_ptr() if self._ws is not None else None
        a.workspace_bytes = self._ws.numel() if self._ws is not None else 0
        a.topk_index = idx.data_ptr() if routing else None
        a.topk_weight = w.data_ptr() if routing else None
        s = torch.cuda.current_stream(self.device) if stream is None else stream
        check(_abi.lib().vvli_cuda_moe_ffn(self.device.index, ctypes.byref(a), ctypes.c_void_p(s.cuda_stream)))
        return (idx, w) if routing else None
