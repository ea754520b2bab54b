"""vvli_cuda_argmax_rows_static: greedy token choice with no library allocation.

The entry point keeps its scratch in a static device array.  Its answers are
compared with the greedy token the context-based path picks
(vvli_cuda_forward_token's argmax) on the same logits, and with the oracle's
restatement of llm.argmax (src/llm.zig:778-789) on edge cases: ties, NaNs,
-inf rows, ragged and maximum sizes.  Device buffers come from torch; every
call goes through the C ABI.
"""

import ctypes

import numpy as np
import pytest

from vvli_b200 import _abi
from vvli_b200 import config as C

pytestmark = pytest.mark.gpu

VVLI_OK = 0
VVLI_ERR_INVALID_ARGUMENT = 25
MAX_ROWS = 64
MAX_PARTIALS = 4096
CHUNK = 4096


@pytest.fixture(scope="module")
def torch():
    import torch
    assert torch.cuda.is_available()
    return torch


def static_argmax(torch, dev_logits, rows, n, stream=None):
    """Calls the entry point on a [rows, n] float32 cuda tensor; returns token ids."""
    tokens = torch.full((rows,), -1, dtype=torch.int32, device=dev_logits.device)
    s = torch.cuda.current_stream() if stream is None else stream
    rc = _abi.lib().vvli_cuda_argmax_rows_static(dev_logits.device.index or 0, ctypes.c_void_p(dev_logits.data_ptr()),
                                                 rows, n, ctypes.c_void_p(tokens.data_ptr()),
                                                 ctypes.c_void_p(s.cuda_stream))
    assert rc == VVLI_OK, _abi.lib().vvli_cuda_last_error()
    s.synchronize()
    return tokens.cpu().numpy().tolist()


def test_matches_context_greedy_token_two_calls(torch):
    # Llama-3.2-1B shape: vocab 128256 -> 32 CTAs per row.
    import vvli_b200
    cfg = C.llama3_2_1b()
    gpu = vvli_b200.Runner(cfg, max_seq=64)
    gpu.fill_synthetic(0)
    rows, expect = [], []
    for pos, tok in enumerate([11, 4000, 77, 128000, 5]):
        rows.append(gpu.forward_token(tok, pos))
        expect.append(gpu.last_argmax)
    gpu.close()
    logits = torch.from_numpy(np.stack(rows)).cuda()
    n = cfg.vocab_size
    # two calls in a row: all rows, then one row (a different grid over the same scratch)
    assert static_argmax(torch, logits, len(rows), n) == expect
    assert static_argmax(torch, logits[3:4].contiguous(), 1, n) == expect[3:4]
    assert static_argmax(torch, logits, len(rows), n) == expect


def test_edge_cases_against_oracle(torch, oracle):
    rng = np.random.default_rng(0)
    cases = []
    n = 3 * CHUNK + 123                                       # ragged last CTA
    a = rng.standard_normal(n).astype(np.float32)
    a[[5000, 9000, n - 1]] = 7.0                              # tie across CTAs: first wins
    cases.append(a)
    cases.append(np.zeros(n, np.float32))                     # all equal -> 0
    cases.append(np.full(n, -np.inf, np.float32))             # all -inf -> 0
    b = rng.standard_normal(n).astype(np.float32)
    b[0] = np.nan                                             # NaN at 0 is never replaced -> 0
    cases.append(b)
    c = rng.standard_normal(n).astype(np.float32)
    c[[1, 4097, 8000]] = np.nan                               # NaNs elsewhere are skipped
    c[4096] = 50.0
    cases.append(c)
    d = rng.standard_normal(n).astype(np.float32)
    d[n - 1] = np.inf
    cases.append(d)
    batch = np.stack(cases)
    expect = [oracle.argmax(r) for r in batch]
    assert expect[:4] == [5000, 0, 0, 0] and expect[4] == 4096 and expect[5] == n - 1
    assert static_argmax(torch, torch.from_numpy(batch).cuda(), len(cases), n) == expect
    # one element; and a second call with the same arrays
    one = torch.tensor([[3.5]], device="cuda")
    assert static_argmax(torch, one, 1, 1) == [0]
    assert static_argmax(torch, torch.from_numpy(batch).cuda(), len(cases), n) == expect


def test_maximum_sizes(torch, oracle):
    g = torch.Generator(device="cuda").manual_seed(1)
    # one row at the largest n: 4096 CTAs
    n = MAX_PARTIALS * CHUNK
    big = torch.randn((1, n), generator=g, device="cuda")
    big[0, n - 5] = 100.0
    assert static_argmax(torch, big, 1, n) == [n - 5]
    del big
    # the most rows, each with 64 CTAs (64 * 64 = 4096 partials)
    rows, n = MAX_ROWS, 64 * CHUNK
    x = torch.randn((rows, n), generator=g, device="cuda")
    expect = [oracle.argmax(r) for r in x.cpu().numpy()]
    assert static_argmax(torch, x, rows, n) == expect
    assert static_argmax(torch, x, rows, n) == expect


def test_rejects_out_of_limit_requests_without_launching(torch):
    lib = _abi.lib()
    x = torch.zeros((2, CHUNK), device="cuda")
    t = torch.zeros(MAX_ROWS + 1, dtype=torch.int32, device="cuda")
    ptr = ctypes.c_void_p(x.data_ptr())
    tp = ctypes.c_void_p(t.data_ptr())
    cases = [
        (0, ptr, MAX_ROWS + 1, 1, tp),         # too many rows
        (0, ptr, 2, MAX_PARTIALS * CHUNK, tp),  # 2 * 4096 partials
        (0, ptr, 0, 8, tp),                     # empty
        (0, ptr, 1, 0, tp),                     # empty
        (0, None, 1, 8, tp),                    # null
        (0, ctypes.c_void_p(x.data_ptr() + 2), 1, 8, tp),  # misaligned
    ]
    for dev, lp, rows, n, tok in cases:
        assert lib.vvli_cuda_argmax_rows_static(dev, lp, rows, n, tok, None) == VVLI_ERR_INVALID_ARGUMENT
        assert b"argmax (static scratch)" in lib.vvli_cuda_last_error()
    host = np.zeros(16, np.float32)
    assert lib.vvli_cuda_argmax_rows_static(0, host.ctypes.data_as(ctypes.c_void_p), 1, 16, tp,
                                            None) == VVLI_ERR_INVALID_ARGUMENT
    # still usable afterwards
    x[1, 17] = 1.0
    assert static_argmax(torch, x, 2, CHUNK) == [0, 17]


def test_allocates_no_device_memory(torch):
    # The point of the entry point: after the first call on a device (which
    # may load this library's device code), calls of any shape leave the
    # device's free memory unchanged.
    g = torch.Generator(device="cuda").manual_seed(2)
    shapes = [(1, 1), (3, 3 * CHUNK + 5), (MAX_ROWS, 64 * CHUNK), (1, MAX_PARTIALS * CHUNK)]
    inputs = [torch.randn(s, generator=g, device="cuda") for s in shapes]
    for x in inputs:  # warm-up: one call per shape
        static_argmax(torch, x, x.shape[0], x.shape[1])
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        for x in inputs:
            static_argmax(torch, x, x.shape[0], x.shape[1])
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before, (free_before, free_after)


VMM_CHILD = r"""
import ctypes, sys
import torch
sys.path.insert(0, sys.argv[1])
from vvli_b200 import _abi
n = 16 * 1024 * 1024                      # 64 MB (the one-row maximum): spans chunks of the segment
pad = torch.empty(3 * 1024 * 1024 + 7, device="cuda")   # moves the next buffer off a chunk boundary
x = torch.zeros((1, n), device="cuda")
x[0, n - 3] = 5.0
x[0, 7] = 4.0
t = torch.full((1,), -1, dtype=torch.int32, device="cuda")
s = torch.cuda.current_stream()
rc = _abi.lib().vvli_cuda_argmax_rows_static(0, ctypes.c_void_p(x.data_ptr()), 1, n,
                                             ctypes.c_void_p(t.data_ptr()), ctypes.c_void_p(s.cuda_stream))
assert rc == 0, _abi.lib().vvli_cuda_last_error()
s.synchronize()
assert t.item() == n - 3, t.item()
print("vmm ok")
"""


def test_buffer_from_virtual_memory_pool(torch):
    # A pool built on cuMemCreate + cuMemMap (torch's expandable segments)
    # maps a large buffer as several physical chunks; the entry point must
    # accept such a buffer.  Runs in a child process so the allocator setting
    # applies from the start.
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, PYTORCH_CUDA_ALLOC_CONF="expandable_segments:True")
    r = subprocess.run([sys.executable, "-c", VMM_CHILD, root], env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0 and "vmm ok" in r.stdout, r.stdout + r.stderr
