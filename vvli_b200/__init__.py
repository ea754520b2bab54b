"""vvli_b200: B200-native (sm_100a) implementation of VVLI's dense decoder hot path.

The compute path is libvvli_cuda.so (hand-written CUDA behind the C ABI of
include/vvli_cuda.h); this package is the host-side mirror of the
reference's Runner / generator API over that library.
"""

from .config import Config, PRESETS, decode_bytes_per_token  # noqa: F401
from .errors import VvliError  # noqa: F401
from .generator import Options, Result, Stats, generate_greedy, generate_greedy_measured  # noqa: F401
from .runner import Runner, nccl_unique_id  # noqa: F401
