"""Status codes of the C ABI and the Python exception that carries them.

The names mirror the reference's Zig error sets: llm.Error
(src/llm.zig:17-27), generator.Error (src/generator.zig:8-12) and
gguf.Error (src/gguf.zig:7-12).  Codes
20 and above are added by the CUDA runtime (device, NCCL, bounded waits).
"""

OK = 0
CODES = {
    1: "ContextFull",
    2: "InvalidConfig",
    3: "InvalidToken",
    4: "InvalidWeight",
    5: "UnsupportedDType",
    6: "UnsupportedModelArchitecture",
    7: "EmptyPrompt",
    8: "OutputTooSmall",
    9: "InvalidSamplingOptions",
    10: "MissingSafetensorsTensor",
    11: "InvalidGguf",
    12: "UnsupportedGgufVersion",
    13: "UnsupportedMetadataType",
    20: "CudaError",
    21: "NcclError",
    22: "Timeout",
    23: "OutOfMemory",
    24: "WeightsNotLoaded",
    25: "InvalidArgument",
    26: "Unimplemented",
}
# Errors raised by the host side only (no C code): config parsing.
MISSING_JSON_FIELD = "MissingJsonField"
CODE_OF = {name: code for code, name in CODES.items()}


class VvliError(Exception):
    """A reference error name (e.g. ``ContextFull``) with its C status code."""

    def __init__(self, name, code=None, detail=""):
        self.name = name
        self.code = code if code is not None else CODE_OF.get(name, -1)
        super().__init__(f"{name}{': ' + detail if detail else ''}")


def check(status, detail=""):
    """Raises VvliError for a non-zero C status, with the library's message."""
    if status != OK:
        if not detail and status >= 20:
            try:
                from . import _abi
                detail = _abi.lib().vvli_cuda_last_error().decode()
            except Exception:
                pass
        raise VvliError(CODES.get(status, f"Status{status}"), status, detail)
