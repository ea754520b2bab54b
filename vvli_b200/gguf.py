"""GGUF container parser: the host-side mirror of src/gguf.zig.

``parse`` follows gguf.parse (src/gguf.zig:234-287) and its Reader
(:288-356): the magic, version 2 or 3, the metadata key/value table (arrays
are recorded by position and read on demand), the tensor table, and the data
section start aligned to ``general.alignment`` (default 32).  The lookups
follow File (:119-232): the first entry of a name wins, ``usize_value`` and
``f32_value`` convert integer and float types as the reference does.  Errors
carry gguf.Error's names (InvalidGguf, UnsupportedGgufVersion,
UnsupportedMetadataType).
"""

from __future__ import annotations

import dataclasses
import struct

from .errors import VvliError

DEFAULT_ALIGNMENT = 32

# gguf.MetadataType (src/gguf.zig:16-30)
UINT8, INT8, UINT16, INT16, UINT32, INT32, FLOAT32, BOOL, STRING, ARRAY, UINT64, INT64, FLOAT64 = range(13)
_SCALAR = {UINT8: "<B", INT8: "<b", UINT16: "<H", INT16: "<h", UINT32: "<I", INT32: "<i", FLOAT32: "<f",
           BOOL: "<B", UINT64: "<Q", INT64: "<q", FLOAT64: "<d"}

# gguf.TensorType (src/gguf.zig:32-72)
F32, F16, BF16 = 0, 1, 30
Q4_0, Q8_0 = 2, 8  # the block-quantised types the device streams (32 weights and an fp16 scale per block)
TENSOR_TYPES = {0, 1, 2, 3, *range(6, 31), 34, 35, 39}
NATIVE_FLOAT = {F32, F16, BF16}  # TensorType.isNativeFloat


@dataclasses.dataclass
class ArrayInfo:
    item_type: int
    len: int
    values_offset: int


@dataclasses.dataclass
class TensorInfo:
    name: str
    dims: tuple
    tensor_type: int
    offset: int

    def shape(self) -> tuple:
        return self.dims

    def element_count(self) -> int:
        n = 1
        for d in self.dims:
            n *= d
        return n


class _Reader:
    def __init__(self, data, index: int = 0):
        self.data = data
        self.index = index

    def read_bytes(self, n: int):
        if n > len(self.data) - self.index:
            raise VvliError("InvalidGguf")
        out = self.data[self.index: self.index + n]
        self.index += n
        return out

    def read(self, fmt: str):
        return struct.unpack(fmt, self.read_bytes(struct.calcsize(fmt)))[0]

    def read_metadata_type(self) -> int:
        t = self.read("<I")
        if t > FLOAT64:
            raise VvliError("UnsupportedMetadataType")
        return t

    def read_string(self) -> bytes:
        return bytes(self.read_bytes(self.read("<Q")))

    def read_value(self, t: int):
        """Reader.readMetadataValue (src/gguf.zig:316-338)."""
        if t == STRING:
            return self.read_string()
        if t == ARRAY:
            item = self.read_metadata_type()
            n = self.read("<Q")
            off = self.index
            for _ in range(n):
                self.skip_value(item)
            return ArrayInfo(item, n, off)
        v = self.read(_SCALAR[t])
        return v != 0 if t == BOOL else v

    def skip_value(self, t: int) -> None:
        """Reader.skipMetadataValue (src/gguf.zig:340-355)."""
        if t == STRING:
            self.read_bytes(self.read("<Q"))
        elif t == ARRAY:
            item = self.read_metadata_type()
            n = self.read("<Q")
            if item in _SCALAR:  # one bounds check for a whole array of numbers
                self.read_bytes(n * struct.calcsize(_SCALAR[item]))
            else:
                for _ in range(n):
                    self.skip_value(item)
        else:
            self.read_bytes(struct.calcsize(_SCALAR[t]))


@dataclasses.dataclass
class File:
    data: object
    version: int
    metadata: list  # [(key: str, type: int, value)]
    tensors: list   # [TensorInfo]
    data_start: int
    alignment: int

    def metadata_value(self, key: str):
        """(type, value) of the first entry named `key`, or None."""
        for k, t, v in self.metadata:
            if k == key:
                return t, v
        return None

    def string(self, key: str):
        mv = self.metadata_value(key)
        if mv is None or mv[0] != STRING:
            return None
        return mv[1].decode("utf-8", errors="replace")

    def usize_value(self, key: str):
        """File.usizeValue (src/gguf.zig:149-162): unsigned, or non-negative signed, integers."""
        mv = self.metadata_value(key)
        if mv is None:
            return None
        t, v = mv
        if t in (UINT8, UINT16, UINT32, UINT64):
            return v
        if t in (INT8, INT16, INT32, INT64):
            return v if v >= 0 else None
        return None

    def f32_value(self, key: str):
        """File.f32Value (src/gguf.zig:164-179): floats and integers as f32."""
        mv = self.metadata_value(key)
        if mv is None:
            return None
        t, v = mv
        if t in (STRING, ARRAY, BOOL):
            return None
        return struct.unpack("<f", struct.pack("<f", float(v)))[0]

    def tensor(self, name: str):
        for info in self.tensors:
            if info.name == name:
                return info
        return None

    def _array(self, key: str) -> ArrayInfo:
        mv = self.metadata_value(key)
        if mv is None or mv[0] != ARRAY:
            raise VvliError("InvalidGguf")
        return mv[1]

    def string_array(self, key: str) -> list:
        """File.stringArrayAlloc (src/gguf.zig:188-202)."""
        a = self._array(key)
        if a.item_type != STRING:
            raise VvliError("InvalidGguf")
        r = _Reader(self.data, a.values_offset)
        return [r.read_string().decode("utf-8", errors="replace") for _ in range(a.len)]

    def f32_array(self, key: str) -> list:
        """File.f32ArrayAlloc (src/gguf.zig:204-231)."""
        a = self._array(key)
        if a.item_type in (STRING, ARRAY, BOOL):
            raise VvliError("InvalidGguf")
        r = _Reader(self.data, a.values_offset)
        return [struct.unpack("<f", struct.pack("<f", float(r.read(_SCALAR[a.item_type]))))[0]
                for _ in range(a.len)]


def parse(data) -> File:
    """gguf.parse (src/gguf.zig:234-287) over bytes, a memoryview or an mmap."""
    r = _Reader(data)
    if bytes(r.read_bytes(4)) != b"GGUF":
        raise VvliError("InvalidGguf")
    version = r.read("<I")
    if version < 2 or version > 3:
        raise VvliError("UnsupportedGgufVersion")
    tensor_count = r.read("<Q")
    metadata_count = r.read("<Q")
    metadata = []
    for _ in range(metadata_count):
        key = r.read_string().decode("utf-8", errors="replace")
        t = r.read_metadata_type()
        metadata.append((key, t, r.read_value(t)))
    tensors = []
    for _ in range(tensor_count):
        name = r.read_string().decode("utf-8", errors="replace")
        dim_count = r.read("<I")
        if dim_count == 0 or dim_count > 8:
            raise VvliError("InvalidGguf")
        dims = tuple(r.read("<Q") for _ in range(dim_count))
        tensor_type = r.read("<I")
        if tensor_type not in TENSOR_TYPES:
            raise VvliError("UnsupportedMetadataType")
        tensors.append(TensorInfo(name, dims, tensor_type, r.read("<Q")))
    f = File(data, version, metadata, tensors, 0, DEFAULT_ALIGNMENT)
    a = f.usize_value("general.alignment")
    f.alignment = DEFAULT_ALIGNMENT if a is None else a
    if f.alignment == 0:
        raise VvliError("InvalidGguf")
    f.data_start = (r.index + f.alignment - 1) // f.alignment * f.alignment
    if f.data_start > len(data):
        raise VvliError("InvalidGguf")
    return f
