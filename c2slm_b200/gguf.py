"""GGUF v2/v3 reader, mirroring gguf/reader.go of hazyhaar/c2slm.

Same surface as the reference: ``open(path) -> File`` with ``tensors``,
``tensor_map`` (name -> TensorInfo{name, dimensions, type, offset, data}),
``metadata`` and the typed getters ``get_uint32`` / ``get_float32`` /
``get_string`` / ``get_string_slice`` (gguf/reader.go:90-118, 549-602).
``data`` is a read-only memoryview into the mmap, like the Go slice.
"""
from __future__ import annotations

import mmap
import struct
from dataclasses import dataclass, field

GGUF_MAGIC = 0x46554747
# gguf/reader.go:21-37
F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q8_1 = 0, 1, 2, 3, 6, 7, 8, 9
Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, Q8_K, BF16 = 10, 11, 12, 13, 14, 15, 28
TYPE_NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q4_1: "Q4_1", Q5_0: "Q5_0", Q5_1: "Q5_1",
              Q8_0: "Q8_0", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K", Q8_K: "Q8_K", BF16: "BF16"}


def tensor_byte_size(t: int, dims) -> int:
    """gguf/reader.go:513-546 (unknown types fall back to 4 bytes/element)."""
    if len(dims) == 0:
        return 0
    n = 1
    for d in dims:
        n *= int(d)
    if t == F32:
        return n * 4
    if t == F16:
        return n * 2
    if t == Q4_0:
        return (n // 32) * 18
    if t == Q5_0:
        return (n // 32) * 22
    if t == Q8_0:
        return (n // 32) * 34
    if t == Q4_K:
        return (n // 256) * 144
    if t == Q6_K:
        return (n // 256) * 210
    return n * 4


@dataclass
class TensorInfo:
    name: str
    dimensions: list
    type: int
    offset: int
    data: memoryview = field(repr=False, default=None)

    def num_elements(self) -> int:
        if not self.dimensions:
            return 0
        n = 1
        for d in self.dimensions:
            n *= int(d)
        return n


class GGUFError(ValueError):
    pass


class _Reader:
    def __init__(self, buf):
        self.buf = buf
        self.pos = 0

    def take(self, n: int):
        if self.pos + n > len(self.buf):
            raise GGUFError("unexpected EOF")
        b = self.buf[self.pos:self.pos + n]
        self.pos += n
        return b

    def u(self, fmt: str):
        size = struct.calcsize(fmt)
        return struct.unpack(fmt, self.take(size))[0]

    def string(self) -> str:
        n = self.u("<Q")
        return bytes(self.take(n)).decode("utf-8", errors="replace")

    def value(self, vt: int):
        fmts = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 10: "<Q", 11: "<q", 12: "<d"}
        if vt in fmts:
            return self.u(fmts[vt])
        if vt == 7:
            return self.u("<B") != 0
        if vt == 8:
            return self.string()
        if vt == 9:
            et = self.u("<I")
            n = self.u("<Q")
            if et == 8:
                return [self.string() for _ in range(n)]
            return [self.value(et) for _ in range(n)]
        raise GGUFError(f"unknown metadata value type: {vt}")


class File:
    def __init__(self, path: str):
        self._f = open(path, "rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        self._view = memoryview(self._mm)
        self.metadata: dict = {}
        self.metadata_types: dict = {}
        self.tensors: list[TensorInfo] = []
        self.tensor_map: dict[str, TensorInfo] = {}
        self._parse()

    def _parse(self) -> None:  # gguf/reader.go:394-510
        if len(self._view) < 24:
            raise GGUFError("gguf: file too small")
        r = _Reader(self._view)
        magic = r.u("<I")
        if magic != GGUF_MAGIC:
            raise GGUFError(f"invalid GGUF magic: 0x{magic:08x}")
        self.version = r.u("<I")
        if self.version < 2 or self.version > 3:
            raise GGUFError(f"unsupported GGUF version {self.version}")
        n_tensors = r.u("<Q")
        n_kv = r.u("<Q")
        for _ in range(n_kv):
            key = r.string()
            vt = r.u("<I")
            self.metadata[key] = r.value(vt)
            self.metadata_types[key] = vt
        alignment = 32
        a = self.metadata.get("general.alignment")
        if isinstance(a, int) and self.metadata_types.get("general.alignment") in (4, 10):
            alignment = a
        for _ in range(n_tensors):
            name = r.string()
            nd = r.u("<I")
            dims = [r.u("<Q") for _ in range(nd)]
            t = r.u("<I")
            off = r.u("<Q")
            ti = TensorInfo(name, dims, t, off)
            self.tensors.append(ti)
            self.tensor_map[name] = ti
        pad = r.pos % alignment
        if pad:
            r.pos += alignment - pad
        self.tensor_data_offset = r.pos
        for ti in self.tensors:
            start = self.tensor_data_offset + ti.offset
            size = tensor_byte_size(ti.type, ti.dimensions)
            if start + size > len(self._view):
                raise GGUFError(f"tensor[{ti.name}] data out of range")
            ti.data = self._view[start:start + size]

    # typed getters, gguf/reader.go:549-602
    def get_uint32(self, key: str):
        v = self.metadata.get(key)
        if self.metadata_types.get(key) in (4, 5, 10, 11):
            return int(v) & 0xFFFFFFFF, True
        return 0, False

    def get_float32(self, key: str):
        if self.metadata_types.get(key) in (6, 12):
            return float(self.metadata[key]), True
        return 0.0, False

    def get_string(self, key: str):
        if self.metadata_types.get(key) == 8:
            return self.metadata[key], True
        return "", False

    def get_string_slice(self, key: str):
        v = self.metadata.get(key)
        if isinstance(v, list) and all(isinstance(s, str) for s in v):
            return v, True
        return None, False

    def close(self) -> None:
        for ti in self.tensors:
            ti.data = None
        try:
            self._view.release()
        except Exception:
            pass
        self._mm.close()
        self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


def open_gguf(path: str) -> File:
    return File(path)
