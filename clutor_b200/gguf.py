"""GGUF files: a writer (for synthetic models) and a reader (for checking them).

The format is llama.cpp's GGUF version 3, as the reference's reader takes it (c/src/gguf.c:113-166, c/src/meta.c):
magic "GGUF", u32 version, u64 tensor count, u64 metadata count; metadata entries (u64-length string key, u32 type, value);
tensor infos (name, u32 dims, u64 dims innermost first, u32 ggml type, u64 offset from the data start); the data section
starts at the next multiple of general.alignment (32 unless stated) and every tensor starts on that alignment.

Tensor dims follow ggml: a weight matrix of `rows` outputs and `cols` inputs is [cols, rows]; the fused expert tensors are
[cols, rows, n_expert] (c/src/forward.c:194-216).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

# metadata value types (gguf.h in llama.cpp; the reference's meta.c reads the same codes)
U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<?", U64: "<Q", I64: "<q",
           F64: "<d"}
ALIGN = 32


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(t: int, v) -> bytes:
    if t == STR:
        return _str(v)
    if t == ARR:
        et, items = v
        body = b"".join(_value(et, x) for x in items)
        return struct.pack("<IQ", et, len(items)) + body
    return struct.pack(_SCALAR[t], v)


@dataclass
class Tensor:
    name: str
    dims: list[int]
    type: int
    data: object          # bytes-like, numpy array, or a callable with .nbytes that makes the array when written

    @property
    def nbytes(self) -> int:
        if isinstance(self.data, np.ndarray) or callable(self.data):
            return int(self.data.nbytes)
        return memoryview(self.data).nbytes

    def raw(self) -> memoryview:
        d = self.data() if callable(self.data) else self.data
        if isinstance(d, np.ndarray):
            return memoryview(np.ascontiguousarray(d).view(np.uint8).reshape(-1))
        return memoryview(d).cast("B")


@dataclass
class Writer:
    """Collects metadata and tensors, then writes one GGUF file. Tensor data is written as given, in order."""
    kv: list[tuple[str, int, object]] = field(default_factory=list)
    tensors: list[Tensor] = field(default_factory=list)

    def add(self, key: str, type_: int, value) -> None:
        self.kv.append((key, type_, value))

    def add_tensor(self, name: str, dims: list[int], type_: int, data) -> None:
        self.tensors.append(Tensor(name, list(dims), type_, data))

    def header(self) -> bytes:
        out = [b"GGUF", struct.pack("<IQQ", 3, len(self.tensors), len(self.kv))]
        out += [_str(k) + struct.pack("<I", t) + _value(t, v) for k, t, v in self.kv]
        off = 0
        for t in self.tensors:
            out.append(_str(t.name) + struct.pack("<I", len(t.dims)) + b"".join(struct.pack("<Q", d) for d in t.dims)
                       + struct.pack("<IQ", t.type, off))
            off += -(-t.nbytes // ALIGN) * ALIGN
        head = b"".join(out)
        return head + b"\0" * (-len(head) % ALIGN)

    def write(self, path: str) -> int:
        """Writes the file; returns its size in bytes."""
        head = self.header()
        n = len(head)
        with open(path, "wb") as f:
            f.write(head)
            for t in self.tensors:
                f.write(t.raw())
                pad = -t.nbytes % ALIGN
                f.write(b"\0" * pad)
                n += t.nbytes + pad
        return n

    def image(self) -> np.ndarray:
        """The whole file as one uint8 array in memory."""
        head = self.header()
        total = len(head) + sum(-(-t.nbytes // ALIGN) * ALIGN for t in self.tensors)
        out = np.zeros(total, dtype=np.uint8)
        out[:len(head)] = np.frombuffer(head, dtype=np.uint8)
        o = len(head)
        for t in self.tensors:
            out[o:o + t.nbytes] = np.frombuffer(t.raw(), dtype=np.uint8)
            o += -(-t.nbytes // ALIGN) * ALIGN
        return out


@dataclass
class TensorInfo:
    name: str
    dims: list[int]
    type: int
    offset: int           # absolute, from the start of the file


def read(buf) -> tuple[dict, dict]:
    """Parses a GGUF image (bytes / memoryview / mmap): returns (metadata {key: value}, tensors {name: TensorInfo})."""
    mv = memoryview(buf)
    pos = 0

    def take(fmt):
        nonlocal pos
        v = struct.unpack_from(fmt, mv, pos)
        pos += struct.calcsize(fmt)
        return v[0] if len(v) == 1 else v

    def rstr():
        nonlocal pos
        n = take("<Q")
        s = bytes(mv[pos:pos + n]).decode()
        pos += n
        return s

    def rval(t):
        if t == STR:
            return rstr()
        if t == ARR:
            et, n = take("<I"), take("<Q")
            return [rval(et) for _ in range(n)]
        return take(_SCALAR[t])

    if bytes(mv[:4]) != b"GGUF":
        raise ValueError("not a GGUF file")
    pos = 4
    version, nt, nkv = take("<I"), take("<Q"), take("<Q")
    if version not in (2, 3):
        raise ValueError(f"GGUF version {version}")
    meta = {}
    for _ in range(nkv):
        k = rstr()
        meta[k] = rval(take("<I"))
    infos = []
    for _ in range(nt):
        name = rstr()
        nd = take("<I")
        dims = [take("<Q") for _ in range(nd)]
        infos.append((name, dims, take("<I"), take("<Q")))
    align = int(meta.get("general.alignment", ALIGN))
    data = -(-pos // align) * align
    return meta, {n: TensorInfo(n, d, t, data + o) for n, d, t, o in infos}
