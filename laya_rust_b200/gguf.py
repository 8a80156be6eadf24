"""GGUF v3 container: writer and reader.

Restates the reference's dependency-free GGUF module (laya-rust ``src/gguf.rs``):

* value types 0..12 with nested arrays whose elements share one type
  (gguf.rs:16-50, 252-287, 490-518);
* key rules: ASCII, ``lower_snake_case`` segments joined by ``.`` (gguf.rs:359-369);
* 32-byte alignment of the data section and of every tensor offset
  (gguf.rs:7, 170-172, 428-475);
* the reader's validation: magic, version 3, plausible counts, 1..4 dims,
  aligned offsets and data inside the file (gguf.rs:289-357).

Errors raise :class:`GGUFError` (the reference calls ``die`` -> exit 2).
Dimensions are written in GGUF order, i.e. the reverse of the framework shape
(convert.rs:243); :meth:`Header.stored_dims` reverses them back
(weights.rs:261-268).
"""
from __future__ import annotations

import re
import struct
from dataclasses import dataclass, field
from typing import Any

import numpy as np

MAGIC = 0x46554747
VERSION = 3
ALIGNMENT = 32
T_F32, T_F16, T_BF16 = 0, 1, 30
FT_ALL_F32, FT_MOSTLY_F16 = 0, 1

U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f",
           U64: "<Q", I64: "<q", F64: "<d"}


class GGUFError(Exception):
    pass


@dataclass
class Value:
    """A typed metadata value (gguf.rs:16-31)."""
    ty: int
    v: Any

    def as_u64(self):
        if self.ty in (U8, U16, U32, U64):
            return int(self.v)
        if self.ty in (I8, I16, I32, I64):
            return int(self.v) & 0xFFFFFFFFFFFFFFFF
        return None

    def as_f32(self):
        if self.ty == F32:
            return float(np.float32(self.v))
        if self.ty == F64:
            return float(np.float32(self.v))
        return None

    def as_str(self):
        return self.v if self.ty == STR else None

    def as_f32s(self):
        if self.ty != ARR:
            return []
        return [x.as_f32() for x in self.v if x.as_f32() is not None]

    def as_strs(self):
        if self.ty != ARR:
            return []
        return [x.as_str() or "" for x in self.v]


def key_ok(k: str) -> bool:
    if not k or len(k) > 65535 or not k.isascii():
        return False
    return all(re.fullmatch(r"[a-z0-9_]+", seg) is not None for seg in k.split("."))


def _align(x: int) -> int:
    return x + (ALIGNMENT - x % ALIGNMENT) % ALIGNMENT


def elem_size(ty: int) -> int:
    if ty == T_F32:
        return 4
    if ty in (T_F16, T_BF16):
        return 2
    raise GGUFError(f"gguf: unsupported tensor type {ty}")


def _put_value(out: bytearray, v: Value) -> None:
    if v.ty in _SCALAR:
        out += struct.pack(_SCALAR[v.ty], v.v)
    elif v.ty == BOOL:
        out += struct.pack("<B", 1 if v.v else 0)
    elif v.ty == STR:
        b = v.v.encode("utf-8")
        out += struct.pack("<Q", len(b)) + b
    elif v.ty == ARR:
        et = v.v[0].ty if v.v else U8
        if any(x.ty != et for x in v.v):
            raise GGUFError("gguf: array elements must share one type")
        out += struct.pack("<IQ", et, len(v.v))
        for x in v.v:
            _put_value(out, x)
    else:
        raise GGUFError(f"gguf: unknown metadata value type {v.ty}")


class Writer:
    """GGUF writer with the reference's validation (gguf.rs:371-475)."""

    def __init__(self):
        self.kv: list[tuple[str, Value]] = []
        self.tensors: list[tuple[str, list[int], int, bytes]] = []

    def add_kv(self, key: str, v: Value) -> "Writer":
        if not key_ok(key):
            raise GGUFError(f"gguf: illegal metadata key {key!r}")
        self.kv.append((key, v))
        return self

    def add_tensor(self, name: str, dims: list[int], ty: int, data: bytes) -> "Writer":
        if not name or len(name) > 64 or not name.isascii():
            raise GGUFError(f"gguf: illegal tensor name {name!r}")
        if not dims or len(dims) > 4:
            raise GGUFError(f"gguf: tensor {name} has {len(dims)} dimensions")
        want = int(np.prod(dims, dtype=np.uint64)) * elem_size(ty)
        if want != len(data):
            raise GGUFError(f"gguf: tensor {name} is {dims} = {want} bytes but {len(data)} were given")
        if any(t[0] == name for t in self.tensors):
            raise GGUFError(f"gguf: duplicate tensor name {name}")
        self.tensors.append((name, list(dims), ty, data))
        return self

    def write(self, path: str) -> None:
        head = bytearray()
        head += struct.pack("<IIQQ", MAGIC, VERSION, len(self.tensors), len(self.kv))
        seen = set()
        for k, v in self.kv:
            if k in seen:
                raise GGUFError(f"gguf: duplicate metadata key {k!r}")
            seen.add(k)
            kb = k.encode()
            head += struct.pack("<Q", len(kb)) + kb + struct.pack("<I", v.ty)
            _put_value(head, v)
        off = 0
        for name, dims, ty, data in self.tensors:
            nb = name.encode()
            head += struct.pack("<Q", len(nb)) + nb + struct.pack("<I", len(dims))
            for d in dims:
                head += struct.pack("<Q", d)
            head += struct.pack("<IQ", ty, off)
            off = _align(off + len(data))
        data_off = _align(len(head))
        with open(path, "wb") as f:
            f.write(head)
            f.write(b"\0" * (data_off - len(head)))
            pos = 0
            for _, _, _, data in self.tensors:
                f.write(data)
                pos += len(data)
                pad = _align(pos) - pos
                f.write(b"\0" * pad)
                pos += pad
            if data_off + pos != data_off + off:
                raise GGUFError(f"gguf: wrote {data_off + pos} bytes but planned {data_off + off}")


@dataclass
class TensorInfo:
    name: str
    dims: list[int]
    ty: int
    offset: int

    def elems(self) -> int:
        return int(np.prod(self.dims, dtype=np.uint64))

    def nbytes(self) -> int:
        return self.elems() * elem_size(self.ty)


@dataclass
class Header:
    path: str
    kv: list[tuple[str, Value]] = field(default_factory=list)
    tensors: list[TensorInfo] = field(default_factory=list)
    data_off: int = 0

    def get(self, key: str):
        for k, v in self.kv:
            if k == key:
                return v
        return None

    def str_or(self, key, d):
        v = self.get(key)
        return v.as_str() if v is not None and v.as_str() is not None else d

    def u64_or(self, key, d):
        v = self.get(key)
        return v.as_u64() if v is not None and v.as_u64() is not None else d

    def f32_or(self, key, d):
        v = self.get(key)
        return v.as_f32() if v is not None and v.as_f32() is not None else d

    def tensor(self, name):
        for t in self.tensors:
            if t.name == name:
                return t
        return None

    def stored_dims(self, name):
        return list(reversed(self.tensor(name).dims))

    def raw(self, name) -> np.ndarray:
        """Tensor bytes as a numpy array of its storage type, in stored shape."""
        t = self.tensor(name)
        if t is None:
            raise GGUFError(f"gguf: no tensor named {name}")
        dt = {T_F32: np.float32, T_F16: np.float16, T_BF16: np.uint16}[t.ty]
        a = np.fromfile(self.path, dtype=dt, count=t.elems(), offset=self.data_off + t.offset)
        return a.reshape(self.stored_dims(name))

    def f32(self, name) -> np.ndarray:
        """gguf.rs:550-571 decode, in stored shape."""
        t = self.tensor(name)
        a = self.raw(name)
        if t.ty == T_BF16:
            return (a.astype(np.uint32) << 16).view(np.float32)
        return a.astype(np.float32)


class _Rd:
    def __init__(self, buf: bytes, path: str):
        self.b, self.pos, self.len, self.path = buf, 0, len(buf), path

    def take(self, n: int, ctx: str) -> bytes:
        if self.pos + n > self.len:
            raise GGUFError(f"gguf: {ctx}: read of {n} bytes at {self.pos} passes end of file ({self.len})")
        out = self.b[self.pos:self.pos + n]
        self.pos += n
        return out

    def unpack(self, fmt: str, ctx: str):
        return struct.unpack(fmt, self.take(struct.calcsize(fmt), ctx))[0]

    def string(self, ctx: str) -> str:
        n = self.unpack("<Q", ctx)
        try:
            return self.take(n, ctx).decode("utf-8")
        except UnicodeDecodeError:
            raise GGUFError(f"gguf: {ctx}: invalid utf-8")


def _read_value(r: _Rd, ty: int, ctx: str) -> Value:
    if ty in _SCALAR:
        return Value(ty, r.unpack(_SCALAR[ty], ctx))
    if ty == BOOL:
        return Value(ty, r.unpack("<B", ctx) != 0)
    if ty == STR:
        return Value(ty, r.string(ctx))
    if ty == ARR:
        et = r.unpack("<I", ctx)
        n = r.unpack("<Q", ctx)
        if n * 8 + 1 > r.len:
            raise GGUFError(f"gguf: {ctx}: array of {n} elements is not plausible in {r.len} bytes")
        return Value(ty, [_read_value(r, et, ctx) for _ in range(n)])
    raise GGUFError(f"gguf: {ctx}: unknown metadata value type {ty}")


def read(path: str) -> Header:
    """gguf.rs:289-357.  Reads the header only; tensor bytes stay on disk."""
    with open(path, "rb") as f:
        f.seek(0, 2)
        flen = f.tell()
        f.seek(0)
        # the header is small: read a generous prefix, grow on demand
        buf = f.read(min(flen, 64 << 20))
    r = _Rd(buf, path)
    r.len = len(buf)
    magic = r.unpack("<I", path)
    if magic != MAGIC:
        raise GGUFError(f"{path}: not a GGUF file (magic {magic:#010x}, want {MAGIC:#010x})")
    version = r.unpack("<I", path)
    if version != VERSION:
        raise GGUFError(f"{path}: GGUF version {version}, want {VERSION}")
    tc = r.unpack("<Q", path)
    kc = r.unpack("<Q", path)
    if tc * 64 + kc * 16 > flen:
        raise GGUFError(f"{path}: header claims {tc} tensors and {kc} metadata entries in {flen} bytes")
    h = Header(path)
    for _ in range(kc):
        key = r.string(path)
        ty = r.unpack("<I", path)
        h.kv.append((key, _read_value(r, ty, key)))
    for _ in range(tc):
        name = r.string(path)
        nd = r.unpack("<I", path)
        if nd == 0 or nd > 4:
            raise GGUFError(f"gguf: tensor {name} has {nd} dimensions")
        dims = [r.unpack("<Q", name) for _ in range(nd)]
        ty = r.unpack("<I", name)
        off = r.unpack("<Q", name)
        h.tensors.append(TensorInfo(name, dims, ty, off))
    h.data_off = _align(r.pos)
    if h.data_off > flen:
        raise GGUFError(f"{path}: tensor data starts past end of file")
    for t in h.tensors:
        if t.offset % ALIGNMENT:
            raise GGUFError(f"gguf: tensor {t.name} offset {t.offset} is not a multiple of {ALIGNMENT}")
        if h.data_off + t.offset + t.nbytes() > flen:
            raise GGUFError(f"gguf: tensor {t.name} data is outside the file")
    return h


def f32_bytes(v) -> bytes:
    return np.asarray(v, dtype="<f4").tobytes()


def f16_bytes(v) -> bytes:
    """f32 -> f16 round-to-nearest-even, the conversion of weights.rs:8-40."""
    return np.asarray(v, dtype=np.float32).astype("<f2").tobytes()
