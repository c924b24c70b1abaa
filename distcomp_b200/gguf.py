"""GGUF v3 writer and a small reader, for building synthetic seeded models.

The layout follows the GGUF definition the reference reads
(src/gguf.c:233-336): little-endian header ``GGUF``, version, uint64 tensor
and key counts, key/value pairs, tensor infos (name, n_dims, uint64 dims,
ggml type, uint64 offset relative to the data block), then the data block
aligned to ``general.alignment`` (32) with each tensor 32-byte aligned.

The writer fills one preallocated ``numpy.uint8`` buffer, so multi-GB models
are built without intermediate copies: tensor payloads are written in place
through ``GGUFBuilder.tensor_view``.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

# GGUF metadata value types
T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 = range(13)

# ggml tensor types
F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q8_1 = 0, 1, 2, 3, 6, 7, 8, 9
Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, Q8_K = 10, 11, 12, 13, 14, 15

BLOCK = {Q4_0: (32, 18), Q4_1: (32, 20), Q5_0: (32, 22), Q5_1: (32, 24), Q8_0: (32, 34),
         Q8_1: (32, 36), Q2_K: (256, 84), Q3_K: (256, 110), Q4_K: (256, 144), Q5_K: (256, 176),
         Q6_K: (256, 210), Q8_K: (256, 292)}
TYPE_NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q4_1: "Q4_1", Q5_0: "Q5_0", Q5_1: "Q5_1",
              Q8_0: "Q8_0", Q8_1: "Q8_1", Q2_K: "Q2_K", Q3_K: "Q3_K", Q4_K: "Q4_K", Q5_K: "Q5_K",
              Q6_K: "Q6_K", Q8_K: "Q8_K"}
ALIGN = 32


def type_nbytes(t: int, n: int) -> int:
    """Bytes of n elements of ggml type t (src/gguf.c:149-174)."""
    if t == F32:
        return 4 * n
    if t == F16:
        return 2 * n
    be, bb = BLOCK[t]
    if n % be:
        raise ValueError(f"{n} elements is not a whole number of {TYPE_NAMES[t]} blocks")
    return n // be * bb


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, vtype: int, val) -> bytes:
    out = _str(key) + struct.pack("<I", vtype)
    if vtype == T_STR:
        return out + _str(val)
    if vtype == T_ARR:
        etype, items = val
        out += struct.pack("<IQ", etype, len(items))
        if etype == T_STR:
            return out + b"".join(_str(s) for s in items)
        fmt = {T_U32: "<I", T_I32: "<i", T_F32: "<f"}[etype]
        return out + b"".join(struct.pack(fmt, x) for x in items)
    fmt = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i", T_F32: "<f",
           T_BOOL: "<B", T_U64: "<Q", T_I64: "<q", T_F64: "<d"}[vtype]
    return out + struct.pack(fmt, val)


@dataclass
class _TInfo:
    name: str
    dims: tuple
    gtype: int
    nbytes: int
    offset: int = 0


@dataclass
class GGUFBuilder:
    """Two-phase writer: declare metadata and tensors, then ``finalize()``
    allocates the file image and ``tensor_view(name)`` exposes each tensor's
    bytes for in-place filling."""
    kvs: list = field(default_factory=list)
    tensors: list = field(default_factory=list)
    buf: np.ndarray | None = None
    data_start: int = 0

    def add_kv(self, key: str, vtype: int, val) -> None:
        self.kvs.append((key, vtype, val))

    def add_tensor(self, name: str, dims, gtype: int) -> None:
        n = 1
        for d in dims:
            n *= int(d)
        self.tensors.append(_TInfo(name, tuple(int(d) for d in dims), gtype, type_nbytes(gtype, n)))

    def finalize(self) -> np.ndarray:
        head = struct.pack("<IIQQ", 0x46554747, 3, len(self.tensors), len(self.kvs))
        body = b"".join(_kv(k, t, v) for k, t, v in self.kvs)
        off = 0
        infos = []
        for t in self.tensors:
            t.offset = off
            infos.append(_str(t.name) + struct.pack("<I", len(t.dims)) +
                         b"".join(struct.pack("<Q", d) for d in t.dims) + struct.pack("<IQ", t.gtype, off))
            off += t.nbytes
            off = (off + ALIGN - 1) // ALIGN * ALIGN
        header = head + body + b"".join(infos)
        self.data_start = (len(header) + ALIGN - 1) // ALIGN * ALIGN
        self.buf = np.zeros(self.data_start + off, dtype=np.uint8)
        self.buf[: len(header)] = np.frombuffer(header, dtype=np.uint8)
        return self.buf

    def tensor_view(self, name: str) -> np.ndarray:
        for t in self.tensors:
            if t.name == name:
                s = self.data_start + t.offset
                return self.buf[s: s + t.nbytes]
        raise KeyError(name)

    def info(self, name: str) -> _TInfo:
        for t in self.tensors:
            if t.name == name:
                return t
        raise KeyError(name)


def read_tensor_table(buf) -> dict:
    """Minimal reader: {name: (gtype, dims, memoryview of the bytes)} plus
    metadata under the key ``"__meta__"``.  For tests and tools."""
    mv = memoryview(buf).cast("B")
    p = 0

    def rd(fmt):
        nonlocal p
        v = struct.unpack_from(fmt, mv, p)
        p += struct.calcsize(fmt)
        return v[0] if len(v) == 1 else v

    def rs():
        n = rd("<Q")
        nonlocal p
        s = bytes(mv[p: p + n]).decode("utf-8", "replace")
        p += n
        return s

    magic, ver, nt, nkv = rd("<IIQQ")
    assert magic == 0x46554747 and ver in (2, 3)
    meta = {}
    scal = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i", T_F32: "<f",
            T_BOOL: "<B", T_U64: "<Q", T_I64: "<q", T_F64: "<d"}
    for _ in range(nkv):
        k = rs()
        t = rd("<I")
        if t == T_STR:
            meta[k] = rs()
        elif t == T_ARR:
            et, n = rd("<IQ")
            meta[k] = [rs() if et == T_STR else rd(scal[et]) for _ in range(n)]
        else:
            meta[k] = rd(scal[t])
    infos = []
    for _ in range(nt):
        name = rs()
        nd = rd("<I")
        dims = [rd("<Q") for _ in range(nd)]
        gt, off = rd("<IQ")
        infos.append((name, gt, dims, off))
    align = int(meta.get("general.alignment", ALIGN))
    base = (p + align - 1) // align * align
    out = {"__meta__": meta}
    for name, gt, dims, off in infos:
        n = int(np.prod(dims)) if dims else 1
        nb = type_nbytes(gt, n)
        out[name] = (gt, dims, mv[base + off: base + off + nb])
    return out
