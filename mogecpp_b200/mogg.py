"""MOGG v1 image writer: packs a model's metadata and tensors into the
container mogecpp loads (synthetic refiner models for the tests and the
benchmark, or any caller that holds weights in memory).

The layout is the one the reference reads (mogecpp
src/mogg.cpp:247-312, written by tools/convert_moge.py:101-180): a 40-byte
header (magic "MOGG\\0\\0\\0\\1", version, metadata count, tensor count,
alignment, metadata offset, data start), metadata records {u16 key length,
key, u8 tag, u32 payload bytes, payload}, tensor records {u16 name length,
name, u16 type, u8 ndim, u8 flags, i64 ne[4], u64 offset, u64 size}, then
the aligned tensor payloads.  ne is ggml order (ne0 fastest): a numpy array
of shape (rows, cols) is stored with ne = (cols, rows).
"""

from __future__ import annotations

import struct

import numpy as np

MAGIC = b"MOGG\x00\x00\x00\x01"
T_F32, T_F16, T_BF16, T_I32, T_Q8_0 = 1, 2, 3, 4, 12
TF_SPARSE, TF_SPARSE_PACKED = 1 << 3, 1 << 4
META_I64, META_F64, META_STR, META_I64_LIST, META_BOOL = 1, 2, 3, 4, 6


def _p16(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<H", len(b)) + b


def _meta(v) -> tuple[int, bytes]:
    if isinstance(v, bool):
        return META_BOOL, struct.pack("<B", int(v))
    if isinstance(v, int):
        return META_I64, struct.pack("<q", v)
    if isinstance(v, float):
        return META_F64, struct.pack("<d", v)
    if isinstance(v, str):
        b = v.encode()
        return META_STR, struct.pack("<I", len(b)) + b
    if isinstance(v, (list, tuple)):
        return META_I64_LIST, struct.pack("<I", len(v)) + b"".join(struct.pack("<q", int(x)) for x in v)
    raise TypeError(type(v))


def build(meta: dict, tensors: list, alignment: int = 64) -> bytes:
    """tensors: (name, type, shape in numpy order, payload bytes, flags)."""
    mblob = b""
    for k, v in meta.items():
        tag, payload = _meta(v)
        mblob += _p16(k) + struct.pack("<BI", tag, len(payload)) + payload

    def index(offs):
        out = b""
        for (name, typ, shape, data, flags), off in zip(tensors, offs):
            ne = list(reversed(shape)) + [1] * (4 - len(shape))
            out += _p16(name) + struct.pack("<HBB", typ, len(shape), flags) + struct.pack("<4q", *ne)
            out += struct.pack("<QQ", off, len(data))
        return out

    up = lambda v: (v + alignment - 1) // alignment * alignment
    data_start = up(40 + len(mblob) + len(index([0] * len(tensors))))
    offs, cur = [], data_start
    for t in tensors:
        cur = up(cur)
        offs.append(cur)
        cur += len(t[3])
    img = bytearray(MAGIC + struct.pack("<IIIIQQ", 1, len(meta), len(tensors), alignment, 40, data_start))
    img += mblob + index(offs)
    img += b"\0" * (data_start - len(img))
    for t, off in zip(tensors, offs):
        img += b"\0" * (off - len(img))
        img += t[3]
    return bytes(img)


def tensor(name: str, a: np.ndarray, typ: int) -> tuple:
    """A float array stored as F32 / F16 (sparse27 names get the packed flags)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    payload = a.tobytes() if typ == T_F32 else a.astype(np.float16).tobytes()
    flags = TF_SPARSE | (TF_SPARSE_PACKED if name.endswith("mogg_sparse27") else 0)
    return (name, typ, a.shape, payload, flags)
