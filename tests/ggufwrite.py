"""Writes GGUF v3 images for the tests: the layout the reference's fixture
writers emit (src/gguf/gguf.zig:335-406 writeFixture): header, metadata
key/values, tensor infos, padding to `general.alignment`, tensor data at
aligned offsets. Values are given as (gguf value type, python value)."""
from __future__ import annotations

import struct

MAGIC = 0x46554747
T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 = range(13)


def _str(s) -> bytes:
    b = s.encode() if isinstance(s, str) else bytes(s)
    return struct.pack("<Q", len(b)) + b


def value(vt: int, v) -> bytes:
    fmt = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i", T_F32: "<f",
           T_BOOL: "<B", T_U64: "<Q", T_I64: "<q", T_F64: "<d"}
    if vt in fmt:
        return struct.pack(fmt[vt], int(v) if vt not in (T_F32, T_F64) else v)
    if vt == T_STR:
        return _str(v)
    if vt == T_ARR:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(value(et, x) for x in items)
    raise ValueError(vt)


def image(meta: list, tensors: list, alignment: int = 32, version: int = 3) -> bytes:
    """meta: [(key, vt, value)]; tensors: [(name, dims, ggml_type, data bytes)].
    Tensor data is laid out in order, each at an `alignment` boundary."""
    head = bytearray(struct.pack("<IIQQ", MAGIC, version, len(tensors), len(meta)))
    for k, vt, v in meta:
        head += _str(k) + struct.pack("<I", vt) + value(vt, v)
    off, offs = 0, []
    for name, dims, ty, data in tensors:
        offs.append(off)
        head += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", ty, off)
        off = (off + len(data) + alignment - 1) // alignment * alignment
    head += b"\0" * ((-len(head)) % alignment)
    body = bytearray(off if tensors else 0)
    for (name, dims, ty, data), o in zip(tensors, offs):
        body[o:o + len(data)] = bytes(data)
    # trim trailing padding after the last tensor, as a writer that stops at its last byte would
    if tensors:
        body = body[:offs[-1] + len(bytes(tensors[-1][3]))]
    return bytes(head) + bytes(body)
