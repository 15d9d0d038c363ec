"""Test oracle: a pure-Python restatement of the reference's GGUF reader, used
only by tests to check the backend's C parser (loom_gguf_* in the library).

Restates src/gguf/gguf.zig:131-210 (Cursor, readValue with the nesting cap),
:251-325 (parse) and src/gguf/llama.zig:259-273 with src/gguf/ggml.zig:100-180
and src/gguf/iq.zig:22-37 (resolve with overflow-checked sizes). Outcomes are
the reference's: a result, or the name of the error the reference returns.
Not part of the product path.
"""
from __future__ import annotations

import struct

MAGIC = 0x46554747
MAX_ARRAY_DEPTH = 4
HEAD_CAP = 64 << 20
U64 = (1 << 64) - 1

# ggml type -> (block width in elements, bytes per block); src/gguf/ggml.zig:126-180
TYPE_GEOM = {
    0: (1, 4), 1: (1, 2), 2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34),
    10: (256, 84), 11: (256, 110), 12: (256, 144), 13: (256, 176), 14: (256, 210),
    16: (256, 66), 17: (256, 74), 18: (256, 98), 19: (256, 50), 20: (32, 18), 21: (256, 110),
    22: (256, 82), 23: (256, 136), 29: (256, 56), 39: (32, 17),
}


class GgufErr(Exception):
    def __init__(self, name):
        super().__init__(name)
        self.name = name


class _Cursor:
    def __init__(self, buf):
        self.buf, self.pos = buf, 0

    def need(self, n):
        if self.pos + n > len(self.buf):
            raise GgufErr("TruncatedGguf")
        s = self.buf[self.pos:self.pos + n]
        self.pos += n
        return s

    def u32(self):
        return struct.unpack("<I", self.need(4))[0]

    def u64(self):
        return struct.unpack("<Q", self.need(8))[0]

    def str(self):
        n = self.u64()
        if n > 1 << 24:
            raise GgufErr("TruncatedGguf")
        return bytes(self.need(n))


def _read_value(c, vt, depth):
    """gguf.zig:166-210. Returns (kind, value) with the kinds of MetaValue."""
    if depth > MAX_ARRAY_DEPTH:
        raise GgufErr("ArrayNestingTooDeep")
    if vt == 0:
        return "uint", c.need(1)[0]
    if vt == 1:
        return "int", struct.unpack("<b", c.need(1))[0]
    if vt == 2:
        return "uint", struct.unpack("<H", c.need(2))[0]
    if vt == 3:
        return "int", struct.unpack("<h", c.need(2))[0]
    if vt == 4:
        return "uint", c.u32()
    if vt == 5:
        return "int", struct.unpack("<i", c.need(4))[0]
    if vt == 6:
        return "float", struct.unpack("<f", c.need(4))[0]
    if vt == 7:
        return "bool", c.need(1)[0] != 0
    if vt == 8:
        return "string", c.str()
    if vt == 10:
        return "uint", c.u64()
    if vt == 11:
        return "int", struct.unpack("<q", c.need(8))[0]
    if vt == 12:
        return "float", struct.unpack("<d", c.need(8))[0]
    if vt == 9:
        et = c.u32()
        count = c.u64()
        if count > 1 << 24:
            raise GgufErr("TruncatedGguf")
        if et == 8:
            return "array_str", [c.str() for _ in range(count)]
        if et == 6:
            return "array_f32", [struct.unpack("<f", c.need(4))[0] for _ in range(count)]
        if et == 5:
            return "array_i32", [struct.unpack("<i", c.need(4))[0] for _ in range(count)]
        for _ in range(count):
            _read_value(c, et, depth + 1)
        return "array", (et, count)
    raise GgufErr("UnknownValueType")


def parse(image: bytes) -> dict:
    """gguf.parse (gguf.zig:251-325) over a whole file image."""
    file_size = len(image)
    c = _Cursor(memoryview(image)[:min(file_size, HEAD_CAP)])
    if c.u32() != MAGIC:
        raise GgufErr("NotGguf")
    version = c.u32()
    if version < 2 or version > 3:
        raise GgufErr("UnsupportedGgufVersion")
    tensor_count = c.u64()
    kv_count = c.u64()
    if tensor_count > 1 << 20 or kv_count > 1 << 20:
        raise GgufErr("TruncatedGguf")
    meta = []
    for _ in range(kv_count):
        start = c.pos
        key = c.str()
        vt = c.u32()
        kind, val = _read_value(c, vt, 0)
        meta.append((key, kind, val, start, c.pos))
    tensors = []
    for _ in range(tensor_count):
        name = c.str()
        n_dims = c.u32()
        if n_dims == 0 or n_dims > 8:
            raise GgufErr("BadTensorDims")
        dims, elems = [], 1
        for _ in range(n_dims):
            d = c.u64()
            if d == 0:
                raise GgufErr("BadTensorDims")
            elems *= d
            if elems > U64:
                raise GgufErr("BadTensorDims")
            dims.append(d)
        ty = c.u32()
        off = c.u64()
        tensors.append((name, tuple(dims), ty, off))
    alignment = 32
    for key, kind, val, _, _ in meta:
        if key == b"general.alignment":
            if kind == "uint":
                alignment = val
            elif kind == "int" and val > 0:
                alignment = val
    if alignment == 0 or alignment & (alignment - 1):
        raise GgufErr("BadAlignment")
    data_offset = (c.pos + alignment - 1) // alignment * alignment
    if data_offset > file_size:
        raise GgufErr("TruncatedGguf")
    return {"version": version, "alignment": alignment, "meta": meta, "tensors": tensors,
            "data_offset": data_offset, "file_size": file_size}


def resolve(parsed: dict, name: bytes):
    """Model.resolve (llama.zig:259-273): (type, start, bytes, ne0, ne1, ne2)."""
    t = next((t for t in parsed["tensors"] if t[0] == name), None)
    if t is None:
        raise GgufErr("MissingTensor")
    _, dims, ty, off = t
    if ty not in TYPE_GEOM:
        raise GgufErr("UnsupportedTensorType")
    blk, bb = TYPE_GEOM[ty]
    ne0 = dims[0]
    ne1 = dims[1] if len(dims) > 1 else 1
    ne2 = dims[2] if len(dims) > 2 else 1
    if blk != 1 and ne0 % blk:
        raise GgufErr("BadTensorShape")
    row = (ne0 // blk) * bb
    slice_ = ne1 * row
    nbytes = slice_ * ne2
    if row > U64 or slice_ > U64 or nbytes > U64:
        raise GgufErr("BadTensorShape")
    start = parsed["data_offset"] + off
    if start > U64 or start + nbytes > U64 or start + nbytes > parsed["file_size"]:
        raise GgufErr("TruncatedGguf")
    return ty, start, nbytes, ne0, ne1, ne2
