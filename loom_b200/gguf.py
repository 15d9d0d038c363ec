"""GGUF tensor table through the backend library (loom_gguf_* in
include/loom_cuda.h): the reader a host engine uses to find every weight's
bytes before it hands them to the device.

Mirrors the reference's `Parsed` API (src/gguf/gguf.zig:82-126: findMeta,
getUint, getFloat, getString, getBool, findTensor) and the engine's checked
`Model.resolve` (src/gguf/llama.zig:259-273). Parse errors raise GgufError
carrying the reference's error name (TruncatedGguf, BadTensorDims, ...).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib

META_INT, META_UINT, META_FLOAT, META_BOOL, META_STRING = 1, 2, 3, 4, 5
META_ARRAY_STR, META_ARRAY_F32, META_ARRAY_I32, META_ARRAY = 6, 7, 8, 9


class GgufError(ValueError):
    def __init__(self, name: str):
        super().__init__(name)
        self.name = name


@dataclass
class TensorInfo:
    name: str
    dims: tuple
    ggml_type: int
    offset: int
    raw_name: bytes = b""


@dataclass
class View:
    """A resolved tensor: its bytes (a zero-copy view of the image) and shape."""
    ggml_type: int
    data: np.ndarray  # uint8 view into the image
    ne0: int
    ne1: int
    ne2: int

    @property
    def ptr(self) -> int:
        return self.data.ctypes.data

    def weight(self) -> _lib.Weight:
        return _lib.Weight(self.ggml_type, self.ptr, self.data.nbytes)


def _b(name) -> bytes:
    return name if isinstance(name, bytes) else name.encode()


def _err() -> str:
    e = _lib.lib().loom_gguf_error()
    return e.decode() if e else "unknown"


class GGUF:
    """A parsed GGUF image: `GGUF(bytes_or_array)` parses memory the object
    keeps alive; `GGUF.open(path)` maps a file read-only."""

    def __init__(self, image=None, *, _handle=None, _keep=None):
        L = _lib.lib()
        if _handle is None:
            buf = np.frombuffer(bytes(image), np.uint8) if not isinstance(image, np.ndarray) else image
            buf = np.ascontiguousarray(buf.view(np.uint8).reshape(-1))
            _keep = buf
            _handle = L.loom_gguf_parse(buf.ctypes.data_as(C.c_void_p) if buf.size else None, buf.size)
            if not _handle:
                raise GgufError(_err())
        self._h = _handle
        self._keep = _keep
        self.version = L.loom_gguf_version(self._h)
        self.alignment = L.loom_gguf_alignment(self._h)
        self.data_offset = L.loom_gguf_data_offset(self._h)
        self.file_size = L.loom_gguf_file_size(self._h)

    @classmethod
    def open(cls, path: str) -> "GGUF":
        h = _lib.lib().loom_gguf_open(path.encode())
        if not h:
            raise GgufError(_err())
        return cls(_handle=h)

    def close(self):
        if self._h:
            _lib.lib().loom_gguf_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    # ---- tensor table ---------------------------------------------------------

    def _info(self, t: _lib.GgufTensor) -> TensorInfo:
        raw = C.string_at(t.name, t.name_len) if t.name_len else b""
        return TensorInfo(raw.decode(errors="replace"), tuple(int(t.dims[d]) for d in range(t.n_dims)),
                          int(t.ggml_type), int(t.offset), raw)

    @property
    def tensors(self) -> list:
        L = _lib.lib()
        out = []
        for k in range(L.loom_gguf_n_tensors(self._h)):
            t = _lib.GgufTensor()
            L.loom_gguf_tensor_info(self._h, k, C.byref(t))
            out.append(self._info(t))
        return out

    def find_tensor(self, name):
        t = _lib.GgufTensor()
        if _lib.lib().loom_gguf_find_tensor(self._h, _b(name), C.byref(t)) != _lib.OK:
            return None
        return self._info(t)

    def resolve(self, name) -> View:
        v = _lib.GgufView()
        if _lib.lib().loom_gguf_resolve(self._h, _b(name), C.byref(v)) != _lib.OK:
            raise GgufError(_err())
        arr = np.ctypeslib.as_array(C.cast(v.data, C.POINTER(C.c_uint8)), shape=(v.bytes,)) if v.bytes else \
            np.zeros(0, np.uint8)
        return View(v.ggml_type, arr, v.ne0, v.ne1, v.ne2)

    # ---- metadata ---------------------------------------------------------------

    def _value(self, m: _lib.GgufValue):
        k = m.kind
        if k == META_INT:
            return int(m.i)
        if k in (META_UINT,):
            return int(m.u)
        if k == META_FLOAT:
            return float(m.f)
        if k == META_BOOL:
            return bool(m.u)
        if k == META_STRING:
            return C.string_at(m.str, m.str_len).decode(errors="replace") if m.str_len else ""
        if k == META_ARRAY_F32:
            return np.frombuffer(C.string_at(m.array, 4 * m.count), "<f4").copy() if m.count else \
                np.zeros(0, np.float32)
        if k == META_ARRAY_I32:
            return np.frombuffer(C.string_at(m.array, 4 * m.count), "<i4").copy() if m.count else \
                np.zeros(0, np.int32)
        if k == META_ARRAY_STR:
            out, p = [], m.array
            for _ in range(m.count):
                n = int.from_bytes(C.string_at(p, 8), "little")
                out.append(C.string_at(p + 8, n).decode(errors="replace") if n else "")
                p += 8 + n
            return out
        return ("array", int(m.elem_type), int(m.count))

    @property
    def metadata(self) -> dict:
        L = _lib.lib()
        out = {}
        for k in range(L.loom_gguf_n_meta(self._h)):
            m = _lib.GgufValue()
            L.loom_gguf_meta(self._h, k, C.byref(m))
            out[C.string_at(m.key, m.key_len).decode(errors="replace")] = self._value(m)
        return out

    def find_meta(self, key: str):
        m = _lib.GgufValue()
        if _lib.lib().loom_gguf_find_meta(self._h, key.encode(), C.byref(m)) != _lib.OK:
            return None
        return self._value(m)

    def get_uint(self, key: str):
        v = C.c_uint64()
        return int(v.value) if _lib.lib().loom_gguf_get_uint(self._h, key.encode(), C.byref(v)) == _lib.OK else None

    def get_float(self, key: str):
        v = C.c_double()
        return float(v.value) if _lib.lib().loom_gguf_get_float(self._h, key.encode(), C.byref(v)) == _lib.OK \
            else None

    def get_string(self, key: str):
        p, n = C.c_void_p(), C.c_size_t()
        if _lib.lib().loom_gguf_get_string(self._h, key.encode(), C.byref(p), C.byref(n)) != _lib.OK:
            return None
        return C.string_at(p.value, n.value).decode(errors="replace") if n.value else ""

    def get_bool(self, key: str):
        v = C.c_int()
        return bool(v.value) if _lib.lib().loom_gguf_get_bool(self._h, key.encode(), C.byref(v)) == _lib.OK \
            else None
