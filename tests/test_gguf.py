"""CPU tests of the backend's GGUF reader (loom_gguf_* in the library) against
the Python restatement of the reference's parser (oracle/gguf_ref.py):
same fields on valid images, the same error name on every malformed one
(src/gguf/gguf.zig:251-325; the issue-29 checks at :288-298, :167, :152,
:184, :272, :315, :318; resolve at src/gguf/llama.zig:259-273)."""
import struct

import numpy as np
import pytest

from tests import ggufwrite as W
from loom_b200.gguf import GGUF, GgufError
from oracle import gguf_ref as R


def _meta_py(meta):
    out = {}
    for key, kind, val, _, _ in meta:
        k = key.decode(errors="replace")
        if kind == "string":
            val = val.decode(errors="replace")
        elif kind == "array_str":
            val = [s.decode(errors="replace") for s in val]
        elif kind == "array":
            val = ("array",) + tuple(val)
        out[k] = val
    return out


def outcome_c(img):
    try:
        g = GGUF(img)
    except GgufError as e:
        return ("err", e.name)
    meta = g.metadata
    for k, v in meta.items():
        if isinstance(v, np.ndarray):
            meta[k] = [float(x) if v.dtype.kind == "f" else int(x) for x in v]
    tens = [(t.name, t.dims, t.ggml_type, t.offset) for t in g.tensors]
    res = {}
    for t in g.tensors:
        try:
            v = g.resolve(t.raw_name)
            res[t.name] = (v.ggml_type, v.ptr - g.resolve_base(), v.data.nbytes, v.ne0, v.ne1, v.ne2)
        except GgufError as e:
            res[t.name] = ("err", e.name)
    if len(set(t.raw_name for t in g.tensors)) < len(g.tensors):
        res["dup"] = True
    return ("ok", g.version, g.alignment, g.data_offset, meta, tens, res)


def outcome_ref(img):
    try:
        p = R.parse(img)
    except R.GgufErr as e:
        return ("err", e.name)
    meta = _meta_py(p["meta"])
    for k, v in meta.items():
        if isinstance(v, list) and v and isinstance(v[0], float):
            meta[k] = [float(np.float32(x)) for x in v]
    tens = [(n.decode(errors="replace"), d, ty, off) for n, d, ty, off in p["tensors"]]
    res = {}
    for n, _, _, _ in p["tensors"]:
        try:
            res[n.decode(errors="replace")] = R.resolve(p, n)
        except R.GgufErr as e:
            res[n.decode(errors="replace")] = ("err", e.name)
    if len(set(t[0] for t in p["tensors"])) < len(p["tensors"]):
        res["dup"] = True
    return ("ok", p["version"], p["alignment"], p["data_offset"], meta, tens, res)


# GGUF.resolve returns a pointer into the image; the test compares offsets
def _base(self):
    import ctypes as C
    from loom_b200 import _lib
    return _lib.lib().loom_gguf_image(self._h)


GGUF.resolve_base = _base


def rich_image(alignment=32):
    rng = np.random.default_rng(7)
    meta = [
        ("general.architecture", W.T_STR, "qwen3moe"),
        ("general.alignment", W.T_U32, alignment),
        ("u8", W.T_U8, 200), ("i8", W.T_I8, -5), ("u16", W.T_U16, 65000), ("i16", W.T_I16, -300),
        ("i32", W.T_I32, -70000), ("f32", W.T_F32, 1.5), ("b", W.T_BOOL, 1), ("u64", W.T_U64, 1 << 40),
        ("i64", W.T_I64, -(1 << 40)), ("f64", W.T_F64, 0.1),
        ("tok", W.T_ARR, (W.T_STR, ["a", "bc", ""])),
        ("scores", W.T_ARR, (W.T_F32, [0.5, -1.25])),
        ("types", W.T_ARR, (W.T_I32, [1, -2, 3])),
        ("merges_u8", W.T_ARR, (W.T_U8, [1, 2, 3])),
        ("nested", W.T_ARR, (W.T_ARR, [(W.T_U32, [1, 2]), (W.T_U32, [])])),
    ]
    tensors = [
        ("token_embd.weight", (64, 3), 0, rng.integers(0, 255, 64 * 3 * 4, dtype=np.uint8).tobytes()),
        ("blk.0.ffn_gate_exps.weight", (256, 2, 4), 12, rng.integers(0, 255, 144 * 8, dtype=np.uint8).tobytes()),
        ("blk.0.ffn_down_exps.weight", (512, 1, 2), 14, rng.integers(0, 255, 210 * 4, dtype=np.uint8).tobytes()),
        ("q8", (64,), 8, rng.integers(0, 255, 68, dtype=np.uint8).tobytes()),
        ("iq4", (32, 2), 20, rng.integers(0, 255, 36, dtype=np.uint8).tobytes()),
        ("mx", (32,), 39, rng.integers(0, 255, 17, dtype=np.uint8).tobytes()),
        ("four_d", (32, 1, 1, 5), 2, rng.integers(0, 255, 18, dtype=np.uint8).tobytes()),
    ]
    return W.image(meta, tensors, alignment=alignment), tensors


@pytest.mark.parametrize("alignment", [32, 64, 256])
def test_valid_image_matches_reference(alignment):
    img, tensors = rich_image(alignment)
    c, r = outcome_c(img), outcome_ref(img)
    assert c[0] == "ok" and r[0] == "ok"
    assert c[1:4] == r[1:4]
    assert c[5] == r[5]
    assert c[6] == r[6]
    for k, v in r[4].items():
        got = c[4][k]
        if isinstance(v, float):
            assert got == pytest.approx(v, rel=0, abs=0) or got == v
        else:
            assert got == v, k
    g = GGUF(img)
    for name, dims, ty, data in tensors:
        v = g.resolve(name)
        assert v.data.tobytes() == data[:v.data.nbytes]
    assert g.get_uint("i32") is None and g.get_uint("u16") == 65000 and g.get_uint("i8") is None
    assert g.get_float("u64") == float(1 << 40) and g.get_float("f32") == 1.5
    assert g.get_string("general.architecture") == "qwen3moe" and g.get_string("u8") is None
    assert g.get_bool("b") is True and g.get_bool("u8") is True and g.get_bool("f32") is None
    assert g.find_tensor("nope") is None and g.find_meta("nope") is None


def test_open_maps_a_file(tmp_path):
    img, tensors = rich_image()
    p = tmp_path / "m.gguf"
    p.write_bytes(img)
    with GGUF.open(str(p)) as g:
        assert [t.name for t in g.tensors] == [t[0] for t in tensors]
        assert g.resolve("q8").data.tobytes() == tensors[3][3]
    with pytest.raises(GgufError) as e:
        GGUF.open(str(tmp_path / "missing.gguf"))
    assert e.value.name == "FileNotFound"


def _hdr(n_t, n_kv, version=3):
    return struct.pack("<IIQQ", W.MAGIC, version, n_t, n_kv)


def _tinfo(name, dims, ty, off):
    return W._str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims) + \
        struct.pack("<IQ", ty, off)


MALFORMED = {
    "bad_magic": (b"GGUG" + _hdr(0, 0)[4:], "NotGguf"),
    "version1": (_hdr(0, 0, 1), "UnsupportedGgufVersion"),
    "version4": (_hdr(0, 0, 4), "UnsupportedGgufVersion"),
    "too_many_tensors": (_hdr((1 << 20) + 1, 0), "TruncatedGguf"),
    "too_many_kv": (_hdr(0, (1 << 20) + 1), "TruncatedGguf"),
    "huge_string": (_hdr(0, 1) + struct.pack("<Q", (1 << 24) + 1), "TruncatedGguf"),
    "zero_dims": (_hdr(1, 0) + _tinfo("t", (), 0, 0), "BadTensorDims"),
    "nine_dims": (_hdr(1, 0) + _tinfo("t", (1,) * 9, 0, 0), "BadTensorDims"),
    "zero_dim": (_hdr(1, 0) + _tinfo("t", (4, 0), 0, 0), "BadTensorDims"),
    "elem_overflow": (_hdr(1, 0) + _tinfo("t", (1 << 32, 1 << 32), 0, 0), "BadTensorDims"),
    "deep_nesting": (_hdr(0, 1) + W._str("k") + struct.pack("<I", W.T_ARR) +
                     b"".join(struct.pack("<IQ", W.T_ARR, 1) for _ in range(5)) + struct.pack("<IQ", W.T_U8, 0),
                     "ArrayNestingTooDeep"),
    "nesting_at_cap": (_hdr(0, 1) + W._str("k") + struct.pack("<I", W.T_ARR) +
                       b"".join(struct.pack("<IQ", W.T_ARR, 1) for _ in range(4)) + struct.pack("<IQ", W.T_U8, 0) +
                       b"\0" * 32, None),
    "unknown_type": (_hdr(0, 1) + W._str("k") + struct.pack("<I", 13) + b"\0" * 8, "UnknownValueType"),
    "huge_array": (_hdr(0, 1) + W._str("k") + struct.pack("<IIQ", W.T_ARR, W.T_U8, (1 << 24) + 1), "TruncatedGguf"),
    "alignment_zero": (_hdr(0, 1) + W._str("general.alignment") + struct.pack("<II", W.T_U32, 0), "BadAlignment"),
    "alignment_48": (_hdr(0, 1) + W._str("general.alignment") + struct.pack("<II", W.T_U32, 48), "BadAlignment"),
    "alignment_neg_int": (_hdr(0, 1) + W._str("general.alignment") + struct.pack("<Ii", W.T_I32, -8) + b"\0" * 16, None),
    "data_past_end": (_hdr(0, 1) + W._str("general.alignment") + struct.pack("<II", W.T_U32, 1 << 20),
                      "TruncatedGguf"),
    "empty": (b"", "TruncatedGguf"),
}


@pytest.mark.parametrize("case", sorted(MALFORMED))
def test_malformed_header_same_error(case):
    img, want = MALFORMED[case]
    c, r = outcome_c(img), outcome_ref(img)
    assert c == r
    if want is None:
        assert c[0] == "ok"
    else:
        assert c == ("err", want)


RESOLVE = {
    "missing_type": ((32,), 15, 64, "UnsupportedTensorType"),
    "ragged_row": ((100,), 12, 144, "BadTensorShape"),
    "bytes_overflow": ((1 << 31, 1 << 31, 2), 0, 144, "BadTensorShape"),
    "offset_overflow": ((32,), 0, 128, "TruncatedGguf"),
    "past_end": ((64,), 0, 128, "TruncatedGguf"),
    "fits": ((32,), 0, 128, None),
}


@pytest.mark.parametrize("case", sorted(RESOLVE))
def test_resolve_checks_same_error(case):
    dims, ty, nbytes, want = RESOLVE[case]
    off = (1 << 64) - 16 if case == "offset_overflow" else 0
    img = _hdr(1, 0) + _tinfo("t", dims, ty, off)
    img += b"\0" * ((-len(img)) % 32) + b"\1" * nbytes
    c, r = outcome_c(img), outcome_ref(img)
    assert c == r
    got = c[6]["t"]
    if want is None:
        assert got[0] == ty
    else:
        assert got == ("err", want)
    g = GGUF(img)
    with pytest.raises(GgufError) as e:
        g.resolve("absent")
    assert e.value.name == "MissingTensor"


def test_every_truncation_agrees():
    """Every prefix of a valid image: the same outcome (mostly TruncatedGguf)."""
    img, _ = rich_image()
    for n in range(0, len(img), 3):
        assert outcome_c(img[:n]) == outcome_ref(img[:n]), n


def test_random_mutations_agree():
    """Bytes of the header flipped at random: the C reader and the restated
    reference reach the same outcome (error name or the same fields)."""
    img, _ = rich_image()
    rng = np.random.default_rng(29)
    head = GGUF(img).data_offset
    for _ in range(400):
        b = bytearray(img)
        for _ in range(int(rng.integers(1, 4))):
            i = int(rng.integers(0, head))
            b[i] = int(rng.integers(0, 256))
        b = bytes(b)
        assert outcome_c(b) == outcome_ref(b)
