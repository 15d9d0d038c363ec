"""CPU checks of the C ABI library: it loads, exports every symbol the public
header declares, and declines cleanly when no device is initialised."""
import ctypes as C

import numpy as np

from loom_b200 import _lib


def test_library_exports_every_header_symbol():
    L = _lib.lib()
    syms = _lib.header_symbols()
    assert len(syms) >= 20
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing


def test_every_exported_symbol_is_declared():
    """The library exports no loom_cuda_* entry that the header leaves out."""
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if ln.split() and ln.split()[-1].startswith(("loom_cuda_", "loom_gguf_"))}
    undeclared = sorted(exported - set(_lib.header_symbols()))
    assert not undeclared, undeclared


def test_seam_declines_before_init():
    L = _lib.lib()
    out = np.zeros(4, np.float32)
    x = np.zeros(256, np.float32)
    w = np.zeros(144 * 4, np.uint8)
    rc = L.loom_cuda_matvec(12, out.ctypes.data_as(C.c_void_p), w.ctypes.data_as(C.c_void_p), w.nbytes,
                            x.ctypes.data_as(C.c_void_p), 4, 256)
    assert rc == _lib.DECLINED
    assert "init" in _lib.last_error()
    assert L.loom_cuda_register_arena(w.ctypes.data_as(C.c_void_p), w.nbytes) == _lib.DECLINED
    assert L.loom_cuda_materialize_arenas() == 0
    assert L.loom_cuda_take_cmdbuf_count() == 0
    # the whole-model batch entries decline the same way, having done nothing
    t = np.array([1, 2, 3], np.uint32)
    nxt = np.zeros(3, np.uint32)
    assert L.loom_cuda_model_prefill(7, t.ctypes.data_as(C.c_void_p), 3, 0, None,
                                     nxt.ctypes.data_as(C.POINTER(C.c_uint32))) == _lib.DECLINED
    assert L.loom_cuda_model_decode_batch(7, t.ctypes.data_as(C.c_void_p), t.ctypes.data_as(C.c_void_p), 3, None,
                                          nxt.ctypes.data_as(C.c_void_p)) == _lib.DECLINED
    assert list(nxt) == [0, 0, 0]


def test_ctypes_structs_match_the_header(tmp_path):
    """Every ctypes mirror of a header struct has the C size (a field missing on
    either side would otherwise pass silently)."""
    import shutil
    import subprocess
    import pytest
    if not shutil.which("gcc"):
        pytest.skip("no C compiler")
    names = {"loom_moe_desc": _lib.MoeDesc, "loom_model_layer": _lib.ModelLayer, "loom_model_desc": _lib.ModelDesc,
             "loom_weight": _lib.Weight, "loom_routed_cfg": _lib.RoutedCfg, "loom_gguf_tensor": _lib.GgufTensor,
             "loom_gguf_value": _lib.GgufValue, "loom_gguf_view": _lib.GgufView, "loom_shard": _lib.Shard}
    src = tmp_path / "sz.c"
    src.write_text('#include <stdio.h>\n#include "%s"\nint main(void){%s return 0;}\n' % (
        _lib.HEADER, " ".join('printf("%%zu\\n", sizeof(%s));' % n for n in names)))
    exe = tmp_path / "sz"
    subprocess.run(["gcc", "-o", str(exe), str(src)], check=True)
    sizes = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    for (n, cls), want in zip(names.items(), sizes):
        assert C.sizeof(cls) == want, (n, C.sizeof(cls), want)
