"""GPU test of the allocation-free MoE layer (loom_cuda_moe_forward_noalloc).

Some callers cannot allocate device memory while they run: code recorded
into a CUDA stream capture that another component owns, or an engine whose
device memory is budgeted once at start-up. For them the backend offers one
entry point whose scratch is a fixed array in the library image instead of
memory obtained from cudaMalloc. This test calls it through the C ABI twice in
a row (the array keeps the previous call's contents, so the second call checks
that nothing stale leaks through) and compares each result with the regular
entry point, loom_cuda_moe_forward, within the FFN tolerance used by the other
MoE tests (2e-3 relative L2). This file is named to be collected last.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from loom_b200 import _lib
from loom_b200.device import DeviceTensor, MoeLayer
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu
TOL = 2e-3


def _noalloc(layer, x, out, residual):
    d = layer.desc()
    rc = _lib.lib().loom_cuda_moe_forward_noalloc(C.byref(d), x.data_ptr(), x.shape[0], out.data_ptr(),
                                                   residual.data_ptr(), torch.cuda.current_stream().cuda_stream)
    _lib.must(rc, "moe_forward_noalloc")


def test_noalloc_layer_matches_regular_entry_point_twice(be, orc):
    ne, k, dim, ffn = 32, 8, 2048, 768  # Qwen3-30B-A3B expert shapes, fewer experts
    g = orc.synth(12, ne * ffn * dim // 256, 901)
    u = orc.synth(12, ne * ffn * dim // 256, 902)
    d = orc.synth(14, ne * dim * ffn // 256, 903)
    rw = orc.synth(0, ne * dim, seed=904, sigma=0.02)
    L = MoeLayer(dim, ffn, ne, k, DeviceTensor.upload(12, g), DeviceTensor.upload(12, u),
                 DeviceTensor.upload(14, d), router=DeviceTensor.upload(0, rw))
    try:
        for call, T in enumerate((1, 3)):
            x = torch.from_numpy(orc.synth(0, T * dim, seed=910 + call).reshape(T, dim)).cuda()
            res = torch.from_numpy(orc.synth(0, T * dim, seed=920 + call).reshape(T, dim)).cuda()
            want = torch.full((T, dim), float("nan"), device="cuda")
            L.forward(x, want, residual=res)
            got = torch.full((T, dim), float("nan"), device="cuda")
            _noalloc(L, x, got, res)
            torch.cuda.synchronize()
            w, o = want.cpu().numpy(), got.cpu().numpy()
            assert np.all(np.isfinite(o))
            assert rel_l2(o, w) < TOL, (call, rel_l2(o, w))
    finally:
        for t in (L.gate, L.up, L.down, L.router):
            t.free()


def test_noalloc_rejects_oversized_layers(be):
    ne, k, dim, ffn = 8, 2, 512, 256
    g = DeviceTensor.synth(12, ne * ffn * dim // 256, 1)
    u = DeviceTensor.synth(12, ne * ffn * dim // 256, 2)
    d = DeviceTensor.synth(14, ne * dim * ffn // 256, 3)
    r = DeviceTensor.synth(0, ne * dim, 4, 0.02)
    L = MoeLayer(dim, ffn, ne, k, g, u, d, router=r)
    try:
        T = 17  # beyond the 16-token limit
        x = torch.zeros((T, dim), device="cuda")
        out = torch.zeros((T, dim), device="cuda")
        dsc = L.desc()
        rc = _lib.lib().loom_cuda_moe_forward_noalloc(C.byref(dsc), x.data_ptr(), T, out.data_ptr(), None, None)
        assert rc == _lib.DECLINED and "16 tokens" in _lib.last_error()
    finally:
        for t in (g, u, d, r):
            t.free()
