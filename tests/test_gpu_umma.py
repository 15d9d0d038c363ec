"""The tcgen05 bf16 GEMM building block (kind::f16, f32 accumulator in TMEM,
K-major no-swizzle shared-memory operands) against a float64 reference on
the same bf16 inputs."""
import ctypes as C

import numpy as np
import pytest

from loom_b200 import _lib

pytestmark = pytest.mark.gpu


def bf16_bits(x):
    f = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return ((f + 0x7FFF + ((f >> 16) & 1)) >> 16).astype(np.uint16)  # round to nearest even


def bf16_val(b):
    return (b.astype(np.uint32) << 16).view(np.float32)


@pytest.mark.parametrize("M,N,K", [(128, 16, 64), (128, 32, 128), (256, 48, 192), (128, 256, 256), (384, 128, 2048)])
def test_umma_bf16_gemm(be, M, N, K):
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    a = bf16_bits(rng.standard_normal((M, K)))
    b = bf16_bits(rng.standard_normal((N, K)))
    d = np.full((M, N), np.nan, np.float32)
    lib = _lib.lib()
    rc = lib.loom_cuda_umma_selftest(a.ctypes.data_as(C.c_void_p), b.ctypes.data_as(C.c_void_p),
                                     d.ctypes.data_as(C.c_void_p), M, N, K)
    assert rc == 0
    want = bf16_val(a).astype(np.float64) @ bf16_val(b).astype(np.float64).T
    err = np.abs(d - want).max() / np.abs(want).max()
    assert err < 1e-5, err
