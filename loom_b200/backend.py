"""Python mirror of Loom's compute-backend seam (src/compute/backend.zig) for
the MoE hot path, bound to the CUDA backend's C ABI (include/loom_cuda.h).

Names, argument meaning and error behaviour follow the seam:
  matvec / matmul / dequantRow   -- always run; raise on failure (the seam's
                                    void ops have no decline path here, and
                                    there is no CPU fallback)
  moeFfnBlock / moeFfnBlockRouted / moeRoute / registerArena
                                 -- return True when done, False when the
                                    backend declines (the caller then runs
                                    its own path); raise on a CUDA error
Slices are numpy arrays: weights are uint8 GGUF bytes, activations float32.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

from . import _lib
from ._lib import DECLINED, OK, LoomCudaError

F32, Q4_0, Q8_0, Q4_K, Q6_K = 0, 2, 8, 12, 14
name = "cuda"


def _p(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _u8(a) -> np.ndarray:
    if a.dtype != np.uint8:
        a = a.view(np.uint8)
    return np.ascontiguousarray(a)


@dataclass
class WeightRef:  # src/compute/cpu.zig:21
    ty: int
    data: np.ndarray

    def c(self) -> _lib.Weight:
        d = _u8(self.data)
        return _lib.Weight(self.ty, d.ctypes.data, d.nbytes)


@dataclass
class ExpertRef:  # src/compute/cpu.zig:23
    gate: WeightRef
    up: WeightRef
    down: WeightRef
    weight: float
    ffn: int


@dataclass
class RoutedCfg:  # src/compute/cpu.zig:61
    n_expert: int
    n_used: int
    gating_sigmoid: bool
    weights_norm: bool
    weights_scale: float


def init(device: int = 0) -> None:
    _lib.must(_lib.lib().loom_cuda_init(device), "loom_cuda_init")


def parallelBegin(n: int) -> None:  # backend.zig:225
    _lib.lib().loom_cuda_parallel_begin(n)


def parallelEnd() -> None:  # backend.zig:226
    _lib.lib().loom_cuda_parallel_end()


def MAX_BATCH() -> int:  # backend.zig:229
    return int(_lib.lib().loom_cuda_max_batch())


def matvec(t: int, out: np.ndarray, data: np.ndarray, x: np.ndarray, rows: int, cols: int) -> None:
    """backend.zig:62: out[r] = dot(W[r], x)."""
    d, xx = _u8(data), _f32(x)
    assert out.dtype == np.float32 and out.size >= rows and out.flags.c_contiguous
    _lib.must(_lib.lib().loom_cuda_matvec(t, _p(out), _p(d), d.nbytes, _p(xx), rows, cols), "matvec")


def matmul(t: int, out: np.ndarray, data: np.ndarray, xs: np.ndarray, n: int, rows: int, cols: int) -> None:
    """backend.zig:66: out[k*rows + r] = dot(W[r], xs[k*cols..]); equals n matvecs."""
    d, xx = _u8(data), _f32(xs)
    assert out.dtype == np.float32 and out.size >= n * rows and out.flags.c_contiguous
    _lib.must(_lib.lib().loom_cuda_matmul(t, _p(out), _p(d), d.nbytes, _p(xx), n, rows, cols), "matmul")


def dequantRow(t: int, out: np.ndarray, data: np.ndarray, r: int, cols: int) -> None:
    """backend.zig:69."""
    d = _u8(data)
    assert out.dtype == np.float32 and out.size >= cols and out.flags.c_contiguous
    _lib.must(_lib.lib().loom_cuda_dequant_row(t, _p(out), _p(d), d.nbytes, r, cols), "dequantRow")


def moeRoute(logits, bias, ids_out: np.ndarray, gates_out: np.ndarray, gating_sigmoid: bool, weights_norm: bool,
             weights_scale: float) -> bool:
    """backend.zig:183 (cpu.zig:86)."""
    lg = _f32(logits)
    b = None if bias is None else _f32(bias)
    assert ids_out.dtype == np.uint32 and gates_out.dtype == np.float32
    rc = _lib.lib().loom_cuda_moe_route(_p(lg), _p(b), lg.size, _p(ids_out), _p(gates_out), ids_out.size,
                                        int(gating_sigmoid), int(weights_norm), float(weights_scale))
    return _lib.check(rc, "moeRoute") == OK


def moeFfnBlock(normed, experts: Sequence[ExpertRef], out: np.ndarray) -> bool:
    """backend.zig:104 (cpu.zig:27)."""
    x = _f32(normed)
    arr = (_lib.ExpertRef * len(experts))()
    keep = []
    for i, e in enumerate(experts):
        refs = [e.gate.c(), e.up.c(), e.down.c()]
        keep.append((e.gate.data, e.up.data, e.down.data))
        arr[i] = _lib.ExpertRef(refs[0], refs[1], refs[2], e.weight, e.ffn)
    rc = _lib.lib().loom_cuda_moe_ffn_block(_p(x), x.size, C.cast(arr, C.c_void_p), len(experts), _p(out))
    del keep
    return _lib.check(rc, "moeFfnBlock") == OK


def moeFfnBlockRouted(normed, logits, bias, gate_w: WeightRef, up_w: WeightRef, down_w: WeightRef,
                      shexp: Optional[Sequence[WeightRef]], ffn: int, shexp_ffn: int, cfg: RoutedCfg,
                      out: np.ndarray) -> bool:
    """backend.zig:189 (cpu.zig:68)."""
    x, lg = _f32(normed), _f32(logits)
    b = None if bias is None else _f32(bias)
    sh = None
    if shexp is not None:
        sh = (_lib.Weight * 3)(*[w.c() for w in shexp])
    c = _lib.RoutedCfg(cfg.n_expert, cfg.n_used, int(cfg.gating_sigmoid), int(cfg.weights_norm), cfg.weights_scale)
    rc = _lib.lib().loom_cuda_moe_ffn_routed(_p(x), x.size, _p(lg), _p(b), gate_w.c(), up_w.c(), down_w.c(),
                                             C.cast(sh, C.c_void_p) if sh is not None else None, ffn, shexp_ffn, c,
                                             _p(out))
    return _lib.check(rc, "moeFfnBlockRouted") == OK


def registerArena(mem: np.ndarray) -> bool:
    """backend.zig:98."""
    m = _u8(mem)
    return _lib.check(_lib.lib().loom_cuda_register_arena(_p(m), m.nbytes), "registerArena") == OK


def materializeArenas() -> int:
    """backend.zig:104."""
    return int(_lib.lib().loom_cuda_materialize_arenas())


def arenaError() -> Optional[str]:
    e = _lib.lib().loom_cuda_arena_error()
    return None if e is None else e.decode()


def takeCmdBufCount() -> int:
    """backend.zig:112."""
    return int(_lib.lib().loom_cuda_take_cmdbuf_count())


def kernelLaunches() -> int:
    return int(_lib.lib().loom_cuda_kernel_launches())


def clearWeightCache() -> None:
    _lib.lib().loom_cuda_clear_weight_cache()
