"""Device-resident API of the CUDA backend (include/loom_cuda.h, second half):
tensors that live on the GPU in the backend's layout and whole MoE layers run
on device buffers. Device buffers are torch CUDA tensors (plumbing only: the
kernels are the backend's own)."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional

import numpy as np

from . import _lib

BLOCK_ELEMS = {0: 1, 2: 32, 8: 32, 12: 256, 14: 256}
BLOCK_BYTES = {0: 4, 2: 18, 3: 20, 6: 22, 7: 24, 8: 34, 10: 84, 11: 110, 12: 144, 13: 176, 14: 210}


def _ptr(t) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _st(stream) -> int:
    """The stream a call runs on: the caller's, else torch's current stream, so
    the backend's kernels are ordered after the copies and fills that torch
    queued for their inputs and before torch's reads of their outputs."""
    if stream is not None:
        return stream
    import torch
    return torch.cuda.current_stream().cuda_stream


class DeviceTensor:
    def __init__(self, handle: int, ty: int, nblk: int):
        self.handle, self.ty, self.nblk = handle, ty, nblk

    @classmethod
    def upload(cls, ty: int, data: np.ndarray) -> "DeviceTensor":
        d = np.ascontiguousarray(data).view(np.uint8)
        h = C.c_uint64(0)
        _lib.must(_lib.lib().loom_cuda_tensor_upload(ty, d.ctypes.data_as(C.c_void_p), d.nbytes, C.byref(h)),
                  "tensor_upload")
        return cls(h.value, ty, d.nbytes // BLOCK_BYTES[ty])

    @classmethod
    def synth(cls, ty: int, nblk: int, seed: int, sigma: float = 1.0) -> "DeviceTensor":
        h = C.c_uint64(0)
        _lib.must(_lib.lib().loom_cuda_tensor_synth(ty, nblk, seed, sigma, C.byref(h)), "tensor_synth")
        return cls(h.value, ty, nblk)

    @classmethod
    def synth_range(cls, ty: int, blk0: int, nblk: int, seed: int, sigma: float = 1.0) -> "DeviceTensor":
        """Blocks [blk0, blk0+nblk) of the seeded tensor (an expert-parallel slice)."""
        h = C.c_uint64(0)
        _lib.must(_lib.lib().loom_cuda_tensor_synth_range(ty, blk0, nblk, seed, sigma, C.byref(h)), "tensor_synth_range")
        return cls(h.value, ty, nblk)

    def download(self) -> np.ndarray:
        out = np.empty(self.nblk * BLOCK_BYTES[self.ty], np.uint8)
        _lib.must(_lib.lib().loom_cuda_tensor_download(self.handle, out.ctypes.data_as(C.c_void_p), out.nbytes),
                  "tensor_download")
        return out

    @property
    def device_bytes(self) -> int:
        return int(_lib.lib().loom_cuda_tensor_device_bytes(self.handle))

    def free(self) -> None:
        if self.handle:
            _lib.lib().loom_cuda_tensor_free(self.handle)
            self.handle = 0


@dataclass
class MoeLayer:
    dim: int
    ffn: int
    n_expert: int
    n_used: int
    gate: DeviceTensor
    up: DeviceTensor
    down: DeviceTensor
    router: Optional[DeviceTensor] = None
    router_bias: Optional[DeviceTensor] = None
    gating: int = 1
    weights_norm: bool = True
    weights_scale: float = 1.0
    shexp: Optional[tuple] = None
    shexp_ffn: int = 0
    expert0: int = 0
    n_local: int = 0
    next_router: Optional[DeviceTensor] = None  # L2-prefetch hint: the following layer's router
    n_group: int = 1      # DeepSeek-V3 group-limited routing: expert groups ...
    topk_group: int = 1   # ... and how many of them stay eligible

    def desc(self) -> _lib.MoeDesc:
        h = lambda t: t.handle if t is not None else 0  # noqa: E731
        sh = self.shexp or (None, None, None)
        return _lib.MoeDesc(self.dim, self.ffn, self.n_expert, self.n_used, self.gating, int(self.weights_norm),
                            self.weights_scale, h(self.router), h(self.router_bias), h(self.gate), h(self.up),
                            h(self.down), h(sh[0]), h(sh[1]), h(sh[2]), self.shexp_ffn, self.expert0,
                            self.n_local or self.n_expert, h(self.next_router), self.n_group, self.topk_group)

    def forward_a2a(self, x, out, residual=None, logits=None, ids=None, stream=None, t_cap=0, desc=None) -> None:
        """All-to-all expert parallelism: x/out are THIS rank's tokens [T, dim]
        (T may be 0); collective over the ranks of ep_init. t_cap > 0 (the same
        on every rank, >= T): fixed-capacity exchanges, no host synchronisation."""
        d = desc if desc is not None else self.desc()
        T = x.shape[0]
        if t_cap:
            rc = _lib.lib().loom_cuda_ep_a2a_forward_cap(C.byref(d), _ptr(x), T, t_cap, _ptr(out), _ptr(residual),
                                                         _ptr(logits), _ptr(ids), _st(stream))
            _lib.must(rc, "ep_a2a_forward_cap")
            return
        rc = _lib.lib().loom_cuda_ep_a2a_forward(C.byref(d), _ptr(x), T, _ptr(out), _ptr(residual), _ptr(logits),
                                                 _ptr(ids), _st(stream))
        _lib.must(rc, "ep_a2a_forward")

    def forward(self, x, out, residual=None, logits=None, ids=None, stream=None, desc=None) -> None:
        """x, out: torch cuda float32 [T, dim]; ids: torch cuda int32 [T, n_used]."""
        d = desc if desc is not None else self.desc()
        T = x.shape[0]
        rc = _lib.lib().loom_cuda_moe_forward(C.byref(d), _ptr(x), T, _ptr(out), _ptr(residual), _ptr(logits),
                                              _ptr(ids), _st(stream))
        _lib.must(rc, "moe_forward")


class Stack:
    """A decode step through several MoE layers as one persistent kernel."""

    def __init__(self, layers):
        descs = (_lib.MoeDesc * len(layers))(*[L.desc() for L in layers])
        h = C.c_uint64(0)
        _lib.must(_lib.lib().loom_cuda_stack_prepare(C.cast(descs, C.c_void_p), len(layers), C.byref(h)), "stack_prepare")
        self.handle = h.value
        self.n_layers = len(layers)

    def forward(self, x, out, ids=None, stream=None) -> None:
        _lib.must(_lib.lib().loom_cuda_stack_forward(self.handle, _ptr(x), _ptr(out), _ptr(ids), _st(stream)), "stack_forward")

    def forward_residual(self, x, residual, out, ids=None, stream=None) -> None:
        """out = residual + MoE(x) for a one-layer stack (the last layer adds to residual)."""
        _lib.must(_lib.lib().loom_cuda_stack_forward_residual(self.handle, _ptr(x), _ptr(residual), _ptr(out),
                                                              _ptr(ids), _st(stream)), "stack_forward_residual")

    def error(self) -> int:
        return int(_lib.lib().loom_cuda_stack_error(self.handle))

    def trace_enable(self) -> None:
        _lib.must(_lib.lib().loom_cuda_stack_trace(self.handle, 1, None, 0), "stack_trace")

    def trace_read(self):
        """[n_layers][12 + 26]: 12 globaltimer ns points, then (max, sum) over
        CTAs of 16 sections' cycles (see loom_cuda_stack_trace)."""
        import numpy as np
        out = np.zeros((self.n_layers, 12 + 2 * 16), np.uint64)
        _lib.must(_lib.lib().loom_cuda_stack_trace(self.handle, 0, out.ctypes.data, out.size), "stack_trace")
        return out

    def free(self) -> None:
        if self.handle:
            _lib.lib().loom_cuda_stack_free(self.handle)
            self.handle = 0


def ep_init(rank: int, world: int, dist=None) -> None:
    """Create the backend's NCCL communicator (one process per GPU). The id is
    made on rank 0 and broadcast with torch.distributed (any backend)."""
    ident = np.zeros(128, np.uint8)
    if rank == 0:
        _lib.must(_lib.lib().loom_cuda_ep_unique_id(ident.ctypes.data_as(C.c_void_p), ident.nbytes), "ep_unique_id")
    if world > 1:
        box = [ident.tobytes()]
        dist.broadcast_object_list(box, src=0)
        ident = np.frombuffer(box[0], np.uint8).copy()
    _lib.must(_lib.lib().loom_cuda_ep_init(world, rank, ident.ctypes.data_as(C.c_void_p), ident.nbytes), "ep_init")


def expert_range(n_expert: int, rank: int, world: int):
    """Contiguous expert shard of a rank: (expert0, n_local)."""
    e0 = rank * n_expert // world
    e1 = (rank + 1) * n_expert // world
    return e0, e1 - e0


def argmax(logits, out=None, stream=None):
    """sampler.zig:7-15 argmax of a cuda float32 vector; returns a cuda int32 [1] (the index)."""
    import torch
    out = torch.zeros(1, dtype=torch.int32, device=logits.device) if out is None else out
    _lib.must(_lib.lib().loom_cuda_argmax(_ptr(logits), logits.numel(), _ptr(out), _st(stream)), "argmax")
    return out


def lm_head_argmax(w: DeviceTensor, vocab: int, dim: int, x, logits=None, out=None, stream=None):
    """Output head + greedy sample of one token: (logits W x, their argmax)."""
    import torch
    out = torch.zeros(1, dtype=torch.int32, device=x.device) if out is None else out
    _lib.must(_lib.lib().loom_cuda_lm_head_argmax(w.handle, vocab, dim, _ptr(x), _ptr(logits), _ptr(out), _st(stream)),
              "lm_head_argmax")
    return out


def reserve(T: int, dim: int, ffn: int, n_expert: int, n_used: int) -> None:
    _lib.must(_lib.lib().loom_cuda_reserve(T, dim, ffn, n_expert, n_used), "reserve")


def tensor_matmul(w: DeviceTensor, rows: int, cols: int, xs, out, stream=None) -> None:
    _lib.must(_lib.lib().loom_cuda_tensor_matmul(w.handle, rows, cols, _ptr(xs), xs.shape[0], _ptr(out), _st(stream)),
              "tensor_matmul")


def force_generic(mode) -> int:
    """Kernel family for MoE layers: 0 automatic, 1 (True) slot kernels, 2 expert-major batch kernels
    (int8 dots), 3 expert-major batch kernels on the tensor cores (tcgen05 MMAs; see tc_exact)."""
    return int(_lib.lib().loom_cuda_force_generic(int(mode)))


def tc_exact(on) -> int:
    """Tensor-core expert kernels: 0 (default) dequantized fp16 tiles, within 2e-3 relative L2 of the
    reference; 1 integer-exact tiles, bit-identical to the CPU. Returns the previous setting."""
    return int(_lib.lib().loom_cuda_tc_exact(int(on)))


def last_path() -> int:
    """Kernel family of the last routed layer: 0 decode, 1 slot, 2 int8 batch, 3 tensor cores."""
    return int(_lib.lib().loom_cuda_last_path())


def trace_enable(n_kernels: int) -> None:
    """Record (first start, last end) of the next n_kernels decode kernels."""
    _lib.must(_lib.lib().loom_cuda_trace_enable(n_kernels), "trace_enable")


def trace_reset() -> None:
    _lib.must(_lib.lib().loom_cuda_trace_reset(), "trace_reset")


def trace_read(n_kernels: int) -> np.ndarray:
    """[n, 2] globaltimer ns (start, end) per traced kernel."""
    out = np.zeros((n_kernels, 2), np.uint64)
    n = _lib.lib().loom_cuda_trace_read(out.ctypes.data_as(C.c_void_p), n_kernels)
    return out[:n]


def sync() -> None:
    _lib.must(_lib.lib().loom_cuda_sync(), "sync")
