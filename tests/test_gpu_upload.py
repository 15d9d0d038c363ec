"""Verified upload on the device: SHA-256 computed by the backend over the
bytes its kernels read (loom_cuda_sha256_device, loom_cuda_tensor_sha256,
loom_cuda_verify_shards) against Python's hashlib, the content address the
reference keeps per weight range (src/core/hash.zig:12-23,
src/p2p/weights.zig:862-879); and a GGUF image read by the backend's parser
feeding the routed MoE seam call, checked against the oracle."""
import ctypes as C
import hashlib

import numpy as np
import pytest

from loom_b200 import _lib
from loom_b200 import backend as B
from loom_b200.gguf import GGUF
from tests import ggufwrite as W

pytestmark = pytest.mark.gpu

BLOCK = {0: (1, 4), 2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34), 10: (256, 84),
         11: (256, 110), 12: (256, 144), 13: (256, 176), 14: (256, 210)}


def _dev_digest(ptr, n):
    out = (C.c_uint8 * 32)()
    _lib.must(_lib.lib().loom_cuda_sha256_device(C.c_void_p(ptr), n, out), "sha256_device")
    return bytes(out)


@pytest.mark.parametrize("n", [0, 1, 55, 56, 63, 64, 65, 119, 120, 128, 1000, (1 << 20) + 3])
@pytest.mark.parametrize("shift", [0, 1, 4])
def test_sha256_device_matches_hashlib(be, n, shift):
    import torch
    rng = np.random.default_rng(n + 7 * shift)
    host = rng.integers(0, 256, n + 16, dtype=np.uint8)
    dev = torch.from_numpy(host).cuda()
    torch.cuda.synchronize()
    got = _dev_digest(dev.data_ptr() + shift, n)
    assert got == hashlib.sha256(host[shift:shift + n].tobytes()).digest()


@pytest.mark.parametrize("ty", sorted(BLOCK))
def test_tensor_sha256_over_gguf_bytes(be, orc, ty):
    """The digest is over the GGUF bytes even where the device layout is
    repacked (Q6_K, Q8_0, Q3_K, ...), for the whole tensor and a block range."""
    nblk = 37 if ty else 37 * 64
    host = orc.synth(ty, nblk, 11).view(np.uint8)
    h = C.c_uint64()
    _lib.must(_lib.lib().loom_cuda_tensor_upload(ty, host.ctypes.data_as(C.c_void_p), host.nbytes, C.byref(h)),
              "upload")
    bb = BLOCK[ty][1]
    try:
        for b0, nb in [(0, nblk), (5, 17), (nblk - 1, 1), (3, 0)]:
            out = (C.c_uint8 * 32)()
            _lib.must(_lib.lib().loom_cuda_tensor_sha256(h.value, b0, nb, out), "tensor_sha256")
            assert bytes(out) == hashlib.sha256(host[b0 * bb:(b0 + nb) * bb].tobytes()).digest(), (b0, nb)
        out = (C.c_uint8 * 32)()
        assert _lib.lib().loom_cuda_tensor_sha256(h.value, nblk, 1, out) == _lib.DECLINED
    finally:
        _lib.lib().loom_cuda_tensor_free(h.value)


def _layer(orc, seed, ne, dim, ffn, gt=12, ut=12, dt=14):
    def plane(t, rows, cols):
        return rows * (cols // BLOCK[t][0]) * BLOCK[t][1]
    g = orc.synth(gt, ne * plane(gt, ffn, dim) // BLOCK[gt][1], seed)
    u = orc.synth(ut, ne * plane(ut, ffn, dim) // BLOCK[ut][1], seed + 1)
    d = orc.synth(dt, ne * plane(dt, dim, ffn) // BLOCK[dt][1], seed + 2)
    return (gt, g, plane(gt, ffn, dim)), (ut, u, plane(ut, ffn, dim)), (dt, d, plane(dt, dim, ffn))


def _shards(tensors, ne, digests_from=None):
    """One shard per expert: its gate, up and down planes, in that order."""
    arr = (_lib.Shard * ne)()
    src = digests_from or tensors
    for e in range(ne):
        s = arr[e]
        s.n_ext = 3
        hsh = hashlib.sha256()
        for k, ((t, buf, pb), (_, good, _)) in enumerate(zip(tensors, src)):
            s.ext[k] = _lib.Weight(t, buf.ctypes.data + e * pb, pb)
            hsh.update(good.view(np.uint8)[e * pb:(e + 1) * pb].tobytes())
        C.memmove(s.digest, hsh.digest(), 32)
    return arr


def _verify(arr, ne):
    bad = (C.c_uint8 * ne)()
    nb = C.c_size_t()
    _lib.must(_lib.lib().loom_cuda_verify_shards(arr, ne, bad, C.byref(nb)), "verify_shards")
    return list(bad), nb.value


def test_verify_shards_catches_a_poisoned_expert_and_rechecks_after_repair(be, orc):
    ne, dim, ffn = 8, 512, 256
    good = _layer(orc, 21, ne, dim, ffn)
    B.clearWeightCache()
    # the layer's tensors are cached by a seam call first, as an engine would
    x = np.random.default_rng(1).standard_normal(dim).astype(np.float32)
    logits = np.random.default_rng(2).standard_normal(ne).astype(np.float32)
    out = np.empty(dim, np.float32)
    cfg = B.RoutedCfg(ne, 2, False, True, 1.0)
    wr = [B.WeightRef(t, b) for t, b, _ in good]
    assert B.moeFfnBlockRouted(x, logits, None, *wr, None, ffn, 0, cfg, out)
    assert _verify(_shards(good, ne), ne) == ([0] * ne, 0)

    # a byte of expert 5's down plane flipped in a second copy of the weights
    poisoned = [(t, b.copy(), pb) for t, b, pb in good]
    t, d, pb = poisoned[2]
    d.view(np.uint8)[5 * pb + 77] ^= 0x10
    bad, nb = _verify(_shards(poisoned, ne, digests_from=good), ne)
    assert nb == 1 and bad == [0, 0, 0, 0, 0, 1, 0, 0]
    # repaired in place (a refetch): the evicted device copy is uploaded and hashed again
    d.view(np.uint8)[5 * pb + 77] ^= 0x10
    assert _verify(_shards(poisoned, ne, digests_from=good), ne) == ([0] * ne, 0)
    B.clearWeightCache()


def test_gguf_image_to_routed_moe(be, orc):
    """A MoE layer written as GGUF, read by the backend's parser (checked
    resolve), verified per expert on the device, then run through the routed
    seam entry from the image's own bytes -- parity with the oracle."""
    ne, k, dim, ffn = 16, 4, 512, 256
    (gt, g, pg), (ut, u, pu), (dt, d, pd) = _layer(orc, 31, ne, dim, ffn)
    img = W.image([("general.architecture", W.T_STR, "qwen3moe"), ("qwen3moe.expert_count", W.T_U32, ne),
                   ("qwen3moe.expert_used_count", W.T_U32, k), ("general.alignment", W.T_U32, 64)],
                  [("blk.0.ffn_gate_exps.weight", (dim, ffn, ne), gt, g.view(np.uint8).tobytes()),
                   ("blk.0.ffn_up_exps.weight", (dim, ffn, ne), ut, u.view(np.uint8).tobytes()),
                   ("blk.0.ffn_down_exps.weight", (ffn, dim, ne), dt, d.view(np.uint8).tobytes())], alignment=64)
    gg = GGUF(img)
    assert gg.get_uint("qwen3moe.expert_count") == ne
    vg, vu, vd = (gg.resolve(f"blk.0.ffn_{n}_exps.weight") for n in ("gate", "up", "down"))
    assert (vg.ne0, vg.ne1, vg.ne2) == (dim, ffn, ne) and vd.data.nbytes == d.nbytes
    B.clearWeightCache()
    views = [(vg.ggml_type, vg.data, pg), (vu.ggml_type, vu.data, pu), (vd.ggml_type, vd.data, pd)]
    assert _verify(_shards(views, ne), ne) == ([0] * ne, 0)
    rng = np.random.default_rng(5)
    x = rng.standard_normal(dim).astype(np.float32)
    logits = rng.standard_normal(ne).astype(np.float32)
    out = np.full(dim, np.nan, np.float32)
    cfg = B.RoutedCfg(ne, k, False, True, 1.0)
    assert B.moeFfnBlockRouted(x, logits, None, B.WeightRef(gt, vg.data), B.WeightRef(ut, vu.data),
                               B.WeightRef(dt, vd.data), None, ffn, 0, cfg, out)
    want = orc.moe_ffn_routed(x, logits, (gt, g), (ut, u), (dt, d), ffn, k)
    rel = float(np.linalg.norm(out - want) / np.linalg.norm(want))
    assert rel < 2e-3, rel
    B.clearWeightCache()
