"""The tensor-core batch path in both arithmetics, against the CPU oracle and
against the int8 batch kernels (the reference's integer arithmetic):
- "exact" (loom_cuda_tc_exact(1)): tcgen05 kind::f16 MMAs carrying the
  reference's integer sub-block products (sc*q weights and int8 activations,
  exact in fp16 and in the f32 accumulator): bit-identical outputs;
- "fp16" (the default): gate/up integer-exact as above, down on dequantized
  fp16 weight tiles against the int8 activations dequantized to fp16, f32
  accumulation over the row: every token within the seam's 2e-3 relative L2.
Expert ids are the router's in both."""
from tests.conftest import bits
import numpy as np
import pytest
import torch

from loom_b200 import _lib
from loom_b200 import device as D
from tests.conftest import rel_l2
from tests.test_gpu_moe import _layer_case, _route_gaps_ok, synth_layer

pytestmark = pytest.mark.gpu
TOL = 2e-3


def _run(L, x, mode, k, path=None, exact=None):
    prev = D.force_generic(mode)
    prev_x = D.tc_exact(exact) if exact is not None else None
    try:
        out = torch.full(x.shape, float("nan"), device="cuda")
        ids = torch.zeros((x.shape[0], k), dtype=torch.int32, device="cuda")
        L.forward(x, out, ids=ids)
        torch.cuda.synchronize()
    finally:
        D.force_generic(prev)
        if prev_x is not None:
            D.tc_exact(prev_x)
    assert _lib.lib().loom_cuda_device_error() == 0
    if path is not None:
        assert D.last_path() == path
    return out.cpu().numpy(), ids.cpu().numpy()


ARITH = pytest.mark.parametrize("arith", ["exact", "fp16"])


def _agree(a, b, arith):
    """exact: bit for bit; fp16: every token within TOL relative L2."""
    if arith == "exact":
        assert np.array_equal(bits(a), bits(b)), rel_l2(a, b)
    else:
        worst = max(rel_l2(a[t], b[t]) for t in range(a.shape[0]))
        assert worst < TOL, worst


@ARITH
@pytest.mark.parametrize("T", [64, 256])
def test_mma_layer_vs_oracle(be, orc, T, arith):
    """Qwen3-30B-A3B layer (config 2) forced onto the tensor cores, against
    the oracle's moeLayer token by token."""
    ne, k, dim, ffn = 128, 8, 2048, 768
    g, u, d = synth_layer(orc, 11, ne, dim, ffn)
    rw = orc.synth(0, ne * dim, seed=111, sigma=0.02)
    x = orc.synth(0, T * dim, seed=112, sigma=1.0).reshape(T, dim)
    L = D.MoeLayer(dim, ffn, ne, k, D.DeviceTensor.upload(12, g), D.DeviceTensor.upload(12, u),
                   D.DeviceTensor.upload(14, d), router=D.DeviceTensor.upload(0, rw))
    got, gids = _run(L, torch.from_numpy(x).cuda(), 3, k, path=3, exact=arith == "exact")
    orc.parallel_begin(16)
    try:
        want, wids = orc.moe_layer(x, rw, (12, g), (12, u), (14, d), ffn, ne, k)
        logits = orc.matmul(0, rw.view(np.uint8), x, ne, dim)
    finally:
        orc.parallel_end()
    compared = 0
    for t in range(T):
        if _route_gaps_ok(logits[t], k):
            assert list(gids[t]) == list(wids[t]), t
            assert rel_l2(got[t], want[t]) < TOL, (t, rel_l2(got[t], want[t]))
            compared += 1
    assert compared >= T * 3 // 4
    for t in (L.gate, L.up, L.down, L.router):
        t.free()


@ARITH
def test_mma_auto_prefill_matches_int8_batch(be, orc, arith):
    """T = 512 (32 tokens per expert): the automatic choice is the tensor-core
    path; it agrees with the int8 expert-major kernels (bit for bit when
    exact, within tolerance in fp16)."""
    ne, k, dim, ffn, T = 128, 8, 2048, 768, 512
    L = _layer_case(orc, 21, ne=ne, k=k, dim=dim, ffn=ffn, gt=12, dt=14)
    x = torch.from_numpy(orc.synth(0, T * dim, seed=212, sigma=1.0).reshape(T, dim)).cuda()
    auto, ids_a = _run(L, x, 0, k, path=3, exact=arith == "exact")
    ref, ids_r = _run(L, x, 2, k, path=2)
    assert np.array_equal(ids_a, ids_r)
    _agree(auto, ref, arith)
    k0 = _lib.lib().loom_cuda_kernel_launches()
    _run(L, x, 0, k)
    assert _lib.lib().loom_cuda_kernel_launches() > k0


@ARITH
def test_mma_shared_expert_and_ragged_groups(be, orc, arith):
    """A layer with a shared expert (DeepSeek-style, sigmoid + bias routing),
    dim 1024 / ffn 512, 40 experts so groups are ragged: tensor cores vs the
    int8 batch kernels."""
    cfg = dict(ne=40, k=4, dim=1024, ffn=512, gt=12, dt=14, shared=512, gating=2, scale=2.5, bias=True)
    L = _layer_case(orc, 31, **cfg)
    T = 200
    x = torch.from_numpy(orc.synth(0, T * cfg["dim"], seed=312, sigma=1.0).reshape(T, cfg["dim"])).cuda()
    mma, ids_m = _run(L, x, 3, cfg["k"], path=3, exact=arith == "exact")
    ref, ids_r = _run(L, x, 2, cfg["k"], path=2)
    assert np.array_equal(ids_m, ids_r)
    _agree(mma, ref, arith)


@ARITH
@pytest.mark.parametrize("T", [1, 8, 40, 1100])
def test_mma_token_counts(be, orc, T, arith):
    """Few tokens per expert (MMA N = 16 with padding), and more than one
    64-token chunk per expert (T = 1100 over 40 experts, ~110 each): the
    tensor-core path equals the int8 batch kernels bit for bit."""
    cfg = dict(ne=40, k=4, dim=1024, ffn=512, gt=12, dt=14)
    L = _layer_case(orc, 41, **cfg)
    x = torch.from_numpy(orc.synth(0, T * cfg["dim"], seed=412, sigma=1.0).reshape(T, cfg["dim"])).cuda()
    mma, ids_m = _run(L, x, 3, cfg["k"], path=3, exact=arith == "exact")
    ref, ids_r = _run(L, x, 2, cfg["k"], path=2)
    assert np.array_equal(ids_m, ids_r)
    _agree(mma, ref, arith)


def _full_range_scales(d, seed, extreme):
    """Q6_K blocks with int8 sub-block scales over the whole range real GGUF
    files use (llama.cpp maps each super-block's largest sub-block to -128 or
    127); `extreme`: every scale -128 and every quant 0, the largest folded
    values (sc * (q - 32) = 4096) the format allows."""
    d = d.copy().reshape(-1, 210)
    rng = np.random.default_rng(seed)
    if extreme:
        d[:, :192] = 0
        d[:, 192:208] = np.uint8(0x80)
    else:
        d[:, 192:208] = rng.integers(0, 256, (d.shape[0], 16), dtype=np.uint8)
        d[:, 192] = np.where(rng.random(d.shape[0]) < 0.5, 0x80, 0x7F)  # -128 / 127 in every block
    return d.reshape(-1)


@ARITH
@pytest.mark.parametrize("extreme", [False, True], ids=["random", "extreme"])
@pytest.mark.parametrize("shared", [False, True], ids=["routed", "shared"])
def test_mma_full_range_q6k_scales(be, orc, extreme, shared, arith):
    """Q6_K down weights with scales beyond +-32 run on the tensor cores (the
    split fold: two fp16 tiles, 8 I_hi + I_lo) and equal the int8 kernels,
    which are the reference's integer arithmetic, bit for bit."""
    ne, k, dim, ffn, T = 16, 4, 1024, 512, 160
    g, u, d = synth_layer(orc, 51, ne, dim, ffn, 12, 12, 14)
    d = _full_range_scales(d, 54, extreme)
    rw = orc.synth(0, ne * dim, seed=52, sigma=0.02)
    kw = {}
    if shared:
        sg, su, sd = synth_layer(orc, 55, 1, dim, ffn, 12, 12, 14)
        kw = dict(shexp=(D.DeviceTensor.upload(12, sg), D.DeviceTensor.upload(12, su),
                         D.DeviceTensor.upload(14, _full_range_scales(sd, 56, extreme))), shexp_ffn=ffn)
    L = D.MoeLayer(dim, ffn, ne, k, D.DeviceTensor.upload(12, g), D.DeviceTensor.upload(12, u),
                   D.DeviceTensor.upload(14, d), router=D.DeviceTensor.upload(0, rw), **kw)
    x = torch.from_numpy(orc.synth(0, T * dim, seed=53, sigma=1.0).reshape(T, dim)).cuda()
    a, ia = _run(L, x, 3, k, path=3, exact=arith == "exact")
    b, ib = _run(L, x, 2, k, path=2)
    assert np.array_equal(ia, ib)
    _agree(a, b, arith)
    assert np.isfinite(a).all()


@ARITH
def test_mma_full_range_q6k_vs_oracle(be, orc, arith):
    """The split fold against the CPU oracle's moeLayer directly."""
    ne, k, dim, ffn, T = 16, 4, 1024, 512, 64
    g, u, d = synth_layer(orc, 61, ne, dim, ffn, 12, 12, 14)
    d = _full_range_scales(d, 62, False)
    rw = orc.synth(0, ne * dim, seed=63, sigma=0.02)
    x = orc.synth(0, T * dim, seed=64, sigma=1.0).reshape(T, dim)
    L = D.MoeLayer(dim, ffn, ne, k, D.DeviceTensor.upload(12, g), D.DeviceTensor.upload(12, u),
                   D.DeviceTensor.upload(14, d), router=D.DeviceTensor.upload(0, rw))
    got, gids = _run(L, torch.from_numpy(x).cuda(), 3, k, path=3, exact=arith == "exact")
    want, wids = orc.moe_layer(x, rw, (12, g), (12, u), (14, d), ffn, ne, k)
    logits = orc.matmul(0, rw.view(np.uint8), x, ne, dim)
    compared = 0
    for t in range(T):
        if _route_gaps_ok(logits[t], k):
            assert list(gids[t]) == list(wids[t]), t
            assert rel_l2(got[t], want[t]) < TOL, (t, rel_l2(got[t], want[t]))
            compared += 1
    assert compared >= T * 3 // 4


@pytest.mark.parametrize("cfg", [
    dict(ne=40, k=4, dim=1024, ffn=512, gt=12, dt=14),
    dict(ne=40, k=4, dim=1024, ffn=512, gt=12, dt=14, shared=512, gating=2, scale=2.5, bias=True),
    dict(ne=128, k=8, dim=2048, ffn=768, gt=12, dt=14),
], ids=["small", "shared", "qwen3"])
@pytest.mark.parametrize("T", [1, 3, 16, 64, 200])
def test_dp4a_tiles_match_int8_batch(be, orc, cfg, T):
    """The tiled dp4a kernels (16-token tiles, one thread per weight row)
    equal the per-expert int8 kernels bit for bit, including experts with more
    than one tile of tokens and a shared expert."""
    L = _layer_case(orc, 61, **cfg)
    x = torch.from_numpy(orc.synth(0, T * cfg["dim"], seed=612, sigma=1.0).reshape(T, cfg["dim"])).cuda()
    a, ia = _run(L, x, 4, cfg["k"], path=4)
    b, ib = _run(L, x, 2, cfg["k"], path=2)
    assert np.array_equal(ia, ib)
    assert np.array_equal(bits(a), bits(b)), rel_l2(a, b)
