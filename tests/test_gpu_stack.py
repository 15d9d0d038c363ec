"""The persistent decode stack (one cooperative kernel for a whole stack of
MoE layers at T = 1) must reproduce, bit for bit, running the same layers one
by one through loom_cuda_moe_forward with the residual add: same expert ids,
same output bits, on every layer."""
import numpy as np
import pytest
import torch

from loom_b200 import _lib
from loom_b200.device import DeviceTensor, MoeLayer, Stack
from tests.conftest import bits
from tests.test_gpu_moe import synth_layer

pytestmark = pytest.mark.gpu


def _qwen_layers(orc, n, ne=128, k=8, dim=2048, ffn=768):
    layers = []
    for i in range(n):
        g, u, d = synth_layer(orc, 100 + i, ne, dim, ffn)
        rw = orc.synth(0, ne * dim, seed=300 + i, sigma=0.02)
        layers.append(MoeLayer(dim, ffn, ne, k, DeviceTensor.upload(12, g), DeviceTensor.upload(12, u),
                               DeviceTensor.upload(14, d), router=DeviceTensor.upload(0, rw)))
    return layers


@pytest.mark.parametrize("n_layers", [1, 2, 5])
def test_stack_bitexact_with_layer_loop(be, orc, n_layers):
    layers = _qwen_layers(orc, n_layers)
    dim, k = layers[0].dim, layers[0].n_used
    x0 = torch.from_numpy(orc.synth(0, dim, seed=501, sigma=1.0).reshape(1, dim)).cuda()
    # layer loop: x_{l+1} = x_l + MoE_l(x_l)
    want_ids = []
    x = x0.clone()
    for L in layers:
        out = torch.empty_like(x)
        ids = torch.zeros((1, k), dtype=torch.int32, device="cuda")
        L.forward(x, out, residual=x, ids=ids)
        want_ids.append(ids)
        x = out
    torch.cuda.synchronize()
    want = x.cpu().numpy()
    S = Stack(layers)
    try:
        for rep in range(2):  # a second launch reuses the barrier words
            out = torch.full((1, dim), float("nan"), device="cuda")
            ids = torch.zeros((n_layers, k), dtype=torch.int32, device="cuda")
            S.forward(x0, out, ids)
            torch.cuda.synchronize()
            assert S.error() == 0
            assert np.array_equal(ids.cpu().numpy(), torch.cat(want_ids).cpu().numpy()), rep
            assert np.array_equal(bits(out.cpu().numpy()), bits(want)), rep
    finally:
        S.free()
    assert _lib.lib().loom_cuda_device_error() == 0
    for L in layers:
        for t in (L.gate, L.up, L.down, L.router):
            t.free()


def test_stack_declines_shared_expert(be, orc):
    from tests.test_gpu_moe import _layer_case
    L = _layer_case(orc, 5, ne=64, k=6, dim=2048, ffn=1408, gt=12, dt=8, shared=2816)
    with pytest.raises(RuntimeError):
        Stack([L])


def test_one_layer_stack_with_residual_bitexact(be, orc):
    """loom_cuda_stack_forward_residual: out = residual + MoE(x), a decoder
    layer's FFN on its normed input, bit for bit the per-layer path's."""
    layers = _qwen_layers(orc, 1)
    L, dim = layers[0], layers[0].dim
    x = torch.from_numpy(orc.synth(0, dim, seed=611, sigma=1.0).reshape(1, dim)).cuda()
    res = torch.from_numpy(orc.synth(0, dim, seed=612, sigma=1.0).reshape(1, dim)).cuda()
    want = torch.empty_like(x)
    L.forward(x, want, residual=res)
    st = Stack(layers)
    try:
        for _ in range(2):
            got = torch.full_like(x, float("nan"))
            st.forward_residual(x, res, got)
            torch.cuda.synchronize()
            assert np.array_equal(bits(got.cpu().numpy()), bits(want.cpu().numpy()))
        assert st.error() == 0
    finally:
        st.free()
        for t in (L.gate, L.up, L.down, L.router):
            t.free()


def test_stack_matches_oracle_layer_by_layer(be, orc):
    """The persistent stack against the oracle directly: three Qwen3-shaped
    layers, x_{l+1} = x_l + moeLayer_l(x_l) with the
    oracle's moeLayer (moe.zig / ggml.zig restated in C); every layer's ids
    equal where the router's top-k margins are clear, the output within the
    path's tolerance."""
    from tests.conftest import rel_l2
    from tests.test_gpu_moe import _route_gaps_ok
    n_layers, ne, k, dim, ffn = 3, 128, 8, 2048, 768
    hosts = []
    for i in range(n_layers):
        g, u, d = synth_layer(orc, 100 + i, ne, dim, ffn)
        rw = orc.synth(0, ne * dim, seed=300 + i, sigma=0.02)
        hosts.append((g, u, d, rw))
    layers = [MoeLayer(dim, ffn, ne, k, DeviceTensor.upload(12, g), DeviceTensor.upload(12, u),
                       DeviceTensor.upload(14, d), router=DeviceTensor.upload(0, rw)) for g, u, d, rw in hosts]
    x0 = orc.synth(0, dim, seed=777, sigma=1.0).reshape(1, dim)
    S = Stack(layers)
    try:
        out = torch.full((1, dim), float("nan"), device="cuda")
        ids = torch.zeros((n_layers, k), dtype=torch.int32, device="cuda")
        S.forward(torch.from_numpy(x0).cuda(), out, ids)
        torch.cuda.synchronize()
        assert S.error() == 0
        got_ids = ids.cpu().numpy()
        x = x0.astype(np.float32)
        for li, (g, u, d, rw) in enumerate(hosts):
            y, wids = orc.moe_layer(x, rw, (12, g), (12, u), (14, d), ffn, ne, k)
            logits = orc.matmul(0, rw.view(np.uint8), x, ne, dim)
            if _route_gaps_ok(logits[0], k):
                assert list(got_ids[li]) == list(wids[0]), li
            x = (x + y).astype(np.float32)
        assert rel_l2(out.cpu().numpy(), x) < 2e-3, rel_l2(out.cpu().numpy(), x)
    finally:
        S.free()
    for L in layers:
        for t in (L.gate, L.up, L.down, L.router):
            t.free()
