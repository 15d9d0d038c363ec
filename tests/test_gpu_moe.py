"""GPU parity of the fused MoE entry points against the CPU oracle at the
benchmark shapes: moeFfnBlock, moeFfnBlockRouted (Qwen3-30B-A3B layer,
DeepSeek-V2-Lite layer with shared experts, sigmoid+bias routing), and the
device-resident layer with its own router at T=1 and T=64.

Tolerances (north star): top-k ids identical wherever the logit gap exceeds
1e-4; FFN outputs within 2e-3 relative L2."""
import numpy as np
import pytest
import torch

from loom_b200 import backend as B
from loom_b200.device import DeviceTensor, MoeLayer
from tests.conftest import bits, rel_l2

pytestmark = pytest.mark.gpu
TOL = 2e-3


def synth_layer(orc, seed, ne, dim, ffn, gt=12, ut=12, dt=14):
    rb = lambda t, n: orc.row_bytes(t, n)  # noqa: E731
    bg, bu = ffn * dim // orc.BLOCK_ELEMS[gt], ffn * dim // orc.BLOCK_ELEMS[ut]
    bd = dim * ffn // orc.BLOCK_ELEMS[dt]
    g = orc.synth(gt, ne * bg, seed * 10 + 1)
    u = orc.synth(ut, ne * bu, seed * 10 + 2)
    d = orc.synth(dt, ne * bd, seed * 10 + 3)
    assert g.size == ne * ffn * rb(gt, dim)
    return g, u, d


def test_moe_ffn_block_mixed_types(be, orc):
    rng = np.random.default_rng(3)
    dim, ffn = 1024, 512
    from tests import npref
    ex, oex = [], []
    for k, (gt, ut, dt, w) in enumerate([(12, 8, 2, 0.5), (14, 12, 12, 0.3), (2, 2, 8, 0.2), (12, 12, 14, 1.0)]):
        g = npref.random_blocks(rng, gt, ffn, dim)
        u = npref.random_blocks(rng, ut, ffn, dim)
        d = npref.random_blocks(rng, dt, dim, ffn)
        ex.append(B.ExpertRef(B.WeightRef(gt, g), B.WeightRef(ut, u), B.WeightRef(dt, d), w, ffn))
        oex.append(dict(gate_type=gt, up_type=ut, down_type=dt, gate=g, up=u, down=d, weight=w, ffn=ffn))
    x = rng.standard_normal(dim).astype(np.float32)
    out = np.full(dim, np.nan, np.float32)
    B.takeCmdBufCount()
    assert B.moeFfnBlock(x, ex, out)
    assert B.takeCmdBufCount() == 1
    want = orc.moe_ffn_block(x, oex, dim)
    assert rel_l2(out, want) < TOL
    assert np.mean(bits(out) == bits(want)) > 0.9  # identical except where an ulp of expf moved an int8


def test_moe_ffn_routed_qwen3_layer(be, orc):
    """BASELINE config 2 (Qwen3-30B-A3B MoE layer): 128 experts, top-8 softmax+renorm,
    gate/up Q4_K [768x2048], down Q6_K [2048x768]."""
    ne, k, dim, ffn = 128, 8, 2048, 768
    g, u, d = synth_layer(orc, 1, ne, dim, ffn)
    rng = np.random.default_rng(9)
    cfg = B.RoutedCfg(ne, k, False, True, 1.0)
    for trial in range(4):
        x = rng.standard_normal(dim).astype(np.float32)
        logits = (rng.standard_normal(ne) * 0.5).astype(np.float32)
        out = np.full(dim, np.nan, np.float32)
        assert B.moeFfnBlockRouted(x, logits, None, B.WeightRef(12, g), B.WeightRef(12, u), B.WeightRef(14, d), None,
                                   ffn, 0, cfg, out)
        want = orc.moe_ffn_routed(x, logits, (12, g), (12, u), (14, d), ffn, k)
        assert rel_l2(out, want) < TOL, rel_l2(out, want)


@pytest.mark.parametrize("sigmoid", [False, True])
def test_moe_ffn_routed_deepseek_shared(be, orc, sigmoid):
    """DeepSeek-V2-Lite-shaped layer: 64 experts top-6, moe_ffn 1408 (down Q8_0:
    1408 is not a multiple of 256), 2 shared experts (2816), optional sigmoid
    gating with selection bias and scale."""
    ne, k, dim, ffn, sffn = 64, 6, 2048, 1408, 2816
    g, u, d = synth_layer(orc, 2, ne, dim, ffn, 12, 12, 8)
    sg, su, sd = synth_layer(orc, 3, 1, dim, sffn, 12, 12, 8)
    rng = np.random.default_rng(4)
    x = rng.standard_normal(dim).astype(np.float32)
    logits = rng.standard_normal(ne).astype(np.float32)
    bias = (rng.standard_normal(ne) * 0.05).astype(np.float32) if sigmoid else None
    scale = 2.5 if sigmoid else 1.0
    cfg = B.RoutedCfg(ne, k, sigmoid, True, scale)
    out = np.full(dim, np.nan, np.float32)
    sh = [B.WeightRef(12, sg), B.WeightRef(12, su), B.WeightRef(8, sd)]
    assert B.moeFfnBlockRouted(x, logits, bias, B.WeightRef(12, g), B.WeightRef(12, u), B.WeightRef(8, d), sh, ffn,
                               sffn, cfg, out)
    want = orc.moe_ffn_routed(x, logits, (12, g), (12, u), (8, d), ffn, k, gating_sigmoid=sigmoid,
                              weights_scale=scale, bias=bias, shexp=[(12, sg), (12, su), (8, sd)], shexp_ffn=sffn)
    assert rel_l2(out, want) < TOL


@pytest.mark.parametrize("t", [0, 2, 3, 6, 7, 8, 10, 11, 12, 13, 14])
def test_device_synth_matches_oracle(be, orc, t):
    nblk = 1000
    dt = DeviceTensor.synth(t, nblk, seed=77, sigma=0.02)
    try:
        got = dt.download()
        want = orc.synth(t, nblk, seed=77, sigma=0.02).view(np.uint8)
        assert np.array_equal(got, want)
    finally:
        dt.free()


def test_arena_materialize_and_lookup(be, orc):
    rng = np.random.default_rng(8)
    from tests import npref
    rows, cols = 96, 2048
    arena = np.zeros(4096 + rows * orc.row_bytes(14, cols) + 1000, np.uint8)
    w = npref.random_blocks(rng, 14, rows, cols)
    arena[4096:4096 + w.size] = w
    assert B.registerArena(arena)
    assert B.materializeArenas() == arena.nbytes
    assert B.arenaError() is None
    x = rng.standard_normal(cols).astype(np.float32)
    out = np.empty(rows, np.float32)
    B.matvec(14, out, arena[4096:4096 + w.size], x, rows, cols)
    assert np.array_equal(bits(out), bits(orc.matvec(14, w, x, rows, cols)))


def _route_gaps_ok(logits_row, k):
    s = np.sort(logits_row.astype(np.float64))[::-1]
    return bool(np.all(s[:k] - s[1:k + 1] > 1e-4))


@pytest.mark.parametrize("T", [1, 4, 64])
def test_device_layer_with_router(be, orc, T):
    """The whole layer on the device (router GEMV -> route -> experts ->
    combine) against the oracle's moeLayer at BASELINE config 2, T in {1, 64}."""
    ne, k, dim, ffn = 128, 8, 2048, 768
    g, u, d = synth_layer(orc, 4, ne, dim, ffn)
    rw = orc.synth(0, ne * dim, seed=41, sigma=0.02)
    x = orc.synth(0, T * dim, seed=42, sigma=1.0).reshape(T, dim)
    L = MoeLayer(dim, ffn, ne, k, DeviceTensor.upload(12, g), DeviceTensor.upload(12, u), DeviceTensor.upload(14, d),
                 router=DeviceTensor.upload(0, rw))
    xt = torch.from_numpy(x).cuda()
    out = torch.full((T, dim), float("nan"), device="cuda")
    ids = torch.zeros((T, k), dtype=torch.int32, device="cuda")
    L.forward(xt, out, ids=ids)
    torch.cuda.synchronize()
    orc.parallel_begin(8)
    try:
        want, wids = orc.moe_layer(x, rw, (12, g), (12, u), (14, d), ffn, ne, k)
        logits = orc.matmul(0, rw.view(np.uint8), x, ne, dim)
    finally:
        orc.parallel_end()
    got, gids = out.cpu().numpy(), ids.cpu().numpy()
    compared = 0
    for t in range(T):
        if _route_gaps_ok(logits[t], k):
            assert list(gids[t]) == list(wids[t]), t
            assert rel_l2(got[t], want[t]) < TOL, (t, rel_l2(got[t], want[t]))
            compared += 1
    assert compared >= max(1, T * 3 // 4)
    for t in (L.gate, L.up, L.down, L.router):
        t.free()


def _layer_case(orc, seed, ne, k, dim, ffn, gt, dt, shared=0, gating=1, scale=1.0, bias=False, groups=(1, 1)):
    g, u, d = synth_layer(orc, seed, ne, dim, ffn, gt, gt, dt)
    rw = orc.synth(0, ne * dim, seed=seed * 7 + 1, sigma=0.02)
    L = MoeLayer(dim, ffn, ne, k, DeviceTensor.upload(gt, g), DeviceTensor.upload(gt, u), DeviceTensor.upload(dt, d),
                 router=DeviceTensor.upload(0, rw), gating=gating, weights_scale=scale, n_group=groups[0],
                 topk_group=groups[1])
    if bias:
        L.router_bias = DeviceTensor.upload(0, (np.random.default_rng(seed).standard_normal(ne) * 0.05).astype(np.float32))
    if shared:
        sg, su, sd = synth_layer(orc, seed + 50, 1, dim, shared, gt, gt, dt)
        L.shexp = (DeviceTensor.upload(gt, sg), DeviceTensor.upload(gt, su), DeviceTensor.upload(dt, sd))
        L.shexp_ffn = shared
    return L


@pytest.mark.parametrize("cfg", [
    dict(ne=128, k=8, dim=2048, ffn=768, gt=12, dt=14),                     # Qwen3-30B-A3B
    dict(ne=64, k=6, dim=2048, ffn=1408, gt=12, dt=8, shared=2816),          # DeepSeek-V2-Lite
    dict(ne=256, k=8, dim=1024, ffn=1024, gt=12, dt=12, shared=1024, gating=2, scale=2.5, bias=True),  # V3-like
    dict(ne=16, k=4, dim=512, ffn=256, gt=14, dt=14),                        # Q6_K gate/up
    dict(ne=256, k=8, dim=1024, ffn=512, gt=12, dt=12, shared=512, gating=2, scale=2.5, bias=True,
         groups=(8, 4)),                                                     # V3 group-limited routing
], ids=["qwen3", "v2lite", "v3like", "q6k", "v3grouped"])
@pytest.mark.parametrize("T", [1, 3, 40])
def test_decode_kernels_bitexact_with_slot_kernels(be, orc, cfg, T):
    """The fused decode kernels, the expert-major batch kernels and the general
    slot kernels implement the same arithmetic: their outputs must agree bit for
    bit."""
    from loom_b200 import device as D
    L = _layer_case(orc, 5, **cfg)
    x = torch.from_numpy(orc.synth(0, T * cfg["dim"], seed=9).reshape(T, cfg["dim"])).cuda()
    res = torch.randn(T, cfg["dim"], device="cuda")
    outs, idss = [], []
    for generic in (0, 2, 1):
        prev = D.force_generic(generic)
        try:
            out = torch.full((T, cfg["dim"]), float("nan"), device="cuda")
            ids = torch.zeros((T, cfg["k"]), dtype=torch.int32, device="cuda")
            L.forward(x, out, residual=res, ids=ids)
            torch.cuda.synchronize()
            outs.append(out.cpu().numpy())
            idss.append(ids.cpu().numpy())
        finally:
            D.force_generic(prev)
    from loom_b200 import _lib
    assert _lib.lib().loom_cuda_device_error() == 0  # no bounded wait gave up
    for i in (1, 2):
        assert np.array_equal(idss[0], idss[i])
        assert np.array_equal(bits(outs[0]), bits(outs[i])), i


def test_expert_parallel_partition_sums_to_full(be, orc):
    """Expert-parallel shards: each rank runs only its expert range; the sum of
    the partial outputs equals the unsharded layer (to rounding: the combine
    order changes)."""
    ne, k, dim, ffn = 64, 6, 1024, 512
    g, u, d = synth_layer(orc, 6, ne, dim, ffn)
    rw = orc.synth(0, ne * dim, seed=61, sigma=0.02)
    x = torch.from_numpy(orc.synth(0, 2 * dim, seed=62).reshape(2, dim)).cuda()
    pg, pd = ffn * orc.row_bytes(12, dim), dim * orc.row_bytes(14, ffn)
    full = MoeLayer(dim, ffn, ne, k, DeviceTensor.upload(12, g), DeviceTensor.upload(12, u),
                    DeviceTensor.upload(14, d), router=DeviceTensor.upload(0, rw))
    want = torch.empty((2, dim), device="cuda")
    full.forward(x, want)
    parts = []
    R = 4
    for rank in range(R):
        e0, n = rank * ne // R, ne // R
        L = MoeLayer(dim, ffn, ne, k, DeviceTensor.upload(12, g[e0 * pg:(e0 + n) * pg]),
                     DeviceTensor.upload(12, u[e0 * pg:(e0 + n) * pg]), DeviceTensor.upload(14, d[e0 * pd:(e0 + n) * pd]),
                     router=full.router, expert0=e0, n_local=n)
        o = torch.empty((2, dim), device="cuda")
        L.forward(x, o)
        parts.append(o)
    got = sum(parts)
    torch.cuda.synchronize()
    assert rel_l2(got.cpu().numpy(), want.cpu().numpy()) < 1e-5


@pytest.mark.parametrize("T", [1, 5, 40])
def test_grouped_routing_layer_vs_oracle(be, orc, T):
    """DeepSeek-V3 group-limited routing (256 experts in 8 groups, the best 4
    groups by the sum of their two best biased sigmoid scores stay eligible,
    top-8, renormalised, scaled) through the device layer: ids equal to the
    oracle's grouped route on the oracle's logits wherever the selection is
    decided by more than 1e-4 (no near-tie between the k-th and (k+1)-th
    eligible choice or between the kept and dropped groups), outputs within
    the FFN tolerance of the oracle's moeFfnBlock over those experts."""
    ne, k, dim, ffn, ng, tg, scale = 256, 8, 1024, 512, 8, 4, 2.5
    g, u, d = synth_layer(orc, 11, ne, dim, ffn)
    rw = orc.synth(0, ne * dim, seed=111, sigma=0.05)
    bias = (np.random.default_rng(12).standard_normal(ne) * 0.05).astype(np.float32)
    x = orc.synth(0, T * dim, seed=112, sigma=1.0).reshape(T, dim)
    L = MoeLayer(dim, ffn, ne, k, DeviceTensor.upload(12, g), DeviceTensor.upload(12, u), DeviceTensor.upload(14, d),
                 router=DeviceTensor.upload(0, rw), router_bias=DeviceTensor.upload(0, bias), gating=2,
                 weights_scale=scale, n_group=ng, topk_group=tg)
    xt = torch.from_numpy(x).cuda()
    out = torch.full((T, dim), float("nan"), device="cuda")
    ids = torch.zeros((T, k), dtype=torch.int32, device="cuda")
    L.forward(xt, out, ids=ids)
    torch.cuda.synchronize()
    got, gids = out.cpu().numpy(), ids.cpu().numpy()
    orc.parallel_begin(8)
    try:
        logits = orc.matmul(0, rw.view(np.uint8), x, ne, dim)
        gp, dp = ffn * orc.row_bytes(12, dim), dim * orc.row_bytes(14, ffn)
        compared = 0
        for t in range(T):
            c = 1.0 / (1.0 + np.exp(-logits[t].astype(np.float64))) + bias
            grp = np.sort(c.reshape(ng, -1), axis=1)[:, ::-1]
            gsc = np.sort(grp[:, 0] + grp[:, 1])[::-1]
            kept = np.sort(c.reshape(ng, -1)[np.argsort(-(grp[:, 0] + grp[:, 1]))[:tg]].ravel())[::-1]
            if gsc[tg - 1] - gsc[tg] <= 1e-4 or kept[k - 1] - kept[k] <= 1e-4:
                continue
            wids, wg = orc.route(logits[t], k, 2, True, scale, bias, n_group=ng, topk_group=tg)
            assert list(gids[t]) == list(wids), t
            assert len(set(int(i) // (ne // ng) for i in wids)) <= tg
            ex = [dict(gate_type=12, up_type=12, down_type=14, gate=g[i * gp:(i + 1) * gp],
                       up=u[i * gp:(i + 1) * gp], down=d[i * dp:(i + 1) * dp], weight=float(w), ffn=ffn)
                  for i, w in zip(wids, wg)]
            want = orc.moe_ffn_block(x[t], ex, dim)
            assert rel_l2(got[t], want) < TOL, (t, rel_l2(got[t], want))
            compared += 1
    finally:
        orc.parallel_end()
    assert compared >= max(1, T * 3 // 4)
    for t_ in (L.gate, L.up, L.down, L.router, L.router_bias):
        t_.free()


def test_grouped_routing_declines_bad_groups(be, orc):
    ne, k, dim, ffn = 64, 6, 512, 256
    g, u, d = synth_layer(orc, 13, ne, dim, ffn)
    L = MoeLayer(dim, ffn, ne, k, DeviceTensor.upload(12, g), DeviceTensor.upload(12, u), DeviceTensor.upload(14, d),
                 router=DeviceTensor.upload(0, orc.synth(0, ne * dim, seed=5, sigma=0.02)), n_group=3, topk_group=1)
    x = torch.zeros((1, dim), device="cuda")
    out = torch.empty((1, dim), device="cuda")
    with pytest.raises(Exception):
        L.forward(x, out)  # 64 experts do not split into 3 groups
    L.n_group, L.topk_group = 8, 0
    with pytest.raises(Exception):
        L.forward(x, out)  # no group kept
    L.n_group, L.topk_group = 16, 1
    with pytest.raises(Exception):
        L.forward(x, out)  # one group of 4 experts cannot supply 6
    for t_ in (L.gate, L.up, L.down, L.router):
        t_.free()


def test_moe_ffn_block_other_k_types(be, orc):
    """Experts in Q5_K / Q2_K / Q3_K / Q4_1 / Q5_1 (the types real Q*_K_M / Q*_K_S
    checkpoints mix in; DeepSeek-Coder-V2-Lite's ffn_down_exps are Q5_1):
    moeFfnBlock through the general slot kernels against the oracle."""
    rng = np.random.default_rng(33)
    dim, ffn = 1024, 512
    from tests import npref
    ex, oex = [], []
    for gt, ut, dt, w in [(13, 13, 13, 0.6), (10, 11, 10, 0.3), (11, 13, 12, 0.1), (12, 12, 7, 0.4), (3, 7, 3, 0.2)]:
        g = npref.random_blocks(rng, gt, ffn, dim)
        u = npref.random_blocks(rng, ut, ffn, dim)
        d = npref.random_blocks(rng, dt, dim, ffn)
        ex.append(B.ExpertRef(B.WeightRef(gt, g), B.WeightRef(ut, u), B.WeightRef(dt, d), w, ffn))
        oex.append(dict(gate_type=gt, up_type=ut, down_type=dt, gate=g, up=u, down=d, weight=w, ffn=ffn))
    x = rng.standard_normal(dim).astype(np.float32)
    out = np.full(dim, np.nan, np.float32)
    assert B.moeFfnBlock(x, ex, out)
    want = orc.moe_ffn_block(x, oex, dim)
    assert rel_l2(out, want) < TOL
