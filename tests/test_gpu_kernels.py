"""GPU parity of the block kernels against the CPU oracle (the reference's CPU
kernels restated): dequantRow bit-exact, matvec/matmul bit-exact (int8
activations, same integer sums, same float tail, same block order), router ids
identical. Every call goes through the C ABI (include/loom_cuda.h)."""
import json
import os

import numpy as np
import pytest

from tests import npref
from tests.conftest import bits

pytestmark = pytest.mark.gpu

GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "known_answers.json")))
QTYPES = [2, 3, 6, 7, 8, 10, 11, 12, 13, 14]


def _data(rng, t, rows, cols):
    if t == 0:
        return rng.standard_normal(rows * cols).astype(np.float32).view(np.uint8)
    return npref.random_blocks(rng, t, rows, cols)


@pytest.mark.parametrize("case", GOLDEN["dequant"], ids=lambda c: c["name"])
def test_known_answer_blocks(be, case):
    blk = np.array(case["block"], np.uint8)
    out = np.empty(case["cols"], np.float32)
    be.dequantRow(case["type"], out, blk, 0, case["cols"])
    if "expect_at" in case:
        for i, v in case["expect_at"].items():
            assert abs(out[int(i)] - v) <= case["tol"]
    if "expect_all" in case:
        assert np.all(np.abs(out - case["expect_all"]) <= case["tol"])
    if "matvec_ones" in case:
        mv = np.empty(1, np.float32)
        be.matvec(case["type"], mv, blk, np.ones(case["cols"], np.float32), 1, case["cols"])
        assert abs(mv[0] - case["matvec_ones"]) <= case["matvec_tol"]


@pytest.mark.parametrize("t", QTYPES + [0])
def test_dequant_row_bitexact(be, orc, t):
    rng = np.random.default_rng(11 + t)
    rows, cols = 7, 512
    data = _data(rng, t, rows, cols)
    for r in range(rows):
        got = np.empty(cols, np.float32)
        be.dequantRow(t, got, data, r, cols)
        assert np.array_equal(bits(got), bits(orc.dequant_row(t, data, r, cols))), (t, r)


@pytest.mark.parametrize("t,rows,cols", [
    (12, 257, 256), (12, 768, 2048), (12, 64, 7168), (14, 257, 256), (14, 2048, 768), (14, 33, 1536),
    (8, 257, 288), (8, 100, 1408), (8, 64, 2048), (2, 257, 288), (2, 96, 768), (2, 40, 2048),
    (0, 128, 2048), (0, 37, 300), (0, 5, 7), (0, 9, 40),
    (3, 257, 288), (3, 100, 1408), (7, 257, 288), (7, 100, 1408), (6, 257, 288), (6, 100, 1408),
    (10, 257, 256), (10, 96, 2048), (11, 257, 256), (11, 96, 2048), (13, 257, 256), (13, 768, 2048)])
def test_matvec_bitexact(be, orc, t, rows, cols):
    rng = np.random.default_rng(rows * 31 + cols + t)
    data = _data(rng, t, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    got = np.full(rows, np.nan, np.float32)
    be.matvec(t, got, data, x, rows, cols)
    want = orc.matvec(t, data, x, rows, cols)
    assert np.array_equal(bits(got), bits(want)), (np.abs(got - want).max(), t)


@pytest.mark.parametrize("t", QTYPES + [0])
def test_matmul_bitexact_and_equals_matvec(be, orc, t):
    rng = np.random.default_rng(0x5EED + t)
    rows, cols = 133, 512
    data = _data(rng, t, rows, cols)
    for n in (2, 3, 5, 8, 17):
        xs = np.stack([(rng.random(cols, dtype=np.float32) - 0.5) * (k + 1) for k in range(n)]).astype(np.float32)
        got = np.full(n * rows, np.nan, np.float32)
        be.matmul(t, got, data, xs, n, rows, cols)
        want = orc.matmul(t, data, xs, rows, cols).ravel()
        assert np.array_equal(bits(got), bits(want)), (t, n)
        one = np.empty(rows, np.float32)
        be.matvec(t, one, data, xs[n - 1], rows, cols)
        assert np.array_equal(bits(one), bits(got[(n - 1) * rows:]))


def test_matvec_nonfinite_activations(be, orc):
    """ggml.zig:2188: NaN/Inf activations quantize to 0 instead of trapping."""
    rng = np.random.default_rng(5)
    rows, cols = 16, 512
    for t in QTYPES:
        data = _data(rng, t, rows, cols)
        x = rng.standard_normal(cols).astype(np.float32)
        x[3], x[300], x[301] = np.nan, np.inf, -np.inf
        x[256:288] = np.nan  # an all-non-finite 32 block
        got = np.empty(rows, np.float32)
        be.matvec(t, got, data, x, rows, cols)
        want = orc.matvec(t, data, x, rows, cols)
        if t == 6:  # q5_0 stays on f32 activations: non-finite values reach the sums (NaN payloads differ by host)
            assert np.array_equal(np.isnan(got), np.isnan(want))
            got, want = np.nan_to_num(got, nan=0.0), np.nan_to_num(want, nan=0.0)
        assert np.array_equal(bits(got), bits(want))


@pytest.mark.parametrize("case", GOLDEN["route"], ids=lambda c: c["name"])
def test_route_known_answers(be, case):
    if case["gating"] == 3:
        pytest.skip("softmax_topk is gpt-oss only; the seam's moeRoute carries softmax|sigmoid")
    k = case["n_used"]
    ids = np.empty(k, np.uint32)
    gates = np.empty(k, np.float32)
    bias = None if case["bias"] is None else np.array(case["bias"], np.float32)
    assert be.moeRoute(np.array(case["logits"], np.float32), bias, ids, gates, case["gating"] == 2, case["norm"],
                       case["scale"])
    if "expect_ids" in case:
        assert list(ids) == case["expect_ids"]
        np.testing.assert_allclose(gates, case["expect_gates"], atol=case["tol"], rtol=0)
    if "expect_gate_sum" in case:
        assert abs(gates.sum() - case["expect_gate_sum"]) <= case["tol"]
    if "expect_gate_sum_below" in case:
        assert gates.sum() < case["expect_gate_sum_below"]


def _check_route(ids, gates, want_ids, want_gates, logits_sel):
    """ids identical wherever the selection gap exceeds 1e-4 (north-star rule)."""
    srt = np.sort(logits_sel)[::-1]
    k = len(ids)
    gaps = srt[:k] - srt[1:k + 1]
    if np.all(gaps > 1e-4):
        assert list(ids) == list(want_ids)
        np.testing.assert_allclose(gates, want_gates, rtol=1e-5, atol=1e-7)
        return True
    return False


@pytest.mark.parametrize("ne,k,sig,bias", [(128, 8, False, False), (64, 6, False, False), (256, 8, True, True),
                                           (1024, 64, False, False), (8, 2, False, False), (256, 8, False, True)])
def test_route_matches_oracle(be, orc, ne, k, sig, bias):
    rng = np.random.default_rng(ne + k)
    checked = 0
    for trial in range(20):
        logits = (rng.standard_normal(ne) * 2).astype(np.float32)
        b = (rng.standard_normal(ne) * 0.1).astype(np.float32) if bias else None
        ids = np.empty(k, np.uint32)
        gates = np.empty(k, np.float32)
        assert be.moeRoute(logits, b, ids, gates, sig, True, 2.5 if sig else 1.0)
        wids, wg = orc.route(logits, k, 2 if sig else 1, True, 2.5 if sig else 1.0, b)
        scores = (1 / (1 + np.exp(-logits.astype(np.float64)))) if sig else logits.astype(np.float64)
        sel = scores + (b if b is not None else 0)
        checked += _check_route(ids, gates, wids, wg, sel)
    assert checked >= 10


def test_route_ties_keep_lowest_index(be):
    ids = np.empty(3, np.uint32)
    gates = np.empty(3, np.float32)
    assert be.moeRoute(np.array([1, 3, 3, 2, 3], np.float32), None, ids, gates, False, True, 1.0)
    assert list(ids) == [1, 2, 4]


def test_declines_bad_shapes(be):
    out = np.empty(4, np.float32)
    assert not be.moeRoute(np.zeros(4, np.float32), None, np.empty(5, np.uint32), np.empty(5, np.float32),
                           False, True, 1.0)
    with pytest.raises(Exception):
        be.matvec(12, out, np.zeros(144 * 4, np.uint8), np.zeros(300, np.float32), 4, 300)  # ragged cols


def test_launch_counter_moves(be):
    """Every seam op is one submission and launches this library's kernels
    (the reference's no-silent-fallback check, vulkan/backend.zig:2153)."""
    rng = np.random.default_rng(1)
    data = _data(rng, 12, 64, 256)
    be.takeCmdBufCount()
    k0 = be.kernelLaunches()
    out = np.empty(64, np.float32)
    be.matvec(12, out, data, np.ones(256, np.float32), 64, 256)
    assert be.takeCmdBufCount() == 1
    assert be.kernelLaunches() > k0


@pytest.mark.parametrize("n", [1, 5, 300, 151936])
def test_device_argmax_matches_sampler(be, orc, n):
    """sampler.zig:7-15 on the device: first maximum, NaN never taken, 0 when
    nothing is above -inf; bit-compatible with the oracle on random logits,
    planted ties, NaN and infinities."""
    import torch
    from loom_b200 import device as D
    rng = np.random.default_rng(n)
    cases = [rng.standard_normal(n).astype(np.float32)]
    v = rng.standard_normal(n).astype(np.float32)
    if n >= 5:
        v[[n // 3, n // 2, n - 1]] = 7.0  # ties: the first one wins
        v[n // 4] = np.nan
    cases.append(v)
    cases.append(np.full(n, -np.inf, np.float32))
    cases.append(np.full(n, np.nan, np.float32))
    w = rng.standard_normal(n).astype(np.float32)
    w[n - 1] = np.inf
    cases.append(w)
    for c in cases:
        got = int(D.argmax(torch.from_numpy(c).cuda()).item())
        assert got == orc.argmax(c)


def test_lm_head_argmax_q6k(be, orc):
    """The output head (Q6_K [151936 x 2048], Qwen3's vocab) and its greedy
    sample: logits bit-identical to the oracle's matvec, the same token."""
    import torch
    from loom_b200 import device as D
    vocab, dim = 151936, 2048
    nblk = vocab * dim // 256
    W = D.DeviceTensor.synth(14, nblk, seed=901, sigma=1.0)
    try:
        x = orc.synth(0, dim, seed=902, sigma=1.0)
        logits = torch.empty(vocab, device="cuda")
        tok = D.lm_head_argmax(W, vocab, dim, torch.from_numpy(x).cuda(), logits=logits)
        want = orc.matvec(14, orc.synth(14, nblk, seed=901), x, vocab, dim)
        assert np.array_equal(bits(logits.cpu().numpy()), bits(want))
        assert int(tok.item()) == orc.argmax(want)
    finally:
        W.free()


@pytest.mark.parametrize("t", [12, 14, 6, 0])
def test_repeated_seam_calls_replay_exactly(be, orc, t):
    """Repeated calls on the same weights and shape (eager, captured, then
    replayed as one graph) stay bit-exact with fresh inputs every call and
    still count their kernel launches."""
    rng = np.random.default_rng(70 + t)
    rows, cols = 96, 512
    data = _data(rng, t, rows, cols)
    for _ in range(5):
        x = rng.standard_normal(cols).astype(np.float32)
        got = np.full(rows, np.nan, np.float32)
        k0 = be.kernelLaunches()
        be.matvec(t, got, data, x, rows, cols)
        assert be.kernelLaunches() > k0
        assert np.array_equal(bits(got), bits(orc.matvec(t, data, x, rows, cols)))


@pytest.mark.parametrize("t,rows,cols", [(12, 8195, 7168), (12, 4100, 16384), (14, 5003, 2048), (14, 4096, 4096)])
def test_streamed_matvec_bitexact(be, orc, t, rows, cols):
    """Large matrices take the streamed matvec (tiles bulk-copied through
    shared memory, one CTA per SM; ragged last tiles): bit-identical to the
    oracle's matvec (ggml.zig:602)."""
    import torch
    from loom_b200 import device as D
    nblk = rows * cols // 256
    W = D.DeviceTensor.synth(t, nblk, seed=911 + t, sigma=1.0)
    try:
        x = orc.synth(0, cols, seed=912, sigma=1.0)
        out = torch.full((1, rows), float("nan"), device="cuda")
        D.tensor_matmul(W, rows, cols, torch.from_numpy(x.reshape(1, cols)).cuda(), out)
        torch.cuda.synchronize()
        want = orc.matvec(t, orc.synth(t, nblk, seed=911 + t), x, rows, cols)
        assert np.array_equal(bits(out.cpu().numpy().reshape(-1)), bits(want))
    finally:
        W.free()
