"""Pins the CPU oracle against the reference's own known-answer tests and
invariants (ch4r10t33r/loom src/gguf/ggml.zig:1906-2210, src/gguf/moe.zig:210-262,
src/core/tensor.zig:77-101), and cross-checks it bit for bit against an
independent numpy restatement of the block decoders."""
import json
import os

import numpy as np
import pytest

from tests import npref

GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "known_answers.json")))
TYPES = [2, 8, 12, 14]  # q4_0, q8_0, q4_k, q6_k


@pytest.mark.parametrize("case", GOLDEN["dequant"], ids=lambda c: c["name"])
def test_known_answer_dequant(orc, case):
    blk = np.array(case["block"], np.uint8)
    vals = orc.dequant_row(case["type"], blk, 0, case["cols"])
    if "expect_at" in case:
        for i, v in case["expect_at"].items():
            assert abs(vals[int(i)] - v) <= case["tol"]
    if "expect_all" in case:
        assert np.all(np.abs(vals - case["expect_all"]) <= case["tol"])
    if "matvec_ones" in case:
        out = orc.matvec(case["type"], blk, np.ones(case["cols"], np.float32), 1, case["cols"])
        assert abs(out[0] - case["matvec_ones"]) <= case["matvec_tol"]


@pytest.mark.parametrize("case", GOLDEN["route"], ids=lambda c: c["name"])
def test_known_answer_route(orc, case):
    ids, gates = orc.route(np.array(case["logits"], np.float32), case["n_used"], case["gating"],
                           case["norm"], case["scale"],
                           None if case["bias"] is None else np.array(case["bias"], np.float32))
    if "expect_ids" in case:
        assert list(ids) == case["expect_ids"]
        np.testing.assert_allclose(gates, case["expect_gates"], atol=case["tol"], rtol=0)
    if "expect_gate_sum" in case:
        assert abs(gates.sum() - case["expect_gate_sum"]) <= case["tol"]
    if "expect_gate_sum_below" in case:
        assert gates.sum() < case["expect_gate_sum_below"]


def test_known_answer_softmax(orc):
    for case in GOLDEN["softmax"]:
        assert abs(orc.softmax(case["x"]).sum() - case["expect_sum"]) <= case["tol"]


@pytest.mark.parametrize("t", TYPES)
def test_dequant_matches_numpy_restatement_bitexact(orc, t):
    rng = np.random.default_rng(100 + t)
    rows, cols = 5, 512
    data = npref.random_blocks(rng, t, rows, cols)
    got = orc.dequant(t, data, rows, cols)
    want = npref.DEQUANT[t](data.tobytes(), rows, cols)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("t", TYPES + [0])
def test_matvec_agrees_with_dequant_row(orc, t):
    """ggml.zig:2021-2087: matvec vs dequant-then-dot, mass*0.01 for int8 kernels."""
    rng = np.random.default_rng(0xC0FFEE)
    cols, rows = 256, 3
    x = ((rng.random(cols, dtype=np.float32) - 0.5) * 4.0).astype(np.float32)
    if t == 0:
        data = rng.standard_normal(rows * cols).astype(np.float32).view(np.uint8)
    else:
        data = npref.random_blocks(rng, t, rows, cols)
    got = orc.matvec(t, data, x, rows, cols)
    for r in range(rows):
        row = orc.dequant_row(t, data, r, cols)
        want = np.float32(0)
        mass = np.float32(0)
        for w, xv in zip(row, x):
            want = np.float32(want + w * xv)
            mass = np.float32(mass + abs(w * xv))
        tol = mass * 0.01 if t != 0 else max(abs(want), abs(got[r])) * 1e-4 + 1e-3
        assert abs(want - got[r]) <= tol, (t, r, got[r], want)


def test_q40_q80_within_quant_error(orc):
    """ggml.zig:1906-1936, with the test's own encoders."""
    rng = np.random.default_rng(3)
    rows, cols = 4, 64
    wf = (rng.random((rows, cols), dtype=np.float32) - 0.5).astype(np.float32)
    x = (rng.random(cols, dtype=np.float32) - 0.5).astype(np.float32)
    ref = orc.matvec(0, wf.view(np.uint8).ravel(), x, rows, cols)
    q4 = np.concatenate([npref.quantize_q40(wf[r]) for r in range(rows)])
    q8 = np.concatenate([npref.quantize_q80(wf[r]) for r in range(rows)])
    o4 = orc.matvec(2, q4, x, rows, cols)
    o8 = orc.matvec(8, q8, x, rows, cols)
    assert np.all(np.abs(o4 - ref) < 0.6)
    assert np.all(np.abs(o8 - ref) < 0.05)


@pytest.mark.parametrize("t", [12, 14, 8, 2, 0])
def test_matmul_bit_identical_to_matvec(orc, t):
    """ggml.zig:2132-2186 with per-token magnitudes differing."""
    rng = np.random.default_rng(0x5EED)
    cols, rows = 512, 133
    if t == 0:
        data = rng.standard_normal(rows * cols).astype(np.float32).view(np.uint8)
    else:
        data = npref.random_blocks(rng, t, rows, cols)
    for n in (2, 3, 5, 8):
        xs = np.stack([(rng.random(cols, dtype=np.float32) - 0.5) * (k + 1) for k in range(n)]).astype(np.float32)
        want = np.stack([orc.matvec(t, data, xs[k], rows, cols) for k in range(n)])
        got = orc.matmul(t, data, xs, rows, cols)
        assert np.array_equal(want.view(np.uint32), got.view(np.uint32))


def test_parallel_bit_identical(orc):
    """ggml.zig:2089-2130: row splitting never perturbs an element."""
    rng = np.random.default_rng(0xBEEF)
    cols, rows = 256, 257
    x = ((rng.random(cols, dtype=np.float32) - 0.5) * 4.0).astype(np.float32)
    for t in (14, 12, 0):
        data = (rng.standard_normal(rows * cols).astype(np.float32).view(np.uint8) if t == 0
                else npref.random_blocks(rng, t, rows, cols))
        serial = orc.matvec(t, data, x, rows, cols)
        orc.parallel_begin(8)
        try:
            assert orc.lib().or_pool_workers() > 0
            for _ in range(4):
                par = orc.matvec(t, data, x, rows, cols)
                assert np.array_equal(serial.view(np.uint32), par.view(np.uint32))
        finally:
            orc.parallel_end()


def test_nonfinite_activations_do_not_trap(orc):
    """ggml.zig:2188-2210."""
    x = (np.arange(64) % 7).astype(np.float32)
    x[0], x[1], x[2] = np.nan, np.inf, -np.inf
    q, d, s = orc.quantize_x32(x)
    assert np.all(np.isfinite(d)) and q.min() >= -127 and q.max() <= 127
    y = np.full(32, np.nan, np.float32)
    q, d, s = orc.quantize_x32(y)
    assert d[0] == 0 and np.all(q == 0)
    q, d, s = orc.quantize_x256(np.full(256, np.nan, np.float32))
    assert d[0] == 0 and np.all(q == 0) and np.all(s == 0)


def test_quantizer_rounding_half_away_from_zero(orc):
    """toI8Saturating (ggml.zig:1067): @round is half away from zero."""
    x = np.zeros(32, np.float32)
    x[0] = 127.0  # d = 1, inv = 1
    x[1], x[2], x[3], x[4] = 0.5, -0.5, 2.5, -2.5
    q, d, s = orc.quantize_x32(x)
    assert d[0] == 1.0
    assert list(q[:5]) == [127, 1, -1, 3, -3]
    assert s[0] == 127 + 1 - 1 + 3 - 3


def test_route_ties_lowest_index_and_selection_order(orc):
    """moe.zig:135-146: strict '>' keeps the first maximum."""
    ids, _ = orc.route(np.array([1.0, 3.0, 3.0, 2.0, 3.0], np.float32), 3, 1, True, 1.0)
    assert list(ids) == [1, 2, 4]


def test_route_renorm_clamp(orc):
    """moe.zig:149-153: divisor clamped to 6.103515625e-5."""
    logits = np.full(4, -200.0, np.float32)
    ids, gates = orc.route(logits, 2, 2, True, 1.0)  # sigmoid(-200) ~ 0
    assert np.all(np.isfinite(gates))


def test_moe_ffn_routed_equals_block(orc):
    """moeFfnBlockRouted == route + moeFfnBlock over the selected planes."""
    rng = np.random.default_rng(7)
    dim, ffn, ne, k = 512, 256, 8, 3
    gate = npref.random_blocks(rng, 12, ne * ffn, dim)
    up = npref.random_blocks(rng, 12, ne * ffn, dim)
    down = npref.random_blocks(rng, 14, ne * dim, ffn)
    x = rng.standard_normal(dim).astype(np.float32)
    logits = rng.standard_normal(ne).astype(np.float32)
    out = orc.moe_ffn_routed(x, logits, (12, gate), (12, up), (14, down), ffn, k)
    ids, gates = orc.route(logits, k)
    gp, dp = ffn * orc.row_bytes(12, dim), dim * orc.row_bytes(14, ffn)
    ex = [dict(gate_type=12, up_type=12, down_type=14, gate=gate[i * gp:(i + 1) * gp],
               up=up[i * gp:(i + 1) * gp], down=down[i * dp:(i + 1) * dp], weight=float(g), ffn=ffn)
          for i, g in zip(ids, gates)]
    want = orc.moe_ffn_block(x, ex, dim)
    assert np.array_equal(out.view(np.uint32), want.view(np.uint32))


def test_synth_matches_spec(orc):
    """The seeded generator emits valid blocks with the configured scale ranges."""
    b = orc.synth(12, 64, seed=11).reshape(64, 144)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32).ravel()
    assert d.min() >= 0.00099 and d.max() <= 0.01001
    b6 = orc.synth(14, 64, seed=11).reshape(64, 210)
    sc = b6[:, 192:208].view(np.int8)
    assert sc.min() >= -32 and sc.max() <= 31
    f = orc.synth(0, 100000, seed=5, sigma=0.02)
    assert abs(f.std() - 0.02) < 0.002 and abs(f.mean()) < 0.001
    again = orc.synth(12, 8, seed=11, blk0=10)
    assert np.array_equal(again, b[10:18].ravel())


def _np_grouped_route(logits, bias, k, n_group, topk_group):
    """Independent restatement of DeepSeek-V3's group-limited top-k (sigmoid
    gating, bias for selection only, renormalised gates): group score = sum of
    the group's two largest biased scores; the topk_group best groups are
    kept; top-k over the kept experts; ties take the lowest index."""
    s = (1.0 / (1.0 + np.exp(-logits.astype(np.float64)))).astype(np.float32)
    c = s + bias
    gs = logits.size // n_group
    grp = np.sort(c.reshape(n_group, gs), axis=1)[:, ::-1]
    gsc = grp[:, 0] + grp[:, 1]
    keep = np.argsort(-gsc, kind="stable")[:topk_group]
    mask = np.full(logits.size, -np.inf, np.float32)
    for g in keep:
        mask[g * gs:(g + 1) * gs] = 0.0
    ids = np.argsort(-(c + mask), kind="stable")[:k]
    g = s[ids]
    return ids, g / g.sum()


@pytest.mark.parametrize("seed", range(6))
def test_grouped_route_matches_restatement(orc, seed):
    """DeepSeek-V3 shape: 256 experts, 8 groups, keep 4, top-8."""
    rng = np.random.default_rng(100 + seed)
    logits = rng.standard_normal(256).astype(np.float32) * 2
    bias = rng.standard_normal(256).astype(np.float32) * 0.1
    ids, gates = orc.route(logits, 8, 2, True, 1.0, bias, n_group=8, topk_group=4)
    rids, rg = _np_grouped_route(logits, bias, 8, 8, 4)
    assert list(ids) == list(rids)
    np.testing.assert_allclose(gates, rg, rtol=1e-5, atol=0)
    kept = set(int(i) // 32 for i in ids)
    assert len(kept) <= 4


@pytest.mark.parametrize("gating", [1, 2, 3])
def test_grouped_route_one_group_is_route(orc, gating):
    """n_group = 1 (or topk_group = n_group) reduces exactly to moe.route."""
    rng = np.random.default_rng(5)
    logits = rng.standard_normal(64).astype(np.float32)
    bias = rng.standard_normal(64).astype(np.float32) * 0.1
    a = orc.route(logits, 6, gating, True, 1.0, bias)
    for ng, tg in [(1, 1), (8, 8)]:
        ids = np.empty(6, np.uint32)
        g = np.empty(6, np.float32)
        assert orc.lib().or_route_grouped(orc._p(logits), orc._p(bias), 64, 6, gating, 1, 1.0, ng, tg,
                                          orc._p(ids), orc._p(g)) == 0
        assert list(ids) == list(a[0])
        assert g.tobytes() == a[1].tobytes()


def test_grouped_route_rejects_bad_groups(orc):
    logits = np.zeros(64, np.float32)
    ids = np.empty(8, np.uint32)
    g = np.empty(8, np.float32)
    L = orc.lib()
    assert L.or_route_grouped(orc._p(logits), None, 64, 8, 2, 1, 1.0, 3, 1, orc._p(ids), orc._p(g)) != 0  # 64 % 3
    assert L.or_route_grouped(orc._p(logits), None, 64, 8, 2, 1, 1.0, 8, 0, orc._p(ids), orc._p(g)) != 0
    assert L.or_route_grouped(orc._p(logits), None, 64, 9, 2, 1, 1.0, 8, 1, orc._p(ids), orc._p(g)) != 0  # k > 8


def test_known_answer_argmax(orc):
    """sampler.zig:33-36."""
    for case in GOLDEN["argmax"]:
        assert orc.argmax(np.array(case["logits"], np.float32)) == case["expect"]


def test_argmax_ties_nan_and_inf(orc):
    """Strict '>' from -inf: the first maximum wins, NaN is never taken, nothing above -inf gives 0."""
    f = lambda v: orc.argmax(np.array(v, np.float32))  # noqa: E731
    assert f([1.0, 5.0, 5.0, 2.0]) == 1
    assert f([np.nan, 1.0, np.nan, 3.0]) == 3
    assert f([-np.inf, -np.inf]) == 0
    assert f([np.nan, np.nan]) == 0
    assert f([-np.inf, -5.0, np.inf, np.inf]) == 2
    assert f([0.0, -0.0]) == 0 and f([-0.0, 0.0]) == 0


def test_q5k_high_bit_adds_16(orc):
    """ggml.zig:1979-1990: d = 1, dmin = 0, sc(sub-block 0) = 1, qh bit 0 of byte 0 set, qs zero."""
    blk = np.zeros(176, np.uint8)
    blk[0:2] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)
    blk[4] = 1
    blk[16] = 1
    v = orc.dequant_row(13, blk, 0, 256)
    assert abs(v[0] - 16.0) < 1e-4 and abs(v[1]) < 1e-4


@pytest.mark.parametrize("t", [3, 6, 7, 10, 11, 13])
def test_new_k_types_matvec_agrees_with_dequant(orc, t):
    """ggml.zig:2021-2087 for q4_1 / q5_1 / q2_k / q3_k / q5_k: random bytes (one f16 exponent
    bit cleared so no scale is NaN/Inf), int8-activation matvec within
    mass * 0.01 of dequant-then-dot; matmul bit-identical to n matvecs."""
    rng = np.random.default_rng(t)
    cols, rows = 512, 3
    data = rng.integers(0, 256, rows * (cols // orc.BLOCK_ELEMS[t]) * orc.BLOCK_BYTES[t], dtype=np.uint8)
    data[1::2] &= 0xFB
    x = ((rng.random(cols) - 0.5) * 4.0).astype(np.float32)
    got = orc.matvec(t, data, x, rows, cols)
    for r in range(rows):
        w = orc.dequant_row(t, data, r, cols).astype(np.float64)
        want, mass = float(np.sum(w * x)), float(np.sum(np.abs(w * x)))
        assert abs(got[r] - want) <= mass * 0.01, (t, r, got[r], want)
    xs = ((rng.random((4, cols)) - 0.5) * 4.0).astype(np.float32)
    mm = orc.matmul(t, data, xs, rows, cols)
    for k in range(4):
        assert np.array_equal(np.asarray(mm).reshape(4, rows)[k].view(np.uint32),
                              orc.matvec(t, data, xs[k], rows, cols).view(np.uint32))


def test_q2k_q3k_decode_matches_numpy_restatement(orc):
    """Independent numpy restatement of dequantBlockQ2K (:1476) and
    dequantBlockQ3K (:1508), including q3kScales (:1173)."""
    rng = np.random.default_rng(3)
    b2 = rng.integers(0, 256, 84, dtype=np.uint8)
    b2[81] &= 0xFB
    b2[83] &= 0xFB
    d, dmin = np.frombuffer(b2[80:82].tobytes(), np.float16)[0], np.frombuffer(b2[82:84].tobytes(), np.float16)[0]
    want = []
    for n in range(2):
        for j in range(4):
            for half in range(2):
                sc = b2[8 * n + 2 * j + half]
                dl, ml = np.float32(d) * np.float32(sc & 15), np.float32(dmin) * np.float32(sc >> 4)
                for l in range(16):
                    q = (int(b2[16 + 32 * n + half * 16 + l]) >> (2 * j)) & 3
                    want.append(np.float32(dl * np.float32(q)) - ml)
    assert np.array_equal(np.array(want, np.float32).view(np.uint32), orc.dequant_row(10, b2, 0, 256).view(np.uint32))
    b3 = rng.integers(0, 256, 110, dtype=np.uint8)
    b3[109] &= 0xFB
    aux = np.frombuffer(b3[96:108].tobytes(), np.uint32).copy()
    a0, a1, tmp = int(aux[0]), int(aux[1]), int(aux[2])
    m1, m2 = 0x03030303, 0x0f0f0f0f
    words = [(a0 & m2) | (((tmp >> 0) & m1) << 4), (a1 & m2) | (((tmp >> 2) & m1) << 4),
             ((a0 >> 4) & m2) | (((tmp >> 4) & m1) << 4), ((a1 >> 4) & m2) | (((tmp >> 6) & m1) << 4)]
    sc16 = np.frombuffer(np.array(words, np.uint32).tobytes(), np.uint8).astype(np.int32) - 32
    d3 = np.float32(np.frombuffer(b3[108:110].tobytes(), np.float16)[0])
    want = []
    for n in range(2):
        for j in range(4):
            m = 1 << (4 * n + j)
            for half in range(2):
                dl = d3 * np.float32(sc16[8 * n + 2 * j + half])
                for l in range(16):
                    idx = half * 16 + l
                    q = (int(b3[32 + 32 * n + idx]) >> (2 * j)) & 3
                    want.append(dl * np.float32(q - (0 if b3[idx] & m else 4)))
    assert np.array_equal(np.array(want, np.float32).view(np.uint32), orc.dequant_row(11, b3, 0, 256).view(np.uint32))


def test_q51_matches_numpy_restatement(orc):
    """matvecQ41Int (:1242) and dequantRow (:1795) for q5_1, restated in numpy."""
    rng = np.random.default_rng(71)
    blk = rng.integers(0, 256, 24, dtype=np.uint8)
    blk[1] &= 0xFB
    blk[3] &= 0xFB
    d, m = (np.float32(v) for v in np.frombuffer(blk[0:4].tobytes(), np.float16))
    qh = int(np.frombuffer(blk[4:8].tobytes(), np.uint32)[0])
    want = np.zeros(32, np.float32)
    for j in range(16):
        lo = (int(blk[8 + j]) & 15) | (((qh >> j) << 4) & 0x10)
        hi = (int(blk[8 + j]) >> 4) | ((qh >> (j + 12)) & 0x10)
        want[j] = np.float32(np.float32(lo) * d) + m
        want[j + 16] = np.float32(np.float32(hi) * d) + m
    assert np.array_equal(want.view(np.uint32), orc.dequant_row(7, blk, 0, 32).view(np.uint32))


def test_q50_f32_path_matches_numpy(orc):
    """matvecQ50 (:1673): f32 activations, per block partial += w0*x[j] + w1*x[j+16]
    in order, zero-scale blocks skipped (even with non-finite activations)."""
    rng = np.random.default_rng(6)
    cols = 96
    data = rng.integers(0, 256, 3 * 22, dtype=np.uint8)
    data[1::2] &= 0xFB
    data[44:46] = 0  # block 2: scale 0
    x = rng.standard_normal(cols).astype(np.float32)
    x[70] = np.inf  # inside the zero-scale block: skipped, so no NaN
    acc = np.float32(0)
    for b in range(3):
        blk = data[b * 22:(b + 1) * 22]
        s = np.float32(np.frombuffer(blk[0:2].tobytes(), np.float16)[0])
        if s == 0:
            continue
        qh = int(np.frombuffer(blk[2:6].tobytes(), np.uint32)[0])
        part = np.float32(0)
        for j in range(16):
            w0 = np.float32(((int(blk[6 + j]) & 15) | (((qh >> j) << 4) & 0x10)) - 16)
            w1 = np.float32(((int(blk[6 + j]) >> 4) | ((qh >> (j + 12)) & 0x10)) - 16)
            part = np.float32(part + np.float32(np.float32(w0 * x[b * 32 + j]) + np.float32(w1 * x[b * 32 + j + 16])))
        acc = np.float32(acc + np.float32(part * s))
    got = orc.matvec(6, data, x, 1, cols)
    assert got.view(np.uint32)[0] == np.float32(acc).view(np.uint32)
