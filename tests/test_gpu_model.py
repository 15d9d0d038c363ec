"""GPU parity of whole-model decode (loom_cuda_model_*) against the oracle's
token step (or_llama_step, restating llama.zig:1111-1228), through the C ABI.

The north star's bar for the small configs: greedy-decoded tokens identical
for 64 steps (tiny llama Q4_0, seeded 8-token prompt).
Logits are compared within 2e-3 relative L2 with the oracle fed the same
tokens; the KV cache rows within the same tolerance."""
import ctypes as C

import numpy as np
import pytest
import torch

from loom_b200 import _lib
from loom_b200.model import DeviceModel, greedy, qwen3_moe, tiny_llama
from tests.conftest import rel_l2
from tests.modelref import host_tensors

pytestmark = pytest.mark.gpu
TOL = 2e-3


def _runner(spec, orc):
    from oracle.oracle import LlamaRunner
    return LlamaRunner(spec, host_tensors(spec, orc))


def test_tiny_llama_64_greedy_tokens_match_oracle(be, orc):
    spec = tiny_llama(ctx_len=256)
    rng = np.random.default_rng(1)
    prompt = [int(t) for t in rng.integers(1, 32000, size=8)]
    ref = _runner(spec, orc)
    want = greedy(lambda t, p: int(np.argmax(ref.step(t, p))), prompt, 64)
    dev = DeviceModel(spec)
    try:
        got = greedy(lambda t, p: dev.decode(t, p)[0], prompt, 64)
        assert got == want
        assert len(set(want)) > 4  # the synthetic model does not collapse to one token
        kvd = spec.n_kv_heads * spec.head_dim
        kc = ref.kc.reshape(spec.n_layers, spec.ctx_len, kvd)
        vc = ref.vc.reshape(spec.n_layers, spec.ctx_len, kvd)
        for li, pos in ((0, 0), (3, 40), (5, 70)):
            k, v = dev.read_kv(li, pos)
            assert rel_l2(k, kc[li, pos]) < TOL and rel_l2(v, vc[li, pos]) < TOL
    finally:
        dev.free()


@pytest.mark.parametrize("spec,exact,tol", [
    (tiny_llama(ctx_len=160), False, TOL),
    (qwen3_moe(n_layers=2, ctx_len=160, n_expert=16, vocab=4096), True, TOL),
    (qwen3_moe(n_layers=2, ctx_len=640, n_expert=16, vocab=4096), True, TOL),
    (qwen3_moe(n_layers=2, ctx_len=640, n_expert=16, vocab=4096), False, 2e-2)],
    ids=["tiny_llama", "qwen3_exact", "qwen3_exact_long_ctx", "qwen3_fast_split"])
def test_model_logits_match_oracle_over_positions(be, orc, spec, exact, tol):
    """Teacher-forced: both sides get the same tokens. Tiny llama (dim 288,
    ctx 160) keeps the reference's order by default; the Qwen3 shape keeps it
    with exact_order. The fast form (tree-summed RMSNorm at dim 2048, split
    attention at ctx 640: chunks of 64 rows, merged) differs by rounding, which
    can move int8 activations of the next matvec: its logits are held to
    2e-2 relative L2."""
    ref = _runner(spec, orc)
    dev = DeviceModel(spec, exact_order=exact)
    rng = np.random.default_rng(7)
    try:
        for pos in range(140):
            tok = int(rng.integers(0, spec.vocab))
            want = ref.step(tok, pos)
            nxt, got = dev.decode(tok, pos, logits=True)
            assert np.all(np.isfinite(got))
            assert rel_l2(got, want) < tol, (pos, rel_l2(got, want))
            top = np.sort(want)[-2:]
            if top[1] - top[0] > 50 * tol * max(1.0, abs(top[1])):
                assert nxt == int(np.argmax(want)), pos
        assert dev.error() == 0
    finally:
        dev.free()


def test_model_step_on_device_buffers_equals_decode(be):
    """loom_cuda_model_step on torch buffers (a caller's stream) gives the same
    logits and token as the host entry point on a second model of the same weights."""
    spec = qwen3_moe(n_layers=2, ctx_len=64, n_expert=16, vocab=4096)
    a, b = DeviceModel(spec), DeviceModel(spec)
    try:
        s = torch.cuda.Stream()
        tok = torch.zeros(1, dtype=torch.int32, device="cuda")
        pos = torch.zeros(1, dtype=torch.int32, device="cuda")
        logits = torch.empty(spec.vocab, dtype=torch.float32, device="cuda")
        nxt = torch.empty(1, dtype=torch.int32, device="cuda")
        t = 11
        for p in range(5):
            with torch.cuda.stream(s):
                tok.fill_(t)
                pos.fill_(p)
                a.step(tok, pos, logits, nxt)
                got_tok = int(nxt.item())
                got = logits.cpu().numpy()
            want_tok, want = b.decode(t, p, logits=True)
            assert got_tok == want_tok
            assert np.array_equal(got, want)  # same kernels, same order
            t = want_tok
    finally:
        a.free()
        b.free()


def test_model_declines_bad_arguments(be):
    spec = tiny_llama(ctx_len=8)
    spec.n_layers = 1
    dev = DeviceModel(spec)
    try:
        nxt = C.c_uint32(0)
        L = _lib.lib()
        assert L.loom_cuda_model_decode(dev.handle, spec.vocab, 0, None, C.byref(nxt)) == _lib.DECLINED
        assert L.loom_cuda_model_decode(dev.handle, 1, spec.ctx_len, None, C.byref(nxt)) == _lib.DECLINED
        assert L.loom_cuda_model_decode(dev.handle + 999, 1, 0, None, C.byref(nxt)) == _lib.DECLINED
    finally:
        dev.free()


def test_fused_attention_block_equals_separate_kernels(be, monkeypatch):
    """The cooperative attention kernel (one launch per layer) against the
    separate kernels on the same weights, over positions that cross several
    attention chunks. The two RMSNorm trees (dim 2048) round differently, which
    can move an int8 activation: logits within the fast form's 2e-2."""
    spec = qwen3_moe(n_layers=2, ctx_len=640, n_expert=16, vocab=4096)
    a = DeviceModel(spec)
    monkeypatch.setenv("LOOM_CUDA_NO_ATTN_BLOCK", "1")
    b = DeviceModel(spec)
    try:
        rng = np.random.default_rng(3)
        for pos in range(100):
            tok = int(rng.integers(0, spec.vocab))
            na, la = a.decode(tok, pos, logits=True)
            nb, lb = b.decode(tok, pos, logits=True)
            assert rel_l2(la, lb) < 2e-2, (pos, rel_l2(la, lb))
        assert a.error() == 0
    finally:
        a.free()
        b.free()


def test_persistent_model_kernel_equals_per_layer_path(be, monkeypatch):
    """Every layer in one persistent launch (model_kernel.cu) against the
    per-layer launches on the same weights: the same kernels' arithmetic, so the
    logits agree to the RMSNorm tree's rounding (held to the fast form's 2e-2),
    over positions that cross several attention chunks, with the routing equal."""
    spec = qwen3_moe(n_layers=3, ctx_len=640, n_expert=16, vocab=4096)
    monkeypatch.setenv("LOOM_CUDA_PERSISTENT", "1")
    a = DeviceModel(spec)
    monkeypatch.delenv("LOOM_CUDA_PERSISTENT")
    b = DeviceModel(spec)
    try:
        rng = np.random.default_rng(11)
        worst = 0.0
        for pos in range(100):
            tok = int(rng.integers(0, spec.vocab))
            na, la = a.decode(tok, pos, logits=True)
            nb, lb = b.decode(tok, pos, logits=True)
            worst = max(worst, rel_l2(la, lb))
            assert rel_l2(la, lb) < 2e-2, (pos, rel_l2(la, lb))
        assert worst < 2e-2
        assert a.error() == 0
    finally:
        a.free()
        b.free()


def _ds_runner(spec, orc):
    from oracle.oracle import DeepseekRunner
    return DeepseekRunner(spec, host_tensors(spec, orc))


def _v3_small():
    from loom_b200.model import deepseek_v3
    spec = deepseek_v3(n_layers=3, ctx_len=96, n_expert=16, dim=1024, n_heads=8, vocab=2048, n_dense=1)
    spec.n_used, spec.n_group, spec.topk_group = 4, 4, 2
    return spec


@pytest.mark.parametrize("which,exact,tol,ctx,steps", [
    ("v2_lite", True, TOL, 96, 40), ("v2_lite", False, 2e-2, 96, 40), ("v3", True, TOL, 96, 40),
    ("v2_lite", False, 2e-2, 640, 100), ("v3", False, 2e-2, 640, 100)],
    ids=["v2_lite_exact", "v2_lite_fast", "v3_qlora_grouped_exact", "v2_lite_split", "v3_split"])
def test_mla_model_matches_oracle(be, orc, which, exact, tol, ctx, steps):
    """MLA decode (deepseek.zig:851-1049) on the device against the oracle:
    DeepSeek-V2-Lite shape (no q_lora, dense first layer, 2 shared experts,
    Q8_0 down projections) and a reduced V3 shape (q_lora, sigmoid + bias,
    grouped top-k, one shared expert); logits every step, the compressed and
    rope cache rows. Contexts past 512 without exact_order take the
    split-position attention (16-position chunks, merged records)."""
    from loom_b200.model import deepseek_v2_lite
    spec = deepseek_v2_lite(n_layers=2, ctx_len=ctx, n_expert=8, vocab=2048) if which == "v2_lite" else _v3_small()
    spec.ctx_len = ctx
    ref = _ds_runner(spec, orc)
    dev = DeviceModel(spec, exact_order=exact)
    rng = np.random.default_rng(13)
    try:
        for pos in range(steps):
            tok = int(rng.integers(0, spec.vocab))
            want = ref.step(tok, pos)
            nxt, got = dev.decode(tok, pos, logits=True)
            assert np.all(np.isfinite(got))
            assert rel_l2(got, want) < tol, (pos, rel_l2(got, want))
        c, r = dev.read_kv(1, steps - 1)
        cc = ref.cc.reshape(spec.n_layers, spec.ctx_len, spec.kv_lora)[1, steps - 1]
        rc = ref.rc.reshape(spec.n_layers, spec.ctx_len, spec.rope_dim)[1, steps - 1]
        assert rel_l2(c, cc) < tol and rel_l2(r, rc) < tol
    finally:
        dev.free()


# ---- batched prefill (loom_cuda_model_prefill, llama.zig:1698 stepBatch) ----------------

def _kv_rows(dev, spec, n):
    return [dev.read_kv(li, p) for li in range(spec.n_layers) for p in range(n)]


def test_prefill_matches_token_by_token(be):
    """The reference's own invariant (llama.zig:2206 "batched prefill matches
    token-by-token prefill"): the tiny llama's 8-token prompt through the
    batched prefill equals 8 decode steps bit for bit -- the last logits and
    every cache row -- and both continue to the same 16 greedy tokens."""
    spec = tiny_llama(ctx_len=256)
    rng = np.random.default_rng(1)
    prompt = [int(t) for t in rng.integers(1, 32000, size=8)]
    a, b = DeviceModel(spec), DeviceModel(spec)
    try:
        na, la = a.prefill(prompt, 0, logits=True)
        for p, t in enumerate(prompt):
            nb, lb = b.decode(t, p, logits=True)
        assert na == nb
        assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
        for (ka, va), (kb, vb) in zip(_kv_rows(a, spec, 8), _kv_rows(b, spec, 8)):
            assert np.array_equal(ka, kb) and np.array_equal(va, vb)
        ta, tb, pos = na, nb, len(prompt)
        for _ in range(16):
            ta, _ = a.decode(ta, pos)
            tb, _ = b.decode(tb, pos)
            assert ta == tb
            pos += 1
    finally:
        a.free()
        b.free()


def test_prefill_matches_oracle_and_greedy(be, orc):
    """Prefill logits against the oracle fed the same prompt token by token
    (2e-3), then 24 greedy tokens decoded after the prefill equal the
    oracle's."""
    spec = tiny_llama(ctx_len=256)
    rng = np.random.default_rng(5)
    prompt = [int(t) for t in rng.integers(1, 32000, size=12)]
    ref = _runner(spec, orc)
    for p, t in enumerate(prompt):
        want = ref.step(t, p)
    dev = DeviceModel(spec)
    try:
        nxt, got = dev.prefill(prompt, 0, logits=True)
        assert rel_l2(got, want) < TOL
        assert nxt == int(np.argmax(want))
        seq_ref, seq_dev, pos = [int(np.argmax(want))], [nxt], len(prompt)
        for _ in range(24):
            seq_ref.append(int(np.argmax(ref.step(seq_ref[-1], pos))))
            seq_dev.append(dev.decode(seq_dev[-1], pos)[0])
            pos += 1
        assert seq_dev == seq_ref
    finally:
        dev.free()


@pytest.mark.parametrize("arith", ["exact", "fp16"])
def test_prefill_qwen3_shape(be, arith):
    """Qwen3-30B-A3B shape (2 layers, 16 experts, ctx 640) with the
    reference's order (exact_order): 100 prompt tokens through the batched
    prefill -- 50 tokens per expert on average, so the experts run on the
    tensor cores -- against 100 decode steps. Integer-exact tensor cores: bit
    for bit, logits and cache rows; the default fp16 down projection: logits
    within 2e-2 (operand rounding can move an int8 rounding of the next
    layer's activation). Chunked (60 then 40 tokens at position 60) equals one
    batch bit for bit."""
    from loom_b200 import device as D
    spec = qwen3_moe(n_layers=2, ctx_len=640, n_expert=16, vocab=4096)
    rng = np.random.default_rng(11)
    prompt = [int(t) for t in rng.integers(0, spec.vocab, size=100)]
    prev = D.tc_exact(1 if arith == "exact" else 0)
    a, b, c = DeviceModel(spec, exact_order=True), DeviceModel(spec, exact_order=True), DeviceModel(spec, exact_order=True)
    try:
        na, la = a.prefill(prompt, 0, logits=True)
        for p, t in enumerate(prompt):
            nb, lb = b.decode(t, p, logits=True)
        c.prefill(prompt[:60], 0)
        nc, lc = c.prefill(prompt[60:], 60, logits=True)
        assert np.array_equal(la.view(np.uint32), lc.view(np.uint32)) and na == nc
        if arith == "exact":
            assert np.array_equal(la.view(np.uint32), lb.view(np.uint32)) and na == nb
            for (ka, va), (kb, vb) in zip(_kv_rows(a, spec, 100)[::7], _kv_rows(b, spec, 100)[::7]):
                assert np.array_equal(ka, kb) and np.array_equal(va, vb)
        else:
            assert rel_l2(la, lb) < 2e-2, rel_l2(la, lb)
        assert a.error() == 0 and c.error() == 0
    finally:
        D.tc_exact(prev)
        a.free()
        b.free()
        c.free()


def test_prefill_batched_attention_form(be):
    """The default form (ctx 640: the batched prefill attention, fused
    multiply-adds and tree sums, beside the decode path's split attention):
    120 prompt tokens through the prefill against 120 decode steps, logits
    within 2e-2 (rounding differences can move an int8 rounding of a later
    activation), the same greedy token when the top two logits are apart, and
    the cache rows within 2e-3."""
    spec = qwen3_moe(n_layers=2, ctx_len=640, n_expert=16, vocab=4096)
    rng = np.random.default_rng(13)
    prompt = [int(t) for t in rng.integers(0, spec.vocab, size=120)]
    a, b = DeviceModel(spec), DeviceModel(spec)
    try:
        na, la = a.prefill(prompt, 0, logits=True)
        for p, t in enumerate(prompt):
            nb, lb = b.decode(t, p, logits=True)
        assert np.all(np.isfinite(la)) and rel_l2(la, lb) < 2e-2, rel_l2(la, lb)
        top = np.sort(lb)[-2:]
        if top[1] - top[0] > 1e-2 * max(1.0, abs(top[1])):
            assert na == nb
        for (ka, va), (kb, vb) in zip(_kv_rows(a, spec, 120)[::11], _kv_rows(b, spec, 120)[::11]):
            assert rel_l2(ka, kb) < 1e-2 and rel_l2(va, vb) < 1e-2
        assert a.error() == 0
    finally:
        a.free()
        b.free()


# ---- batched decode of many sequences (loom_cuda_model_decode_batch, llama.zig:1939) --------

def test_decode_batch_matches_single_sequences(be):
    """Three sequences of the tiny llama decoded together, one token each per
    call, sequence 2 starting 5 positions later (its earlier cache rows zero,
    as in a fresh single-sequence model): every row's logits equal the same
    sequence decoded alone, bit for bit, over 12 steps, and so does the
    greedy token."""
    spec = tiny_llama(ctx_len=256)
    rng = np.random.default_rng(21)
    off = [0, 0, 5]
    toks = rng.integers(1, 32000, size=(12, 3))
    batch = DeviceModel(spec)
    singles = [DeviceModel(spec) for _ in range(3)]
    try:
        for s in range(12):
            pos = [s + o for o in off]
            nxt, lg = batch.decode_batch(toks[s], pos, logits=True)
            for b in range(3):
                n1, l1 = singles[b].decode(int(toks[s, b]), pos[b], logits=True)
                assert np.array_equal(lg[b].view(np.uint32), l1.view(np.uint32)), (s, b)
                assert int(nxt[b]) == n1
    finally:
        batch.free()
        for m in singles:
            m.free()


def test_decode_batch_qwen3_shape(be):
    """Qwen3 shape (2 layers, 16 experts, ctx 640), 4 sequences at different
    positions: the batched form (per-row attention against each sequence's
    cache, the experts of all rows together) within 2e-2 of each sequence
    decoded alone (the single-sequence path's split attention and fused
    kernels round differently)."""
    spec = qwen3_moe(n_layers=2, ctx_len=640, n_expert=16, vocab=4096)
    rng = np.random.default_rng(22)
    off = [0, 3, 7, 11]
    toks = rng.integers(0, spec.vocab, size=(16, 4))
    batch = DeviceModel(spec)
    singles = [DeviceModel(spec) for _ in range(4)]
    try:
        for s in range(16):
            pos = [s + o for o in off]
            nxt, lg = batch.decode_batch(toks[s], pos, logits=True)
            for b in range(4):
                n1, l1 = singles[b].decode(int(toks[s, b]), pos[b], logits=True)
                assert np.all(np.isfinite(lg[b])) and rel_l2(lg[b], l1) < 2e-2, (s, b, rel_l2(lg[b], l1))
        assert batch.error() == 0
    finally:
        batch.free()
        for m in singles:
            m.free()
