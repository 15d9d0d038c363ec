"""CPU checks of the oracle's token step (or_llama_step, llama.zig:1111-1228)
against an independent numpy restatement, on the tiny llama config (BASELINE
config 1: dense Q4_0, ropeNorm) and on a reduced Qwen3-MoE shape (QK-norm,
ropeNeox, GQA 8:1, routed MoE FFN)."""
import numpy as np
import pytest

from loom_b200.model import qwen3_moe, tiny_llama
from tests.conftest import rel_l2
from tests.modelref import host_tensors, numpy_step


def _compare(spec, orc, steps, tol):
    from oracle.oracle import LlamaRunner
    T = host_tensors(spec, orc)
    run = LlamaRunner(spec, T)
    kvd = spec.n_kv_heads * spec.head_dim
    kc = np.zeros((spec.n_layers, spec.ctx_len, kvd), np.float32)
    vc = np.zeros_like(kc)
    rng = np.random.default_rng(5)
    tok = int(rng.integers(1, spec.vocab))
    for pos in range(steps):
        got = run.step(tok, pos)
        want = numpy_step(spec, T, orc, kc, vc, tok, pos)
        assert np.all(np.isfinite(got))
        assert rel_l2(got, want) < tol, (pos, rel_l2(got, want))
        ck = run.kc.reshape(spec.n_layers, spec.ctx_len, kvd)[:, pos]
        assert rel_l2(ck, kc[:, pos]) < tol
        tok = int(np.argmax(got))


def test_oracle_step_tiny_llama(orc):
    _compare(tiny_llama(ctx_len=16), orc, steps=10, tol=2e-3)


def test_oracle_step_qwen3_moe_reduced(orc):
    _compare(qwen3_moe(n_layers=2, ctx_len=16, n_expert=16, vocab=1024), orc, steps=6, tol=2e-3)


def test_oracle_rejects_bad_token_and_position(orc):
    from oracle.oracle import LlamaRunner
    spec = tiny_llama(ctx_len=4)
    spec.n_layers = 1
    run = LlamaRunner(spec, host_tensors(spec, orc))
    with pytest.raises(AssertionError):
        run.step(spec.vocab, 0)  # llama.zig:1121 TokenOutOfRange
    with pytest.raises(AssertionError):
        run.step(1, spec.ctx_len)


def _compare_ds(spec, orc, steps, tol):
    from oracle.oracle import DeepseekRunner
    from tests.modelref import numpy_ds_step
    T = host_tensors(spec, orc)
    run = DeepseekRunner(spec, T)
    cc = np.zeros((spec.n_layers, spec.ctx_len, spec.kv_lora), np.float32)
    rc = np.zeros((spec.n_layers, spec.ctx_len, spec.rope_dim), np.float32)
    rng = np.random.default_rng(9)
    for pos in range(steps):
        tok = int(rng.integers(0, spec.vocab))
        got = run.step(tok, pos)
        want = numpy_ds_step(spec, T, orc, cc, rc, tok, pos)
        assert np.all(np.isfinite(got))
        assert rel_l2(got, want) < tol, (pos, rel_l2(got, want))
        oc = run.cc.reshape(spec.n_layers, spec.ctx_len, spec.kv_lora)[:, pos]
        assert rel_l2(oc, cc[:, pos]) < tol


def test_oracle_deepseek_v2_lite_reduced(orc):
    """MLA without q_lora, dense first layer, routed layer with shared experts."""
    from loom_b200.model import deepseek_v2_lite
    _compare_ds(deepseek_v2_lite(n_layers=2, ctx_len=8, n_expert=8, vocab=512), orc, steps=5, tol=2e-3)


def test_oracle_deepseek_v3_shape_reduced(orc):
    """MLA with q_lora, sigmoid + bias gating, grouped top-k, one shared expert."""
    from loom_b200.model import deepseek_v3
    spec = deepseek_v3(n_layers=2, ctx_len=8, n_expert=16, dim=1024, n_heads=8, vocab=512, n_dense=1)
    spec.n_used, spec.n_group, spec.topk_group = 4, 4, 2
    _compare_ds(spec, orc, steps=4, tol=2e-3)
