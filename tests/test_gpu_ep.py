"""Expert parallelism on 2 GPUs: two processes (torchrun, NCCL), each holding
half of the experts; the combined output must equal the unsharded layer
(within 1e-5 relative L2: only the order of the partial sums changes)."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("combine", ["peer", "nccl"])
def test_two_rank_expert_parallel_layer(combine):
    """Sharded layers (T = 1, 5 through the peer-memory combine unless NCCL is
    forced; T = 40 through NCCL) against the unsharded layer, and the
    whole-token model sharded over 2 GPUs against the same model on one."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    if combine == "nccl":
        env["LOOM_CUDA_EP_NCCL"] = "1"
    p = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
                        "--master-addr", "127.0.0.1", "--master-port", str(29600 + os.getpid() % 300),
                        os.path.join(ROOT, "tests", "ep_worker.py")], env=env, capture_output=True, text=True,
                       timeout=600)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-3000:]
    assert "EP_MAX_REL_L2" in p.stdout
    assert f"PEER_COMBINE {1 if combine == 'peer' else 0}" in p.stdout


@pytest.mark.parametrize("cfg", [
    dict(ne=128, k=8, dim=2048, ffn=768, gt=12, dt=14),                                              # Qwen3
    dict(ne=64, k=6, dim=2048, ffn=1408, gt=12, dt=8, shared=2816),                                   # V2-Lite
    dict(ne=256, k=8, dim=1024, ffn=512, gt=12, dt=12, shared=512, gating=2, scale=2.5, bias=True,
         groups=(8, 4)),                                                                             # V3-like
], ids=["qwen3", "v2lite", "v3grouped"])
@pytest.mark.parametrize("T", [0, 1, 7, 64])
@pytest.mark.parametrize("mode", [0, 1, 3], ids=["auto", "slot", "mma"])
@pytest.mark.parametrize("cap", [0, 1, 5], ids=["counted", "cap_exact", "cap_padded"])
def test_a2a_single_rank_bitexact(be, orc, cfg, T, mode, cap):
    """The all-to-all layer as one rank (every row goes to itself through the
    pack, the self copy, the per-row expert run and the ordered combine) is
    bit-identical to the ordinary layer, shared expert and groups included;
    so is the fixed-capacity form, with a run exactly T*n_used long and one
    padded with unused entries."""
    from tests.test_gpu_moe import _layer_case
    from tests.conftest import bits
    import numpy as np
    L = _layer_case(orc, 21, **cfg)
    dim, k = cfg["dim"], cfg["k"]
    x = torch.from_numpy(orc.synth(0, max(T, 1) * dim, seed=22).reshape(max(T, 1), dim)[:T].copy()).cuda()
    res = torch.randn(T, dim, device="cuda")
    want = torch.full((T, dim), float("nan"), device="cuda")
    wids = torch.zeros((T, k), dtype=torch.int32, device="cuda")
    if T:
        L.forward(x, want, residual=res, ids=wids)
    got = torch.full((T, dim), float("nan"), device="cuda")
    gids = torch.zeros((T, k), dtype=torch.int32, device="cuda")
    from loom_b200 import device as D
    prev = D.force_generic(mode)  # how the arriving rows run: batch / slot kernels / tensor cores
    prev_x = D.tc_exact(1)  # the integer-exact tensor-core form: bit-comparable
    try:
        L.forward_a2a(x, got, residual=res, ids=gids, t_cap=0 if cap == 0 else max(T, 1) + (cap - 1))
    finally:
        D.force_generic(prev)
        D.tc_exact(prev_x)
    torch.cuda.synchronize()
    assert np.array_equal(gids.cpu().numpy(), wids.cpu().numpy())
    assert np.array_equal(bits(got.cpu().numpy()), bits(want.cpu().numpy()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_all_to_all_layer():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    p = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
                        "--master-addr", "127.0.0.1", "--master-port", str(29650 + os.getpid() % 300),
                        os.path.join(ROOT, "tests", "ep_a2a_worker.py")], env=env, capture_output=True, text=True,
                       timeout=600)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-3000:]
    assert "A2A_BITEXACT 1" in p.stdout
