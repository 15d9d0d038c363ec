"""Worker for the 2-GPU expert-parallel test (launched by torchrun from
tests/test_gpu_ep.py): every rank holds half of each layer's experts; the
NCCL combine must reproduce the unsharded layer that rank 0 also runs."""
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from loom_b200 import backend as B  # noqa: E402
from loom_b200 import device as D  # noqa: E402
from loom_b200.device import DeviceTensor, MoeLayer  # noqa: E402


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    B.init(local)
    D.tc_exact(1)  # integer-exact tensor-core kernels: the sharded layer is compared with tight bounds
    D.ep_init(rank, world, dist)
    ne, k, dim, ffn = 32, 8, 2048, 768
    pg, pd = ffn * dim // 256, dim * ffn // 256
    e0, nl = D.expert_range(ne, rank, world)
    router = DeviceTensor.synth(0, ne * dim, 44, 0.02)
    shard = MoeLayer(dim, ffn, ne, k, DeviceTensor.synth_range(12, e0 * pg, nl * pg, 41),
                     DeviceTensor.synth_range(12, e0 * pg, nl * pg, 42), DeviceTensor.synth_range(14, e0 * pd, nl * pd, 43),
                     router=router, expert0=e0, n_local=nl)
    full = MoeLayer(dim, ffn, ne, k, DeviceTensor.synth(12, ne * pg, 41), DeviceTensor.synth(12, ne * pg, 42),
                    DeviceTensor.synth(14, ne * pd, 43), router=router)
    worst = 0.0
    for T in (1, 5, 40):
        x = torch.randn((T, dim), device="cuda", generator=torch.Generator("cuda").manual_seed(T))
        res = torch.randn((T, dim), device="cuda", generator=torch.Generator("cuda").manual_seed(100 + T))
        out = torch.empty((T, dim), device="cuda")
        shard.forward(x, out, residual=res)
        want = torch.empty((T, dim), device="cuda")
        full.desc()  # the unsharded layer runs without the collective (its range is all experts)
        full.forward(x, want, residual=res)
        torch.cuda.synchronize()
        err = float((out - want).norm() / want.norm())
        worst = max(worst, err)
    from loom_b200 import _lib
    lib = _lib.lib()
    assert lib.loom_cuda_ep_error() == 0
    # the whole-token model, experts sharded, against the same model unsharded (rank 0)
    from loom_b200.model import DeviceModel, qwen3_moe
    spec = qwen3_moe(n_layers=2, ctx_len=640, n_expert=16, vocab=4096)
    sharded = DeviceModel(spec, expert_shard=D.expert_range(spec.n_expert, rank, world))
    single = DeviceModel(spec) if rank == 0 else None
    mworst = 0.0
    for pos in range(24):
        tok = (37 * pos + 11) % spec.vocab
        nxt, lg = sharded.decode(tok, pos, logits=True)
        if single is not None:
            n1, l1 = single.decode(tok, pos, logits=True)
            mworst = max(mworst, float(np.linalg.norm(lg - l1) / np.linalg.norm(l1)))
    assert lib.loom_cuda_ep_error() == 0
    t = torch.tensor([worst, mworst], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        print(f"EP_MAX_REL_L2 {float(t[0].item()):.3e} MODEL_REL_L2 {float(t[1].item()):.3e} "
              f"PEER_COMBINE {lib.loom_cuda_ep_peer_combine()}", flush=True)
    dist.destroy_process_group()
    return 0 if float(t[0].item()) < 1e-5 and float(t[1].item()) < 2e-2 else 1


if __name__ == "__main__":
    sys.exit(main())
