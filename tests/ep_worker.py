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
    t = torch.tensor([worst], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        print(f"EP_MAX_REL_L2 {float(t.item()):.3e}", flush=True)
    dist.destroy_process_group()
    return 0 if float(t.item()) < 1e-5 else 1


if __name__ == "__main__":
    sys.exit(main())
