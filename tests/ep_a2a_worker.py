"""Worker for the 2-GPU all-to-all expert-parallel test (launched by torchrun
from tests/test_gpu_ep.py): each rank holds its contiguous half of the
experts and its own tokens (different counts per rank, one round with no
tokens on one rank), in both exchange forms (counted, and fixed capacity with
and without unused entries); the all-to-all layer must equal, bit for bit,
the unsharded layer each rank also runs on its own tokens."""
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
    ne, k, dim, ffn, sffn = 64, 6, 2048, 1408, 1408
    pg, pd = ffn * dim // 256, dim * ffn // 32
    e0, nl = D.expert_range(ne, rank, world)
    router = DeviceTensor.synth(0, ne * dim, 54, 0.02)
    shexp = (DeviceTensor.synth(12, sffn * dim // 256, 55), DeviceTensor.synth(12, sffn * dim // 256, 56),
             DeviceTensor.synth(8, dim * sffn // 32, 57))
    shard = MoeLayer(dim, ffn, ne, k, DeviceTensor.synth_range(12, e0 * pg, nl * pg, 51),
                     DeviceTensor.synth_range(12, e0 * pg, nl * pg, 52), DeviceTensor.synth_range(8, e0 * pd, nl * pd, 53),
                     router=router, shexp=shexp, shexp_ffn=sffn, expert0=e0, n_local=nl)
    full = MoeLayer(dim, ffn, ne, k, DeviceTensor.synth(12, ne * pg, 51), DeviceTensor.synth(12, ne * pg, 52),
                    DeviceTensor.synth(8, ne * pd, 53), router=router, shexp=shexp, shexp_ffn=sffn)
    ok = 1
    for rnd, (counts, t_cap) in enumerate([((5, 3), 0), ((1, 1), 0), ((40, 0), 0), ((0, 17), 0),
                                            ((5, 3), 5), ((1, 1), 1), ((2, 0), 4), ((0, 3), 3)]):
        T = counts[rank % 2]
        g = torch.Generator("cuda").manual_seed(1000 * rnd + rank)
        x = torch.randn((T, dim), device="cuda", generator=g)
        res = torch.randn((T, dim), device="cuda", generator=g)
        out = torch.full((T, dim), float("nan"), device="cuda")
        ids = torch.zeros((T, k), dtype=torch.int32, device="cuda")
        shard.forward_a2a(x, out, residual=res, ids=ids, t_cap=t_cap)
        if T:
            want = torch.empty((T, dim), device="cuda")
            wids = torch.zeros((T, k), dtype=torch.int32, device="cuda")
            full.forward(x, want, residual=res, ids=wids)
            torch.cuda.synchronize()
            same = np.array_equal(out.cpu().numpy().view(np.uint32), want.cpu().numpy().view(np.uint32))
            same = same and np.array_equal(ids.cpu().numpy(), wids.cpu().numpy())
            if not same:
                print(f"rank {rank} round {rnd}: max diff {float((out - want).abs().max())}", flush=True)
                ok = 0
    # a collective that one rank cannot complete must not leave the other blocked:
    # (a) rank 0 has more tokens than the capacity: it takes part, sends none of its
    #     rows and declines; rank 1's tokens are still served, bit for bit;
    # (b) the ranks pass different capacities: both decline, neither exchanges
    import ctypes as C
    from loom_b200 import _lib
    from loom_b200.device import _ptr, _st
    L = _lib.lib()
    for name, counts, caps in [("over", (6, 3), (4, 4)), ("mismatch", (2, 2), (6, 7))]:
        T = counts[rank % 2]
        g = torch.Generator("cuda").manual_seed(77 + rank)
        x = torch.randn((T, dim), device="cuda", generator=g)
        res = torch.randn((T, dim), device="cuda", generator=g)
        out = torch.full((T, dim), float("nan"), device="cuda")
        d = shard.desc()
        rc = L.loom_cuda_ep_a2a_forward_cap(C.byref(d), _ptr(x), T, caps[rank % 2], _ptr(out), _ptr(res), None,
                                            None, _st(None))
        want_rc = (_lib.DECLINED if rank == 0 else _lib.OK) if name == "over" else _lib.DECLINED
        if rc != want_rc:
            print(f"rank {rank} {name}: rc {rc}, expected {want_rc}", flush=True)
            ok = 0
        elif rc == _lib.OK:
            want = torch.empty((T, dim), device="cuda")
            full.forward(x, want, residual=res)
            torch.cuda.synchronize()
            if not np.array_equal(out.cpu().numpy().view(np.uint32), want.cpu().numpy().view(np.uint32)):
                print(f"rank {rank} {name}: served tokens differ", flush=True)
                ok = 0
    t = torch.tensor([ok], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    if rank == 0:
        print(f"A2A_BITEXACT {int(t.item())}", flush=True)
    dist.destroy_process_group()
    return 0 if int(t.item()) == 1 else 1


if __name__ == "__main__":
    sys.exit(main())
