"""Expert-parallel decomposition on CPU ranks (gloo, world size 2): each rank
runs only its contiguous expert shard of the routed layer (the same selection
on every rank), the partial outputs are summed with an all-reduce, and the sum
equals the unsharded layer computed by the CPU oracle."""
import os

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from loom_b200.device import expert_range


def test_expert_ranges_partition_the_experts():
    for ne in (64, 128, 256):
        for world in (1, 2, 3, 4, 8):
            got = []
            for r in range(world):
                e0, n = expert_range(ne, r, world)
                got.extend(range(e0, e0 + n))
            assert got == list(range(ne))


def _worker(rank, world, port, q):
    import torch
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as orc
        ne, k, dim, ffn = 16, 4, 256, 256
        g = orc.synth(12, ne * ffn * dim // 256, 1)
        u = orc.synth(12, ne * ffn * dim // 256, 2)
        d = orc.synth(14, ne * dim * ffn // 256, 3)
        x = orc.synth(0, dim, 4)
        logits = orc.synth(0, ne, 5)
        ids, gates = orc.route(logits, k)  # replicated routing
        e0, n = expert_range(ne, rank, world)
        gp, dp = ffn * orc.row_bytes(12, dim), dim * orc.row_bytes(14, ffn)
        local = [dict(gate_type=12, up_type=12, down_type=14, gate=g[e * gp:(e + 1) * gp], up=u[e * gp:(e + 1) * gp],
                      down=d[e * dp:(e + 1) * dp], weight=float(w), ffn=ffn)
                 for e, w in zip(ids, gates) if e0 <= e < e0 + n]
        part = orc.moe_ffn_block(x, local, dim) if local else np.zeros(dim, np.float32)
        t = torch.from_numpy(part.copy())
        dist.all_reduce(t)
        if rank == 0:
            want = orc.moe_ffn_routed(x, logits, (12, g), (12, u), (14, d), ffn, k)
            q.put(float(np.linalg.norm(t.numpy() - want) / np.linalg.norm(want)))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_sharded_layer_sums_to_unsharded_on_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(90)
    assert all(p.exitcode == 0 for p in ps)
    assert q.get(timeout=5) < 1e-5


def _a2a_worker(rank, world, port, q):
    """The all-to-all decomposition on gloo ranks, restated with the oracle:
    each rank routes its own tokens, sends each routed row (a stable
    partition by owner rank) to the expert's owner with all_to_all_single,
    the owner applies that one expert with weight 1, the rows come back in the
    same order and the home rank combines them in selection order. The result
    must equal the oracle's unsharded routed block bit for bit."""
    import torch
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as orc
        ne, k, dim, ffn = 16, 4, 256, 256
        g = orc.synth(12, ne * ffn * dim // 256, 1)
        u = orc.synth(12, ne * ffn * dim // 256, 2)
        d = orc.synth(14, ne * dim * ffn // 256, 3)
        gp, dp = ffn * orc.row_bytes(12, dim), dim * orc.row_bytes(14, ffn)
        plane = lambda e, w: dict(gate_type=12, up_type=12, down_type=14, gate=g[e * gp:(e + 1) * gp],  # noqa: E731
                                  up=u[e * gp:(e + 1) * gp], down=d[e * dp:(e + 1) * dp], weight=w, ffn=ffn)
        T = 3 if rank == 0 else 2
        xs = orc.synth(0, T * dim, 10 + rank).reshape(T, dim)
        logits = orc.synth(0, T * ne, 20 + rank).reshape(T, ne)
        routes = [orc.route(logits[t], k) for t in range(T)]
        owner = lambda e: next(r for r in range(world) if expert_range(ne, r, world)[0] <= e  # noqa: E731
                               < sum(expert_range(ne, r, world)))
        slots = [(t, int(e)) for t in range(T) for e in routes[t][0]]
        order = sorted(range(len(slots)), key=lambda i: (owner(slots[i][1]), i))  # stable partition
        pos = {i: p for p, i in enumerate(order)}
        scnt = [sum(1 for i in order if owner(slots[i][1]) == r) for r in range(world)]
        rcnt_t = torch.zeros(world, dtype=torch.int64)
        dist.all_to_all_single(rcnt_t, torch.tensor(scnt, dtype=torch.int64))
        rcnt = rcnt_t.tolist()
        send = torch.from_numpy(np.stack([np.append(xs[slots[i][0]], np.float32(slots[i][1])) for i in order]))
        recv = torch.empty((sum(rcnt), dim + 1))
        dist.all_to_all_single(recv, send, rcnt, scnt)
        ys = torch.from_numpy(np.stack([orc.moe_ffn_block(r[:dim].numpy(), [plane(int(r[dim]), 1.0)], dim)
                                        for r in recv])) if sum(rcnt) else torch.empty((0, dim))
        back = torch.empty((len(slots), dim))
        dist.all_to_all_single(back, ys.float(), scnt, rcnt)
        ok = True
        for t in range(T):
            acc = np.zeros(dim, np.float32)
            for kk in range(k):
                acc = (acc + np.float32(routes[t][1][kk]) * back[pos[t * k + kk]].numpy()).astype(np.float32)
            want = orc.moe_ffn_routed(xs[t], logits[t], (12, g), (12, u), (14, d), ffn, k)
            ok &= np.array_equal(acc.view(np.uint32), want.view(np.uint32))
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_all_to_all_decomposition_on_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 28500 + os.getpid() % 1000
    ps = [ctx.Process(target=_a2a_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(90)
    assert all(p.exitcode == 0 for p in ps)
    res = dict(q.get(timeout=5) for _ in range(2))
    assert res == {0: True, 1: True}
