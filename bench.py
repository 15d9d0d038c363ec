"""Benchmark of the B200 CUDA backend on BASELINE's headline metric:
decode tok/s + expert-matvec HBM GB/s at Qwen3-30B-A3B Q4_K.

Default workload (--workload model; one "step"): one decode token at batch 1
through the FULL Qwen3-30B-A3B-shaped model (48 layers,
hidden 2048, 32/4 heads of 128, QK-RMSNorm, RoPE NEOX, 128 experts top-8 of
768, vocab 151936, Q4_K_M mix) at position 2047 of a 2048-token context whose
KV cache the run first fills by decoding: embedding, per layer RMSNorm +
q/k/v + QK-norm + RoPE + KV append + attention over 2048 positions + output
projection + MoE FFN, final norm, lm_head and argmax (loom_cuda_model_*).
~2.5 GB is read per token, far more than the 126 MB L2.
  value      tok/s of loom_cuda_model_step replayed from a CUDA graph
  e2e        loom_cuda_model_decode: host token in, host token out (one
             8-byte H2D and one 4-byte D2H copy per step), wall clock
  roofline   algorithmic bytes of the token (every weight byte read once,
             8 experts per layer, the KV cache rows, the head) / step time
  moe_stack  the MoE-only measurement below (expert-matvec GB/s)
  cpu_baseline  the oracle's token step (oracle/ restatement of llama.zig
             step) on sampled layers of the same model, extrapolated
With torchrun (N > 1) the model runs expert-parallel: experts of every layer
sharded contiguously over the ranks, attention/norms/router/head replicated,
the MoE partial outputs summed by an NCCL all-reduce (strong scaling: the
same token on every rank).

--workload moe (one "step"): one decode token (T=1 by default, --tokens T for a
batch) through the 48 MoE layers of a Qwen3-30B-A3B-shaped model with
distinct random-init weights per layer: router f32 [128x2048] -> softmax top-8
with renorm -> gate/up Q4_K [768x2048] + SwiGLU -> down Q6_K [2048x768] ->
weighted combine -> residual add. Attention is outside this backend's hot
path and not timed. Weights come from the seeded generator (synthetic: no
checkpoint or dataset is available offline); 48 distinct layers touch
~1.2 GB per token, far more than the 126 MB L2, so no flush is needed.

  value      tok/s of the device-resident path, inputs already in HBM, max
             over ranks. T=1 unsharded (the default): the persistent stack
             kernel, one launch per token for all 48 layers
             (loom_cuda_stack_forward); otherwise the per-layer kernels
             (loom_cuda_moe_forward) replayed from a CUDA graph
  e2e        the same token through the reference-facing seam calls with
             HOST buffers (loom_cuda_matvec for the router +
             loom_cuda_moe_ffn_routed per layer, as deepseek.zig:1334-1380
             drives its backend)
  e2e_device the device-resident path with the token copied in from pinned
             host memory and the output read back every step
  roofline   HBM bytes the layer must move (router + the distinct selected
             experts' planes + activations) / measured layer time
  cpu_baseline  the CPU restatement of the reference kernels (oracle/) on
             the host cores, on sampled layers of the same model

--impl reference times the reference's CPU path (the oracle restatement,
Zig being unavailable) on the same workload and prints the same JSON line.
Multi-GPU (torchrun): each rank runs an independent replica of the decode
stream (weak scaling); expert-parallel sharding is a separate mode.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

DIM, FFN, NE, NK, LAYERS = 2048, 768, 128, 8, 48
LAYERS_DEFAULT = LAYERS
Q4K, Q6K, F32 = 12, 14, 0
METRIC = "decode tok/s (Qwen3-30B-A3B MoE stack, Q4_K/Q6_K, T=1)"


def layer_bytes_model(T_ids: np.ndarray, e0: int = 0, nl: int = NE) -> int:
    """Algorithmic HBM bytes of one layer: router + every distinct selected
    expert's gate/up/down plane once (those held in [e0, e0+nl)) + activations."""
    plane = 2 * FFN * (DIM // 256) * 144 + DIM * (FFN // 256) * 210
    u = np.unique(T_ids)
    n_distinct = int(np.sum((u >= e0) & (u < e0 + nl)))
    T = T_ids.shape[0]
    return NE * DIM * 4 + n_distinct * plane + T * DIM * 4 * 3


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """Samples the SM clock and the throttle reasons during the timed region
    (NVML every 2 ms; nvidia-smi every 100 ms when NVML is unavailable)."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4}

    def __init__(self, gpu: int):
        self.gpu, self.samples, self.stop = gpu, [], threading.Event()

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self.max = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)

            def poll():
                while not self.stop.is_set():
                    self.samples.append((pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
                                         pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)))
                    time.sleep(0.002)
            self.t = threading.Thread(target=poll, daemon=True)
            self.t.start()
        except Exception:  # noqa: BLE001 -- clocks are reported, never required
            self.max = None
        return self

    def __exit__(self, *a):
        self.stop.set()
        if hasattr(self, "t"):
            self.t.join(timeout=1)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max, "reasons": ["unsampled"]}
        reasons = sorted({n for _, r in self.samples for n, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(s for s, _ in self.samples), "sm_max_mhz": self.max, "reasons": reasons,
                "samples": len(self.samples)}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


# ---- CPU reference path (the oracle restatement of the reference kernels) ----------

def cpu_time_layers(n_layers_sample: int, threads: int, reps: int, seed_base: int = 1000):
    """Median seconds per MoE layer of the CPU restatement over sampled layers."""
    from oracle import oracle as orc
    rng = np.random.default_rng(0)
    layers = []
    for l in range(n_layers_sample):
        s = seed_base + l
        g = orc.synth(Q4K, NE * FFN * DIM // 256, s * 10 + 1)
        u = orc.synth(Q4K, NE * FFN * DIM // 256, s * 10 + 2)
        d = orc.synth(Q6K, NE * DIM * FFN // 256, s * 10 + 3)
        r = orc.synth(F32, NE * DIM, s * 10 + 4, sigma=0.02)
        layers.append((g, u, d, r))
    x = rng.standard_normal((1, DIM)).astype(np.float32)
    if threads > 1:
        orc.parallel_begin(threads)
    times = []
    try:
        for rep in range(reps + 1):
            t0 = time.perf_counter()
            for (g, u, d, r) in layers:
                out, _ = orc.moe_layer(x, r, (Q4K, g), (Q4K, u), (Q6K, d), FFN, NE, NK)
                x = x + out
            dt = (time.perf_counter() - t0) / len(layers)
            if rep:
                times.append(dt)
    finally:
        if threads > 1:
            orc.parallel_end()
    return statistics.median(times)


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    sample_layers = 4
    # warmup + steps: each step is one token through `sample_layers` layers,
    # extrapolated to the 48-layer stack
    per_layer = cpu_time_layers(sample_layers, threads, max(args.steps, 1))
    tok_s = 1.0 / (per_layer * LAYERS)
    line = {"impl": "reference", "metric": METRIC, "value": round(tok_s, 3), "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_layer * LAYERS * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8xq4/q6 (f32 accum)",
            "data": "synthetic (seeded generator), random-init weights",
            "config": {"workload": "qwen3-30b-a3b moe stack decode, T=1, 48 layers", "tokens": 1,
                       "layers": LAYERS, "n_expert": NE, "n_used": NK, "dim": DIM, "ffn": FFN,
                       "parallelism": "host threads"},
            "cpu_baseline": {"value": round(tok_s, 3), "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": f"1 token x {sample_layers} sampled layers per step, extrapolated to {LAYERS}"},
            "e2e": {"value": round(tok_s, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---- GPU path ----------------------------------------------------------------------

def build_model(T: int, seed_base: int = 1000, e0: int = 0, nl: int = NE):
    """The 48 layers; with expert parallelism only experts [e0, e0+nl) of each
    layer are generated (the same bytes the full model holds there)."""
    from loom_b200.device import DeviceTensor, MoeLayer
    pg, pd = FFN * DIM // 256, DIM * FFN // 256  # blocks per expert plane
    layers = []
    for l in range(LAYERS):
        s = seed_base + l
        layers.append(MoeLayer(
            DIM, FFN, NE, NK,
            gate=DeviceTensor.synth_range(Q4K, e0 * pg, nl * pg, s * 10 + 1),
            up=DeviceTensor.synth_range(Q4K, e0 * pg, nl * pg, s * 10 + 2),
            down=DeviceTensor.synth_range(Q6K, e0 * pd, nl * pd, s * 10 + 3),
            router=DeviceTensor.synth(F32, NE * DIM, s * 10 + 4, sigma=0.02),
            expert0=e0, n_local=nl))
    return layers


def run_gpu(args, emit=True):
    import torch
    import torch.distributed as dist
    from loom_b200 import backend as B
    from loom_b200 import device as D

    rank, world, local = dist_env()
    if world > 1 and not dist.is_initialized():
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    B.init(local)
    T = args.tokens
    ep = args.ep and world > 1
    a2a = ep and args.ep_mode in ("a2a", "a2a-counted")
    a2a_cap = T if args.ep_mode == "a2a" else 0  # fixed-capacity runs: every rank decodes T tokens
    ex0, nloc = D.expert_range(NE, rank, world) if ep else (0, NE)
    if ep:
        D.ep_init(rank, world, dist)
    layers = build_model(T, e0=ex0, nl=nloc)
    for l in range(LAYERS - 1):
        layers[l].next_router = layers[l + 1].router  # prefetch hint
    # size the scratch once for decode and prefill: graphs keep the pointers they captured
    D.reserve(max(T, args.prefill_tokens if not ep else 0), DIM, FFN, NE, NK)
    descs = [L.desc() for L in layers]
    stream = torch.cuda.Stream()
    # replicas decode independent streams; expert-parallel ranks share one stream
    # all-to-all ranks own different tokens (token-sharded attention)
    x0 = torch.from_numpy(np.random.default_rng(0 if ep and not a2a else rank).standard_normal((T, DIM))
                          .astype(np.float32)).cuda()
    bufs = [torch.empty((T, DIM), device="cuda") for _ in range(2)]
    ids = torch.zeros((LAYERS, T, NK), dtype=torch.int32, device="cuda")

    stack = None
    engine = args.engine
    if engine == "auto":
        engine = "stack" if T == 1 and not ep else "layers"
    if engine == "stack":
        if T != 1 or ep:
            raise SystemExit("--engine stack runs the T=1 decode of unsharded layers")
        stack = D.Stack(layers)

    def step(sh):
        if stack is not None:
            stack.forward(x0, bufs[(LAYERS - 1) % 2], ids, stream=sh)
            return
        cur = x0
        for l, L in enumerate(layers):
            nxt = bufs[l % 2]
            if a2a:
                L.forward_a2a(cur, nxt, residual=cur, ids=ids[l], stream=sh, t_cap=a2a_cap, desc=descs[l])
            else:
                L.forward(cur, nxt, residual=cur, ids=ids[l], stream=sh, desc=descs[l])
            cur = nxt

    with torch.cuda.stream(stream):
        step(stream.cuda_stream)  # sizes all scratch before capture
    torch.cuda.synchronize()
    k0 = B.kernelLaunches()
    if a2a and not a2a_cap:  # the receive counts go to the host every layer: no graph, eager launches
        class _Eager:
            def replay(self):
                step(stream.cuda_stream)
        g = _Eager()
        with torch.cuda.stream(stream):
            g.replay()
        torch.cuda.synchronize()
    else:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step(torch.cuda.current_stream().cuda_stream)
    launches_per_step = B.kernelLaunches() - k0
    with torch.cuda.stream(stream):  # replay, events and timing all on the launching stream
        for _ in range(args.warmup):
            g.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with Clocks(local) as ck:
            torch.cuda.synchronize()
            e0.record(stream)
            for _ in range(args.steps):
                g.replay()
            e1.record(stream)
            torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    if stack is not None:
        assert stack.error() == 0, "stack kernel grid barrier timed out"
    phases = None
    if args.trace:
        phases = trace_phases(D, step, stream, torch) if stack is None else trace_stack(stack, step, stream, torch)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    ids_np = ids.cpu().numpy()
    if ep:  # this rank's bytes: router + its own selected experts + activations
        bytes_step = sum(layer_bytes_model(ids_np[l].reshape(-1), ex0, nloc) for l in range(LAYERS))
    else:
        bytes_step = sum(layer_bytes_model(ids_np[l].reshape(-1)) for l in range(LAYERS))
    achieved = bytes_step / (ms * 1e-3) / 1e9
    # DRAM bytes (read + write) per layer of k_stack from one ncu capture of a
    # 4-layer launch (dram__bytes_read.sum 102,891,776 + dram__bytes_write.sum
    # 9,694,464), scaled by layers: traffic grows in proportion to the layers
    traffic = (102891776 + 9694464) * LAYERS // 4 if stack is not None else None
    peak, peak_kind = peaks()
    value = (T if ep and not a2a else world * T) / (ms * 1e-3)

    # e2e through the seam with host buffers
    e2e = None
    prefill = batch = None
    if args.prefill_tokens > 0 and not ep:
        prefill = run_prefill(args, layers, stream, torch, D)
        if args.batch_tokens > 0:
            batch = run_prefill(args, layers, stream, torch, D, T=args.batch_tokens,
                                label=f"decode batch {args.batch_tokens} (one step of {args.batch_tokens} streams)")
            btc = run_prefill(args, layers, stream, torch, D, T=args.batch_tokens, force_tc=True, with_exact=False,
                              label="the same step forced onto the tensor-core kernels")
            batch["tensor_cores"] = {k: btc[k] for k in ("workload", "value", "unit", "ms_per_step", "engine")}
    e2e_device = None
    if args.e2e_layers > 0 and not ep:
        e2e = run_e2e(args, B)
    if ep or stack is not None:
        e2e_device = run_e2e_device(args, g, stream, x0, bufs[(LAYERS - 1) % 2], torch, dist, world,
                                    job_tokens=T if ep and not a2a else world * T)
        if ep:
            e2e = e2e_device

    if rank != 0:
        return
    cpu = None
    if not args.no_cpu:
        threads = os.cpu_count() or 1
        per_layer = cpu_time_layers(2, threads, 3)
        cpu = {"value": round(1.0 / (per_layer * LAYERS), 3), "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"1 token x 2 sampled layers x 3 reps, extrapolated to {LAYERS} layers"}
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "strong" if ep and not a2a else "weak",
        "vs_baseline": None, "dtype": "int8xq4/q6 (f32 accum)", "data": "synthetic (seeded generator), random-init weights",
        "config": {"workload": f"qwen3-30b-a3b moe stack decode, T={T}, {LAYERS} layers", "tokens": T,
                   "layers": LAYERS, "n_expert": NE, "n_used": NK, "dim": DIM, "ffn": FFN,
                   "parallelism": (f"ep{world} (experts sharded, tokens sharded, NCCL all-to-all dispatch and "
                                   f"combine)" if a2a else
                                   f"ep{world} (experts sharded, NCCL all-reduce combine)" if ep else
                                   f"replicas x{world}" if world > 1 else "1 gpu"),
                   "engine": engine,
                   **({"a2a_exchange": "fixed capacity (T*n_used rows per rank), graph-captured" if a2a_cap else
                       "counted (host sync per layer)"} if a2a else {}),
                   "l2": "inputs > L2 (48 distinct layers, ~1.2 GB touched per token)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "kernel": ("k_stack: every layer's router GEMV, route, gate/up, down and combine in one "
                                "persistent launch" if stack is not None else
                                "moe layer (router gemv + route + gate/up + down/combine)"),
                     "peak_kind": peak_kind, "bytes_per_step": bytes_step},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": ck.summary(),
    }
    if phases:
        line["phase_us"] = phases
    if e2e:
        line["e2e"] = e2e
    if e2e_device and e2e_device is not e2e:
        line["e2e_device"] = e2e_device
    if prefill:
        line["prefill"] = prefill
    if batch:
        line["batch"] = batch
    if cpu:
        line["cpu_baseline"] = cpu
    if emit:
        print(json.dumps(line), flush=True)
    if stack is not None:
        stack.free()
    for L in layers:
        for t in (L.gate, L.up, L.down, L.router):
            t.free()
    return line


def trace_stack(stack, step, stream, torch):
    """One extra traced launch of the stack kernel: per layer, the mean time
    from the layer's start to each phase point, in microseconds."""
    stack.trace_enable()
    with torch.cuda.stream(stream):
        step(stream.cuda_stream)
    tr = stack.trace_read().astype(np.float64)
    rel = tr[1:] - tr[1:, :1]
    names = ["start", "router_rows_done", "unused", "route_done", "gateup_done",
             "unused", "act_quantized", "down_done", "gateup_half2_landed", "gateup_tiles_landed",
             "down_tiles_landed"]
    out = {n: round(float(np.mean(rel[:, i])) / 1e3, 2) for i, n in enumerate(names) if i and n != "unused"}
    out["worst_layer_total"] = round(float(np.max(np.diff(tr[:, 0]))) / 1e3, 2)
    out["layer_total"] = round(float(np.mean(np.diff(tr[:, 0]))) / 1e3, 2)
    sec = ["p1_load", "router_dot", "logits_wait", "route", "stage_issue_w0", "gateup_tiles_wait", "gateup_compute",
           "unused", "act_wait", "act_quant", "down_tiles_wait", "down_compute", "unused2", "gateup_dots_w0", "act_store_w0", "spare"]
    cyc = tr[1:, 12:].reshape(-1, 16, 2)
    G = torch.cuda.get_device_properties(0).multi_processor_count
    out["cycles_max_mean"] = {n: [int(np.mean(cyc[:, i, 0])), int(np.mean(cyc[:, i, 1]) / G)] for i, n in enumerate(sec)}
    return out


def trace_phases(D, step, stream, torch):
    """One extra replay of a separately captured, traced graph: per decode
    kernel the mean span (first CTA start to last CTA end) and the mean gap
    between consecutive kernels, in microseconds (not part of the timed
    region)."""
    n = 12 * LAYERS
    D.trace_enable(n)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        step(torch.cuda.current_stream().cuda_stream)
    with torch.cuda.stream(stream):
        for _ in range(2):
            D.trace_reset()
            g.replay()
            torch.cuda.synchronize()
    tr = D.trace_read(n).astype(np.float64).reshape(LAYERS, 12, 2)
    D.trace_enable(0)
    if tr.shape[0] < LAYERS:
        return None
    # per layer, relative to the previous layer's down end (layer 0 skipped)
    prev_end = tr[:-1, 2, 1]
    L = tr[1:]
    rel = lambda v: round(float(np.mean(v - prev_end)) / 1e3, 2)  # noqa: E731
    return {
        "router_first_start": rel(L[:, 0, 0]), "router_x_staged": rel(L[:, 3, 0]),
        "router_cluster_synced": rel(L[:, 3, 1]), "router_routed": rel(L[:, 6, 0]),
        "router_quantized": rel(L[:, 6, 1]), "router_end": rel(L[:, 0, 1]),
        "gateup_first_start": rel(L[:, 1, 0]), "gateup_post_wait": rel(L[:, 4, 0]), "gateup_end": rel(L[:, 1, 1]),
        "down_first_start": rel(L[:, 2, 0]), "down_post_wait": rel(L[:, 5, 0]), "down_end": rel(L[:, 2, 1]),
        "cycles": {"router_copy_wait": float(np.median(L[:, 7, 0])), "router_dots": float(np.median(L[:, 7, 1])),
                   "router_tail": float(np.median(L[:, 8, 1])), "gateup_stage": float(np.median(L[:, 9, 0])),
                   "gateup_dots": float(np.median(L[:, 9, 1])), "down_quant": float(np.median(L[:, 10, 0])),
                   "down_dots": float(np.median(L[:, 10, 1]))},
        "unit": "us after the previous layer's down end",
    }


def run_prefill(args, layers, stream, torch, D, T=None, label="prefill", force_tc=False, with_exact=True):
    """T tokens (default --prefill-tokens) through the same layers on the
    expert-major batch path, captured in one CUDA graph: a prefill (the
    experts average >= 16 tokens, so gate/up and down run as tcgen05 MMAs) or
    a batched decode step (the tiled dp4a kernels)."""
    T = args.prefill_tokens if T is None else T
    D.reserve(T, DIM, FFN, NE, NK)
    x0 = torch.from_numpy(np.random.default_rng(7).standard_normal((T, DIM)).astype(np.float32)).cuda()
    bufs = [torch.empty((T, DIM), device="cuda") for _ in range(2)]
    ids = torch.zeros((LAYERS, T, NK), dtype=torch.int32, device="cuda")
    descs = [L.desc() for L in layers]

    def step(sh):
        cur = x0
        for l, L in enumerate(layers):
            nxt = bufs[l % 2]
            L.forward(cur, nxt, residual=cur, ids=ids[l], stream=sh, desc=descs[l])
            cur = nxt

    steps = max(2, min(args.steps, 5))

    def timed():
        with torch.cuda.stream(stream):
            step(stream.cuda_stream)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step(torch.cuda.current_stream().cuda_stream)
        with torch.cuda.stream(stream):
            for _ in range(max(args.warmup, 3)):
                g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(steps):
                g.replay()
            e1.record(stream)
            torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps, D.last_path()

    extra = {}
    if force_tc:  # the tensor-core kernels at this T (below their automatic threshold)
        prev = D.force_generic(3)
        try:
            ms, last = timed()
        finally:
            D.force_generic(prev)
    else:
        ms, last = timed()
    if last == 3 and with_exact:  # the integer-exact tensor-core form beside the default fp16 one
        prev = D.tc_exact(1)
        try:
            ms_x, _ = timed()
        finally:
            D.tc_exact(prev)
        extra["integer_exact"] = {"value": round(T / (ms_x * 1e-3), 1), "unit": "tok/s", "ms_per_step": round(ms_x, 3),
                                  "engine": "tcgen05 kind::f16 on integer sub-block products (bit-identical to "
                                            "the CPU), per-super-block float tail"}
    ids_np = ids.cpu().numpy()
    bytes_step = sum(layer_bytes_model(ids_np[l].reshape(-1)) for l in range(LAYERS))
    flops = 2.0 * T * NK * 3 * DIM * FFN * LAYERS  # gate, up, down per routed token
    peak, peak_kind = peaks()
    tpeak = float(json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["bf16_tflops"]) \
        if os.path.exists(os.path.join(ROOT, "MEASURED_PEAKS.json")) else 1590.0
    gbs = bytes_step / (ms * 1e-3) / 1e9
    tfs = flops / (ms * 1e-3) / 1e12
    path = {0: "fused decode kernels", 1: "slot kernels", 2: "per-expert int8 dot kernels",
            3: "tcgen05 kind::f16 gate/up and down on dequantized fp16 tiles (f32 accumulation over the row, "
               "within 2e-3 of the reference), warp-specialized",
            4: "tiled dp4a gate/up and down (TMA-staged rows, integer-exact)"}.get(last, "?")
    return {"workload": label, "tokens": T, "layers": LAYERS, "value": round(T / (ms * 1e-3), 1), "unit": "tok/s",
            "ms_per_step": round(ms, 3), "steps": steps,
            "engine": "expert-major batch: tiled router GEMV, " + path,
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "peak_kind": peak_kind, "bytes_per_step": bytes_step,
                         "tensor_tflops": round(tfs, 2), "tensor_peak": tpeak,
                         "tensor_frac": round(tfs / tpeak, 5)}, **extra}


def run_e2e_device(args, g, stream, x0, out, torch, dist, world, job_tokens=None):
    """End to end through the device-resident API: every step copies the
    token's activation in from pinned host memory, replays the step and reads
    the final output back."""
    hx = torch.empty(x0.shape, dtype=torch.float32, pin_memory=True)
    hx.copy_(x0.cpu())
    ho = torch.empty(out.shape, dtype=torch.float32, pin_memory=True)
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 1)):
            x0.copy_(hx, non_blocking=True)
            g.replay()
            ho.copy_(out, non_blocking=True)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            x0.copy_(hx, non_blocking=True)
            g.replay()
            ho.copy_(out, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    T = x0.shape[0] if job_tokens is None else job_tokens  # whole job: every rank's own tokens
    return {"value": round(T / (ms * 1e-3), 2), "unit": "tok/s", "h2d_bytes_per_step": int(hx.numel() * 4),
            "d2h_bytes_per_step": int(ho.numel() * 4), "path": "device API with pinned host input/output per step"}


def run_e2e(args, B):
    """Seam calls with host buffers: per layer, router matvec (F32) then
    moeFfnBlockRouted, then the residual add on the host."""
    from loom_b200.device import DeviceTensor

    def host_bytes(ty, nblk, seed, sigma=1.0):
        t = DeviceTensor.synth(ty, nblk, seed, sigma)  # the seeded generator, read back as GGUF bytes
        b = t.download()
        t.free()
        return b

    nl = args.e2e_layers
    host = []
    for l in range(nl):
        s = 1000 + l
        host.append((host_bytes(Q4K, NE * FFN * DIM // 256, s * 10 + 1), host_bytes(Q4K, NE * FFN * DIM // 256, s * 10 + 2),
                     host_bytes(Q6K, NE * DIM * FFN // 256, s * 10 + 3), host_bytes(F32, NE * DIM, s * 10 + 4, 0.02)))
    import ctypes as C
    from loom_b200 import _lib
    # the C ABI called the way the reference's Zig arm would: argument structs built
    # once, the host buffers reused, one matvec + one moe_ffn_routed per layer
    lib = _lib.lib()
    mv, fr = lib.loom_cuda_matvec, lib.loom_cuda_moe_ffn_routed
    cfg = _lib.RoutedCfg(NE, NK, 0, 1, 1.0)
    x = np.random.default_rng(0).standard_normal(DIM).astype(np.float32)
    logits = np.empty(NE, np.float32)
    out = np.empty(DIM, np.float32)
    xp, lp, op = (C.c_void_p(a.ctypes.data) for a in (x, logits, out))
    args_l = [(C.c_void_p(r.ctypes.data), r.nbytes, _lib.Weight(Q4K, g.ctypes.data, g.nbytes),
               _lib.Weight(Q4K, u.ctypes.data, u.nbytes), _lib.Weight(Q6K, d.ctypes.data, d.nbytes))
              for (g, u, d, r) in host]

    def token(_x):
        for (rp, rn, wg, wu, wd) in args_l:
            if mv(F32, lp, rp, rn, xp, NE, DIM) != 0:
                raise RuntimeError("matvec declined")
            if fr(xp, DIM, lp, None, wg, wu, wd, None, FFN, 0, cfg, op) != 0:
                raise RuntimeError("moe_ffn_routed declined")
            np.add(x, out, out=x)  # the residual, on the host as the reference's engine does
        return x

    for _ in range(max(args.warmup, 1)):
        token(x)
    reps = max(args.steps, 3)
    t0 = time.perf_counter()
    for _ in range(reps):
        token(x)
    dt = (time.perf_counter() - t0) / reps / nl * LAYERS
    h2d = LAYERS * (DIM * 4 + DIM * 4 + NE * 4)
    d2h = LAYERS * (NE * 4 + DIM * 4)
    return {"value": round(1.0 / dt, 2), "unit": "tok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "path": f"seam calls with host buffers, {nl} distinct layers cycled to {LAYERS}"}


# ---- full-model decode (--workload model) -------------------------------------------

MODEL_METRIC = "decode tok/s (Qwen3-30B-A3B full model, Q4_K_M, batch 1, ctx 2048)"
DS_METRIC = "decode tok/s (DeepSeek-V2-Lite-shaped full model, Q4_K/Q8_0, batch 1)"
# DRAM bytes of one headline step (48 layers + head at position 2047), from the
# 4-layer ncu capture of profiles/model_step_qwen3_ctx2048_dram.md: 48 x 56.43 MB + 257.7 MB
MODEL_TRAFFIC = 2966436352


def model_bytes(spec, pos: int, n_local: int = None) -> int:
    """Algorithmic HBM bytes of one decode token at position pos: every
    replicated weight once (attention, norms, router, head, the embedding
    row), the n_used selected experts' gate/up/down planes (on a shard: the
    expected share n_used * n_local / n_expert), the KV rows read (pos + 1 per
    layer, keys and values) and written (one)."""
    n_local = spec.n_expert if n_local is None else n_local
    kvd = spec.n_kv_heads * spec.head_dim
    b = 0
    for t in spec.plan():
        if t.name == "token_embd":
            b += t.nbytes // spec.vocab
        elif t.planes > 1:
            b += t.nbytes // t.planes * spec.n_used * n_local / spec.n_expert
        else:
            b += t.nbytes
    if getattr(spec, "mla", False):  # compressed row + rope row per position
        b += spec.n_layers * (pos + 2) * (spec.kv_lora + spec.rope_dim) * 4
    else:
        b += spec.n_layers * (pos + 2) * kvd * 4 * 2
    return int(b)


def cpu_model_time(spec, threads: int, reps: int, pos: int):
    """Seconds per token of the oracle's token step (llama.zig:1111-1228
    restated) for `spec`, measured on 2- and 4-layer cuts of the model (same
    shapes, KV cache filled with synthetic rows up to pos) and extrapolated:
    head = t2 - 2 * layer, layer = (t4 - t2) / 2. Medians of `reps` runs."""
    import copy
    from oracle import oracle as orc
    from oracle.oracle import LlamaRunner
    from tests.modelref import host_tensors
    if threads > 1:
        orc.parallel_begin(threads)
    try:
        med = {}
        for nl in (2, 4):
            sp = copy.copy(spec)
            sp.n_layers = nl
            sp.ctx_len = pos + 1
            run = LlamaRunner(sp, host_tensors(sp, orc))
            rng = np.random.default_rng(0)
            run.kc[:] = rng.standard_normal(run.kc.size).astype(np.float32)
            run.vc[:] = rng.standard_normal(run.vc.size).astype(np.float32)
            run.step(1, pos)  # warm-up
            ts = []
            for r in range(reps):
                t0 = time.perf_counter()
                run.step(1 + r, pos)
                ts.append(time.perf_counter() - t0)
            med[nl] = statistics.median(ts)
    finally:
        if threads > 1:
            orc.parallel_end()
    layer = max((med[4] - med[2]) / 2, 1e-9)
    head = max(med[2] - 2 * layer, 0.0)
    return head + spec.n_layers * layer


def cpu_model_baseline(spec, pos, reps=9):
    """The reference CPU path's own policy: nproc - 2 worker threads
    (generator.zig:265-304), plus the single-thread figure."""
    n = max(1, (os.cpu_count() or 1) - 2)
    t_n = cpu_model_time(spec, n, reps, pos)
    t_1 = cpu_model_time(spec, 1, max(3, reps // 3), pos)
    try:
        import cpuinfo
        model = cpuinfo.get_cpu_info().get("brand_raw", "?")
    except Exception:  # noqa: BLE001
        model = "?"
    return {"value": round(1.0 / t_n, 3), "unit": "tok/s", "cores": n, "kind": "port",
            "value_1_thread": round(1.0 / t_1, 3), "host_cores": os.cpu_count(), "cpu_model": model,
            "sample": (f"oracle token step at position {pos} on 2- and 4-layer cuts of the model (KV cache "
                       f"synthetic), medians of {reps} runs ({max(3, reps // 3)} at 1 thread), extrapolated to "
                       f"{spec.n_layers} layers")}


def prefill_bytes(spec, T: int) -> int:
    """Algorithmic HBM bytes of a T-token prefill: every replicated weight once
    (attention, norms, router, the head for the last token; T embedding rows),
    each routed layer's expected distinct experts (n_expert (1 - (1 - n_used /
    n_expert)^T)) once, the T cache rows written per layer."""
    kvd = spec.n_kv_heads * spec.head_dim
    touched = spec.n_expert * (1.0 - (1.0 - spec.n_used / spec.n_expert) ** T)
    b = 0
    for t in spec.plan():
        if t.name == "token_embd":
            b += t.nbytes // spec.vocab * T
        elif t.planes > 1:
            b += t.nbytes // t.planes * touched
        else:
            b += t.nbytes
    return int(b + spec.n_layers * T * kvd * 4 * 2)


def run_model_prefill(args, dev, spec, peak, peak_kind):
    """A T-token prompt through the whole model at position 0 by the batched
    prefill (loom_cuda_model_prefill: host token ids in, the last token's next
    token out), wall clock of the synchronous call, median of 3 after one
    warm-up."""
    T = args.model_prefill
    rng = np.random.default_rng(3)
    prompt = [int(t) for t in rng.integers(0, spec.vocab, size=T)]
    dev.prefill(prompt, 0)
    ts = []
    for _ in range(3):
        t0 = time.perf_counter()
        dev.prefill(prompt, 0)
        ts.append(time.perf_counter() - t0)
    sec = statistics.median(ts)
    b = prefill_bytes(spec, T)
    return {"workload": f"prefill of a {T}-token prompt through the full model (batched, layer-major)",
            "tokens": T, "value": round(T / sec, 1), "unit": "tok/s", "ms_per_step": round(sec * 1e3, 3),
            "engine": "loom_cuda_model_prefill: row-batched norms, tiled q/k/v/output matmuls, causal ordered "
                      "attention per (head, token), experts on the tensor cores",
            "roofline": {"bound": "hbm", "achieved": round(b / sec / 1e9, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(b / sec / 1e9 / peak, 4), "peak_kind": peak_kind, "bytes_per_step": b},
            "e2e": {"value": round(T / sec, 1), "unit": "tok/s", "h2d_bytes_per_step": 4 * T + 4,
                    "d2h_bytes_per_step": 4}}


def run_model_batch(args, dev, spec, peak, peak_kind):
    """One decode step of B sequences through the whole model
    (loom_cuda_model_decode_batch: B host tokens and positions in, B next tokens
    out), every sequence at position ctx - 1 of its own cache (zeroed rows:
    the same kernels and bytes as a filled one), wall clock of the synchronous
    call, median of 5 after two warm-ups."""
    B = args.model_batch
    pos = spec.ctx_len - 1
    rng = np.random.default_rng(4)
    toks = [int(t) for t in rng.integers(0, spec.vocab, size=B)]
    for _ in range(2):
        dev.decode_batch(toks, [pos] * B)
    ts = []
    for _ in range(5):
        t0 = time.perf_counter()
        dev.decode_batch(toks, [pos] * B)
        ts.append(time.perf_counter() - t0)
    sec = statistics.median(ts)
    kvd = spec.n_kv_heads * spec.head_dim
    touched = spec.n_expert * (1.0 - (1.0 - spec.n_used / spec.n_expert) ** B)
    b = 0
    for t in spec.plan():
        if t.name == "token_embd":
            b += t.nbytes // spec.vocab * B
        elif t.planes > 1:
            b += t.nbytes // t.planes * touched
        else:
            b += t.nbytes
    b = int(b + B * spec.n_layers * (pos + 2) * kvd * 4 * 2)  # every sequence's cache rows read, one written
    return {"workload": f"decode of {B} sequences, one token each, at position {pos} of a {spec.ctx_len}-token "
                        f"context (each its own cache)",
            "tokens": B, "value": round(B / sec, 1), "unit": "tok/s", "ms_per_step": round(sec * 1e3, 3),
            "engine": "loom_cuda_model_decode_batch: row-batched norms, tiled matmuls, per-row attention over each "
                      "sequence's cache, the experts of all rows on the expert-major path, every row's head",
            "roofline": {"bound": "hbm", "achieved": round(b / sec / 1e9, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(b / sec / 1e9 / peak, 4), "peak_kind": peak_kind, "bytes_per_step": b},
            "e2e": {"value": round(B / sec, 1), "unit": "tok/s", "h2d_bytes_per_step": 8 * B,
                    "d2h_bytes_per_step": 4 * B}}


def run_model(args):
    import torch
    import torch.distributed as dist
    from loom_b200 import backend as B
    from loom_b200 import device as D
    from loom_b200.model import DeviceModel, deepseek_v2_lite, qwen3_moe

    rank, world, local = dist_env()
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    B.init(local)
    from loom_b200.model import deepseek_v3
    ds_main = args.model in ("ds-v2-lite", "ds-v3")
    if args.model == "ds-v2-lite":
        spec = deepseek_v2_lite(n_layers=args.layers if args.layers != LAYERS_DEFAULT else 27, ctx_len=args.ctx)
    elif args.model == "ds-v3":
        spec = deepseek_v3(n_layers=args.v3_layers, ctx_len=args.ctx)
    else:
        spec = qwen3_moe(n_layers=args.layers, ctx_len=args.ctx)
    shard = D.expert_range(spec.n_expert, rank, world) if world > 1 else None
    if world > 1:
        D.ep_init(rank, world, dist)
    dev = DeviceModel(spec, expert_shard=shard)
    if args.prefill_only or args.batch_only:  # one sub-measurement alone (profiling captures), then exit
        if rank == 0:
            peak, peak_kind = peaks()
            run = run_model_prefill if args.prefill_only else run_model_batch
            print(json.dumps(run(args, dev, spec, peak, peak_kind)), flush=True)
        dev.free()
        return
    pos = spec.ctx_len - 1
    # fill the KV cache: greedy decode of positions 0 .. ctx-2 (every rank the same tokens)
    tok = 1
    t0 = time.perf_counter()
    for p in range(0 if args.no_fill else pos):
        tok, _ = dev.decode(tok, p)
    fill_s = time.perf_counter() - t0

    stream = torch.cuda.Stream()
    d_tok = torch.tensor([tok], dtype=torch.int32, device="cuda")
    d_pos = torch.tensor([pos], dtype=torch.int32, device="cuda")
    d_next = torch.zeros(1, dtype=torch.int32, device="cuda")
    d_logits = torch.empty(spec.vocab, dtype=torch.float32, device="cuda")
    with torch.cuda.stream(stream):
        dev.step(d_tok, d_pos, d_logits, d_next, stream=stream.cuda_stream)
    torch.cuda.synchronize()
    k0 = B.kernelLaunches()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        dev.step(d_tok, d_pos, d_logits, d_next, stream=torch.cuda.current_stream().cuda_stream)
    launches_per_step = B.kernelLaunches() - k0
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            g.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with Clocks(local) as ck:
            torch.cuda.synchronize()
            e0.record(stream)
            for _ in range(args.steps):
                g.replay()
            e1.record(stream)
            torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    # e2e: the host entry point, host token in and out, wall clock per token
    for _ in range(args.warmup):
        dev.decode(tok, pos)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        dev.decode(tok, pos)
    e2e_ms = (time.perf_counter() - t0) / args.steps * 1e3
    if world > 1:
        t = torch.tensor([ms, e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = (float(v) for v in t.tolist())
        dist.barrier()
    n_local = shard[1] if shard else spec.n_expert
    bytes_step = model_bytes(spec, pos, n_local)
    achieved = bytes_step / (ms * 1e-3) / 1e9
    peak, peak_kind = peaks()
    prefill = mbatch = None
    if world == 1 and not ds_main and args.model_batch > 0:
        try:
            mbatch = run_model_batch(args, dev, spec, peak, peak_kind)
        except Exception as e:  # reported in the line, never fatal to the headline
            mbatch = {"error": f"{type(e).__name__}: {e}"[:300]}
    if world == 1 and not ds_main and args.model_prefill > 0:
        try:
            prefill = run_model_prefill(args, dev, spec, peak, peak_kind)
        except Exception as e:  # reported in the line, never fatal to the headline
            prefill = {"error": f"{type(e).__name__}: {e}"[:300]}
    dev.free()

    ds = None
    if world == 1 and not args.no_deepseek and not ds_main:
        try:
            ds = run_model_deepseek(args, peak, peak_kind)
        except Exception as e:  # reported in the line, never fatal to the headline
            ds = {"error": f"{type(e).__name__}: {e}"[:300]}
    moe = None
    if world == 1 and not args.no_moe_stack and not ds_main:
        margs = argparse.Namespace(**vars(args))
        margs.tokens, margs.ep, margs.engine, margs.trace = 1, False, "auto", False
        margs.layers = args.layers
        moe = run_gpu(margs, emit=False)
    if rank != 0:
        return
    cpu = None
    if not args.no_cpu and world == 1 and not ds_main:
        cpu = cpu_model_baseline(spec, pos)
    line = {
        "metric": (MODEL_METRIC if not ds_main else DS_METRIC if args.model == "ds-v2-lite" else
                   f"decode tok/s (DeepSeek-V3-shaped model, first {spec.n_layers} of 61 layers at full width, Q4_K, "
                   f"batch 1)"), "value": round(1e3 / ms, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "dtype": "int8xq4/q6 matvecs (f32 accum), f32 attention and KV",
        "data": "synthetic (seeded generator), random-init weights",
        "config": {"workload": f"{spec.name} full-model decode, batch 1, position {pos} of a {spec.ctx_len}-token "
                               f"context", "model": spec.name, "layers": spec.n_layers, "batch": 1,
                   "ctx": spec.ctx_len, "dim": spec.dim, "n_heads": spec.n_heads, "n_kv_heads": spec.n_kv_heads,
                   "n_expert": spec.n_expert, "n_used": spec.n_used, "vocab": spec.vocab,
                   "parallelism": (f"ep{world} (experts sharded, attention replicated, NCCL all-reduce combine)"
                                   if world > 1 else "1 gpu"),
                   "engine": "loom_cuda_model_step in a CUDA graph",
                   "l2": f"inputs > L2 ({bytes_step / 1e9:.2f} GB read per token)",
                   "kv_fill_s": round(fill_s, 2)},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4),
                     "traffic": MODEL_TRAFFIC if (args.model == "qwen3" and spec.n_layers == 48 and spec.ctx_len == 2048)
                     else None,
                     "traffic_note": "DRAM bytes per step from an ncu capture of 4 layers + head (caches flushed per "
                                     "kernel, scaled to 48 layers): profiles/model_step_qwen3_ctx2048_dram.md",
                     "kernel": "whole decode step (all kernels of the token, CUDA-event timed)",
                     "peak_kind": peak_kind, "bytes_per_step": bytes_step},
        "e2e": {"value": round(1e3 / e2e_ms, 2), "unit": "tok/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 4,
                "path": "loom_cuda_model_decode (graph replay, host token in/out), wall clock"},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": ck.summary(),
    }
    if moe:
        line["moe_stack"] = {k: moe[k] for k in ("metric", "value", "unit", "ms_per_step", "roofline", "config",
                                                 "e2e", "e2e_device", "prefill", "batch", "gpu_launches")
                             if k in moe}
    if ds:
        line["deepseek_v2_lite"] = ds
    if prefill is not None:
        line["prefill"] = prefill
    if mbatch is not None:
        line["batch"] = mbatch
    if world == 1 and not args.no_deepseek and not ds_main and args.v3_layers > 0:
        try:
            line["deepseek_v3_cut"] = run_model_deepseek(args, peak, peak_kind, which="v3")
        except Exception as e:
            line["deepseek_v3_cut"] = {"error": f"{type(e).__name__}: {e}"[:300]}
    if cpu:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


def run_model_deepseek(args, peak, peak_kind, which="v2-lite"):
    """A DeepSeek-shaped model: V2-Lite (MLA attention,
    layer 0 dense, 64 routed experts top-6 + 2 shared), or a cut of the V3
    shape (config 5 at full width: dim 7168, 128 MLA heads with q-LoRA, 256
    experts top-8 with sigmoid + bias and grouped top-k, one shared expert; the
    first `layers` of its 61, three dense). One decode token at position
    ctx - 1 after filling the cache by decoding, graph-replayed and event-timed
    like the headline; e2e through loom_cuda_model_decode."""
    import torch
    from loom_b200.model import DeviceModel, deepseek_v2_lite, deepseek_v3
    spec = deepseek_v2_lite(ctx_len=args.ctx) if which == "v2-lite" else deepseek_v3(n_layers=args.v3_layers,
                                                                                       ctx_len=args.ctx)
    dev = DeviceModel(spec)
    try:
        pos = spec.ctx_len - 1
        tok = 1
        t0 = time.perf_counter()
        for p in range(pos):
            tok, _ = dev.decode(tok, p)
        fill_s = time.perf_counter() - t0
        stream = torch.cuda.Stream()
        d_tok = torch.tensor([tok], dtype=torch.int32, device="cuda")
        d_pos = torch.tensor([pos], dtype=torch.int32, device="cuda")
        d_next = torch.zeros(1, dtype=torch.int32, device="cuda")
        d_logits = torch.empty(spec.vocab, dtype=torch.float32, device="cuda")
        with torch.cuda.stream(stream):
            dev.step(d_tok, d_pos, d_logits, d_next, stream=stream.cuda_stream)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            dev.step(d_tok, d_pos, d_logits, d_next, stream=torch.cuda.current_stream().cuda_stream)
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.steps):
                g.replay()
            e1.record(stream)
            torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        for _ in range(args.warmup):
            dev.decode(tok, pos)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            dev.decode(tok, pos)
        e2e_ms = (time.perf_counter() - t0) / args.steps * 1e3
        err = dev.error()
    finally:
        dev.free()
    bytes_step = model_bytes(spec, pos)
    achieved = bytes_step / (ms * 1e-3) / 1e9
    metric = DS_METRIC if which == "v2-lite" else (
        f"decode tok/s (DeepSeek-V3-shaped model, first {spec.n_layers} of 61 layers at full width, Q4_K, batch 1)")
    return {"metric": metric,
            "value": round(1e3 / ms, 2), "unit": "tok/s", "ms_per_step": round(ms, 4),
            "config": {"workload": f"{spec.name} decode ({spec.n_layers} layers), batch 1, position {pos} of a "
                                   f"{spec.ctx_len}-token context", "model": spec.name, "layers": spec.n_layers,
                       "ms_per_layer": round(ms / spec.n_layers, 4),
                       "dim": spec.dim, "n_heads": spec.n_heads, "kv_lora": spec.kv_lora, "n_expert": spec.n_expert,
                       "n_used": spec.n_used, "shared_ffn": spec.shexp_ffn, "vocab": spec.vocab,
                       "engine": "loom_cuda_model_step (MLA kernels + fused MoE) in a CUDA graph",
                       "kv_fill_s": round(fill_s, 2)},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind, "bytes_per_step": bytes_step},
            "e2e": {"value": round(1e3 / e2e_ms, 2), "unit": "tok/s", "h2d_bytes_per_step": 8,
                    "d2h_bytes_per_step": 4, "path": "loom_cuda_model_decode, wall clock"},
            "device_error": err}


def run_reference_model(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from loom_b200.model import qwen3_moe
    spec = qwen3_moe(n_layers=args.layers, ctx_len=args.ctx)
    pos = spec.ctx_len - 1
    cpu = cpu_model_baseline(spec, pos, reps=max(args.steps, 9))
    v = cpu["value"]
    line = {"impl": "reference", "metric": MODEL_METRIC, "value": v, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 / v, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8xq4/q6 matvecs (f32 accum), f32 attention and KV",
            "data": "synthetic (seeded generator), random-init weights",
            "config": {"workload": f"qwen3-30b-a3b full-model decode, batch 1, position {pos} of a {spec.ctx_len}-"
                                   f"token context", "model": spec.name, "layers": spec.n_layers, "batch": 1,
                       "ctx": spec.ctx_len, "parallelism": "host threads"},
            "cpu_baseline": cpu,
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--impl", default="cuda", choices=["cuda", "reference"])
    ap.add_argument("--e2e-layers", type=int, default=8)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--prefill-tokens", type=int, default=512,
                    help="also time a prefill of this many tokens through the same layers (0: skip)")
    ap.add_argument("--batch-tokens", type=int, default=32,
                    help="also time one batched decode step of this many tokens (0: skip)")
    ap.add_argument("--engine", default="auto", choices=["auto", "layers", "stack"],
                    help="layers: per-layer kernels in a CUDA graph; stack: one persistent kernel for all layers "
                         "(T=1); auto: stack for unsharded T=1, else layers")
    ap.add_argument("--trace", action="store_true", help="add per-kernel phase times (one extra traced replay)")
    ap.add_argument("--ep", action="store_true",
                    help="with torchrun: shard each layer's experts over the ranks (expert parallel) instead of "
                         "running independent replicas")
    ap.add_argument("--ep-mode", default="allreduce", choices=["allreduce", "a2a", "a2a-counted"],
                    help="allreduce: every rank runs the same tokens, partial outputs summed; a2a: every rank owns "
                         "its own T tokens, routed rows travel to the experts' ranks and back (NCCL send/recv) in fixed "
                         "runs of T*n_used rows per rank, captured in a CUDA graph; a2a-counted: the same with "
                         "exactly the routed rows (their counts go to the host each layer, eager launches)")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="layers in the stack (default 48; smaller only for profiling captures)")
    ap.add_argument("--workload", default="model", choices=["model", "moe"],
                    help="model: full Qwen3-30B-A3B decode (the headline); moe: the 48 MoE layers only")
    ap.add_argument("--ctx", type=int, default=2048, help="context length of the model workload")
    ap.add_argument("--no-moe-stack", action="store_true", help="model workload: skip the MoE-only sub-measurement")
    ap.add_argument("--model", default="qwen3", choices=["qwen3", "ds-v2-lite", "ds-v3"],
                    help="model workload: the headline Qwen3-30B-A3B shape, or the DeepSeek-V2-Lite shape (MLA)")
    ap.add_argument("--v3-layers", type=int, default=8,
                    help="model workload: layers of the DeepSeek-V3-shaped cut measured beside the headline (0: skip)")
    ap.add_argument("--no-fill", action="store_true",
                    help="model workload: leave the KV cache unfilled (profiling captures only; the kernels and "
                         "bytes are the same, the cached values are zeros)")
    ap.add_argument("--model-prefill", type=int, default=512,
                    help="model workload: also time a prefill of this many tokens through the full model (0: skip)")
    ap.add_argument("--model-batch", type=int, default=32,
                    help="model workload: also time one decode step of this many sequences (0: skip)")
    ap.add_argument("--batch-only", action="store_true",
                    help="model workload: time only the --model-batch decode step (profiling captures)")
    ap.add_argument("--prefill-only", action="store_true",
                    help="model workload: time only the --model-prefill prefill (profiling captures)")
    ap.add_argument("--no-deepseek", action="store_true",
                    help="model workload: skip the DeepSeek-V2-Lite full-model sub-measurement")
    args = ap.parse_args()
    globals()["LAYERS"] = args.layers
    if args.workload == "model":
        run_reference_model(args) if args.impl == "reference" else run_model(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
