#!/usr/bin/env python3
"""Benchmark of the W4A16 grouped-MoE layer on B200 (one JSON line on stdout).

Workload (default, N=1): benchmark configuration 1 -- decode, M=1 token, one
MoE layer with E=256 experts, top-10, H=3072, I=1024, int4 group-32 weights
(random-init, seeded), bf16 activations ~ N(0,1).  A "step" is one full
``fused_experts_w4a16`` call: routing align + w13 GEMM (+SiLU*up) + w2 GEMM
(+ weighted top-k sum).  ``value`` is achieved weight bandwidth: unique routed
experts x 5,308,416 bytes per step / device time per step (the reference's
metric, bench/bench_moe.py:250-263, :742-743).  Each step is replayed from a
CUDA graph (as the reference's --cudagraph mode) with a 256 MiB L2 flush
before it, outside the timed events.

``--workload ep`` runs benchmark configuration 4 instead: a stack of four
such layers, expert-parallel over the N ranks (E/N experts and their weights
per rank), M=8192 tokens per step split evenly over the ranks as source
batches, Zipf(1.1)-biased top-10 routing, NCCL all-to-all dispatch and
combine; ``value`` is tokens/s of the whole job.

``--impl reference`` times the reference algorithm's CPU path (the numpy
oracle port; the reference itself is PyTorch and cannot travel to the GPU box)
on all host cores, same config and metric.  With N>1 GPUs every rank runs its
own replica of the workload (weak scaling); rank 0 prints the aggregate.
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
from pathlib import Path

REPO = Path(__file__).resolve().parent
PKG = REPO / "gb10-laguna-s-2.1-w4a16-moe_b200"
for _p in (str(PKG), str(REPO)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

E, TOPK, H, I, GROUP = 256, 10, 3072, 1024, 32
BYTES_PER_EXPERT = 2 * I * (H // 2) + H * (I // 2) + 2 * I * (H // GROUP) * 2 + H * (I // GROUP) * 2
W13_BYTES_PER_EXPERT = 2 * I * (H // 2) + 2 * I * (H // GROUP) * 2
FLUSH_BYTES = 256 << 20
METRIC = "weight_GBps"


def _peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.is_file():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d.get("bf16_tflops", 1590.0)),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", 1400.0)), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


def _traffic(M: int, key: str = "decode") -> float | None:
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    p = REPO / "profiles" / "traffic.json"
    if not p.is_file():
        return None
    d = json.loads(p.read_text())
    v = d.get(f"{key}_M{M}")
    return float(v) if v is not None else None


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:  # noqa: BLE001
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:  # noqa: BLE001
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def _dist():
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        import datetime

        # a collective that one rank never joins fails in two minutes, not ten
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=120))
    return world, rank, local


def _max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def _barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def cpu_port_time(M: int, layer_cpu: dict, hidden, tw, ids, threads: int, budget_s: float,
                  max_iters: int) -> tuple[float, int]:
    """Mean seconds of one oracle forward on the host cores (bounded sample)."""
    import numpy as np
    from threadpoolctl import threadpool_limits

    from oracle import moe_oracle as O

    x = hidden.float().cpu().numpy()
    tw_c = tw.float().cpu().numpy()
    ids_c = ids.cpu().numpy().astype(np.int64)
    times = []
    with threadpool_limits(limits=threads):
        t_end = time.perf_counter() + budget_s
        while len(times) < max_iters and (not times or time.perf_counter() < t_end):
            t0 = time.perf_counter()
            O.moe_reference(x, layer_cpu["w1_q"], layer_cpu["w1_s"], layer_cpu["w2_q"], layer_cpu["w2_s"],
                            tw_c, ids_c, GROUP)
            times.append(time.perf_counter() - t0)
    return sum(times) / len(times), len(times)


def routed_layer_to_cpu(layer: dict, ids):
    """Copy only the routed experts to host memory (ids remapped to them)."""
    import numpy as np
    import torch

    used = torch.unique(ids).to(torch.int64)
    bits = lambda t: t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)  # noqa: E731
    sub = {"w1_q": layer["w1_q"][used].cpu().numpy(), "w1_s": bits(layer["w1_s"][used]),
           "w2_q": layer["w2_q"][used].cpu().numpy(), "w2_s": bits(layer["w2_s"][used])}
    remap = torch.full((E,), -1, dtype=torch.int64, device=ids.device)
    remap[used] = torch.arange(used.numel(), device=ids.device)
    return sub, remap[ids.to(torch.int64)]


def decode_workload(M: int) -> str:
    cfg = 1 if M == 1 else (2 if M <= 256 else 3)
    return f"decode M={M} (config {cfg}): E=256 top-10 H=3072 I=1024 int4 g32, one layer"


EP_WORKLOAD = ("config 4: expert-parallel stack of 4 MoE layers (E=256 top-10 H=3072 I=1024 int4 g32), "
               "8192 tokens per step, Zipf(1.1)-biased routing")


def run_reference_ep(args, world: int) -> int:
    """Reference arm of configuration 4: the numpy oracle port (the reference's
    per-expert fp32 dequant-then-GEMM, bench/bench_moe.py:run_reference) on all
    host cores, timed on a bounded sample of tokens of one layer and scaled to
    the 4-layer stack; the reference has no multi-GPU path."""
    import torch

    from kernels.synthetic import make_hidden, make_layer, make_routing, zipf_bias

    sub_tok = 8
    lay = make_layer(E // world, H, I, seed=0, device="cpu")
    bias = zipf_bias(E, 1.1, seed=0)
    tw, ids = make_routing(EP_TOKENS // world, E, TOPK, seed=0, device="cpu", bias=bias)
    tw, ids = tw[:sub_tok], ids[:sub_tok] % (E // world)  # route into the generated experts
    x = make_hidden(EP_TOKENS // world, H, seed=0, device="cpu")[:sub_tok]
    sub, local_ids = routed_layer_to_cpu(lay, ids)
    cores = os.cpu_count() or 1
    cpu_port_time(sub_tok, sub, x, tw, local_ids, cores, 0.0, 1)
    per, n = cpu_port_time(sub_tok, sub, x, tw, local_ids, cores, 20.0, max(args.steps, 3))
    tps = sub_tok / per / EP_LAYERS
    line = {
        "impl": "reference", "metric": "ep_tokens_per_s", "value": tps, "unit": "tokens/s", "n_gpus": world,
        "steps": n, "warmup": args.warmup, "ms_per_step": EP_TOKENS / tps * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": EP_WORKLOAD, "tokens_per_step": EP_TOKENS, "layers": EP_LAYERS},
        "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{n} numpy-oracle forwards of one layer for {sub_tok} tokens (per-call "
                                   f"dequant of their routed experts), scaled to the 4-layer stack"},
        "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_reference_arm(args) -> int:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    if args.workload == "ep":
        return run_reference_ep(args, world)
    import torch

    from kernels.synthetic import make_hidden, make_layer, make_routing

    M = args.M
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    layer = make_layer(E, H, I, seed=0, device=dev)
    hidden = make_hidden(M, H)
    tw, ids = make_routing(M, E, TOPK)
    n_act = int(torch.unique(ids).numel())
    wbytes = n_act * BYTES_PER_EXPERT
    sub, local_ids = routed_layer_to_cpu(layer, ids.to(dev))
    del layer
    cores = os.cpu_count() or 1
    for _ in range(args.warmup):
        cpu_port_time(M, sub, hidden, tw, local_ids.cpu(), cores, 0.0, 1)
    per, n = cpu_port_time(M, sub, hidden, tw, local_ids.cpu(), cores, 1e9, args.steps)
    gbs = wbytes / per / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": world,
        "steps": n, "warmup": args.warmup, "ms_per_step": per * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": decode_workload(M), "M": M, "unique_experts": n_act,
                   "weight_bytes_per_step": wbytes},
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"{n} full forwards of the numpy oracle (restating bench/bench_moe.py:"
                                   f"run_reference, per-call dequant) at M={M} on the routed experts"},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args) -> int:
    import torch

    from kernels import w4a16_moe as K
    from kernels.synthetic import make_hidden, make_layer, make_routing

    world, rank, local = _dist()
    if world == 1 and args.gpus > 1:
        print("note: --gpus > 1 requested without torchrun; running one replica", file=sys.stderr)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    K.load_library()
    M = args.M

    layer = make_layer(E, H, I, seed=0, device=dev)
    w1r, s1r = K.repack_weights(layer["w1_q"], layer["w1_s"])
    w2r, s2r = K.repack_weights(layer["w2_q"], layer["w2_s"])
    hidden = make_hidden(M, H, device=dev)
    tw, ids = make_routing(M, E, TOPK, device=dev)
    n_act = int(torch.unique(ids).numel())
    wbytes = n_act * BYTES_PER_EXPERT
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def step(h, w, i):
        return K.fused_experts_w4a16(h, w1r, w2r, s1r, s2r, w, i)

    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    for _ in range(max(args.warmup, 3)):
        step(hidden, tw, ids)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step(hidden, tw, ids)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out_static = step(hidden, tw, ids)
    for _ in range(max(args.warmup, 3)):
        flush.zero_()
        graph.replay()
    torch.cuda.synchronize()

    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    step_ms, align_ms, w13_ms, w2_ms = [], [], [], []
    _barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        for _ in range(args.steps):
            flush.zero_()
            t0.record()
            graph.replay()
            t1.record()
            t1.synchronize()
            step_ms.append(t0.elapsed_time(t1))
        torch.cuda.synchronize()
    _barrier(world)
    # Per-kernel device time of the same steps: eager launches with events
    # recorded on the forward's stream at its stage boundaries (graph replays
    # above carry no event nodes, which would add microseconds per node).
    K.set_stage_events(ev)
    for _ in range(args.steps):
        flush.zero_()
        step(hidden, tw, ids)
        ev[3].synchronize()
        align_ms.append(ev[0].elapsed_time(ev[1]))
        w13_ms.append(ev[1].elapsed_time(ev[2]))
        w2_ms.append(ev[2].elapsed_time(ev[3]))
    K.set_stage_events(None)
    total_ms = _max_over_ranks(sum(step_ms), world)
    total_bytes = _sum_over_ranks(float(wbytes * args.steps), world)
    value = total_bytes / (total_ms * 1e-3) / 1e9

    # ---- end to end through the public API with pinned host buffers ----
    h_host = hidden.cpu().pin_memory()
    tw_host = tw.cpu().pin_memory()
    ids_host = ids.cpu().pin_memory()
    out_host = torch.empty((M, H), dtype=torch.bfloat16).pin_memory()
    hd, twd, idd = torch.empty_like(hidden), torch.empty_like(tw), torch.empty_like(ids)
    e2e_ms = []
    for it in range(args.warmup + args.steps):
        flush.zero_()
        t0.record()
        hd.copy_(h_host, non_blocking=True)
        twd.copy_(tw_host, non_blocking=True)
        idd.copy_(ids_host, non_blocking=True)
        o = step(hd, twd, idd)
        out_host.copy_(o, non_blocking=True)
        t1.record()
        t1.synchronize()
        if it >= args.warmup:
            e2e_ms.append(t0.elapsed_time(t1))
    e2e_total = _max_over_ranks(sum(e2e_ms), world)
    e2e_value = total_bytes / (e2e_total * 1e-3) / 1e9
    h2d = hidden.numel() * 2 + tw.numel() * 4 + ids.numel() * 4
    d2h = M * H * 2

    # ---- parity spot check of the timed output (cheap, outside timing) ----
    torch.cuda.synchronize()
    assert torch.isfinite(out_static.float()).all()
    assert torch.equal(out_host.to(dev), out_static)

    peaks = _peaks()
    w13_mean = sum(w13_ms) / len(w13_ms)
    # the library runs M*topk <= 4096 slots through its single fused kernel
    fused = M * TOPK <= 4096
    if fused:  # one persistent kernel does routing + w13 + w2 + top-k sum
        kname = "moe_decode_fused_kernel (routing + w13 + w2 + top-k sum)"
        kbytes = wbytes
        achieved = kbytes / (w13_mean * 1e-3) / 1e9
        roofline = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": achieved / peaks["hbm_gbs"], "traffic": _traffic(M), "kernel": kname,
                    "kernel_us": 1e3 * w13_mean, "peak_src": f"{peaks['src']} hbm_gbs (STREAM copy)",
                    "algorithmic_bytes_per_launch": kbytes}
    else:  # tensor-core prefill: the w13 grouped GEMM is the dominant kernel
        kflops = 2.0 * M * TOPK * (2 * I) * H
        achieved = kflops / (w13_mean * 1e-3) / 1e12
        roofline = {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                    "frac": achieved / peaks["bf16_tflops"], "traffic": _traffic(M, "prefill_w13"),
                    "kernel": "moe_prefill_kernel<0> (w13 + SiLU*up, tcgen05)", "kernel_us": 1e3 * w13_mean,
                    "w2_and_sum_us": 1e3 * sum(w2_ms) / len(w2_ms),
                    "peak_src": f"{peaks['src']} bf16_tflops (cuBLAS burst)",
                    "algorithmic_flops_per_launch": kflops,
                    "layer_tflops": 2.0 * M * TOPK * 18874368 / 2 / (1e-3 * (w13_mean + sum(w2_ms) / len(w2_ms))) / 1e12}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sub, local_ids = routed_layer_to_cpu(layer, ids)
        per, n = cpu_port_time(M, sub, hidden.cpu(), tw.cpu(), local_ids.cpu(), 1, args.cpu_budget, 1000)
        cpu = {"value": wbytes / per / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
               "sample": f"{n} forwards (~{args.cpu_budget:.0f}s budget) of the numpy oracle (restating "
                         f"bench/bench_moe.py:run_reference with per-call dequant) at M={M}, 1 thread"}

    sweep = None
    if rank == 0 and world == 1 and not args.no_sweep:
        sweep = run_sweep(K, layer, w1r, s1r, w2r, s2r, dev, flush, peaks)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": decode_workload(M),
                       "M": M, "unique_experts": n_act, "weight_bytes_per_step": wbytes,
                       "us_per_layer": 1e3 * total_ms / args.steps,
                       # the fused decode path is one kernel: only its time is a measurement
                       "stage_us": ({"fused_kernel": 1e3 * w13_mean} if fused else
                                    {"align": 1e3 * sum(align_ms) / len(align_ms), "w13": 1e3 * w13_mean,
                                     "w2_and_sum": 1e3 * sum(w2_ms) / len(w2_ms)}),
                       "parallelism": f"replicas x{world}" if world > 1 else "single",
                       "l2": "flushed before every step (256 MiB write, untimed)",
                       "timing": "CUDA-graph replay per step, CUDA events, sum over steps, max over ranks; "
                                 "kernel times from event-bracketed eager launches of the same steps"},
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "us_per_step": 1e3 * e2e_total / args.steps},
            "gpu_launches": (1 if fused else 5) * args.steps,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
            "sweep": sweep,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


SWEEP_MS = (4, 16, 64, 256, 1024, 4096, 16384)


def run_sweep(K, layer, w1r, s1r, w2r, s2r, dev, flush, peaks, reps: int = 5) -> list:
    """Benchmark configurations 2 and 3 on the same layer: per M, the layer's
    device time (CUDA-graph replay, L2 flushed before each step, median of
    `reps`), weight bandwidth and, where the tensor-core path runs, TFLOP/s,
    each against the measured peaks, plus a parity spot check of 4 tokens
    against the fp32 oracle (untimed)."""
    import numpy as np
    import torch

    from kernels.synthetic import make_hidden, make_routing
    from oracle import moe_oracle as O

    out = []
    for M in SWEEP_MS:
        hidden = make_hidden(M, H, device=dev)
        tw, ids = make_routing(M, E, TOPK, device=dev)

        def step():
            return K.fused_experts_w4a16(hidden, w1r, w2r, s1r, s2r, tw, ids)

        for _ in range(3):
            step()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step()
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            o = step()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        times = []
        for _ in range(reps):
            flush.zero_()
            t0.record()
            graph.replay()
            t1.record()
            t1.synchronize()
            times.append(t0.elapsed_time(t1) * 1e3)
        us = sorted(times)[len(times) // 2]
        n_act = int(torch.unique(ids).numel())
        wbytes = n_act * BYTES_PER_EXPERT
        gbs = wbytes / (us * 1e-6) / 1e9
        flops = float(M * TOPK * FLOP_PER_SLOT)
        tflops = flops / (us * 1e-6) / 1e12
        fused = M * TOPK <= 4096
        # parity: 4 tokens against the fp32 oracle on their routed experts
        toks = np.random.default_rng(M).choice(M, size=4, replace=False)
        tt = torch.as_tensor(toks, device=dev)
        sub, local = routed_layer_to_cpu(layer, ids[tt])
        ref = O.moe_reference(hidden[tt].float().cpu().numpy(), sub["w1_q"], sub["w1_s"], sub["w2_q"], sub["w2_s"],
                              tw[tt].float().cpu().numpy(), local.cpu().numpy(), GROUP)
        got = o[tt].float().cpu().numpy()
        rf = float(O.rel_frobenius(got, ref))
        out.append({
            "M": M, "config": 2 if M <= 256 else 3, "path": "fused decode" if fused else "tcgen05 prefill",
            "us_per_layer": us, "unique_experts": n_act, "weight_GBps": gbs,
            "frac_hbm": gbs / peaks["hbm_gbs"], "TFLOPs": tflops, "frac_bf16": tflops / peaks["bf16_tflops"],
            "parity_rel_frobenius_4tok": rf,
        })
        assert rf <= 1e-2, (M, rf)
        del graph, o
    return out


EP_LAYERS, EP_TOKENS = 4, 8192
FLOP_PER_SLOT = 2 * (2 * I * H + H * I)


def run_ep(args) -> int:
    """Benchmark configuration 4: expert-parallel 4-layer stack, M=8192 per step."""
    import torch

    from kernels import ep
    from kernels import w4a16_moe as K
    from kernels.synthetic import make_hidden, make_layer, make_routing, zipf_bias

    world, rank, local = _dist()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    K.load_library()
    assert EP_TOKENS % world == 0 and E % world == 0
    m_src = EP_TOKENS // world
    own = ep.owned_experts(E, world, rank)
    emap = ep.local_expert_map(E, world, rank, dev)
    bias = zipf_bias(E, 1.1, seed=0)
    perm = None
    if args.placement == "balanced" and world > 1:
        # load-aware placement from a calibration batch of the same routing
        # distribution (another seed): a load-time relabelling of the experts
        _, calib = make_routing(EP_TOKENS, E, TOPK, seed=424_242, device="cpu", bias=bias)
        perm = ep.balanced_placement(torch.bincount(calib.flatten().long(), minlength=E), world).to(dev)
    layers, routing = [], []
    for l in range(EP_LAYERS):
        lay = make_layer(len(own), H, I, seed=1000 * l + rank, device=dev)  # this rank's experts only
        w1r, s1r = K.repack_weights(lay["w1_q"], lay["w1_s"])
        w2r, s2r = K.repack_weights(lay["w2_q"], lay["w2_s"])
        del lay
        layers.append(ep.LocalExperts(w1r, s1r, w2r, s2r))
        tw, ids = make_routing(m_src, E, TOPK, seed=7919 * l + 31 * rank, device=dev, bias=bias)
        if perm is not None:  # what the permuted router emits
            ids = perm[ids.long()].to(torch.int32)
        routing.append((tw, ids))
    x0 = make_hidden(m_src, H, seed=rank, device=dev)
    # fixed-capacity exchange (no host read of counts) unless asked otherwise
    cap = m_src if args.ep_exchange == "fixed" else None

    def step(x):
        for l in range(EP_LAYERS):
            x = ep.moe_layer(x, routing[l][0], routing[l][1], layers[l], E, emap, capacity=cap)
        return x

    for _ in range(max(args.warmup, 3)):
        step(x0)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        t0.record()
        for _ in range(args.steps):
            out = step(x0)
        t1.record()
        t1.synchronize()
    _barrier(world)
    my_ms = t0.elapsed_time(t1)
    total_ms = _max_over_ranks(my_ms, world)
    value = EP_TOKENS * args.steps / (total_ms * 1e-3)

    # rows this rank sends per step (dispatch + combine each move them once)
    sent_rows = 0
    for l in range(EP_LAYERS):
        pl = ep.plan(routing[l][1], E)
        sent_rows += sum(c for r, c in enumerate(pl.send_counts) if r != rank)
    nvlink_bytes = 2 * sent_rows * H * 2
    max_sent = _max_over_ranks(float(nvlink_bytes), world)

    # ---- end to end: source tokens from pinned host memory, result back ----
    x_host = x0.cpu().pin_memory()
    out_host = torch.empty((m_src, H), dtype=torch.bfloat16).pin_memory()
    xd = torch.empty_like(x0)
    _barrier(world)
    torch.cuda.synchronize()
    t0.record()
    for _ in range(args.steps):
        xd.copy_(x_host, non_blocking=True)
        o = step(xd)
        out_host.copy_(o, non_blocking=True)
    t1.record()
    t1.synchronize()
    e2e_ms = _max_over_ranks(t0.elapsed_time(t1), world)
    assert torch.isfinite(out.float()).all()

    # ---- per-stage breakdown (separate, untimed pass with stage events) ----
    nst = len(ep.EP_STAGES)
    stage_ms = [0.0] * nst
    reps = min(args.steps, 5)
    for _ in range(reps):
        x = x0
        for l in range(EP_LAYERS):
            evs = [torch.cuda.Event(enable_timing=True) for _ in range(nst + 1)]
            x = ep.moe_layer(x, routing[l][0], routing[l][1], layers[l], E, emap, stage_events=evs, capacity=cap)
            evs[-1].synchronize()
            for i in range(nst):
                stage_ms[i] += evs[i].elapsed_time(evs[i + 1]) / (reps * EP_LAYERS)
    stage_us = {name: 1e3 * _max_over_ranks(v, world) for name, v in zip(ep.EP_STAGES, stage_ms)}
    # expert load: rows and routed slots this rank's experts receive per layer
    recv_rows = sum(sum(ep.plan(routing[l][1], E).recv_counts) for l in range(EP_LAYERS)) / EP_LAYERS
    max_recv_rows = _max_over_ranks(float(recv_rows), world)
    mean_recv_rows = _sum_over_ranks(float(recv_rows), world) / world
    # communicator check: every rank sees the same world through NCCL
    comm_ok = True
    if world > 1:
        import torch.distributed as dist

        t = torch.ones(1, device=dev)
        dist.all_reduce(t)
        comm_ok = int(t.item()) == world == dist.get_world_size()

    # ---- parity spot check (rank 0, untimed): layer 0 on 4 of its tokens vs the oracle ----
    parity = None
    # the layer's exchange is a collective: every rank runs it, rank 0 checks
    x1 = None if args.no_parity else ep.moe_layer(x0, routing[0][0], routing[0][1], layers[0], E, emap, capacity=cap)
    if rank == 0 and not args.no_parity:
        import numpy as np

        from oracle import moe_oracle as O

        sub_tok = 4
        ids_s = routing[0][1][:sub_tok].to(torch.int64).cpu()
        tw_s = routing[0][0][:sub_tok].float().cpu().numpy()
        per = E // world
        used = torch.unique(ids_s)
        ws = {k: [] for k in ("w1_q", "w1_s", "w2_q", "w2_s")}
        owners = sorted({int(e) // per for e in used})
        for r in owners:  # the owner's layer-0 weights (same device generator), routed experts to host
            lay = make_layer(per, H, I, seed=1000 * 0 + r, device=dev)
            for e in used.tolist():
                if e // per == r:
                    for k in ws:
                        ws[k].append((e, lay[k][e % per].cpu()))
            del lay
        for k in ws:  # ascending expert order, as `used`
            ws[k] = [v for _, v in sorted(ws[k], key=lambda ev: ev[0])]
        bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
        w1 = torch.stack(ws["w1_q"]).numpy()
        s1 = bits(torch.stack(ws["w1_s"]))
        w2 = torch.stack(ws["w2_q"]).numpy()
        s2 = bits(torch.stack(ws["w2_s"]))
        local = np.searchsorted(used.numpy(), ids_s.numpy())
        ref = O.moe_reference(x0[:sub_tok].float().cpu().numpy(), w1, s1, w2, s2, tw_s, local, GROUP)
        got = x1[:sub_tok].float().cpu().numpy()
        parity = {"tokens": sub_tok, "layer": 0, "rel_frobenius": float(O.rel_frobenius(got, ref)),
                  "max_abs": float(O.max_abs_err(got, ref)), "tol_rel_frobenius": 1e-2}
        assert parity["rel_frobenius"] <= 1e-2, parity

    peaks = _peaks()
    flops = EP_LAYERS * EP_TOKENS * TOPK * FLOP_PER_SLOT  # whole job per step
    per_gpu_tflops = flops / world / (total_ms / args.steps * 1e-3) / 1e12
    ms_step = total_ms / args.steps
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import moe_oracle as O  # noqa: F401  (checker only)
        sub_tok = 4
        lay0 = make_layer(E, H, I, seed=0, device=dev)
        tw_s, ids_s = routing[0][0][:sub_tok], routing[0][1][:sub_tok]
        subl, lid = routed_layer_to_cpu(lay0, ids_s)
        del lay0
        per, n = cpu_port_time(sub_tok, subl, x0[:sub_tok].cpu(), tw_s.cpu(), lid.cpu(), 1, args.cpu_budget, 1000)
        cpu = {"value": sub_tok / per / EP_LAYERS, "unit": "tokens/s", "cores": 1, "kind": "port",
               "sample": f"{n} numpy-oracle forwards of one layer for {sub_tok} tokens (per-call dequant of "
                         f"their routed experts), scaled to the 4-layer stack, 1 thread"}
    if rank == 0:
        line = {
            "metric": "ep_tokens_per_s", "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": EP_WORKLOAD,
                       "tokens_per_step": EP_TOKENS, "layers": EP_LAYERS, "experts_per_rank": len(own),
                       "parallelism": f"ep{world}", "exchange": args.ep_exchange,
                       "placement": args.placement if world > 1 else "single rank",
                       "l2": "inputs larger than L2 (each layer's expert weights stream from HBM)",
                       "timing": "CUDA events around all steps on each rank, max over ranks",
                       "nvlink_bytes_per_step_max_rank": max_sent,
                       "stage_us_per_layer_max_rank": stage_us,
                       "recv_rows_per_layer": {"max_rank": max_recv_rows, "mean": mean_recv_rows},
                       "comm_nranks_ok": comm_ok, "parity_spot_check": parity},
            "e2e": {"value": EP_TOKENS * args.steps / (e2e_ms * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": m_src * H * 2, "d2h_bytes_per_step": m_src * H * 2,
                    "ms_per_step": e2e_ms / args.steps},
            "gpu_launches": EP_LAYERS * 8 * args.steps,
            "roofline": {"bound": "tensor", "achieved": per_gpu_tflops, "peak": peaks["bf16_tflops_sustained"],
                         "unit": "TFLOP/s", "frac": per_gpu_tflops / peaks["bf16_tflops_sustained"],
                         "traffic": None, "kernel": "whole expert-parallel step (per GPU)",
                         "peak_src": f"{peaks['src']} bf16_tflops_sustained"},
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--M", type=int, default=1, help="tokens per step (config 1: 1)")
    ap.add_argument("--cpu-budget", type=float, default=10.0, help="seconds of CPU baseline sampling")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["decode", "ep"], default=None,
                    help="decode: configs 1-3 (--M); ep: config 4, expert-parallel over the ranks "
                         "(default: ep when launched by torchrun, decode otherwise)")
    ap.add_argument("--no-parity", action="store_true", help="skip the untimed parity spot check")
    ap.add_argument("--no-sweep", action="store_true", help="skip the configuration 2/3 sweep of the N=1 line")
    ap.add_argument("--placement", choices=["balanced", "contiguous"], default="balanced",
                    help="expert-parallel expert placement: balanced by calibration load (a load-time "
                         "relabelling) or contiguous id ranges")
    ap.add_argument("--ep-exchange", choices=["fixed", "counts"], default="fixed",
                    help="ep: fixed-capacity all-to-all (no host sync) or exact counts read back to the host")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        args.warmup = 3
    if args.workload is None:
        # launched by torchrun (WORLD_SIZE set): the multi-GPU configuration 4
        args.workload = "ep" if "WORLD_SIZE" in os.environ else "decode"
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.workload == "ep":
        return run_ep(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
