"""Benchmark of the silogic_b200 hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c2|c1|c3|c4|c5] [--no-soft]

Workload (default): FC LogicNet 784 -> 10000 x 6, Walsh nodes,
Top-K (k=8) wiring, GroupSum 10 classes tau=10, every parameter N(0,1) (seeded),
inputs Bernoulli(0.3) (seeded, synthetic).
  * headline step = hard bit-packed inference of 65,536 samples per GPU
    (pack -> 6 FC layers -> popcount GroupSum);
  * "soft" = soft forward + backward of 4,096 samples per GPU (+ one NCCL
    all-reduce of the parameter gradients when N > 1).
Timing: CUDA events around each step on the launching stream, L2 flushed (a
256 MB write) between steps, W warm-up steps; barrier + synchronize around the
timed loop; the max over ranks is reported.  e2e = the same work through the
public API from pinned host memory (H2D of the uint8 batch, D2H of the logits)
inside the timed region.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    "c2": dict(ctor="LogicNet", kwargs=dict(in_dim=784, width=10000, depth=6, node="walsh",
                                             connectome="topk", k=8, tau=10.0, seed=0),
               hard_batch=65536, soft_batch=4096,
               name="C2 FC LogicNet 784->10000x6 walsh topk8 GroupSum10 tau10"),
    "c1": dict(ctor="LogicNet", kwargs=dict(in_dim=784, width=8000, depth=4, node="gate16",
                                             connectome="fixed", tau=10.0, seed=0),
               hard_batch=1024, soft_batch=1024,
               name="C1 FC LogicNet 784->8000x4 gate16 fixed GroupSum10 tau10"),
}


# ------------------------------------------------------------------ helpers
def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def build_model(cfg, seed=0):
    import silogic_b200 as S
    torch.manual_seed(seed)
    m = getattr(S, cfg["ctor"])(**cfg["kwargs"])
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for p in m.parameters():
            p.copy_(torch.randn(p.shape, generator=g))
    return m


def make_input(cfg, B, seed):
    g = torch.Generator().manual_seed(seed)
    F = cfg["kwargs"]["in_dim"]
    return (torch.rand(B, F, generator=g) < 0.3).to(torch.uint8)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.rows, self._stop = index, [], threading.Event()

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                      "--format=csv,noheader,nounits"], capture_output=True,
                                     text=True, timeout=5).stdout.strip()
                if out:
                    self.rows.append([s.strip() for s in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self.t.join(timeout=10)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4)
                          if len(r) > 3 + i and r[3 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(self.rows)}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ------------------------------------------------------------------ hard leg
class KernelTimer:
    """CUDA events around launches of one kernel on the current stream."""

    def __init__(self):
        self.pairs = []

    def start(self):
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    def stop(self, e0):
        e1 = torch.cuda.Event(enable_timing=True)
        e1.record()
        self.pairs.append((e0, e1))

    def mean_ms(self):
        return statistics.mean(a.elapsed_time(b) for a, b in self.pairs) if self.pairs else None


def run_hard(cfg, B, steps, warmup, rank, ws, dev):
    from silogic_b200 import _hard
    from silogic_b200.bitpacking import convert_logic_net
    from silogic_b200.bitpacking.plan import HardPlan
    model = build_model(cfg).to(dev)
    plan = HardPlan.from_model(model)
    bp = convert_logic_net(model)
    x_host = make_input(cfg, B, seed=1 + rank).pin_memory()
    x_dev = x_host.to(dev)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.int32, device=dev)   # 256 MB > L2
    in_dim, width = cfg["kwargs"]["in_dim"], cfg["kwargs"]["width"]
    fc_timer = KernelTimer()
    launches = [0]

    def step_device():
        h = plan.pack_input(x_dev)
        launches[0] += 1
        for i, st in enumerate(plan.steps):
            t0 = fc_timer.start() if i > 0 else None
            h = _hard.fc(h, st["idx"], st["tt"], st["wire_r"])
            if t0 is not None:
                fc_timer.stop(t0)
            launches[0] += 1
        c = _hard.groupsum(h, B, plan.num_classes)
        launches[0] += 1
        return c

    def step_e2e():
        # public API: host uint8 in (pinned), logits out to host
        out = bp.forward(x_host.to(dev, non_blocking=True))
        return out.to("cpu", non_blocking=True)

    ref = step_device()
    torch.cuda.synchronize()
    for _ in range(warmup):
        step_device()
        step_e2e()
    torch.cuda.synchronize()
    fc_timer.pairs.clear()
    launches[0] = 0
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    times = []
    with ClockSampler(torch.cuda.current_device()) as clk:
        torch.cuda.nvtx.range_push("timed_hard")
        for _ in range(steps):
            flush.fill_(1)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            step_device()
            e1.record()
            times.append((e0, e1))
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        ms = statistics.mean(a.elapsed_time(b) for a, b in times)
        e2e_times = []
        for _ in range(steps):
            flush.fill_(1)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            out = step_e2e()
            e1.record()
            e1.synchronize()
            e2e_times.append(e0.elapsed_time(e1))
        e2e_ms = statistics.mean(e2e_times)
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    fc_ms = fc_timer.mean_ms()
    nw = (B + 63) // 64
    return dict(ms=ms, e2e_ms=e2e_ms, fc_ms=fc_ms, launches_per_step=launches[0] / steps,
                clocks=clk.summary(), counts=ref,
                h2d=int(x_host.numel()), d2h=int(B * plan.num_classes * 4),
                fc_bytes=(width + width) * nw * 8)


# ------------------------------------------------------------------ soft leg
def soft_bytes_per_sample(cfg):
    """Layer-wise algorithmic fp32 bytes per sample of soft fwd+bwd (each stage reads its
    inputs once and writes its outputs once; the data input needs no gradient)."""
    kw = cfg["kwargs"]
    dims = [kw["in_dim"]] + [kw["width"]] * kw["depth"]
    fwd = sum((a + b) * 4 for a, b in zip(dims[:-1], dims[1:]))
    bwd = sum((b + a + (a if i > 0 else 0)) * 4 for i, (a, b) in enumerate(zip(dims[:-1], dims[1:])))
    W = dims[-1]
    return fwd + bwd + (4 * W + 40) * 2


def run_soft(cfg, B, steps, warmup, rank, ws, dev):
    model = build_model(cfg).to(dev).train()
    x = make_input(cfg, B, seed=100 + rank).float().to(dev)
    g = torch.Generator().manual_seed(5)
    rmat = torch.randn(B, 10, generator=g).to(dev)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.int32, device=dev)
    params = [p for p in model.parameters()]
    bucket = None

    def step():
        nonlocal bucket
        for p in params:
            p.grad = None
        logits = model(x)
        (logits * rmat).sum().backward()
        if ws > 1:      # data parallel: one all-reduce of every parameter gradient
            bucket = torch.cat([p.grad.reshape(-1) for p in params])
            torch.distributed.all_reduce(bucket)
        return logits

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
    times = []
    torch.cuda.nvtx.range_push("timed_soft")
    for _ in range(steps):
        flush.fill_(1)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        step()
        e1.record()
        times.append((e0, e1))
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    ms = statistics.mean(a.elapsed_time(b) for a, b in times)
    return dict(ms=ms)


# ------------------------------------------------------------ CPU baselines
_SPEC_CACHE = {}


def cpu_hard_sample(cfg, n_samples, threads=1):
    """Oracle (numpy bit-packed restatement of the reference) on a bounded sample."""
    from concurrent.futures import ThreadPoolExecutor
    from oracle import hard as OH
    from oracle.spec import net_spec
    key = cfg["name"]
    if key not in _SPEC_CACHE:
        model = build_model(cfg)
        sd = {k: v.numpy() for k, v in model.state_dict().items()}
        _SPEC_CACHE[key] = (net_spec(cfg["ctor"], cfg["kwargs"], sd),
                            make_input(cfg, n_samples, seed=1).numpy())
    spec, x = _SPEC_CACHE[key]
    chunk = max(64, (n_samples // threads) // 64 * 64)
    parts = [x[i:i + chunk] for i in range(0, n_samples, chunk)]
    t0 = time.perf_counter()
    with ThreadPoolExecutor(max_workers=threads) as ex:
        list(ex.map(lambda p: OH.net_counts(spec, p), parts))
    dt = time.perf_counter() - t0
    return n_samples / dt, dt


# ------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS))
    ap.add_argument("--cpu-sample", type=int, default=4096)
    ap.add_argument("--no-soft", action="store_true")
    a = ap.parse_args()
    cfg = CONFIGS[a.config]
    ws, rank, local = dist_env()
    warmup = max(3, a.warmup)
    metric = "hard-circuit samples/s (bit-packed inference)"

    if a.impl == "reference":
        if rank != 0:
            return
        threads = os.cpu_count() or 1
        vals = []
        for _ in range(warmup):
            cpu_hard_sample(cfg, a.cpu_sample, threads)
        for _ in range(a.steps):
            v, _ = cpu_hard_sample(cfg, a.cpu_sample, threads)
            vals.append(v)
        v = statistics.mean(vals)
        line = {"metric": metric, "value": v, "unit": "samples/s", "n_gpus": a.gpus,
                "steps": a.steps, "warmup": warmup, "ms_per_step": a.cpu_sample / v * 1e3,
                "higher_is_better": True, "impl": "reference", "dtype": "u64",
                "data": "synthetic", "config": {"workload": cfg["name"], "batch": a.cpu_sample},
                "cpu_baseline": {"value": v, "unit": "samples/s", "cores": threads, "kind": "port",
                                 "sample": f"{a.cpu_sample} samples per step, numpy bit-packed "
                                           f"restatement of the reference, {threads} threads"},
                "e2e": {"value": v, "unit": "samples/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    if ws > 1:
        torch.distributed.init_process_group("nccl")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    B = cfg["hard_batch"]
    r = run_hard(cfg, B, a.steps, warmup, rank, ws, dev)
    soft = None
    if not a.no_soft:
        soft = run_soft(cfg, cfg["soft_batch"], a.steps, warmup, rank, ws, dev)
    ms = torch.tensor([r["ms"], r["e2e_ms"], soft["ms"] if soft else 0.0], device=dev)
    if ws > 1:
        torch.distributed.all_reduce(ms, op=torch.distributed.ReduceOp.MAX)
    ms_step, e2e_ms, soft_ms = ms.tolist()
    hbm, kind = peaks()
    fc_gbs = r["fc_bytes"] / (r["fc_ms"] * 1e-3) / 1e9
    if rank == 0:
        line = {
            "metric": metric, "value": B * ws / (ms_step * 1e-3), "unit": "samples/s",
            "n_gpus": ws, "steps": a.steps, "warmup": warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u64",
            "data": "synthetic (Bernoulli(0.3) inputs, N(0,1) parameters, seeded)",
            "config": {"workload": cfg["name"], "batch_per_gpu": B, "global_batch": B * ws,
                       "parallelism": f"batch-shard x{ws}", "l2": "flushed (256 MB write) between steps"},
            "e2e": {"value": B * ws / (e2e_ms * 1e-3), "unit": "samples/s",
                    "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"]},
            "gpu_launches": int(round(r["launches_per_step"] * a.steps)),
            "roofline": {"kernel": "slg_fc_hard (layers 2-6)", "bound": "hbm",
                         "achieved": fc_gbs, "peak": hbm, "unit": "GB/s", "frac": fc_gbs / hbm,
                         "peak_kind": kind, "traffic": None,
                         "algorithmic_bytes_per_launch": r["fc_bytes"]},
            "clocks": r["clocks"],
        }
        if soft:
            Bs = cfg["soft_batch"]
            bps = soft_bytes_per_sample(cfg)
            ach = bps * Bs / (soft_ms * 1e-3) / 1e9
            line["soft_fwd_bwd"] = {
                "metric": "soft fwd+bwd samples/s", "value": Bs * ws / (soft_ms * 1e-3),
                "unit": "samples/s", "ms_per_step": soft_ms, "batch_per_gpu": Bs, "dtype": "f32",
                "roofline": {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s",
                             "frac": ach / hbm, "algorithmic_bytes_per_sample": bps,
                             "scope": "whole step (layer-wise bytes)"},
                "collective": "one NCCL all-reduce of all parameter gradients" if ws > 1 else None}
        if ws == 1:
            v, dt = cpu_hard_sample(cfg, a.cpu_sample, 1)
            line["cpu_baseline"] = {"value": v, "unit": "samples/s", "cores": 1, "kind": "port",
                                    "sample": f"{a.cpu_sample} samples, numpy bit-packed "
                                              f"restatement of the reference ({dt:.2f} s)"}
        print(json.dumps(line))
    if ws > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
