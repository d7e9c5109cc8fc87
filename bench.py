"""Benchmark of the silogic_b200 hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c1|c2|c3|c4|c5] [--extras c2,..|none] [--no-soft]
                    [--no-cpu] [--no-reference-gpu] [--batch B]

Configs are BASELINE.json's (synthetic, seeded inputs; every parameter N(0,1)):
  c1  FC LogicNet 784 -> 8000 x 4, gate16, fixed wiring; hard + soft at B=1024
  c2  FC LogicNet 784 -> 10000 x 6, Walsh, Top-K 8; hard bit-packed inference at
      B=65,536 per GPU, soft fwd+bwd at B=4,096 per GPU (weak scaling)
  c3  LogicTreeNet 3x32x32 thermometer (5 thresholds) -> gate16 trees depth 2,
      channels 128/256/512 + OR-pool, head 1280; B=4,096
  c4  LogicConvNet, learned thermometer (3 bits), multilinear arity-6 trees,
      channels 128/256, head 16000 x 2, STE selection; B=8,192
  c5  (default, the headline: the largest single-GPU config) LogicTreeNet 3x32x32
      thermometer (31 thresholds), gate16 depth 2, channels 1024/2048/4096/8192,
      head 12800/6400/3200; 1,048,576 samples split across the GPUs (strong
      scaling), processed in 131,072-sample device chunks
With the default c5 headline, c2 (hard + soft) is measured in the same run and
reported under the key "c2".
A "step" is one pass of the hard circuit over the per-GPU batch (value); the
soft fwd+bwd leg (key "soft_fwd_bwd") is one forward + backward of its batch,
plus one NCCL all-reduce of the parameter gradients when N > 1.  Hard inference
shards the batch and all-gathers only the class counts.
Timing: CUDA events on the launching stream around each step, L2 flushed (a
256 MB write read back, untimed) before each step, W >= 3 warm-up steps, barrier +
synchronize around the timed loop, max over ranks.  "e2e" runs the same work
through the public API from pinned host memory with the host<->device copies
inside the timed region; image configs send uint8 pixels (pixel k = fp32 k/255, as
torchvision's ToTensor gives), and "e2e_f32" sends the same images as fp32.  "parity" compares (untimed) the timed step's counts of
the first 128 samples with the CPU oracle; "cpu_baseline" times the reference's
own CPU path (baseline/_ref) on a bounded sample of the same batch and says
whether its counts equal the GPU's.
--impl reference times the reference's own CPU path (rank 0 only) on a bounded
sample per step.  At N=1 the reference's own GPU (Triton) path is also timed, in a
child process, under "reference_gpu" (--no-reference-gpu skips it).
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

FIVE = [1 / 6, 2 / 6, 3 / 6, 4 / 6, 5 / 6]
THIRTY_ONE = [(i + 1) / 32 for i in range(31)]

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the dominant
# kernel, averaged over the launches of one step, from one ncu capture of the same
# command (the summaries under profiles/ name the command and list the figures).
NCU_TRAFFIC = {
    ("c2", "fc_chain"): (6.73e6, "profiles/fc_chain_c2_b65536.md"),
    ("c4", "conv_hard"): ((9.517e6 + 33.738e6) / 2, "profiles/conv_hard_c4_b8192.md"),
    # four C5 blocks captured at 32,768 samples, scaled x4 to the 131,072-sample chunk
    ("c5", "conv_hard"): (4.80e9, "profiles/conv_gate2_c5_b32768.md"),
}

CONFIGS = {
    "c1": dict(ctor="LogicNet", inp="bern",
               kwargs=dict(in_dim=784, width=8000, depth=4, node="gate16", connectome="fixed",
                           tau=10.0, seed=0),
               hard_batch=1024, soft_batch=1024, scaling="weak",
               name="C1 FC LogicNet 784->8000x4 gate16 fixed GroupSum10 tau10"),
    "c2": dict(ctor="LogicNet", inp="bern",
               kwargs=dict(in_dim=784, width=10000, depth=6, node="walsh", connectome="topk", k=8,
                           tau=10.0, seed=0),
               hard_batch=65536, soft_batch=4096, scaling="weak",
               name="C2 FC LogicNet 784->10000x6 walsh topk8 GroupSum10 tau10"),
    "c3": dict(ctor="LogicTreeNet", inp="image", thresholds=FIVE,
               kwargs=dict(in_channels=15, in_hw=32, channels=[128, 256, 512], head_widths=[1280],
                           tree_depth=2, node="gate16", tau=20.0, seed=0),
               hard_batch=4096, soft_batch=4096, scaling="weak",
               name="C3 LogicTreeNet 3x32x32 thermo5 gate16 d2 [128,256,512]+OrPool head1280"),
    "c4": dict(ctor="LogicConvNet", inp="encoder", bits=3,
               kwargs=dict(in_channels=9, in_hw=32, channels=[128, 256], head_widths=[16000, 16000],
                           tree_depth=1, node="multilinear", arity=6, connect="topk", k=8, n_chan=4,
                           gate_select="hard", tau=12.0, seed=0),
               hard_batch=8192, soft_batch=8192, scaling="weak",
               name="C4 LogicConvNet learned-thermo3 multilinear a6 d1 [128,256] head 16000x2"),
    "c5": dict(ctor="LogicTreeNet", inp="image", thresholds=THIRTY_ONE,
               kwargs=dict(in_channels=93, in_hw=32, channels=[1024, 2048, 4096, 8192],
                           head_widths=[12800, 6400, 3200], head_connect="F", tree_depth=2,
                           node="gate16", tau=20.0, seed=0),
               hard_batch=1048576, soft_batch=0, scaling="strong", chunk=131072,
               name="C5 LogicTreeNet 3x32x32 thermo31 gate16 d2 [1024..8192] head 12800/6400/3200"),
}


# ------------------------------------------------------------------ helpers
def dist_env():
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def build_model(cfg, seed=0):
    import silogic_b200 as S
    torch.manual_seed(seed)
    m = getattr(S, cfg["ctor"])(**cfg["kwargs"])
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for p in m.parameters():
            p.copy_(torch.randn(p.shape, generator=g))
    enc = None
    if cfg["inp"] == "encoder":
        enc = S.LearnedThermometerEncoder(3 * 32 * 32, cfg["bits"])
    return m, enc


def make_input(cfg, B, seed):
    """Synthetic batch: Bernoulli(0.3) features (uint8), or uniform 3x32x32 uint8 pixels,
    the form CIFAR images are stored in; pixel k stands for the fp32 value k / 255 that
    torchvision's ToTensor gives (``image_float``)."""
    g = torch.Generator().manual_seed(seed)
    if cfg["inp"] == "bern":
        return (torch.rand(B, cfg["kwargs"]["in_dim"], generator=g) < 0.3).to(torch.uint8)
    return torch.randint(0, 256, (B, 3, 32, 32), generator=g, dtype=torch.uint8)


def image_float(x):
    """uint8 pixels -> the fp32 images k / 255 (ToTensor) that float-input paths take."""
    return x.float() / 255 if x.dtype == torch.uint8 else x


class ClockSampler:
    """nvidia-smi clocks / throttle reasons every 200 ms during the timed region."""

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
        num = lambda s: s.replace(".", "", 1).isdigit()
        sm = [float(r[0]) for r in self.rows if num(r[0])]
        mx = [float(r[1]) for r in self.rows if num(r[1])]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4)
                          if len(r) > 3 + i and r[3 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(self.rows)}


_SYNC = None


def flush_l2(buf):
    """Evict the step's data from L2 before a timed step: write a buffer larger than L2,
    then read it back, so L2 ends up holding clean lines of the flush buffer and the
    step does not pay for writing back the flush's own dirty lines."""
    buf.fill_(1)
    buf.sum()
    # With several ranks, line their streams up after the flush (a one-element
    # all-reduce, untimed) so a step's time does not include another rank's flush.
    if torch.distributed.is_initialized() and torch.distributed.get_world_size() > 1:
        global _SYNC
        if _SYNC is None or _SYNC.device != buf.device:
            _SYNC = torch.zeros(1, device=buf.device)
        torch.distributed.all_reduce(_SYNC)


def soak_until_sampled(step, clk, min_s=1.0, min_samples=4):
    """Untimed extra warm-up steps until the clock sampler has seen the GPU under this
    load (at least ``min_s`` seconds and ``min_samples`` samples), so a step much
    shorter than the 200 ms sampling period still gets a clock record."""
    t0 = time.perf_counter()
    n0 = len(clk.rows)
    while True:
        for _ in range(8):
            step()
        torch.cuda.synchronize()
        if time.perf_counter() - t0 >= min_s and len(clk.rows) - n0 >= min_samples:
            return
        if time.perf_counter() - t0 > 10 * min_s:
            return


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def events():
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


# ------------------------------------------------------- algorithmic bytes
def hard_stage_bytes(cfg, plan):
    """Layer-wise algorithmic bytes PER SAMPLE of each hard stage: every stage reads its
    input bits once and writes its output bits once; the first stage reads the raw
    input (uint8 features, or uint8 pixels for the image configs)."""
    out = []
    if cfg["inp"] == "bern":
        F = cfg["kwargs"]["in_dim"]
        out.append(("pack", F + F / 8))
        bits = F
    else:
        T = len(cfg["thresholds"]) if cfg["inp"] == "image" else cfg["bits"]
        out.append(("pack", 3 * 32 * 32 + 3 * T * 32 * 32 / 8))
        bits, hw = 3 * T * 32 * 32, 32
    for st in plan.steps:
        if st["op"] == "fc":
            o = st["idx"].shape[0]
            out.append(("fc_hard", (bits + o) / 8))
            bits = o
        else:
            hw //= st["pool"]
            o = st["n"] * hw * hw
            out.append(("conv_hard", (bits + o) / 8))
            bits = o
    out.append(("groupsum", bits / 8 + 40))
    return out


def soft_bytes_per_sample(cfg, model):
    """Layer-wise fp32 bytes per sample of soft fwd+bwd: fwd (in + out) * 4 per layer,
    bwd (out + in + in) * 4 (the data input needs no gradient; the learned encoder's
    does), conv blocks count their pooled output, GroupSum 4W + 40 each way."""
    from silogic_b200.layers import ConvLogicTree
    if cfg["ctor"] == "LogicNet":
        dims = [cfg["kwargs"]["in_dim"]] + [L.out_dim for L in model.layers]
    else:
        hw = cfg["kwargs"]["in_hw"]
        dims = [cfg["kwargs"]["in_channels"] * hw * hw]
        for b in model.blocks:
            if isinstance(b, ConvLogicTree):
                hw //= 2
                dims.append(b.n * hw * hw)
        dims += [L.out_dim for L in model.head_layers]
    first_grad = cfg["inp"] == "encoder"
    fwd = sum((a + b) * 4 for a, b in zip(dims[:-1], dims[1:]))
    bwd = sum((b + a + (a if (i > 0 or first_grad) else 0)) * 4
              for i, (a, b) in enumerate(zip(dims[:-1], dims[1:])))
    return fwd + bwd + 2 * (4 * dims[-1] + 40)


# ------------------------------------------------------------------ hard leg
def run_hard(cfg, B, steps, warmup, rank, ws, dev):
    from silogic_b200 import _hard
    from silogic_b200.bitpacking import convert_logic_net, convert_logic_conv_net
    from silogic_b200.bitpacking.plan import HardPlan, HardGraph
    model, enc = build_model(cfg)
    model = model.to(dev)
    plan = HardPlan.from_model(model)
    bp = convert_logic_net(model) if cfg["ctor"] == "LogicNet" else convert_logic_conv_net(model)
    chunk = min(B, cfg.get("chunk", B))
    x_host = make_input(cfg, chunk, seed=1 + rank).pin_memory()
    x_dev = x_host.to(dev)
    thr = None
    if cfg["inp"] == "image":
        thr = list(cfg["thresholds"])
    elif cfg["inp"] == "encoder":
        thr = enc.thresholds.detach().to(dev).contiguous()
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.int32, device=dev)   # 256 MB > L2
    timers = {}
    launches = [0]
    nchunks = (B + chunk - 1) // chunk
    counts_all = torch.empty((B, plan.num_classes), dtype=torch.int32, device=dev)
    # counts cross NVLink in the narrowest type that holds them (int16 for <= 32767 per class)
    from silogic_b200.distributed import wire_dtype
    last = plan.steps[-1]
    wdt = wire_dtype(last["idx"].shape[0] // plan.num_classes if last["op"] == "fc" else 1 << 30)
    gathered = torch.empty((ws * B, plan.num_classes), dtype=wdt, device=dev) if ws > 1 else None
    mode = 0 if cfg["inp"] == "image" else 1

    def pack_chunk(n):
        if cfg["inp"] == "bern":
            return plan.pack_input(x_dev[:n])
        return _hard.thermo_pack(x_dev[:n], thr, mode=mode)

    def timed(name, fn, record):
        if not record:
            return fn()
        # keep the GPU busy while the host enqueues, so the events bracket the
        # kernel alone and not the host's launch gap
        torch.cuda._sleep(200_000)
        e0, e1 = events()
        e0.record()
        r = fn()
        e1.record()
        timers.setdefault(name, []).append((e0, e1))
        return r

    def uses_chain(n):
        return plan.use_chain and n >= plan.chain_min_batch and plan.chain() is not None

    def step_eager(record=False):
        """Kernel-by-kernel launch of one step (per-kernel timing pass)."""
        for c in range(nchunks):
            n = min(chunk, B - c * chunk)
            h = timed("pack", lambda: pack_chunk(n), record)
            if uses_chain(n):
                timed("fc_chain", lambda: plan.chain().counts(h, n, out=counts_all[c * chunk:c * chunk + n]),
                      record)
                continue
            for st in plan.steps:
                hh = h
                if st["op"] == "fc":
                    hh = h.reshape(-1, h.shape[-1])
                    h = timed("fc_hard", lambda: _hard.fc(hh, st["idx"], st["tt"], st["wire_r"]), record)
                else:
                    h = timed("conv_hard", lambda: _hard.conv(hh, st["leaf"], st["tt"], st["arity"],
                                                              st["depth"], st["kernel"], st["pad"],
                                                              st["wire_r"], st["pool"]), record)
            hh = h.reshape(-1, h.shape[-1])
            timed("groupsum", lambda: _hard.groupsum(hh, n, plan.num_classes,
                                                      out=counts_all[c * chunk:c * chunk + n]), record)

    # one CUDA graph per chunk shape over the resident input: pack, every layer and
    # GroupSum replay as one launch
    graph_thr = None if cfg["inp"] == "bern" else thr
    graphs = {}
    for c in range(nchunks):
        n = min(chunk, B - c * chunk)
        if n not in graphs:
            graphs[n] = HardGraph(plan, x_dev[:n], graph_thr, mode)

    def step_device(collective=True):
        for c in range(nchunks):
            n = min(chunk, B - c * chunk)
            counts_all[c * chunk:c * chunk + n].copy_(graphs[n].replay())
            launches[0] += 2 if uses_chain(n) else 2 + len(plan.steps)
        if ws > 1 and collective:   # only the class counts leave the GPU
            # bytes on the wire: neither NCCL nor gloo moves int16 itself
            torch.distributed.all_gather_into_tensor(gathered.view(torch.uint8),
                                                     counts_all.to(wdt).view(torch.uint8))
        return counts_all

    # the same images as fp32 k / 255 on the host, for the fp32-input end-to-end figure
    # (one GPU only: 4x the pinned host memory of the uint8 batch per rank)
    x_host_f32 = image_float(x_host).pin_memory() if cfg["inp"] != "bern" and ws == 1 else None

    def step_e2e(src=x_host):
        outs = []
        for c in range(nchunks):
            n = min(chunk, B - c * chunk)
            xd = src[:n]        # pinned host batch: copied into the graph's static input
            if cfg["inp"] == "bern":
                outs.append(bp.forward(xd).to("cpu", non_blocking=True))
            else:
                outs.append(bp.forward_images(xd, thr, mode=mode).to("cpu", non_blocking=True))
        return outs

    step_device()
    torch.cuda.synchronize()
    for _ in range(warmup):
        step_device()
        step_e2e()
    torch.cuda.synchronize()
    launches[0] = 0
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    times = []
    with ClockSampler(torch.cuda.current_device()) as clk:
        soak_until_sampled(lambda: step_device(collective=False), clk)
        launches[0] = 0
        if ws > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("timed_hard")
        for _ in range(steps):
            flush_l2(flush)
            e0, e1 = events()
            e0.record()
            step_device()
            e1.record()
            times.append((e0, e1))
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        ms = statistics.mean(a.elapsed_time(b) for a, b in times)
        e2e_times = []
        for _ in range(steps):
            flush_l2(flush)
            e0, e1 = events()
            e0.record()
            step_e2e()
            e1.record()
            e1.synchronize()
            e2e_times.append(e0.elapsed_time(e1))
        e2e_ms = statistics.mean(e2e_times)
        e2e_f32_ms = 0.0
        if x_host_f32 is not None:
            step_e2e(x_host_f32)
            torch.cuda.synchronize()
            e2e_times = []
            for _ in range(steps):
                flush_l2(flush)
                e0, e1 = events()
                e0.record()
                step_e2e(x_host_f32)
                e1.record()
                e1.synchronize()
                e2e_times.append(e0.elapsed_time(e1))
            e2e_f32_ms = statistics.mean(e2e_times)
            del x_host_f32
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    step_eager()                # allocator warm-up for the eager pass
    torch.cuda.synchronize()
    for _ in range(steps):      # per-kernel durations, outside the headline region
        flush_l2(flush)
        step_eager(record=True)
    torch.cuda.synchronize()
    kern = {k: (sum(a.elapsed_time(b) for a, b in v) / steps, len(v) / steps) for k, v in timers.items()}
    stage = hard_stage_bytes(cfg, plan)
    per_kind = {}
    for name, bps in stage:
        per_kind[name] = per_kind.get(name, 0.0) + bps
    # the fused whole-stack kernel is credited with the layer-wise bytes of the
    # stages it replaces (every FC layer and the GroupSum)
    per_kind["fc_chain"] = per_kind.get("fc_hard", 0.0) + per_kind.get("groupsum", 0.0)
    in_bytes = x_host[:1].numel() * x_host.element_size()
    step_device(collective=False)
    torch.cuda.synchronize()
    return dict(ms=ms, e2e_ms=e2e_ms, e2e_f32_ms=e2e_f32_ms, kern=kern, per_kind=per_kind, x_first=x_host,
                counts_first=counts_all[:chunk].cpu(), enc=enc, model=model,
                bytes_per_sample=sum(b for _, b in stage), launches_per_step=launches[0] / steps,
                clocks=clk.summary(), h2d=int(in_bytes * B), d2h=int(B * plan.num_classes * 4))


# ------------------------------------------------------------------ soft leg
def run_soft(cfg, B, steps, warmup, rank, ws, dev):
    import silogic_b200 as S
    model, enc = build_model(cfg)
    model = model.to(dev).train()
    if enc is not None:
        enc = enc.to(dev)
    x = make_input(cfg, B, seed=100 + rank).to(dev)
    if cfg["inp"] == "bern":
        x = x.float()
    elif cfg["inp"] == "image":
        x = S.binarize_spatial(image_float(x), cfg["thresholds"]).float()
    else:
        x = image_float(x).reshape(B, -1)
    rmat = torch.randn(B, 10, generator=torch.Generator().manual_seed(5)).to(dev)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.int32, device=dev)
    params = list(model.parameters()) + (list(enc.parameters()) if enc is not None else [])

    def step():
        for p in params:
            p.grad = None
        xi = x
        if enc is not None:
            xi = enc(x).view(B, 3, 32, 32, cfg["bits"]).permute(0, 1, 4, 2, 3).reshape(B, -1, 32, 32)
        logits = model(xi)
        (logits * rmat).sum().backward()
        if ws > 1:      # data parallel: one all-reduce of every parameter gradient
            from silogic_b200.distributed import allreduce_gradients
            allreduce_gradients(params)
        return logits

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
    times = []
    torch.cuda.nvtx.range_push("timed_soft")
    for _ in range(steps):
        flush_l2(flush)
        e0, e1 = events()
        e0.record()
        step()
        e1.record()
        times.append((e0, e1))
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    return dict(ms=statistics.mean(a.elapsed_time(b) for a, b in times),
                bytes_per_sample=soft_bytes_per_sample(cfg, model))


# ------------------------------------------------------------ CPU baselines
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def import_reference():
    """The unmodified reference package installed in baseline/_ref (pure Python:
    numpy for the bit-packed CPU path, Triton for its GPU path), or None."""
    if not os.path.isdir(os.path.join(REF_DIR, "silogic")):
        return None
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    try:
        import silogic
    except Exception:
        return None
    return silogic


def reference_net(silogic, cfg, seed=0):
    """The config's network built with the REFERENCE's own constructors and the same
    seeded N(0,1) parameters as build_model (identical state_dicts)."""
    torch.manual_seed(seed)
    m = getattr(silogic, cfg["ctor"])(**cfg["kwargs"])
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for p in m.parameters():
            p.copy_(torch.randn(p.shape, generator=g))
    from silogic.bitpacking import convert_logic_net, convert_logic_conv_net
    bp = convert_logic_net(m) if cfg["ctor"] == "LogicNet" else convert_logic_conv_net(m)
    enc = None
    if cfg["inp"] == "encoder":
        torch.manual_seed(seed)
        enc = silogic.LearnedThermometerEncoder(3 * 32 * 32, cfg["bits"])
    return m, bp, enc


def reference_cpu_step(silogic, cfg, bp, enc, x):
    """One pass of the reference's fastest CPU path over host batch ``x`` through its
    public API: the input encoding (``binarize_spatial`` / the learned encoder) and
    ``BitpackedNet`` / ``BitpackedConvNet`` (``bitpacking/packed_model.py``).  Returns
    integer counts (logits x tau)."""
    if cfg["inp"] == "bern":
        xb = x.numpy()
    elif cfg["inp"] == "image":
        from silogic.data import binarize_spatial
        xb = binarize_spatial(image_float(x), cfg["thresholds"]).numpy()
    else:
        n = x.shape[0]
        e = enc.forward_hard(image_float(x).reshape(n, -1))
        xb = e.view(n, 3, 32, 32, cfg["bits"]).permute(0, 1, 4, 2, 3).reshape(n, -1, 32, 32).numpy()
    return np.rint(bp(xb) * cfg["kwargs"]["tau"]).astype(np.int64)


def cpu_port_sample(cfg, x):
    """The numpy restatement of the reference's bit-packed path (oracle/hard.py) on
    host batch ``x``; returns integer counts."""
    from oracle import hard as OH
    from oracle.spec import net_spec
    model, enc = build_model(cfg)
    sd = {k: v.numpy() for k, v in model.state_dict().items()}
    spec = net_spec(cfg["ctor"], cfg["kwargs"], sd)
    n = x.shape[0]
    xn = x.numpy() if cfg["inp"] == "bern" else image_float(x).numpy()
    if cfg["inp"] == "image":
        xn = OH.thermometer_bits(xn, cfg["thresholds"])
    elif cfg["inp"] == "encoder":
        e = OH.learned_thermometer_bits(xn.reshape(n, -1), enc.thresholds.detach().numpy())
        xn = e.reshape(n, 3, 32, 32, cfg["bits"]).transpose(0, 1, 4, 2, 3).reshape(n, -1, 32, 32)
    return OH.net_counts(spec, xn)


# bounded CPU samples (about 5-15 s of the reference's CPU path on a 32-core host)
CPU_SAMPLE = {"c1": 8192, "c2": 65536, "c3": 1024, "c4": 256, "c5": 2048}


def cpu_baseline(cfg_key, cfg, x_host, counts):
    """Time the reference's CPU path (baseline/_ref) on the first samples of the GPU
    batch and check that it gives the same counts as the GPU; falls back to the numpy
    port when the reference is not installed."""
    n = min(CPU_SAMPLE[cfg_key], x_host.shape[0])
    x = x_host[:n].clone()
    silogic = import_reference()
    threads = torch.get_num_threads()
    if silogic is not None:
        m, bp, enc = reference_net(silogic, cfg)
        reference_cpu_step(silogic, cfg, bp, enc, x[:64])         # warm-up
        t0 = time.perf_counter()
        ref = reference_cpu_step(silogic, cfg, bp, enc, x)
        dt = time.perf_counter() - t0
        kind, what = "reference", ("the reference's own CPU path from baseline/_ref: input "
                                   "encoding + BitpackedNet/BitpackedConvNet (numpy)")
    else:
        t0 = time.perf_counter()
        ref = cpu_port_sample(cfg, x)
        dt = time.perf_counter() - t0
        kind, what, threads = "port", "the numpy restatement of the reference (oracle/hard.py)", 1
    same = bool(np.array_equal(ref, counts[:n].numpy().astype(np.int64)))
    return {"value": n / dt, "unit": "samples/s", "cores": threads, "kind": kind,
            "sample": f"{n} samples of the same batch through {what}, {dt:.2f} s, "
                      f"torch threads {threads}, host cpus {os.cpu_count()}",
            "counts_equal_gpu": same}


SOFT_CPU_SAMPLE = {"c1": 256, "c2": 64, "c3": 8, "c4": 2}


def soft_cpu_baseline(cfg):
    """The reference's soft training step on the host cores: ``model(x)`` and
    ``.backward()`` through its own PyTorch path (baseline/_ref; its fused kernels need
    CUDA, so the CPU path is the eager one), on a bounded batch of the config."""
    silogic = import_reference()
    if silogic is None:
        return {"unavailable": "reference not installed in baseline/_ref"}
    key = [k for k, v in CONFIGS.items() if v is cfg or v["name"] == cfg["name"]][0]
    n = SOFT_CPU_SAMPLE[key]
    m, _, enc = reference_net(silogic, cfg)
    m.train()
    x = make_input(cfg, n, seed=100)
    if cfg["inp"] == "bern":
        x = x.float()
    elif cfg["inp"] == "image":
        from silogic.data import binarize_spatial
        x = binarize_spatial(image_float(x), cfg["thresholds"]).float()
    else:
        x = image_float(x)
    rmat = torch.randn(n, 10, generator=torch.Generator().manual_seed(5))

    def step():
        m.zero_grad()
        (m(x) * rmat).sum().backward()
    step()
    t0 = time.perf_counter()
    step()
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": "samples/s", "cores": torch.get_num_threads(),
            "kind": "reference", "sample": f"{n} samples, one model(x) + backward of the "
            f"reference's PyTorch path (baseline/_ref) on the host, {dt:.2f} s"}


def parity_check(cfg, x_host, counts, n=128):
    """Untimed: the GPU counts of the first ``n`` samples of the timed batch against the
    oracle (numpy restatement of the reference's bit-packed path)."""
    n = min(n, x_host.shape[0])
    ref = cpu_port_sample(cfg, x_host[:n].clone())
    got = counts[:n].numpy().astype(np.int64)
    return {"samples": n, "oracle": "oracle/hard.py", "equal": bool(np.array_equal(ref, got))}


def reference_gpu(cfg_key, batch, steps=3, warmup=1):
    """The reference's own GPU (Triton) bit-packed path on this box, in a child
    process, as a same-hardware bar: ``BitpackedConvGPUNet`` (conv configs) or
    ``BitpackedNet`` layers on ``BitpackedGPULayer`` (FC configs)."""
    cmd = [sys.executable, os.path.abspath(__file__), "--impl", "reference-gpu", "--config", cfg_key,
           "--batch", str(batch), "--steps", str(steps), "--warmup", str(warmup)]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
        lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
        if r.returncode == 0 and lines:
            return json.loads(lines[-1])
        err = (r.stderr.strip().splitlines() or ["no output"])[-1]
        return {"unavailable": f"exit {r.returncode}: {err[:300]}"}
    except subprocess.TimeoutExpired:
        return {"unavailable": "timed out after 900 s"}


def run_reference_gpu(cfg_key, cfg, a):
    """Child process of reference_gpu(): time the reference's Triton path end to end
    through its public API (numpy uint8 in, numpy logits out; host packing included,
    as in the reference's own benchmark harness, bitpacking/benchmark.py)."""
    silogic = import_reference()
    if silogic is None:
        print(json.dumps({"unavailable": "reference not installed in baseline/_ref"}))
        return
    from silogic.bitpacking import HAS_TRITON
    if not HAS_TRITON:
        print(json.dumps({"unavailable": "reference Triton path not importable on this box"}))
        return
    m, bp, enc = reference_net(silogic, cfg)
    B = a.batch
    x = make_input(cfg, B, seed=1)
    if cfg["inp"] == "bern":
        xb = x.numpy()
        from silogic.bitpacking.kernels import BitpackedGPULayer
        from silogic.bitpacking.ops import pack_bits, mask_last_word
        layers = [BitpackedGPULayer.from_fc_layer(L, "cuda") for L in bp.packed_layers]

        def run():
            h = torch.from_numpy(pack_bits(xb)).cuda()
            for L in layers:
                h = L.forward(h)
            p = h.cpu().numpy()
            mask_last_word(p, B)
            return bp.head.forward(p, B)
        what = "BitpackedGPULayer per FC layer (Triton) + host pack/head"
    else:
        from silogic.bitpacking import BitpackedConvGPUNet, packed_unfold_gpu, packed_or_pool_gpu
        from silogic.bitpacking.packed_layer import pack_conv_input
        from silogic.bitpacking.ops import n_words
        from silogic.data import binarize_spatial
        xb = binarize_spatial(image_float(x), cfg["thresholds"]).numpy()
        gnet = BitpackedConvGPUNet.from_conv_net(bp, 32, 32, "cuda")
        run = lambda: gnet(xb)
        what = "BitpackedConvGPUNet (Triton gate trees, torch unfold/OR-pool) + host pack/head"
        # the same network's device work alone, from the packed input already on the GPU:
        # the sequence BitpackedConvGPUNet.forward runs (packed_model.py:523-600), timed
        # with CUDA events
        x3 = torch.from_numpy(pack_conv_input(xb, n_words(B))).cuda()

        def device_only():
            h = x3
            for (H_, W_, Ho, Wo, ps), gl in zip(gnet.block_spatial, gnet.gpu_conv_layers):
                u = packed_unfold_gpu(h, gl.kh, gl.kw, gl.stride, gl.padding, H_, W_)
                h = packed_or_pool_gpu(gl.forward_packed(u), Ho, Wo, ps)
            h = h.reshape(-1, h.shape[-1]).contiguous()
            for gl in gnet.gpu_head_layers:
                h = gl.forward(h)
            return h
    for _ in range(warmup_n(a)):
        out = run()
    torch.cuda.synchronize()
    ts = []
    for _ in range(a.steps):
        t0 = time.perf_counter()
        out = run()
        torch.cuda.synchronize()
        ts.append(time.perf_counter() - t0)
    device_ms = None
    if cfg["inp"] != "bern":
        device_only()
        torch.cuda.synchronize()
        evs = []
        for _ in range(a.steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            device_only()
            e1.record()
            evs.append((e0, e1))
        torch.cuda.synchronize()
        device_ms = statistics.mean(p.elapsed_time(q) for p, q in evs)
    counts = np.rint(out * cfg["kwargs"]["tau"]).astype(np.int64)
    ours_ok = None
    try:
        ours_ok = bool(np.array_equal(counts[:128], cpu_port_sample(cfg, x[:128].clone())))
    except Exception:
        pass
    dt = statistics.mean(ts)
    extra = {}
    if device_ms is not None:
        extra = {"device_only": {"value": B / (device_ms * 1e-3), "unit": "samples/s",
                                 "ms": device_ms, "what": "the reference's conv/head kernels on a "
                                 "GPU-resident packed input (CUDA events), no host pack or head"}}
    print(json.dumps({**extra, "value": B / dt, "unit": "samples/s", "batch": B, "ms_per_step": dt * 1e3,
                      "path": what, "timing": "host wall clock around the reference's numpy-in/"
                      "numpy-out call (its own API), mean of steps", "counts_equal_oracle_128": ours_ok}))


def warmup_n(a):
    return max(1, a.warmup)


# ----------------------------------------------------------- one config, ours
def measure_ours(cfg_key, cfg, a, ws, rank, dev, warmup, with_soft=True, check=True):
    """Hard (and optionally soft) legs of one config; MAX over ranks of every time."""
    B = cfg["hard_batch"] // (ws if cfg["scaling"] == "strong" else 1)
    r = run_hard(cfg, B, a.steps, warmup, rank, ws, dev)
    soft = None
    if with_soft and cfg["soft_batch"]:
        soft = run_soft(cfg, cfg["soft_batch"], a.steps, warmup, rank, ws, dev)
    ms = torch.tensor([r["ms"], r["e2e_ms"], soft["ms"] if soft else 0.0, r["e2e_f32_ms"]],
                      device=dev)
    if ws > 1:
        torch.distributed.all_reduce(ms, op=torch.distributed.ReduceOp.MAX)
    ms_step, e2e_ms, soft_ms, e2e_f32_ms = ms.tolist()
    hbm, kind = peaks()
    dom = max(r["kern"], key=lambda k: r["kern"][k][0])
    dom_ms, dom_n = r["kern"][dom]
    dom_bytes = r["per_kind"][dom] * B
    ach = dom_bytes / (dom_ms * 1e-3) / 1e9
    total = B * ws if cfg["scaling"] == "weak" else cfg["hard_batch"]
    out = {
        "value": total / (ms_step * 1e-3), "ms_per_step": ms_step, "B": B, "total": total,
        "e2e": {"value": total / (e2e_ms * 1e-3), "unit": "samples/s",
                "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"]},
        "e2e_f32": ({"value": total / (e2e_f32_ms * 1e-3), "unit": "samples/s",
                     "h2d_bytes_per_step": r["h2d"] * 4, "d2h_bytes_per_step": r["d2h"],
                     "input": "the same images as fp32 k/255 from pinned host memory"}
                    if e2e_f32_ms > 0 else None),
        "gpu_launches": int(round(r["launches_per_step"] * a.steps)),
        "roofline": {"kernel": f"slg_{dom} ({dom_n:.0f} launches/step)", "bound": "hbm",
                     "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                     "peak_kind": kind,
                     "traffic": NCU_TRAFFIC.get((cfg_key, dom), (None,))[0] if not a.batch else None,
                     "traffic_source": NCU_TRAFFIC.get((cfg_key, dom), (None, None))[1],
                     "algorithmic_bytes_per_step": dom_bytes,
                     "step_frac": r["bytes_per_sample"] * B / (ms_step * 1e-3) / 1e9 / hbm,
                     "algorithmic_bytes_per_sample": r["bytes_per_sample"]},
        "kernels_ms_per_step": {k: v[0] for k, v in r["kern"].items()},
        "clocks": r["clocks"], "r": r,
    }
    if soft:
        Bs = cfg["soft_batch"]
        ach_s = soft["bytes_per_sample"] * Bs / (soft_ms * 1e-3) / 1e9
        out["soft_fwd_bwd"] = {
            "metric": "soft fwd+bwd samples/s", "value": Bs * ws / (soft_ms * 1e-3),
            "unit": "samples/s", "ms_per_step": soft_ms, "batch_per_gpu": Bs, "dtype": "f32",
            "roofline": {"bound": "hbm (layer-wise bytes; gathers are L2-bound)",
                         "achieved": ach_s, "peak": hbm, "unit": "GB/s", "frac": ach_s / hbm,
                         "algorithmic_bytes_per_sample": soft["bytes_per_sample"]},
            "collective": "one NCCL all-reduce of all parameter gradients" if ws > 1 else None}
    if check and rank == 0:
        out["parity"] = parity_check(cfg, r["x_first"], r["counts_first"])
    return out


# ------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-gpu"])
    ap.add_argument("--config", default="c5", choices=sorted(CONFIGS))
    ap.add_argument("--extras", default=None,
                    help="comma list of further configs measured in the same run "
                         "(default: c2 when the headline is c5; 'none' for none)")
    ap.add_argument("--no-soft", action="store_true")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip the reference's Triton path (timed in a child process, N=1 only)")
    ap.add_argument("--soft-only", action="store_true", help="profile the soft leg alone")
    ap.add_argument("--soft-batch", type=int, default=None,
                    help="soft fwd+bwd batch (default: the config's; smaller for profiling)")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the hard batch (small cases for profiling)")
    a = ap.parse_args()
    cfg = dict(CONFIGS[a.config])
    if a.soft_batch:
        cfg["soft_batch"] = a.soft_batch
    if a.batch:
        cfg["hard_batch"] = a.batch
        cfg["chunk"] = min(cfg.get("chunk", a.batch), a.batch)
    ws, rank, local = dist_env()
    warmup = max(3, a.warmup)
    metric = "hard-circuit samples/s (bit-packed inference)"

    if a.impl == "reference-gpu":
        run_reference_gpu(a.config, cfg, a)
        return

    if a.impl == "reference":
        # the reference's own CPU path on the host cores, rank 0 only
        if rank != 0:
            return
        silogic = import_reference()
        n = CPU_SAMPLE[a.config] // (4 if a.config == "c5" else 1)
        x = make_input(cfg, n, seed=1)
        if silogic is not None:
            m, bp, enc = reference_net(silogic, cfg)
            step = lambda: reference_cpu_step(silogic, cfg, bp, enc, x)
            kind = "reference"
            what = ("the reference's CPU path from baseline/_ref (input encoding + "
                    "BitpackedNet/BitpackedConvNet, numpy)")
        else:
            step = lambda: cpu_port_sample(cfg, x)
            kind, what = "port", "the numpy restatement of the reference (oracle/hard.py)"
        for _ in range(warmup):
            step()
        ts = []
        for _ in range(a.steps):
            t0 = time.perf_counter()
            step()
            ts.append(time.perf_counter() - t0)
        v = n / statistics.mean(ts)
        threads = torch.get_num_threads()
        print(json.dumps({
            "metric": metric, "value": v, "unit": "samples/s", "n_gpus": ws, "steps": a.steps,
            "warmup": warmup, "ms_per_step": statistics.mean(ts) * 1e3, "higher_is_better": True,
            "impl": "reference", "dtype": "u64", "data": "synthetic",
            "config": {"workload": cfg["name"], "batch": n,
                       "sample": f"{n} samples per step (bounded sample of the workload)"},
            "cpu_baseline": {"value": v, "unit": "samples/s", "cores": threads, "kind": kind,
                             "sample": f"{n} samples per step through {what}; torch threads "
                                       f"{threads}, host cpus {os.cpu_count()}"},
            "e2e": {"value": v, "unit": "samples/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}))
        return

    if ws > 1:
        if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
            os.environ["NCCL_DEBUG"] = "WARN"      # keep stdout to the one JSON line
    torch.cuda.set_device(local)
    if ws > 1:
        torch.distributed.init_process_group("nccl", device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    if a.soft_only:
        soft = run_soft(cfg, cfg["soft_batch"], a.steps, warmup, rank, ws, dev)
        if rank == 0:
            print(json.dumps({"metric": "soft fwd+bwd samples/s", "config": cfg["name"],
                              "value": cfg["soft_batch"] * ws / (soft["ms"] * 1e-3),
                              "ms_per_step": soft["ms"]}))
        return
    res = measure_ours(a.config, cfg, a, ws, rank, dev, warmup, with_soft=not a.no_soft)
    if a.extras is None:
        extras = ["c2"] if (a.config == "c5" and not a.batch) else []
    else:
        extras = [e for e in a.extras.split(",") if e and e != "none"]
    extra_res = {}
    for e in extras:
        torch.cuda.empty_cache()
        extra_res[e] = measure_ours(e, dict(CONFIGS[e]), a, ws, rank, dev, warmup,
                                    with_soft=not a.no_soft)
    if rank == 0:
        line = {
            "metric": metric, "value": res["value"], "unit": "samples/s", "n_gpus": ws,
            "steps": a.steps, "warmup": warmup, "ms_per_step": res["ms_per_step"],
            "higher_is_better": True, "scaling": cfg["scaling"], "vs_baseline": None,
            "dtype": "u64", "data": "synthetic (seeded inputs, N(0,1) parameters)",
            "config": {"workload": cfg["name"], "batch_per_gpu": res["B"],
                       "input": ("seeded uint8 3x32x32 pixels, pixel k = fp32 k/255 (ToTensor); the "
                                 "reference arms take the same images as fp32"
                                 if cfg["inp"] != "bern" else "seeded Bernoulli(0.3) uint8 features"),
                       "global_batch": res["total"],
                       "parallelism": f"batch shard x{ws}, counts all-gathered (int16 on the wire)",
                       "l2": "flushed before each step (256 MB write, then read back so L2 is clean)",
                       "launch": "one CUDA graph per chunk shape (pack + every layer + GroupSum)",
                       "clocks": "sampled over >= 1 s of untimed replays of the same step, then the timed steps"},
            "e2e": res["e2e"], "e2e_f32": res.get("e2e_f32"), "gpu_launches": res["gpu_launches"], "roofline": res["roofline"],
            "kernels_ms_per_step": res["kernels_ms_per_step"], "clocks": res["clocks"],
            "parity": res.get("parity"),
        }
        if "soft_fwd_bwd" in res:
            line["soft_fwd_bwd"] = res["soft_fwd_bwd"]
        for e, er in extra_res.items():
            line[e] = {k: er[k] for k in ("value", "ms_per_step", "e2e", "roofline", "parity",
                                          "kernels_ms_per_step", "soft_fwd_bwd") if k in er}
            line[e].update(workload=CONFIGS[e]["name"], batch_per_gpu=er["B"],
                           scaling=CONFIGS[e]["scaling"], unit="samples/s")
        if ws == 1 and not a.no_cpu:
            for e, er in extra_res.items():
                if "soft_fwd_bwd" in er:
                    line[e]["soft_fwd_bwd"]["cpu_baseline"] = soft_cpu_baseline(CONFIGS[e])
            r = res["r"]
            line["cpu_baseline"] = cpu_baseline(a.config, cfg, r["x_first"], r["counts_first"])
            for e, er in extra_res.items():
                line[e]["cpu_baseline"] = cpu_baseline(e, CONFIGS[e], er["r"]["x_first"],
                                                       er["r"]["counts_first"])
        if ws == 1 and not a.no_reference_gpu and not a.batch:
            keys = list(extra_res)
            del res, extra_res
            torch.cuda.empty_cache()
            line["reference_gpu"] = reference_gpu(a.config, 16384 if a.config == "c5" else 65536)
            for e in keys:
                line[e]["reference_gpu"] = reference_gpu(e, 16384 if e == "c5" else 65536)
        print(json.dumps(line))
    if ws > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
