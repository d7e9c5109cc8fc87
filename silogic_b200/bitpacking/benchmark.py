"""Inference-speed benchmark helpers with the API of ``silogic/bitpacking/benchmark.py``
(``run_benchmark``, ``run_conv_benchmark``, ``print_report``, ``speedup_summary``,
``BenchResult``), measuring this package's CUDA paths.

Rows per batch size:
  * ``soft (float32)``             -- ``model(x)`` (fused soft kernels), no grad;
  * ``hard uint8 (CUDA)``          -- ``model.forward_hard(x)`` (pack, one kernel per
                                      layer, GroupSum; the reference's "hard uint8 (torch)");
  * ``bitpacked GPU (CUDA graph)`` -- the converted net, numpy uint8 in -> numpy logits
                                      out, every layer replayed as one CUDA graph;
  * ``bitpacked GPU resident``     -- the same circuit on a device-resident batch
                                      (counts only; no host copies).
There is no CPU path in this package, so ``device`` must be ``"cuda"``.  Timing follows
the reference: warm-up runs, then the mean and standard deviation of ``n_runs`` (CUDA
events for device work, wall clock for the numpy-in/numpy-out call).
"""
import gc
import time
from collections import defaultdict
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from .convert import convert_logic_net, convert_logic_conv_net

HARD_ROW = "hard uint8 (CUDA)"
BITPACKED_ROW = "bitpacked GPU (CUDA graph)"


def _time_host(fn, n_warmup=3, n_runs=20):
    for _ in range(n_warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(n_runs):
        t0 = time.perf_counter()
        fn()
        torch.cuda.synchronize()
        ts.append((time.perf_counter() - t0) * 1e3)
    a = np.asarray(ts)
    return float(a.mean()), float(a.std())


def _time_cuda(fn, n_warmup=3, n_runs=20):
    for _ in range(n_warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(n_runs):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        ts.append(s.elapsed_time(e))
    a = np.asarray(ts)
    return float(a.mean()), float(a.std())


@dataclass
class BenchResult:
    """One timed method at one batch size (``benchmark.py:64-81``)."""
    name: str
    batch_size: int
    mean_ms: float
    std_ms: float
    throughput_kps: float     # thousands of samples per second
    accuracy: Optional[float] = None
    extra: dict = field(default_factory=dict)

    def as_row(self) -> str:
        acc = f"{self.accuracy * 100:.2f}%" if self.accuracy is not None else "  n/a  "
        return (f"  {self.name:<28s}  {self.batch_size:>6d}  {self.mean_ms:>9.3f}ms ± "
                f"{self.std_ms:>6.3f}  {self.throughput_kps:>10.1f}  {acc}")


def _row(name, B, ms, sd, acc=None, **extra):
    return BenchResult(name=name, batch_size=B, mean_ms=ms, std_ms=sd,
                       throughput_kps=B / (ms / 1e3) / 1e3, accuracy=acc, extra=dict(extra))


def _acc(logits, y):
    if y is None:
        return None
    logits = logits.cpu().numpy() if torch.is_tensor(logits) else np.asarray(logits)
    return float((logits.argmax(1) == y).mean())


def _run(model, convert, x_test, y_test, batch_sizes, device, n_warmup, n_runs):
    if not str(device).startswith("cuda"):
        raise RuntimeError("silogic_b200 runs on CUDA only (no CPU implementation); pass device='cuda'")
    results: List[BenchResult] = []
    model.eval()
    dev = torch.device(device)
    model.to(dev)
    bp = convert(model)
    for B in batch_sizes:
        idx = np.arange(B) % len(x_test)
        x_b = np.ascontiguousarray(x_test[idx])
        y_b = y_test[idx] if y_test is not None else None
        x_float = torch.from_numpy(x_b).float().to(dev)
        x_u8 = torch.from_numpy(x_b).to(torch.uint8).to(dev)
        with torch.no_grad():
            m, s = _time_cuda(lambda: model(x_float), n_warmup, n_runs)
            results.append(_row("soft (float32)", B, m, s))
            m, s = _time_cuda(lambda: model.forward_hard(x_u8), n_warmup, n_runs)
            results.append(_row(HARD_ROW, B, m, s, _acc(model.forward_hard(x_u8), y_b)))
        m, s = _time_host(lambda: bp(x_b), n_warmup, n_runs)
        results.append(_row(BITPACKED_ROW, B, m, s, _acc(bp(x_b), y_b),
                            path="numpy uint8 in -> numpy float32 logits out"))
        m, s = _time_cuda(lambda: bp.counts(x_u8), n_warmup, n_runs)
        results.append(_row("bitpacked GPU resident", B, m, s, _acc(bp.counts(x_u8), y_b)))
        gc.collect()
    return results


def run_benchmark(model, x_test: np.ndarray, y_test: Optional[np.ndarray],
                  batch_sizes: Tuple[int, ...] = (64, 512, 2048, 8192), device: str = "cuda",
                  include_gpu: bool = True, n_warmup: int = 3, n_runs: int = 20) -> List[BenchResult]:
    """Benchmark a ``LogicNet``: soft, hard and bit-packed inference on ``x_test``
    ``[N, in_dim]`` uint8 (``benchmark.py:84-211``).  ``include_gpu`` is accepted for
    signature parity: every path here is a GPU path."""
    return _run(model, convert_logic_net, x_test, y_test, batch_sizes, device,
                n_warmup, n_runs)


def run_conv_benchmark(model, x_test: np.ndarray, y_test: Optional[np.ndarray],
                       H_in: Optional[int] = None, W_in: Optional[int] = None,
                       batch_sizes: Tuple[int, ...] = (64, 256, 1024, 4096), device: str = "cuda",
                       include_gpu: bool = True, n_warmup: int = 3,
                       n_runs: int = 20) -> List[BenchResult]:
    """Benchmark a ``LogicConvNet`` on ``x_test`` ``[N, C, H, W]`` uint8
    (``benchmark.py:249-367``)."""
    return _run(model, convert_logic_conv_net, x_test, y_test, batch_sizes, device,
                n_warmup, n_runs)


def print_report(results: List[BenchResult], title: str = "Inference Speed Report") -> None:
    """Print the results grouped by batch size (``benchmark.py:379-398``)."""
    header = "  {:<28s}  {:>6s}  {:>16s}  {:>10s}  {:>7s}".format(
        "Method", "Batch", "Latency (ms)", "Throughput", "Accuracy")
    rule = "  " + "-" * 80
    print()
    print("=" * 84)
    print(f"  {title}")
    print("=" * 84)
    last = None
    for r in results:
        if r.batch_size != last:
            if last is not None:
                print(rule)
            print(f"\n  Batch size = {r.batch_size}")
            print(header)
            print(rule)
            last = r.batch_size
        print(r.as_row())
        for k, v in r.extra.items():
            print(f"      └─ {k}: {v}")
    print("=" * 84)
    print()


def speedup_summary(results: List[BenchResult]) -> Dict[int, Dict[str, float]]:
    """Per batch size: hard-path and bit-packed throughput (k samples/s) and the
    bit-packed speed-up over the hard path (``benchmark.py:401-416``; same keys)."""
    by_batch: Dict[int, Dict[str, float]] = defaultdict(dict)
    for r in results:
        by_batch[r.batch_size][r.name] = r.throughput_kps
    out = {}
    for B, methods in by_batch.items():
        base = methods.get(HARD_ROW, methods.get("hard uint8 (torch)", 1.0))
        bp = methods.get(BITPACKED_ROW, methods.get("bitpacked CPU (gate-grouped)", 0.0))
        out[B] = {"hard_kps": round(base, 1), "bitpacked_kps": round(bp, 1),
                  "speedup_x": round(bp / base, 2) if base > 0 else 0.0}
    return out
