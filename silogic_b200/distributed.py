"""Batch data parallelism for the logic-gate-network path (one process per GPU).

* Hard inference: samples never interact, so each rank evaluates a contiguous,
  64-sample-aligned shard of the batch and only the ``[B, num_classes]`` int32
  counts are gathered (:func:`gather_counts`).
* Soft training: data parallel with ONE all-reduce per step over a single flat
  bucket of every parameter gradient (:func:`allreduce_gradients`); the bucket is
  a few MB for the BASELINE configs, so latency, not bandwidth, dominates.
Works with any ``torch.distributed`` backend (NCCL on GPUs, gloo in CPU tests).
"""
import torch
import torch.distributed as dist


def shard_range(total, world_size, rank, align=64):
    """``[start, stop)`` of ``rank``'s shard: contiguous, ``align``-aligned starts, the
    remainder spread over the first ranks, so packed words never straddle ranks."""
    units = (total + align - 1) // align
    base, extra = divmod(units, world_size)
    u0 = rank * base + min(rank, extra)
    u1 = u0 + base + (1 if rank < extra else 0)
    return min(total, u0 * align), min(total, u1 * align)


def wire_dtype(max_count):
    """Narrowest integer type that carries counts up to ``max_count`` (a class count is at
    most the group size, e.g. 1,000 for a 10,000-wide layer and 10 classes): int16
    halves the bytes of the gather against int32."""
    return torch.int16 if max_count <= 32767 else torch.int32


def gather_counts(local_counts, total, group=None, max_count=None):
    """All-gather per-rank ``[b_r, C]`` counts into ``[total, C]`` in rank order.  With
    ``max_count`` the counts travel in :func:`wire_dtype` and come back in the input's
    dtype."""
    ws = dist.get_world_size(group)
    C = local_counts.shape[1]
    sizes = [shard_range(total, ws, r)[1] - shard_range(total, ws, r)[0] for r in range(ws)]
    mx = max(sizes)
    wd = wire_dtype(max_count) if max_count is not None else local_counts.dtype
    buf = torch.zeros((mx, C), dtype=wd, device=local_counts.device)
    buf[:local_counts.shape[0]] = local_counts
    raw = buf.view(torch.uint8)                 # bytes on the wire (any backend moves uint8)
    parts = [torch.empty_like(raw) for _ in range(ws)]
    dist.all_gather(parts, raw, group=group)
    return torch.cat([p.view(wd)[:n] for p, n in zip(parts, sizes)], 0).to(local_counts.dtype)


def sharded_hard_counts(plan, x, group=None):
    """Counts of the whole batch ``x`` (present on every rank) computed shard-wise.

    Each rank runs the circuit on its shard only; the result is identical on all
    ranks and equal to ``plan.counts(x)``."""
    ws, rank = dist.get_world_size(group), dist.get_rank(group)
    a, b = shard_range(x.shape[0], ws, rank)
    local = plan.counts(x[a:b]) if b > a else torch.zeros(
        (0, plan.num_classes), dtype=torch.int32, device=x.device)
    steps = getattr(plan, "steps", None)
    width = steps[-1]["idx"].shape[0] if steps and steps[-1]["op"] == "fc" else None
    max_count = width // plan.num_classes if width and plan.num_classes else None
    return gather_counts(local, x.shape[0], group, max_count)


def allreduce_gradients(params, group=None, average=True):
    """One all-reduce of all parameter gradients through a single flat bucket."""
    params = [p for p in params if p.grad is not None]
    if not params:
        return
    flat = torch.cat([p.grad.reshape(-1) for p in params])
    dist.all_reduce(flat, group=group)
    if average:
        flat /= dist.get_world_size(group)
    off = 0
    for p in params:
        n = p.grad.numel()
        p.grad.copy_(flat[off:off + n].view_as(p.grad))
        off += n
