"""Multi-process logic of the data-parallel path on CPU (gloo, world size 2).

No GPU is involved: the sharding/gather/all-reduce helpers are backend-agnostic.
Failure detection is exercised on the host: a rank that never joins a collective
makes the survivor's collective fail within its process-group timeout."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from silogic_b200 import distributed as D


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, ws, port, timeout=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws,
                            timeout=datetime.timedelta(seconds=timeout))


def test_shard_range_covers_batch_aligned():
    for total in (1, 63, 64, 65, 1000, 65536, 1048576):
        for ws in (1, 2, 3, 4, 8):
            spans = [D.shard_range(total, ws, r) for r in range(ws)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            for (a0, b0), (a1, b1) in zip(spans, spans[1:]):
                assert b0 == a1
            assert all(a % 64 == 0 or a == total for a, _ in spans)


def _worker_gather(rank, ws, port, q):
    try:
        _init(rank, ws, port)
        total = 1000
        a, b = D.shard_range(total, ws, rank)
        counts = torch.arange(a, b, dtype=torch.int32).view(-1, 1).repeat(1, 10)
        full = D.gather_counts(counts, total)
        ok = torch.equal(full[:, 0], torch.arange(total, dtype=torch.int32))
        # counts up to 1000 travel as int16 and come back as int32, unchanged
        small = (counts % 1000).contiguous()
        narrow = D.gather_counts(small, total, max_count=1000)
        ok = ok and narrow.dtype == torch.int32 and torch.equal(narrow[:, 0], torch.arange(total) % 1000)
        ok = ok and D.wire_dtype(1000) == torch.int16 and D.wire_dtype(40000) == torch.int32
        # gradient all-reduce: each rank contributes rank+1
        p = torch.nn.Parameter(torch.zeros(3, 4))
        p.grad = torch.full((3, 4), float(rank + 1))
        r = torch.nn.Parameter(torch.zeros(5))
        r.grad = torch.full((5,), 2.0 * (rank + 1))
        D.allreduce_gradients([p, r])
        ok = ok and torch.allclose(p.grad, torch.full((3, 4), 1.5)) and \
            torch.allclose(r.grad, torch.full((5,), 3.0))
        # sharded_hard_counts: each rank runs only its shard (a stand-in plan whose
        # counts are a function of the rows), and every rank gets the whole batch
        seen = []

        class _Plan:
            num_classes = 3

            def counts(self, xs):
                seen.append(xs.shape[0])
                return (xs[:, :3] * 2).to(torch.int32)
        x = torch.arange(777 * 5, dtype=torch.int32).view(777, 5)
        got = D.sharded_hard_counts(_Plan(), x)
        a, b = D.shard_range(777, ws, rank)
        ok = ok and torch.equal(got, (x[:, :3] * 2).to(torch.int32)) and seen == [b - a]
        q.put((rank, bool(ok)))
        dist.destroy_process_group()
    except Exception as e:   # report instead of hanging the parent
        q.put((rank, repr(e)))


def test_gather_counts_and_gradient_allreduce_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker_gather, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert sorted(res) == [(0, True), (1, True)], res


def _worker_dropout(rank, ws, port, q):
    try:
        _init(rank, ws, port, timeout=5)
        if rank == 1:
            q.put((rank, "left"))      # leaves between steps, never joins the collective
            q.close()
            q.join_thread()
            os._exit(0)
        t = torch.ones(4)
        try:
            dist.all_reduce(t)
            q.put((rank, "no error"))
        except Exception as e:
            q.put((rank, "error:" + type(e).__name__))
    except Exception as e:
        q.put((rank, repr(e)))


def test_rank_dropout_is_detected_by_survivor():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker_dropout, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[1] == "left"
    assert res[0].startswith("error"), res
