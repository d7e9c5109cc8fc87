"""Input wiring ("connectomes"), with the reference's names, buffers and seeded draws.

The random candidate draws use the same generator calls in the same order as
``silogic/connectomes.py:37-43,49-55,97-113`` so that a given ``seed`` produces the
same wiring in both libraries (state_dicts are interchangeable).  Layers read
the wiring buffers and run the fused CUDA kernels; ``select_soft`` /
``select_hard`` here are plain tensor-indexing utilities that no layer calls.
"""
import torch
import torch.nn as nn
import torch.nn.functional as F

_ALIASES = {"f": "fixed", "fixed": "fixed", "l": "dense", "dense": "dense",
            "topk": "topk", "blocktopk": "blocktopk", "st": "st", "stw": "stw", "stt": "stt"}


def _candidates(in_dim, out_dim, arity, k, gen):
    """``[out, arity, k]``: per (node, slot) the first k of a random permutation."""
    rows = []
    for _ in range(out_dim):
        rows.append(torch.stack([torch.randperm(in_dim, generator=gen)[:k]
                                 for _ in range(arity)]))
    return torch.stack(rows)


class FixedConnectome(nn.Module):
    """One random wire per (node, slot)."""

    kind = "fixed"

    def __init__(self, in_dim, out_dim, arity, gen=None):
        super().__init__()
        self.in_dim, self.out_dim, self.arity = in_dim, out_dim, arity
        idx = torch.randint(0, in_dim, (out_dim, arity), generator=gen)
        self.register_buffer("idx", idx)
        self.register_buffer("cand_i32", idx.unsqueeze(-1).to(torch.int32))

    def candidates_i32(self):
        return self.cand_i32

    def weights(self):
        return torch.ones(self.out_dim, self.arity, 1, device=self.idx.device)

    def hard_index(self):
        return self.idx

    def select_soft(self, x):
        return x[:, self.idx]

    select_hard = select_soft


class DenseConnectome(nn.Module):
    """Softmax over every input per slot; hard path = argmax wire."""

    kind = "dense"

    def __init__(self, in_dim, out_dim, arity, gen=None):
        super().__init__()
        self.in_dim, self.out_dim, self.arity = in_dim, out_dim, arity
        self.conn = nn.Parameter(torch.randn(out_dim, arity, in_dim, generator=gen) * 0.1)

    def hard_index(self):
        return self.conn.argmax(dim=2)

    def select_soft(self, x):
        return torch.einsum("bi,oai->boa", x, F.softmax(self.conn, dim=2))

    def select_hard(self, x):
        return x[:, self.hard_index()]


class TopKConnectome(nn.Module):
    """Each slot mixes ``k`` random candidates with a learnable softmax."""

    kind = "topk"

    def __init__(self, in_dim, out_dim, arity, k, gen=None, block=False, window=0):
        super().__init__()
        self.in_dim, self.out_dim, self.arity = in_dim, out_dim, arity
        kk = min(k, in_dim)
        self.k = kk
        if block:
            Wn = min(in_dim, window if window else max(4 * kk, 256))
            starts = (torch.arange(out_dim).float() / max(1, out_dim)
                      * max(1, in_dim - Wn)).long()
            cand = torch.stack([
                torch.stack([starts[o] + torch.randperm(Wn, generator=gen)[:kk]
                             for _ in range(arity)]) for o in range(out_dim)])
        else:
            cand = _candidates(in_dim, out_dim, arity, kk, gen)
        self.register_buffer("cand", cand)
        self.register_buffer("cand_i32", cand.to(torch.int32))
        self.conn = nn.Parameter(torch.randn(out_dim, arity, kk, generator=gen))
        self.ste = False

    def weights(self):
        w = F.softmax(self.conn, dim=2)
        if self.ste:
            hard = F.one_hot(self.conn.argmax(dim=2), w.shape[-1]).to(w.dtype)
            w = hard + w - w.detach()
        return w

    def candidates_i32(self):
        return self.cand_i32

    def hard_index(self):
        sel = self.conn.argmax(dim=2)
        return torch.gather(self.cand, 2, sel.unsqueeze(-1)).squeeze(-1)

    def select_soft(self, x):
        return torch.einsum("boak,oak->boa", x[:, self.cand], self.weights())

    def select_hard(self, x):
        return x[:, self.hard_index()]


class SumThresholdConnectome(nn.Module):
    """Sum-threshold inputs (BNN-style).  Kept for checkpoint compatibility; it has
    no static wiring, so no kernel of this package evaluates it."""

    kind = "sumthreshold"

    def __init__(self, in_dim, out_dim, arity, k, mode="none", gen=None):
        super().__init__()
        self.in_dim, self.out_dim, self.arity, self.mode = in_dim, out_dim, arity, mode
        kk = min(k, in_dim)
        self.k = kk
        self.register_buffer("cand", _candidates(in_dim, out_dim, arity, kk, gen))
        self.bn = nn.ModuleList([nn.BatchNorm1d(out_dim) for _ in range(arity)])
        if mode != "none":
            scale = 0.1 if mode == "binary" else 1.0
            self.w = nn.Parameter(torch.randn(out_dim, arity, kk) * scale)


def build_connectome(kind, in_dim, out_dim, arity=2, k=8, seed=None, window=0):
    """Construct a connectome by name (same names and aliases as the reference)."""
    key = _ALIASES.get(str(kind).lower())
    if key is None:
        raise ValueError(f"unknown connectome {kind!r}")
    gen = torch.Generator().manual_seed(seed) if seed is not None else None
    if key == "fixed":
        return FixedConnectome(in_dim, out_dim, arity, gen)
    if key == "dense":
        return DenseConnectome(in_dim, out_dim, arity, gen)
    if key == "topk":
        return TopKConnectome(in_dim, out_dim, arity, k, gen)
    if key == "blocktopk":
        return TopKConnectome(in_dim, out_dim, arity, k, gen, block=True, window=window)
    mode = {"st": "none", "stw": "binary", "stt": "ternary"}[key]
    return SumThresholdConnectome(in_dim, out_dim, arity, k, mode=mode, gen=gen)
