"""Hard-circuit execution plan: a trained network flattened into a list of kernel
launches over bit-packed activations (the device-side form of
``silogic/bitpacking/convert.py`` + ``packed_model.py``).

Packed activations never leave the GPU between layers; a conv block and its
OR-pool are one launch; GroupSum is a popcount kernel.
"""
import torch

from .. import _hard


#: relabel conv output channels for L2 locality (see _order_channels_for_locality)
LOCALITY_ORDER = True


def _order_channels_for_locality(steps):
    """Relabel the output channels of every conv block that feeds another step so that
    channels reading the same input channels are adjacent.  The conv kernel walks output
    channels in order, so neighbouring CTAs then share input planes in L2 instead of
    fetching them from HBM again; the next step's taps (or the FC head's feature
    indices) are renamed to match, so the circuit and its outputs are unchanged."""
    for i, st in enumerate(steps[:-1]):
        if st["op"] != "conv":
            continue
        kk = st["kernel"] * st["kernel"]
        key = (st["leaf"].long() // kk).min(dim=1).values
        perm = torch.argsort(key, stable=True)                  # new position -> old channel
        inv = torch.empty_like(perm)
        inv[perm] = torch.arange(perm.numel(), device=perm.device)
        st["leaf"], st["tt"] = st["leaf"][perm].contiguous(), st["tt"][perm].contiguous()
        nxt = steps[i + 1]
        if nxt["op"] == "conv":
            kk2 = nxt["kernel"] * nxt["kernel"]
            leaf = nxt["leaf"].long()
            nxt["leaf"] = (inv[leaf // kk2] * kk2 + leaf % kk2).to(torch.int32).contiguous()
        else:
            hw = nxt["in_dim"] // st["n"]                         # pooled positions
            idx = nxt["idx"].long()
            nxt["idx"] = (inv[idx // hw] * hw + idx % hw).to(nxt["idx"].dtype).contiguous()


def validate_steps(steps, width):
    """Check every gather index of a plan against the width it reads (once, at build):
    FC wiring < the layer's input width, conv leaves < cin * k * k.  ``width`` is the
    input feature count (FC) or input channel count (conv)."""
    for i, st in enumerate(steps):
        if st["op"] == "conv":
            kk = st["kernel"] * st["kernel"]
            _hard.check_index_range(st["leaf"], width * kk, f"conv block {i} leaf taps")
            width = st["n"]
        else:
            if "in_dim" in st:
                width = st["in_dim"]
            _hard.check_index_range(st["idx"], width, f"FC layer {i} wiring")
            width = st["idx"].shape[0]


class HardPlan:
    """Wiring + truth tables of every layer, on the parameters' device."""

    #: batches at least this large run an all-FC arity-2 plan as one persistent
    #: kernel (``_hard.FCChain``: activations stay in shared memory between layers);
    #: measured faster than the per-layer kernels from 1,024 samples up
    chain_min_batch = 0

    def __init__(self, steps, in_shape, num_classes, tau):
        self.steps = steps            # list of dicts, see from_model
        self.in_shape = in_shape      # ("fc", F) or ("conv", C, H, W)
        self.num_classes = num_classes
        self.tau = tau
        self.use_chain = True
        self._chain = None
        self._chain_ok = (in_shape[0] == "fc" and
                          _hard.FCChain.supported(steps, in_shape[1], num_classes))

    def chain(self):
        """The fused whole-stack kernel for this plan, or None when it does not apply."""
        if not self._chain_ok:
            return None
        if self._chain is None:
            self._chain = _hard.FCChain(self.steps, self.in_shape[1], self.num_classes,
                                        self.steps[0]["tt"].device)
            if not self._chain.fits:
                self._chain_ok, self._chain = False, None
        return self._chain

    # ----------------------------------------------------------- building
    @classmethod
    @torch.no_grad()
    def from_model(cls, model):
        from ..models import LogicNet, LogicConvNet
        steps = []
        if isinstance(model, LogicNet):
            d_in = model.layers[0].in_dim
            for layer in model.layers:
                idx, tt = layer.hard_spec()
                wr = model.wire_r if (model.wire_r and layer.in_dim == layer.out_dim) else 0
                steps.append(dict(op="fc", idx=idx, tt=tt, wire_r=wr))
            in_shape = ("fc", d_in)
            validate_steps(steps, d_in)
        elif isinstance(model, LogicConvNet):
            convs = [b for b in model.blocks[0::2]]
            pools = [b for b in model.blocks[1::2]]
            first = convs[0]
            for conv, pool in zip(convs, pools):
                leaf, tt = conv.hard_spec()
                steps.append(dict(op="conv", leaf=leaf, tt=tt, arity=conv.node_arity,
                                  depth=conv.d, kernel=conv.kh, pad=conv.padding,
                                  wire_r=model.wire_channels(conv, conv.cin), pool=pool.size,
                                  n=conv.n))
            for layer in model.head_layers:
                idx, tt = layer.hard_spec()
                steps.append(dict(op="fc", idx=idx, tt=tt, wire_r=0, in_dim=layer.in_dim))
            in_shape = ("conv", first.cin, None, None)
            validate_steps(steps, first.cin)
            if LOCALITY_ORDER and all(st["wire_r"] == 0 for st in steps):
                _order_channels_for_locality(steps)
        else:
            raise TypeError(f"unsupported model {type(model).__name__}")
        head = model.head
        nc = getattr(head, "num_classes", None)
        tau = getattr(head, "tau", 1.0)
        return cls(steps, in_shape, nc, tau)

    # ---------------------------------------------------------- execution
    def pack_input(self, x):
        """Pack a binary input batch (``[B, F]`` or ``[B, C, H, W]``)."""
        B = x.shape[0]
        want = self.in_shape[1]
        got = x.shape[1] if x.dim() == 4 else x.reshape(B, -1).shape[1]
        if x.dim() == 4 and self.in_shape[0] == "fc":
            got = x[0].numel()
        if got != want:
            raise ValueError(f"the circuit expects {want} input "
                             f"{'features' if self.in_shape[0] == 'fc' else 'channels'}, got {got}")
        h = _hard.pack(x.reshape(B, -1))
        if x.dim() == 4:
            h = h.view(x.shape[1], x.shape[2], x.shape[3], -1)
        return h

    def run_packed(self, h):
        """Run every layer on packed input ``h``; returns packed ``[width, ldw]``."""
        for st in self.steps:
            if st["op"] == "fc":
                if h.dim() != 2:
                    h = h.reshape(-1, h.shape[-1])
                h = _hard.fc(h, st["idx"], st["tt"], st["wire_r"])
            else:
                h = _hard.conv(h, st["leaf"], st["tt"], st["arity"], st["depth"], st["kernel"],
                               st["pad"], st["wire_r"], st["pool"])
        return h.reshape(-1, h.shape[-1])

    def counts(self, x):
        """Integer GroupSum counts ``[B, num_classes]`` (int32) of binary input ``x``."""
        B = x.shape[0]
        return self.counts_from_packed(self.pack_input(x), B)

    def counts_from_packed(self, h, B, out=None):
        if self.use_chain and B >= self.chain_min_batch and self.chain() is not None:
            return self._chain.counts(h, B, out=out)
        return _hard.groupsum(self.run_packed(h), B, self.num_classes, out=out)

    def features(self, x):
        """Last-layer bits ``[B, width]`` uint8."""
        return _hard.unpack(self.run_packed(self.pack_input(x)), x.shape[0])


class HardGraph:
    """One batch shape of a :class:`HardPlan` captured as a CUDA graph.

    Packing (or the fused thermometer packing), every layer and GroupSum replay as
    one graph launch, so batches whose kernels last a few microseconds are not bound
    by the host's per-kernel launch cost.  ``x`` is the graph's static input: pass
    the tensor that will hold every batch (it is used in place, not copied), or any
    tensor of the right shape and copy batches in with :meth:`__call__`.  ``out``
    optionally names the int32 ``[B, num_classes]`` counts buffer to fill.
    ``thresholds`` / ``mode`` select thermometer input as in ``_hard.thermo_pack``
    (``None``: ``x`` is already binary).  ``tau`` adds a float32 ``logits`` output
    ``counts / tau`` to the graph; ``head`` (a ``PackedLearnedHead``) replaces GroupSum
    and produces ``logits`` only.
    """

    def __init__(self, plan, x, thresholds=None, mode=0, out=None, tau=None, head=None):
        self.plan, self.x, self.thresholds, self.mode, self.tau = plan, x, thresholds, mode, tau
        self.head = head     # a learned bit-packed readout replacing GroupSum (logits only)
        self._out = out
        dev = x.device
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):      # warm-up: caches thresholds, kernel attributes
            self._body()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.counts, self.logits = self._body()

    def _body(self):
        B = self.x.shape[0]
        if self.thresholds is None:
            h = self.plan.pack_input(self.x)
        else:
            h = _hard.thermo_pack(self.x, self.thresholds, mode=self.mode)
            if self.plan.in_shape[0] == "conv" and h.shape[0] != self.plan.in_shape[1]:
                raise ValueError(f"thermometer encoding gives {h.shape[0]} channels, the "
                                 f"circuit expects {self.plan.in_shape[1]}")
        if self.head is not None:
            return None, self.head.apply(self.plan.run_packed(h), B)
        counts = self.plan.counts_from_packed(h, B, out=self._out)
        logits = counts.float() / self.tau if self.tau is not None else None
        return counts, logits

    def replay(self):
        self.graph.replay()
        return self.counts

    def __call__(self, x):
        """Copy ``x`` (device or pinned host tensor) into the static input and replay."""
        if x is not self.x:
            self.x.copy_(x, non_blocking=True)
        self.graph.replay()
        return self.counts
