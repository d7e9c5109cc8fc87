"""Bit-packed inference objects with the API of ``silogic/bitpacking/packed_model.py``,
``packed_layer.py`` and ``kernels/triton_*.py`` -- all evaluated by the CUDA kernels.

Inputs may be numpy arrays (copied to the GPU; results copied back to numpy, as
the reference's CPU classes return) or CUDA tensors (results stay on the GPU).
"""
import numpy as np
import torch

from .. import _hard
from ..functional import gate16_lut_codes
from .plan import HardGraph


def _dev(device=None):
    return torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())


def _as_cuda(x, device=None):
    if isinstance(x, np.ndarray):
        return torch.from_numpy(np.ascontiguousarray(x)).to(_dev(device), non_blocking=True)
    return x


def _plan_device(plan):
    for st in plan.steps:
        return st["tt"].device
    return _dev()


def _packed_in(x, device=None):
    """numpy/torch ``[rows, nw]`` int64 -> CUDA ``[rows, ldw]`` (ldw even), plus nw."""
    was_np = isinstance(x, np.ndarray)
    t = _as_cuda(x, device)
    nw = t.shape[-1]
    if nw % 2:
        t = torch.nn.functional.pad(t, (0, 1))
    return t.contiguous(), nw, was_np


def _packed_out(t, nw, was_np):
    t = t[..., :nw]
    return t.cpu().numpy() if was_np else t


class PackedFCLayer:
    """One hard FC layer: wiring ``[out, arity]`` int32 + truth tables ``[out]`` int64."""

    def __init__(self, idx, tt):
        self.idx = idx.to(torch.int32).contiguous()
        self.tt = tt.to(torch.int64).contiguous()
        self.out_dim, self.arity = self.idx.shape
        # the input width this wiring needs (checked once here: no index may be
        # negative; forward checks the input has more rows than the largest index)
        _hard.check_index_range(self.idx, 2**31 - 1, "FC wiring")
        self.min_in_dim = int(self.idx.max()) + 1 if self.idx.numel() else 0

    def forward(self, x):
        """``[in, n_words]`` int64 (numpy or CUDA) -> ``[out, n_words]``."""
        t, nw, was_np = _packed_in(x, self.idx.device)
        if t.shape[0] < self.min_in_dim:
            raise IndexError(f"FC wiring reads input row {self.min_in_dim - 1} but the input "
                             f"has {t.shape[0]} rows")
        return _packed_out(_hard.fc(t, self.idx, self.tt), nw, was_np)

    __call__ = forward


class BitpackedGPULayer(PackedFCLayer):
    """Gate16 layer from gate codes (``triton_layer.py:124-149`` signature)."""

    def __init__(self, gate_types, a_idx, b_idx, device="cuda"):
        dev = torch.device(device)
        g = torch.as_tensor(np.asarray(gate_types), dtype=torch.int64)
        idx = torch.stack([torch.as_tensor(np.asarray(a_idx)), torch.as_tensor(np.asarray(b_idx))], 1)
        super().__init__(idx.to(dev), gate16_lut_codes()[g].to(dev))
        self.device = device

    @classmethod
    def from_fc_layer(cls, fc_layer, device="cuda"):
        """From a converted FC layer: this package's (wiring + truth tables) or one with the
        reference ``BitpackedFCLayer`` fields ``gate_types`` / ``a_idx`` / ``b_idx``
        (``triton_layer.py:176-179``)."""
        if hasattr(fc_layer, "gate_types"):
            return cls(fc_layer.gate_types, fc_layer.a_idx, fc_layer.b_idx, device)
        obj = cls.__new__(cls)
        PackedFCLayer.__init__(obj, fc_layer.idx.to(device), fc_layer.tt.to(device))
        obj.device = device
        return obj


class PackedConvLayer:
    """One hard conv tree block: leaves ``[n, leaves]`` + truth tables ``[n, nodes]``."""

    def __init__(self, leaf, tt, arity, depth, kernel, pad, cin, n):
        self.leaf, self.tt = leaf.contiguous(), tt.contiguous()
        self.arity, self.depth, self.kh, self.kw = arity, depth, kernel, kernel
        self.padding, self.stride, self.cin, self.n_out = pad, 1, cin, n
        self.n_leaves = leaf.shape[1]
        _hard.check_index_range(self.leaf, cin * kernel * kernel, "conv leaf taps")

    def forward(self, x4, pool=2, wire_r=0):
        """Packed ``[C, H, W, ldw]`` CUDA -> ``[n, Ho/pool, Wo/pool, ldw]``."""
        if x4.shape[0] != self.cin:
            raise ValueError(f"conv layer built for {self.cin} input channels, got {x4.shape[0]}")
        return _hard.conv(x4, self.leaf, self.tt, self.arity, self.depth, self.kh,
                          self.padding, wire_r, pool)

    def forward_packed(self, x_3d):
        """Reference form on an already-unfolded ``[P, L, nw]`` input (no pool):
        the taps become 1x1 taps over ``P`` channels."""
        t, nw, was_np = _packed_in(x_3d, self.leaf.device)
        P, L, ldw = t.shape
        if P != self.cin * self.kh * self.kw:
            raise ValueError(f"unfolded input must have cin*k*k = {self.cin * self.kh * self.kw} "
                             f"rows, got {P}")
        y = _hard.conv(t.view(P, L, 1, ldw), self.leaf, self.tt, self.arity, self.depth,
                       kernel=1, pad=0, wire_r=0, pool=1)
        return _packed_out(y.view(self.n_out, L, ldw), nw, was_np)


class BitpackedConvGPULayer(PackedConvLayer):
    @classmethod
    def from_cpu_layer(cls, layer, device="cuda"):
        return cls(layer.leaf.to(device), layer.tt.to(device), layer.arity, layer.depth,
                   layer.kh, layer.padding, layer.cin, layer.n_out)


class PackedGroupSumHead:
    def __init__(self, num_classes, tau=1.0):
        self.num_classes, self.tau = num_classes, tau

    def forward(self, x, B):
        t, nw, was_np = _packed_in(x)
        c = _hard.groupsum(t, B, self.num_classes).float() / self.tau
        return c.cpu().numpy() if was_np else c


class PackedLearnedHead:
    """Learned linear readout on packed features (``BitpackedLearnedHead``,
    ``packed_layer.py:574-605``): ``weight`` ``[C, width]``, optional ``bias`` ``[C]``."""

    def __init__(self, weight, bias=None):
        self.weight = torch.as_tensor(weight, dtype=torch.float32)
        self.bias = None if bias is None else torch.as_tensor(bias, dtype=torch.float32)
        self.num_classes = self.weight.shape[0]

    def to(self, device):
        self.weight = self.weight.to(device)
        self.bias = self.bias.to(device) if self.bias is not None else None
        return self

    def apply(self, t, B):
        """Packed CUDA ``[width, ldw]`` -> fp32 logits ``[B, C]`` on the GPU."""
        t = t.reshape(-1, t.shape[-1])
        if self.weight.device != t.device:
            self.to(t.device)
        return _hard.packed_linear(t, self.weight, self.bias, B)

    def forward(self, x, B):
        t, nw, was_np = _packed_in(x)
        out = self.apply(t, B)
        return out.cpu().numpy() if was_np else out


class BitpackedNet:
    """End-to-end bit-packed ``LogicNet`` on the GPU.  ``net(x)`` with ``x`` ``[B, in]``
    uint8 -> ``[B, num_classes]`` float32 = counts / tau (``packed_model.py:75-102``)."""

    #: batch shapes whose CUDA graphs are kept (each holds its activations' memory)
    max_graphs = 4

    def __init__(self, plan, head, graphs=True):
        self.plan, self.head = plan, head
        self.num_layers = len(plan.steps)
        self.graphs = graphs
        self._graphs = {}
        self.device = _plan_device(plan)

    def _graph_for(self, x, thresholds=None, mode=0, slot=0):
        """Cached :class:`HardGraph` for this input shape/dtype (and thresholds);
        ``slot`` tells apart the double-buffered graphs of the pipelined path."""
        if isinstance(thresholds, (list, tuple)):
            tkey = tuple(float(v) for v in thresholds)
        elif thresholds is not None:
            thresholds = torch.as_tensor(thresholds, dtype=torch.float32,
                                         device=self.device).contiguous()
            tkey = (thresholds.data_ptr(), tuple(thresholds.shape))
        else:
            tkey = None
        key = (tuple(x.shape), x.dtype, mode, tkey, slot)
        g = self._graphs.get(key)
        if g is None:
            if len(self._graphs) >= self.max_graphs:
                torch.cuda.synchronize(self.device)     # no replay of it still pending
                self._graphs.pop(next(iter(self._graphs)))
            static = torch.empty(x.shape, dtype=x.dtype, device=self.device)
            static.copy_(x)
            if isinstance(self.head, PackedLearnedHead):
                g = HardGraph(self.plan, static, thresholds, mode, head=self.head)
            else:
                g = HardGraph(self.plan, static, thresholds, mode, tau=self.head.tau)
            self._graphs[key] = g
        return g

    def _run_pipelined(self, t, thresholds, mode):
        """A large host batch in slices of ~``pipeline_bytes``: the host-to-device copy of
        slice i+1 (side stream) overlaps the graph replay of slice i, alternating two
        graphs with their own static inputs."""
        B, sb = t.shape[0], self._slice(t)
        dev = self.device
        main = torch.cuda.current_stream(dev)
        if getattr(self, "_copy_stream", None) is None:
            self._copy_stream = torch.cuda.Stream(dev)
        cs = self._copy_stream
        logits = torch.empty((B, self.head.num_classes), dtype=torch.float32, device=dev)
        freed = [None, None]          # replay k no longer reads its static input
        cs.wait_stream(main)
        for i, s0 in enumerate(range(0, B, sb)):
            part = t[s0:s0 + sb]
            k = i % 2 if part.shape[0] == sb else 2
            g = self._graph_for(part, thresholds, mode, slot=k)
            with torch.cuda.stream(cs):
                if k < 2 and freed[k] is not None:
                    cs.wait_event(freed[k])
                g.x.copy_(part, non_blocking=True)
                copied = torch.cuda.Event()
                copied.record(cs)
            main.wait_event(copied)
            g.graph.replay()
            logits[s0:s0 + part.shape[0]].copy_(g.logits)
            if k < 2:
                freed[k] = torch.cuda.Event()
                freed[k].record(main)
        return logits

    #: host batches are pipelined (see _run_pipelined) in slices of about this many
    #: input bytes (a multiple of 1024 samples), when there are at least two slices ...
    pipeline_bytes = 8 << 20
    #: ... and of at least this many samples, so that each replay still fills the GPU
    #: (C5 from uint8 pixels: 3,072-sample slices ran at 8.3 M samples/s end to end,
    #: 16,384-sample ones at 11.1 M, 65,536-sample ones at 8.7 M)
    min_slice_samples = 16384

    def _slice(self, t):
        per = max(1, t[:1].numel() * t.element_size())
        by_bytes = -(-(self.pipeline_bytes // per) // 1024) * 1024
        return max(1024, self.min_slice_samples, by_bytes)

    def _run(self, x, thresholds=None, mode=0):
        """Logits of a numpy / host / device batch; host tensors are copied straight
        into the graph's static input (pinned memory makes that asynchronous)."""
        was_np = isinstance(x, np.ndarray)
        t = torch.from_numpy(np.ascontiguousarray(x)) if was_np else x
        if self.graphs and not t.is_cuda and t.shape[0] >= 2 * self._slice(t):
            logits = self._run_pipelined(t, thresholds, mode)
        elif self.graphs and t.shape[0] > 0:
            g = self._graph_for(t, thresholds, mode)
            g(t)
            logits = g.logits.clone()
        else:
            t = t.to(self.device, non_blocking=True)
            h = (self.plan.pack_input(t) if thresholds is None
                 else _hard.thermo_pack(t, thresholds, mode=mode))
            if isinstance(self.head, PackedLearnedHead):
                logits = self.head.apply(self.plan.run_packed(h), t.shape[0])
            else:
                logits = self.plan.counts_from_packed(h, t.shape[0]).float() / self.head.tau
        return logits.cpu().numpy() if was_np else logits

    def forward(self, x):
        return self._run(x)

    __call__ = forward

    def counts(self, x):
        """Integer counts ``[B, C]`` int32 on the GPU (no ``/tau``)."""
        return self.plan.counts(_as_cuda(x))

    def layer_summary(self):
        rows = []
        for i, st in enumerate(self.plan.steps):
            rows.append({"layer": i, "mode": st["op"], "out_dim": int(st.get("idx", st.get("leaf")).shape[0])})
        return rows


class BitpackedConvNet(BitpackedNet):
    """End-to-end bit-packed ``LogicConvNet``: ``[B, C, H, W]`` uint8 -> logits."""

    def forward_images(self, img, thresholds, mode=0):
        """Logits from real-valued images ``[B, C, H, W]`` with the thermometer encoding
        fused into the packing kernel (never materialising the bit planes as bytes).
        ``mode`` 0: shared ``thresholds`` [T] as in ``binarize_spatial``; 1: per-feature
        learned thresholds ``[C*H*W, T]`` as in ``LearnedThermometerEncoder``."""
        return self._run(img, thresholds, mode)

    @classmethod
    def from_conv_net(cls, bp_conv_net, H_in=None, W_in=None, device="cuda"):
        """Reference ``BitpackedConvGPUNet.from_conv_net`` signature: the net is already
        GPU-resident, so this returns it (moved to ``device``)."""
        return bp_conv_net


BitpackedConvGPUNet = BitpackedConvNet


def packed_unfold_gpu(x_3d, kh, kw, stride, padding, H_in, W_in):
    """``[C, H*W, nw]`` -> ``[C*kh*kw, L_out, nw]`` (API utility; the fused conv kernel
    never materialises this)."""
    C, L, nw = x_3d.shape
    Ho = (H_in + 2 * padding - kh) // stride + 1
    Wo = (W_in + 2 * padding - kw) // stride + 1
    x4 = torch.nn.functional.pad(x_3d.view(C, H_in, W_in, nw), (0, 0, padding, padding, padding, padding))
    cols = []
    for dy in range(kh):
        for dx in range(kw):
            cols.append(x4[:, dy:dy + stride * Ho:stride, dx:dx + stride * Wo:stride])
    return torch.stack(cols, 1).reshape(C * kh * kw, Ho * Wo, nw)


def packed_or_pool_gpu(x_3d, H, W, pool_size=2):
    """OR-pool ``[C, H*W, nw]`` -> ``[C, (H/ps)*(W/ps), nw]`` (API utility)."""
    C, L, nw = x_3d.shape
    ps = pool_size
    x4 = x_3d.view(C, H, W, nw)[:, :H // ps * ps, :W // ps * ps]
    x5 = x4.reshape(C, H // ps, ps, W // ps, ps, nw)
    out = x5[:, :, 0, :, 0]
    for dy in range(ps):
        for dx in range(ps):
            out = out | x5[:, :, dy, :, dx]
    return out.reshape(C, -1, nw)
