"""Logic networks with the reference model API (``silogic/models.py``), CUDA-only.

Inside a network, activations stay in the kernels' native layouts between layers:
soft activations feature-major ``[F, B]``, hard activations bit-packed
``[F, ceil(B/64)]`` words; a conv block and the ``OrPool`` after it run as one
fused kernel.  Constructor arguments, submodule names and per-layer seeds follow
the reference so checkpoints load unchanged.
"""
import torch
import torch.nn as nn

from . import _soft
from .heads import build_decoder, GroupSum
from .layers import LogicLayer, ConvLogicTree, OrPool


def _per_layer(v, i):
    return v[i] if isinstance(v, (list, tuple)) else v


class LogicNet(nn.Module):
    """Stack of :class:`LogicLayer` + a head (same arguments as the reference)."""

    def __init__(self, in_dim, width, depth, num_classes=10, node="gate16",
                 connectome="topk", arity=2, k=8, tau=1.0, gate_eval="basis",
                 node_tau=1.0, residual_p=0.0, seed=0, wire_residual=0.0,
                 decoder="groupsum", degree=None, seed_mult=1000, gate_select="softmax",
                 gumbel_tau=1.0, decoder_ste=True, use_triton=True):
        super().__init__()
        layers, d_in = [], in_dim
        for i in range(depth):
            layers.append(LogicLayer(
                d_in, width, node=_per_layer(node, i), connectome=connectome, arity=arity,
                k=k, gate_eval=gate_eval, residual_p=residual_p, degree=degree, tau=node_tau,
                gate_select=_per_layer(gate_select, i), gumbel_tau=gumbel_tau,
                use_triton=use_triton, seed=None if seed is None else seed * seed_mult + i))
            d_in = width
        self.layers = nn.ModuleList(layers)
        self.head = build_decoder(decoder, width, num_classes, tau, feature_ste=decoder_ste)
        self.width = width
        self.depth = depth
        self.node = node
        self.connectome = connectome
        self.k = k
        self.decoder_kind = decoder
        self.wire_r = int(width * wire_residual)

    def _run(self, x, hard):
        if hard:
            from .bitpacking.plan import HardPlan
            return HardPlan.from_model(self).features(x)
        return _soft.logic_net_features(self, x)

    def forward(self, x):
        if isinstance(self.head, GroupSum):
            return _soft.logic_net_logits(self, x)
        return self.head(self._run(x, hard=False))

    @torch.no_grad()
    def forward_hard(self, x):
        from .bitpacking.plan import HardPlan
        plan = HardPlan.from_model(self)
        # per-layer kernels: the fused FC stack's host-side layout planning and record
        # upload pay off on a converted, reused BitpackedNet, not on every call
        plan.use_chain = False
        if isinstance(self.head, GroupSum):
            return plan.counts(x).float()
        return self.head.forward_hard(plan.features(x))

    def num_gates(self):
        return self.width * self.depth


class WARPNet(LogicNet):
    def __init__(self, in_dim, width, depth, num_classes=10, k=8, tau=1.0, residual_p=0.0,
                 seed=0, gate_select="softmax"):
        super().__init__(in_dim, width, depth, num_classes=num_classes, node="walsh", arity=2,
                         k=k, node_tau=tau, tau=20.0, residual_p=residual_p, seed=seed,
                         gate_select=gate_select)


class WARPNetN(LogicNet):
    def __init__(self, in_dim, width, depth, arity=6, num_classes=10, k=8, tau=1.0,
                 residual_p=0.0, seed=0, gate_select="softmax"):
        super().__init__(in_dim, width, depth, num_classes=num_classes, node="walsh",
                         arity=arity, k=k, node_tau=tau, tau=20.0, residual_p=residual_p,
                         seed=seed, gate_select=gate_select)


class LUTkNet(LogicNet):
    def __init__(self, in_dim, width, depth, k=4, num_classes=10, tau=4.0, cand_k=4, seed=0):
        super().__init__(in_dim, width, depth, num_classes=num_classes, node="multilinear",
                         arity=k, k=cand_k, tau=tau, seed=seed)
        self.lut_inputs = k

    def num_luts(self):
        return self.width * self.depth


class LUTNodeNet(LogicNet):
    def __init__(self, in_dim, width, depth, arity=4, relaxation="probabilistic",
                 num_classes=10, k=8, tau=10.0, residual_p=0.0, seed=0):
        super().__init__(in_dim, width, depth, num_classes=num_classes, node=relaxation,
                         arity=arity, k=k, tau=tau, residual_p=residual_p, seed=seed)


class LogicConvNet(nn.Module):
    """Conv logic-tree blocks (``ConvLogicTree`` + ``OrPool``) + a logic head."""

    def __init__(self, in_channels, in_hw, channels, head_width=None, num_classes=10,
                 tree_depth=None, kernel=3, connect="topk", k=4, head_connect="topk",
                 head_k=8, head_depth=2, n_chan=2, residual_init=True, tau=100.0, seed=0,
                 wire_residual=0.0, head_widths=None, decoder="groupsum", node="gate16",
                 arity=2, node_tau=1.0, degree=None, gate_select="softmax", gumbel_tau=1.0,
                 decoder_ste=True, use_triton=True):
        super().__init__()
        self.blocks = nn.ModuleList()
        c = in_channels
        for i, n in enumerate(channels):
            self.blocks.append(ConvLogicTree(
                c, n, kernel=kernel, tree_depth=tree_depth, stride=1, padding=kernel // 2,
                connect=connect, k=k, n_chan=n_chan, residual_init=residual_init,
                seed=seed * 17 + i, node=node, arity=arity, tau=node_tau, degree=degree,
                gate_select=gate_select, gumbel_tau=gumbel_tau, use_triton=use_triton))
            self.blocks.append(OrPool(2))
            c = n
            in_hw = in_hw // 2
        self.feat_dim = c * in_hw * in_hw
        if head_widths is None:
            head_widths = [head_width] * head_depth
        layers, d_in = [], self.feat_dim
        for j, w in enumerate(head_widths):
            layers.append(LogicLayer(d_in, w, connectome=head_connect, k=head_k, node=node,
                                     gate_select=gate_select, use_triton=use_triton,
                                     seed=seed * 31 + j))
            d_in = w
        self.head_layers = nn.ModuleList(layers)
        self.head = build_decoder(decoder, head_widths[-1], num_classes, tau,
                                  feature_ste=decoder_ste)
        self.decoder_kind = decoder
        self._head_widths = head_widths
        self.wire_residual = wire_residual

    def wire_channels(self, conv, cin):
        if self.wire_residual <= 0:
            return 0
        return max(0, min(int(conv.n * self.wire_residual), cin))

    def _run(self, x, hard):
        if hard:
            from .bitpacking.plan import HardPlan
            return HardPlan.from_model(self).features(x)
        return _soft.logic_conv_net_features(self, x)

    def forward(self, x):
        if isinstance(self.head, GroupSum):
            return _soft.logic_conv_net_logits(self, x)
        return self.head(self._run(x, hard=False))

    @torch.no_grad()
    def forward_hard(self, x):
        from .bitpacking.plan import HardPlan
        plan = HardPlan.from_model(self)
        # per-layer kernels: the fused FC stack's host-side layout planning and record
        # upload pay off on a converted, reused BitpackedNet, not on every call
        plan.use_chain = False
        if isinstance(self.head, GroupSum):
            return plan.counts(x).float()
        return self.head.forward_hard(plan.features(x))

    def gate_count(self, in_hw):
        total, hw = 0, in_hw
        for blk in self.blocks:
            if isinstance(blk, ConvLogicTree):
                total += blk.n * hw * hw * blk.gates_per_output
            elif isinstance(blk, OrPool):
                hw = hw // 2
        return total + sum(self._head_widths)


class LogicTreeNet(LogicConvNet):
    """Paper-named preset of :class:`LogicConvNet` (Petersen et al. trees + Top-K wiring)."""
