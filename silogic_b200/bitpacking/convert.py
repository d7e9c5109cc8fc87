"""Trained model -> bit-packed inference objects (API of ``silogic/bitpacking/convert.py``).

Conversion is device-side: hard wiring (``argmax`` of the connection logits) and
truth tables (each node's ``forward_hard`` at the 2^arity cube corners) are
computed from the parameters where they live and stay on the GPU.
"""
import torch

from .. import _hard
from ..connectomes import SumThresholdConnectome
from .packed import (PackedLearnedHead, PackedFCLayer, PackedConvLayer, BitpackedNet, BitpackedConvNet,
                     PackedGroupSumHead)


def convert_layer(layer):
    """``LogicLayer`` -> :class:`PackedFCLayer` (``None`` for sum-threshold wiring)."""
    if isinstance(layer._conn, SumThresholdConnectome):
        return None
    idx, tt = layer.hard_spec()
    return PackedFCLayer(idx, tt)


def convert_conv_tree_layer(conv):
    leaf, tt = conv.hard_spec()
    return PackedConvLayer(leaf, tt, conv.node_arity, conv.d, conv.kh, conv.padding,
                           conv.cin, conv.n)


def convert_head(head):
    """GroupSum -> popcount head; LearnedDecoder ``linear`` / ``linfull`` / ``ternary`` ->
    :class:`PackedLearnedHead` with its effective weight (``convert.py:300-328``);
    ``sumlinear`` needs batch-norm folding and is refused, as in the reference."""
    from ..heads import GroupSum, LearnedDecoder
    from ..functional import ternary_ste
    if isinstance(head, GroupSum):
        return PackedGroupSumHead(head.num_classes, head.tau)
    if isinstance(head, LearnedDecoder):
        with torch.no_grad():
            if head.kind in ("linear", "linfull"):
                return PackedLearnedHead(head.dec.weight.detach().clone(), head.dec.bias.detach().clone())
            if head.kind == "ternary":
                return PackedLearnedHead(ternary_ste(head.dec_w).detach().clone(), None)
            if head.kind == "sumlinear":
                raise NotImplementedError("sumlinear decoder requires BN folding; use forward_hard")
        raise ValueError(f"unknown decoder kind {head.kind!r}")
    raise TypeError(f"no bit-packed form for head {type(head).__name__}")


def convert_logic_net(model):
    """``LogicNet`` -> :class:`BitpackedNet` (GPU-resident)."""
    from .plan import HardPlan
    for L in model.layers:
        if isinstance(L._conn, SumThresholdConnectome):
            raise NotImplementedError("sum-threshold connectomes have no static wiring")
    return BitpackedNet(HardPlan.from_model(model), convert_head(model.head))


def convert_logic_conv_net(model):
    """``LogicConvNet`` / ``LogicTreeNet`` -> :class:`BitpackedConvNet` (GPU-resident)."""
    from .plan import HardPlan
    return BitpackedConvNet(HardPlan.from_model(model), convert_head(model.head))
