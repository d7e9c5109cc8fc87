"""Trained model -> bit-packed inference objects (API of ``silogic/bitpacking/convert.py``).

Conversion is device-side: hard wiring (``argmax`` of the connection logits) and
truth tables (each node's ``forward_hard`` at the 2^arity cube corners) are
computed from the parameters where they live and stay on the GPU.
"""
import torch

from .. import _hard
from ..connectomes import SumThresholdConnectome
from .packed import (PackedFCLayer, PackedConvLayer, BitpackedNet, BitpackedConvNet,
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
    from ..heads import GroupSum
    if isinstance(head, GroupSum):
        return PackedGroupSumHead(head.num_classes, head.tau)
    raise TypeError(f"no bit-packed form for head {type(head).__name__} in silogic_b200")


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
