"""Soft (relaxed, differentiable) ops -- host side of the fp32 CUDA kernels."""
import torch

from . import _hard


def _todo(*a, **k):
    raise NotImplementedError("soft kernels are not built yet")


fc_supported = lambda layer: True
logic_layer_forward = _todo
node_forward = _todo
conv_tree_forward = _todo
group_sum_forward = _todo
logic_net_features = _todo
logic_net_logits = _todo
logic_conv_net_features = _todo
logic_conv_net_logits = _todo
thermometer_forward = _todo
or_pool = _todo


@torch.no_grad()
def or_pool_hard(x, size):
    raise NotImplementedError


@torch.no_grad()
def thermometer_hard(x, thresholds):
    B, F = x.shape
    T = thresholds.shape[1]
    h = _hard.thermo_pack(x.view(B, F, 1, 1), thresholds, mode=1)   # [F*T, 1, 1, ldw]
    return _hard.unpack(h.view(F * T, -1), B)
