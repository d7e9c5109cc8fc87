"""Thermometer thresholds and spatial binarization (``silogic/data.py:18-20,71-92``).

Dataset download/augmentation is not part of this package (no datasets are
needed for the kernels).  ``binarize_spatial`` on a CUDA tensor runs the fused
thermometer + pack kernel and unpacks; hard-circuit pipelines use
:func:`silogic_b200._hard.thermo_pack` directly and never materialise the bytes.
"""
import torch

MNIST_THRESH = [0.25]
SEVEN_THRESH = [0.125, 0.25, 0.375, 0.5, 0.625, 0.75, 0.875]
FOUR_THRESH = [0.2, 0.4, 0.6, 0.8]
CIFAR3_THRESH = [0.25, 0.5, 0.75]
FIVE_THRESH = [1 / 6, 2 / 6, 3 / 6, 4 / 6, 5 / 6]
EDGE_THRESH = [0.12, 0.25]


def binarize_spatial(x, thresholds):
    """``[N, C, H, W]`` in [0,1] -> ``[N, C*T, H, W]`` uint8, plane t*C+c = ``x >= f32(t)``."""
    from . import _hard
    B, C, H, W = x.shape
    h = _hard.thermo_pack(x, thresholds, mode=0)          # [C*T, H, W, ldw]
    return _hard.unpack(h.view(-1, h.shape[-1]), B).view(B, C * len(thresholds), H, W)
