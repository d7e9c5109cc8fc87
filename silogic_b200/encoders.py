"""Learned thermometer encoder (``silogic/encoders.py``), CUDA-only."""
import torch
import torch.nn as nn

from . import _soft


class LearnedThermometerEncoder(nn.Module):
    """``bits`` learnable thresholds per feature; forward = ``1[x_f > t_{f,i}]`` with a
    ``sigmoid(scale * (x - t))`` straight-through gradient.  ``[B, F] -> [B, F*bits]``."""

    def __init__(self, num_features, bits, init_lo=0.0, init_hi=1.0, scale=10.0):
        super().__init__()
        self.num_features = num_features
        self.bits = bits
        self.scale = scale
        t = torch.linspace(init_lo, init_hi, bits + 2)[1:-1]
        self.thresholds = nn.Parameter(t.repeat(num_features, 1))

    def forward(self, x):
        return _soft.thermometer_forward(x, self.thresholds, self.scale)

    @torch.no_grad()
    def forward_hard(self, x):
        return _soft.thermometer_hard(x, self.thresholds)
