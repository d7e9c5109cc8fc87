"""Decoders (``silogic/heads.py``): the parameter-free GroupSum runs as a CUDA
popcount (hard) / thresholded block-sum (soft) kernel; the learned decoders are
ordinary torch modules (dense readouts, outside the logic-gate hot path)."""
import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _hard, _soft
from .functional import binarize_ste, ternary_ste


class GroupSum(nn.Module):
    """Class logits = per-class block sums of the logic outputs, divided by ``tau``.

    ``feature_ste=True`` sums the thresholded bits ``x > 0.5`` with an identity
    gradient (the setting every ``LogicNet``/``LogicConvNet`` uses).
    """

    def __init__(self, num_classes=10, tau=1.0, feature_ste=False):
        super().__init__()
        self.num_classes = num_classes
        self.tau = tau
        self.feature_ste = feature_ste

    def forward(self, x):
        return _soft.group_sum_forward(x, self.num_classes, self.tau, self.feature_ste)

    @torch.no_grad()
    def forward_hard(self, x):
        """Integer block counts (as float, no ``/tau``) of binary features ``[B, W]``."""
        B = x.shape[0]
        return _hard.groupsum(_hard.pack(x), B, self.num_classes).float()


class LearnedDecoder(nn.Module):
    """Learned readouts ``linear`` / ``linfull`` / ``sumlinear`` / ``ternary``."""

    def __init__(self, kind, width, num_classes=10, feature_ste=True):
        super().__init__()
        self.kind = kind
        self.feature_ste = feature_ste
        if kind == "linear":
            self.dec = nn.Linear(width, num_classes)
        elif kind == "linfull":
            assert width % num_classes == 0
            self.dec = nn.Linear(width, num_classes)
            g = width // num_classes
            with torch.no_grad():
                self.dec.weight.zero_()
                for c in range(num_classes):
                    self.dec.weight[c, c * g:(c + 1) * g] = 1.0 / g
                self.dec.bias.zero_()
        elif kind == "ternary":
            assert width % num_classes == 0
            g = width // num_classes
            w = torch.zeros(num_classes, width)
            for c in range(num_classes):
                w[c, c * g:(c + 1) * g] = 1.0
            self.dec_w = nn.Parameter(w)
        elif kind == "sumlinear":
            self.hidden = 256
            assert width % self.hidden == 0, "width must be divisible by 256"
            self.dec_bn = nn.BatchNorm1d(self.hidden)
            self.dec_lin = nn.Linear(self.hidden, num_classes)
        else:
            raise ValueError(f"unknown decoder {kind!r}")

    def _decode(self, x):
        if self.kind == "linear":
            return self.dec(x)
        if self.feature_ste:
            x = binarize_ste(x)
        if self.kind == "ternary":
            return F.linear(x, ternary_ste(self.dec_w))
        if self.kind == "linfull":
            return self.dec(x)
        x = x.view(x.shape[0], self.hidden, -1).sum(2)
        return self.dec_lin(self.dec_bn(x))

    def forward(self, x):
        return self._decode(x)

    @torch.no_grad()
    def forward_hard(self, x):
        return self._decode(x.float())


def build_decoder(kind, width, num_classes=10, tau=1.0, feature_ste=True):
    """``"groupsum"`` (default) or a :class:`LearnedDecoder` kind."""
    if kind == "groupsum":
        assert width % num_classes == 0, "width must be divisible by classes"
        return GroupSum(num_classes=num_classes, tau=tau, feature_ste=feature_ste)
    return LearnedDecoder(kind, width, num_classes, feature_ste=feature_ste)
