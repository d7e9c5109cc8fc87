"""Logic-node parameterizations (same names, parameters and init as ``silogic/nodes.py``).

A node maps operands ``[B, out, arity]`` in [0, 1] to ``[B, out]``.  In this
package a node is the parameter holder of a layer; its ``forward`` and
``forward_hard`` run the same CUDA kernels as :class:`~silogic_b200.layers.LogicLayer`
with an identity wiring (operand ``j`` of node ``o`` is input column ``o*arity + j``).
"""
from itertools import combinations

import torch
import torch.nn as nn

from .functional import BASIS_COEFFS, TRUTH_TABLES, GATE_A, residual_logit, corner_bits

NODES = ("gate16", "walsh", "multilinear", "hybrid", "linear", "polynomial")
RELAXATIONS = ("probabilistic", "hybrid", "linear", "polynomial")
_NODE_ALIASES = {
    "gate16": "gate16", "gate": "gate16", "walsh": "walsh",
    "multilinear": "multilinear", "probabilistic": "multilinear",
    "hybrid": "hybrid", "linear": "linear", "polynomial": "polynomial",
}


class Node(nn.Module):
    """Base class; ``kind`` names the kernel family."""

    kind = None
    param_name = None

    def __init__(self, out_dim, arity):
        super().__init__()
        self.out_dim = out_dim
        self.arity = arity

    @property
    def param(self):
        return getattr(self, self.param_name)

    def _identity_call(self, operands, hard):
        from . import _soft, _hard
        B = operands.shape[0]
        x = operands.reshape(B, self.out_dim * self.arity)
        idx = torch.arange(self.out_dim * self.arity, device=operands.device,
                           dtype=torch.int32).view(self.out_dim, self.arity)
        if hard:
            tt = _hard.node_truth_tables(self.kind, self.param, self.arity,
                                         getattr(self, "mono_mask", None))
            h = _hard.fc(_hard.pack(x), idx, tt)
            return _hard.unpack(h, B)
        return _soft.node_forward(self, x, idx)

    def forward(self, operands):
        return self._identity_call(operands, hard=False)

    @torch.no_grad()
    def forward_hard(self, operands):
        return self._identity_call(operands, hard=True)

    def residual_init(self, p):
        raise NotImplementedError


class Gate16Node(Node):
    """Softmax mixture over the 16 two-input gates (arity 2)."""

    kind, param_name = "gate16", "gate_logits"

    def __init__(self, out_dim, arity=2, gate_eval="basis", gate_select="softmax",
                 gumbel_tau=1.0):
        super().__init__(out_dim, 2)
        assert arity == 2, "gate16 nodes are two-input"
        self.gate_eval = gate_eval
        self.gate_select = gate_select
        self.gumbel_tau = gumbel_tau
        self.gate_logits = nn.Parameter(torch.randn(out_dim, 16) * 0.1)
        self.register_buffer("basis", BASIS_COEFFS.clone())
        self.register_buffer("truth", TRUTH_TABLES.clone())

    def coef(self):
        """BasisProj coefficients ``[out, 4]`` = ``gate_probs(logits) @ basis``."""
        from .functional import gate_probs
        p = gate_probs(self.gate_logits, self.training, dim=1, gate_select=self.gate_select,
                       gumbel_tau=self.gumbel_tau)
        return p @ self.basis

    @torch.no_grad()
    def residual_init(self, p):
        self.gate_logits.normal_(0, 0.1)
        self.gate_logits[:, GATE_A] = residual_logit(p)


class WalshNode(Node):
    """Walsh-Hadamard node ``sigmoid(sum_M theta_M prod_{j in M}(2a_j-1) / tau)``."""

    kind, param_name = "walsh", "theta"

    def __init__(self, out_dim, arity=2, tau=1.0, gate_select="softmax"):
        super().__init__(out_dim, arity)
        self.tau = tau
        self.gate_select = gate_select
        self.theta = nn.Parameter(torch.randn(out_dim, 2 ** arity) * 0.1)

    @property
    def inv_tau(self):
        return 1.0 / self.tau

    def coef(self):
        """Arity-2 coefficients of ``z`` in the (1, a, b, ab) basis."""
        t = self.theta
        return torch.stack([t[:, 0] - t[:, 1] - t[:, 2] + t[:, 3], 2 * (t[:, 1] - t[:, 3]),
                            2 * (t[:, 2] - t[:, 3]), 4 * t[:, 3]], dim=1)

    def _z(self, *vals):
        u = [2 * v - 1 for v in vals]
        if self.arity == 2:
            t = self.theta
            return t[:, 0] + t[:, 1] * u[0] + t[:, 2] * u[1] + t[:, 3] * (u[0] * u[1])
        from .functional import walsh_monomials
        return (walsh_monomials(torch.stack(u, dim=2)) * self.theta[None]).sum(2)

    @torch.no_grad()
    def residual_init(self, p):
        self.theta.zero_()
        self.theta[:, 2 ** (self.arity - 1)] = residual_logit(p, self.tau)


class MultilinearNode(Node):
    """One logit per truth-table entry, multilinear interpolation (a LUT_k)."""

    kind, param_name = "multilinear", "logits"

    def __init__(self, out_dim, arity=2):
        super().__init__(out_dim, arity)
        self.register_buffer("corners", corner_bits(arity))
        self.logits = nn.Parameter(torch.randn(out_dim, 2 ** arity) * 0.1)

    @torch.no_grad()
    def residual_init(self, p):
        c = residual_logit(p)
        bit0 = self.corners[:, 0]
        self.logits.copy_((2 * bit0 - 1) * c + 0.1 * torch.randn_like(self.logits))


class HybridNode(MultilinearNode):
    """Discrete forward on thresholded operands, multilinear surrogate gradient."""

    kind = "hybrid"


class LinearNode(Node):
    """Perceptron node ``sigmoid(theta_0 + sum_j theta_j a_j)``."""

    kind, param_name = "linear", "theta"

    def __init__(self, out_dim, arity=2):
        super().__init__(out_dim, arity)
        self.theta = nn.Parameter(torch.randn(out_dim, arity + 1) * 0.1)

    @torch.no_grad()
    def residual_init(self, p):
        c = residual_logit(p)
        self.theta.zero_()
        self.theta[:, 1] = c
        self.theta[:, 0] = -c / 2


class PolynomialNode(Node):
    """Degree-``d`` multilinear polynomial node ``sigmoid(sum_s theta_s prod_{j in s} a_j)``.

    The soft kernels evaluate it in the Walsh form: with ``a_j = (u_j + 1) / 2``,
    ``prod_{j in s} a_j = 2^-|s| sum_{M subset s} prod_{j in M} u_j``, so
    ``theta_walsh = theta @ T`` with ``T[s, M] = 2^-|s|`` for ``M`` a subset of ``s``
    (a fixed linear map, differentiated by autograd) and ``inv_tau = 1``."""

    kind, param_name = "polynomial", "theta"

    def __init__(self, out_dim, arity=2, degree=None):
        super().__init__(out_dim, arity)
        d = min(2, arity) if degree is None else min(degree, arity)
        self.degree = d
        subs = [()]
        for r in range(1, d + 1):
            subs += list(combinations(range(arity), r))
        self._subs = subs
        mask = torch.zeros(len(subs), arity)
        for i, s in enumerate(subs):
            for j in s:
                mask[i, j] = 1.0
        self.register_buffer("mono_mask", mask)
        self.theta = nn.Parameter(torch.randn(out_dim, len(subs)) * 0.1)
        T = torch.zeros(len(subs), 1 << arity)
        for i, sub in enumerate(subs):
            S = sum(1 << j for j in sub)
            M = S
            while True:                      # every subset M of S
                T[i, M] += 2.0 ** -len(sub)
                if M == 0:
                    break
                M = (M - 1) & S
        self.register_buffer("_to_walsh", T, persistent=False)

    def walsh_theta(self):
        """``[out, 2^arity]`` coefficients of the same function in the ``u = 2a - 1``
        monomial basis (index = subset bitmask), for the Walsh-form soft kernels."""
        return self.theta @ self._to_walsh

    @torch.no_grad()
    def residual_init(self, p):
        c = residual_logit(p)
        self.theta.zero_()
        self.theta[:, self._subs.index(())] = -c / 2
        self.theta[:, self._subs.index((0,))] = c


_BUILDERS = {"gate16": Gate16Node, "walsh": WalshNode, "multilinear": MultilinearNode,
             "hybrid": HybridNode, "linear": LinearNode, "polynomial": PolynomialNode}


def build_node(name, out_dim, arity=2, **kw):
    """Construct a node by name (aliases as in the reference registry)."""
    key = _NODE_ALIASES.get(str(name).lower())
    if key is None:
        raise ValueError(f"unknown node {name!r}; choose from {NODES}")
    if key == "gate16":
        return Gate16Node(out_dim, arity, gate_eval=kw.get("gate_eval", "basis"),
                          gate_select=kw.get("gate_select", "softmax"),
                          gumbel_tau=kw.get("gumbel_tau", 1.0))
    if key == "walsh":
        return WalshNode(out_dim, arity, tau=kw.get("tau", 1.0),
                         gate_select=kw.get("gate_select", "softmax"))
    if key == "polynomial":
        return PolynomialNode(out_dim, arity, degree=kw.get("degree"))
    return _BUILDERS[key](out_dim, arity)
