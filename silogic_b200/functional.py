"""Gate algebra constants and straight-through helpers (same public names and
semantics as ``silogic/functional.py``).

These are parameter-side utilities: the 16-gate basis table, the truth tables,
and the small STE helpers users compose with.  The activation path of every
layer runs in the CUDA kernels of this package, not here.
"""
import math

import torch
import torch.nn.functional as F

# Coefficients of (1, a, b, a*b) for the 16 two-input gates, in the DiffLogic
# order used by the reference (silogic/functional.py:24-44): gate g computes
# c0 + c1*a + c2*b + c3*a*b on {0,1} inputs.
BASIS_COEFFS = torch.tensor([
    [0, 0, 0, 0], [0, 0, 0, 1], [0, 1, 0, -1], [0, 1, 0, 0],
    [0, 0, 1, -1], [0, 0, 1, 0], [0, 1, 1, -2], [0, 1, 1, -1],
    [1, -1, -1, 1], [1, -1, -1, 2], [1, 0, -1, 0], [1, 0, -1, 1],
    [1, -1, 0, 0], [1, -1, 0, 1], [1, 0, 0, -1], [1, 0, 0, 0],
], dtype=torch.float32)

GATE_A = 3   # pass-through of the first input


def _gate_truth_tables():
    c = BASIS_COEFFS
    # column order (a, b) = 00, 01, 10, 11, i.e. column index (a << 1) | b
    cols = [c[:, 0], c[:, 0] + c[:, 2], c[:, 0] + c[:, 1], c.sum(1)]
    return torch.stack(cols, dim=1).round().to(torch.uint8)


TRUTH_TABLES = _gate_truth_tables()   # [16, 4]


def gate16_lut_codes():
    """``[16]`` int64: gate g as a 4-entry LUT in the address order a | b << 1."""
    tt = TRUTH_TABLES.to(torch.int64)
    code = torch.zeros(16, dtype=torch.int64)
    for p in range(4):
        a, b = p & 1, p >> 1
        code |= tt[:, (a << 1) | b] << p
    return code


def ste_threshold(s):
    """Forward ``s > 0`` in {0,1}, gradient of ``sigmoid(s)``."""
    soft = torch.sigmoid(s)
    return (s > 0).float() + soft - soft.detach()


def sign_ste(w):
    """Forward sign in {-1,+1} (``w >= 0`` -> +1), clipped straight-through gradient."""
    clip = torch.clamp(w, -1, 1)
    return clip + (torch.where(w >= 0, 1.0, -1.0) - clip).detach()


def ternary_ste(w, delta=0.5):
    """Forward {-1,0,+1} with dead zone ``|w| <= delta``, clipped STE gradient."""
    hard = torch.where(w > delta, 1.0, torch.where(w < -delta, -1.0, 0.0))
    clip = torch.clamp(w, -1, 1)
    return clip + (hard - clip).detach()


def binarize_ste(x, thresh=0.5):
    """Forward ``x > thresh`` in {0,1}, identity gradient."""
    return (x > thresh).float() + (x - x.detach())


def residual_logit(p, tau=1.0):
    """Logit whose sigmoid is ``p`` (clamped to [1e-4, 1-1e-4]), times ``tau``."""
    p = min(max(float(p), 1e-4), 1 - 1e-4)
    return tau * math.log(p / (1 - p))


def gate_probs(logits, training, dim=-1, gate_select="softmax", gumbel_tau=1.0):
    """Selection weights over the 16 gates: softmax, or (training) Gumbel / argmax STE."""
    if training and gate_select == "gumbel":
        return F.gumbel_softmax(logits, tau=gumbel_tau, hard=True, dim=dim)
    soft = F.softmax(logits, dim=dim)
    if training and gate_select == "hard":
        hard = torch.zeros_like(soft).scatter_(dim, soft.argmax(dim=dim, keepdim=True), 1.0)
        return soft + (hard - soft).detach()
    return soft


def corner_bits(n, dtype=torch.float32):
    """``[2^n, n]`` table: row p holds the bits of p (bit j in column j)."""
    p = torch.arange(2 ** n).unsqueeze(1)
    return ((p >> torch.arange(n)) & 1).to(dtype)


def walsh_monomials(u):
    """``[B, out, n]`` -> ``[B, out, 2^n]``; column i = prod of u_j over bits j of i."""
    cols = [torch.ones_like(u[..., :1])]
    for j in range(u.shape[-1]):
        cols = cols + [c * u[..., j:j + 1] for c in cols]
    return torch.cat(cols, dim=-1)
