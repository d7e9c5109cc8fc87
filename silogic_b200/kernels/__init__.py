"""The reference's fused-kernel function API (``silogic/kernels/__init__.py:21-55``), on
this package's sm_100a CUDA kernels.

Each function keeps the reference's signature, argument meaning, shapes and return
value: activations are batch-major (``[B, IN]`` / ``[B, C, H, W]``), connection
weights and gate coefficients arrive already transformed (post-softmax weights,
BasisProj coefficients, ``sigmoid(logits)`` LUT values), and autograd returns
gradients with respect to exactly those tensors.  Underneath, the batch is
transposed once to the feature-major layout of the kernels (``slg_to_feature_major``)
and the soft FC / conv-tree kernels run in their "direct parameter" modes
(``conn_ste = 2`` = weights as given; node kinds 5 coef, 6 coef-sigmoid, 7 hybrid
with given LUT values).

There is no Triton and no CPU fallback: every ``HAS_*`` flag is ``True`` and means
"the CUDA kernel is available"; calling a function on CPU tensors raises.
"""
import torch

from .. import _soft
from .._soft import ConvSoft, FCSoft, FromFeatureMajor, ToFeatureMajor

N_COEF, N_COEF_SIG, N_HYBRID_S = 5, 6, 7
DIRECT_WEIGHTS = 2

HAS_DENSE = True
HAS_CONV = True
HAS_CONV_TOPK = True
HAS_WARP = True
HAS_MULTILINEAR = True
HAS_CONV_HYBRID = True

__all__ = ["dense_logic", "warp_logic", "multilinear_logic", "tree_conv", "tree_conv_af",
           "tree_conv_topk", "conv_hybrid", "build_inverse_map", "HAS_DENSE", "HAS_CONV",
           "HAS_CONV_TOPK", "HAS_WARP", "HAS_MULTILINEAR", "HAS_CONV_HYBRID"]


# ----------------------------------------------------------------------- FC
def _fc(x, cand, w, params, node, arity, inv_tau=1.0):
    if x.dim() != 2:
        raise ValueError(f"x must be [B, IN], got {tuple(x.shape)}")
    B, IN = x.shape
    OUT, n, K = cand.shape
    if n != arity or w.shape != cand.shape:
        raise ValueError("cand / w must be [OUT, arity, K] with matching shapes")
    cand = cand.to(torch.int32).contiguous()
    from .. import _hard
    _hard.check_index_range(cand, IN, "candidate indices")
    meta = dict(cand=cand, K=K, ste=DIRECT_WEIGHTS, node=node, arity=arity, gate_hard=0,
                inv_tau=float(inv_tau), out_dim=OUT, wire_r=0)
    xt = ToFeatureMajor.apply(x.float())
    yt = FCSoft.apply(xt, params, w.float(), meta)
    return FromFeatureMajor.apply(yt, B).to(x.dtype)


def dense_logic(x, ca, cb, wa, wb, coef):
    """``x[B,IN]``, ``ca/cb[OUT,K]`` int32, ``wa/wb[OUT,K]`` post-softmax weights,
    ``coef[OUT,4]`` BasisProj coefficients -> ``[B,OUT]`` =
    ``c0 + c1 a + c2 b + c3 a b`` with ``a = sum_k wa[o,k] x[:, ca[o,k]]``
    (``silogic/kernels/dense.py:91-125``)."""
    cand = torch.stack([ca, cb], dim=1)
    w = torch.stack([wa, wb], dim=1)
    return _fc(x, cand, w, coef, N_COEF, 2)


def warp_logic(x, ca, cb, wa, wb, coef, inv_tau):
    """As :func:`dense_logic` with ``sigmoid((c0 + c1 a + c2 b + c3 a b) * inv_tau)``
    (the Walsh node in BasisProj form, ``silogic/kernels/warp.py:79-105``)."""
    cand = torch.stack([ca, cb], dim=1)
    w = torch.stack([wa, wb], dim=1)
    return _fc(x, cand, w, coef, N_COEF_SIG, 2, inv_tau)


def multilinear_logic(x, cand, w, s, arity):
    """Hybrid (discrete forward, multilinear surrogate gradient) LUT layer:
    ``cand/w[OUT,arity,K]``, ``s[OUT,2**arity] = sigmoid(logits)`` -> ``[B,OUT]``
    (``silogic/kernels/multilinear.py:130-176``)."""
    return _fc(x, cand, w, s, N_HYBRID_S, int(arity))


# --------------------------------------------------------------------- conv
def _kernel_size(H, W, pad, Ho, Wo, stride):
    if stride != 1:
        raise NotImplementedError("the conv-tree kernels support stride 1 (every reference model)")
    kh, kw = H + 2 * pad - Ho + 1, W + 2 * pad - Wo + 1
    if kh != kw or kh <= 0:
        raise ValueError(f"output {Ho}x{Wo} does not follow from a square kernel on {H}x{W}")
    return kh


def _conv(x, cm, ch, cw, w, params, node, arity, depth, stride, pad, Ho, Wo,
          deterministic=False):
    if x.dim() != 4:
        raise ValueError(f"x must be [B, C, H, W], got {tuple(x.shape)}")
    B, C, H, W = x.shape
    k = _kernel_size(H, W, pad, Ho, Wo, stride)
    if cm.dim() == 2:                                # fixed leaves [N, leaves] -> K = 1
        cm, ch, cw = cm.unsqueeze(-1), ch.unsqueeze(-1), cw.unsqueeze(-1)
    N, L, K = cm.shape
    if L != arity ** depth:
        raise ValueError(f"{L} leaves for an arity-{arity} tree of depth {depth}")
    cand = (cm.long() * (k * k) + ch.long() * k + cw.long()).to(torch.int32).contiguous()
    from .. import _hard
    _hard.check_index_range(cand, C * k * k, "conv leaf candidates")
    meta = dict(cand=cand, K=K, ste=DIRECT_WEIGHTS if w is not None else 0, node=node,
                arity=arity, depth=depth, gate_hard=0, inv_tau=1.0, kernel=k, pad=pad, n_out=N,
                wire_r=0, pool=1)
    if deterministic:
        meta["deterministic"] = True
    xt = ToFeatureMajor.apply(x.reshape(B, -1).float())
    yt = ConvSoft.apply(xt, params, w.float() if w is not None else None, meta, (C, H, W))
    return FromFeatureMajor.apply(yt, B).view(B, N, Ho, Wo).to(x.dtype)


def tree_conv(x, coef, cm, ch, cw, depth, stride, pad, Ho, Wo):
    """Fixed-connectome gate-tree convolution: ``coef[N, 2**depth-1, 4]`` BasisProj
    coefficients (nodes level 0 first), leaves ``cm/ch/cw[N, 2**depth]`` = (channel,
    dy, dx) -> ``[B, N, Ho, Wo]`` (``silogic/kernels/conv.py:354-400``)."""
    return _conv(x, cm, ch, cw, None, coef, N_COEF, 2, int(depth), stride, pad, Ho, Wo)


def tree_conv_topk(x, coef, w, cm, ch, cw, depth, K, stride, pad, Ho, Wo):
    """Top-K gate-tree convolution: ``w[N, 2**depth, K]`` post-softmax leaf weights,
    candidates ``cm/ch/cw[N, 2**depth, K]`` (``silogic/kernels/conv_topk.py:139-189``)."""
    if cm.shape[-1] != K:
        raise ValueError(f"candidates carry {cm.shape[-1]} per leaf, K = {K}")
    return _conv(x, cm, ch, cw, w, coef, N_COEF, 2, int(depth), stride, pad, Ho, Wo)


def conv_hybrid(x, s, w, cm, ch, cw, depth, node_arity, K, stride, pad, Ho, Wo):
    """Hybrid LUT-tree convolution: ``s[N, total_nodes, 2**node_arity]`` =
    ``sigmoid(logits)`` (levels concatenated, level 0 first), ``w[N, leaves, K]``
    (``silogic/kernels/conv_hybrid.py:161-213``)."""
    if cm.shape[-1] != K:
        raise ValueError(f"candidates carry {cm.shape[-1]} per leaf, K = {K}")
    return _conv(x, cm, ch, cw, w, s, N_HYBRID_S, int(node_arity), int(depth), stride, pad,
                 Ho, Wo)


def build_inverse_map(cm, ch, cw, C):
    """For each input channel, the (output channel n, leaf l, dy, dx) entries that read
    it, as CSR arrays ``(off[C+1], en, el, edy, edx)`` int32, entries of a channel in
    (n, l) order (``silogic/kernels/conv.py:247-265``).  The CUDA backward of
    :func:`tree_conv_af` does not need it (it is accepted for signature parity)."""
    N, L = cm.shape
    c = cm.reshape(-1).long().cpu()
    order = torch.argsort(c * (N * L) + torch.arange(N * L), stable=True)
    counts = torch.bincount(c, minlength=C)
    off = torch.zeros(C + 1, dtype=torch.int32)
    off[1:] = torch.cumsum(counts, 0).to(torch.int32)
    flat_n = torch.arange(N).repeat_interleave(L)
    flat_l = torch.arange(L).repeat(N)
    t = lambda a: a[order].to(torch.int32)
    return off, t(flat_n), t(flat_l), t(ch.reshape(-1).cpu()), t(cw.reshape(-1).cpu())


def tree_conv_af(x, coef, cm, ch, cw, inv, depth, stride, pad, Ho, Wo):
    """:func:`tree_conv` with a deterministic input gradient: the backward writes every
    leaf gradient once and gathers each input element's sum in a fixed order instead of
    accumulating it with atomics (``silogic/kernels/conv.py:301-351``), so ``x.grad`` is
    bit-identical from run to run.  ``inv`` (from :func:`build_inverse_map`) is
    accepted for signature parity."""
    return _conv(x, cm, ch, cw, None, coef, N_COEF, 2, int(depth), stride, pad, Ho, Wo,
                 deterministic=True)
