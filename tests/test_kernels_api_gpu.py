"""The reference's fused-kernel function API (``silogic.kernels``) on the CUDA kernels,
against plain torch fp32 restatements of the reference's formulas
(``silogic/kernels/{dense,warp,multilinear,conv,conv_topk,conv_hybrid}.py``): forward
values and the gradients with respect to every tensor argument within
1e-5 (|ref| + max|ref|) + 1e-7 (fp32; the summation order differs)."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import silogic_b200.kernels as K
from test_soft_gpu import assert_grad_close

pytestmark = pytest.mark.gpu
dev = "cuda"


def _leaf(t):
    return t.detach().clone().to(dev).requires_grad_(True)


def _check(got, ref, inputs_got, inputs_ref, gout):
    assert_grad_close(got, ref.detach().numpy(), "forward")
    (got * gout.to(dev)).sum().backward()
    (ref * gout).sum().backward()
    for i, (a, b) in enumerate(zip(inputs_got, inputs_ref)):
        assert_grad_close(a.grad, b.grad.numpy(), f"arg {i}")


def test_flags():
    assert all([K.HAS_DENSE, K.HAS_CONV, K.HAS_CONV_TOPK, K.HAS_WARP, K.HAS_MULTILINEAR,
                K.HAS_CONV_HYBRID])


@pytest.mark.parametrize("which", ["dense", "warp"])
@pytest.mark.parametrize("B,IN,OUT,Kc", [(1, 50, 70, 1), (37, 300, 200, 8), (515, 784, 1000, 16)])
def test_dense_and_warp_logic(which, B, IN, OUT, Kc):
    g = torch.Generator().manual_seed(B + Kc)
    x = torch.rand(B, IN, generator=g)
    ca = torch.randint(0, IN, (OUT, Kc), generator=g, dtype=torch.int32)
    cb = torch.randint(0, IN, (OUT, Kc), generator=g, dtype=torch.int32)
    wa = torch.softmax(torch.randn(OUT, Kc, generator=g), 1)
    wb = torch.softmax(torch.randn(OUT, Kc, generator=g), 1)
    coef = torch.randn(OUT, 4, generator=g)
    gout = torch.randn(B, OUT, generator=g)
    ref_in = [t.clone().requires_grad_(True) for t in (x, wa, wb, coef)]
    xr, war, wbr, cr = ref_in
    a = (xr[:, ca.long()] * war).sum(-1)
    b = (xr[:, cb.long()] * wbr).sum(-1)
    z = cr[:, 0] + cr[:, 1] * a + cr[:, 2] * b + cr[:, 3] * (a * b)
    got_in = [_leaf(t) for t in (x, wa, wb, coef)]
    if which == "dense":
        got = K.dense_logic(got_in[0], ca.to(dev), cb.to(dev), *got_in[1:])
        ref = z
    else:
        got = K.warp_logic(got_in[0], ca.to(dev), cb.to(dev), *got_in[1:], 0.5)
        ref = torch.sigmoid(z * 0.5)
    _check(got, ref, got_in, ref_in, gout)


def _corners(n):
    return torch.tensor([[(p >> j) & 1 for j in range(n)] for p in range(2 ** n)], dtype=torch.float32)


def _hybrid(ops, s):
    """ops [..., n] (children), s [..., 2^n] broadcastable -> discrete value with the soft
    multilinear gradient (silogic/nodes.py:198-207)."""
    n = ops.shape[-1]
    c = _corners(n)
    au = ops.unsqueeze(-2)                                          # [..., 1, n]
    soft = ((c * au + (1 - c) * (1 - au)).prod(-1) * s).sum(-1)
    idx = ((ops >= 0.5).long() << torch.arange(n)).sum(-1, keepdim=True)
    # the discrete value carries no gradient (HybridNode evaluates it under no_grad, and
    # the fused kernel's s-gradient is the soft surrogate's alone)
    disc = torch.gather(s.detach().expand(*ops.shape[:-1], s.shape[-1]), -1, idx).squeeze(-1)
    return disc + soft - soft.detach()


@pytest.mark.parametrize("arity,Kc,B", [(2, 4, 33), (3, 1, 200), (6, 8, 64)])
def test_multilinear_logic(arity, Kc, B):
    g = torch.Generator().manual_seed(arity * 10 + Kc)
    IN, OUT = 120, 90
    x = torch.rand(B, IN, generator=g)
    cand = torch.randint(0, IN, (OUT, arity, Kc), generator=g, dtype=torch.int32)
    w = torch.softmax(torch.randn(OUT, arity, Kc, generator=g), -1)
    s = torch.sigmoid(torch.randn(OUT, 2 ** arity, generator=g))
    gout = torch.randn(B, OUT, generator=g)
    ref_in = [t.clone().requires_grad_(True) for t in (x, w, s)]
    xr, wr, sr = ref_in
    ops = (xr[:, cand.long()] * wr).sum(-1)                          # [B, OUT, n]
    ref = _hybrid(ops, sr.unsqueeze(0))
    got_in = [_leaf(t) for t in (x, w, s)]
    got = K.multilinear_logic(got_in[0], cand.to(dev), got_in[1], got_in[2], arity)
    _check(got, ref, got_in, ref_in, gout)


def _ref_tree_conv(x, cm, ch, cw, w, pad, Ho, Wo, node, params, depth, arity):
    """Plain torch: leaf = sum_k w * padded x at (channel, y + dy, x + dx), then the tree
    level by level (node m takes children m*arity ..), node ids level 0 first."""
    xp = F.pad(x, (pad, pad, pad, pad))
    ys = torch.arange(Ho).view(Ho, 1)
    xs = torch.arange(Wo).view(1, Wo)
    cmL, chL, cwL = (t.long()[..., None, None] for t in (cm, ch, cw))
    v = xp[:, cmL, chL + ys, cwL + xs]                               # [B, N, L, K, Ho, Wo]
    vals = (v * w[None, ..., None, None]).sum(3)                     # [B, N, L, Ho, Wo]
    vals = [vals[:, :, l] for l in range(vals.shape[2])]
    nid = 0
    for _ in range(depth):
        nxt = []
        for m in range(0, len(vals), arity):
            ch_ = vals[m:m + arity]
            prm = params[:, nid]                                     # [N, P]
            if node == "coef":
                c = prm[None, :, :, None, None]
                nxt.append(c[:, :, 0] + c[:, :, 1] * ch_[0] + c[:, :, 2] * ch_[1] + c[:, :, 3] * (ch_[0] * ch_[1]))
            else:
                ops = torch.stack(ch_, -1)                           # [B, N, Ho, Wo, n]
                nxt.append(_hybrid(ops, prm[None, :, None, None, :]))
            nid += 1
        vals = nxt
    return vals[0]


@pytest.mark.parametrize("fn", ["tree_conv", "tree_conv_af", "tree_conv_topk", "conv_hybrid"])
@pytest.mark.parametrize("depth", [1, 2, 3])
def test_conv_functions(fn, depth):
    arity = 3 if (fn == "conv_hybrid" and depth == 1) else 2
    if fn == "conv_hybrid" and depth == 3:
        depth = 2
    g = torch.Generator().manual_seed(depth * 7 + len(fn))
    B, C, H, Wd, N, pad = 20, 5, 9, 7, 12, 1
    Ho, Wo = H, Wd
    L = arity ** depth
    Kc = 1 if fn in ("tree_conv", "tree_conv_af") else 4
    cm = torch.randint(0, C, (N, L, Kc), generator=g, dtype=torch.int32)
    ch = torch.randint(0, 3, (N, L, Kc), generator=g, dtype=torch.int32)
    cw = torch.randint(0, 3, (N, L, Kc), generator=g, dtype=torch.int32)
    x = torch.rand(B, C, H, Wd, generator=g)
    nodes = (L - 1) // (arity - 1)
    if fn == "conv_hybrid":
        prm = torch.sigmoid(torch.randn(N, nodes, 2 ** arity, generator=g))
    else:
        prm = torch.randn(N, nodes, 4, generator=g)
    w = torch.softmax(torch.randn(N, L, Kc, generator=g), -1) if Kc > 1 else torch.ones(N, L, 1)
    gout = torch.randn(B, N, Ho, Wo, generator=g)
    node = "hybrid" if fn == "conv_hybrid" else "coef"
    ref_in = [t.clone().requires_grad_(True) for t in ((x, prm, w) if Kc > 1 else (x, prm))]
    ref = _ref_tree_conv(ref_in[0], cm, ch, cw, ref_in[2] if Kc > 1 else w, pad, Ho, Wo, node,
                         ref_in[1], depth, arity)
    got_in = [_leaf(t) for t in ((x, prm, w) if Kc > 1 else (x, prm))]
    d = lambda t: t.to(dev)
    if fn == "tree_conv":
        got = K.tree_conv(got_in[0], got_in[1], d(cm[..., 0]), d(ch[..., 0]), d(cw[..., 0]), depth, 1,
                          pad, Ho, Wo)
    elif fn == "tree_conv_af":
        inv = K.build_inverse_map(cm[..., 0], ch[..., 0], cw[..., 0], C)
        got = K.tree_conv_af(got_in[0], got_in[1], d(cm[..., 0]), d(ch[..., 0]), d(cw[..., 0]), inv,
                             depth, 1, pad, Ho, Wo)
    elif fn == "tree_conv_topk":
        got = K.tree_conv_topk(got_in[0], got_in[1], got_in[2], d(cm), d(ch), d(cw), depth, Kc, 1,
                               pad, Ho, Wo)
    else:
        got = K.conv_hybrid(got_in[0], got_in[1], got_in[2], d(cm), d(ch), d(cw), depth, arity, Kc,
                            1, pad, Ho, Wo)
    _check(got, ref, got_in, ref_in, gout)


def test_tree_conv_af_input_gradient_is_bit_reproducible():
    """Two backward passes of tree_conv_af give bit-identical x.grad (no atomics), equal
    to tree_conv's within rounding."""
    g = torch.Generator().manual_seed(3)
    B, C, H, N, depth = 300, 6, 16, 40, 2
    cm = torch.randint(0, C, (N, 4), generator=g, dtype=torch.int32).to(dev)
    ch = torch.randint(0, 3, (N, 4), generator=g, dtype=torch.int32).to(dev)
    cw = torch.randint(0, 3, (N, 4), generator=g, dtype=torch.int32).to(dev)
    coef = torch.randn(N, 3, 4, generator=g).to(dev)
    x0 = torch.rand(B, C, H, H, generator=g).to(dev)
    gout = torch.randn(B, N, H, H, generator=g).to(dev)
    inv = K.build_inverse_map(cm, ch, cw, C)
    grads = []
    for fn in ("af", "af", "plain"):
        x = x0.clone().requires_grad_(True)
        y = (K.tree_conv_af(x, coef, cm, ch, cw, inv, depth, 1, 1, H, H) if fn == "af"
             else K.tree_conv(x, coef, cm, ch, cw, depth, 1, 1, H, H))
        (y * gout).sum().backward()
        grads.append(x.grad.clone())
    assert torch.equal(grads[0], grads[1])
    assert_grad_close(grads[2], grads[0].cpu().numpy(), "tree_conv vs tree_conv_af")
