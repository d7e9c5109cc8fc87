"""Generate the golden fixtures in this folder by running the REFERENCE silogic.

Run it in a container where the reference source tree is importable:

    PYTHONPATH=<path to reference checkout> PYTHONDONTWRITEBYTECODE=1 \
        python tests/golden/make_golden.py <path to reference checkout> [prims fc conv cont]

Every case builds a network with the reference constructors, overwrites every
learnable parameter with N(0, 1) draws from a seeded generator (so gate choices
are not all the residual-init "A" gate), draws seeded inputs, and records

* ``ctor`` / ``kwargs``: the constructor call (JSON) -- silogic_b200 exposes the
  same classes, so a test rebuilds the net and loads ``sd/*``;
* ``sd/<name>``: the full reference ``state_dict`` (parameters and buffers);
* ``x``: the input batch;
* ``hard``: ``model.forward_hard(x)`` -- integer GroupSum counts (float dtype);
* ``feat``: the soft activations that enter the head (``model._run(x, False)``);
* ``logits``: the soft forward ``model(x)`` (training mode, as in a train step);
* ``grad/<name>``: gradients of ``(logits * R).sum()`` w.r.t. every parameter
  (and ``grad/x`` w.r.t. the input where it is a leaf), ``R`` = ``rmat``.

The reference is only imported here; nothing at test time reads it.
"""
import json
import os
import sys

import numpy as np
import torch

OUT_DIR = os.path.dirname(os.path.abspath(__file__))


def _randomise(model, seed):
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for p in model.parameters():
            p.copy_(torch.randn(p.shape, generator=g))


def _bits(shape, seed, p=0.3):
    g = torch.Generator().manual_seed(seed)
    return (torch.rand(shape, generator=g) < p).float()


def _uniform(shape, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.rand(shape, generator=g)


def _record(name, model, x, extra_pre=None, x_leaf=True, ctor=None, kwargs=None,
            store=None, img_shape=None, x_hard=None):
    """Run hard + soft fwd/bwd on the reference and save an .npz fixture.  ``x_hard``:
    a separate binary input for the hard path (fixtures with continuous soft inputs)."""
    import silogic  # noqa: F401  (reference)
    store = dict(store or {})
    if x_hard is not None:
        store["x_hard"] = x_hard.numpy()
    model.train()
    with torch.no_grad():
        xh = x if x_hard is None else x_hard
        xin = extra_pre.forward_hard(xh) if extra_pre is not None else xh
        if extra_pre is not None:
            xin = _encoded_to_image(xin, img_shape)
        hard = model.forward_hard(xin)
    xr = x.clone().requires_grad_(x_leaf)
    xs = xr
    if extra_pre is not None:
        xs = _encoded_to_image(extra_pre(xr), img_shape)
    feat = model._run(xs, hard=False)
    logits = model.head(feat)
    g = torch.Generator().manual_seed(12345)
    rmat = torch.randn(logits.shape, generator=g)
    (logits * rmat).sum().backward()
    out = {
        "ctor": np.array(ctor), "kwargs": np.array(json.dumps(kwargs)),
        "x": x.numpy(), "hard": hard.numpy(), "feat": feat.detach().numpy(),
        "logits": logits.detach().numpy(), "rmat": rmat.numpy(),
    }
    for k, v in model.state_dict().items():
        out["sd/" + k] = v.numpy()
    for k, p in model.named_parameters():
        if p.grad is not None:
            out["grad/" + k] = p.grad.numpy()
    if extra_pre is not None:
        for k, v in extra_pre.state_dict().items():
            out["encsd/" + k] = v.numpy()
        for k, p in extra_pre.named_parameters():
            out["encgrad/" + k] = p.grad.numpy()
    if x_leaf and xr.grad is not None:
        out["grad/x"] = xr.grad.numpy()
    out.update(store)
    np.savez_compressed(os.path.join(OUT_DIR, name + ".npz"), **out)
    print(f"{name}: hard {hard.shape} logits {logits.shape}")


def _encoded_to_image(enc, shape):
    """[B, C*H*W*bits] encoder output -> [B, C*bits, H, W], channel = c*bits + bit."""
    B, C, H, W = shape
    bits = enc.shape[1] // (C * H * W)
    return enc.view(B, C, H, W, bits).permute(0, 1, 4, 2, 3).reshape(B, C * bits, H, W)


def fc_cases():
    from silogic.models import LogicNet
    cases = [
        ("fc_gate16_fixed", dict(in_dim=64, width=120, depth=3, node="gate16",
                                 connectome="fixed", tau=10.0, seed=0)),
        ("fc_gate16_topk", dict(in_dim=64, width=120, depth=3, node="gate16",
                                connectome="topk", k=8, tau=10.0, seed=1)),
        ("fc_gate16_topk_hardsel", dict(in_dim=64, width=120, depth=2, node="gate16",
                                        connectome="topk", k=4, tau=10.0, seed=2,
                                        gate_select="hard", wire_residual=0.25)),
        ("fc_walsh_topk", dict(in_dim=64, width=120, depth=3, node="walsh",
                               connectome="topk", k=8, tau=10.0, seed=3)),
        ("fc_walsh_fixed_a3", dict(in_dim=64, width=120, depth=2, node="walsh",
                                   arity=3, connectome="fixed", tau=10.0, seed=4,
                                   node_tau=2.0)),
        ("fc_multilinear_a2_ste", dict(in_dim=64, width=120, depth=2, node="multilinear",
                                       connectome="topk", k=8, tau=10.0, seed=5,
                                       gate_select="hard")),
        ("fc_multilinear_a6", dict(in_dim=64, width=120, depth=2, node="multilinear",
                                   arity=6, connectome="topk", k=3, tau=10.0, seed=6)),
        ("fc_hybrid_a4", dict(in_dim=64, width=120, depth=2, node="hybrid", arity=4,
                              connectome="topk", k=4, tau=10.0, seed=7)),
        ("fc_hybrid_a3_fixed", dict(in_dim=64, width=120, depth=2, node="hybrid",
                                    arity=3, connectome="fixed", tau=10.0, seed=8)),
    ]
    for i, (name, kw) in enumerate(cases):
        torch.manual_seed(100 + i)
        m = LogicNet(**kw)
        _randomise(m, 200 + i)
        x = _bits((100, 64), 300 + i)
        _record(name, m, x, ctor="LogicNet", kwargs=kw)


def conv_cases():
    from silogic.models import LogicTreeNet, LogicConvNet
    from silogic.encoders import LearnedThermometerEncoder
    from silogic.data import binarize_spatial
    cases = [
        ("conv_gate16_topk_d2", "LogicTreeNet",
         dict(in_channels=6, in_hw=8, channels=[16, 32], head_widths=[80],
              tree_depth=2, node="gate16", tau=20.0, seed=0)),
        ("conv_gate16_fixed_d2", "LogicTreeNet",
         dict(in_channels=6, in_hw=8, channels=[16, 32], head_widths=[80],
              tree_depth=2, node="gate16", connect="fixed", head_connect="fixed",
              tau=20.0, seed=1)),
        ("conv_gate16_topk_d3_wire", "LogicConvNet",
         dict(in_channels=6, in_hw=8, channels=[16, 24], head_widths=[60, 40],
              tree_depth=3, node="gate16", tau=5.0, seed=2, wire_residual=0.25,
              gate_select="hard")),
        ("conv_hybrid_a4_d1", "LogicConvNet",
         dict(in_channels=6, in_hw=8, channels=[16, 32], head_widths=[80],
              tree_depth=1, node="hybrid", arity=4, k=4, n_chan=2, tau=20.0, seed=3)),
    ]
    for i, (name, ctor, kw) in enumerate(cases):
        torch.manual_seed(400 + i)
        cls = {"LogicTreeNet": LogicTreeNet, "LogicConvNet": LogicConvNet}[ctor]
        m = cls(**kw)
        _randomise(m, 500 + i)
        img = _uniform((40, 3, 8, 8), 600 + i)
        x = binarize_spatial(img, [1 / 3, 2 / 3]).float()   # 6 channels
        _record(name, m, x, x_leaf=True, ctor=ctor, kwargs=kw,
                store={"img": img.numpy()})

    # multilinear arity-6 conv with the learned thermometer encoder (C4 family)
    torch.manual_seed(450)
    kw = dict(in_channels=9, in_hw=8, channels=[16, 32], head_widths=[100, 100],
              tree_depth=1, node="multilinear", arity=6, connect="topk", k=8,
              n_chan=4, gate_select="hard", tau=12.0, seed=4)
    m = LogicConvNet(**kw)
    enc = LearnedThermometerEncoder(3 * 8 * 8, 3)
    _randomise(m, 550)
    img = _uniform((24, 3, 8, 8), 650)
    x = img.reshape(24, -1)
    _record("conv_multilinear_a6_enc", m, x, extra_pre=enc, x_leaf=True,
            ctor="LogicConvNet", kwargs=kw, img_shape=(24, 3, 8, 8),
            store={"enc_kwargs": np.array(json.dumps(dict(num_features=192, bits=3))),
                   "img_shape": np.array([24, 3, 8, 8])})


def prim_cases():
    """Packing / GroupSum / thermometer known answers from the reference ops."""
    from silogic.bitpacking.ops import pack_bits, group_sum_packed, n_words
    from silogic.data import binarize_spatial, FIVE_THRESH
    out = {}
    rng = np.random.default_rng(7)
    for B, F in [(1, 1), (63, 8), (64, 64), (65, 256), (200, 784)]:
        x = rng.integers(0, 2, (B, F), dtype=np.uint8)
        out[f"pack_{B}_{F}/x"] = x
        out[f"pack_{B}_{F}/packed"] = pack_bits(x)
    xs = rng.integers(0, 2, (130, 200), dtype=np.uint8)
    p = pack_bits(xs)
    out["gsum/x"] = xs
    out["gsum/logits_tau4"] = group_sum_packed(p, 130, 10, 4.0)
    out["nwords"] = np.array([n_words(b) for b in [1, 64, 65, 128, 129]])
    img = torch.rand(5, 3, 6, 6, generator=torch.Generator().manual_seed(3))
    img[0, 0, 0, :] = torch.tensor([1 / 6, 2 / 6, 3 / 6, 4 / 6, 5 / 6, 0.0])
    out["thermo/img"] = img.numpy()
    out["thermo/bits"] = binarize_spatial(img, FIVE_THRESH).numpy()
    np.savez_compressed(os.path.join(OUT_DIR, "prims.npz"), **out)
    print("prims written")


def continuous_conv_cases():
    """Conv nets on continuous U[0,1] inputs: OR-pool windows then tie only at padding, so
    the soft gradients pin the reference's own pool routing (binary inputs tie
    everywhere).  The hard path gets the thresholded input ``x >= 0.5`` (``x_hard``)."""
    from silogic.models import LogicTreeNet, LogicConvNet
    cases = [
        ("conv_cont_gate16_topk_d2", "LogicTreeNet",
         dict(in_channels=6, in_hw=8, channels=[16, 32], head_widths=[80],
              tree_depth=2, node="gate16", tau=20.0, seed=10)),
        ("conv_cont_gate16_fixed_d1", "LogicConvNet",
         dict(in_channels=6, in_hw=8, channels=[12, 24], head_widths=[60],
              tree_depth=1, node="gate16", connect="fixed", tau=5.0, seed=11)),
        ("conv_cont_walsh_k8_d2", "LogicConvNet",
         dict(in_channels=6, in_hw=8, channels=[12, 20], head_widths=[100],
              tree_depth=2, node="walsh", k=8, n_chan=2, tau=5.0, seed=12)),
        ("conv_cont_multilinear_a3_d1", "LogicConvNet",
         dict(in_channels=6, in_hw=8, channels=[12, 20], head_widths=[100],
              tree_depth=1, node="multilinear", arity=3, k=4, tau=5.0, seed=13)),
    ]
    for i, (name, ctor, kw) in enumerate(cases):
        torch.manual_seed(700 + i)
        cls = {"LogicTreeNet": LogicTreeNet, "LogicConvNet": LogicConvNet}[ctor]
        m = cls(**kw)
        _randomise(m, 800 + i)
        # the input seed whose pool windows are farthest from a near-tie (largest two
        # values of a window apart by more than 1e-6, relative, unless exactly equal: an
        # exact tie comes from identical all-padding taps and resolves the same way in
        # any implementation) on the reference's own forward, so the routing -- and
        # every gradient -- is fixed beyond fp32 rounding
        best = None
        for s in range(900 + 40 * i, 940 + 40 * i):
            gap = _min_pool_gap(m, _uniform((16, 6, 8, 8), s))
            if best is None or gap > best[0]:
                best = (gap, s)
        gap, s = best
        assert gap > 1e-6, f"{name}: every input seed has a near-tie ({gap:.1e})"
        x = _uniform((16, 6, 8, 8), s)
        print(f"{name}: input seed {s}, smallest pool-window gap {gap:.2e}")
        _record(name, m, x, x_leaf=True, ctor=ctor, kwargs=kw, x_hard=(x >= 0.5).float(),
                store={"input_seed": np.array(s), "min_pool_gap": np.array(gap)})


@torch.no_grad()
def _min_pool_gap(model, x):
    """Smallest nonzero relative gap between the two largest values of any 2x2 pool
    window of the reference's soft conv outputs (training mode) over all conv blocks."""
    model.train()
    h, gap = x, float("inf")
    blocks = list(model.blocks)
    for j in range(0, len(blocks), 2):
        y = blocks[j](h)
        B, n, H, W = y.shape
        w = y[:, :, :H // 2 * 2, :W // 2 * 2].reshape(B, n, H // 2, 2, W // 2, 2)
        w = w.permute(0, 1, 2, 4, 3, 5).reshape(-1, 4)
        top = torch.topk(w, 2, dim=1).values
        rel = (top[:, 0] - top[:, 1]) / top[:, 0].abs().clamp_min(1e-30)
        rel = rel[rel > 0]                       # exact ties resolve identically
        if rel.numel():
            gap = min(gap, float(rel.min()))
        h = blocks[j + 1](y)
    return gap


if __name__ == "__main__":
    if len(sys.argv) > 1:
        sys.path.insert(0, sys.argv[1])
    only = sys.argv[2:]
    if not only or "prims" in only:
        prim_cases()
    if not only or "fc" in only:
        fc_cases()
    if not only or "conv" in only:
        conv_cases()
    if not only or "cont" in only:
        continuous_conv_cases()
