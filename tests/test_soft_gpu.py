"""Soft forward + backward on the GPU vs the reference golden vectors and the
torch-fp32 oracle.

Tolerances: activations |got - ref| <= 1e-5 |ref| + 1e-6; gradients norm-wise
|got - ref| <= 1e-5 (|ref| + max|ref|) + 1e-7 (fp32, summation order differs);
GroupSum logits exact except where a feature lies within 1e-5 of the 0.5
threshold (a 1-ulp difference there flips a count by design of feature_ste).
"""
import numpy as np
import pytest
import torch

from helpers import FIXTURES, build_model, encoder_image

pytestmark = pytest.mark.gpu
dev = "cuda"
FC = [n for n in FIXTURES if n.startswith("fc_")]
CONV = [n for n in FIXTURES if n.startswith("conv_")]


def assert_grad_close(got, ref, what, atol=1e-7):
    got = got.detach().cpu().numpy() if torch.is_tensor(got) else got
    tol = 1e-5 * (np.abs(ref) + np.abs(ref).max()) + atol
    bad = np.abs(got - ref) > tol
    assert not bad.any(), f"{what}: {bad.sum()} of {bad.size} entries off, max err " \
                          f"{np.abs(got - ref).max():.3e} (ref max {np.abs(ref).max():.3e})"


def assert_logits_close(logits, ref, feat_ref, tau):
    d = np.abs(logits - ref) * tau                        # in counts
    near = (np.abs(feat_ref - 0.5) <= 1e-5).sum(1)[:, None]   # per sample
    assert np.all(d <= near + 1e-3), f"logit counts differ beyond threshold ties: {d.max()}"


def _conv_grads_vs_oracle(name, m, enc, z, x):
    import json
    from oracle import soft as OS
    from oracle.spec import net_spec
    with torch.no_grad():
        xs = encoder_image(enc(x), z) if enc is not None else x
    routing = our_pool_routing(m, xs.detach())
    sd = {k: v.detach().cpu() for k, v in m.state_dict().items()}
    spec = net_spec(str(z["ctor"]), json.loads(str(z["kwargs"])), {k: v.numpy() for k, v in sd.items()})
    P = OS.params_from_sd(sd)
    xr = torch.from_numpy(z["x"]).clone().requires_grad_(True)
    xo = xr
    thr = None
    if enc is not None:
        thr = torch.from_numpy(z["encsd/thresholds"]).clone().requires_grad_(True)
        xo = encoder_image(OS.learned_thermometer(xr, thr), z)
    feat = OS.net_features(spec, P, xo, training=True, pool_index=routing)
    lo = OS.group_sum(feat, spec["num_classes"], spec["tau"])
    (lo * torch.from_numpy(z["rmat"])).sum().backward()
    assert_grad_close(x.grad, xr.grad.numpy(), f"{name} x")
    for n, p in m.named_parameters():
        assert_grad_close(p.grad, P[n].grad.numpy(), f"{name} {n}")
    if enc is not None:
        assert_grad_close(enc.thresholds.grad, thr.grad.numpy(), "encoder thresholds")


def run_soft(name):
    m, enc, z, _ = build_model(name, dev)
    m.train()
    x = torch.from_numpy(z["x"]).to(dev).requires_grad_(True)
    xs = x
    if enc is not None:
        xs = encoder_image(enc(x), z)
    feat = m._run(xs, hard=False)
    logits = m(xs)
    (logits * torch.from_numpy(z["rmat"]).to(dev)).sum().backward()
    return m, enc, z, x, feat, logits


@pytest.mark.parametrize("name", FIXTURES)
def test_soft_matches_reference_golden(name):
    """Forward: strict vs the reference.  Gradients: FC nets and conv nets on continuous
    inputs (``conv_cont_*``, where pool windows tie only at padding) strict vs the
    reference; conv nets on binary inputs (OR-pool) strict vs the oracle -- itself pinned
    to these fixtures on the CPU -- replaying this package's pool routing, because the
    reference's choice at windows tied within fp32 rounding depends on its own rounding."""
    m, enc, z, x, feat, logits = run_soft(name)
    np.testing.assert_allclose(feat.detach().cpu().numpy(), z["feat"], rtol=1e-5, atol=1e-6)
    assert_logits_close(logits.detach().cpu().numpy(), z["logits"], z["feat"], m.head.tau)
    params = dict(m.named_parameters())
    if name.startswith("conv_") and "x_hard" not in z.files:
        # binary inputs: pool windows tie, see the docstring
        _conv_grads_vs_oracle(name, m, enc, z, x)
        return
    # conv nets: a deep block's gradient can be a near-total cancellation of O(1) terms
    # (max |grad| ~1e-5 while the model's are ~1), so its fp32 noise is ~1e-7 absolute
    atol = 1e-6 if name.startswith("conv_") else 1e-7
    for k in z.files:
        if k.startswith("grad/"):
            n = k[5:]
            got = x.grad if n == "x" else params[n].grad
            assert got is not None, n
            assert_grad_close(got, z[k], f"{name} grad {n}", atol)
    if enc is not None:
        assert_grad_close(enc.thresholds.grad, z["encgrad/thresholds"], "encoder thresholds")


def _rand_model(ctor, kw, seed):
    import silogic_b200 as S
    torch.manual_seed(seed)
    m = getattr(S, ctor)(**kw)
    g = torch.Generator().manual_seed(seed + 1)
    with torch.no_grad():
        for p in m.parameters():
            p.copy_(torch.randn(p.shape, generator=g))
    return m


@torch.no_grad()
def our_pool_routing(m, x):
    """Per conv block, the window element our first-max OR-pool selects (flat index into
    H*W), computed from this package's own unpooled block outputs."""
    idx, h = [], x
    blocks = list(m.blocks)
    for i in range(0, len(blocks), 2):
        conv = blocks[i]
        y = conv(h)                                              # unpooled, our kernel
        r = m.wire_channels(conv, h.shape[1])
        if r:
            y = torch.cat([h[:, :r], y[:, r:]], 1)
        B, n, H, W = y.shape
        Hp, Wp = H // 2, W // 2
        win = y[:, :, :Hp * 2, :Wp * 2].reshape(B, n, Hp, 2, Wp, 2).permute(0, 1, 2, 4, 3, 5)
        a = win.reshape(B, n, Hp, Wp, 4).argmax(-1)              # first maximum
        hp = torch.arange(Hp, device=y.device).view(1, 1, Hp, 1)
        wp = torch.arange(Wp, device=y.device).view(1, 1, 1, Wp)
        idx.append(((2 * hp + a // 2) * W + 2 * wp + a % 2).cpu())
        h = torch.nn.functional.max_pool2d(y, 2, 2)
    return idx


def oracle_soft(ctor, kw, m, x, rmat, pool_index=None):
    from oracle import soft as OS
    from oracle.spec import net_spec
    sd = {k: v.detach().cpu() for k, v in m.state_dict().items()}
    spec = net_spec(ctor, kw, {k: v.numpy() for k, v in sd.items()})
    P = OS.params_from_sd(sd)
    xr = x.detach().cpu().clone().requires_grad_(True)
    feat = OS.net_features(spec, P, xr, training=True, pool_index=pool_index)
    logits = OS.group_sum(feat, spec["num_classes"], spec["tau"])
    (logits * rmat).sum().backward()
    return feat.detach().numpy(), logits.detach().numpy(), P, xr.grad


@pytest.mark.parametrize("kw", [
    dict(in_dim=784, width=2000, depth=3, node="walsh", connectome="topk", k=8, tau=10.0, seed=0),
    dict(in_dim=784, width=1600, depth=2, node="gate16", connectome="fixed", tau=10.0, seed=1),
    dict(in_dim=300, width=1000, depth=2, node="gate16", connectome="topk", k=16, tau=3.0, seed=2),
    dict(in_dim=300, width=500, depth=2, node="multilinear", arity=6, connectome="topk", k=2,
         tau=5.0, seed=3),
    dict(in_dim=300, width=500, depth=2, node="linear", arity=3, connectome="topk", k=4, tau=5.0,
         seed=4),
    dict(in_dim=300, width=500, depth=2, node="polynomial", arity=3, degree=2, connectome="topk",
         k=4, tau=5.0, seed=5),
    dict(in_dim=300, width=400, depth=2, node="polynomial", arity=4, connectome="fixed", tau=5.0,
         seed=6, degree=4),
], ids=["walsh_topk8", "gate16_fixed", "gate16_topk16", "multilinear6", "linear3", "poly3_d2",
        "poly4_full"])
@pytest.mark.parametrize("B", [1, 515])
def test_fc_soft_vs_oracle(kw, B):
    m = _rand_model("LogicNet", kw, 11)
    g = torch.Generator().manual_seed(B)
    x = (torch.rand(B, kw["in_dim"], generator=g) < 0.3).float()
    rmat = torch.randn(B, 10, generator=g)
    f_ref, l_ref, P, gx_ref = oracle_soft("LogicNet", kw, m, x, rmat)
    m = m.to(dev).train()
    xd = x.to(dev).requires_grad_(True)
    feat = m._run(xd, hard=False)
    np.testing.assert_allclose(feat.detach().cpu().numpy(), f_ref, rtol=1e-5, atol=1e-6)
    logits = m(xd)
    assert_logits_close(logits.detach().cpu().numpy(), l_ref, f_ref, m.head.tau)
    (logits * rmat.to(dev)).sum().backward()
    assert_grad_close(xd.grad, gx_ref.numpy(), "x")
    for n, p in m.named_parameters():
        assert_grad_close(p.grad, P[n].grad.numpy(), n)


def test_layer_and_node_level_soft_vs_torch_math():
    """LogicLayer.forward / Node.forward on [B, in] match the reference formulas."""
    import silogic_b200 as S
    torch.manual_seed(0)
    layer = S.LogicLayer(64, 96, node="walsh", connectome="topk", k=4, seed=3).to(dev)
    x = torch.rand(37, 64, device=dev)
    y = layer(x)
    w = torch.softmax(layer._conn.conn, 2)
    ops = torch.einsum("boak,oak->boa", x[:, layer._conn.cand], w)
    u = 2 * ops - 1
    t = layer.node.theta
    z = t[:, 0] + t[:, 1] * u[..., 0] + t[:, 2] * u[..., 1] + t[:, 3] * u[..., 0] * u[..., 1]
    torch.testing.assert_close(y, torch.sigmoid(z), rtol=1e-5, atol=1e-6)
    node = S.build_node("multilinear", 20, arity=3).to(dev)
    opnd = torch.rand(9, 20, 3, device=dev)
    c = node.corners
    ref = ((c * opnd.unsqueeze(2) + (1 - c) * (1 - opnd.unsqueeze(2))).prod(3)
           * torch.sigmoid(node.logits)[None]).sum(2)
    torch.testing.assert_close(node(opnd), ref, rtol=1e-5, atol=1e-6)


def test_groupsum_orpool_thermometer_soft():
    import silogic_b200 as S
    x = torch.rand(33, 50, device=dev, requires_grad=True)
    gs = S.GroupSum(5, tau=2.0, feature_ste=True)
    y = gs(x)
    ref = (x > 0.5).float().view(33, 5, 10).sum(2) / 2.0
    torch.testing.assert_close(y, ref)
    y.sum().backward()
    torch.testing.assert_close(x.grad, torch.full_like(x, 0.5))
    # OrPool: max with first-max gradient routing (ties are common on binary inputs)
    xi = (torch.rand(3, 4, 7, 6, device=dev) < 0.5).float().requires_grad_(True)
    xr = xi.detach().clone().requires_grad_(True)
    p = S.OrPool(2)
    yi = p(xi)
    yr = torch.nn.functional.max_pool2d(xr.cpu(), 2, 2)
    torch.testing.assert_close(yi.cpu(), yr)
    g = torch.randn_like(yi)
    yi.backward(g)
    xc = xr.detach().cpu().requires_grad_(True)
    torch.nn.functional.max_pool2d(xc, 2, 2).backward(g.cpu())
    torch.testing.assert_close(xi.grad.cpu(), xc.grad)
    # learned thermometer
    from oracle import soft as OS
    enc = S.LearnedThermometerEncoder(40, 3).to(dev)
    with torch.no_grad():
        enc.thresholds.copy_(torch.rand(40, 3))
    xe = torch.rand(21, 40, device=dev, requires_grad=True)
    out = enc(xe)
    thr = enc.thresholds.detach().cpu().clone().requires_grad_(True)
    xc = xe.detach().cpu().clone().requires_grad_(True)
    ref = OS.learned_thermometer(xc, thr)
    torch.testing.assert_close(out.cpu(), ref, rtol=0, atol=1e-6)
    gg = torch.randn_like(out)
    out.backward(gg)
    ref.backward(gg.cpu())
    assert_grad_close(xe.grad, xc.grad.numpy(), "enc x")
    assert_grad_close(enc.thresholds.grad, thr.grad.numpy(), "enc thr")


@pytest.mark.parametrize("kw", [
    dict(in_channels=15, in_hw=16, channels=[32, 64], head_widths=[320], tree_depth=2,
         node="gate16", tau=20.0, seed=0),
    dict(in_channels=6, in_hw=12, channels=[16, 24], head_widths=[90], tree_depth=3,
         node="gate16", connect="fixed", tau=3.0, seed=1, wire_residual=0.5),
    dict(in_channels=9, in_hw=12, channels=[16, 24], head_widths=[120, 60], tree_depth=1,
         node="multilinear", arity=6, k=8, n_chan=4, gate_select="hard", tau=12.0, seed=2),
    dict(in_channels=6, in_hw=10, channels=[12, 20], head_widths=[100], tree_depth=2,
         node="walsh", k=16, n_chan=2, tau=5.0, seed=3),
    dict(in_channels=6, in_hw=10, channels=[12, 20], head_widths=[100], tree_depth=2,
         node="hybrid", arity=3, k=4, tau=5.0, seed=4),
], ids=["gate16_topk_d2", "gate16_fixed_d3_wire", "multilinear6_ste", "walsh_k16_d2", "hybrid3_d2"])
@pytest.mark.parametrize("B", [3, 300])
def test_conv_soft_vs_oracle(kw, B):
    m = _rand_model("LogicConvNet", kw, 21)
    g = torch.Generator().manual_seed(B)
    C, hw = kw["in_channels"], kw["in_hw"]
    x = (torch.rand(B, C, hw, hw, generator=g) < 0.5).float()
    rmat = torch.randn(B, 10, generator=g)
    routing = our_pool_routing(m.to(dev).train(), x.to(dev))
    f_ref, l_ref, P, gx_ref = oracle_soft("LogicConvNet", kw, m.cpu(), x, rmat, routing)
    m = m.to(dev).train()
    xd = x.to(dev).requires_grad_(True)
    feat = m._run(xd, hard=False)
    np.testing.assert_allclose(feat.detach().cpu().numpy(), f_ref, rtol=1e-5, atol=1e-6)
    logits = m(xd)
    assert_logits_close(logits.detach().cpu().numpy(), l_ref, f_ref, m.head.tau)
    (logits * rmat.to(dev)).sum().backward()
    assert_grad_close(xd.grad, gx_ref.numpy(), "x")
    for n, p in m.named_parameters():
        assert_grad_close(p.grad, P[n].grad.numpy(), n)


def test_conv_layer_soft_unpooled_vs_oracle():
    import silogic_b200 as S
    from oracle import soft as OS
    from oracle.spec import conv_block_spec
    torch.manual_seed(1)
    conv = S.ConvLogicTree(5, 12, tree_depth=2, connect="topk", k=4, seed=7)
    with torch.no_grad():
        for p in conv.parameters():
            p.normal_()
    x = torch.rand(40, 5, 9, 7)
    sd = {k: v.detach() for k, v in conv.state_dict().items()}
    Bk = conv_block_spec({k: v.numpy() for k, v in sd.items()}, "", 5, 12, 3, 2, "topk", 4,
                         "gate16", 2, "softmax", 1.0)
    P = OS.params_from_sd(sd)
    ref = OS.conv_block(Bk, P, x, training=True)
    got = conv.to(dev)(x.to(dev))
    np.testing.assert_allclose(got.detach().cpu().numpy(), ref.detach().numpy(), rtol=1e-5, atol=1e-6)


def test_conv_backward_with_saved_pool_argmax_matches_recompute():
    """The backward that reads the forward's saved window argmax gives the gradients of
    the one that re-evaluates every window (gx within atomic-order rounding)."""
    import silogic_b200._soft as SS
    kw = dict(in_channels=15, in_hw=16, channels=[32, 64], head_widths=[320], tree_depth=2,
              node="gate16", tau=20.0, seed=0)
    m = _rand_model("LogicConvNet", kw, 31).to(dev).train()
    g = torch.Generator().manual_seed(5)
    x = (torch.rand(200, 15, 16, 16, generator=g) < 0.5).float().to(dev)
    rmat = torch.randn(200, 10, generator=g).to(dev)
    grads = []
    for save in (True, False):
        SS.SAVE_POOL_ARGMAX = save
        try:
            m.zero_grad()
            xd = x.clone().requires_grad_(True)
            (m(xd) * rmat).sum().backward()
            grads.append([xd.grad.clone()] + [p.grad.clone() for p in m.parameters()])
        finally:
            SS.SAVE_POOL_ARGMAX = True
    for a, b in zip(*grads):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("ctor", ["LogicNet", "LogicTreeNet"])
def test_torch_compile_traces_the_custom_ops(ctor):
    """The kernels are torch.library custom ops with fake implementations: torch.compile
    (AOT autograd, no code generation) traces forward + backward of a whole network and
    gives the eager results."""
    import silogic_b200 as S
    torch.manual_seed(0)
    if ctor == "LogicNet":
        m = S.LogicNet(64, 200, 2, node="walsh", connectome="topk", k=8, tau=10.0, seed=0)
        x = (torch.rand(50, 64) < 0.3).float()
    else:
        m = S.LogicTreeNet(in_channels=6, in_hw=8, channels=[16, 32], head_widths=[80],
                           tree_depth=2, node="gate16", tau=20.0, seed=0)
        x = (torch.rand(50, 6, 8, 8) < 0.5).float()
    m = m.to(dev).train()
    x = x.to(dev)
    eager_out = m(x)
    eager_out.sum().backward()
    ref = [p.grad.clone() for p in m.parameters()]
    m.zero_grad()
    cm = torch.compile(m, backend="aot_eager", fullgraph=True)
    out = cm(x)
    out.sum().backward()
    torch.testing.assert_close(out, eager_out, rtol=1e-6, atol=1e-6)
    for p, r in zip(m.parameters(), ref):
        torch.testing.assert_close(p.grad, r, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("ctor", ["LogicNet", "LogicTreeNet"])
def test_train_model_graphed_step_matches_eager(ctor):
    """train_model's CUDA-graphed step (fwd + bwd + Adam, cosine learning rate) trains like
    the eager step: the same data order gives parameters within rounding (gx atomics)
    after two epochs.  The graphed step with on-device augmentation (bit flips, cutout)
    runs as well."""
    import silogic_b200 as S
    from silogic_b200.train import train_model
    g = torch.Generator().manual_seed(0)
    if ctor == "LogicNet":
        X = (torch.rand(1024, 64, generator=g) < 0.5).to(torch.uint8)
        y = (X[:, :10].sum(1) > 5).long() * 3
        make = lambda: S.LogicNet(64, 200, 2, node="walsh", connectome="topk", k=4, tau=3.0, seed=0)
    else:
        X = (torch.rand(512, 6, 8, 8, generator=g) < 0.5).to(torch.uint8)
        y = (X[:, 0].sum((1, 2)) > 32).long() * 3
        make = lambda: S.LogicTreeNet(in_channels=6, in_hw=8, channels=[16, 32], head_widths=[80],
                                      tree_depth=2, node="gate16", tau=5.0, seed=0)
    params = []
    for graph in (True, False):
        torch.manual_seed(1)
        m = make()
        res = train_model(m, X, y, X, y, dev, epochs=2, bs=128, lr=0.05, val_every=100,
                          log=lambda *a: None, graph=graph, cosine=True)
        params.append([p.detach().clone() for p in m.parameters()])
        assert set(res) == {"test_soft", "test_hard", "train_min", "history"}
    for a, b in zip(*params):
        if ctor == "LogicNet":
            torch.testing.assert_close(a, b, rtol=1e-3, atol=1e-4)
        else:
            # conv gx atomics differ in order run to run, and Adam normalises each entry's
            # gradient, so entries whose gradient is ~0 may move apart: bound the aggregate
            d = (a - b).abs()
            assert d.mean() < 1e-4 and d.max() < 1e-2, (d.mean().item(), d.max().item())
    res = train_model(make(), X, y, X, y, dev, epochs=1, bs=128, val_every=1,
                      log=lambda *a: None, flip_p=0.05, cutout=3)
    assert 0.0 <= res["test_hard"] <= 100.0 and res["history"]["epoch"] == [1]


@pytest.mark.parametrize("B", [37, 300])
@pytest.mark.parametrize("k, sel", [(8, "softmax"), (5, "softmax"), (1, "softmax"), (8, "hard")])
def test_multilinear6_conv_backward_kernels_agree(B, k, sel):
    """One-level arity-6 multilinear conv trees: the factorised low-register backward
    (tuning key 5 = 1) and the generic tree backward (key 5 = 0) give the same input,
    connection and LUT gradients within the fp32 tolerance, for softmax and hard Top-K
    selection, K below the template width, and batches that end inside a warp round."""
    from silogic_b200 import _lib
    L = _lib.lib()
    kw = dict(in_channels=9, in_hw=12, channels=[16, 24], head_widths=[120, 60], tree_depth=1,
              node="multilinear", arity=6, k=k, n_chan=4, gate_select=sel, tau=12.0, seed=2)
    m = _rand_model("LogicConvNet", kw, 23).to(dev).train()
    g = torch.Generator().manual_seed(B + k)
    x = torch.rand(B, 9, 12, 12, generator=g)
    rmat = torch.randn(B, 10, generator=g).to(dev)
    grads = {}
    try:
        for key in (0, 1):
            assert L.slg_tuning_set(5, key) == 0
            m.zero_grad()
            xd = x.to(dev).requires_grad_(True)
            (m(xd) * rmat).sum().backward()
            grads[key] = {"x": xd.grad.detach().cpu().numpy()}
            grads[key].update({n: p.grad.detach().cpu().numpy() for n, p in m.named_parameters()
                               if p.grad is not None})
    finally:
        L.slg_tuning_set(5, 1)
    assert grads[0].keys() == grads[1].keys()
    for name in grads[0]:
        assert_grad_close(grads[1][name], grads[0][name], name)
