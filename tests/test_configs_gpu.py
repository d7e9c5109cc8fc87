"""Parity at the benchmark's own configurations (C1-C5, the shapes bench.py times).

Each network is built exactly as bench.py builds it (seeded N(0,1) parameters), run
on the GPU through the public API, and compared with the CPU oracle:
  * hard counts bit-exactly (the reference's ``forward_hard`` semantics,
    ``silogic/models.py:100``, ``silogic/heads.py:42-45``), at the config's batch or on
    slices of it where the oracle would take minutes;
  * soft features / logits / gradients within 1e-5 (fp32), on small batches.
"""
import numpy as np
import pytest
import torch

import bench
from oracle import hard as OH
from oracle.spec import net_spec

pytestmark = pytest.mark.gpu
dev = "cuda"


def _oracle_counts(cfg, model, enc, x):
    """Oracle counts for a host batch of the config's raw input (uint8 pixels are the
    fp32 images k / 255)."""
    sd = {k: v.detach().cpu().numpy() for k, v in model.state_dict().items()}
    spec = net_spec(cfg["ctor"], cfg["kwargs"], sd)
    n = x.shape[0]
    xn = x.numpy() if cfg["inp"] == "bern" else bench.image_float(x).numpy()
    if cfg["inp"] == "image":
        xn = OH.thermometer_bits(xn, cfg["thresholds"])
    elif cfg["inp"] == "encoder":
        e = OH.learned_thermometer_bits(xn.reshape(n, -1), enc.thresholds.detach().cpu().numpy())
        xn = e.reshape(n, 3, 32, 32, cfg["bits"]).transpose(0, 1, 4, 2, 3).reshape(n, -1, 32, 32)
    return OH.net_counts(spec, xn)


def _bp(cfg, model):
    from silogic_b200.bitpacking import convert_logic_net, convert_logic_conv_net
    return convert_logic_net(model) if cfg["ctor"] == "LogicNet" else convert_logic_conv_net(model)


def _bp_counts(cfg, bp, enc, x):
    """Counts through the bit-packed API: uint8 features, or uint8 images with the
    thermometer fused into packing (shared or learned thresholds)."""
    tau = cfg["kwargs"]["tau"]
    if cfg["inp"] == "bern":
        logits = bp(x.numpy())
    elif cfg["inp"] == "image":
        logits = bp.forward_images(x, cfg["thresholds"])
    else:
        logits = bp.forward_images(x, enc.thresholds.detach().to(dev).contiguous(), mode=1)
    logits = logits.cpu().numpy() if torch.is_tensor(logits) else logits
    return np.rint(np.asarray(logits, np.float64) * tau).astype(np.int64)


def test_c1_full_batch_vs_oracle():
    cfg = bench.CONFIGS["c1"]
    m, _ = bench.build_model(cfg)
    x = bench.make_input(cfg, cfg["hard_batch"], seed=1)
    ref = _oracle_counts(cfg, m, None, x)
    m = m.to(dev)
    got = m.forward_hard(x.to(dev).float()).cpu().numpy()
    np.testing.assert_array_equal(got, ref)
    np.testing.assert_array_equal(_bp_counts(cfg, _bp(cfg, m), None, x), ref)


@pytest.mark.parametrize("B", [4160, 65536])
def test_c2_fused_stack_full_width_vs_oracle(B):
    """784 -> 10000 x 6 Walsh through BitpackedNet: the fused whole-stack kernel with
    the planner's node reordering and class-block padding, at a batch that is not a
    multiple of 64 and at the benchmark's 65,536.  The oracle checks a 4,160-sample
    slice; at 65,536 the whole batch must also equal the per-layer kernels."""
    cfg = bench.CONFIGS["c2"]
    m, _ = bench.build_model(cfg)
    x = bench.make_input(cfg, B, seed=1)
    m = m.to(dev)
    bp = _bp(cfg, m)
    assert bp.plan.chain() is not None, "C2 must run on the fused FC stack"
    got = _bp_counts(cfg, bp, None, x)
    n = min(B, 4160)
    ref = _oracle_counts(cfg, m.cpu(), None, x[:n])
    np.testing.assert_array_equal(got[:n], ref)
    if B > n:
        per_layer = bp.plan
        per_layer.use_chain = False
        try:
            h = per_layer.counts(x.to(dev))
        finally:
            per_layer.use_chain = True
        np.testing.assert_array_equal(got, h.cpu().numpy())


def test_c3_full_batch_vs_oracle():
    cfg = bench.CONFIGS["c3"]
    m, _ = bench.build_model(cfg)
    x = bench.make_input(cfg, cfg["hard_batch"], seed=1)
    ref = _oracle_counts(cfg, m, None, x)
    m = m.to(dev)
    np.testing.assert_array_equal(_bp_counts(cfg, _bp(cfg, m), None, x), ref)
    import silogic_b200 as S
    xb = S.binarize_spatial(bench.image_float(x).to(dev), cfg["thresholds"])
    np.testing.assert_array_equal(m.forward_hard(xb).cpu().numpy(), ref)


def test_c4_encoder_lut6_vs_oracle():
    """Learned thermometer + arity-6 LUT trees + 16000-wide head at the full 8,192
    batch on the GPU; the oracle checks the first 512 and the last 64 samples."""
    cfg = bench.CONFIGS["c4"]
    m, enc = bench.build_model(cfg)
    with torch.no_grad():   # spread the thresholds so every bit plane carries information
        enc.thresholds.copy_(torch.rand(enc.thresholds.shape,
                                        generator=torch.Generator().manual_seed(3)))
    B = cfg["hard_batch"]
    x = bench.make_input(cfg, B, seed=1)
    m, enc = m.to(dev), enc.to(dev)
    got = _bp_counts(cfg, _bp(cfg, m), enc, x)
    mc, ec = m.cpu(), enc.cpu()
    np.testing.assert_array_equal(got[:512], _oracle_counts(cfg, mc, ec, x[:512]))
    np.testing.assert_array_equal(got[-64:], _oracle_counts(cfg, mc, ec, x[-64:]))


@pytest.fixture(scope="module")
def c5():
    cfg = bench.CONFIGS["c5"]
    m, _ = bench.build_model(cfg)
    return cfg, m


def test_c5_full_net_across_slice_boundaries_vs_oracle(c5):
    """The full C5 network (93 -> 1024 ... 8192 channels + 3-layer head) on 2,112
    samples fed from host memory in 1,024-sample pipelined slices (so samples cross
    two slice boundaries); the oracle checks samples on both sides of each."""
    cfg, m = c5
    B = 2112
    x = bench.make_input(cfg, B, seed=1)
    bp = _bp(cfg, m.to(dev))
    bp.pipeline_bytes = 1024 * 3 * 32 * 32              # 1,024-sample slices of uint8 pixels
    bp.min_slice_samples = 1024
    got = _bp_counts(cfg, bp, None, x)
    mc = m.cpu()
    for lo, hi in ((0, 96), (1000, 1056), (2040, 2112)):
        np.testing.assert_array_equal(got[lo:hi], _oracle_counts(cfg, mc, None, x[lo:hi]),
                                      err_msg=f"samples {lo}:{hi}")


def test_c5_device_chunk_of_the_benchmark_vs_oracle(c5):
    """One 131,072-sample device chunk (the benchmark's) through the captured graph;
    the oracle checks the first 128 and the last 64 samples."""
    from silogic_b200.bitpacking.plan import HardPlan, HardGraph
    cfg, m = c5
    B = cfg["chunk"]
    x = bench.make_input(cfg, B, seed=1)
    plan = HardPlan.from_model(m.to(dev))
    g = HardGraph(plan, x.to(dev), list(cfg["thresholds"]), 0)
    got = g.replay().cpu().numpy().astype(np.int64)
    mc = m.cpu()
    np.testing.assert_array_equal(got[:128], _oracle_counts(cfg, mc, None, x[:128]))
    np.testing.assert_array_equal(got[-64:], _oracle_counts(cfg, mc, None, x[-64:]))
    del g
    torch.cuda.empty_cache()


# ------------------------------------------------------------------ soft
def _soft_case(key, B):
    """Model and (host) model input of a config, for soft checks."""
    cfg = bench.CONFIGS[key]
    m, enc = bench.build_model(cfg)
    x = bench.make_input(cfg, B, seed=7)
    if cfg["inp"] == "bern":
        x = x.float()
    elif cfg["inp"] == "image":
        x = torch.from_numpy(OH.thermometer_bits(bench.image_float(x).numpy(), cfg["thresholds"])).float()
    else:
        x = bench.image_float(x)
    return cfg, m, enc, x


@pytest.mark.parametrize("key,B", [("c1", 256), ("c2", 64)])
def test_fc_configs_soft_vs_oracle(key, B):
    from test_soft_gpu import assert_grad_close, assert_logits_close, oracle_soft
    cfg, m, _, x = _soft_case(key, B)
    rmat = torch.randn(B, 10, generator=torch.Generator().manual_seed(9))
    f_ref, l_ref, P, gx_ref = oracle_soft(cfg["ctor"], cfg["kwargs"], m, x, rmat)
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


@pytest.mark.parametrize("key,B", [("c3", 16), ("c4", 2)])
def test_conv_configs_soft_vs_oracle(key, B):
    """C3 / C4 networks at full width on small batches.  Inputs are binary
    (thermometer bits), so OR-pool windows tie; the oracle replays this package's
    first-max routing for the gradients (forward values are compared strictly)."""
    from oracle import soft as OS
    from test_soft_gpu import assert_grad_close, assert_logits_close, our_pool_routing
    cfg, m, enc, x = _soft_case(key, B)
    rmat = torch.randn(B, 10, generator=torch.Generator().manual_seed(9))
    md = m.to(dev).train()
    if enc is not None:
        with torch.no_grad():
            enc.thresholds.copy_(torch.rand(enc.thresholds.shape,
                                            generator=torch.Generator().manual_seed(3)))
        encd = enc.to(dev)
        xr = x.reshape(B, -1).to(dev).requires_grad_(True)
        xi = encd(xr).view(B, 3, 32, 32, cfg["bits"]).permute(0, 1, 4, 2, 3).reshape(B, -1, 32, 32)
    else:
        xr = x.to(dev).requires_grad_(True)
        xi = xr
    routing = our_pool_routing(md, xi.detach())
    feat = md._run(xi, hard=False)
    logits = md(xi)
    (logits * rmat.to(dev)).sum().backward()
    # oracle on the CPU
    sd = {k: v.detach().cpu() for k, v in md.state_dict().items()}
    spec = net_spec(cfg["ctor"], cfg["kwargs"], {k: v.numpy() for k, v in sd.items()})
    P = OS.params_from_sd(sd)
    xc = x.reshape(B, -1).clone().requires_grad_(True) if enc is not None else \
        x.clone().requires_grad_(True)
    thr = None
    if enc is not None:
        thr = enc.thresholds.detach().cpu().clone().requires_grad_(True)
        xo = OS.learned_thermometer(xc, thr).view(B, 3, 32, 32, cfg["bits"]).permute(
            0, 1, 4, 2, 3).reshape(B, -1, 32, 32)
    else:
        xo = xc
    f_ref = OS.net_features(spec, P, xo, training=True, pool_index=routing)
    l_ref = OS.group_sum(f_ref, spec["num_classes"], spec["tau"])
    (l_ref * rmat).sum().backward()
    f_ref = f_ref.detach().numpy()
    np.testing.assert_allclose(feat.detach().cpu().numpy(), f_ref, rtol=1e-5, atol=1e-6)
    assert_logits_close(logits.detach().cpu().numpy(), l_ref.detach().numpy(), f_ref, md.head.tau)
    assert_grad_close(xr.grad, xc.grad.numpy(), "x")
    for n, p in md.named_parameters():
        assert_grad_close(p.grad, P[n].grad.numpy(), n)
    if enc is not None:
        assert_grad_close(encd.thresholds.grad, thr.grad.numpy(), "encoder thresholds")
