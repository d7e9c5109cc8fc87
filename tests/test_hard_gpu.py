"""Hard (bit-packed) circuit on the GPU vs the reference golden counts and the oracle."""
import numpy as np
import pytest
import torch

from helpers import FIXTURES, build_model, encoder_image, hard_input, load
from oracle import hard as OH
from oracle.spec import net_spec

pytestmark = pytest.mark.gpu
dev = "cuda"


@pytest.mark.parametrize("name", FIXTURES)
def test_forward_hard_matches_reference_golden(name):
    m, enc, z, _ = build_model(name, dev)
    x = torch.from_numpy(hard_input(z)).to(dev)
    if enc is not None:
        x = encoder_image(enc.forward_hard(x), z)
    got = m.forward_hard(x)
    np.testing.assert_array_equal(got.cpu().numpy(), z["hard"])


@pytest.mark.parametrize("name", FIXTURES)
def test_bitpacked_api_matches_reference_golden(name):
    from silogic_b200.bitpacking import convert_logic_net, convert_logic_conv_net
    m, enc, z, _ = build_model(name, dev)
    x = torch.from_numpy(hard_input(z)).to(dev)
    if enc is not None:
        x = encoder_image(enc.forward_hard(x), z)
    conv = "conv" in name
    bp = convert_logic_conv_net(m) if conv else convert_logic_net(m)
    logits = bp(x.to(torch.uint8).cpu().numpy())                # numpy in -> numpy out
    tau = m.head.tau
    np.testing.assert_array_equal(np.rint(logits * tau), z["hard"])


def _rand_fc(in_dim, width, depth, seed, **kw):
    import silogic_b200 as S
    torch.manual_seed(seed)
    m = S.LogicNet(in_dim, width, depth, seed=seed, **kw)
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for p in m.parameters():
            p.copy_(torch.randn(p.shape, generator=g))
    return m


@pytest.mark.parametrize("B", [1, 63, 64, 65, 127, 128, 129, 1000, 4097])
def test_fc_ragged_batches_vs_oracle(B):
    m = _rand_fc(100, 300, 3, 7, node="walsh", connectome="topk", k=8, tau=10.0)
    g = torch.Generator().manual_seed(B)
    x = (torch.rand(B, 100, generator=g) < 0.3).float()
    sd = {k: v.numpy() for k, v in m.state_dict().items()}
    ref = OH.model_counts("LogicNet", dict(in_dim=100, width=300, depth=3, node="walsh",
                                           connectome="topk", k=8, tau=10.0, seed=7), sd,
                          x.numpy().astype(np.uint8))
    got = m.to(dev).forward_hard(x.to(dev))
    np.testing.assert_array_equal(got.cpu().numpy(), ref)


@pytest.mark.parametrize("arity", [1, 2, 3, 4, 5, 6])
def test_fc_lut_arities_vs_oracle(arity):
    node = "multilinear" if arity > 1 else "linear"
    kw = dict(in_dim=64, width=200, depth=2, node=node, arity=arity, connectome="topk", k=3,
              tau=1.0, seed=arity)
    m = _rand_fc(64, 200, 2, arity, **{k: v for k, v in kw.items()
                                       if k not in ("in_dim", "width", "depth", "seed")})
    sd = {k: v.numpy() for k, v in m.state_dict().items()}
    x = (torch.rand(333, 64, generator=torch.Generator().manual_seed(1)) < 0.5).float()
    ref = OH.model_counts("LogicNet", kw, sd, x.numpy().astype(np.uint8))
    got = m.to(dev).forward_hard(x.to(dev))
    np.testing.assert_array_equal(got.cpu().numpy(), ref)


@pytest.mark.parametrize("depth,node,arity,connect", [
    (1, "gate16", 2, "topk"), (2, "gate16", 2, "fixed"), (3, "gate16", 2, "topk"),
    (4, "gate16", 2, "topk"), (1, "multilinear", 6, "topk"), (1, "hybrid", 4, "fixed"),
    (2, "multilinear", 3, "topk"), (2, "walsh", 2, "topk")])
def test_conv_trees_vs_oracle(depth, node, arity, connect):
    import silogic_b200 as S
    kw = dict(in_channels=6, in_hw=12, channels=[24, 40], head_widths=[120], tree_depth=depth,
              node=node, arity=arity, connect=connect, k=4, tau=3.0, seed=depth)
    torch.manual_seed(5)
    m = S.LogicConvNet(**kw)
    g = torch.Generator().manual_seed(9)
    with torch.no_grad():
        for p in m.parameters():
            p.copy_(torch.randn(p.shape, generator=g))
    sd = {k: v.numpy() for k, v in m.state_dict().items()}
    x = (torch.rand(150, 6, 12, 12, generator=g) < 0.5).float()
    ref = OH.model_counts("LogicConvNet", kw, sd, x.numpy().astype(np.uint8))
    got = m.to(dev).forward_hard(x.to(dev))
    np.testing.assert_array_equal(got.cpu().numpy(), ref)


def test_layer_level_forward_hard_vs_oracle():
    import silogic_b200 as S
    torch.manual_seed(3)
    conv = S.ConvLogicTree(4, 8, tree_depth=2, connect="topk", seed=3)
    with torch.no_grad():
        for p in conv.parameters():
            p.normal_()
    x = (torch.rand(70, 4, 7, 9) < 0.5).float()
    y = conv.to(dev).forward_hard(x.to(dev)).cpu().numpy()
    leaf, tts = conv.cpu().hard_spec()
    otts = [OH.node_truth_tables("gate16", p.detach().reshape(-1, 16).numpy(), 2).reshape(8, -1, 4)
            for p in conv.gate_logits]
    h = OH.pack_bits(x.numpy().reshape(70, -1)).reshape(4, 7, 9, -1)
    ref = OH.conv_forward(h, leaf.numpy().astype(np.int64), otts, 2, pool=1)
    ref = OH.unpack_bits(ref.reshape(-1, ref.shape[-1]), 70).reshape(70, 8, 7, 9)
    np.testing.assert_array_equal(y, ref)


def test_pack_unpack_and_thermometer_vs_golden():
    from silogic_b200 import _hard
    from silogic_b200.bitpacking import pack_bits, unpack_bits
    z = load("prims")
    for B, F in [(1, 1), (63, 8), (64, 64), (65, 256), (200, 784)]:
        x = z[f"pack_{B}_{F}/x"]
        p = pack_bits(x)
        np.testing.assert_array_equal(p, z[f"pack_{B}_{F}/packed"])
        np.testing.assert_array_equal(unpack_bits(p, B), x)
        xf = torch.from_numpy(x).float().cuda()
        np.testing.assert_array_equal(_hard.pack(xf)[:, :p.shape[1]].cpu().numpy(), p)
    import silogic_b200 as S
    bits = S.binarize_spatial(torch.from_numpy(z["thermo/img"]).cuda(), S.FIVE_THRESH)
    np.testing.assert_array_equal(bits.cpu().numpy(), z["thermo/bits"])


def test_groupsum_vs_golden():
    from silogic_b200 import _hard
    z = load("prims")
    x = torch.from_numpy(z["gsum/x"]).cuda()
    c = _hard.groupsum(_hard.pack(x), 130, 10)
    np.testing.assert_array_equal((c.float() / 4.0).cpu().numpy(), z["gsum/logits_tau4"])


def test_large_group_groupsum_vs_oracle():
    from silogic_b200 import _hard
    x = (torch.rand(1000, 20000) < 0.5)
    c = _hard.groupsum(_hard.pack(x.cuda()), 1000, 10).cpu().numpy()
    np.testing.assert_array_equal(c, x.view(1000, 10, 2000).sum(-1).numpy())


def test_learned_thermometer_hard_vs_oracle():
    import silogic_b200 as S
    enc = S.LearnedThermometerEncoder(50, 3)
    with torch.no_grad():
        enc.thresholds.copy_(torch.rand(50, 3))
    x = torch.rand(77, 50)
    got = enc.cuda().forward_hard(x.cuda()).cpu().numpy()
    ref = OH.learned_thermometer_bits(x.numpy(), enc.thresholds.detach().cpu().numpy())
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("B,W,C", [(1, 10, 10), (70, 40000, 2), (3000, 1280, 10), (1025, 60, 3)])
def test_groupsum_shapes_vs_oracle(B, W, C):
    from silogic_b200 import _hard
    x = torch.rand(B, W, generator=torch.Generator().manual_seed(B)) < 0.5
    c = _hard.groupsum(_hard.pack(x.cuda()), B, C).cpu().numpy()
    np.testing.assert_array_equal(c, OH.group_sum_counts(OH.pack_bits(x.numpy()), B, C))


@pytest.mark.parametrize("F", [1, 15, 16, 33, 784])
def test_pack_widths_u8_f32_vs_oracle(F):
    from silogic_b200 import _hard
    x = torch.rand(131, F, generator=torch.Generator().manual_seed(F)) < 0.4
    ref = OH.pack_bits(x.numpy())
    for t in (x.to(torch.uint8), x.float()):
        got = _hard.pack(t.cuda())[:, :ref.shape[1]].cpu().numpy().view(np.uint64)
        np.testing.assert_array_equal(got, ref)


def test_forward_images_fuses_thermometer_vs_oracle():
    """BitpackedConvNet.forward_images(img) == oracle counts of binarize_spatial(img)."""
    import silogic_b200 as S
    from silogic_b200.bitpacking import convert_logic_conv_net
    kw = dict(in_channels=15, in_hw=16, channels=[24, 40], head_widths=[160], tree_depth=2,
              node="gate16", tau=4.0, seed=3)
    torch.manual_seed(2)
    m = S.LogicTreeNet(**kw)
    with torch.no_grad():
        for p in m.parameters():
            p.normal_()
    img = torch.rand(200, 3, 16, 16, generator=torch.Generator().manual_seed(4))
    sd = {k: v.numpy() for k, v in m.state_dict().items()}
    th = [1 / 6, 2 / 6, 3 / 6, 4 / 6, 5 / 6]
    ref = OH.model_counts("LogicTreeNet", kw, sd, OH.thermometer_bits(img.numpy(), th))
    bp = convert_logic_conv_net(m.cuda())
    got = bp.forward_images(img.cuda(), th) * 4.0
    np.testing.assert_array_equal(np.rint(got.cpu().numpy()), ref)


@pytest.mark.parametrize("th", [[0.5], [1 / 6, 2 / 6, 3 / 6, 4 / 6, 5 / 6],
                                [(i + 1) / 32 for i in range(31)], [0.7, 0.2, 0.5],
                                [(i + 1) / 40 for i in range(39)], [0.3, 0.3, 0.6]])
def test_thermometer_pack_sorted_unsorted_and_long_vs_oracle(th):
    from silogic_b200 import _hard
    img = torch.rand(70, 3, 5, 7, generator=torch.Generator().manual_seed(len(th)))
    img[0, 0, 0, :len(th[:7])] = torch.tensor(th[:7])                  # exact threshold values
    h = _hard.thermo_pack(img.cuda(), th)
    got = _hard.unpack(h.view(-1, h.shape[-1]), 70).view(70, -1).cpu().numpy()
    ref = OH.thermometer_bits(img.numpy(), th).reshape(70, -1)
    np.testing.assert_array_equal(got, ref)
    h2 = _hard.thermo_pack(img.cuda(), torch.tensor(th).cuda())      # tensor thresholds path
    np.testing.assert_array_equal(h2.cpu().numpy(), h.cpu().numpy())


def test_cuda_graph_replay_matches_eager_and_oracle():
    """BitpackedNet replays a cached CUDA graph per batch shape; every input form
    (device, pinned host, numpy, a second batch through the same graph, ragged
    shapes that evict older graphs) gives the oracle's counts."""
    from silogic_b200.bitpacking import convert_logic_net
    kw = dict(node="walsh", connectome="topk", k=8, tau=10.0)
    m = _rand_fc(100, 300, 3, 11, **kw)
    sd = {k: v.numpy() for k, v in m.state_dict().items()}
    bp = convert_logic_net(m.to(dev))
    bp.max_graphs = 2
    for i, B in enumerate([129, 129, 64, 3000, 129]):
        x = (torch.rand(B, 100, generator=torch.Generator().manual_seed(i)) < 0.3).to(torch.uint8)
        ref = OH.model_counts("LogicNet", dict(in_dim=100, width=300, depth=3, seed=11, **kw), sd,
                              x.numpy())
        for xin in (x.cuda(), x.pin_memory(), x.numpy()):
            got = bp(xin)
            got = got if isinstance(got, np.ndarray) else got.cpu().numpy()
            np.testing.assert_array_equal(np.rint(got * 10.0), ref)
    assert len(bp._graphs) <= 2
    bp.graphs = False                                      # eager path, same answers
    np.testing.assert_array_equal(np.rint(bp(x.numpy()) * 10.0), ref)


def test_cuda_graph_thermometer_learned_and_shared():
    """forward_images through the graph cache: shared (mode 0) and learned per-feature
    (mode 1) thresholds, against the eager path."""
    import silogic_b200 as S
    from silogic_b200.bitpacking import convert_logic_conv_net
    kw = dict(in_channels=15, in_hw=8, channels=[16, 24], head_widths=[60], tree_depth=2,
              node="gate16", tau=4.0, seed=5)
    torch.manual_seed(3)
    m = S.LogicTreeNet(**kw)
    with torch.no_grad():
        for p in m.parameters():
            p.normal_()
    bp = convert_logic_conv_net(m.cuda())
    img = torch.rand(77, 3, 8, 8, generator=torch.Generator().manual_seed(6))
    th = [0.2, 0.4, 0.5, 0.6, 0.8]
    a = bp.forward_images(img.cuda(), th)
    bp.graphs = False
    b = bp.forward_images(img.cuda(), th)
    np.testing.assert_array_equal(a.cpu().numpy(), b.cpu().numpy())
    thr = torch.rand(3 * 8 * 8, 5, generator=torch.Generator().manual_seed(7)).cuda()
    b = bp.forward_images(img.cuda(), thr, mode=1)
    bp.graphs = True
    a = bp.forward_images(img.pin_memory(), thr, mode=1)
    np.testing.assert_array_equal(a.cpu().numpy(), b.cpu().numpy())


@pytest.mark.parametrize("B", [1, 64, 100, 1000, 4097, 20000])
@pytest.mark.parametrize("kw", [dict(node="walsh", connectome="topk", k=8, tau=10.0),
                                dict(node="gate16", connectome="fixed", tau=10.0),
                                dict(node="gate16", connectome="topk", k=4, tau=10.0,
                                     wire_residual=0.25),
                                dict(node="multilinear", connectome="topk", k=8, tau=10.0)])
def test_fc_chain_whole_stack_kernel_vs_oracle(B, kw):
    """The one-launch FC stack + GroupSum (slg_fc_chain_counts) == oracle counts."""
    m = _rand_fc(100, 300, 3, 13, **kw)
    g = torch.Generator().manual_seed(B)
    x = (torch.rand(B, 100, generator=g) < 0.3).to(torch.uint8)
    sd = {k: v.numpy() for k, v in m.state_dict().items()}
    ref = OH.model_counts("LogicNet", dict(in_dim=100, width=300, depth=3, seed=13, **kw), sd,
                          x.numpy())
    from silogic_b200.bitpacking.plan import HardPlan
    plan = HardPlan.from_model(m.to(dev))
    assert plan.chain() is not None
    plan.chain_min_batch = 0
    got = plan.counts(x.cuda()).cpu().numpy()
    np.testing.assert_array_equal(got, ref)
    plan.use_chain = False
    np.testing.assert_array_equal(plan.counts(x.cuda()).cpu().numpy(), ref)


def test_fc_chain_large_group_and_unsupported_plans():
    """Wide last layer (group of 1300 rows per class) and the plans the chain declines."""
    m = _rand_fc(50, 2600, 2, 17, node="walsh", connectome="topk", k=8, tau=10.0)
    from silogic_b200.bitpacking.plan import HardPlan
    plan = HardPlan.from_model(m.to(dev))
    x = (torch.rand(777, 50, generator=torch.Generator().manual_seed(3)) < 0.5).to(torch.uint8)
    plan.chain_min_batch = 0
    a = plan.counts(x.cuda()).cpu().numpy()
    plan.use_chain = False
    np.testing.assert_array_equal(a, plan.counts(x.cuda()).cpu().numpy())
    m3 = _rand_fc(50, 120, 2, 5, node="walsh", arity=3, connectome="fixed", tau=10.0)
    assert HardPlan.from_model(m3.to(dev)).chain() is None


def test_pipelined_host_batches_match_one_shot():
    """Host batches split into double-buffered, copy-overlapped slices give the same
    logits as one graph over the whole batch (ragged last slice included)."""
    from silogic_b200.bitpacking import convert_logic_net
    m = _rand_fc(100, 300, 3, 21, node="walsh", connectome="topk", k=8, tau=10.0)
    bp = convert_logic_net(m.to(dev))
    x = (torch.rand(5000, 100, generator=torch.Generator().manual_seed(9)) < 0.3).to(torch.uint8)
    ref = bp(x.cuda()).cpu().numpy()
    bp.pipeline_bytes = 100 * 1024            # 1024-sample slices of 100 features
    bp.min_slice_samples = 1024
    for xin in (x.pin_memory(), x, x.numpy()):
        got = bp(xin)
        got = got if isinstance(got, np.ndarray) else got.cpu().numpy()
        np.testing.assert_array_equal(got, ref)


def test_chain_encode_records_on_device():
    """slg_fc_chain_encode packs (in_a, in_b, table) records, residual wires included."""
    from silogic_b200 import _hard
    g = torch.Generator().manual_seed(4)
    idx = torch.randint(0, 9000, (5000, 2), generator=g, dtype=torch.int32)
    tt = torch.randint(0, 16, (5000,), generator=g, dtype=torch.int64)
    rec = _hard.chain_encode(idx.cuda(), tt.cuda(), wire_r=100).cpu().numpy().view(np.uint32)
    i, t = idx.numpy().astype(np.uint32), tt.numpy().astype(np.uint32)
    ref = i[:, 0] | (i[:, 1] << 14) | (t << 28)
    o = np.arange(100, dtype=np.uint32)
    ref[:100] = o | (o << 14) | np.uint32(0xA << 28)
    np.testing.assert_array_equal(rec, ref)


@pytest.mark.parametrize("decoder", ["linear", "linfull", "ternary"])
def test_learned_decoder_bitpacked_head(decoder):
    """BitpackedNet with a learned readout: the packed-feature linear head equals the
    model's own forward_hard (unpacked bits @ W.T + b); ternary weights are exact."""
    import silogic_b200 as S
    from silogic_b200.bitpacking import convert_logic_net
    torch.manual_seed(4)
    m = S.LogicNet(100, 320, 2, node="walsh", connectome="topk", k=8, decoder=decoder, seed=4)
    with torch.no_grad():
        for p in m.parameters():
            p.normal_()
    m = m.to(dev)
    x = (torch.rand(333, 100, generator=torch.Generator().manual_seed(8)) < 0.3).to(torch.uint8)
    ref = m.forward_hard(x.to(dev).float()).cpu().numpy()
    bp = convert_logic_net(m)
    for graphs in (True, False):
        bp.graphs = graphs
        got = bp(x.numpy())
        if decoder == "ternary":
            np.testing.assert_array_equal(got, ref)
        else:
            np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-4)


def test_device_index_check_names_the_first_bad_entry():
    """slg_check_index_range on device wiring: in-range passes, one bad entry is refused
    with its position and value, and a circuit built from it never launches."""
    from silogic_b200 import _hard
    idx = torch.randint(0, 100, (5000, 2), dtype=torch.int32, device=dev)
    _hard.check_index_range(idx, 100, "wiring")
    bad = idx.clone()
    bad[1234, 1] = 100
    bad[4000, 0] = -3
    with pytest.raises(IndexError, match=r"2 of 10000 entries outside \[0, 100\), first at "
                                         r"position 2469 \(value 100\)"):
        _hard.check_index_range(bad, 100, "wiring")
    from silogic_b200.bitpacking.packed import PackedFCLayer
    layer = PackedFCLayer(idx, torch.zeros(5000, dtype=torch.int64, device=dev))
    x = torch.zeros(50, 2, dtype=torch.int64, device=dev)            # only 50 input rows
    with pytest.raises(IndexError, match="reads input row"):
        layer(x)


@pytest.mark.parametrize("thr", [
    [(i + 1) / 32 for i in range(31)],                       # C5's grid
    [1 / 6, 2 / 6, 3 / 6, 4 / 6, 5 / 6],                      # C3's grid
    [0.1 + 0.03 * i + (0.007 if i % 3 == 0 else -0.006) for i in range(20)],   # near uniform
    [0.01, 0.02, 0.5, 0.51, 0.9],                             # far from uniform: searched
    [0.3],                                                    # one threshold
], ids=["grid31", "grid5", "perturbed20", "nonuniform5", "single"])
def test_thermometer_pack_exact_at_threshold_boundaries(thr):
    """binarize_spatial bits (x >= f32(t)) for values exactly at each threshold, one ulp
    either side, +-inf and NaN, against the oracle: the sorted-threshold count (grid
    guess corrected by two comparisons, or a binary search) must be exact."""
    from silogic_b200 import _hard
    t32 = np.asarray(thr, np.float32)
    specials = np.concatenate([t32, np.nextafter(t32, -np.inf), np.nextafter(t32, np.inf),
                               np.float32([np.inf, -np.inf, np.nan, 0.0, -0.0, 1.0, 2.0, -1.0])])
    g = np.random.default_rng(len(thr))
    B = 700
    img = g.random((B, 3, 8, 8), dtype=np.float32)
    flat = img.reshape(-1)
    pick = g.choice(flat.size, size=flat.size // 3, replace=False)
    flat[pick] = g.choice(specials, size=pick.size)
    ref = OH.pack_bits(OH.thermometer_bits(img, thr).reshape(B, -1))
    got = _hard.thermo_pack(torch.from_numpy(img).to(dev), list(thr))
    got = got.reshape(got.shape[0] * got.shape[1] * got.shape[2], -1)
    np.testing.assert_array_equal(got[:, :ref.shape[1]].cpu().numpy().view(np.uint64), ref)
    assert not got[:, ref.shape[1]:].any(), "padding words must be zero"


# (key 0 gate dispatch, key 4 staged window: 1 below its size cut-over, 2 always, key 3
# node form): every conv path for arity-2 trees, the first entry being the default
CONV_PATHS = [(1, 1, 0), (1, 2, 0), (1, 2, 1), (1, 0, 0), (1, 0, 1), (1, 0, 2), (0, 0, 0)]


@pytest.mark.parametrize("B", [100, 4096])
def test_conv_gate_dispatch_kernel_equals_generic_tree_kernel(B):
    """The arity-2 conv kernels -- the staged shared-memory window, the gate-dispatch
    kernel with each node form, and the generic LUT-tree kernel -- give the same bits
    (depths 1-3, pool 1 and 2, pad 0 and 1, wire residual, image sizes down to 2x2,
    odd sizes, near the staged kernel's shared-memory limit and past it)."""
    from silogic_b200 import _hard, _lib
    L = _lib.lib()
    g = torch.Generator().manual_seed(B)
    cases = [(1, 2, 5, 9, 7, 0, 1), (2, 2, 15, 32, 40, 0, 1), (3, 1, 4, 6, 9, 0, 1),
             (2, 2, 16, 4, 24, 8, 1), (2, 2, 8, 2, 300, 0, 1), (2, 2, 6, 11, 33, 0, 0),
             (3, 2, 7, 13, 20, 3, 1), (2, 2, 118, 10, 70, 0, 1), (2, 2, 134, 6, 30, 0, 1),
             (2, 2, 9, 19, 17, 2, 0)]
    for depth, pool, C, H, n, wr, pad in cases:
        ldw = _hard.ldw_for(B)
        x = torch.randint(-2**62, 2**62, (C, H, H, ldw), generator=g).to(dev)
        leaves = 2 ** depth
        leaf = torch.randint(0, C * 9, (n, leaves), generator=g, dtype=torch.int32).to(dev)
        tt = torch.randint(0, 16, (n, leaves - 1), generator=g).to(dev)
        outs = []
        for k0, k4, k3 in CONV_PATHS:
            assert L.slg_tuning_set(0, k0) == 0 and L.slg_tuning_set(4, k4) == 0
            assert L.slg_tuning_set(3, k3) == 0
            try:
                outs.append(_hard.conv(x, leaf, tt, 2, depth, 3, pad, wr, pool))
            finally:
                for key, val in ((0, 1), (4, 1), (3, 0)):
                    L.slg_tuning_set(key, val)
        for (k0, k4, k3), o in zip(CONV_PATHS[1:], outs[1:]):
            assert torch.equal(outs[0], o), (depth, pool, C, H, n, wr, pad, k0, k4, k3)


def test_loaded_packed_artefact_gives_the_same_counts(tmp_path):
    import silogic_b200 as S
    from silogic_b200.bitpacking import convert_logic_conv_net, save_packed, load_packed
    torch.manual_seed(0)
    m = S.LogicTreeNet(in_channels=6, in_hw=8, channels=[16, 32], head_widths=[80], tree_depth=2,
                       node="gate16", tau=5.0, seed=0).to(dev)
    bp = convert_logic_conv_net(m)
    save_packed(bp, tmp_path / "net.npz")
    back = load_packed(tmp_path / "net.npz", device=dev)
    x = (np.random.default_rng(0).random((300, 6, 8, 8)) < 0.5).astype(np.uint8)
    np.testing.assert_array_equal(back(x), bp(x))


@pytest.mark.parametrize("th", [[0.5], [1 / 6, 2 / 6, 3 / 6, 4 / 6, 5 / 6],
                                [(i + 1) / 32 for i in range(31)], [0.7, 0.2, 0.5],
                                [(i + 1) / 40 for i in range(39)],
                                [k / 255 for k in (0, 1, 2, 127, 128, 254, 255)]])
@pytest.mark.parametrize("shape", [(70, 3, 5, 7), (1100, 3, 32, 32), (65, 1, 4, 4)])
def test_thermometer_pack_uint8_equals_float_quotient(th, shape):
    """uint8 pixels k packed like the fp32 image k / 255 (torchvision ToTensor), for shared
    sorted / unsorted / long threshold lists, thresholds exactly on k / 255, every pixel
    value, vector and scalar load paths (3072 and 35 features), and learned per-feature
    thresholds; checked against the oracle on the float image."""
    from silogic_b200 import _hard
    g = torch.Generator().manual_seed(len(th) + shape[0])
    u8 = torch.randint(0, 256, shape, generator=g, dtype=torch.uint8)
    u8.view(-1)[:256] = torch.arange(256, dtype=torch.uint8)      # every value appears
    f32 = u8.float() / 255
    ref = OH.pack_bits(OH.thermometer_bits(u8.numpy().astype(np.float32) / np.float32(255), th)
                       .reshape(shape[0], -1))
    for mode_thr in (th, torch.tensor(th)):                      # sorted-list and tensor paths
        got = _hard.thermo_pack(u8.to(dev), mode_thr)
        assert torch.equal(got, _hard.thermo_pack(f32.to(dev), mode_thr))
        got = got.reshape(-1, got.shape[-1])
        np.testing.assert_array_equal(got[:, :ref.shape[1]].cpu().numpy().view(np.uint64), ref)
    F = shape[1] * shape[2] * shape[3]
    learned = torch.rand(F, len(th), generator=g)
    assert torch.equal(_hard.thermo_pack(u8.to(dev), learned.to(dev), mode=1),
                       _hard.thermo_pack(f32.to(dev), learned.to(dev), mode=1))


def test_forward_images_uint8_host_batch_equals_float():
    """BitpackedConvNet.forward_images on a pinned uint8 host batch (pipelined copies)
    gives the logits of the same images as fp32 k / 255."""
    import silogic_b200 as S
    from silogic_b200.bitpacking import convert_logic_conv_net
    kw = dict(in_channels=15, in_hw=16, channels=[24, 40], head_widths=[160], tree_depth=2,
              node="gate16", tau=4.0, seed=3)
    torch.manual_seed(5)
    m = S.LogicTreeNet(**kw)
    with torch.no_grad():
        for p in m.parameters():
            p.normal_()
    bp = convert_logic_conv_net(m.cuda())
    u8 = torch.randint(0, 256, (5000, 3, 16, 16), generator=torch.Generator().manual_seed(6),
                       dtype=torch.uint8).pin_memory()
    th = [1 / 6, 2 / 6, 3 / 6, 4 / 6, 5 / 6]
    old = bp.pipeline_bytes
    bp.pipeline_bytes = 1 << 20           # several pipelined slices
    bp.min_slice_samples = 1024
    try:
        got = bp.forward_images(u8, th)
    finally:
        bp.pipeline_bytes = old
    ref = bp.forward_images((u8.float() / 255).cuda(), th)
    assert torch.equal(got.cpu(), ref.cpu())



@pytest.mark.parametrize("B, ldw", [(1000, None), (777, 13), (4160, 70), (300, 9), (64, 1)])
@pytest.mark.parametrize("T", [1, 5, 31, 39])
def test_thermometer_pack_any_row_length_vs_oracle(B, ldw, T):
    """Caller-chosen row lengths: odd ldw (rows not 16-byte aligned, so 8-byte stores),
    rows padded past the batch (zero words) and a ragged batch, for sorted threshold
    lists of one, a few, 31 and more than one 32-threshold chunk."""
    from silogic_b200 import _hard
    g = torch.Generator().manual_seed(B + T)
    u8 = torch.randint(0, 256, (B, 3, 8, 16), generator=g, dtype=torch.uint8)
    u8.view(-1)[:256] = torch.arange(256, dtype=torch.uint8)
    th = sorted(torch.rand(T, generator=g).tolist())
    got = _hard.thermo_pack(u8.to(dev), th, ldw=ldw)
    ref = OH.pack_bits(OH.thermometer_bits(u8.numpy().astype(np.float32) / np.float32(255), th)
                       .reshape(B, -1))
    w = got.reshape(-1, got.shape[-1]).cpu().numpy().view(np.uint64)
    assert w.shape[1] >= ref.shape[1]
    np.testing.assert_array_equal(w[:, :ref.shape[1]], ref)
    assert not w[:, ref.shape[1]:].any()
