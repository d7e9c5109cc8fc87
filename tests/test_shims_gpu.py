"""The reference-signature bit-packed layer objects and GPU helpers
(``silogic/bitpacking/kernels/triton_layer.py:108-185``,
``triton_conv_layer.py:123-278``, ``packed_model.py:287-382``) and the benchmark API
(``bitpacking/benchmark.py``), against the numpy oracle."""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import hard as OH

pytestmark = pytest.mark.gpu
dev = "cuda"


def _gate_ref(xp, gates, a, b, B):
    """Gate g of each output at address (a << 1) | b (gate16 order, functional.py:50-69)."""
    bits = OH.unpack_bits(xp, B)                                   # [B, in]
    av, bv = bits[:, a].astype(np.int64), bits[:, b].astype(np.int64)
    out = OH.GATE_TT[gates][np.arange(len(gates))[None, :], (av << 1) | bv]
    return OH.pack_bits(out)


@pytest.mark.parametrize("B", [1, 64, 200, 4097])
def test_bitpacked_gpu_layer_from_gate_codes(B):
    from silogic_b200.bitpacking import BitpackedGPULayer
    g = np.random.default_rng(B)
    IN, OUT = 77, 300
    gates = g.integers(0, 16, OUT).astype(np.int32)
    a, b = g.integers(0, IN, OUT).astype(np.int32), g.integers(0, IN, OUT).astype(np.int32)
    xp = OH.pack_bits(g.integers(0, 2, (B, IN)))
    ref = _gate_ref(xp, gates, a, b, B)
    layer = BitpackedGPULayer(gates, a, b, device=dev)
    got = layer.forward(torch.from_numpy(xp.view(np.int64)).to(dev))  # [in, nw] int64 CUDA
    assert got.is_cuda and got.dtype == torch.int64 and tuple(got.shape) == ref.shape
    # padding samples of the last word are unspecified (a NOT gate sets them), as in the
    # reference, which masks them only before the head (ops.py:107-115)
    mask = lambda p: OH.mask_last_word(np.array(p, dtype=np.uint64), B)
    np.testing.assert_array_equal(mask(got.cpu().numpy().view(np.uint64)), ref)
    # numpy in -> numpy out, and from a reference-style converted layer
    again = BitpackedGPULayer.from_fc_layer(SimpleNamespace(gate_types=gates, a_idx=a, b_idx=b), dev)
    np.testing.assert_array_equal(mask(again.forward(xp.view(np.int64)).view(np.uint64)), ref)


def test_from_fc_layer_of_converted_model_matches_forward_hard():
    import silogic_b200 as S
    from silogic_b200.bitpacking import BitpackedGPULayer, convert_layer
    torch.manual_seed(0)
    layer = S.LogicLayer(64, 150, node="walsh", connectome="topk", k=4, seed=1).to(dev)
    with torch.no_grad():
        layer.node.theta.normal_()
    x = (torch.rand(300, 64, device=dev) < 0.5).float()
    gl = BitpackedGPULayer.from_fc_layer(convert_layer(layer), dev)
    packed = S.bitpacking.pack_bits(x.to(torch.uint8))
    out = S.bitpacking.unpack_bits(gl.forward(packed), 300)
    np.testing.assert_array_equal(out.cpu().numpy(), layer.forward_hard(x).cpu().numpy())


def _unfold_ref(x3, kh, pad, H, W):
    C, L, nw = x3.shape
    x4 = np.zeros((C, H + 2 * pad, W + 2 * pad, nw), np.uint64)
    x4[:, pad:pad + H, pad:pad + W] = x3.reshape(C, H, W, nw)
    Ho, Wo = H + 2 * pad - kh + 1, W + 2 * pad - kh + 1
    out = np.zeros((C * kh * kh, Ho * Wo, nw), np.uint64)
    for c in range(C):
        for dy in range(kh):
            for dx in range(kh):
                out[c * kh * kh + dy * kh + dx] = x4[c, dy:dy + Ho, dx:dx + Wo].reshape(-1, nw)
    return out


def test_packed_unfold_and_or_pool_gpu():
    from silogic_b200.bitpacking import packed_unfold_gpu, packed_or_pool_gpu
    g = np.random.default_rng(1)
    C, H, W, nw = 5, 7, 6, 3
    x3 = g.integers(0, 2**63, (C, H * W, nw), dtype=np.uint64)
    got = packed_unfold_gpu(torch.from_numpy(x3.view(np.int64)).to(dev), 3, 3, 1, 1, H, W)
    np.testing.assert_array_equal(got.cpu().numpy().view(np.uint64), _unfold_ref(x3, 3, 1, H, W))
    pooled = packed_or_pool_gpu(torch.from_numpy(x3.view(np.int64)).to(dev), H, W, 2)
    x4 = x3.reshape(C, H, W, nw)[:, :6, :6]
    ref = (x4[:, 0::2, 0::2] | x4[:, 0::2, 1::2] | x4[:, 1::2, 0::2] | x4[:, 1::2, 1::2])
    np.testing.assert_array_equal(pooled.cpu().numpy().view(np.uint64), ref.reshape(C, 9, nw))


@pytest.mark.parametrize("depth", [1, 2, 3])
def test_conv_gpu_layer_forward_packed_on_unfolded_input(depth):
    """BitpackedConvGPULayer.from_cpu_layer + forward_packed on an unfolded [P, L, nw]
    input (the reference's GPU conv path) equals the oracle's conv tree (no pool)."""
    from silogic_b200.bitpacking import BitpackedConvGPULayer, packed_unfold_gpu
    from silogic_b200.bitpacking.convert import convert_conv_tree_layer
    import silogic_b200 as S
    torch.manual_seed(depth)
    conv = S.ConvLogicTree(4, 9, tree_depth=depth, connect="topk", k=4, seed=depth).to(dev)
    with torch.no_grad():
        for p in conv.parameters():
            p.normal_()
    cpu_layer = convert_conv_tree_layer(conv)
    gl = BitpackedConvGPULayer.from_cpu_layer(cpu_layer, dev)
    g = np.random.default_rng(depth)
    B, H, W = 150, 6, 5
    bits = g.integers(0, 2, (B, 4, H, W))
    x3 = OH.pack_bits(bits.reshape(B, -1)).reshape(4, H * W, -1)
    unf = packed_unfold_gpu(torch.from_numpy(x3.view(np.int64)).to(dev), 3, 3, 1, 1, H, W)
    got = gl.forward_packed(unf).cpu().numpy().view(np.uint64)      # [n, L, nw]
    leaf = cpu_layer.leaf.cpu().numpy().astype(np.int64)
    tt = cpu_layer.tt.cpu().numpy().astype(np.int64).view(np.uint64)
    P = 4
    tts, base = [], 0
    for lev in range(depth):
        m = 2 ** (depth - 1 - lev)
        codes = tt[:, base:base + m]
        tts.append(((codes[..., None] >> np.arange(P, dtype=np.uint64)) & np.uint64(1)).astype(bool))
        base += m
    ref = OH.conv_forward(x3.reshape(4, H, W, -1), leaf, tts, 2, kernel=3, pad=1, pool=1)
    np.testing.assert_array_equal(got, ref.reshape(9, H * W, -1))


def test_benchmark_api_runs_and_reports(capsys):
    import silogic_b200 as S
    from silogic_b200.bitpacking import run_benchmark, run_conv_benchmark, print_report, speedup_summary
    torch.manual_seed(0)
    net = S.LogicNet(64, 200, 2, node="gate16", connectome="topk", k=4, tau=4.0, seed=0)
    x = (np.random.default_rng(0).random((500, 64)) < 0.4).astype(np.uint8)
    y = np.random.default_rng(1).integers(0, 10, 500)
    res = run_benchmark(net, x, y, batch_sizes=(64, 256), n_warmup=1, n_runs=2)
    names = {r.name for r in res}
    assert {"soft (float32)", "hard uint8 (CUDA)", "bitpacked GPU (CUDA graph)"} <= names
    accs = {(r.name, r.batch_size): r.accuracy for r in res if r.accuracy is not None}
    for B in (64, 256):      # the hard and bit-packed paths compute the same circuit
        assert accs[("hard uint8 (CUDA)", B)] == accs[("bitpacked GPU (CUDA graph)", B)]
    summ = speedup_summary(res)
    assert set(summ) == {64, 256} and set(summ[64]) == {"hard_kps", "bitpacked_kps", "speedup_x"}
    print_report(res)
    assert "Batch size = 256" in capsys.readouterr().out
    conv = S.LogicTreeNet(in_channels=3, in_hw=8, channels=[8, 16], head_widths=[40],
                          tree_depth=2, node="gate16", tau=4.0, seed=0)
    xc = (np.random.default_rng(2).random((100, 3, 8, 8)) < 0.5).astype(np.uint8)
    resc = run_conv_benchmark(conv, xc, None, batch_sizes=(64,), n_warmup=1, n_runs=2)
    assert len(resc) == 4 and all(r.mean_ms > 0 for r in resc)
    with pytest.raises(RuntimeError, match="CUDA"):
        run_benchmark(net, x, y, batch_sizes=(64,), device="cpu")
