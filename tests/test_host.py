"""Host-side logic on CPU: constructor parity (seeded wiring), state_dict layout,
parameter -> truth-table conversion, plan building.  No kernel launches."""
import numpy as np
import pytest
import torch

from helpers import FIXTURES, build_model, load
from oracle import hard as OH
from oracle.spec import net_spec
from silogic_b200 import _hard


@pytest.mark.parametrize("name", FIXTURES)
def test_constructor_matches_reference_state_dict(name):
    """Same seed -> identical wiring buffers and identical state_dict keys/shapes."""
    m, enc, z, fresh = build_model(name)
    ref_keys = {k[3:] for k in z.files if k.startswith("sd/")}
    assert set(fresh) == ref_keys
    for k, v in fresh.items():
        ref = z["sd/" + k]
        assert tuple(v.shape) == ref.shape, k
        if v.dtype in (torch.int64, torch.int32) or k.endswith(("basis", "truth", "corners")):
            np.testing.assert_array_equal(v.numpy(), ref, err_msg=k)


@pytest.mark.parametrize("name", FIXTURES)
def test_truth_tables_match_oracle(name):
    m, enc, z, _ = build_model(name)
    sd = {k[3:]: z[k] for k in z.files if k.startswith("sd/")}
    spec = net_spec(str(z["ctor"]), str(z["kwargs"]), sd)
    fc_layers = spec["layers"] if spec["type"] == "fc" else spec["head"]
    mods = m.layers if spec["type"] == "fc" else m.head_layers
    for L, mod in zip(fc_layers, mods):
        idx, tt = mod.hard_spec()
        oidx, ott = OH.fc_hard_spec(L)
        np.testing.assert_array_equal(idx.numpy(), oidx)
        P = ott.shape[1]
        bits = ((tt.unsqueeze(1) >> torch.arange(P)) & 1).bool().numpy()
        np.testing.assert_array_equal(bits, ott)
    if spec["type"] == "conv":
        for Bk, conv in zip(spec["blocks"], m.blocks[0::2]):
            leaf, tt = conv.hard_spec()
            oleaf, otts = OH.conv_hard_spec(Bk)
            np.testing.assert_array_equal(leaf.numpy(), oleaf)
            ott = np.concatenate(otts, axis=1)            # [n, total, P]
            P = ott.shape[2]
            bits = ((tt.unsqueeze(-1) >> torch.arange(P)) & 1).bool().numpy()
            np.testing.assert_array_equal(bits, ott)


def test_gate16_lut_codes():
    from silogic_b200.functional import gate16_lut_codes, TRUTH_TABLES
    codes = gate16_lut_codes()
    for g in range(16):
        for a in (0, 1):
            for b in (0, 1):
                assert ((int(codes[g]) >> (a | (b << 1))) & 1) == int(TRUTH_TABLES[g, (a << 1) | b])


def test_ldw_and_words():
    assert [_hard.n_words(b) for b in (1, 64, 65, 128, 129)] == [1, 1, 2, 2, 3]
    assert _hard.ldw_for(1) == 2 and _hard.ldw_for(129) == 4 and _hard.ldw_for(256) == 4


def test_cpu_tensors_are_rejected():
    import silogic_b200 as S
    net = S.LogicNet(16, 20, 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        net.forward_hard(torch.zeros(4, 16))


def _emulate_chain(rec, widths, class_off, xp, num_classes, B):
    """Evaluate chain node records on packed uint64 words (numpy), then GroupSum."""
    cur = xp
    o = 0
    for w in widths:
        r = rec[o:o + w].astype(np.uint64)
        o += w
        a, b, g = cur[(r & 0x3fff).astype(np.int64)], cur[((r >> 14) & 0x3fff).astype(np.int64)], r >> 28
        m = [(0 - ((g >> np.uint64(k)) & np.uint64(1))).astype(np.uint64)[:, None] for k in range(4)]
        f0 = (a & m[1]) | (~a & m[0])
        f1 = (a & m[3]) | (~a & m[2])
        cur = (b & f1) | (~b & f0)
    bits = np.unpackbits(cur.view(np.uint8), axis=1, bitorder="little")[:, :B].astype(np.int64)
    return np.stack([bits[class_off[c]:class_off[c + 1]].sum(0) for c in range(num_classes)], 1)


@pytest.mark.parametrize("kw", [dict(node="walsh", connectome="topk", k=8, tau=10.0),
                                dict(node="gate16", connectome="topk", k=4, tau=10.0,
                                     wire_residual=0.25)])
def test_chain_layout_bank_grouping_preserves_the_circuit(kw):
    """The fused FC kernel's reordered, bank-conflict-free node layout computes the same
    counts as the oracle (records emulated on the CPU), and every half-warp of 16 slots
    reads 16 distinct shared-memory bank pairs (no conflicts)."""
    import silogic_b200 as S
    from silogic_b200.bitpacking.plan import HardPlan
    torch.manual_seed(3)
    m = S.LogicNet(64, 320, 3, seed=3, **kw)
    with torch.no_grad():
        for p in m.parameters():
            p.normal_()
    plan = HardPlan.from_model(m)
    rec, widths, off = _hard.chain_layout(plan.steps, 64, 10)
    assert all(w % 32 == 0 for w in widths)
    x = (torch.rand(150, 64, generator=torch.Generator().manual_seed(1)) < 0.4).numpy().astype(np.uint8)
    xp = OH.pack_bits(x)
    sd = {k: v.numpy() for k, v in m.state_dict().items()}
    ref = OH.model_counts("LogicNet", dict(in_dim=64, width=320, depth=3, seed=3, **kw), sd, x)
    np.testing.assert_array_equal(_emulate_chain(rec, widths, off, xp, 10, 150), ref)
    off = 0
    for w in widths:
        r = rec[off:off + w].astype(np.int64)
        for g in range(0, w, 16):                      # each half-warp: distinct pairs
            for sh in (0, 14):
                slots = np.unique((r[g:g + 16] >> sh) & 0x3fff)
                assert np.bincount(slots % 16, minlength=16).max() <= 1
        off += w


def test_build_inverse_map_lists_every_reader_in_order():
    import silogic_b200.kernels as K
    cm = torch.tensor([[0, 2], [1, 0]], dtype=torch.int32)
    ch = torch.tensor([[0, 1], [2, 1]], dtype=torch.int32)
    cw = torch.tensor([[1, 2], [0, 0]], dtype=torch.int32)
    off, en, el, edy, edx = K.build_inverse_map(cm, ch, cw, 3)
    assert off.tolist() == [0, 2, 3, 4]
    assert list(zip(en.tolist(), el.tolist())) == [(0, 0), (1, 1), (1, 0), (0, 1)]
    assert edy.tolist() == [0, 1, 2, 1] and edx.tolist() == [1, 0, 0, 2]


def test_packed_artefact_round_trip_and_corrupt_wiring(tmp_path):
    """save_packed / load_packed keep every step's wiring, tables and geometry and the
    head; a file whose wiring reads past its input is refused on load."""
    import silogic_b200 as S
    from silogic_b200.bitpacking import convert_logic_net, convert_logic_conv_net, save_packed, load_packed
    torch.manual_seed(0)
    for m, conv in ((S.LogicNet(30, 40, 2, node="walsh", connectome="topk", k=4, tau=3.0, seed=0), False),
                    (S.LogicTreeNet(in_channels=3, in_hw=8, channels=[4, 8], head_widths=[40],
                                    tree_depth=2, node="gate16", tau=2.0, seed=0), True)):
        bp = convert_logic_conv_net(m) if conv else convert_logic_net(m)
        path = tmp_path / ("c.npz" if conv else "f.npz")
        save_packed(bp, path)
        back = load_packed(path, device="cpu")
        assert type(back).__name__ == type(bp).__name__
        assert back.plan.in_shape == tuple(bp.plan.in_shape) and back.head.tau == bp.head.tau
        for a, b in zip(bp.plan.steps, back.plan.steps):
            assert a["op"] == b["op"]
            key = "idx" if a["op"] == "fc" else "leaf"
            assert torch.equal(a[key].to(torch.int32), b[key]) and torch.equal(a["tt"], b["tt"])
    z = dict(np.load(tmp_path / "f.npz"))
    z["step1/wiring"] = z["step1/wiring"].copy()
    z["step1/wiring"][0, 0] = 40                     # layer 1 reads only 40 rows
    np.savez(tmp_path / "bad.npz", **z)
    with pytest.raises(IndexError):
        load_packed(tmp_path / "bad.npz", device="cpu")
    z["format"] = np.array("something else")
    np.savez(tmp_path / "other.npz", **z)
    with pytest.raises(ValueError):
        load_packed(tmp_path / "other.npz", device="cpu")


def test_pipeline_slice_size_rule():
    """Host batches are sliced by bytes (multiples of 1024 samples) with a floor of
    min_slice_samples, so per-slice replays of heavy networks still fill the GPU."""
    from types import SimpleNamespace
    from silogic_b200.bitpacking.packed import BitpackedConvNet
    ns = SimpleNamespace(pipeline_bytes=8 << 20, min_slice_samples=16384)
    img_u8 = torch.zeros(4, 3, 32, 32, dtype=torch.uint8)     # 3,072 B per sample
    feats = torch.zeros(4, 784, dtype=torch.uint8)             # 784 B per sample
    assert BitpackedConvNet._slice(ns, img_u8) == 16384
    assert BitpackedConvNet._slice(ns, img_u8.float()) == 16384
    ns.min_slice_samples = 1024
    assert BitpackedConvNet._slice(ns, img_u8) == 3072
    assert BitpackedConvNet._slice(ns, feats) == 11264
    ns.pipeline_bytes = 1
    assert BitpackedConvNet._slice(ns, feats) == 1024
