"""The C-ABI library loads, exports every symbol the header declares, and rejects
bad arguments with status codes (validation only: no kernel is launched)."""
import ctypes
import os
import re

import pytest

from conftest import ROOT
from silogic_b200 import _lib

HEADER = os.path.join(ROOT, "include", "silogic_b200.h")


def _declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"\b(?:int|int64_t|const char\*)\s+(slg_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def L():
    if not os.path.exists(_lib.LIB_PATH):
        from silogic_b200 import build
        build.build()
    return _lib.lib()


def test_every_declared_symbol_is_exported(L):
    names = _declared()
    assert len(names) >= 8
    for n in names:
        assert hasattr(L, n), n


def test_version(L):
    assert L.slg_version() >= 100


def _p(v):
    return ctypes.c_void_p(v)


def test_bad_arguments_are_rejected(L):
    # odd leading dimension
    st = L.slg_fc_hard(_p(256), 10, 3, _p(512), _p(1024), 2, 10, 0, _p(2048), _p(0))
    assert st == 2 and b"even" in L.slg_last_error()
    # misaligned pointer
    st = L.slg_fc_hard(_p(258), 10, 2, _p(512), _p(1024), 2, 10, 0, _p(2048), _p(0))
    assert st == 2
    # unsupported arity
    st = L.slg_fc_hard(_p(256), 10, 2, _p(512), _p(1024), 7, 10, 0, _p(2048), _p(0))
    assert st == 3
    # conv tree shape not built
    st = L.slg_conv_hard(_p(256), 4, 8, 8, 2, _p(512), _p(1024), 2, 7, 3, 1, 4, 0, 2, _p(2048), _p(0))
    assert st == 3
    # groupsum: width not divisible
    st = L.slg_groupsum(_p(256), 11, 2, 64, 10, _p(512), _p(0))
    assert st == 1
    # empty work is a no-op success
    assert L.slg_pack_u8(_p(0), 0, 5, _p(0), 2, _p(0)) == 0


def test_chain_planner_runs_on_the_host_and_rejects_bad_wiring():
    """slg_fc_chain_plan is host code: it runs without a GPU, lays the last layer out in
    per-class blocks padded to whole warps, and refuses a wiring that reads past the
    previous layer."""
    import numpy as np
    from silogic_b200._hard import CHAIN_MAX_WIDTH
    P = ctypes.c_void_p
    in_dim, out, C = 40, 50, 5
    rng = np.random.default_rng(0)
    idx = rng.integers(0, in_dim, (out, 2)).astype(np.int32)
    tt = rng.integers(0, 16, out).astype(np.uint64)
    outs, wr = np.array([out], np.int64), np.array([0], np.int64)
    rec = np.zeros(2 * CHAIN_MAX_WIDTH, np.uint32)
    widths, off = np.zeros(1, np.int32), np.zeros(C + 1, np.int32)

    def plan(idx_arr, reorder):
        return _lib.lib().slg_fc_chain_plan(in_dim, 1, P(outs.ctypes.data), P(idx_arr.ctypes.data),
                                           P(tt.ctypes.data), P(wr.ctypes.data), C, reorder,
                                           P(rec.ctypes.data), CHAIN_MAX_WIDTH,
                                           P(widths.ctypes.data), P(off.ctypes.data))
    assert plan(idx, 0) == 0
    assert widths[0] % 32 == 0 and list(off) == [32 * c for c in range(C + 1)]
    for c in range(C):                 # each class's 10 nodes sit in its own block
        r = rec[off[c]:off[c + 1]].astype(np.int64)
        have = set(zip((r & 0x3fff).tolist(), ((r >> 14) & 0x3fff).tolist(), (r >> 28).tolist()))
        want = set(zip(idx[10 * c:10 * c + 10, 0].tolist(), idx[10 * c:10 * c + 10, 1].tolist(),
                       tt[10 * c:10 * c + 10].astype(np.int64).tolist()))
        assert want <= have
    bad = idx.copy()
    bad[3, 1] = in_dim                 # one past the input layer
    assert plan(bad, 1) != 0
    assert b"out of range" in _lib.lib().slg_last_error()


def test_index_check_rejects_null_and_bad_sizes(L):
    """slg_check_index_range validates its arguments before touching any memory."""
    assert L.slg_check_index_range(None, 0, 10, None, None) == 0          # nothing to check
    assert L.slg_check_index_range(None, 5, 10, None, None) == 1
    assert L.slg_check_index_range(None, -1, 10, None, None) == 1


def test_plan_and_layers_reject_out_of_range_wiring():
    """A wiring index outside the layer's input (e.g. from a corrupted checkpoint) is
    refused when the circuit is built, before any kernel could read past the input."""
    import torch
    import silogic_b200 as S
    from silogic_b200.bitpacking.plan import HardPlan
    from silogic_b200.bitpacking.packed import PackedFCLayer, PackedConvLayer
    torch.manual_seed(0)
    m = S.LogicNet(20, 30, 2, node="gate16", connectome="topk", k=4, tau=1.0, seed=0)
    HardPlan.from_model(m)                                           # valid wiring builds
    with torch.no_grad():
        m.layers[1]._conn.cand[0, 0, :] = 30                         # layer 1 reads 30 rows
    with pytest.raises(IndexError, match="FC layer 1"):
        HardPlan.from_model(m)
    with pytest.raises(IndexError):
        PackedFCLayer(torch.tensor([[0, -1]], dtype=torch.int32), torch.tensor([6]))
    conv = S.LogicTreeNet(in_channels=3, in_hw=8, channels=[4, 8], head_widths=[40], tree_depth=1,
                          node="gate16", tau=1.0, seed=0)
    HardPlan.from_model(conv)
    with torch.no_grad():
        blk = conv.blocks[2]
        (blk.leaf_cand if blk.connect != "fixed" else blk.leaf_idx)[0, 0] = 4 * 9   # cin*k*k
    with pytest.raises(IndexError, match="conv block 1"):
        HardPlan.from_model(conv)
    with pytest.raises(IndexError):
        PackedConvLayer(torch.tensor([[0, 27]], dtype=torch.int32), torch.tensor([[6]]), 2, 1, 3,
                        1, 3, 1)


def test_tuning_keys_and_env():
    """slg_tuning_set accepts each key's documented range and refuses the rest;
    SLG_TUNING applies settings when the library loads and rejects bad ones."""
    import subprocess
    import sys
    L = _lib.lib()
    ranges = {0: (0, 1), 1: (1, 64), 2: (0, 1), 3: (0, 2), 4: (0, 2), 5: (0, 1)}
    defaults = {0: 1, 1: 32, 2: 1, 3: 0, 4: 1, 5: 1}
    try:
        for key, (lo, hi) in ranges.items():
            assert L.slg_tuning_set(key, lo) == 0 and L.slg_tuning_set(key, hi) == 0
            assert L.slg_tuning_set(key, lo - 1) != 0 and L.slg_tuning_set(key, hi + 1) != 0
        assert L.slg_tuning_set(6, 0) != 0 and L.slg_tuning_set(-1, 0) != 0
    finally:
        for key, val in defaults.items():
            L.slg_tuning_set(key, val)
    code = "import silogic_b200._lib as l; l.lib()"
    env = dict(os.environ, SLG_TUNING="4=2, 3=1")
    assert subprocess.run([sys.executable, "-c", code], env=env, cwd=ROOT).returncode == 0
    for bad in ("4=9", "4", "x=1"):
        env["SLG_TUNING"] = bad
        r = subprocess.run([sys.executable, "-c", code], env=env, cwd=ROOT, capture_output=True, text=True)
        assert r.returncode != 0 and "SLG_TUNING" in r.stderr
