"""The allocation-free soft FC backward (``slg_fc_soft_bwd_noalloc``), called through
the C ABI, matches the workspace form (``slg_fc_soft_bwd``) on two calls in a row.

It serves callers that cannot allocate device memory (a plugin whose host framework
owns every device buffer, or a loop that must not enter the allocator); its scratch
is a static 16 MiB device array shared by every call on the GPU.  This file is
collected last so that a failure here comes after every other test has run.
"""
import ctypes

import numpy as np
import pytest
import torch

from silogic_b200 import _lib

pytestmark = pytest.mark.gpu

_p, _i64, _i32, _f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_float
NOALLOC_ARGS = [_p, _i64, _i64, _p, _p, _i32, _i32, _i32, _i32, _p, _i32, _f32, _i64, _i64, _p, _p,
                _p, _p, _p]
LIMIT = 16 << 20          # SLG_FC_NOALLOC_SCRATCH_BYTES
GATE16, WALSH = 0, 1


def _close(got, ref, what):
    """Same tolerance as the other gradient tests: 1e-5 (|ref| + max|ref|) + 1e-7."""
    got, ref = got.cpu().numpy(), ref.cpu().numpy()
    tol = 1e-5 * (np.abs(ref) + np.abs(ref).max()) + 1e-7
    assert np.all(np.abs(got - ref) <= tol), f"{what}: max err {np.abs(got - ref).max():.3e}"


def _case(IN, OUT, B, K, node, with_conn=True, wire_r=0, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    ldb = (B + 3) // 4 * 4
    x = torch.zeros(IN, ldb)
    x[:, :B] = (torch.rand(IN, B, generator=g) < 0.3).float()
    gy = torch.zeros(OUT, ldb)
    gy[:, :B] = torch.randn(OUT, B, generator=g)
    cand = torch.randint(0, IN, (OUT, 2, K), generator=g, dtype=torch.int32)
    conn = torch.randn(OUT, 2, K, generator=g) if with_conn else None
    params = torch.randn(OUT, 16 if node == GATE16 else 4, generator=g)
    dev = "cuda"
    t = [v.to(dev).contiguous() if v is not None else None for v in (x, gy, cand, conn, params)]
    return ldb, t


def _run_both(IN, OUT, B, K, node, with_conn=True, wire_r=0):
    _lib.declare("slg_fc_soft_bwd_noalloc", NOALLOC_ARGS)
    L = _lib.lib()
    ldb, (x, gy, cand, conn, params) = _case(IN, OUT, B, K, node, with_conn, wire_r)
    Kc = K if with_conn else 1
    if not with_conn:
        cand = cand[:, :, :1].contiguous()
    st = _lib.stream_ptr()
    common = (_lib.ptr(x), IN, ldb, _lib.ptr(cand), _lib.ptr(conn), Kc, 0, node, 2,
              _lib.ptr(params), 0, 1.0, OUT, wire_r, _lib.ptr(gy))

    def outs():
        gc = torch.empty_like(conn) if conn is not None else None
        return torch.zeros_like(x), gc, torch.empty_like(params)

    nbytes = L.slg_fc_soft_workspace_bytes(ldb, Kc, node, 2, OUT)
    assert nbytes <= LIMIT
    gx0, gc0, gp0 = outs()
    ws = torch.empty(nbytes // 4 + 1, device="cuda")
    _lib.call("slg_fc_soft_bwd", *common, _lib.ptr(gx0), _lib.ptr(gc0), _lib.ptr(gp0),
              _lib.ptr(ws), ws.numel() * 4, st)
    for call in range(2):
        gx, gc, gp = outs()
        _lib.call("slg_fc_soft_bwd_noalloc", *common, _lib.ptr(gx), _lib.ptr(gc), _lib.ptr(gp), st)
        torch.cuda.synchronize()
        _close(gx, gx0, f"call {call} gx")
        if gc is not None:
            _close(gc, gc0, f"call {call} gconn")
        _close(gp, gp0, f"call {call} gparams")
    return nbytes


@pytest.mark.parametrize("node", [GATE16, WALSH], ids=["gate16", "walsh"])
@pytest.mark.parametrize("K", [1, 8, 16])
def test_fc_soft_bwd_noalloc_matches_workspace_form(node, K):
    _run_both(700, 900, 1000, K, node)


def test_fc_soft_bwd_noalloc_fixed_wiring_and_wire_residual():
    _run_both(600, 800, 777, 4, WALSH, with_conn=False, wire_r=300)


def test_fc_soft_bwd_noalloc_at_exactly_the_array_size():
    """K = 14 Walsh: 32 floats of partials per (node, 512-sample chunk); 16,384 nodes x 8
    chunks fill the 16 MiB array exactly, and one more node is refused."""
    assert _run_both(500, 16384, 4096, 14, WALSH) == LIMIT
    L = _lib.lib()
    assert L.slg_fc_soft_workspace_bytes(4096, 14, WALSH, 2, 16385) > LIMIT


def test_fc_soft_bwd_noalloc_rejects_sizes_beyond_its_array():
    """The scratch size is checked before any pointer, so the question needs no buffers:
    10000 nodes x 16 candidates at batch 65536 need far more than 16 MiB of partials."""
    _lib.declare("slg_fc_soft_bwd_noalloc", NOALLOC_ARGS)
    L = _lib.lib()
    st = L.slg_fc_soft_bwd_noalloc(None, 10000, 65536, None, None, 16, 0, WALSH, 2, None,
                                   0, 1.0, 10000, 0, None, None, None, None, None)
    assert st == 5 and b"static array" in L.slg_last_error()
    # scalar arguments are still checked first, with slg_fc_soft_bwd's codes
    st = L.slg_fc_soft_bwd_noalloc(None, 10000, 65536, None, None, 17, 0, WALSH, 2, None,
                                   0, 1.0, 10000, 0, None, None, None, None, None)
    assert st == 3
    st = L.slg_fc_soft_bwd_noalloc(None, 10000, 65538, None, None, 8, 0, WALSH, 2, None,
                                   0, 1.0, 10000, 0, None, None, None, None, None)
    assert st == 2
