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


def _close(got, ref, what):
    """Same tolerance as the other gradient tests: 1e-5 (|ref| + max|ref|) + 1e-7."""
    got, ref = got.cpu().numpy(), ref.cpu().numpy()
    tol = 1e-5 * (np.abs(ref) + np.abs(ref).max()) + 1e-7
    assert np.all(np.abs(got - ref) <= tol), f"{what}: max err {np.abs(got - ref).max():.3e}"


def test_fc_soft_bwd_noalloc_matches_workspace_form():
    _lib.declare("slg_fc_soft_bwd_noalloc", NOALLOC_ARGS)
    L = _lib.lib()
    dev = "cuda"
    g = torch.Generator(device="cpu").manual_seed(0)
    IN, OUT, B, K, AR, node = 700, 900, 1000, 8, 2, 1          # walsh nodes, Top-K 8
    ldb = (B + 3) // 4 * 4
    x = torch.zeros(IN, ldb)
    x[:, :B] = (torch.rand(IN, B, generator=g) < 0.3).float()
    gy = torch.zeros(OUT, ldb)
    gy[:, :B] = torch.randn(OUT, B, generator=g)
    cand = torch.randint(0, IN, (OUT, AR, K), generator=g, dtype=torch.int32)
    conn = torch.randn(OUT, AR, K, generator=g)
    theta = torch.randn(OUT, 4, generator=g)
    x, gy, cand, conn, theta = (t.to(dev).contiguous() for t in (x, gy, cand, conn, theta))
    st = _lib.stream_ptr()
    common = (_lib.ptr(x), IN, ldb, _lib.ptr(cand), _lib.ptr(conn), K, 0, node, AR, _lib.ptr(theta),
              0, 1.0, OUT, 0, _lib.ptr(gy))

    def outs():
        return torch.zeros_like(x), torch.empty_like(conn), torch.empty_like(theta)

    gx0, gc0, gp0 = outs()
    nbytes = L.slg_fc_soft_workspace_bytes(ldb, K, node, AR, OUT)
    ws = torch.empty(nbytes // 4 + 1, device=dev)
    _lib.call("slg_fc_soft_bwd", *common, _lib.ptr(gx0), _lib.ptr(gc0), _lib.ptr(gp0),
              _lib.ptr(ws), ws.numel() * 4, st)
    for call in range(2):
        gx, gc, gp = outs()
        _lib.call("slg_fc_soft_bwd_noalloc", *common, _lib.ptr(gx), _lib.ptr(gc), _lib.ptr(gp), st)
        torch.cuda.synchronize()
        _close(gx, gx0, f"call {call} gx")
        _close(gc, gc0, f"call {call} gconn")
        _close(gp, gp0, f"call {call} gtheta")


def test_fc_soft_bwd_noalloc_rejects_sizes_beyond_its_array():
    _lib.declare("slg_fc_soft_bwd_noalloc", NOALLOC_ARGS)
    L = _lib.lib()
    # 10000 nodes x 16 candidates at batch 65536 needs far more than 16 MiB of partials
    st = L.slg_fc_soft_bwd_noalloc(_p(256), 10000, 65536, _p(512), _p(768), 16, 0, 1, 2, _p(1024),
                                   0, 1.0, 10000, 0, _p(2048), _p(0), _p(4096), _p(8192), _p(0))
    assert st == 5 and b"static array" in L.slg_last_error()
