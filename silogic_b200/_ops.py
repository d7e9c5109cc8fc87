"""The soft-path kernels as ``torch.library`` custom ops (namespace ``silogic_b200``).

Each op wraps one C-ABI entry point functionally (new output tensors, no mutation of
its inputs) and has a fake (meta) implementation that only computes shapes, so
``torch.compile`` / ``torch.export`` can trace the autograd Functions of ``_soft`` that
call them without breaking the graph (:func:`op` picks the registered op while tracing
and the plain function in eager mode).  Absent optional outputs are returned as empty
tensors (custom ops cannot return ``None``).
"""
from typing import Optional, Tuple

import torch
from torch import Tensor

from ._lib import call, lib, ptr, require_cuda, stream_ptr


#: the undecorated implementations, called directly in eager mode: the custom-op
#: dispatcher costs tens of microseconds a call, which small soft steps would notice
IMPL = {}


def _op(name):
    """Register ``fn`` as ``torch.ops.silogic_b200.<name>`` and keep the raw function."""
    def deco(fn):
        IMPL[name] = fn
        return torch.library.custom_op(f"silogic_b200::{name}", mutates_args=())(fn)
    return deco


def op(name):
    """The op to call: the registered custom op while torch.compile traces (so the graph
    holds an opaque node with a fake implementation), the raw function otherwise."""
    if torch.compiler.is_compiling():
        return getattr(torch.ops.silogic_b200, name)
    return IMPL[name]


def _none_if_empty(t):
    return None if t is None or t.numel() == 0 else t


def _empty(device, dtype=torch.float32):
    return torch.empty(0, dtype=dtype, device=device)


# ------------------------------------------------------------- transposes
@_op("to_feature_major")
def to_feature_major(x: Tensor, ldb: int) -> Tensor:
    """``[B, F]`` -> ``[F, ldb]`` fp32, padding columns zero."""
    require_cuda(x)
    x = x.float().contiguous()
    B, F = x.shape
    out = torch.empty((F, ldb), dtype=torch.float32, device=x.device)
    call("slg_to_feature_major", ptr(x), B, F, ptr(out), ldb, stream_ptr(x.device))
    return out


@to_feature_major.register_fake
def _(x, ldb):
    return x.new_empty((x.shape[1], ldb), dtype=torch.float32)


@_op("from_feature_major")
def from_feature_major(xt: Tensor, B: int) -> Tensor:
    """``[F, ldb]`` -> ``[B, F]`` fp32."""
    require_cuda(xt)
    xt = xt.float().contiguous()
    F, ldb = xt.shape
    out = torch.empty((B, F), dtype=torch.float32, device=xt.device)
    call("slg_from_feature_major", ptr(xt), F, ldb, B, ptr(out), stream_ptr(xt.device))
    return out


@from_feature_major.register_fake
def _(xt, B):
    return xt.new_empty((B, xt.shape[0]), dtype=torch.float32)


# --------------------------------------------------------------- FC layer
@_op("fc_soft_fwd")
def fc_soft_fwd(xt: Tensor, cand: Tensor, conn: Optional[Tensor], params: Tensor, K: int,
                ste: int, node: int, arity: int, gate_hard: int, inv_tau: float, out_dim: int,
                wire_r: int) -> Tensor:
    require_cuda(xt)
    in_dim, ldb = xt.shape
    y = torch.empty((out_dim, ldb), dtype=torch.float32, device=xt.device)
    call("slg_fc_soft_fwd", ptr(xt), in_dim, ldb, ptr(cand), ptr(conn), K, ste, node, arity,
         ptr(params), gate_hard, inv_tau, out_dim, wire_r, ptr(y), stream_ptr(xt.device))
    return y


@fc_soft_fwd.register_fake
def _(xt, cand, conn, params, K, ste, node, arity, gate_hard, inv_tau, out_dim, wire_r):
    return xt.new_empty((out_dim, xt.shape[1]))


@_op("fc_soft_bwd")
def fc_soft_bwd(xt: Tensor, cand: Tensor, conn: Optional[Tensor], params: Tensor, K: int,
                ste: int, node: int, arity: int, gate_hard: int, inv_tau: float, out_dim: int,
                wire_r: int, gy: Tensor, need_gx: bool) -> Tuple[Tensor, Tensor, Tensor]:
    """(gx or empty, gparams, gconn or empty)."""
    require_cuda(xt)
    in_dim, ldb = xt.shape
    gy = gy.contiguous()
    gx = torch.zeros_like(xt) if need_gx else None
    gparams = torch.empty_like(params)
    gconn = torch.empty_like(conn) if conn is not None else None
    nbytes = lib().slg_fc_soft_workspace_bytes(ldb, K, node, arity, out_dim)
    ws = torch.empty(max(nbytes, 4) // 4 + 1, dtype=torch.float32, device=xt.device)
    call("slg_fc_soft_bwd", ptr(xt), in_dim, ldb, ptr(cand), ptr(conn), K, ste, node, arity,
         ptr(params), gate_hard, inv_tau, out_dim, wire_r, ptr(gy), ptr(gx), ptr(gconn),
         ptr(gparams), ptr(ws), ws.numel() * 4, stream_ptr(xt.device))
    return (gx if gx is not None else _empty(xt.device), gparams,
            gconn if gconn is not None else _empty(xt.device))


@fc_soft_bwd.register_fake
def _(xt, cand, conn, params, K, ste, node, arity, gate_hard, inv_tau, out_dim, wire_r, gy,
      need_gx):
    gx = torch.empty_like(xt) if need_gx else xt.new_empty((0,))
    gconn = torch.empty_like(conn) if conn is not None else xt.new_empty((0,))
    return gx, torch.empty_like(params), gconn


# ---------------------------------------------------------------- GroupSum
@_op("groupsum_soft_fwd")
def groupsum_soft_fwd(xt: Tensor, B: int, C: int, tau: float, ste: int) -> Tensor:
    require_cuda(xt)
    xt = xt.contiguous()
    W, ldb = xt.shape
    out = torch.empty((B, C), dtype=torch.float32, device=xt.device)
    call("slg_groupsum_soft_fwd", ptr(xt), W, ldb, B, C, tau, ste, ptr(out), stream_ptr(xt.device))
    return out


@groupsum_soft_fwd.register_fake
def _(xt, B, C, tau, ste):
    return xt.new_empty((B, C))


@_op("groupsum_soft_bwd")
def groupsum_soft_bwd(g: Tensor, W: int, ldb: int, tau: float) -> Tensor:
    require_cuda(g)
    g = g.float().contiguous()
    B, C = g.shape
    gx = torch.empty((W, ldb), dtype=torch.float32, device=g.device)
    call("slg_groupsum_soft_bwd", ptr(g), W, ldb, B, C, tau, ptr(gx), stream_ptr(g.device))
    return gx


@groupsum_soft_bwd.register_fake
def _(g, W, ldb, tau):
    return g.new_empty((W, ldb))


# --------------------------------------------------------------- conv tree
def _conv_out(C, H, W, kernel, pad, pool, n_out):
    Ho, Wo = H + 2 * pad - kernel + 1, W + 2 * pad - kernel + 1
    return n_out * (Ho // pool) * (Wo // pool)


@_op("conv_soft_fwd")
def conv_soft_fwd(xt: Tensor, C: int, H: int, W: int, cand: Tensor, conn: Optional[Tensor],
                  params: Tensor, K: int, ste: int, node: int, arity: int, depth: int,
                  gate_hard: int, inv_tau: float, kernel: int, pad: int, n_out: int, wire_r: int,
                  pool: int, keep_arg: bool) -> Tuple[Tensor, Tensor]:
    """(y [n*Hp*Wp, ldb], pool-window argmax uint8 of the same shape or empty)."""
    require_cuda(xt)
    ldb = xt.shape[-1]
    rows = _conv_out(C, H, W, kernel, pad, pool, n_out)
    y = torch.empty((rows, ldb), dtype=torch.float32, device=xt.device)
    arg = torch.empty((rows, ldb), dtype=torch.uint8, device=xt.device) if keep_arg else None
    call("slg_conv_soft_fwd", ptr(xt), C, H, W, ldb, ptr(cand), ptr(conn), K, ste, node, arity,
         depth, ptr(params), gate_hard, inv_tau, kernel, pad, n_out, wire_r, pool, ptr(y),
         ptr(arg), stream_ptr(xt.device))
    return y, arg if arg is not None else _empty(xt.device, torch.uint8)


@conv_soft_fwd.register_fake
def _(xt, C, H, W, cand, conn, params, K, ste, node, arity, depth, gate_hard, inv_tau, kernel,
      pad, n_out, wire_r, pool, keep_arg):
    rows = _conv_out(C, H, W, kernel, pad, pool, n_out)
    y = xt.new_empty((rows, xt.shape[-1]))
    arg = xt.new_empty((rows, xt.shape[-1]) if keep_arg else (0,), dtype=torch.uint8)
    return y, arg


@_op("conv_soft_bwd")
def conv_soft_bwd(xt: Tensor, C: int, H: int, W: int, cand: Tensor, conn: Optional[Tensor],
                  params: Tensor, K: int, ste: int, node: int, arity: int, depth: int,
                  gate_hard: int, inv_tau: float, kernel: int, pad: int, n_out: int, wire_r: int,
                  pool: int, gy: Tensor, arg: Optional[Tensor],
                  need_gx: bool) -> Tuple[Tensor, Tensor, Tensor]:
    """(gx or empty, gparams, gconn or empty)."""
    require_cuda(xt)
    ldb = xt.shape[-1]
    gy = gy.contiguous()
    arg = _none_if_empty(arg)
    gx = torch.zeros_like(xt) if need_gx else None
    gparams = torch.empty_like(params)
    gconn = torch.empty_like(conn) if conn is not None else None
    nbytes = lib().slg_conv_soft_workspace_bytes(H, W, ldb, K, node, arity, depth, kernel, pad,
                                                 pool, n_out)
    ws = torch.empty(max(nbytes, 4) // 4 + 1, dtype=torch.float32, device=xt.device)
    call("slg_conv_soft_bwd", ptr(xt), C, H, W, ldb, ptr(cand), ptr(conn), K, ste, node, arity,
         depth, ptr(params), gate_hard, inv_tau, kernel, pad, n_out, wire_r, pool, ptr(gy),
         ptr(arg), ptr(gx), ptr(gconn), ptr(gparams), ptr(ws), ws.numel() * 4,
         stream_ptr(xt.device))
    return (gx if gx is not None else _empty(xt.device), gparams,
            gconn if gconn is not None else _empty(xt.device))


@conv_soft_bwd.register_fake
def _(xt, C, H, W, cand, conn, params, K, ste, node, arity, depth, gate_hard, inv_tau, kernel,
      pad, n_out, wire_r, pool, gy, arg, need_gx):
    gx = torch.empty_like(xt) if need_gx else xt.new_empty((0,))
    gconn = torch.empty_like(conn) if conn is not None else xt.new_empty((0,))
    return gx, torch.empty_like(params), gconn


# ------------------------------------------------------------------ OrPool
@_op("or_pool_fwd")
def or_pool_fwd(x: Tensor, size: int) -> Tensor:
    require_cuda(x)
    x = x.float().contiguous()
    B, C, H, W = x.shape
    y = torch.empty((B, C, H // size, W // size), dtype=torch.float32, device=x.device)
    call("slg_or_pool_fwd", ptr(x), B * C, H, W, size, ptr(y), stream_ptr(x.device))
    return y


@or_pool_fwd.register_fake
def _(x, size):
    B, C, H, W = x.shape
    return x.new_empty((B, C, H // size, W // size), dtype=torch.float32)


@_op("or_pool_bwd")
def or_pool_bwd(x: Tensor, gy: Tensor, size: int) -> Tensor:
    require_cuda(x)
    B, C, H, W = x.shape
    gy = gy.contiguous()
    gx = torch.zeros_like(x)
    call("slg_or_pool_bwd", ptr(x), ptr(gy), B * C, H, W, size, ptr(gx), stream_ptr(x.device))
    return gx


@or_pool_bwd.register_fake
def _(x, gy, size):
    return torch.empty_like(x)


# ---------------------------------------------------------------- encoder
@_op("thermo_soft_fwd")
def thermo_soft_fwd(x: Tensor, thr: Tensor) -> Tensor:
    require_cuda(x)
    B, F = x.shape
    T = thr.shape[1]
    out = torch.empty((B, F * T), dtype=torch.float32, device=x.device)
    call("slg_thermo_soft_fwd", ptr(x), ptr(thr), B, F, T, ptr(out), stream_ptr(x.device))
    return out


@thermo_soft_fwd.register_fake
def _(x, thr):
    return x.new_empty((x.shape[0], x.shape[1] * thr.shape[1]))


@_op("thermo_soft_bwd")
def thermo_soft_bwd(x: Tensor, thr: Tensor, g: Tensor, scale: float,
                    need_gx: bool) -> Tuple[Tensor, Tensor]:
    """(gx or empty, gthr)."""
    require_cuda(x)
    B, F = x.shape
    T = thr.shape[1]
    g = g.float().contiguous()
    gx = torch.zeros_like(x) if need_gx else None
    gthr = torch.zeros_like(thr)
    call("slg_thermo_soft_bwd", ptr(x), ptr(thr), ptr(g), B, F, T, scale, ptr(gx), ptr(gthr),
         stream_ptr(x.device))
    return gx if gx is not None else _empty(x.device), gthr


@thermo_soft_bwd.register_fake
def _(x, thr, g, scale, need_gx):
    return (torch.empty_like(x) if need_gx else x.new_empty((0,))), torch.empty_like(thr)
