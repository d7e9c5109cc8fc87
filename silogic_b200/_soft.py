"""Soft (relaxed, fp32) path: autograd Functions around the CUDA kernels.

Inside a network the activations are feature-major ``[F, ldb]`` (``ldb`` = batch
rounded up to a multiple of 4, padding columns zero) so each connectome gather
reads whole rows; the module boundary transposes once with a CUDA kernel.
Every Function's backward is a CUDA kernel too; parameter-side transforms
(connection softmax, gate_probs @ basis, sigmoid of LUT logits) are fused into
the layer kernels.
"""
import torch

from . import _hard
from ._ops import op
from ._lib import require_cuda


NODE_ID = {"gate16": 0, "walsh": 1, "multilinear": 2, "hybrid": 3, "linear": 4}


def ldb_for(B):
    return max(4, (int(B) + 3) // 4 * 4)


# ------------------------------------------------------------- transposes
class ToFeatureMajor(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        require_cuda(x)
        B = x.shape[0]
        ctx.shape = x.shape
        return op("to_feature_major")(x.reshape(B, -1), ldb_for(B))

    @staticmethod
    def backward(ctx, g):
        return op("from_feature_major")(g, ctx.shape[0]).view(ctx.shape)


class FromFeatureMajor(torch.autograd.Function):
    @staticmethod
    def forward(ctx, xt, B):
        ctx.ldb = xt.shape[1]
        return op("from_feature_major")(xt, B)

    @staticmethod
    def backward(ctx, g):
        return op("to_feature_major")(g, ctx.ldb), None


# --------------------------------------------------------------- FC layer
def fc_supported(layer):
    from .connectomes import FixedConnectome, TopKConnectome
    if layer.node.kind not in NODE_ID and layer.node.kind != "polynomial":
        return False
    if not isinstance(layer._conn, (FixedConnectome, TopKConnectome)):
        return False
    if isinstance(layer._conn, TopKConnectome) and layer._conn.k > 16:
        return False
    if layer.node.kind == "walsh" and layer.node.gate_select == "gumbel" and layer.training:
        return False
    return 1 <= layer.arity <= 6


def _fc_meta(layer, wire_r=0):
    """Static launch description of a LogicLayer's soft kernel."""
    from .connectomes import FixedConnectome, TopKConnectome
    if not fc_supported(layer):
        raise NotImplementedError(
            f"no soft kernel for node={layer.node.kind!r} connectome={type(layer._conn).__name__} "
            f"arity={layer.arity} in silogic_b200")
    node = layer.node
    kind = node.kind
    if isinstance(layer._conn, FixedConnectome):
        cand, K, ste, conn = layer._conn.cand_i32, 1, 0, None
    else:
        cand, K, ste, conn = layer._conn.cand_i32, layer._conn.k, int(layer._conn.ste), layer._conn.conn
    gate_hard = 0
    params = node.param
    if kind == "gate16" and layer.training:
        if node.gate_select == "hard":
            gate_hard = 1
        elif node.gate_select == "gumbel":
            g = -torch.empty_like(params).exponential_().log()
            params = (params + g) / node.gumbel_tau
            gate_hard = 1
    inv_tau = float(node.inv_tau) if kind == "walsh" else 1.0
    if kind == "polynomial":    # same function in the Walsh basis (see PolynomialNode)
        params, kind = node.walsh_theta(), "walsh"
    _hard.check_index_range(cand, layer.in_dim, "LogicLayer candidates")
    return dict(cand=cand.contiguous(), K=K, ste=ste, node=NODE_ID[kind], arity=layer.arity,
                gate_hard=gate_hard, inv_tau=inv_tau, out_dim=layer.out_dim,
                wire_r=wire_r), params, conn


class FCSoft(torch.autograd.Function):
    """Feature-major soft FC layer: xt [in, ldb] -> yt [out, ldb]."""

    @staticmethod
    def _args(meta):
        return (meta["K"], meta["ste"], meta["node"], meta["arity"], meta["gate_hard"],
                float(meta["inv_tau"]), meta["out_dim"], meta["wire_r"])

    @staticmethod
    def forward(ctx, xt, params, conn, meta):
        require_cuda(xt)
        xt = xt.contiguous()
        params = params.float().contiguous()
        connc = conn.float().contiguous() if conn is not None else None
        y = op("fc_soft_fwd")(xt, meta["cand"], connc, params, *FCSoft._args(meta))
        ctx.save_for_backward(xt, params, connc)
        ctx.meta = meta
        return y

    @staticmethod
    def backward(ctx, gy):
        xt, params, connc = ctx.saved_tensors
        m = ctx.meta
        gx, gparams, gconn = op("fc_soft_bwd")(xt, m["cand"], connc, params, *FCSoft._args(m), gy,
                                             bool(ctx.needs_input_grad[0]))
        return (gx if ctx.needs_input_grad[0] else None, gparams,
                gconn if connc is not None else None, None)


def fc_layer_fm(layer, xt, wire_r=0):
    meta, params, conn = _fc_meta(layer, wire_r)
    return FCSoft.apply(xt, params, conn, meta)


def logic_layer_forward(layer, x):
    """``LogicLayer.forward`` on ``[B, in]``."""
    require_cuda(x)
    B = x.shape[0]
    return FromFeatureMajor.apply(fc_layer_fm(layer, ToFeatureMajor.apply(x)), B)


def node_forward(node, x, idx):
    """``Node.forward`` on operands flattened to ``[B, out*arity]`` (identity wiring)."""
    from types import SimpleNamespace
    from .connectomes import FixedConnectome
    conn = FixedConnectome.__new__(FixedConnectome)
    torch.nn.Module.__init__(conn)
    conn.cand_i32 = idx.unsqueeze(-1).contiguous()
    fake = SimpleNamespace(node=node, _conn=conn, arity=node.arity, out_dim=node.out_dim,
                           in_dim=x.reshape(x.shape[0], -1).shape[1], training=node.training)
    meta, params, c = _fc_meta(fake)
    B = x.shape[0]
    return FromFeatureMajor.apply(FCSoft.apply(ToFeatureMajor.apply(x), params, c, meta), B)


# ---------------------------------------------------------------- GroupSum
class GroupSumSoft(torch.autograd.Function):
    """Feature-major GroupSum: xt [W, ldb] -> logits [B, C]."""

    @staticmethod
    def forward(ctx, xt, B, C, tau, ste):
        ctx.dims = (xt.shape[0], xt.shape[1], float(tau))
        return op("groupsum_soft_fwd")(xt, B, C, float(tau), int(ste))

    @staticmethod
    def backward(ctx, g):
        W, ldb, tau = ctx.dims
        return op("groupsum_soft_bwd")(g, W, ldb, tau), None, None, None, None


def group_sum_forward(x, num_classes, tau, feature_ste):
    """``GroupSum.forward`` on ``[B, W]``."""
    require_cuda(x)
    B = x.shape[0]
    return GroupSumSoft.apply(ToFeatureMajor.apply(x), B, num_classes, tau, feature_ste)


# ----------------------------------------------------------------- networks
def logic_net_features_fm(net, x):
    B = x.shape[0]
    xt = ToFeatureMajor.apply(x)
    for layer in net.layers:
        wr = net.wire_r if (net.wire_r and layer.in_dim == layer.out_dim) else 0
        xt = fc_layer_fm(layer, xt, wr)
    return xt, B


def logic_net_features(net, x):
    require_cuda(x)
    xt, B = logic_net_features_fm(net, x)
    return FromFeatureMajor.apply(xt, B)


def logic_net_logits(net, x):
    require_cuda(x)
    xt, B = logic_net_features_fm(net, x)
    h = net.head
    return GroupSumSoft.apply(xt, B, h.num_classes, h.tau, h.feature_ste)


# --------------------------------------------------------------- conv tree
CONV_BUILT = {
    "gate16": {(2, 1), (2, 2), (2, 3), (2, 4)},
    "walsh": {(2, 1), (2, 2), (2, 3)},
    "multilinear": {(2, 1), (2, 2), (3, 1), (3, 2), (4, 1), (4, 2), (5, 1), (6, 1)},
    "hybrid": {(2, 1), (2, 2), (3, 1), (3, 2), (4, 1), (4, 2), (5, 1), (6, 1)},
    "linear": {(2, 1), (2, 2), (3, 1), (4, 1), (6, 1)},
}


def _conv_meta(conv, wire_r=0, pool=1):
    kind = conv.node_name
    if kind not in CONV_BUILT or (conv.node_arity, conv.d) not in CONV_BUILT[kind]:
        raise NotImplementedError(f"no soft conv kernel for node={kind!r} arity={conv.node_arity} "
                                  f"depth={conv.d} in silogic_b200")
    if conv.stride != 1:
        raise NotImplementedError("soft conv kernels support stride 1")
    if conv.connect == "fixed":
        src = conv.leaf_idx
        cand = src.unsqueeze(-1).to(torch.int32).contiguous()
        conn, K, ste = None, 1, 0
    else:
        src = conv.leaf_cand
        cand = src.to(torch.int32).contiguous()
        conn, K, ste = conv.conn, conv.k, int(conv.gate_select == "hard")
    if K > 16:
        raise NotImplementedError("soft conv kernels support at most 16 candidates per leaf")
    # checked on the module's own buffer (remembered until it changes), not on the
    # per-call int32 copy, so a step replayed from a CUDA graph never re-checks
    _hard.check_index_range(src, conv.cin * conv.kh * conv.kw, "ConvLogicTree leaf candidates")
    levels = conv.level_params()
    if kind == "gate16":
        params = torch.cat(list(levels), dim=1)                        # [n, nodes, 16]
    else:
        params = torch.cat([p.view(conv.n, -1, p.shape[-1]) for p in levels], dim=1)
    gate_hard = 0
    if kind == "gate16" and conv.training:
        if conv.gate_select == "hard":
            gate_hard = 1
        elif conv.gate_select == "gumbel":
            g = -torch.empty_like(params).exponential_().log()
            params = (params + g) / conv.gumbel_tau
            gate_hard = 1
    inv_tau = 1.0 / conv.tau if kind == "walsh" else 1.0
    meta = dict(cand=cand, K=K, ste=ste, node=NODE_ID[kind], arity=conv.node_arity, depth=conv.d,
                gate_hard=gate_hard, inv_tau=float(inv_tau), kernel=conv.kh, pad=conv.padding,
                n_out=conv.n, wire_r=wire_r, pool=pool)
    return meta, params, conn


#: keep the OR-pool window argmax from the conv forward for the backward (False: the
#: backward re-evaluates every window; same results, more work)
SAVE_POOL_ARGMAX = True


class ConvSoft(torch.autograd.Function):
    """Feature-major conv tree block (+ OR-pool): xt [C*H*W, ldb] -> [n*Hp*Wp, ldb]."""

    @staticmethod
    def _args(meta):
        return (meta["K"], meta["ste"], meta["node"], meta["arity"], meta["depth"],
                meta["gate_hard"], float(meta["inv_tau"]), meta["kernel"], meta["pad"],
                meta["n_out"], meta["wire_r"], meta["pool"])

    @staticmethod
    def forward(ctx, xt, params, conn, meta, shape):
        require_cuda(xt)
        xt = xt.contiguous()
        params = params.float().contiguous()
        connc = conn.float().contiguous() if conn is not None else None
        C, H, W = shape
        # keep each pooled output's window argmax for the backward (1 byte per output)
        # instead of re-evaluating all the window's trees there
        keep = bool(SAVE_POOL_ARGMAX and meta["pool"] > 1 and any(ctx.needs_input_grad[:3]))
        y, arg = op("conv_soft_fwd")(xt, C, H, W, meta["cand"], connc, params,
                                     *ConvSoft._args(meta),
                                   keep)
        ctx.save_for_backward(xt, params, connc, arg)
        ctx.meta, ctx.shape = meta, shape
        return y

    @staticmethod
    def backward(ctx, gy):
        xt, params, connc, arg = ctx.saved_tensors
        m = ctx.meta
        C, H, W = ctx.shape
        if m.get("deterministic") and ctx.needs_input_grad[0]:
            gx, gparams, gconn = conv_soft_bwd_deterministic(xt, (C, H, W), m, params, connc, gy)
            return gx, gparams, gconn, None, None
        gx, gparams, gconn = op("conv_soft_bwd")(xt, C, H, W, m["cand"], connc, params,
                                               *ConvSoft._args(m), gy, arg,
                                               bool(ctx.needs_input_grad[0]))
        return (gx if ctx.needs_input_grad[0] else None, gparams,
                gconn if connc is not None else None, None, None)


def conv_inverse_map(cand, C, kernel, pad, K):
    """For each input channel, the (output channel n, leaf candidate e = l*K + k, tap
    dy - pad, tap dx - pad) rows that read it, ordered by (n, e): CSR offsets [C+1] and
    [nnz, 4] int32 rows on cand's device (the inverse map of ``build_inverse_map``,
    ``silogic/kernels/conv.py:247-265``, extended to Top-K candidates)."""
    N = cand.shape[0]
    flat = cand.reshape(N, -1).long()
    LK = flat.shape[1]
    kk = kernel * kernel
    c = flat // kk
    dy = (flat % kk) // kernel - pad
    dx = flat % kernel - pad
    n_idx = torch.arange(N, device=cand.device).unsqueeze(1).expand(N, LK)
    e_idx = torch.arange(LK, device=cand.device).unsqueeze(0).expand(N, LK)
    key = (c * N + n_idx) * LK + e_idx
    order = torch.argsort(key.reshape(-1))
    rows = torch.stack([n_idx.reshape(-1), e_idx.reshape(-1), dy.reshape(-1), dx.reshape(-1)], 1)
    ent = rows[order].to(torch.int32).contiguous()
    off = torch.zeros(C + 1, dtype=torch.int64, device=cand.device)
    off[1:] = torch.cumsum(torch.bincount(c.reshape(-1), minlength=C), 0)
    return off.to(torch.int32), ent


def conv_soft_bwd_deterministic(xt, shape, m, params, connc, gy):
    """Backward of one pool-1 conv block with a bit-reproducible input gradient
    (``slg_conv_soft_bwd_det``: leaf gradients stored once, then gathered per input
    element in inverse-map order)."""
    from ._lib import call, lib, ptr, stream_ptr
    C, H, W = shape
    if m["pool"] != 1 or m["wire_r"]:
        raise NotImplementedError("the deterministic conv backward covers pool-1 blocks without wire residual")
    ldb = xt.shape[-1]
    gy = gy.contiguous()
    off, ent = conv_inverse_map(m["cand"], C, m["kernel"], m["pad"], m["K"])
    gx = torch.empty_like(xt)
    gparams = torch.empty_like(params)
    gconn = torch.empty_like(connc) if connc is not None else None
    nb = lib().slg_conv_soft_workspace_bytes(H, W, ldb, m["K"], m["node"], m["arity"], m["depth"],
                                             m["kernel"], m["pad"], 1, m["n_out"])
    ws = torch.empty(max(nb, 4) // 4 + 1, dtype=torch.float32, device=xt.device)
    Ho, Wo = H + 2 * m["pad"] - m["kernel"] + 1, W + 2 * m["pad"] - m["kernel"] + 1
    LK = m["cand"][0].numel()
    gleaf = torch.empty(m["n_out"] * LK * Ho * Wo * ldb, dtype=torch.float32, device=xt.device)
    call("slg_conv_soft_bwd_det", ptr(xt), C, H, W, ldb, ptr(m["cand"]), ptr(connc), m["K"],
         m["ste"], m["node"], m["arity"], m["depth"], ptr(params), m["gate_hard"],
         float(m["inv_tau"]), m["kernel"], m["pad"], m["n_out"], ptr(gy), ptr(gx), ptr(gconn),
         ptr(gparams), ptr(off), ptr(ent), ptr(ws), ws.numel() * 4, ptr(gleaf),
         gleaf.numel() * 4, stream_ptr(xt.device))
    return gx, gparams, gconn


def conv_block_fm(conv, xt, shape, wire_r=0, pool=1):
    """One conv block on feature-major ``xt`` ([C*H*W, ldb]); returns (yt, (n, Hp, Wp))."""
    meta, params, conn = _conv_meta(conv, wire_r, pool)
    C, H, W = shape
    Ho = H + 2 * conv.padding - conv.kh + 1
    Wo = W + 2 * conv.padding - conv.kw + 1
    return ConvSoft.apply(xt, params, conn, meta, shape), (conv.n, Ho // pool, Wo // pool)


def logic_conv_net_features_fm(net, x):
    from .layers import OrPool
    B, C, H, W = x.shape
    xt = ToFeatureMajor.apply(x)
    shape = (C, H, W)
    blocks = list(net.blocks)
    for i in range(0, len(blocks), 2):
        conv, pool = blocks[i], blocks[i + 1]
        assert isinstance(pool, OrPool)
        xt, shape = conv_block_fm(conv, xt, shape, net.wire_channels(conv, shape[0]), pool.size)
    for layer in net.head_layers:
        xt = fc_layer_fm(layer, xt)
    return xt, B


def logic_conv_net_features(net, x):
    require_cuda(x)
    xt, B = logic_conv_net_features_fm(net, x)
    return FromFeatureMajor.apply(xt, B)


def logic_conv_net_logits(net, x):
    require_cuda(x)
    xt, B = logic_conv_net_features_fm(net, x)
    h = net.head
    return GroupSumSoft.apply(xt, B, h.num_classes, h.tau, h.feature_ste)


def conv_tree_forward(conv, x, pool=1):
    """``ConvLogicTree.forward`` on ``[B, C, H, W]`` -> ``[B, n, Ho, Wo]``."""
    require_cuda(x)
    B, C, H, W = x.shape
    yt, (n, Hp, Wp) = conv_block_fm(conv, ToFeatureMajor.apply(x), (C, H, W), 0, pool)
    return FromFeatureMajor.apply(yt, B).view(B, n, Hp, Wp)


# ------------------------------------------------------------------ OrPool
class OrPoolSoft(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, size):
        x = x.float().contiguous()
        ctx.save_for_backward(x)
        ctx.size = size
        return op("or_pool_fwd")(x, size)

    @staticmethod
    def backward(ctx, gy):
        (x,) = ctx.saved_tensors
        return op("or_pool_bwd")(x, gy, ctx.size), None


def or_pool(x, size):
    require_cuda(x)
    return OrPoolSoft.apply(x, size)


@torch.no_grad()
def or_pool_hard(x, size):
    require_cuda(x)
    return OrPoolSoft.apply(x.float(), size).to(torch.uint8)


# -------------------------------------------------------------- encoder
class ThermometerSoft(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, thr, scale):
        x = x.float().contiguous()
        thr = thr.float().contiguous()
        ctx.save_for_backward(x, thr)
        ctx.scale = float(scale)
        return op("thermo_soft_fwd")(x, thr)

    @staticmethod
    def backward(ctx, g):
        x, thr = ctx.saved_tensors
        gx, gthr = op("thermo_soft_bwd")(x, thr, g, ctx.scale, bool(ctx.needs_input_grad[0]))
        return (gx if ctx.needs_input_grad[0] else None), gthr, None


def thermometer_forward(x, thresholds, scale):
    require_cuda(x)
    return ThermometerSoft.apply(x, thresholds, scale)


@torch.no_grad()
def thermometer_hard(x, thresholds):
    require_cuda(x)
    B, F = x.shape
    T = thresholds.shape[1]
    h = _hard.thermo_pack(x.view(B, F, 1, 1), thresholds, mode=1)   # [F*T, 1, 1, ldw]
    return _hard.unpack(h.view(F * T, -1), B)
