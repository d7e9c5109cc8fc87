"""numpy restatement of silogic's bit-packed hard circuit -- TEST ORACLE ONLY.

Layout (``silogic/bitpacking/ops.py:1-10``): activations are ``uint64``
``[dim, nw]`` with ``nw = ceil(B/64)``; sample ``b`` is bit ``b % 64`` of word
``b // 64``.  Conv activations keep the spatial axes: ``[C, H, W, nw]``
(``packed_layer.py:183-209`` uses ``[C, H*W, nw]``, the same memory order).

Truth tables use the LUT address convention ``addr = sum_j bit_j << j`` (slot 0
is the least significant bit, ``nodes.py:184-189``); gate16 nodes are mapped into
it from their own address ``(a << 1) | b`` (``nodes.py:101-106``).
"""
import numpy as np

from .spec import net_spec

# silogic/functional.py:24-44 -- row g = coefficients of 1, a, b, a*b for gate g.
BASIS = np.array([
    [0, 0, 0, 0], [0, 0, 0, 1], [0, 1, 0, -1], [0, 1, 0, 0],
    [0, 0, 1, -1], [0, 0, 1, 0], [0, 1, 1, -2], [0, 1, 1, -1],
    [1, -1, -1, 1], [1, -1, -1, 2], [1, 0, -1, 0], [1, 0, -1, 1],
    [1, -1, 0, 0], [1, -1, 0, 1], [1, 0, 0, -1], [1, 0, 0, 0]], dtype=np.int64)

# gate16 truth tables, column (a<<1)|b  (functional.py:50-69)
GATE_TT = np.stack([BASIS[:, 0], BASIS[:, 0] + BASIS[:, 2], BASIS[:, 0] + BASIS[:, 1],
                    BASIS.sum(1)], axis=1).astype(np.uint8)

ALL = np.uint64(0xFFFFFFFFFFFFFFFF)


def n_words(B):
    """``ops.py:27-29``."""
    return (B + 63) >> 6


def pack_bits(x):
    """``[B, dim]`` {0,1} -> ``[dim, nw]`` uint64, little-endian (``ops.py:32-49``)."""
    x = np.asarray(x)
    B, dim = x.shape
    nw = n_words(B)
    buf = np.zeros((nw * 64, dim), dtype=np.uint8)
    buf[:B] = (x != 0)
    packed = np.packbits(np.ascontiguousarray(buf.T), axis=1, bitorder="little")
    return np.ascontiguousarray(packed).view(np.uint64)


def unpack_bits(p, B):
    """``[dim, nw]`` uint64 -> ``[B, dim]`` uint8 (``ops.py:52-63``)."""
    p = np.ascontiguousarray(p).view(np.uint8)
    bits = np.unpackbits(p, axis=1, bitorder="little")
    return np.ascontiguousarray(bits[:, :B].T)


def mask_last_word(p, B):
    """Zero padding samples in the last word (``ops.py:107-115``)."""
    r = B % 64
    if r:
        p[..., -1] &= np.uint64((1 << r) - 1)
    return p


def group_sum_counts(p, B, num_classes):
    """Integer GroupSum counts ``[B, C]`` (``ops.py:66-104`` without the /tau)."""
    dim = p.shape[0]
    gs = dim // num_classes
    out = np.empty((B, num_classes), dtype=np.int64)
    for c in range(num_classes):
        out[:, c] = unpack_bits(p[c * gs:(c + 1) * gs], B).sum(axis=1, dtype=np.int64)
    return out


# ---------------------------------------------------------------------------
# truth tables (restating convert.py:78-138 and the nodes' forward_hard)
# ---------------------------------------------------------------------------
def _corner_bits(n):
    return np.array([[(p >> j) & 1 for j in range(n)] for p in range(2 ** n)], dtype=np.int64)


def node_truth_tables(node, params, arity, mono_mask=None):
    """``[out, 2**arity]`` bool truth tables in the LUT address convention."""
    P = 2 ** arity
    cb = _corner_bits(arity)                                  # [P, n]
    if node == "gate16":
        g = np.argmax(params, axis=1)                         # nodes.py:103 (first max)
        a, b = cb[:, 0], cb[:, 1]
        return GATE_TT[g][:, (a << 1) | b].astype(bool)
    if node in ("multilinear", "hybrid"):
        return params > 0                                     # nodes.py:188
    if node == "walsh":
        # z = sum_M theta_M prod_{j in M} (2 bit_j - 1) > 0 in fp32, monomials added in
        # index order as the reference's forward_hard sums them (nodes.py:153-156;
        # walsh_monomials column order, functional.py:176-185); the arity-2 bit-packed
        # conversion (convert.py:84-97) adds the same fp32 terms in the same order.
        u = (2 * cb - 1).astype(np.float32)                   # [P, n]
        mono = np.ones((P, P), dtype=np.float32)
        for m in range(P):
            for j in range(arity):
                if (m >> j) & 1:
                    mono[:, m] *= u[:, j]
        th = params.astype(np.float32)
        z = np.zeros((th.shape[0], P), dtype=np.float32)
        for m in range(P):
            z = z + th[:, m:m + 1] * mono[None, :, m]
        return z > 0
    if node == "linear":
        # fp32: bias + sum_j theta_j a_j, inputs added in slot order (nodes.py:225-233)
        th = params.astype(np.float32)
        cbf = cb.astype(np.float32)
        z = np.repeat(th[:, :1], P, axis=1)
        for j in range(arity):
            z = z + th[:, 1 + j:2 + j] * cbf[None, :, j]
        return z >= 0
    if node == "polynomial":
        # fp32 sum over the monomials in mask-row order (nodes.py:256-268)
        mk = np.asarray(mono_mask, dtype=np.float32)          # [M, n]
        mono = np.prod(np.where(mk[None] > 0, cb[:, None, :], 1), axis=2).astype(np.float32)
        th = params.astype(np.float32)
        z = np.zeros((th.shape[0], P), dtype=np.float32)
        for m in range(mono.shape[1]):
            z = z + th[:, m:m + 1] * mono[None, :, m]
        return z >= 0
    raise ValueError(node)


def fc_hard_spec(L):
    """Hard wiring ``[out, arity]`` + truth tables of one FC layer (convert.py:170-218)."""
    if L["conn"] == "fixed":
        idx = L["idx"]
    elif L["conn"] == "topk":
        sel = np.argmax(L["conn_logits"], axis=2)             # connectomes.py:130
        idx = np.take_along_axis(L["cand"], sel[..., None], 2)[..., 0]
    else:
        idx = np.argmax(L["dense_logits"], axis=2)
    tt = node_truth_tables(L["node"], L["params"], L["arity"], L.get("mono_mask"))
    return idx.astype(np.int64), tt


def eval_lut(operands, tt):
    """Evaluate ``[out, P]`` truth tables on packed operands (list of ``[out, ...]``).

    Sum-of-products over the active entries of each table, the evaluation order of
    ``BitpackedLUTLayer`` (``packed_layer.py:158-178``); for arity 2 this equals the
    gate-grouped form of ``BitpackedFCLayer`` (``packed_layer.py:85-116``).
    """
    arity = len(operands)
    out = np.zeros_like(operands[0])
    for p in range(2 ** arity):
        rows = np.nonzero(tt[:, p])[0]
        if rows.size == 0:
            continue
        m = np.full((rows.size,) + operands[0].shape[1:], ALL, dtype=np.uint64)
        for j in range(arity):
            v = operands[j][rows]
            m &= v if (p >> j) & 1 else ~v
        out[rows] |= m
    return out


# the 16 two-input functions by LUT code (bit p = output at a = p & 1, b = p >> 1),
# as single numpy bitwise expressions (packed_layer.py:85-116, ops.py:123-140)
_GATE2 = {
    0b0000: lambda a, b: np.zeros_like(a), 0b1000: lambda a, b: a & b,
    0b0010: lambda a, b: a & ~b, 0b1010: lambda a, b: a.copy(),
    0b0100: lambda a, b: ~a & b, 0b1100: lambda a, b: b.copy(),
    0b0110: lambda a, b: a ^ b, 0b1110: lambda a, b: a | b,
    0b0001: lambda a, b: ~(a | b), 0b1001: lambda a, b: ~(a ^ b),
    0b0101: lambda a, b: ~a, 0b1101: lambda a, b: ~a | b,
    0b0011: lambda a, b: ~b, 0b1011: lambda a, b: a | ~b,
    0b0111: lambda a, b: ~(a & b), 0b1111: lambda a, b: np.full_like(a, ALL),
}


def fc_forward_gate2(x, idx, tt):
    """Arity-2 layer, outputs grouped by gate so each group is one bitwise op."""
    code = (tt.astype(np.int64) << np.arange(4)).sum(1)
    out = np.empty((idx.shape[0], x.shape[1]), dtype=np.uint64)
    for c in np.unique(code):
        rows = np.nonzero(code == c)[0]
        out[rows] = _GATE2[int(c)](x[idx[rows, 0]], x[idx[rows, 1]])
    return out


def fc_forward(x, idx, tt, wire_r=0):
    """One FC layer on ``[in, nw]`` packed input."""
    if idx.shape[1] == 2:
        y = fc_forward_gate2(x, idx, tt)
    else:
        y = eval_lut([x[idx[:, j]] for j in range(idx.shape[1])], tt)
    if wire_r and x.shape[0] == y.shape[0]:                   # models.py:91-92
        y[:wire_r] = x[:wire_r]
    return y


def conv_hard_spec(Bk):
    """Hard leaves ``[n, leaves]`` + per-level truth tables ``[n, nodes, P]``."""
    if Bk["connect"] == "fixed":
        leaf = Bk["leaf_idx"]
    else:
        sel = np.argmax(Bk["conn_logits"], axis=2)
        leaf = np.take_along_axis(Bk["leaf_cand"], sel[..., None], 2)[..., 0]
    n, k = Bk["n"], Bk["node_arity"]
    tts = []
    for i, lv in enumerate(Bk["levels"]):
        nodes = k ** (Bk["depth"] - 1 - i)
        if Bk["node"] == "gate16":
            t = node_truth_tables("gate16", lv.reshape(n * nodes, 16), 2)
        else:
            t = node_truth_tables(Bk["node"], lv, k, Bk.get("mono_mask"))
        tts.append(t.reshape(n, nodes, 2 ** k))
    return leaf.astype(np.int64), tts


def conv_forward(x4, leaf, tts, node_arity, kernel=3, pad=1, wire_r=0, pool=2):
    """One conv tree block + OR-pool on ``[C, H, W, nw]`` (layers.py:515-541,560-563)."""
    C, H, W, nw = x4.shape
    n = leaf.shape[0]
    xp = np.zeros((C, H + 2 * pad, W + 2 * pad, nw), dtype=np.uint64)
    xp[:, pad:pad + H, pad:pad + W] = x4
    Ho, Wo = H + 2 * pad - kernel + 1, W + 2 * pad - kernel + 1
    kk = kernel * kernel
    vals = []
    for l in range(leaf.shape[1]):
        r = leaf[:, l]
        c, dy, dx = r // kk, (r % kk) // kernel, r % kernel
        yy = np.arange(Ho)[None, :, None] + dy[:, None, None]
        xx = np.arange(Wo)[None, None, :] + dx[:, None, None]
        vals.append(xp[c[:, None, None], yy, xx])              # [n, Ho, Wo, nw]
    k = node_arity
    for t in tts:                                              # level 0 first
        nxt = []
        for m in range(t.shape[1]):
            nxt.append(eval_lut(vals[m * k:(m + 1) * k], t[:, m]))
        vals = nxt
    y = vals[0]
    if wire_r:
        y[:wire_r] = x4[:wire_r, :Ho, :Wo]                     # models.py:254-258
    if pool > 1:
        Hp, Wp = Ho // pool, Wo // pool
        z = np.zeros((n, Hp, Wp, nw), dtype=np.uint64)
        for py in range(pool):
            for px in range(pool):
                z |= y[:, py:Hp * pool:pool, px:Wp * pool:pool]
        y = z
    return y


def net_counts(spec, x):
    """Integer GroupSum counts of ``forward_hard`` (float dtype in the reference)."""
    x = np.asarray(x)
    B = x.shape[0]
    if spec["type"] == "fc":
        h = pack_bits(x.reshape(B, -1))
        for L in spec["layers"]:
            idx, tt = fc_hard_spec(L)
            h = fc_forward(h, idx, tt, spec["wire_r"])
    else:
        Bn, C, H, W = x.shape
        h = pack_bits(x.reshape(B, -1)).reshape(C, H, W, -1)
        for Bk in spec["blocks"]:
            leaf, tts = conv_hard_spec(Bk)
            r = min(int(Bk["n"] * spec["wire_residual"]), h.shape[0]) \
                if spec["wire_residual"] > 0 else 0
            h = conv_forward(h, leaf, tts, Bk["node_arity"], Bk["kernel"], Bk["pad"], r)
        h = h.reshape(-1, h.shape[-1])
        for L in spec["head"]:
            idx, tt = fc_hard_spec(L)
            h = fc_forward(h, idx, tt)
    h = mask_last_word(h, B)
    return group_sum_counts(h, B, spec["num_classes"])


def thermometer_bits(img, thresholds):
    """``binarize_spatial`` (``silogic/data.py:75-92``): ``x >= f32(t)``, channel t*C+c."""
    img = np.asarray(img, dtype=np.float32)
    return np.concatenate([(img >= np.float32(t)).astype(np.uint8) for t in thresholds], 1)


def learned_thermometer_bits(x, thresholds):
    """``LearnedThermometerEncoder.forward_hard`` (``encoders.py:46-50``): ``x - t > 0``."""
    d = np.asarray(x, np.float32)[..., None] - np.asarray(thresholds, np.float32)[None]
    return (d > 0).astype(np.uint8).reshape(x.shape[0], -1)


def model_counts(ctor, kwargs, sd, x):
    return net_counts(net_spec(ctor, kwargs, sd), x)
