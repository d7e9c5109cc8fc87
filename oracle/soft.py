"""fp32 torch restatement of silogic's soft (relaxed) forward -- TEST ORACLE ONLY.

Gradients come from torch autograd over these plain tensor expressions.  Each
function names the reference lines it restates.  Parameters are passed as a
``{state_dict name: tensor}`` mapping so gradients can be compared by name.
"""
import torch
import torch.nn.functional as F

from .hard import BASIS as _BASIS_NP

BASIS = torch.tensor(_BASIS_NP, dtype=torch.float32)


def _probs(logits, dim, training, gate_select):
    """``gate_probs`` (``functional.py:144-163``), softmax / hard-STE only."""
    soft = F.softmax(logits, dim=dim)
    if training and gate_select == "hard":
        hard = torch.zeros_like(soft).scatter_(dim, soft.argmax(dim=dim, keepdim=True), 1.0)
        return soft + (hard - soft).detach()
    if training and gate_select == "gumbel":
        raise NotImplementedError("gumbel selection is random; no oracle")
    return soft


def _corners(n):
    return torch.tensor([[(p >> j) & 1 for j in range(n)] for p in range(2 ** n)],
                        dtype=torch.float32)


def _walsh_mono(u):
    """``walsh_monomials`` (``functional.py:176-185``) on ``[..., n]``."""
    phi = torch.ones(u.shape[:-1] + (1,), dtype=u.dtype)
    for j in range(u.shape[-1]):
        phi = torch.cat([phi, phi * u[..., j:j + 1]], dim=-1)
    return phi


def _multilinear(a, logits):
    """``MultilinearNode._f`` (``nodes.py:174-178``): a ``[..., out, n]``."""
    n = a.shape[-1]
    c = _corners(n)                                            # [P, n]
    au = a.unsqueeze(-2)                                       # [..., out, 1, n]
    prod = (c * au + (1 - c) * (1 - au)).prod(-1)              # [..., out, P]
    return (prod * torch.sigmoid(logits)).sum(-1)


def node_soft(node, params, ops, training, gate_select, node_tau=1.0, mono_mask=None):
    """Node relaxations on operands ``[B, out, arity]`` (``nodes.py:86-272``)."""
    if node == "gate16":
        c = _probs(params, -1, training, gate_select) @ BASIS   # nodes.py:82-90
        a, b = ops[..., 0], ops[..., 1]
        return c[:, 0] + c[:, 1] * a + c[:, 2] * b + c[:, 3] * (a * b)
    if node == "walsh":
        z = (_walsh_mono(2 * ops - 1) * params).sum(-1)          # nodes.py:145-150
        return torch.sigmoid(z * (1.0 / node_tau))
    if node == "multilinear":
        return _multilinear(ops, params)
    if node == "hybrid":                                          # nodes.py:198-207
        f_soft = _multilinear(ops, params)
        with torch.no_grad():
            f_disc = _multilinear((ops >= 0.5).float(), params)
        return f_disc + f_soft - f_soft.detach()
    if node == "linear":                                          # nodes.py:222-227
        return torch.sigmoid(params[:, 0] + torch.einsum("boa,oa->bo", ops, params[:, 1:]))
    if node == "polynomial":                                      # nodes.py:256-264
        mk = mono_mask
        mono = (ops.unsqueeze(-2) * mk + (1 - mk)).prod(-1)
        return torch.sigmoid((mono * params).sum(-1))
    raise ValueError(node)


def fc_layer(L, P, x, training=True):
    """``LogicLayer.forward`` on the PyTorch path (``layers.py:125-129``)."""
    pre = L["prefix"]
    if L["conn"] == "fixed":
        ops = x[:, torch.as_tensor(L["idx"])]                     # connectomes.py:58-59
    elif L["conn"] == "topk":
        conn = P[pre + "_conn.conn"]
        w = F.softmax(conn, dim=2)                                # connectomes.py:114-118
        if L.get("ste"):
            hard = F.one_hot(conn.argmax(dim=2), w.shape[-1]).to(w.dtype)
            w = hard + w - w.detach()
        g = x[:, torch.as_tensor(L["cand"])]                      # [B, out, a, k]
        ops = torch.einsum("boak,oak->boa", g, w)
    else:
        ops = torch.einsum("bi,oai->boa", x, F.softmax(P[pre + "_conn.conn"], dim=2))
    pname = {"gate16": "gate_logits", "walsh": "theta", "multilinear": "logits",
             "hybrid": "logits", "linear": "theta", "polynomial": "theta"}[L["node"]]
    mm = torch.as_tensor(L["mono_mask"]) if "mono_mask" in L else None
    return node_soft(L["node"], P[pre + "node." + pname], ops, training,
                     L["gate_select"], L["node_tau"], mm)


def conv_block(Bk, P, x, training=True):
    """``ConvLogicTree.forward`` PyTorch path (``layers.py:375-485``), no pool."""
    pre = Bk["prefix"]
    B, C, H, W = x.shape
    kz, pad = Bk["kernel"], Bk["pad"]
    Ho, Wo = H + 2 * pad - kz + 1, W + 2 * pad - kz + 1
    patches = F.unfold(x, (kz, kz), padding=pad)                  # [B, C*k*k, L]
    n, nl = Bk["n"], Bk["leaves"]
    if Bk["connect"] == "fixed":
        idx = torch.as_tensor(Bk["leaf_idx"]).reshape(-1)
        leaves = patches[:, idx, :].view(B, n, nl, -1)
    else:
        conn = P[pre + "conn"]
        w = F.softmax(conn, dim=2)                                # layers.py:487-497
        if Bk["gate_select"] == "hard":
            hard = F.one_hot(conn.argmax(dim=2), w.shape[-1]).to(w.dtype)
            w = hard + w - w.detach()
        K = conn.shape[2]
        g = patches[:, torch.as_tensor(Bk["leaf_cand"]).reshape(-1), :].view(B, n, nl, K, -1)
        leaves = torch.einsum("bnlkL,nlk->bnlL", g, w)
    vals = leaves
    if Bk["node"] == "gate16":                                    # layers.py:388-401
        for i in range(Bk["depth"]):
            p = _probs(P[pre + f"gate_logits.{i}"], 2, training, Bk["gate_select"])
            c = (p @ BASIS).unsqueeze(0).unsqueeze(-1)
            a, b = vals[:, :, 0::2, :], vals[:, :, 1::2, :]
            vals = c[:, :, :, 0] + c[:, :, :, 1] * a + c[:, :, :, 2] * b + c[:, :, :, 3] * (a * b)
    else:                                                         # layers.py:432-446
        k = Bk["node_arity"]
        pname = {"walsh": "theta", "multilinear": "logits", "hybrid": "logits",
                 "linear": "theta", "polynomial": "theta"}[Bk["node"]]
        mm = torch.as_tensor(Bk["mono_mask"], dtype=torch.float32) if "mono_mask" in Bk else None
        for i in range(Bk["depth"]):
            nn_, km, L = vals.shape[1], vals.shape[2], vals.shape[3]
            m = km // k
            ops = vals.view(B, nn_, m, k, L).permute(0, 4, 1, 2, 3).reshape(B * L, nn_ * m, k)
            out = node_soft(Bk["node"], P[pre + f"tree_nodes.{i}.{pname}"], ops, training,
                            Bk["gate_select"], Bk["node_tau"], mm)
            vals = out.view(B, L, nn_, m).permute(0, 2, 3, 1)
    return vals[:, :, 0, :].reshape(B, n, Ho, Wo)


def group_sum(x, num_classes, tau):
    """``GroupSum.forward`` with ``feature_ste=True`` (``heads.py:34-39``)."""
    x = (x > 0.5).float() + (x - x.detach())
    B, Wd = x.shape
    return x.view(B, num_classes, Wd // num_classes).sum(dim=2) / tau


def _pool_at(y, idx):
    """2x2 pooling that takes the value at given flat window indices (into H*W)."""
    B, n, H, W = y.shape
    return y.reshape(B, n, H * W).gather(2, idx.reshape(B, n, -1)).view(idx.shape)


def net_features(spec, P, x, training=True, pool_index=None):
    """``model._run(x, hard=False)``: activations entering the head.

    ``pool_index`` (optional, one LongTensor ``[B, n, Hp, Wp]`` per block) fixes
    which window element each OR-pool output takes; by default the routing is
    ``F.max_pool2d``'s.  Tests use it to replay another implementation's choice
    at windows whose values tie to within fp32 rounding."""
    if spec["type"] == "fc":
        for L in spec["layers"]:
            y = fc_layer(L, P, x, training)
            if spec["wire_r"] and x.shape[1] == y.shape[1]:
                y = torch.cat([x[:, :spec["wire_r"]], y[:, spec["wire_r"]:]], dim=1)
            x = y
        return x
    for Bk in spec["blocks"]:
        y = conv_block(Bk, P, x, training)
        if spec["wire_residual"] > 0:
            r = min(int(Bk["n"] * spec["wire_residual"]), x.shape[1])
            if r > 0:
                y = torch.cat([x[:, :r], y[:, r:]], dim=1)
        if pool_index is None:
            x = F.max_pool2d(y, 2, 2)                             # layers.py:558-559
        else:
            x = _pool_at(y, pool_index[spec["blocks"].index(Bk)])
    x = x.flatten(1)
    for L in spec["head"]:
        x = fc_layer(L, P, x, training)
    return x


def net_logits(spec, P, x, training=True):
    return group_sum(net_features(spec, P, x, training), spec["num_classes"], spec["tau"])


def learned_thermometer(x, thresholds, scale=10.0):
    """``LearnedThermometerEncoder.forward`` (``encoders.py:39-44``)."""
    d = x.unsqueeze(-1) - thresholds[None]
    hard = (d > 0).float()
    soft = torch.sigmoid(d * scale)
    return (hard + soft - soft.detach()).reshape(x.shape[0], -1)


def params_from_sd(sd, requires_grad=True):
    """state_dict (numpy or torch) -> float leaf tensors for the learnable entries."""
    P = {}
    for k, v in sd.items():
        t = torch.as_tensor(v).clone()
        if t.dtype == torch.float32 and requires_grad:
            t.requires_grad_(True)
        P[k] = t
    return P
