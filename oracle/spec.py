"""Constructor call + state_dict -> plain per-layer description (test oracle only).

Follows the constructor defaults and parameter layouts of the reference:
``LogicNet`` (``silogic/models.py:23-104``), ``LogicConvNet``/``LogicTreeNet``
(``silogic/models.py:153-293``), ``LogicLayer`` (``silogic/layers.py:20-135``),
``ConvLogicTree`` (``silogic/layers.py:226-541``) and the alias tables in
``silogic/nodes.py:29-35`` and ``silogic/connectomes.py:26-31``.
"""
import json

import numpy as np

NODE_ALIASES = {"gate16": "gate16", "gate": "gate16", "walsh": "walsh",
                "multilinear": "multilinear", "probabilistic": "multilinear",
                "hybrid": "hybrid", "linear": "linear", "polynomial": "polynomial"}
CONN_ALIASES = {"f": "fixed", "fixed": "fixed", "l": "dense", "dense": "dense",
                "topk": "topk", "blocktopk": "topk"}


def _per_layer(v, i):
    return v[i] if isinstance(v, (list, tuple)) else v


def _np(sd, key):
    v = sd[key]
    return v.detach().cpu().numpy() if hasattr(v, "detach") else np.asarray(v)


def fc_layer_spec(sd, prefix, in_dim, out_dim, node, connectome, arity, k,
                  gate_select="softmax", node_tau=1.0):
    """One ``LogicLayer`` (``silogic/layers.py:46-76``)."""
    node = NODE_ALIASES[str(node).lower()]
    if node == "gate16":
        arity = 2
    conn = CONN_ALIASES[str(connectome).lower()]
    L = dict(kind="fc", prefix=prefix, k=k, in_dim=in_dim, out_dim=out_dim, node=node, arity=arity,
             conn=conn, gate_select=gate_select, node_tau=float(node_tau))
    if conn == "fixed":
        L["idx"] = _np(sd, prefix + "_conn.idx").astype(np.int64)
    elif conn == "topk":
        L["cand"] = _np(sd, prefix + "_conn.cand").astype(np.int64)
        L["conn_logits"] = _np(sd, prefix + "_conn.conn").astype(np.float32)
        L["ste"] = gate_select == "hard"       # layers.py:68-69
    else:
        L["dense_logits"] = _np(sd, prefix + "_conn.conn").astype(np.float32)
    pname = {"gate16": "gate_logits", "walsh": "theta", "multilinear": "logits",
             "hybrid": "logits", "linear": "theta", "polynomial": "theta"}[node]
    L["params"] = _np(sd, prefix + "node." + pname).astype(np.float32)
    if node == "polynomial":
        L["mono_mask"] = _np(sd, prefix + "node.mono_mask").astype(np.float32)
    return L


def conv_block_spec(sd, prefix, cin, n, kernel, tree_depth, connect, k, node,
                    arity, gate_select, node_tau):
    """One ``ConvLogicTree`` (``silogic/layers.py:279-365``)."""
    node = NODE_ALIASES[str(node).lower()]
    node_arity = 2 if node in ("gate16", "walsh") else arity
    depth = tree_depth if tree_depth is not None else (2 if node_arity == 2 else 1)
    B = dict(kind="conv", prefix=prefix, cin=cin, n=n, kernel=kernel, pad=kernel // 2, stride=1,
             node=node, node_arity=node_arity, depth=depth, connect=connect,
             leaves=node_arity ** depth, gate_select=gate_select,
             node_tau=float(node_tau))
    if connect == "fixed":
        B["leaf_idx"] = _np(sd, prefix + "leaf_idx").astype(np.int64)
    else:
        B["leaf_cand"] = _np(sd, prefix + "leaf_cand").astype(np.int64)
        B["conn_logits"] = _np(sd, prefix + "conn").astype(np.float32)
    if node == "gate16":
        B["levels"] = [_np(sd, prefix + f"gate_logits.{i}").astype(np.float32)
                       for i in range(depth)]                  # [n, nodes, 16]
    else:
        pname = {"walsh": "theta", "multilinear": "logits", "hybrid": "logits",
                 "linear": "theta", "polynomial": "theta"}[node]
        B["levels"] = [_np(sd, prefix + f"tree_nodes.{i}.{pname}").astype(np.float32)
                       for i in range(depth)]                  # [n*nodes, P]
        if node == "polynomial":
            B["mono_mask"] = _np(sd, prefix + "tree_nodes.0.mono_mask")
    return B


def net_spec(ctor, kwargs, sd):
    """Describe a ``LogicNet`` / ``LogicConvNet`` / ``LogicTreeNet`` call."""
    if isinstance(kwargs, str):
        kwargs = json.loads(kwargs)
    kw = dict(kwargs)
    if ctor == "LogicNet":
        d = dict(num_classes=10, node="gate16", connectome="topk", arity=2, k=8,
                 tau=1.0, node_tau=1.0, wire_residual=0.0, gate_select="softmax")
        d.update(kw)
        layers, d_in = [], d["in_dim"]
        for i in range(d["depth"]):
            layers.append(fc_layer_spec(
                sd, f"layers.{i}.", d_in, d["width"], _per_layer(d["node"], i),
                d["connectome"], d["arity"], d["k"],
                _per_layer(d["gate_select"], i), d["node_tau"]))
            d_in = d["width"]
        return dict(type="fc", layers=layers, wire_r=int(d["width"] * d["wire_residual"]),
                    num_classes=d["num_classes"], tau=float(d["tau"]))
    if ctor in ("LogicConvNet", "LogicTreeNet"):
        d = dict(head_width=None, num_classes=10, tree_depth=None, kernel=3,
                 connect="topk", k=4, head_connect="topk", head_k=8, head_depth=2,
                 n_chan=2, tau=100.0, wire_residual=0.0, head_widths=None,
                 node="gate16", arity=2, node_tau=1.0, gate_select="softmax")
        d.update(kw)
        blocks, c, hw = [], d["in_channels"], d["in_hw"]
        for i, n in enumerate(d["channels"]):
            blocks.append(conv_block_spec(
                sd, f"blocks.{2 * i}.", c, n, d["kernel"], d["tree_depth"],
                d["connect"], d["k"], d["node"], d["arity"], d["gate_select"],
                d["node_tau"]))
            c, hw = n, hw // 2
        widths = d["head_widths"] or [d["head_width"]] * d["head_depth"]
        head, d_in = [], c * hw * hw
        for j, w in enumerate(widths):
            head.append(fc_layer_spec(sd, f"head_layers.{j}.", d_in, w, d["node"],
                                      d["head_connect"], 2, d["head_k"],
                                      d["gate_select"], 1.0))
            d_in = w
        return dict(type="conv", blocks=blocks, head=head, in_hw=d["in_hw"],
                    wire_residual=float(d["wire_residual"]),
                    num_classes=d["num_classes"], tau=float(d["tau"]))
    raise ValueError(f"unknown constructor {ctor!r}")


def load_fixture(path):
    """Read a golden ``.npz`` into (ctor, kwargs dict, state_dict of numpy arrays, raw)."""
    z = np.load(path)
    sd = {k[3:]: z[k] for k in z.files if k.startswith("sd/")}
    return str(z["ctor"]), json.loads(str(z["kwargs"])), sd, z
