"""Packed-artefact format: a converted circuit saved to and loaded from one ``.npz`` file,
so inference needs neither the trained model nor its conversion.

The reference keeps a converted net only as live Python objects
(``silogic/bitpacking/convert.py:170-218, 333-402``: wiring ``[out, arity]`` int32 plus a
gate code or a truth table per node); this format stores the same information:

  ``format``            "silogic_b200.packed/1"
  ``in_shape``          ["fc", F] or ["conv", C, ...] (JSON)
  ``num_classes``, ``tau``
  ``step{i}/kind``      "fc" | "conv"; meta JSON (arity, depth, kernel, pad, wire_r,
                        pool, n, in_dim)
  ``step{i}/wiring``    int32 FC wiring ``[out, arity]`` or conv leaves ``[n, leaves]``
                        (leaf = c*k*k + dy*k + dx)
  ``step{i}/tables``    uint64 truth tables, bit p = output at address sum_j in_j << j
                        (FC ``[out]``; conv ``[n, nodes]``, nodes level-major)
  ``head/kind``         "groupsum" | "learned" (+ ``head/weight``, ``head/bias``)

Loading validates every wiring index against the width it reads before the circuit can
run, so a corrupted or hand-edited file is refused instead of becoming out-of-bounds
device reads.
"""
import json

import numpy as np
import torch

FORMAT = "silogic_b200.packed/1"


def save_packed(net, path):
    """Write a :class:`BitpackedNet` / :class:`BitpackedConvNet` to ``path`` (.npz)."""
    from .packed import PackedLearnedHead
    plan = net.plan
    arrays = {"format": np.array(FORMAT), "in_shape": np.array(json.dumps(list(plan.in_shape))),
              "num_classes": np.array(plan.num_classes if plan.num_classes is not None else -1),
              "tau": np.array(float(plan.tau)), "n_steps": np.array(len(plan.steps))}
    for i, st in enumerate(plan.steps):
        key = "idx" if st["op"] == "fc" else "leaf"
        meta = {k: (int(v) if isinstance(v, (int, np.integer)) else v) for k, v in st.items()
                if k not in ("idx", "leaf", "tt", "op")}
        arrays[f"step{i}/kind"] = np.array(st["op"])
        arrays[f"step{i}/meta"] = np.array(json.dumps(meta))
        arrays[f"step{i}/wiring"] = st[key].detach().cpu().numpy().astype(np.int32)
        arrays[f"step{i}/tables"] = st["tt"].detach().cpu().numpy().astype(np.int64).view(np.uint64)
    head = net.head
    if isinstance(head, PackedLearnedHead):
        arrays["head/kind"] = np.array("learned")
        arrays["head/weight"] = head.weight.detach().cpu().numpy().astype(np.float32)
        if head.bias is not None:
            arrays["head/bias"] = head.bias.detach().cpu().numpy().astype(np.float32)
    else:
        arrays["head/kind"] = np.array("groupsum")
    np.savez(path, **arrays)


def load_packed(path, device="cuda"):
    """Read a file written by :func:`save_packed`; returns the bit-packed net on ``device``.
    Raises ``ValueError`` for another format and ``IndexError`` for out-of-range wiring."""
    from .packed import BitpackedConvNet, BitpackedNet, PackedGroupSumHead, PackedLearnedHead
    from .plan import HardPlan, validate_steps
    z = np.load(path, allow_pickle=False)
    if "format" not in z.files or str(z["format"]) != FORMAT:
        raise ValueError(f"{path}: not a {FORMAT} file")
    dev = torch.device(device)
    in_shape = tuple(json.loads(str(z["in_shape"])))
    steps = []
    for i in range(int(z["n_steps"])):
        kind = str(z[f"step{i}/kind"])
        meta = json.loads(str(z[f"step{i}/meta"]))
        wiring = torch.from_numpy(np.ascontiguousarray(z[f"step{i}/wiring"])).to(torch.int32)
        tables = torch.from_numpy(np.ascontiguousarray(z[f"step{i}/tables"]).view(np.int64))
        st = dict(op=kind, tt=tables.to(dev), **meta)
        st["idx" if kind == "fc" else "leaf"] = wiring.to(dev)
        steps.append(st)
    validate_steps(steps, in_shape[1])
    nc = int(z["num_classes"])
    plan = HardPlan(steps, in_shape, nc if nc >= 0 else None, float(z["tau"]))
    if str(z["head/kind"]) == "learned":
        bias = torch.from_numpy(z["head/bias"]) if "head/bias" in z.files else None
        head = PackedLearnedHead(torch.from_numpy(z["head/weight"]), bias).to(dev)
    else:
        head = PackedGroupSumHead(nc, float(z["tau"]))
    cls = BitpackedNet if in_shape[0] == "fc" else BitpackedConvNet
    return cls(plan, head)
