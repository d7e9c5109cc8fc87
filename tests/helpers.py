"""Shared test helpers: rebuild golden-fixture models with silogic_b200 classes."""
import glob
import json
import os

import numpy as np
import torch

from conftest import GOLDEN

FIXTURES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "*.npz"))
                  if not p.endswith("prims.npz"))
SEEDS = {}   # fixture name -> torch.manual_seed used before construction in make_golden.py
_fc = ["fc_gate16_fixed", "fc_gate16_topk", "fc_gate16_topk_hardsel", "fc_walsh_topk",
       "fc_walsh_fixed_a3", "fc_multilinear_a2_ste", "fc_multilinear_a6", "fc_hybrid_a4",
       "fc_hybrid_a3_fixed"]
_conv = ["conv_gate16_topk_d2", "conv_gate16_fixed_d2", "conv_gate16_topk_d3_wire",
         "conv_hybrid_a4_d1"]
SEEDS.update({n: 100 + i for i, n in enumerate(_fc)})
SEEDS.update({n: 400 + i for i, n in enumerate(_conv)})
SEEDS["conv_multilinear_a6_enc"] = 450
_cont = ["conv_cont_gate16_topk_d2", "conv_cont_gate16_fixed_d1", "conv_cont_walsh_k8_d2",
         "conv_cont_multilinear_a3_d1"]
SEEDS.update({n: 700 + i for i, n in enumerate(_cont)})


def hard_input(z):
    """The binary input of the hard path: ``x_hard`` where the soft input is continuous."""
    return z["x_hard"] if "x_hard" in z.files else z["x"]


def load(name):
    return np.load(os.path.join(GOLDEN, name + ".npz"))


def build_model(name, device="cpu", seed_like_golden=True):
    """Construct the fixture's network with silogic_b200 and load its state_dict."""
    import silogic_b200 as S
    z = load(name)
    ctor, kw = str(z["ctor"]), json.loads(str(z["kwargs"]))
    if seed_like_golden:
        torch.manual_seed(SEEDS[name])
    m = getattr(S, ctor)(**kw)
    sd = {k[3:]: torch.from_numpy(z[k]) for k in z.files if k.startswith("sd/")}
    fresh = {k: v.clone() for k, v in m.state_dict().items()}
    m.load_state_dict(sd)
    enc = None
    if "enc_kwargs" in z.files:
        enc = S.LearnedThermometerEncoder(**json.loads(str(z["enc_kwargs"])))
        enc.load_state_dict({"thresholds": torch.from_numpy(z["encsd/thresholds"])})
        enc = enc.to(device)
    return m.to(device), enc, z, fresh


def encoder_image(enc_out, z):
    B, C, H, W = [int(v) for v in z["img_shape"]]
    bits = enc_out.shape[1] // (C * H * W)
    return enc_out.view(B, C, H, W, bits).permute(0, 1, 4, 2, 3).reshape(B, C * bits, H, W)
