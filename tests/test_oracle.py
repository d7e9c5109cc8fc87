"""Pin the CPU oracle against golden vectors produced by the reference itself."""
import glob
import json
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import hard as H
from oracle import soft as S
from oracle.spec import load_fixture, net_spec

CASES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "*.npz"))
               if not p.endswith("prims.npz"))


def _encode(z, x):
    """Apply the learned thermometer encoder of an encoder case ([B,F] -> image)."""
    ekw = json.loads(str(z["enc_kwargs"]))
    B, C, Hh, W = [int(v) for v in z["img_shape"]]
    return ekw["bits"], (B, C, Hh, W)


def _img(enc, shape, bits):
    B, C, Hh, W = shape
    return enc.view(B, C, Hh, W, bits).permute(0, 1, 4, 2, 3).reshape(B, C * bits, Hh, W)


@pytest.mark.parametrize("case", CASES)
def test_oracle_hard_counts_match_reference(case):
    ctor, kw, sd, z = load_fixture(os.path.join(GOLDEN, case + ".npz"))
    spec = net_spec(ctor, kw, sd)
    x = z["x_hard"] if "x_hard" in z.files else z["x"]
    if "enc_kwargs" in z.files:
        bits, shape = _encode(z, x)
        e = H.learned_thermometer_bits(x, z["encsd/thresholds"])
        x = _img(torch.from_numpy(e), shape, bits).numpy()
    counts = H.net_counts(spec, x.astype(np.uint8))
    np.testing.assert_array_equal(counts, z["hard"].astype(np.int64))


@pytest.mark.parametrize("case", CASES)
def test_oracle_soft_matches_reference(case):
    ctor, kw, sd, z = load_fixture(os.path.join(GOLDEN, case + ".npz"))
    spec = net_spec(ctor, kw, sd)
    P = S.params_from_sd(sd)
    x = torch.from_numpy(z["x"]).clone().requires_grad_(True)
    xs = x
    if "enc_kwargs" in z.files:
        bits, shape = _encode(z, x)
        thr = torch.from_numpy(z["encsd/thresholds"]).clone().requires_grad_(True)
        xs = _img(S.learned_thermometer(x, thr), shape, bits)
    feat = S.net_features(spec, P, xs, training=True)
    logits = S.group_sum(feat, spec["num_classes"], spec["tau"])
    (logits * torch.from_numpy(z["rmat"])).sum().backward()
    np.testing.assert_allclose(feat.detach().numpy(), z["feat"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(logits.detach().numpy(), z["logits"], rtol=1e-5, atol=1e-6)
    for k in z.files:
        if not k.startswith("grad/"):
            continue
        name = k[5:]
        got = x.grad if name == "x" else P[name].grad
        ref = z[k]
        tol = 1e-5 * (np.abs(ref) + np.abs(ref).max())
        assert np.all(np.abs(got.numpy() - ref) <= tol + 1e-7), f"{case}: grad {name}"


def test_oracle_primitives_match_reference():
    z = np.load(os.path.join(GOLDEN, "prims.npz"))
    for B, F in [(1, 1), (63, 8), (64, 64), (65, 256), (200, 784)]:
        x = z[f"pack_{B}_{F}/x"]
        p = H.pack_bits(x)
        np.testing.assert_array_equal(p.view(np.int64), z[f"pack_{B}_{F}/packed"])
        np.testing.assert_array_equal(H.unpack_bits(p, B), x)
    c = H.group_sum_counts(H.pack_bits(z["gsum/x"]), 130, 10)
    np.testing.assert_array_equal((c / 4.0).astype(np.float32), z["gsum/logits_tau4"])
    assert [H.n_words(b) for b in [1, 64, 65, 128, 129]] == list(z["nwords"])
    th = [1 / 6, 2 / 6, 3 / 6, 4 / 6, 5 / 6]
    np.testing.assert_array_equal(H.thermometer_bits(z["thermo/img"], th), z["thermo/bits"])
