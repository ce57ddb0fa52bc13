"""The CPU oracle, pinned before it is trusted (CPU only).

* against the golden vectors (tests/golden/dw_cases.npz), produced by the
  reference's own correctness check F.conv2d(groups=C) on fp16 inputs
  (benchmark_sensitivity.py:254-259), run in float64;
* the three restatements (C, numpy, torch) against each other;
* binary16 rounding against numpy's IEEE conversion;
* the fp16-accumulation emulation against the reference's published
  tolerance for its own k31 kernel (max |diff| < 3.0 at N(0,1) weights,
  benchmark_sensitivity.py:343).
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest

from conftest import make_problem

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "dw_cases.npz")


def _golden_cases():
    z = np.load(GOLDEN)
    meta = json.loads(str(z["__meta__"]))
    cases = []
    for m in meta:
        n = m["name"]
        c = {k.split("__", 1)[1]: z[k] for k in z.files if k.startswith(n + "__")}
        c.update(m)
        cases.append(c)
    return cases


CASES = _golden_cases()


def _f16(a):
    return np.asarray(a).view(np.float16)


def _epi(c):
    act = {0: "none", 1: "relu", 2: "gelu"}[int(c["act"])] if "act" in c else "none"
    bias = _f16(c["bias"]) if "bias" in c else None
    scale = _f16(c["scale"]) if "scale" in c else None
    shift = _f16(c["shift"]) if "shift" in c else None
    residual = _f16(c["x"]) if "residual" in c else None
    return dict(bias=bias, scale=scale, shift=shift, residual=residual, act=act)


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_c_oracle_matches_golden(oracle_mod, case):
    x, w = _f16(case["x"]), _f16(case["w"])
    y32, y16 = oracle_mod.dw_forward(x, w, **_epi(case))
    ref = case["y"]
    assert y32.shape == ref.shape
    # double accumulation, output stored as float32: float32 rounding only
    np.testing.assert_allclose(y32, ref, rtol=2e-6, atol=2e-6)
    # the fp16 output is the correctly rounded fixture value (ties are measure-zero)
    expect16 = ref.astype(np.float16)
    mism = np.count_nonzero(y16.view(np.uint16) != expect16.view(np.uint16))
    assert mism <= max(1, ref.size // 10000)


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_numpy_and_torch_restatements_match_golden(oracle_mod, case):
    x, w = _f16(case["x"]), _f16(case["w"])
    e = _epi(case)
    yn = oracle_mod.dw_forward_numpy(x, w, **e)
    np.testing.assert_allclose(yn, case["y"], rtol=1e-12, atol=1e-12)
    yt = oracle_mod.dw_forward_torch(x, w, **e)  # float32, the reference's check precision
    np.testing.assert_allclose(yt, case["y"], rtol=1e-4, atol=1e-4)


def test_pixels_and_channel_sums_agree_with_full(oracle_mod):
    x, w = make_problem(3, 2, 11, 9, 24, 9)
    y32, _ = oracle_mod.dw_forward(x, w)
    pix = np.array([0, 5, 98, 2 * 11 * 9 - 1])
    p32, _ = oracle_mod.dw_forward_pixels(x, w, pix)
    np.testing.assert_array_equal(p32, y32.reshape(-1, 24)[pix])
    sums = oracle_mod.channel_sums(x, w)
    np.testing.assert_allclose(sums, y32.astype(np.float64).sum(axis=(1, 2)), rtol=1e-6, atol=1e-4)


def test_half_rounding_matches_ieee(oracle_mod):
    rng = np.random.default_rng(11)
    vals = rng.standard_normal(20000) * 10.0 ** rng.integers(-9, 6, 20000)
    vals = np.concatenate([vals, [0.0, -0.0, 65504.0, 65519.9, 65520.0, 1e9, 2 ** -24, 2 ** -25, 3 * 2 ** -26,
                                  6.1e-5, -6.1e-5]])
    mine = np.array([oracle_mod.half_round(v) for v in vals], np.uint16)
    np.testing.assert_array_equal(mine, vals.astype(np.float16).view(np.uint16))


def test_fp16_emulation_within_reference_published_tolerance(oracle_mod):
    # benchmark_sensitivity.py:243-262,343: k31 with N(0,1) weights passes if max_diff < 3.0
    x, w = make_problem(42, 1, 24, 24, 16, 31, wscale=1.0)
    exact, _ = oracle_mod.dw_forward(x, w)
    emu = oracle_mod.dw_forward_f16acc(x, w)
    max_err, rel = oracle_mod.parity(emu, exact)
    assert max_err < 3.0
    # and it really is the lossy fp16 path (not the exact one)
    assert rel > 1e-4


def test_fp16_emulation_distance_grows_with_k(oracle_mod):
    rels = []
    for K in (7, 31):
        x, w = make_problem(5, 1, 20, 20, 16, K)
        exact, _ = oracle_mod.dw_forward(x, w)
        rels.append(oracle_mod.parity(oracle_mod.dw_forward_f16acc(x, w), exact)[1])
    assert rels[1] > rels[0]


@pytest.mark.parametrize("B,H,W,C,K", [(2, 7, 9, 8, 3), (1, 5, 4, 16, 7), (2, 6, 6, 8, 1)])
def test_backward_restatement_matches_torch_autograd(oracle_mod, B, H, W, C, K):
    """The numpy gradients agree with PyTorch autograd through F.conv2d(groups=C) in float64."""
    import torch
    import torch.nn.functional as F
    rng = np.random.default_rng(K * 10 + B)
    x = rng.standard_normal((B, H, W, C)).astype(np.float16)
    w = (rng.standard_normal((K, K, C)) / K).astype(np.float16)
    dy = rng.standard_normal((B, H, W, C)).astype(np.float16)
    dx, dw, db = oracle_mod.dw_backward_numpy(x, w, dy)
    xt = torch.tensor(x.astype(np.float64)).permute(0, 3, 1, 2).requires_grad_()
    wt = torch.tensor(w.astype(np.float64)).permute(2, 0, 1).unsqueeze(1).requires_grad_()
    bt = torch.zeros(C, dtype=torch.float64, requires_grad=True)
    y = F.conv2d(xt, wt, bt, padding=K // 2, groups=C)
    y.backward(torch.tensor(dy.astype(np.float64)).permute(0, 3, 1, 2))
    np.testing.assert_allclose(dx, xt.grad.permute(0, 2, 3, 1).numpy(), rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(dw, wt.grad.squeeze(1).permute(1, 2, 0).numpy(), rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(db, bt.grad.numpy(), rtol=1e-12, atol=1e-12)
