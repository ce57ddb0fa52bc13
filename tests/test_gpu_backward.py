"""Gradients of the depthwise convolution on the GPU (the reference is inference-only).

Checked against the float64 numpy adjoints in oracle/oracle.py, which are
themselves pinned to PyTorch autograd through F.conv2d(groups=C)
(tests/test_oracle.py).  The input gradient runs the forward kernel (mixed
accumulation) and is held to the forward's bar; the weight gradient sums
B*H*W products per tap in fp32 and is held to a relative 1e-5.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import make_problem

pytestmark = pytest.mark.gpu

MAX_TOL, REL_TOL = 1e-2, 1e-3


@pytest.fixture(scope="module")
def eng():
    import depthwise_conv_b200 as d
    return d


def to_dev(a):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.permute(0, 3, 1, 2) if t.dim() == 4 else t


def to_host(t):
    return t.permute(0, 2, 3, 1).contiguous().cpu().numpy() if t.dim() == 4 else t.cpu().numpy()


# The last two need more than one weight-gradient column tile (W > 64, W not a multiple of 64: the
# right-edge zero fill and the column-tile offsets of the loads); in (2, 5, 130, 72, 31) the B*H = 10
# rows split into chunks of 3, so one row chunk spans two images.
SHAPES = [(2, 19, 21, 72, 7), (1, 9, 30, 64, 31), (3, 5, 11, 64, 9), (1, 14, 14, 512, 27), (2, 1, 1, 8, 1),
          (2, 23, 17, 136, 13), (1, 3, 40, 16, 29), (1, 6, 100, 64, 7), (2, 5, 130, 72, 31)]


def _problem(B, H, W, C, K):
    x, w = make_problem(500 + K + C, B, H, W, C, K)
    dy = np.random.default_rng(K + H).standard_normal((B, H, W, C)).astype(np.float16)
    return x, w, dy


@pytest.mark.parametrize("B,H,W,C,K", SHAPES)
def test_weight_gradient(eng, oracle_mod, B, H, W, C, K):
    x, w, dy = _problem(B, H, W, C, K)
    _, dw_exact, _ = oracle_mod.dw_backward_numpy(x, w, dy)
    dw = eng.dw_ops.conv2d_nhwc_backward_weight(to_dev(x), to_dev(dy), K)
    torch.cuda.synchronize()
    got = dw.cpu().numpy().astype(np.float64)
    scale = np.abs(dw_exact).max() + 1e-30
    assert np.abs(got - dw_exact).max() <= 1e-5 * scale + 1e-6
    assert np.linalg.norm(got - dw_exact) <= 1e-5 * np.linalg.norm(dw_exact) + 1e-6


@pytest.mark.parametrize("B,H,W,C,K", SHAPES)
def test_input_gradient(eng, oracle_mod, B, H, W, C, K):
    x, w, dy = _problem(B, H, W, C, K)
    dx_exact, _, _ = oracle_mod.dw_backward_numpy(x, w, dy)
    dx = eng.dw_ops.conv2d_nhwc_backward_input(to_dev(dy), to_dev(w))
    torch.cuda.synchronize()
    assert dx.is_contiguous(memory_format=torch.channels_last)
    max_err, rel = oracle_mod.parity(to_host(dx).astype(np.float64), dx_exact)
    assert max_err <= MAX_TOL and rel <= REL_TOL, f"max {max_err:.3e} rel {rel:.3e}"


def test_weight_gradient_accumulates_into_dw(eng, oracle_mod):
    """dwb_conv2d_nhwc_bwd_weight adds to dw: two calls give twice the gradient."""
    from depthwise_conv_b200 import _lib
    B, H, W, C, K = 2, 12, 12, 64, 9
    x, w, dy = _problem(B, H, W, C, K)
    _, dw_exact, _ = oracle_mod.dw_backward_numpy(x, w, dy)
    xd, gd = to_dev(x), to_dev(dy)
    dw = torch.zeros((K, K, C), dtype=torch.float32, device="cuda")
    for _ in range(2):
        assert _lib.load().dwb_conv2d_nhwc_bwd_weight(xd.data_ptr(), gd.data_ptr(), dw.data_ptr(), B, H, W, C, K,
                                                      torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    got = dw.cpu().numpy().astype(np.float64)
    assert np.abs(got - 2 * dw_exact).max() <= 2e-5 * np.abs(dw_exact).max()


@pytest.mark.parametrize("with_bias", [True, False])
def test_autograd_through_the_op(eng, oracle_mod, with_bias):
    """loss = sum(conv2d_nhwc(x, w, b) * g): x.grad, w.grad, b.grad from the engine's backward."""
    B, H, W, C, K = 2, 16, 20, 128, 9
    x, w, dy = _problem(B, H, W, C, K)
    b = (np.random.default_rng(3).standard_normal(C) * 0.1).astype(np.float16)
    xt = to_dev(x).requires_grad_()
    wt = to_dev(w).requires_grad_()
    bt = to_dev(b).requires_grad_() if with_bias else None
    y = torch.ops.depthwise.conv2d_nhwc(xt, wt, bt)
    y.backward(to_dev(dy))
    torch.cuda.synchronize()
    dx_exact, dw_exact, db_exact = oracle_mod.dw_backward_numpy(x, w, dy)
    max_err, rel = oracle_mod.parity(to_host(xt.grad).astype(np.float64), dx_exact)
    assert max_err <= MAX_TOL and rel <= REL_TOL
    assert wt.grad.dtype == torch.float16 and wt.grad.shape == (K, K, C)
    gw = wt.grad.cpu().numpy().astype(np.float64)
    assert np.abs(gw - dw_exact).max() <= 1e-3 * np.abs(dw_exact).max()  # fp16 rounding of the fp32 sum
    if with_bias:
        gb = bt.grad.cpu().numpy().astype(np.float64)
        assert np.abs(gb - db_exact).max() <= 1e-3 * np.abs(db_exact).max() + 1e-3
    assert eng.device_error() == 0


@pytest.mark.parametrize("act", ["none", "relu", "gelu"])
def test_autograd_through_the_fused_op(eng, act):
    """loss = sum(conv2d_nhwc_fused(x, w, b, s, t, x, act) * g): every gradient against float64 torch
    autograd of the same composition (F.conv2d groups=C, activation, scale/shift, residual)."""
    import torch.nn.functional as F
    B, H, W, C, K = 2, 12, 14, 64, 7
    x, w, dy = _problem(B, H, W, C, K)
    rng = np.random.default_rng(11)
    b = (rng.standard_normal(C) * 0.1).astype(np.float16)
    s = rng.uniform(0.5, 1.5, C).astype(np.float16)
    t = (rng.standard_normal(C) * 0.1).astype(np.float16)
    code = {"none": 0, "relu": 1, "gelu": 2}[act]
    leaves = [to_dev(a).requires_grad_() for a in (x, w, b, s, t)]
    xt, wt, bt, st, tt = leaves
    y = torch.ops.depthwise.conv2d_nhwc_fused(xt, wt, bt, st, tt, xt, code)
    y.backward(to_dev(dy))
    torch.cuda.synchronize()
    # float64 reference on the CPU
    r = [torch.from_numpy(a.astype(np.float64)).requires_grad_() for a in (x, w, b, s, t)]
    rx, rw, rb, rs, rt = r
    xc = rx.permute(0, 3, 1, 2)
    z = F.conv2d(xc, rw.permute(2, 0, 1).unsqueeze(1), rb, padding=K // 2, groups=C)
    a = {"none": z, "relu": torch.relu(z), "gelu": F.gelu(z)}[act]
    yr = a * rs.view(1, -1, 1, 1) + rt.view(1, -1, 1, 1) + xc
    yr.backward(torch.from_numpy(dy.astype(np.float64)).permute(0, 3, 1, 2))
    for name, got, ref in zip("x w b s t".split(), leaves, r):
        gv = to_host(got.grad).astype(np.float64) if got.dim() == 4 else got.grad.cpu().numpy().astype(np.float64)
        rv = ref.grad.numpy()
        rel = np.linalg.norm(gv - rv) / (np.linalg.norm(rv) + 1e-30)
        # ReLU's derivative jumps at 0: where the fp16 pre-activation and the exact one straddle 0
        # (|z| within the forward's error) the mask differs, which is the gradient's own conditioning
        assert rel < (2e-2 if act == "relu" else 5e-3), f"d{name}: rel-L2 {rel:.2e}"
    assert eng.device_error() == 0


@pytest.mark.parametrize("B,H,W,C,K", SHAPES + [(8, 56, 56, 1024, 7)])
def test_deterministic_weight_gradient(eng, oracle_mod, B, H, W, C, K):
    """The fixed-order mode: the oracle's bar, and the same bits on every run (the atomic mode's
    partial sums land in any order)."""
    if B * H * W * C > (1 << 22):  # the large case: repeatability only, the oracle would take minutes
        rng = np.random.default_rng(K)
        xd = torch.from_numpy(rng.standard_normal((B, H, W, C)).astype(np.float16)).cuda().permute(0, 3, 1, 2)
        dyd = torch.from_numpy(rng.standard_normal((B, H, W, C)).astype(np.float16)).cuda().permute(0, 3, 1, 2)
        dw_exact = None
    else:
        x, w, dy = _problem(B, H, W, C, K)
        _, dw_exact, _ = oracle_mod.dw_backward_numpy(x, w, dy)
        xd, dyd = to_dev(x), to_dev(dy)
    runs = [eng.dw_ops.conv2d_nhwc_backward_weight(xd, dyd, K, deterministic=True) for _ in range(3)]
    torch.cuda.synchronize()
    assert all(torch.equal(runs[0], r) for r in runs[1:])
    fast = eng.dw_ops.conv2d_nhwc_backward_weight(xd, dyd, K, deterministic=False)
    torch.cuda.synchronize()
    scale = fast.abs().max().item() + 1e-30
    assert (runs[0] - fast).abs().max().item() <= 1e-5 * scale + 1e-6
    if dw_exact is not None:
        got = runs[0].cpu().numpy().astype(np.float64)
        assert np.abs(got - dw_exact).max() <= 1e-5 * (np.abs(dw_exact).max() + 1e-30) + 1e-6


def test_autograd_weight_gradient_follows_torch_determinism(eng):
    """Under torch.use_deterministic_algorithms(True) the op's backward takes the fixed-order path."""
    rng = np.random.default_rng(3)
    x = torch.from_numpy(rng.standard_normal((4, 32, 32, 256)).astype(np.float16)).cuda().permute(0, 3, 1, 2)
    w = torch.from_numpy((rng.standard_normal((9, 9, 256)) / 9).astype(np.float16)).cuda()
    prev = torch.are_deterministic_algorithms_enabled()
    torch.use_deterministic_algorithms(True, warn_only=True)
    try:
        grads = []
        for _ in range(3):
            wr = w.clone().requires_grad_(True)
            y = torch.ops.depthwise.conv2d_nhwc(x, wr)
            y.float().square().sum().backward()
            grads.append(wr.grad.clone())
        torch.cuda.synchronize()
    finally:
        torch.use_deterministic_algorithms(prev)
    assert all(torch.equal(grads[0], g) for g in grads[1:])
