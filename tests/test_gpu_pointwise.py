"""The pointwise block's tensor-core kernel (``dwb_pointwise_conv_nhwc``) against float64 math.

y = act(x @ w^T + bias) * scale + shift: the 1x1 convolution, bias, activation and
inference BatchNorm of a ConvMixer block (convmixer/convmixer.py:116-118) and the
patch stem's GEMM, computed by tcgen05 MMAs into tensor memory with the epilogue
applied before the one fp16 store.  The bar: every output within 2 fp16 ulps of the
float64 result (+2e-5 absolute for fp32 accumulation near zero).
"""
from __future__ import annotations

from math import erf, sqrt

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def eng():
    import depthwise_conv_b200 as d
    return d


def problem(seed, M, K, N, params=True):
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((M, K), dtype=np.float32).astype(np.float16)
    w = (rng.standard_normal((N, K), dtype=np.float32) / np.sqrt(K)).astype(np.float16)
    if not params:
        return a, w, None, None, None
    b = (rng.standard_normal(N) * 0.5).astype(np.float16)
    s = rng.uniform(0.5, 1.5, N).astype(np.float16)
    t = (rng.standard_normal(N) * 0.5).astype(np.float16)
    return a, w, b, s, t


def exact(a, w, b, s, t, act):
    v = torch.from_numpy(a).double() @ torch.from_numpy(w).double().t()
    if b is not None:
        v = v + torch.from_numpy(b).double()
    if act == "relu":
        v = v.clamp_min(0)
    elif act == "gelu":
        v = 0.5 * v * (1 + torch.erf(v / sqrt(2)))
    if s is not None:
        v = v * torch.from_numpy(s).double()
    if t is not None:
        v = v + torch.from_numpy(t).double()
    return v.numpy()


def assert_within_2ulp(got, ref, what):
    a = np.abs(ref)
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(a, 2.0 ** -14))) - 10)
    err = np.abs(got.astype(np.float64) - ref)
    bad = err > 2 * ulp + 2e-5
    assert not bad.any(), f"{what}: {int(bad.sum())} outputs off, worst {err.max():.3e} at {np.argmax(err)}"


def dev(v):
    return None if v is None else torch.from_numpy(np.ascontiguousarray(v)).cuda()


SHAPES = [
    (1024, 1536, 1536),  # ConvMixer-1536/20 block at batch 1
    (1024, 152, 1536),   # its patch stem: 147 taps padded to 152
    (1024, 768, 768),    # ConvMixer-768/32
    (1000, 136, 200),    # ragged: rows, K blocks and channel tiles all partial
    (1, 64, 64),         # one pixel
    (300, 8, 8),         # the smallest channel counts
]


@pytest.mark.parametrize("M,K,N", SHAPES)
@pytest.mark.parametrize("act", ["none", "relu", "gelu"])
def test_pointwise_gemm_matches_float64(eng, M, K, N, act):
    a, w, b, s, t = problem(M + K + N, M, K, N)
    y = eng.dw_ops.pointwise_gemm(dev(a), dev(w), dev(b), dev(s), dev(t), act)
    torch.cuda.synchronize()
    assert y.shape == (M, N) and y.dtype == torch.float16
    assert_within_2ulp(y.cpu().numpy(), exact(a, w, b, s, t, act), f"{M}x{K}x{N} {act}")


@pytest.mark.parametrize("tile_n", [64, 96, 128, 256])
def test_every_tile_width(eng, tile_n):
    M, K, N = 517, 320, 392  # 392 = 4 x 96 + 8: a partial last tile for every width
    a, w, b, s, t = problem(tile_n, M, K, N)
    y = eng.dw_ops.pointwise_gemm(dev(a), dev(w), dev(b), dev(s), dev(t), "gelu", tile_n=tile_n)
    torch.cuda.synchronize()
    assert_within_2ulp(y.cpu().numpy(), exact(a, w, b, s, t, "gelu"), f"tile_n {tile_n}")


def test_without_parameters_and_batched(eng):
    M, K, N = 4 * 1024, 1536, 1536  # batch 4: several waves of tiles
    a, w, _, _, _ = problem(11, M, K, N, params=False)
    y = eng.dw_ops.pointwise_gemm(dev(a), dev(w))
    torch.cuda.synchronize()
    assert_within_2ulp(y.cpu().numpy(), exact(a, w, None, None, None, "none"), "plain product")


def test_nhwc_form_matches_the_unfused_block(eng):
    """pointwise_conv_nhwc on a channels_last tensor == Conv2d(1x1) -> GELU -> BatchNorm2d (eval)."""
    import torch.nn as nn
    torch.manual_seed(5)
    C_in, C_out = 256, 384
    conv, bn = nn.Conv2d(C_in, C_out, 1).half(), nn.BatchNorm2d(C_out).eval()
    with torch.no_grad():
        bn.weight.uniform_(0.5, 1.5)
        bn.bias.normal_(0, 0.5)
        bn.running_mean.normal_(0, 0.2)
        bn.running_var.uniform_(0.5, 2.0)
        sc = (bn.weight / torch.sqrt(bn.running_var + bn.eps)).half()
        sh = (bn.bias - bn.running_mean * bn.weight / torch.sqrt(bn.running_var + bn.eps)).half()
    x = torch.randn(2, C_in, 14, 14).half().cuda().contiguous(memory_format=torch.channels_last)
    y = eng.dw_ops.pointwise_conv_nhwc(x, conv.weight.detach().cuda(), conv.bias.detach().cuda(), sc.cuda(),
                                       sh.cuda(), "gelu")
    torch.cuda.synchronize()
    assert y.is_contiguous(memory_format=torch.channels_last) and y.shape == (2, C_out, 14, 14)
    with torch.no_grad():
        z = torch.nn.functional.conv2d(x.double().cpu(), conv.weight.double(), conv.bias.double())
        folded = 0.5 * z * (1 + torch.erf(z / sqrt(2))) * sc.double().view(1, -1, 1, 1) + sh.double().view(1, -1, 1, 1)
        exp = nn.Sequential(nn.GELU(), bn.double())(z)
    got = y.double().cpu()
    assert_within_2ulp(got.numpy(), folded.numpy(), "nhwc form")
    assert (got - exp).abs().max().item() < 2e-2  # and the unfolded fp64 block up to the fp16 BN fold


def test_argument_errors(eng):
    a = torch.zeros(64, 64, dtype=torch.float16, device="cuda")
    w = torch.zeros(64, 64, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError):
        eng.dw_ops.pointwise_gemm(a, w, tile_n=80)  # not a compiled tile width
    with pytest.raises(RuntimeError):
        eng.dw_ops.pointwise_gemm(a, torch.zeros(60, 64, dtype=torch.float16, device="cuda"))  # C_out % 8
    with pytest.raises(RuntimeError):
        eng.dw_ops.pointwise_gemm(a, torch.zeros(64, 32, dtype=torch.float16, device="cuda"))  # K mismatch
    y = eng.dw_ops.pointwise_gemm(a[:0], w)  # no pixels: a no-op
    assert y.shape == (0, 64)


def test_no_device_error_left(eng):
    a, w, b, s, t = problem(1, 1024, 1536, 1536)
    eng.dw_ops.pointwise_gemm(dev(a), dev(w), dev(b), dev(s), dev(t), "gelu")
    torch.cuda.synchronize()
    code = eng._lib.device_error(clear=False)
    assert code == 0, f"device error word {code}"
