"""The reference-facing torch ops and the C ABI on the GPU.

Mirrors how the reference's scripts exercise the path: the fixed-shape ops
(depthwise_torch_ops.py:93-133, depthwise_replknet_nhwc_ops.py:71-86), the
nn.Module swappers, torch.compile in default and reduce-overhead modes, and
the CUDA-graph replay check of verify_e5b_correctness.py:26-37.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch
import torch.nn as nn

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
    return t.permute(0, 2, 3, 1).contiguous().cpu().numpy()


def check(O, y, exact, what=""):
    max_err, rel = O.parity(to_host(y).astype(np.float64), exact)
    assert max_err <= MAX_TOL and rel <= REL_TOL, f"{what}: max {max_err:.3e} rel {rel:.3e}"


FIXED = [("conv2d_32_768_7", 32, 768, 7), ("conv2d_32_1536_9", 32, 1536, 9), ("conv2d_32_1536_9_v2", 32, 1536, 9),
         ("conv2d_16_1536_9", 16, 1536, 9), ("conv2d_32_1536_13", 32, 1536, 13)]


@pytest.mark.parametrize("op,HW,C,K", FIXED, ids=[f[0] for f in FIXED])
@pytest.mark.parametrize("B", [1, 3])
def test_convmixer_ops(eng, oracle_mod, op, HW, C, K, B):
    x, w = make_problem(K + B, B, HW, HW, C, K)
    y = getattr(torch.ops.depthwise, op)(to_dev(x), to_dev(w))
    torch.cuda.synchronize()
    assert y.is_contiguous(memory_format=torch.channels_last)
    exact, _ = oracle_mod.dw_forward(x, w)
    check(oracle_mod, y, exact, op)


REPL = [("conv_56_128_31", 56, 128, 31), ("conv_28_256_29", 28, 256, 29), ("conv_14_512_27", 14, 512, 27),
        ("conv_7_1024_13", 7, 1024, 13)]


@pytest.mark.parametrize("op,HW,C,K", REPL, ids=[r[0] for r in REPL])
@pytest.mark.parametrize("with_bias", [True, False])
def test_replknet_ops(eng, oracle_mod, op, HW, C, K, with_bias):
    x, w = make_problem(K, 2, HW, HW, C, K)
    b = (np.random.default_rng(K).standard_normal(C) * 0.1).astype(np.float16)
    bias = to_dev(b) if with_bias else torch.empty(0, dtype=torch.float16, device="cuda")
    y = getattr(torch.ops.replknet_dw, op)(to_dev(x), to_dev(w), bias)
    torch.cuda.synchronize()
    exact, _ = oracle_mod.dw_forward(x, w, b if with_bias else None)
    check(oracle_mod, y, exact, op)


def test_fixed_ops_reject_wrong_shapes_with_runtime_error(eng):
    x = torch.zeros(1, 768, 16, 16, dtype=torch.float16, device="cuda").contiguous(memory_format=torch.channels_last)
    w = torch.zeros(7, 7, 768, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError):
        torch.ops.depthwise.conv2d_32_768_7(x, w)  # reference: prints and exit(1)
    x2 = torch.zeros(1, 128, 56, 56, dtype=torch.float16, device="cuda")  # NCHW, not channels_last
    w2 = torch.zeros(31, 31, 128, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError):
        torch.ops.replknet_dw.conv_56_128_31(x2, w2, torch.empty(0, dtype=torch.float16, device="cuda"))
    with pytest.raises(RuntimeError):
        torch.ops.depthwise.conv2d_nhwc(x.float(), w)


def test_c_abi_direct_call(eng, oracle_mod):
    """The C entry point a non-Python host would bind, with raw device pointers."""
    from depthwise_conv_b200 import _lib
    x, w = make_problem(1, 2, 28, 28, 256, 29)
    xd, wd = to_dev(x), to_dev(w)
    y = torch.empty_like(xd)
    lib = _lib.load()
    rc = lib.dwb_depthwise_29x29_256_nhwc(xd.data_ptr(), wd.data_ptr(), None, y.data_ptr(), 2, 256, 28, 28,
                                          torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    exact, _ = oracle_mod.dw_forward(x, w)
    check(oracle_mod, y, exact)
    # bad shape / alignment are statuses, not crashes
    assert lib.dwb_depthwise_29x29_256_nhwc(xd.data_ptr(), wd.data_ptr(), None, y.data_ptr(), 2, 256, 27, 28,
                                            None) == _lib.ERR_BAD_SHAPE
    assert lib.dwb_conv2d_nhwc_fwd(xd.data_ptr() + 2, wd.data_ptr(), y.data_ptr(), 2, 28, 28, 256, 29,
                                   None) == _lib.ERR_BAD_ALIGN


def test_custom_module_and_swapper(eng, oracle_mod):
    from depthwise_conv_b200.depthwise_torch_ops import replace_depthwise_convs
    torch.manual_seed(0)
    conv = nn.Conv2d(1536, 1536, 9, groups=1536, padding=4).cuda()
    model = nn.Sequential(conv)
    x = torch.randn(2, 1536, 32, 32, device="cuda").half().contiguous(memory_format=torch.channels_last)
    with torch.no_grad():
        ref = conv.double()(x.double()).float()
    conv.float()
    replace_depthwise_convs(model, verbose=False)
    with torch.no_grad():
        y = model(x)
    torch.cuda.synchronize()
    # weights went through an fp16 cast in the swap, so compare with a relative bar on fp32 reference
    err = (y.float() - ref).abs()
    assert err.max().item() < 2e-2
    assert (err.norm() / ref.norm()).item() < 2e-3


def test_replknet_swapper_stage3(eng):
    from depthwise_conv_b200.depthwise_replknet_nhwc_ops import replace_replknet_depthwise_nhwc
    m = nn.Sequential(nn.Conv2d(1024, 1024, 13, groups=1024, padding=6, bias=False)).cuda()
    x = torch.randn(1, 1024, 7, 7, device="cuda").half().contiguous(memory_format=torch.channels_last)
    with torch.no_grad():
        ref = m.float()(x.float())
    replace_replknet_depthwise_nhwc(m, verbose=False)
    with torch.no_grad():
        y = m(x)
    assert ((y.float() - ref).norm() / ref.norm()).item() < 2e-3


class _Block(nn.Module):
    def __init__(self):
        super().__init__()
        self.w = nn.Parameter(torch.randn(9, 9, 256, dtype=torch.float16) / 9)
        self.b = nn.Parameter(torch.randn(256, dtype=torch.float16) * 0.1)
        self.s = nn.Parameter(torch.rand(256, dtype=torch.float16) + 0.5)
        self.t = nn.Parameter(torch.randn(256, dtype=torch.float16) * 0.1)

    def forward(self, x):
        y = torch.ops.depthwise.conv2d_nhwc_fused(x, self.w, self.b, self.s, self.t, x, 2)
        return torch.ops.depthwise.conv2d_nhwc(y * 0.5 + 1.0, self.w, None)


@pytest.mark.parametrize("mode", ["default", "reduce-overhead"])
def test_torch_compile_modes_and_replay(eng, mode):
    torch.manual_seed(0)
    blk = _Block().cuda()
    mk = lambda: torch.randn(2, 256, 32, 32, device="cuda").half().contiguous(memory_format=torch.channels_last)  # noqa: E731
    compiled = torch.compile(blk, mode=mode, fullgraph=True)
    with torch.no_grad():
        x1, x2 = mk(), mk()
        y1 = compiled(x1).clone()
        y2 = compiled(x2).clone()
        r1, r2 = blk(x1), blk(x2)
        assert (y1 - r1).abs().max().item() == 0.0
        assert (y2 - r2).abs().max().item() == 0.0
        assert (y1 - y2).abs().max().item() > 0.1
        # replay follows a changing input (verify_e5b_correctness.py:30-37)
        outs = [compiled(mk()).clone() for _ in range(5)]
        diffs = [(outs[i] - outs[i + 1]).abs().max().item() for i in range(4)]
        assert all(d > 0.1 for d in diffs)
        again = compiled(x1).clone()
        assert (again - y1).abs().max().item() == 0.0


def test_cuda_graph_capture_of_c_abi(eng, oracle_mod):
    x, w = make_problem(3, 2, 32, 32, 512, 13)
    xd, wd = to_dev(x), to_dev(w)
    y = torch.empty_like(xd)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        eng.conv2d_nhwc_fused(xd, wd, out=y)  # warm-up (device init, attributes) outside capture
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        eng.conv2d_nhwc_fused(xd, wd, out=y)
    y.zero_()
    g.replay()
    torch.cuda.synchronize()
    exact, _ = oracle_mod.dw_forward(x, w)
    check(oracle_mod, y, exact, "graph replay")
    # new data in the captured input buffer is picked up
    x2, _ = make_problem(4, 2, 32, 32, 512, 13)
    xd.copy_(to_dev(x2))
    g.replay()
    torch.cuda.synchronize()
    exact2, _ = oracle_mod.dw_forward(x2, w)
    check(oracle_mod, y, exact2, "graph replay 2")


def test_dependent_launch_chain_matches_synchronised_chain(eng):
    """Kernels start early under programmatic dependent launch but read their inputs only after the
    previous kernel has finished: a chain of dependent launches (each reading the previous output,
    in place updates in between) equals the same chain with a device synchronisation between steps."""
    torch.manual_seed(5)
    C = 512
    x0 = torch.randn(2, C, 20, 20, device="cuda").half().contiguous(memory_format=torch.channels_last)
    ws = [(torch.randn(k, k, C, device="cuda") / k).half() for k in (7, 13, 27, 9)]
    b = (torch.randn(C, device="cuda") * 0.1).half()
    s = (torch.rand(C, device="cuda") + 0.5).half()

    def chain(sync):
        x = x0.clone()
        for i in range(6):
            w = ws[i % len(ws)]
            y = eng.conv2d_nhwc_fused(x, w, b, s, None, x, "gelu")
            if sync:
                torch.cuda.synchronize()
            eng.dw_ops.bias_act_affine(y, b, s, None, "relu", out=y)  # in place, read by the next launch
            if sync:
                torch.cuda.synchronize()
            x = y
        torch.cuda.synchronize()
        return x

    a, b2 = chain(False), chain(True)
    assert torch.isfinite(a.float()).all()
    assert torch.equal(a, b2)


@pytest.mark.parametrize("act", ["none", "relu", "gelu"])
def test_bias_act_affine(eng, act):
    """The pointwise-block epilogue: y = act(x + b) * s + t, against float64 math."""
    from math import erf, sqrt
    rng = np.random.default_rng(3)
    B, C, H, W = 2, 1536, 7, 9
    x = (rng.standard_normal((B, H, W, C)) * 2).astype(np.float16)
    b = (rng.standard_normal(C) * 0.5).astype(np.float16)
    s = rng.uniform(0.5, 1.5, C).astype(np.float16)
    t = (rng.standard_normal(C) * 0.5).astype(np.float16)
    v = x.astype(np.float64) + b.astype(np.float64)
    if act == "relu":
        v = np.maximum(v, 0)
    elif act == "gelu":
        v = 0.5 * v * (1 + np.vectorize(erf)(v / sqrt(2)))
    exact = v * s.astype(np.float64) + t.astype(np.float64)
    xd = to_dev(x)
    y = eng.dw_ops.bias_act_affine(xd, to_dev(b), to_dev(s), to_dev(t), act)
    torch.cuda.synchronize()
    got = to_host(y).astype(np.float64)
    a = np.abs(exact)
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(a, 2.0 ** -14))) - 10)
    assert (np.abs(got - exact) <= 2 * ulp + 1e-7).all()
    # in place (x == y), as the ConvMixer pointwise block uses it
    eng.dw_ops.bias_act_affine(xd, to_dev(b), to_dev(s), to_dev(t), act, out=xd)
    torch.cuda.synchronize()
    assert torch.equal(xd, y)


@pytest.mark.parametrize("B,H,W,C,offset,with_scale", [(4, 32, 32, 1536, 0, True), (4, 64, 64, 200, 0, False),
                                                        (4, 64, 64, 200, 2, True), (1, 3, 5, 24, 2, False)])
def test_bias_act_affine_strides_and_parameter_alignment(eng, B, H, W, C, offset, with_scale):
    """More 8-channel groups than the grid has threads (the channel index advances across grid
    strides), channel counts that do not divide the grid, parameter vectors only 4-byte aligned
    (offset halves into their allocation), and an absent scale."""
    from math import sqrt

    from scipy.special import erf
    rng = np.random.default_rng(B * 1000 + C + offset)
    x = (rng.standard_normal((B, H, W, C)) * 2).astype(np.float16)
    b = (rng.standard_normal(C) * 0.5).astype(np.float16)
    s = rng.uniform(0.5, 1.5, C).astype(np.float16)
    t = (rng.standard_normal(C) * 0.5).astype(np.float16)
    v = x.astype(np.float64) + b.astype(np.float64)
    gs = 0.5 * v * (1 + erf(v / sqrt(2))) * (s.astype(np.float64) if with_scale else 1.0)
    exact = gs + t.astype(np.float64)

    def vec(a):
        buf = torch.zeros(C + offset, dtype=torch.float16, device="cuda")
        buf[offset:] = torch.from_numpy(a).cuda()
        return buf[offset:]

    y = eng.dw_ops.bias_act_affine(to_dev(x), vec(b), vec(s) if with_scale else None, vec(t), "gelu")
    torch.cuda.synchronize()
    got = to_host(y).astype(np.float64)
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(exact), 2.0 ** -14))) - 10)
    # 2 ulp of the result, plus 1e-4 of the GELU term: where act(v) * s nearly cancels t, the erfc
    # approximation's tail error (about 4e-5 of the term near v = -2.9, well inside one fp16 ulp of
    # the term) outgrows the ulp of the small result
    assert (np.abs(got - exact) <= 2 * ulp + 1e-7 + 1e-4 * np.abs(gs)).all()


def test_probe_fma_peak_reports_plausible_rates(eng):
    h, f = eng.probe_fma_peak()
    assert 10.0 < h < 200.0 and 10.0 < f < 200.0


def test_device_error_word_clear(eng):
    assert eng.device_error() == 0


def test_expired_wait_reports_and_context_survives(eng, oracle_mod):
    """Failure path on the GPU without a fault: a kernel whose mbarrier wait nothing completes gives up
    after ~1 ms, leaves code 5 in the device error word and returns; the next convolution still runs
    and matches the oracle, and the word reads clean again."""
    from depthwise_conv_b200 import _lib
    assert eng.device_error() == 0
    assert _lib.selftest_bounded_wait(2_000_000) == 5
    assert eng.device_error() == 0  # cleared by the read
    x, w = make_problem(5, 1, 16, 16, 64, 7)
    y = eng.conv2d_nhwc_fused(to_dev(x), to_dev(w))
    torch.cuda.synchronize()
    exact, _ = oracle_mod.dw_forward(x, w)
    check(oracle_mod, y, exact, "after the self-test")
    assert eng.device_error() == 0
    with pytest.raises(_lib.DwbError):
        _lib.selftest_bounded_wait(0)


def test_expired_wait_raises_in_torch_path_when_checked(eng, oracle_mod):
    """With the opt-in post-launch check on (DWB_CHECK_DEVICE_ERROR=1 or set_check_device_error), an
    expired bounded wait surfaces as an exception from the next torch op on that device.  The expiry
    is made without a fault: the bounded-wait self-test kernel gives up after ~1 ms and leaves code 5;
    the op after it raises DeviceTimeoutError (a RuntimeError); the context stays usable and the op
    then runs and matches the oracle."""
    from depthwise_conv_b200 import _lib
    assert eng.device_error() == 0
    x, w = make_problem(6, 1, 16, 16, 64, 7)
    xd, wd = to_dev(x), to_dev(w)
    prev = _lib.set_check_device_error(True)
    try:
        stream = torch.cuda.current_stream().cuda_stream
        assert _lib.load().dwb_selftest_bounded_wait(2_000_000, stream) == _lib.OK  # leaves code 5
        with pytest.raises(RuntimeError, match="bounded wait expired"):
            eng.conv2d_nhwc_fused(xd, wd)
        y = eng.conv2d_nhwc_fused(xd, wd)  # the read cleared the word: this call passes the check
        y2 = torch.ops.depthwise.conv2d_nhwc(xd, wd, None)
    finally:
        _lib.set_check_device_error(prev)
    torch.cuda.synchronize()
    exact, _ = oracle_mod.dw_forward(x, w)
    check(oracle_mod, y, exact, "after the expired wait")
    assert torch.equal(y, y2)
    assert eng.device_error() == 0
