"""The reference's bare module names (``compat/``).

The reference's harness imports its op modules by bare name after putting
their directory on ``sys.path``: ``from depthwise_torch_ops import
CustomDepthwiseConv2d`` (bench_custom_warm.py:42), ``from
depthwise_replknet_nhwc_ops import NHWCDepthwise29x29_256`` (:43),
``replace_depthwise_convs`` (benchmark_compile_modes.py:28,
convmixer/benchmark.py:31) and ``replace_replknet_depthwise_nhwc``
(replknet/benchmark.py:215).  With ``compat/`` first on ``sys.path`` the
same lines import the engine.  The CPU test checks the import and the
names; the GPU test runs the imported modules exactly as those scripts do
and compares with the oracle.
"""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest
import torch
import torch.nn as nn

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
COMPAT = os.path.join(ROOT, "compat")


@pytest.fixture()
def compat_path():
    sys.path.insert(0, COMPAT)
    try:
        yield
    finally:
        sys.path.remove(COMPAT)


def test_bare_names_are_the_engine_modules(compat_path):
    import depthwise_conv_b200.depthwise_replknet_nhwc_ops as eng_r
    import depthwise_conv_b200.depthwise_torch_ops as eng_c
    import depthwise_replknet_nhwc_ops
    import depthwise_torch_ops
    assert depthwise_torch_ops is eng_c
    assert depthwise_replknet_nhwc_ops is eng_r
    from depthwise_replknet_nhwc_ops import (NHWCDepthwise27x27_512, NHWCDepthwise29x29_256,  # noqa: F401
                                             NHWCDepthwise31x31_128, replace_replknet_depthwise_nhwc)
    from depthwise_torch_ops import CustomDepthwiseConv2d, replace_depthwise_convs  # noqa: F401
    assert callable(replace_depthwise_convs) and callable(replace_replknet_depthwise_nhwc)
    assert hasattr(torch.ops.depthwise, "conv2d_32_1536_9") and hasattr(torch.ops.replknet_dw, "conv_56_128_31")


def test_bare_import_in_a_fresh_process():
    """A process that knows only the compat directory (as the reference's scripts do) imports the engine."""
    code = ("import sys; sys.path.insert(0, %r)\n"
            "from depthwise_torch_ops import CustomDepthwiseConv2d, replace_depthwise_convs\n"
            "from depthwise_replknet_nhwc_ops import replace_replknet_depthwise_nhwc\n"
            "import depthwise_torch_ops as m\n"
            "print(m.__name__)\n") % COMPAT
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, cwd="/", timeout=300)
    assert res.returncode == 0, res.stderr[-2000:]
    assert res.stdout.strip().endswith("depthwise_conv_b200.depthwise_torch_ops")


@pytest.mark.gpu
def test_reference_harness_lines_run_on_the_engine(compat_path, oracle_mod):
    # bench_custom_warm.py:40-55: seeded modules built by their constructors, fed channels_last fp16
    torch.manual_seed(0)
    from depthwise_replknet_nhwc_ops import NHWCDepthwise29x29_256
    from depthwise_torch_ops import CustomDepthwiseConv2d, replace_depthwise_convs
    for mod, (C, K, HW) in ((CustomDepthwiseConv2d(1536, 9), (1536, 9, 32)),
                            (NHWCDepthwise29x29_256(), (256, 29, 28))):
        m = mod.cuda().half()
        with torch.no_grad():  # BASELINE's layer init: w ~ N(0, 1/K^2); a small bias
            m.weight.copy_(torch.randn(m.weight.shape) / K)
            if getattr(m, "bias", None) is not None:
                m.bias.copy_(torch.randn(C) * 0.1)
        x = torch.randn(1, C, HW, HW).cuda().half().contiguous(memory_format=torch.channels_last)
        with torch.no_grad():
            y = m(x)
        torch.cuda.synchronize()
        xn = x.permute(0, 2, 3, 1).contiguous().cpu().numpy()
        w = m.weight.detach()
        if w.dim() == 4:  # [C, 1, K, K] -> [K, K, C]
            w = w[:, 0].permute(1, 2, 0)
        b = getattr(m, "bias", None)
        bn = None if b is None else b.detach().cpu().numpy().astype(np.float16)
        exact, _ = oracle_mod.dw_forward(xn, w.contiguous().cpu().numpy().astype(np.float16), bn)
        max_err, rel = oracle_mod.parity(y.permute(0, 2, 3, 1).float().cpu().numpy(), exact)
        assert max_err <= 1e-2 and rel <= 1e-3, (type(mod).__name__, max_err, rel)

    # benchmark_compile_modes.py:28 / convmixer/benchmark.py:31: swap a ConvMixer residual block's DW conv
    torch.manual_seed(1)
    block = nn.Sequential(nn.Conv2d(768, 768, 7, groups=768, padding=3), nn.ReLU(), nn.BatchNorm2d(768)).cuda().eval()
    x = torch.randn(1, 768, 32, 32, device="cuda").half().contiguous(memory_format=torch.channels_last)
    with torch.no_grad():
        ref = block.double()(x.double()).float()
    block.half()
    replace_depthwise_convs(block, verbose=False)
    assert type(block[0]).__name__ == "CustomDepthwiseConv2d"
    with torch.no_grad():
        y = block(x)
    err = (y.float() - ref).abs()
    assert err.max().item() < 2e-2 and (err.norm() / ref.norm()).item() < 2e-3
