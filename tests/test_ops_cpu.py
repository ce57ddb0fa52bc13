"""The drop-in boundary without a GPU: op names and schemas identical to the
reference's, fake impls for torch.compile, the module swappers' weight repack
identical to the reference's, and loud failure instead of a CPU fallback."""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np
import pytest
import torch
import torch.nn as nn

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def eng():
    import depthwise_conv_b200 as d
    return d


def _schemas():
    with open(os.path.join(GOLDEN, "op_schemas.json")) as f:
        return json.load(f)


def test_op_schemas_identical_to_reference(eng):
    ref = _schemas()["schemas"]
    assert len(ref) == 8
    for name, schema in ref.items():
        ns, op = name.split("::")
        assert str(getattr(getattr(torch.ops, ns), op).default._schema) == schema


def test_dispatch_tables_cover_reference(eng):
    from depthwise_conv_b200.depthwise_replknet_nhwc_ops import _REPLACEMENT_MAP
    from depthwise_conv_b200.depthwise_torch_ops import CustomDepthwiseConv2d
    ref = _schemas()
    ours = {f"{k[0]},{k[1]},{k[2]}": v for k, v in CustomDepthwiseConv2d.SUPPORTED_CONFIGS.items()}
    assert ours == ref["supported_configs"]
    repl = {f"{k[0]},{k[1]}": v.__name__ for k, v in _REPLACEMENT_MAP.items()}
    for key, cls in ref["replacement_map"].items():
        assert repl[key] == cls
    assert repl["1024,13"] == "NHWCDepthwise13x13_1024"  # the stage the reference leaves on nn.Conv2d


@pytest.mark.parametrize("op,args", [
    ("depthwise.conv2d_32_1536_9", ((2, 1536, 32, 32), (9, 9, 1536))),
    ("depthwise.conv2d_32_768_7", ((2, 768, 32, 32), (7, 7, 768))),
    ("replknet_dw.conv_56_128_31", ((1, 128, 56, 56), (31, 31, 128), (128,))),
    ("depthwise.conv2d_nhwc", ((3, 64, 20, 20), (5, 5, 64))),
])
def test_fake_impls_keep_channels_last(eng, op, args):
    from torch._subclasses.fake_tensor import FakeTensorMode
    ns, name = op.split(".")
    fn = getattr(getattr(torch.ops, ns), name)
    with FakeTensorMode():
        x = torch.empty(args[0], dtype=torch.float16, device="cuda").contiguous(memory_format=torch.channels_last)
        rest = [torch.empty(a, dtype=torch.float16, device="cuda") for a in args[1:]]
        y = fn(x, *rest)
        assert y.shape == x.shape and y.stride() == x.stride() and y.dtype == torch.float16


def test_bias_act_affine_op_fake_impl(eng):
    """The pointwise-epilogue op traces under FakeTensorMode (what torch.compile needs) and keeps
    channels_last strides."""
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        x = torch.empty((1, 1536, 32, 32), dtype=torch.float16, device="cuda").contiguous(
            memory_format=torch.channels_last)
        v = torch.empty((1536,), dtype=torch.float16, device="cuda")
        y = torch.ops.depthwise.bias_act_affine(x, v, v, v, 2)
        assert y.shape == x.shape and y.stride() == x.stride()


def test_fake_impl_strides_match_reference_check(eng):
    # the reference's own fake impl gives strides (1572864, 1, 49152, 1536) for a
    # [1, 1536, 32, 32] channels_last input
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        x = torch.empty(1, 1536, 32, 32, dtype=torch.float16, device="cuda").contiguous(
            memory_format=torch.channels_last)
        y = torch.ops.depthwise.conv2d_32_1536_9(x, torch.empty(9, 9, 1536, dtype=torch.float16, device="cuda"))
        assert y.stride() == (1572864, 1, 49152, 1536)


def test_cpu_tensors_raise_instead_of_falling_back(eng):
    x = torch.zeros(1, 64, 8, 8, dtype=torch.float16).contiguous(memory_format=torch.channels_last)
    w = torch.zeros(3, 3, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA"):
        torch.ops.depthwise.conv2d_nhwc(x, w)
    with pytest.raises(RuntimeError):
        eng.conv2d_nhwc_fused(x, w)
    with pytest.raises(RuntimeError):
        torch.ops.replknet_dw.conv_56_128_31(torch.zeros(1, 128, 56, 56, dtype=torch.float16),
                                             torch.zeros(31, 31, 128, dtype=torch.float16),
                                             torch.zeros(0, dtype=torch.float16))


def _digest(t):
    return hashlib.sha256(t.detach().contiguous().view(torch.int16).numpy().tobytes()).hexdigest()


def test_swapper_repack_identical_to_reference(eng):
    sys.path.insert(0, GOLDEN)
    from make_golden import REPACK_CASES, repack_model
    from depthwise_conv_b200.depthwise_replknet_nhwc_ops import replace_replknet_depthwise_nhwc
    from depthwise_conv_b200.depthwise_torch_ops import replace_depthwise_convs
    with open(os.path.join(GOLDEN, "swap_repack.json")) as f:
        ref = json.load(f)
    for i, (tag, C, K, bias, which) in enumerate(REPACK_CASES):
        m = repack_model(C, K, bias, 500 + i)
        if which == "convmixer":
            replace_depthwise_convs(m, verbose=False)
        else:
            replace_replknet_depthwise_nhwc(m, verbose=False)
        mod = m.body[0]
        exp = ref[tag]
        assert type(mod).__name__ == exp["type"]
        assert list(mod.weight.shape) == exp["weight_shape"]
        assert _digest(mod.weight) == exp["weight_sha256"], tag
        if exp["bias_sha256"] is None:
            assert mod.bias is None
        else:
            assert _digest(mod.bias) == exp["bias_sha256"], tag


def test_swapper_skips_non_depthwise_and_unsupported(eng):
    from depthwise_conv_b200.depthwise_torch_ops import CustomDepthwiseConv2d, replace_depthwise_convs
    m = nn.Sequential(nn.Conv2d(64, 64, 3, padding=1), nn.Conv2d(64, 64, 5, groups=64, padding=2),
                      nn.Conv2d(768, 768, 7, groups=768, padding=3))
    replace_depthwise_convs(m, verbose=False)
    assert isinstance(m[0], nn.Conv2d) and isinstance(m[1], nn.Conv2d)  # dense / unsupported stay
    assert isinstance(m[2], CustomDepthwiseConv2d)
    m2 = nn.Sequential(nn.Conv2d(64, 64, 5, groups=64, padding=2))
    replace_depthwise_convs(m2, verbose=False, any_shape=True)
    assert isinstance(m2[0], CustomDepthwiseConv2d)


def test_strict_module_keeps_reference_error(eng):
    from depthwise_conv_b200.depthwise_torch_ops import CustomDepthwiseConv2d
    mod = CustomDepthwiseConv2d(64, 5, strict=True)
    with pytest.raises(ValueError):
        mod._get_op_name(20)
    assert CustomDepthwiseConv2d(64, 5)._get_op_name(20) == "depthwise::conv2d_nhwc"


def test_convmixer_models_share_weights_with_cpu_reference():
    """The GPU model and the CPU baseline model draw identical weights for a seed."""
    from depthwise_conv_b200.convmixer import ConvMixer, init_baseline_
    from oracle.convmixer_ref import ConvMixerCPU
    gpu_model = init_baseline_(ConvMixer(64, 2, kernel_size=5, patch_size=7, n_classes=10, activation='gelu'), 3).eval()
    cpu_model = ConvMixerCPU(64, 2, 5, 7, 'gelu', 10, seed=3)
    convs = [m for m in gpu_model.modules() if isinstance(m, nn.Conv2d)]
    assert torch.equal(convs[0].weight, cpu_model.patch_w)
    assert torch.equal(convs[1].weight, cpu_model.dw_w[0]) and torch.equal(convs[2].weight, cpu_model.pw_w[0])
    assert torch.equal(convs[3].weight, cpu_model.dw_w[1]) and torch.equal(convs[4].weight, cpu_model.pw_w[1])
    x = torch.randn(1, 3, 28, 28)
    with torch.no_grad():
        np.testing.assert_allclose(gpu_model(x).numpy(), cpu_model(x).numpy(), rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("B,Cin,H,W,p,C,channels_last", [(2, 3, 224, 224, 7, 64, True), (1, 3, 30, 29, 7, 16, True),
                                                         (2, 3, 28, 28, 14, 8, False), (1, 5, 9, 9, 3, 12, False)])
def test_stem_patch_gemm_equals_patch_conv(eng, B, Cin, H, W, p, C, channels_last):
    """The ConvMixer stem's GEMM form (patch matrix x [kh, kw, c_in] x C weight, rows zero-padded to a
    multiple of 8) equals the strided patch convolution, including sizes that do not divide by p."""
    from depthwise_conv_b200.convmixer import FusedStem, patch_matrix
    torch.manual_seed(p * 100 + C)
    conv = nn.Conv2d(Cin, C, p, stride=p)
    stem = FusedStem(conv, "gelu", nn.BatchNorm2d(C).eval())
    K = p * p * Cin
    assert stem.patch == p and stem.k_pad % 8 == 0 and stem.k_pad - K < 8
    x = torch.randn(B, Cin, H, W)
    if channels_last:
        x = x.contiguous(memory_format=torch.channels_last)
    a = patch_matrix(x, p, stem.k_pad)
    assert a.shape == (B * (H // p) * (W // p), stem.k_pad) and (a[:, K:] == 0).all()
    z = (a @ stem.weight_t.float()).view(B, H // p, W // p, C).permute(0, 3, 1, 2)
    ref = torch.nn.functional.conv2d(x, conv.weight.detach().half().float(), None, p)
    assert torch.allclose(z, ref, atol=1e-4, rtol=1e-4)


def test_stem_keeps_the_convolution_for_overlapping_patches(eng):
    from depthwise_conv_b200.convmixer import FusedStem
    assert FusedStem(nn.Conv2d(3, 16, 7, stride=4), "gelu", nn.BatchNorm2d(16).eval()).patch == 0
    assert FusedStem(nn.Conv2d(3, 16, 7, stride=7, padding=1), "gelu", nn.BatchNorm2d(16).eval()).patch == 0


def test_module_direct_path_covers_every_fixed_op():
    """In eager inference CustomDepthwiseConv2d calls the fixed-shape launchers itself; every op it can
    select has its entry point and shape listed."""
    from depthwise_conv_b200 import depthwise_torch_ops as m
    for op in set(m.CustomDepthwiseConv2d.SUPPORTED_CONFIGS.values()) | {"depthwise::conv2d_32_1536_9_v2"}:
        fn, H, W, C, K, stride = m._FIXED_ARGS[op]
        assert fn.startswith("dwb_depthwise_forward_")
        # the op name spells the shape: conv2d_<HW>_<C>_<K>[_v2]
        hw, c, k = (int(v) for v in op.split("::conv2d_")[1].split("_")[:3])
        assert (H, W, C, K) == (hw, hw, c, k) and stride == (C == 1536 and K == 9 and H == 32)
