"""Drop-in replacement for ``replknet/kernels/depthwise_replknet_nhwc_ops.py``.

Same ``replknet_dw::*`` op names and schemas (depthwise_replknet_nhwc_ops.py:53-66),
"default" impls and fake impls (:71-104), NHWC modules (:108-145),
``_REPLACEMENT_MAP`` (:148-152) and ``replace_replknet_depthwise_nhwc``
(:155-210), backed by the sm_100a engine.

Differences, all deliberate:

* the bias add is fused into the convolution's epilogue (the reference
  launches a separate ``bias_add_nhwc_kernel`` per image,
  depthwise_replknet_nhwc_integration.cu:23-28,92-95) and the batch runs in
  one launch instead of a per-image loop (:82-96);
* the 13x13 / 1024-channel stage that the reference leaves on PyTorch's
  conv (:16) has its own op and module here (``conv_7_1024_13``).
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import _lib
from . import dw_ops

_LOADED = False


def _load_kernels():
    global _LOADED
    lib = _lib.load()
    _LOADED = True
    return lib


def _replknet_op(fn: str, input, weight, bias, C: int, HW: int, K: int):
    dw_ops.check_input(input)
    if not weight.is_contiguous() or weight.dtype != torch.float16:
        raise RuntimeError("weight must be contiguous float16")
    B, Ci, Hi, Wi = input.shape
    if (Ci, Hi, Wi) != (C, HW, HW):
        raise RuntimeError(f"expected input [B, {C}, {HW}, {HW}], got {tuple(input.shape)}")
    if tuple(weight.shape) != (K, K, C) or not weight.is_cuda:
        raise RuntimeError(f"weight must be a CUDA tensor [{K}, {K}, {C}], got {tuple(weight.shape)}")
    bp = dw_ops.check_vec(bias, C, "bias", input.device)  # empty tensor = no bias (reference :73)
    output = torch.empty_like(input)
    with dw_ops._DeviceGuard(input.device):
        stream = dw_ops._stream_of(input)
        if fn:
            _lib.call(fn, input.data_ptr(), weight.data_ptr(), bp or None, output.data_ptr(), B, Ci, Hi, Wi, stream)
        else:
            _lib.call("dwb_conv2d_nhwc_fused_fwd", input.data_ptr(), weight.data_ptr(), bp or None, None, None,
                      None, output.data_ptr(), B, Hi, Wi, Ci, K, _lib.ACT_NONE, _lib.ACCUM_DEFAULT, stream)
        _lib.after_launch(stream, fn or "dwb_conv2d_nhwc_fused_fwd")
    return output


# ---- torch.library custom op definitions ----
torch.library.define("replknet_dw::conv_56_128_31", "(Tensor input, Tensor weight, Tensor bias) -> Tensor")
torch.library.define("replknet_dw::conv_28_256_29", "(Tensor input, Tensor weight, Tensor bias) -> Tensor")
torch.library.define("replknet_dw::conv_14_512_27", "(Tensor input, Tensor weight, Tensor bias) -> Tensor")
torch.library.define("replknet_dw::conv_7_1024_13", "(Tensor input, Tensor weight, Tensor bias) -> Tensor")


@torch.library.impl("replknet_dw::conv_56_128_31", "default")
def _conv_56_128_31_impl(input, weight, bias):
    return _replknet_op("dwb_depthwise_31x31_128_nhwc", input, weight, bias, 128, 56, 31)


@torch.library.impl("replknet_dw::conv_28_256_29", "default")
def _conv_28_256_29_impl(input, weight, bias):
    return _replknet_op("dwb_depthwise_29x29_256_nhwc", input, weight, bias, 256, 28, 29)


@torch.library.impl("replknet_dw::conv_14_512_27", "default")
def _conv_14_512_27_impl(input, weight, bias):
    return _replknet_op("dwb_depthwise_27x27_512_nhwc", input, weight, bias, 512, 14, 27)


@torch.library.impl("replknet_dw::conv_7_1024_13", "default")
def _conv_7_1024_13_impl(input, weight, bias):
    return _replknet_op(None, input, weight, bias, 1024, 7, 13)


# ---- Fake (meta) implementations for torch.compile shape inference ----

@torch.library.register_fake("replknet_dw::conv_56_128_31")
def _conv_56_128_31_fake(input, weight, bias):
    return torch.empty_like(input)


@torch.library.register_fake("replknet_dw::conv_28_256_29")
def _conv_28_256_29_fake(input, weight, bias):
    return torch.empty_like(input)


@torch.library.register_fake("replknet_dw::conv_14_512_27")
def _conv_14_512_27_fake(input, weight, bias):
    return torch.empty_like(input)


@torch.library.register_fake("replknet_dw::conv_7_1024_13")
def _conv_7_1024_13_fake(input, weight, bias):
    return torch.empty_like(input)


# ---- nn.Module wrappers ----

class NHWCDepthwise31x31_128(nn.Module):
    """31x31 depthwise conv, 128ch, 56x56. Zero-copy NHWC."""

    def __init__(self):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(31, 31, 128, dtype=torch.float16))
        self.bias = nn.Parameter(torch.empty(128, dtype=torch.float16))
        _load_kernels()

    def forward(self, x):
        if dw_ops.direct_call_ok(x, self.weight, self.bias):  # eager inference: no dispatcher round trip
            return _replknet_op('dwb_depthwise_31x31_128_nhwc', x, self.weight, self.bias, 128, 56, 31)
        return torch.ops.replknet_dw.conv_56_128_31(x, self.weight, self.bias)


class NHWCDepthwise29x29_256(nn.Module):
    """29x29 depthwise conv, 256ch, 28x28. Zero-copy NHWC."""

    def __init__(self):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(29, 29, 256, dtype=torch.float16))
        self.bias = nn.Parameter(torch.empty(256, dtype=torch.float16))
        _load_kernels()

    def forward(self, x):
        if dw_ops.direct_call_ok(x, self.weight, self.bias):  # eager inference: no dispatcher round trip
            return _replknet_op('dwb_depthwise_29x29_256_nhwc', x, self.weight, self.bias, 256, 28, 29)
        return torch.ops.replknet_dw.conv_28_256_29(x, self.weight, self.bias)


class NHWCDepthwise27x27_512(nn.Module):
    """27x27 depthwise conv, 512ch, 14x14. Zero-copy NHWC."""

    def __init__(self):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(27, 27, 512, dtype=torch.float16))
        self.bias = nn.Parameter(torch.empty(512, dtype=torch.float16))
        _load_kernels()

    def forward(self, x):
        if dw_ops.direct_call_ok(x, self.weight, self.bias):  # eager inference: no dispatcher round trip
            return _replknet_op('dwb_depthwise_27x27_512_nhwc', x, self.weight, self.bias, 512, 14, 27)
        return torch.ops.replknet_dw.conv_14_512_27(x, self.weight, self.bias)


class NHWCDepthwise13x13_1024(nn.Module):
    """13x13 depthwise conv, 1024ch, 7x7 (RepLKNet stage 3). Zero-copy NHWC."""

    def __init__(self):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(13, 13, 1024, dtype=torch.float16))
        self.bias = nn.Parameter(torch.empty(1024, dtype=torch.float16))
        _load_kernels()

    def forward(self, x):
        if dw_ops.direct_call_ok(x, self.weight, self.bias):  # eager inference: no dispatcher round trip
            return _replknet_op(None, x, self.weight, self.bias, 1024, 7, 13)
        return torch.ops.replknet_dw.conv_7_1024_13(x, self.weight, self.bias)


# Map (channels, kernel_size) -> NHWC module class (reference :148-152, plus stage 3)
_REPLACEMENT_MAP = {
    (128, 31): NHWCDepthwise31x31_128,
    (256, 29): NHWCDepthwise29x29_256,
    (512, 27): NHWCDepthwise27x27_512,
    (1024, 13): NHWCDepthwise13x13_1024,
}


def replace_replknet_depthwise_nhwc(model, verbose=True, include_stage3=True):
    """Replace RepLKNet depthwise Conv2d layers with the NHWC engine modules (reference :155-210).

    Weights are repacked [C,1,K,K] -> [K,K,C] fp16; the bias is copied, or
    zeroed when the conv has none (reference :191-194).  With
    ``include_stage3=False`` the 13x13 stage stays on nn.Conv2d, as in the
    reference.
    """
    replaced = 0
    for name, module in list(model.named_modules()):
        if not isinstance(module, nn.Conv2d):
            continue
        if module.groups != module.in_channels or module.groups != module.out_channels:
            continue
        key = (module.in_channels, module.kernel_size[0])
        if key not in _REPLACEMENT_MAP or (key == (1024, 13) and not include_stage3):
            continue
        custom = _REPLACEMENT_MAP[key]().to(module.weight.device)
        with torch.no_grad():
            w = module.weight.squeeze(1).permute(1, 2, 0).contiguous().half()
            custom.weight.copy_(w)
            if module.bias is not None:
                custom.bias.copy_(module.bias.half())
            else:
                custom.bias.zero_()
        parts = name.split('.')
        parent = model
        for p in parts[:-1]:
            parent = getattr(parent, p)
        setattr(parent, parts[-1], custom)
        replaced += 1
        if verbose:
            print(f"  Replaced {name}: {key[0]}ch, {key[1]}x{key[1]} -> {custom.__class__.__name__}")
    if verbose:
        print(f"Replaced {replaced} depthwise conv(s) with NHWC custom kernels")
    return model
