"""Drop-in replacement for ``convmixer/kernels/depthwise_torch_ops.py``.

Same op names and schemas (depthwise_torch_ops.py:65-90), the same
"default" impls and fake impls (:93-154), the same ``CustomDepthwiseConv2d``
module and ``replace_depthwise_convs`` swapper (:162-340) -- backed by the
sm_100a engine through its C ABI instead of the reference's JIT-built
shape-specialised kernels.

Differences, all deliberate:

* the whole batch runs in one launch (the reference loops over images in
  Python for conv2d_32_768_7 / 16_1536_9 / 32_1536_13, :113,122,131);
* ``conv2d_32_1536_13`` is implemented (the reference stub calls exit(1),
  depthwise_integration.cu:1013-1030);
* a wrong shape, dtype or layout raises RuntimeError (the reference's
  launchers print and exit(1), depthwise_integration.cu:123-126);
* ``CustomDepthwiseConv2d`` fuses its bias into the kernel epilogue and
  accepts any (C, K, H) the engine supports (pass ``strict=True`` to keep the
  reference's ValueError for configurations outside SUPPORTED_CONFIGS).
"""
from __future__ import annotations

import os

import torch
import torch.nn as nn

from . import _lib
from . import dw_ops

_KERNELS_LOADED = False


def _load_kernels():
    """Load the engine's C-ABI library (the analogue of the reference's JIT build, :31-60)."""
    global _KERNELS_LOADED
    lib = _lib.load()
    _KERNELS_LOADED = True
    return lib


def _stream(t: torch.Tensor) -> int:
    return torch._C._cuda_getCurrentRawStream(t.device.index)


def _fixed_op(fn: str, input: torch.Tensor, weight: torch.Tensor, H: int, W: int, C: int, K: int,
              with_stride: bool) -> torch.Tensor:
    dw_ops.check_input(input)
    if not weight.is_cuda or weight.dtype != torch.float16 or not weight.is_contiguous():
        raise RuntimeError("weight must be a contiguous float16 CUDA tensor [K, K, C]")
    if tuple(weight.shape) != (K, K, C):
        raise RuntimeError(f"weight must be [{K}, {K}, {C}], got {tuple(weight.shape)}")
    B, Ci, Hi, Wi = input.shape
    output = torch.empty_like(input)
    args = [input.data_ptr(), weight.data_ptr(), output.data_ptr(), Hi, Wi, Ci, K, B]
    if with_stride:
        args.append(Hi * Wi * Ci)
    with dw_ops._DeviceGuard(input.device):
        stream = _stream(input)
        args.append(stream)
        _lib.call(fn, *args)
        _lib.after_launch(stream, fn)
    return output


# Ops accept channels_last [B, C, H, W] tensors (physical NHWC memory)
torch.library.define("depthwise::conv2d_32_1536_9", "(Tensor input, Tensor weight) -> Tensor")
torch.library.define("depthwise::conv2d_32_1536_9_v2", "(Tensor input, Tensor weight) -> Tensor")
torch.library.define("depthwise::conv2d_32_768_7", "(Tensor input, Tensor weight) -> Tensor")
torch.library.define("depthwise::conv2d_16_1536_9", "(Tensor input, Tensor weight) -> Tensor")
torch.library.define("depthwise::conv2d_32_1536_13", "(Tensor input, Tensor weight) -> Tensor")


@torch.library.impl("depthwise::conv2d_32_1536_9", "default")
def _depthwise_conv2d_32_1536_9_impl(input, weight):
    return _fixed_op("dwb_depthwise_forward_32_1536_9", input, weight, 32, 32, 1536, 9, True)


@torch.library.impl("depthwise::conv2d_32_1536_9_v2", "default")
def _depthwise_conv2d_32_1536_9_v2_impl(input, weight):
    return _fixed_op("dwb_depthwise_forward_32_1536_9_v2", input, weight, 32, 32, 1536, 9, True)


@torch.library.impl("depthwise::conv2d_32_768_7", "default")
def _depthwise_conv2d_32_768_7_impl(input, weight):
    return _fixed_op("dwb_depthwise_forward_32_768_7", input, weight, 32, 32, 768, 7, False)


@torch.library.impl("depthwise::conv2d_16_1536_9", "default")
def _depthwise_conv2d_16_1536_9_impl(input, weight):
    return _fixed_op("dwb_depthwise_forward_16_1536_9", input, weight, 16, 16, 1536, 9, False)


@torch.library.impl("depthwise::conv2d_32_1536_13", "default")
def _depthwise_conv2d_32_1536_13_impl(input, weight):
    return _fixed_op("dwb_depthwise_forward_32_1536_13", input, weight, 32, 32, 1536, 13, False)


@torch.library.register_fake("depthwise::conv2d_32_1536_9")
def _depthwise_conv2d_32_1536_9_fake(input, weight):
    return torch.empty_like(input)


@torch.library.register_fake("depthwise::conv2d_32_1536_9_v2")
def _depthwise_conv2d_32_1536_9_v2_fake(input, weight):
    return torch.empty_like(input)


@torch.library.register_fake("depthwise::conv2d_32_768_7")
def _depthwise_conv2d_32_768_7_fake(input, weight):
    return torch.empty_like(input)


@torch.library.register_fake("depthwise::conv2d_16_1536_9")
def _depthwise_conv2d_16_1536_9_fake(input, weight):
    return torch.empty_like(input)


@torch.library.register_fake("depthwise::conv2d_32_1536_13")
def _depthwise_conv2d_32_1536_13_fake(input, weight):
    return torch.empty_like(input)


# (op name) -> the C entry point and fixed shape its "default" impl launches; the modules call
# _fixed_op with these directly in eager inference (torch.library.impl used as a decorator does not
# return the function, so the impls above cannot be called by name)
_FIXED_ARGS = {
    'depthwise::conv2d_32_1536_9': ("dwb_depthwise_forward_32_1536_9", 32, 32, 1536, 9, True),
    'depthwise::conv2d_32_1536_9_v2': ("dwb_depthwise_forward_32_1536_9_v2", 32, 32, 1536, 9, True),
    'depthwise::conv2d_32_768_7': ("dwb_depthwise_forward_32_768_7", 32, 32, 768, 7, False),
    'depthwise::conv2d_16_1536_9': ("dwb_depthwise_forward_16_1536_9", 16, 16, 1536, 9, False),
    'depthwise::conv2d_32_1536_13': ("dwb_depthwise_forward_32_1536_13", 32, 32, 1536, 13, False),
}


class CustomDepthwiseConv2d(nn.Module):
    """Depthwise conv on the B200 engine; drop-in for the reference module (:162-265).

    Replaces ``nn.Conv2d(channels, channels, kernel_size, groups=channels,
    padding=kernel_size//2)``.  Input/output: float16, channels_last.
    The weight is stored [K, K, C] like the reference.
    """

    # 32x32x1536 9x9 op selected by DEPTHWISE_9X9_VARIANT env var (default v1), as in the reference.
    SUPPORTED_CONFIGS = {
        (768, 7, 32): 'depthwise::conv2d_32_768_7',
        (1536, 9, 32): ('depthwise::conv2d_32_1536_9_v2'
                        if os.environ.get('DEPTHWISE_9X9_VARIANT', 'v1') == 'v2'
                        else 'depthwise::conv2d_32_1536_9'),
        (1536, 9, 16): 'depthwise::conv2d_16_1536_9',
        (1536, 13, 32): 'depthwise::conv2d_32_1536_13',
    }

    def __init__(self, channels, kernel_size, bias=True, strict=False):
        super().__init__()
        self.channels = channels
        self.kernel_size = kernel_size
        self.padding = kernel_size // 2
        self.strict = strict
        self.weight = nn.Parameter(torch.randn(kernel_size, kernel_size, channels, dtype=torch.float16))
        if bias:
            self.bias = nn.Parameter(torch.zeros(channels, dtype=torch.float16))
        else:
            self.register_parameter('bias', None)
        _load_kernels()
        self.spatial_size = None
        self.op_name = None

    def _get_op_name(self, spatial_size):
        config = (self.channels, self.kernel_size, spatial_size)
        if config not in self.SUPPORTED_CONFIGS:
            if self.strict:
                raise ValueError(
                    f"Unsupported configuration: {self.channels} channels, "
                    f"{self.kernel_size}×{self.kernel_size} kernel, "
                    f"{spatial_size}×{spatial_size} spatial. "
                    f"Supported configs: {list(self.SUPPORTED_CONFIGS.keys())}")
            return 'depthwise::conv2d_nhwc'
        return self.SUPPORTED_CONFIGS[config]

    def forward(self, x):
        B, C, H, W = x.shape
        if self.spatial_size is None:
            self.spatial_size = H
            self.op_name = self._get_op_name(H)
        if dw_ops.direct_call_ok(x, self.weight, self.bias):
            # eager inference: the op's own implementation, without the dispatcher round trip
            # (the same kernel launch; torch.compile and autograd keep going through the ops)
            if self.bias is not None or self.op_name == 'depthwise::conv2d_nhwc':
                return dw_ops.conv2d_nhwc_fused(x, self.weight, bias=self.bias)
            fn, H_, W_, C_, K_, stride = _FIXED_ARGS[self.op_name]
            return _fixed_op(fn, x, self.weight, H_, W_, C_, K_, stride)
        if self.bias is not None or self.op_name == 'depthwise::conv2d_nhwc':
            # bias fused into the kernel epilogue (one launch instead of conv + add)
            return torch.ops.depthwise.conv2d_nhwc(x, self.weight, self.bias)
        if self.op_name == 'depthwise::conv2d_32_1536_9':
            return torch.ops.depthwise.conv2d_32_1536_9(x, self.weight)
        if self.op_name == 'depthwise::conv2d_32_1536_9_v2':
            return torch.ops.depthwise.conv2d_32_1536_9_v2(x, self.weight)
        if self.op_name == 'depthwise::conv2d_32_768_7':
            return torch.ops.depthwise.conv2d_32_768_7(x, self.weight)
        if self.op_name == 'depthwise::conv2d_16_1536_9':
            return torch.ops.depthwise.conv2d_16_1536_9(x, self.weight)
        if self.op_name == 'depthwise::conv2d_32_1536_13':
            return torch.ops.depthwise.conv2d_32_1536_13(x, self.weight)
        raise RuntimeError(f"Unknown operator: {self.op_name}")

    def extra_repr(self):
        s = f'{self.channels}, kernel_size={self.kernel_size}'
        if self.bias is not None:
            s += ', bias=True'
        if self.spatial_size is not None:
            s += f', spatial_size={self.spatial_size}'
            s += f', op={self.op_name}'
        return s


def replace_depthwise_convs(model, verbose=True, any_shape=False):
    """Replace depthwise ``nn.Conv2d`` layers with ``CustomDepthwiseConv2d`` (reference :268-340).

    A layer is replaced when ``groups == in_channels == out_channels`` and,
    as in the reference, its (C, K) matches SUPPORTED_CONFIGS at 32x32 or
    16x16 -- or for any odd K <= 31 with ``any_shape=True``.  Weights are
    repacked [C,1,K,K] -> [K,K,C] fp16 and the bias is copied.
    """
    replaced = 0
    for name, module in list(model.named_modules()):
        if not isinstance(module, nn.Conv2d):
            continue
        if not (module.groups == module.in_channels == module.out_channels):
            continue
        channels = module.in_channels
        kernel_size = module.kernel_size[0]
        supported = ((channels, kernel_size, 32) in CustomDepthwiseConv2d.SUPPORTED_CONFIGS or
                     (channels, kernel_size, 16) in CustomDepthwiseConv2d.SUPPORTED_CONFIGS)
        generic_ok = (any_shape and module.kernel_size[0] == module.kernel_size[1] and kernel_size % 2 == 1
                      and kernel_size <= 31 and module.stride == (1, 1) and module.dilation == (1, 1)
                      and channels % 8 == 0)
        if not (supported or generic_ok):
            continue
        custom_conv = CustomDepthwiseConv2d(channels, kernel_size, bias=(module.bias is not None))
        custom_conv = custom_conv.to(module.weight.device)
        with torch.no_grad():
            # PyTorch: [C, 1, K, K] -> engine: [K, K, C]
            weight_custom = module.weight.squeeze(1).permute(1, 2, 0).contiguous()
            custom_conv.weight.copy_(weight_custom.to(dtype=torch.float16, device=module.weight.device))
            if module.bias is not None and custom_conv.bias is not None:
                custom_conv.bias.copy_(module.bias.to(dtype=torch.float16, device=module.bias.device))
        parent_name = '.'.join(name.split('.')[:-1])
        child_name = name.split('.')[-1]
        parent = model.get_submodule(parent_name) if parent_name else model
        setattr(parent, child_name, custom_conv)
        replaced += 1
        if verbose:
            print(f"Replaced {name}: {channels} channels, {kernel_size}x{kernel_size} kernel")
    if verbose:
        print(f"Replaced {replaced} depthwise convolution(s) with torch.library custom ops")
    return model
