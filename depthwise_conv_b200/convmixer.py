"""ConvMixer host model for the end-to-end metric, with the engine's fused DW block.

The network follows the reference's ``convmixer/convmixer.py`` layer for
layer (``ConvMixerWrapper`` :62-161, configs :17-42): patch conv -> act ->
BN, then ``depth`` blocks of [Residual(DW conv -> act -> BN) -> 1x1 conv ->
act -> BN], then avg-pool, flatten, linear.  Weights are random, initialised
as the benchmark configuration prescribes (no checkpoints are involved):
conv/linear weights N(0, 0.02), biases 0, BN gamma=1 beta=0, running mean 0,
running var 1.

``fuse_dw_blocks`` swaps each Residual(DW conv, act, BN) for one
``depthwise::conv2d_nhwc_fused`` call that computes
``act(conv(x) + b) * s + t + x`` in a single kernel, with s, t the
inference-mode BN fold (benchmark_cudnn_fused_e2e.py:115-134, :125-131), and
each 1x1 conv -> act -> BN (and the patch-conv stem) for a GEMM plus one
fused elementwise kernel.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import dw_ops  # noqa: F401  (registers depthwise::conv2d_nhwc_fused)

CONVMIXER_MODELS = {
    '768_32': {'dim': 768, 'depth': 32, 'kernel_size': 7, 'patch_size': 7, 'activation': 'relu', 'n_classes': 1000},
    '1024_20': {'dim': 1024, 'depth': 20, 'kernel_size': 9, 'patch_size': 14, 'activation': 'gelu',
                'n_classes': 1000},
    '1536_20': {'dim': 1536, 'depth': 20, 'kernel_size': 9, 'patch_size': 7, 'activation': 'gelu',
                'n_classes': 1000},
}


class Residual(nn.Module):
    def __init__(self, fn):
        super().__init__()
        self.fn = fn

    def forward(self, x):
        return self.fn(x) + x


class ConvMixer(nn.Module):
    """Same Sequential indexing as the reference's ConvMixerWrapper (convmixer/convmixer.py:93-127)."""

    def __init__(self, dim, depth, kernel_size=9, patch_size=7, n_classes=1000, activation='gelu'):
        super().__init__()
        self.dim, self.depth, self.kernel_size = dim, depth, kernel_size
        self.patch_size, self.n_classes, self.activation = patch_size, n_classes, activation
        act_fn = nn.ReLU if activation == 'relu' else nn.GELU
        layers = [nn.Conv2d(3, dim, kernel_size=patch_size, stride=patch_size), act_fn(), nn.BatchNorm2d(dim)]
        for _ in range(depth):
            layers.append(nn.Sequential(
                Residual(nn.Sequential(
                    nn.Conv2d(dim, dim, kernel_size, groups=dim, padding='same'),
                    act_fn(),
                    nn.BatchNorm2d(dim))),
                nn.Conv2d(dim, dim, kernel_size=1),
                act_fn(),
                nn.BatchNorm2d(dim)))
        layers += [nn.AdaptiveAvgPool2d((1, 1)), nn.Flatten(), nn.Linear(dim, n_classes)]
        self.model = nn.Sequential(*layers)

    def forward(self, x):
        if not x.is_contiguous(memory_format=torch.channels_last):
            x = x.contiguous(memory_format=torch.channels_last)
        return self.model(x)


def init_baseline_(model: nn.Module, seed: int = 0) -> nn.Module:
    """Random init of the benchmark configuration (seeded, CPU generator)."""
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for m in model.modules():
            if isinstance(m, (nn.Conv2d, nn.Linear)):
                m.weight.copy_(torch.randn(m.weight.shape, generator=g) * 0.02)
                if m.bias is not None:
                    m.bias.zero_()
            elif isinstance(m, nn.BatchNorm2d):
                m.weight.fill_(1.0)
                m.bias.zero_()
                m.running_mean.zero_()
                m.running_var.fill_(1.0)
    return model


def convmixer(name: str, seed: int = 0) -> ConvMixer:
    cfg = CONVMIXER_MODELS[name]
    return init_baseline_(ConvMixer(**cfg), seed).eval()


class FusedDWBlock(nn.Module):
    """Residual(DW conv -> act -> BN) as one engine kernel: act(conv(x) + b) * s + t + x."""

    def __init__(self, conv: nn.Conv2d, act: str, bn: nn.BatchNorm2d):
        super().__init__()
        C = conv.in_channels
        self.act = act
        with torch.no_grad():
            w = conv.weight.detach().squeeze(1).permute(1, 2, 0).contiguous().half()  # [K,K,C]
            b = conv.bias.detach().half() if conv.bias is not None else torch.zeros(C, dtype=torch.float16)
            scale = bn.weight / torch.sqrt(bn.running_var + bn.eps)
            shift = bn.bias - bn.running_mean * scale
        self.register_buffer("weight", w)
        self.register_buffer("bias", b.contiguous())
        self.register_buffer("scale", scale.half().contiguous())
        self.register_buffer("shift", shift.half().contiguous())
        self.act_code = dw_ops.ACT_CODES[act]

    def forward(self, x):
        return torch.ops.depthwise.conv2d_nhwc_fused(x, self.weight, self.bias, self.scale, self.shift, x,
                                                     self.act_code)


def _epilogue(z, bias, scale, shift, act):
    """act(z + bias) * scale + shift: in place in eager mode; under torch.compile through the
    registered op ``depthwise::bias_act_affine`` (out of place, so the graph stays functional)."""
    if torch.compiler.is_compiling():
        return torch.ops.depthwise.bias_act_affine(z, bias, scale, shift, dw_ops.ACT_CODES[act])
    return dw_ops.bias_act_affine(z, bias, scale, shift, act, out=z)


class FusedPointwiseBlock(nn.Module):
    """1x1 conv -> act -> BN as a cuBLAS GEMM on the NHWC pixels plus one elementwise pass.

    channels_last data is a [B*H*W, C] row-major matrix, so the 1x1 convolution is
    z = X @ W^T with no layout change; ``bias_act_affine`` then applies the bias,
    the activation and the inference BatchNorm (scale/shift) in one kernel.
    """

    def __init__(self, conv: nn.Conv2d, act: str, bn: nn.BatchNorm2d):
        super().__init__()
        C_out, C_in = conv.out_channels, conv.in_channels
        with torch.no_grad():
            w = conv.weight.detach().reshape(C_out, C_in).t().contiguous().half()  # [C_in, C_out]
            b = conv.bias.detach().half() if conv.bias is not None else torch.zeros(C_out, dtype=torch.float16)
            scale = bn.weight / torch.sqrt(bn.running_var + bn.eps)
            shift = bn.bias - bn.running_mean * scale
        self.register_buffer("weight_t", w)
        self.register_buffer("bias", b.contiguous())
        self.register_buffer("scale", scale.half().contiguous())
        self.register_buffer("shift", shift.half().contiguous())
        self.act = act

    def forward(self, x):
        B, C, H, W = x.shape
        z = torch.mm(x.permute(0, 2, 3, 1).reshape(B * H * W, C), self.weight_t)  # [BHW, C_out], NHWC
        z = z.view(B, H, W, -1).permute(0, 3, 1, 2)  # channels_last view
        return _epilogue(z, self.bias, self.scale, self.shift, self.act)


def patch_matrix(x: torch.Tensor, p: int, k_pad: int) -> torch.Tensor:
    """The non-overlapping p x p patches of an image batch as a [B*Ho*Wo, k_pad] row-major matrix.

    Row (b, ho, wo) holds the patch's taps in (kh, kw, c_in) order, so a patch
    convolution (stride = kernel, no padding) is this matrix times its weight
    arranged [kh, kw, c_in] x C_out, and the product is already NHWC.  Columns
    past p*p*C_in are zero (rows padded to a multiple of 8 halves keep the GEMM's
    operand rows 16-byte aligned).  One copy for the rearrangement plus one fill.
    """
    B, Cin, H, W = x.shape
    Ho, Wo = H // p, W // p
    K = p * p * Cin
    xs = x[:, :, :Ho * p, :Wo * p].permute(0, 2, 3, 1).reshape(B, Ho, p, Wo, p, Cin)  # NHWC patches
    a = x.new_zeros(B * Ho * Wo, k_pad) if k_pad > K else x.new_empty(B * Ho * Wo, K)
    a[:, :K].view(B, Ho, Wo, p, p, Cin).copy_(xs.permute(0, 1, 3, 2, 4, 5))
    return a


class FusedStem(nn.Module):
    """Patch conv -> act -> BN.

    With stride = kernel and no padding (every ConvMixer stem) the patches do
    not overlap and the convolution is one GEMM: ``patch_matrix`` times the
    [p*p*C_in, C] weight (cuBLAS), whose output is the NHWC activation, then one
    elementwise pass for the bias, the activation and the BN fold.  Any other
    stem runs cuDNN's convolution before the same elementwise pass.
    """

    def __init__(self, conv: nn.Conv2d, act: str, bn: nn.BatchNorm2d):
        super().__init__()
        C = conv.out_channels
        with torch.no_grad():
            b = conv.bias.detach().half() if conv.bias is not None else torch.zeros(C, dtype=torch.float16)
            scale = bn.weight / torch.sqrt(bn.running_var + bn.eps)
            shift = bn.bias - bn.running_mean * scale
        self.register_buffer("weight", conv.weight.detach().half().contiguous(memory_format=torch.channels_last))
        self.register_buffer("bias", b.contiguous())
        self.register_buffer("scale", scale.half().contiguous())
        self.register_buffer("shift", shift.half().contiguous())
        self.stride = conv.stride
        self.act = act
        kh, kw = conv.kernel_size
        self.patch = kh if (kh == kw and conv.stride == (kh, kw) and conv.groups == 1 and conv.dilation == (1, 1)
                            and conv.padding in ((0, 0), "valid")) else 0
        if self.patch:
            K = kh * kw * conv.in_channels
            self.k_pad = (K + 7) // 8 * 8
            with torch.no_grad():
                wt = torch.zeros(self.k_pad, C, dtype=torch.float16, device=conv.weight.device)
                wt[:K] = conv.weight.detach().permute(2, 3, 1, 0).reshape(K, C).half()  # [kh, kw, c_in] x C
            self.register_buffer("weight_t", wt)

    def forward(self, x):
        if self.patch:
            B, _, H, W = x.shape
            Ho, Wo = H // self.patch, W // self.patch
            z = torch.mm(patch_matrix(x, self.patch, self.k_pad), self.weight_t)  # [B*Ho*Wo, C], NHWC
            z = z.view(B, Ho, Wo, -1).permute(0, 3, 1, 2)  # channels_last view
        else:
            z = torch.nn.functional.conv2d(x, self.weight, None, self.stride)
            if not z.is_contiguous(memory_format=torch.channels_last):
                z = z.contiguous(memory_format=torch.channels_last)
        return _epilogue(z, self.bias, self.scale, self.shift, self.act)


def fuse_dw_blocks(model: ConvMixer, pointwise: bool = True) -> ConvMixer:
    """Replace every Residual(DW conv, act, BN) of a ConvMixer with a FusedDWBlock and, with
    ``pointwise``, every 1x1 conv -> act -> BN with a FusedPointwiseBlock."""
    n = 0
    for block in model.model:
        if not isinstance(block, nn.Sequential):
            continue
        for i, sub in enumerate(block):
            if isinstance(sub, Residual) and isinstance(sub.fn, nn.Sequential) and len(sub.fn) == 3:
                conv, act, bn = sub.fn
                if isinstance(conv, nn.Conv2d) and conv.groups == conv.in_channels == conv.out_channels:
                    act_name = 'relu' if isinstance(act, nn.ReLU) else 'gelu'
                    block[i] = FusedDWBlock(conv, act_name, bn).to(conv.weight.device)
                    n += 1
        if pointwise and len(block) == 4 and isinstance(block[1], nn.Conv2d) and block[1].kernel_size == (1, 1):
            conv, act, bn = block[1], block[2], block[3]
            act_name = 'relu' if isinstance(act, nn.ReLU) else 'gelu'
            fused = FusedPointwiseBlock(conv, act_name, bn).to(conv.weight.device)
            block[1], block[2], block[3] = fused, nn.Identity(), nn.Identity()
    if pointwise and isinstance(model.model[0], nn.Conv2d) and isinstance(model.model[2], nn.BatchNorm2d):
        conv, act, bn = model.model[0], model.model[1], model.model[2]
        act_name = 'relu' if isinstance(act, nn.ReLU) else 'gelu'
        model.model[0] = FusedStem(conv, act_name, bn).to(conv.weight.device)
        model.model[1], model.model[2] = nn.Identity(), nn.Identity()
    model.fused_blocks = n
    return model
