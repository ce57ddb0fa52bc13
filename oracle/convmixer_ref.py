"""ConvMixer restated on the CPU in fp32 -- TEST INFRASTRUCTURE / CPU BASELINE ONLY.

The reference's model (convmixer/convmixer.py:62-134): patch conv -> act ->
BN, ``depth`` x [Residual(depthwise conv k, padding='same' -> act -> BN) ->
1x1 conv -> act -> BN], avg-pool, flatten, linear -- run through PyTorch's
CPU kernels, i.e. the depthwise layers go through ``F.conv2d(groups=C)`` in
fp32, which is the reference's CPU path for this op
(convmixer/convmixer.py:109, replknet/kernels/depthwise_replknet_nhwc_ops.py:16).

Weights follow the benchmark's random initialisation: conv/linear weights
N(0, 0.02) from a seeded CPU generator, biases 0, BN gamma 1 / beta 0 /
mean 0 / var 1 -- the same construction and the same generator sequence as
``depthwise_conv_b200.convmixer.init_baseline_``, so the two models hold
identical weights for the same seed.

Used by tests (end-to-end parity of the GPU model) and by bench.py's CPU
baseline / reference arm.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

CONFIGS = {
    '768_32': dict(dim=768, depth=32, kernel_size=7, patch_size=7, act='relu', n_classes=1000),
    '1536_20': dict(dim=1536, depth=20, kernel_size=9, patch_size=7, act='gelu', n_classes=1000),
}


class ConvMixerCPU(nn.Module):
    """fp32 ConvMixer with the reference's layer order, written as plain tensors."""

    def __init__(self, dim, depth, kernel_size, patch_size, act, n_classes, seed=0):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        rnd = lambda *shape: torch.randn(shape, generator=g) * 0.02  # noqa: E731
        self.dim, self.depth, self.k, self.p, self.act = dim, depth, kernel_size, patch_size, act
        # generator order mirrors nn.Module registration order of the GPU model:
        # patch conv, then per block DW conv then 1x1 conv, then the head.
        self.patch_w = rnd(dim, 3, patch_size, patch_size)
        self.dw_w, self.pw_w = [], []
        for _ in range(depth):
            self.dw_w.append(rnd(dim, 1, kernel_size, kernel_size))
            self.pw_w.append(rnd(dim, dim, 1, 1))
        self.head_w = rnd(n_classes, dim)
        self.eps = 1e-5

    def _act(self, x):
        return F.relu(x) if self.act == 'relu' else F.gelu(x)

    def _bn(self, x):
        # inference BN with gamma 1, beta 0, running mean 0, running var 1
        return x / (1.0 + self.eps) ** 0.5

    @torch.no_grad()
    def trunk(self, x, blocks=None):
        """Feature maps after the patch embedding and the first `blocks` blocks (all by default)."""
        x = x.float()
        x = self._bn(self._act(F.conv2d(x, self.patch_w, stride=self.p)))
        for i in range(self.depth if blocks is None else blocks):
            y = F.conv2d(x, self.dw_w[i], padding=self.k // 2, groups=self.dim)
            x = self._bn(self._act(y)) + x
            x = self._bn(self._act(F.conv2d(x, self.pw_w[i])))
        return x

    @torch.no_grad()
    def forward(self, x):
        x = self.trunk(x).mean(dim=(2, 3))
        return F.linear(x, self.head_w)


def convmixer_cpu(name: str, seed: int = 0) -> ConvMixerCPU:
    return ConvMixerCPU(**CONFIGS[name], seed=seed)
