"""Tensor-level entry points of the engine and the generic torch ops.

Everything here validates tensors, allocates the output with the torch
caching allocator and calls the C ABI on ``torch.cuda.current_stream()``;
the arithmetic happens only in ``libdwconv_b200.so``.  There is no CPU or
PyTorch fallback: a CPU tensor, a wrong dtype or layout raises RuntimeError.

Generic ops (new; the reference only has fixed-shape ops):

* ``depthwise::conv2d_nhwc(Tensor input, Tensor weight, Tensor? bias=None) -> Tensor``
* ``depthwise::conv2d_nhwc_fused(Tensor input, Tensor weight, Tensor? bias, Tensor? scale,
  Tensor? shift, Tensor? residual, int act) -> Tensor`` computing
  ``act(conv + bias) * scale + shift + residual`` in one kernel -- the
  semantics of the reference's fused baseline
  (benchmark_cudnn_fused_e2e.py:44-84,115-134) plus ConvMixer's residual
  (convmixer/convmixer.py:58-59).

``depthwise::conv2d_nhwc`` and ``depthwise::conv2d_nhwc_fused`` are
differentiable (``torch.library.register_autograd``): the input gradient runs
the forward kernel on dy with the taps rotated by 180 degrees, the weight
gradient a dedicated kernel accumulating in fp32, the bias gradient a channel
sum; the fused op recomputes its pre-activation with the engine and takes the
elementwise adjoints (activation, BN scale/shift, residual) in fp32.  The
reference's ops are inference-only.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

ACT_CODES = _lib.ACT_CODES


def _stream_of(t: torch.Tensor) -> int:
    """Raw handle of PyTorch's current stream on the tensor's device (no Stream object is built)."""
    return torch._C._cuda_getCurrentRawStream(t.device.index)


def check_input(x: torch.Tensor, name: str = "input") -> None:
    if not x.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (the engine has no CPU path)")
    if x.dtype != torch.float16:
        raise RuntimeError(f"{name} must be float16, got {x.dtype}")
    if x.dim() != 4:
        raise RuntimeError(f"{name} must be 4-D [B, C, H, W], got {tuple(x.shape)}")
    if not x.is_contiguous(memory_format=torch.channels_last):
        raise RuntimeError(f"{name} must be channels_last")


def check_weight(w: torch.Tensor, C: int) -> int:
    if not w.is_cuda or w.dtype != torch.float16:
        raise RuntimeError("weight must be a float16 CUDA tensor")
    if w.dim() != 3 or w.shape[0] != w.shape[1] or w.shape[2] != C or not w.is_contiguous():
        raise RuntimeError(f"weight must be contiguous [K, K, C={C}], got {tuple(w.shape)}")
    return int(w.shape[0])


def check_vec(v, C: int, name: str, device) -> int:
    if v is None or v.numel() == 0:
        return 0
    if not v.is_cuda or v.dtype != torch.float16 or v.numel() != C or not v.is_contiguous():
        raise RuntimeError(f"{name} must be a contiguous float16 CUDA tensor with {C} elements")
    if v.device != device:
        raise RuntimeError(f"{name} is on {v.device}, input on {device}")
    return v.data_ptr()


class _DeviceGuard:
    """Make the tensor's device current for the C ABI (cheap when it already is)."""

    __slots__ = ("idx", "prev")

    def __init__(self, device: torch.device):
        self.idx = device.index
        self.prev = None

    def __enter__(self):
        cur = torch._C._cuda_getDevice()
        if cur != self.idx:
            self.prev = cur
            torch.cuda.set_device(self.idx)

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


def direct_call_ok(*tensors) -> bool:
    """Whether a module may call the op's implementation directly instead of through torch.ops:
    eager mode (not tracing for torch.compile) and no gradient needed for any of ``tensors``."""
    if torch.compiler.is_compiling():
        return False
    if torch.is_grad_enabled():
        for t in tensors:
            if t is not None and t.requires_grad:
                return False
    return True


def conv2d_nhwc_fused(x: torch.Tensor, w: torch.Tensor, bias=None, scale=None, shift=None, residual=None,
                      act: int | str = 0, accum: int = _lib.ACCUM_DEFAULT, out: torch.Tensor | None = None,
                      plan: dict | None = None):
    """y = act(conv(x, w) + bias) * scale + shift + residual (each term optional).

    x: channels_last [B, C, H, W] fp16; w: [K, K, C] fp16.  Returns y like x.
    ``accum``: ``_lib.ACCUM_MIXED`` (default; fp16x2 FMA chains of at most 24
    taps added into fp32 accumulators) or ``_lib.ACCUM_F32`` (every tap in fp32).
    ``plan``: an explicit launch plan (a dict from ``plan_candidates``) instead
    of the planner's choice -- for autotuning.
    """
    check_input(x)
    B, C, H, W = x.shape
    K = check_weight(w, C)
    if w.device != x.device:
        raise RuntimeError(f"weight is on {w.device}, input on {x.device}")
    act_code = ACT_CODES[act] if isinstance(act, str) else int(act)
    bp = check_vec(bias, C, "bias", x.device)
    sp = check_vec(scale, C, "scale", x.device)
    hp = check_vec(shift, C, "shift", x.device)
    rp = 0
    if residual is not None:
        check_input(residual, "residual")
        if residual.shape != x.shape or residual.device != x.device:
            raise RuntimeError("residual must match input in shape and device")
        rp = residual.data_ptr()
    y = torch.empty_like(x, memory_format=torch.channels_last) if out is None else out
    if out is not None:
        check_input(out, "out")
        if out.shape != x.shape:
            raise RuntimeError("out must match input in shape")
    with _DeviceGuard(x.device):
        stream = _stream_of(x)
        if plan is None:
            _lib.call("dwb_conv2d_nhwc_fused_fwd", x.data_ptr(), w.data_ptr(), bp or None, sp or None, hp or None,
                      rp or None, y.data_ptr(), B, H, W, C, K, act_code, int(accum), stream)
        else:
            pl = _lib.Plan.from_dict(plan)
            _lib.call("dwb_conv2d_nhwc_fwd_planned", x.data_ptr(), w.data_ptr(), bp or None, sp or None,
                      hp or None, rp or None, y.data_ptr(), B, H, W, C, K, act_code, ctypes.byref(pl), stream)
        _lib.after_launch(stream, "depthwise conv2d_nhwc_fused")
    return y


def bias_act_affine(x: torch.Tensor, bias=None, scale=None, shift=None, act: int | str = 0,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """y = act(x + bias) * scale + shift per channel, for a channels_last fp16 CUDA tensor [B, C, H, W]."""
    check_input(x)
    B, C, H, W = x.shape
    act_code = ACT_CODES[act] if isinstance(act, str) else int(act)
    bp = check_vec(bias, C, "bias", x.device)
    sp = check_vec(scale, C, "scale", x.device)
    hp = check_vec(shift, C, "shift", x.device)
    y = torch.empty_like(x) if out is None else out
    if out is not None:
        check_input(out, "out")
    with _DeviceGuard(x.device):
        _lib.call("dwb_bias_act_affine_nhwc", x.data_ptr(), bp or None, sp or None, hp or None, y.data_ptr(),
                  B * H * W, C, act_code, _stream_of(x))
        _lib.after_launch(_stream_of(x), "depthwise bias_act_affine")
    return y


def pointwise_gemm(a: torch.Tensor, w: torch.Tensor, bias=None, scale=None, shift=None, act: int | str = 0,
                   out: torch.Tensor | None = None, tile_n: int = 0) -> torch.Tensor:
    """y = act(a @ w^T + bias) * scale + shift as one tensor-core kernel (``dwb_pointwise_conv_nhwc``).

    ``a``: [M, K] fp16 CUDA, row-major (the NHWC pixels of a channels_last tensor, or a patch
    matrix); ``w``: [N, K] fp16 row-major (a 1x1 convolution's weight as PyTorch stores it);
    bias/scale/shift: [N] or None.  Returns [M, N] fp16 (NHWC pixels x output channels);
    accumulation in fp32.  ``tile_n`` forces the output-channel tile (64, 96, 128, 256).
    """
    if not a.is_cuda or a.dtype != torch.float16 or a.dim() != 2 or not a.is_contiguous():
        raise RuntimeError(f"input must be a contiguous float16 CUDA matrix [M, K], got {tuple(a.shape)}")
    if w.dim() == 4 and w.shape[2:] == (1, 1):
        w = w.reshape(w.shape[0], w.shape[1])
    if not w.is_cuda or w.dtype != torch.float16 or w.dim() != 2 or w.shape[1] != a.shape[1] or not w.is_contiguous():
        raise RuntimeError(f"weight must be a contiguous float16 CUDA matrix [N, K={a.shape[1]}], got {tuple(w.shape)}")
    if w.device != a.device:
        raise RuntimeError(f"weight is on {w.device}, input on {a.device}")
    M, K = a.shape
    N = w.shape[0]
    act_code = ACT_CODES[act] if isinstance(act, str) else int(act)
    bp = check_vec(bias, N, "bias", a.device)
    sp = check_vec(scale, N, "scale", a.device)
    hp = check_vec(shift, N, "shift", a.device)
    if out is None:
        y = torch.empty((M, N), dtype=torch.float16, device=a.device)
    else:
        if not out.is_cuda or out.dtype != torch.float16 or out.shape != (M, N) or not out.is_contiguous():
            raise RuntimeError(f"out must be a contiguous float16 CUDA matrix [{M}, {N}]")
        y = out
    with _DeviceGuard(a.device):
        stream = _stream_of(a)
        _lib.call("dwb_pointwise_conv_nhwc", a.data_ptr(), w.data_ptr(), bp or None, sp or None, hp or None,
                  y.data_ptr(), M, K, N, act_code, int(tile_n), stream)
        _lib.after_launch(stream, "depthwise pointwise_gemm")
    return y


def pointwise_conv_nhwc(x: torch.Tensor, w: torch.Tensor, bias=None, scale=None, shift=None,
                        act: int | str = 0) -> torch.Tensor:
    """A 1x1 convolution with its bias, activation and BN fold on a channels_last fp16 tensor
    [B, C_in, H, W]; ``w``: [C_out, C_in] (or [C_out, C_in, 1, 1]).  Returns channels_last
    [B, C_out, H, W] -- the pixel matrix needs no layout change on either side."""
    check_input(x)
    B, C, H, W = x.shape
    z = pointwise_gemm(x.permute(0, 2, 3, 1).reshape(B * H * W, C), w, bias, scale, shift, act)
    return z.view(B, H, W, -1).permute(0, 3, 1, 2)


def weight_rot180(w: torch.Tensor) -> torch.Tensor:
    """[K, K, C] taps rotated by 180 degrees (the input-gradient filter)."""
    C = w.shape[2]
    check_weight(w, C)
    wr = torch.empty_like(w)
    with _DeviceGuard(w.device):
        _lib.call("dwb_weight_rot180", w.data_ptr(), wr.data_ptr(), C, w.shape[0], _stream_of(w))
    return wr


def conv2d_nhwc_backward_input(dy: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """dx of y = conv(x, w): the convolution of dy with the rotated taps."""
    check_input(dy, "grad_output")
    B, C, H, W = dy.shape
    K = check_weight(w, C)
    wr = weight_rot180(w)
    dx = torch.empty_like(dy)
    with _DeviceGuard(dy.device):
        _lib.call("dwb_conv2d_nhwc_bwd_data", dy.data_ptr(), wr.data_ptr(), dx.data_ptr(), B, H, W, C, K,
                  _stream_of(dy))
        _lib.after_launch(_stream_of(dy), "depthwise conv2d_nhwc input gradient")
    return dx


def conv2d_nhwc_backward_weight(x: torch.Tensor, dy: torch.Tensor, K: int, deterministic: bool | None = None
                                ) -> torch.Tensor:
    """dw of y = conv(x, w) as [K, K, C] float32 (summed over the batch and the image).

    ``deterministic`` (default: ``torch.are_deterministic_algorithms_enabled()``) sums the partial
    sums in a fixed order through a workspace instead of adding them atomically, so repeated calls
    give the same bits."""
    check_input(x)
    check_input(dy, "grad_output")
    if dy.shape != x.shape:
        raise RuntimeError(f"grad_output shape {tuple(dy.shape)} != input shape {tuple(x.shape)}")
    B, C, H, W = x.shape
    if deterministic is None:
        deterministic = torch.are_deterministic_algorithms_enabled()
    dw = torch.zeros((K, K, C), dtype=torch.float32, device=x.device)
    with _DeviceGuard(x.device):
        if deterministic:
            nbytes = ctypes.c_int64(0)
            _lib.call("dwb_conv2d_nhwc_bwd_weight_workspace", B, H, W, C, K, ctypes.byref(nbytes))
            ws = torch.empty(max(16, nbytes.value), dtype=torch.uint8, device=x.device)
            _lib.call("dwb_conv2d_nhwc_bwd_weight_det", x.data_ptr(), dy.data_ptr(), dw.data_ptr(), ws.data_ptr(),
                      nbytes.value, B, H, W, C, K, _stream_of(x))
        else:
            _lib.call("dwb_conv2d_nhwc_bwd_weight", x.data_ptr(), dy.data_ptr(), dw.data_ptr(), B, H, W, C, K,
                      _stream_of(x))
        _lib.after_launch(_stream_of(x), "depthwise conv2d_nhwc weight gradient")
    return dw


def conv2d_nhwc(x: torch.Tensor, w: torch.Tensor, bias=None) -> torch.Tensor:
    """y = conv(x, w) (+ bias): the plain depthwise convolution."""
    return conv2d_nhwc_fused(x, w, bias=bias)


# ---- generic torch.library ops ---------------------------------------------------

torch.library.define("depthwise::conv2d_nhwc", "(Tensor input, Tensor weight, Tensor? bias=None) -> Tensor")
torch.library.define(
    "depthwise::conv2d_nhwc_fused",
    "(Tensor input, Tensor weight, Tensor? bias, Tensor? scale, Tensor? shift, Tensor? residual, int act) -> Tensor",
)
torch.library.define(
    "depthwise::bias_act_affine",
    "(Tensor input, Tensor? bias, Tensor? scale, Tensor? shift, int act) -> Tensor",
)
torch.library.define(
    "depthwise::pointwise_gemm",
    "(Tensor input, Tensor weight, Tensor? bias, Tensor? scale, Tensor? shift, int act) -> Tensor",
)


@torch.library.impl("depthwise::conv2d_nhwc", "default")
def _conv2d_nhwc_impl(input, weight, bias=None):
    return conv2d_nhwc_fused(input, weight, bias=bias)


@torch.library.impl("depthwise::conv2d_nhwc_fused", "default")
def _conv2d_nhwc_fused_impl(input, weight, bias, scale, shift, residual, act):
    return conv2d_nhwc_fused(input, weight, bias, scale, shift, residual, act)


@torch.library.register_fake("depthwise::conv2d_nhwc")
def _conv2d_nhwc_fake(input, weight, bias=None):
    return torch.empty_like(input)


@torch.library.register_fake("depthwise::conv2d_nhwc_fused")
def _conv2d_nhwc_fused_fake(input, weight, bias, scale, shift, residual, act):
    return torch.empty_like(input)


@torch.library.impl("depthwise::bias_act_affine", "default")
def _bias_act_affine_impl(input, bias, scale, shift, act):
    return bias_act_affine(input, bias, scale, shift, act)


@torch.library.register_fake("depthwise::bias_act_affine")
def _bias_act_affine_fake(input, bias, scale, shift, act):
    return torch.empty_like(input)


@torch.library.impl("depthwise::pointwise_gemm", "default")
def _pointwise_gemm_impl(input, weight, bias, scale, shift, act):
    return pointwise_gemm(input, weight, bias, scale, shift, act)


@torch.library.register_fake("depthwise::pointwise_gemm")
def _pointwise_gemm_fake(input, weight, bias, scale, shift, act):
    return input.new_empty((input.shape[0], weight.shape[0]))


def _conv2d_nhwc_setup(ctx, inputs, output):
    x, w, bias = inputs
    ctx.save_for_backward(x, w)
    ctx.has_bias = bias is not None


def _conv2d_nhwc_backward(ctx, grad):
    x, w = ctx.saved_tensors
    g = grad if grad.is_contiguous(memory_format=torch.channels_last) else grad.contiguous(
        memory_format=torch.channels_last)
    dx = conv2d_nhwc_backward_input(g, w) if ctx.needs_input_grad[0] else None
    dw = conv2d_nhwc_backward_weight(x, g, w.shape[0]).to(w.dtype) if ctx.needs_input_grad[1] else None
    db = g.float().sum(dim=(0, 2, 3)).to(g.dtype) if ctx.has_bias and ctx.needs_input_grad[2] else None
    return dx, dw, db


torch.library.register_autograd("depthwise::conv2d_nhwc", _conv2d_nhwc_backward, setup_context=_conv2d_nhwc_setup)


# Backward of the fused op y = act(z) * scale + shift + residual, z = conv(x, w) + bias.  The
# forward keeps nothing but its inputs; the backward recomputes z with the engine (one launch), takes
# the elementwise adjoints in fp32 with PyTorch, and runs the engine's two gradient kernels on
#   gz = dy * scale * act'(z):   dx = conv_input_grad(gz) (+ dy through the residual),
#   dw = conv_weight_grad(x, gz), dbias = sum gz, dscale = sum dy * act(z), dshift = sum dy.
# act'(z): ReLU 1[z > 0]; GELU (exact form) Phi(z) + z * phi(z).

def _conv2d_nhwc_fused_setup(ctx, inputs, output):
    x, w, bias, scale, shift, residual, act = inputs
    ctx.save_for_backward(x, w, bias, scale)
    ctx.act = int(act)
    ctx.flags = (bias is not None, scale is not None, shift is not None, residual is not None)


def _conv2d_nhwc_fused_backward(ctx, grad):
    x, w, bias, scale = ctx.saved_tensors
    has_bias, has_scale, has_shift, has_res = ctx.flags
    g = grad if grad.is_contiguous(memory_format=torch.channels_last) else grad.contiguous(
        memory_format=torch.channels_last)
    gf = g.float()
    need = ctx.needs_input_grad
    dims = (0, 2, 3)
    gz = gf
    a = None
    if ctx.act != _lib.ACT_NONE or (has_scale and need[3]):
        z = conv2d_nhwc_fused(x, w, bias=bias).float()
        if ctx.act == _lib.ACT_RELU:
            a = torch.relu(z)
            gz = gz * (z > 0).to(gz.dtype)
        elif ctx.act == _lib.ACT_GELU:
            cdf = 0.5 * (1.0 + torch.erf(z * 0.7071067811865476))
            pdf = torch.exp(-0.5 * z * z) * 0.3989422804014327
            a = z * cdf
            gz = gz * (cdf + z * pdf)
        else:
            a = z
    if has_scale:
        gz = gz * scale.float().view(1, -1, 1, 1)
    gz16 = gz.to(x.dtype).contiguous(memory_format=torch.channels_last)
    dx = conv2d_nhwc_backward_input(gz16, w) if need[0] else None
    dw = conv2d_nhwc_backward_weight(x, gz16, w.shape[0]).to(w.dtype) if need[1] else None
    db = gz.sum(dim=dims).to(x.dtype) if has_bias and need[2] else None
    ds = (gf * a).sum(dim=dims).to(x.dtype) if has_scale and need[3] else None
    dt = gf.sum(dim=dims).to(x.dtype) if has_shift and need[4] else None
    dr = g if has_res and need[5] else None
    return dx, dw, db, ds, dt, dr, None


torch.library.register_autograd("depthwise::conv2d_nhwc_fused", _conv2d_nhwc_fused_backward,
                                setup_context=_conv2d_nhwc_fused_setup)
