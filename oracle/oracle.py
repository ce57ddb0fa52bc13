"""CPU oracle for the depthwise path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg import this module, and only as the checker / the timed CPU reference.
The product package (``depthwise_conv_b200``) never imports it.

Three independent restatements of the reference's computation, each citing
the reference lines it follows (luckychen/depthwise_conv):

* ``dw_forward`` / ``dw_forward_pixels`` -- plain C (``dwconv_oracle.c``),
  double accumulation, the fused epilogue of
  ``benchmark_cudnn_fused_e2e.py:65-74,125-131`` and the residual of
  ``convmixer/convmixer.py:58-59``;
* ``dw_forward_numpy`` -- numpy float64, sum of shifted input slices;
* ``dw_forward_torch`` -- ``F.conv2d(groups=C)`` on the fp16-rounded inputs,
  the reference's own correctness check (``benchmark_sensitivity.py:254-259``,
  ``benchmark_triton.py:141-144``) and the reference model's CPU path
  (``convmixer/convmixer.py:109``, ``replknet/kernels/depthwise_replknet_nhwc_ops.py:16``).

Plus ``dw_forward_f16acc``: the reference kernels' fp16 accumulation
(``depthwise_integration.cu:88-99``, ``depthWise_ch_128_k_31_t_56_half_forward.cu:694``),
used to report the reference kernels' own distance from the exact result.

Arrays: NHWC ``numpy.float16`` inputs ``x[B,H,W,C]``, weights ``w[K,K,C]``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle_dw.so")

ACT = {"none": 0, "relu": 1, "gelu": 2}

_lib = None


def build() -> str:
    """Compile the C oracle (gcc) if it is missing or stale."""
    src = os.path.join(HERE, "dwconv_oracle.c")
    if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        p, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.oracle_dw_forward.argtypes = [p, p, p, p, p, p, i64, i64, i64, i64, i32, i32, p, p, i32]
        L.oracle_dw_forward_pixels.argtypes = [p, p, p, p, p, p, i64, i64, i64, i64, i32, i32, p, i64, p, p, i32]
        L.oracle_dw_forward_f16acc.argtypes = [p, p, p, i64, i64, i64, i64, i32, p, i32]
        L.oracle_dw_channel_sums.argtypes = [p, p, i64, i64, i64, i64, i32, p, p]
        L.oracle_double_to_half.argtypes = [ctypes.c_double]
        L.oracle_double_to_half.restype = ctypes.c_uint16
        L.oracle_half_to_double.argtypes = [ctypes.c_uint16]
        L.oracle_half_to_double.restype = ctypes.c_double
        for f in ("oracle_dw_forward", "oracle_dw_forward_pixels", "oracle_dw_forward_f16acc",
                  "oracle_dw_channel_sums"):
            getattr(L, f).restype = ctypes.c_int
        _lib = L
    return _lib


def _threads(n):
    return int(n) if n else (os.cpu_count() or 1)


def _h(a):
    """float16 array (or None) -> contiguous uint16 view and its pointer."""
    if a is None:
        return None, None
    a = np.ascontiguousarray(a, dtype=np.float16).view(np.uint16)
    return a, a.ctypes.data


def _check_shapes(x, w):
    if x.ndim != 4 or w.ndim != 3 or w.shape[0] != w.shape[1] or w.shape[2] != x.shape[3]:
        raise ValueError(f"expected x[B,H,W,C], w[K,K,C]; got {x.shape}, {w.shape}")
    if w.shape[0] % 2 == 0:
        raise ValueError("kernel size must be odd")


def dw_forward(x, w, bias=None, scale=None, shift=None, residual=None, act="none", nthreads=None):
    """Exact (double-accumulated) forward.  Returns (y_float32, y_float16)."""
    _check_shapes(x, w)
    B, H, W, C = x.shape
    K = w.shape[0]
    xs, xp = _h(x)
    ws, wp = _h(w)
    bs, bp = _h(bias)
    ss, sp = _h(scale)
    hs, hp = _h(shift)
    rs, rp = _h(residual)
    y32 = np.empty((B, H, W, C), np.float32)
    y16 = np.empty((B, H, W, C), np.uint16)
    rc = lib().oracle_dw_forward(xp, wp, bp, sp, hp, rp, B, H, W, C, K, ACT[act], y32.ctypes.data, y16.ctypes.data,
                                 _threads(nthreads))
    if rc:
        raise ValueError("oracle_dw_forward rejected the problem")
    return y32, y16.view(np.float16)


def dw_forward_pixels(x, w, pix, bias=None, scale=None, shift=None, residual=None, act="none", nthreads=None):
    """Exact forward at the given linear output pixels ((b*H + h)*W + w): [npix, C]."""
    _check_shapes(x, w)
    B, H, W, C = x.shape
    K = w.shape[0]
    pix = np.ascontiguousarray(pix, dtype=np.int64)
    xs, xp = _h(x)
    ws, wp = _h(w)
    bs, bp = _h(bias)
    ss, sp = _h(scale)
    hs, hp = _h(shift)
    rs, rp = _h(residual)
    out32 = np.empty((len(pix), C), np.float32)
    out16 = np.empty((len(pix), C), np.uint16)
    rc = lib().oracle_dw_forward_pixels(xp, wp, bp, sp, hp, rp, B, H, W, C, K, ACT[act], pix.ctypes.data, len(pix),
                                        out32.ctypes.data, out16.ctypes.data, _threads(nthreads))
    if rc:
        raise ValueError("oracle_dw_forward_pixels rejected the problem")
    return out32, out16.view(np.float16)


def dw_forward_f16acc(x, w, bias=None, nthreads=None):
    """The reference kernels' fp16-accumulating arithmetic (row-major taps)."""
    _check_shapes(x, w)
    B, H, W, C = x.shape
    K = w.shape[0]
    xs, xp = _h(x)
    ws, wp = _h(w)
    bs, bp = _h(bias)
    y16 = np.empty((B, H, W, C), np.uint16)
    lib().oracle_dw_forward_f16acc(xp, wp, bp, B, H, W, C, K, y16.ctypes.data, _threads(nthreads))
    return y16.view(np.float16)


def channel_sums(x, w):
    """sum over (h, w) of the plain convolution, per (image, channel), float64 [B, C]."""
    _check_shapes(x, w)
    B, H, W, C = x.shape
    K = w.shape[0]
    xs, xp = _h(x)
    ws, wp = _h(w)
    sums = np.empty((B, C), np.float64)
    scratch = np.empty(((H + 1) * (W + 1) * C,), np.float64)
    lib().oracle_dw_channel_sums(xp, wp, B, H, W, C, K, sums.ctypes.data, scratch.ctypes.data)
    return sums


def half_round(v: float) -> int:
    """binary16 bits of v rounded to nearest even (the C restatement)."""
    return int(lib().oracle_double_to_half(float(v)))


# ---- numpy restatement -------------------------------------------------------

def _epilogue_np(acc, C, bias, scale, shift, residual, act):
    v = acc
    if bias is not None:
        v = v + np.asarray(bias, np.float64).reshape(1, 1, 1, C)
    if act == "relu":
        v = np.maximum(v, 0.0)
    elif act == "gelu":
        from math import erf, sqrt
        v = 0.5 * v * (1.0 + np.vectorize(erf)(v / sqrt(2.0)))
    if scale is not None:
        v = v * np.asarray(scale, np.float64).reshape(1, 1, 1, C)
    if shift is not None:
        v = v + np.asarray(shift, np.float64).reshape(1, 1, 1, C)
    if residual is not None:
        v = v + np.asarray(residual, np.float64)
    return v


def dw_forward_numpy(x, w, bias=None, scale=None, shift=None, residual=None, act="none"):
    """float64 forward as a sum of K*K shifted input slices (independent of the C code)."""
    _check_shapes(x, w)
    B, H, W, C = x.shape
    K = w.shape[0]
    p = K // 2
    xd = np.zeros((B, H + 2 * p, W + 2 * p, C), np.float64)
    xd[:, p:p + H, p:p + W, :] = np.asarray(x, np.float64)
    wd = np.asarray(w, np.float64)
    acc = np.zeros((B, H, W, C), np.float64)
    for ki in range(K):
        for kj in range(K):
            acc += xd[:, ki:ki + H, kj:kj + W, :] * wd[ki, kj]
    return _epilogue_np(acc, C, bias, scale, shift, residual, act)


def dw_backward_numpy(x, w, dy):
    """float64 gradients of y = conv(x, w) ("same" padding, stride 1), for loss = sum(y * dy).

    The reference is inference-only; these are the adjoints of its forward
    definition (the tap sum of dw_forward_numpy):
      dx[b,h,w,c]   = sum_{ki,kj} dy[b, h-ki+p, w-kj+p, c] * w[ki,kj,c]
      dw[ki,kj,c]   = sum_{b,h,w} dy[b,h,w,c] * x[b, h+ki-p, w+kj-p, c]
      dbias[c]      = sum_{b,h,w} dy[b,h,w,c]
    Returns (dx NHWC, dw [K,K,C], dbias [C]).
    """
    _check_shapes(x, w)
    B, H, W, C = x.shape
    K = w.shape[0]
    p = K // 2
    xd = np.zeros((B, H + 2 * p, W + 2 * p, C), np.float64)
    xd[:, p:p + H, p:p + W, :] = np.asarray(x, np.float64)
    g = np.asarray(dy, np.float64)
    wd = np.asarray(w, np.float64)
    gd = np.zeros_like(xd)  # dy scattered back onto the padded input grid
    dw = np.zeros((K, K, C), np.float64)
    for ki in range(K):
        for kj in range(K):
            gd[:, ki:ki + H, kj:kj + W, :] += g * wd[ki, kj]
            dw[ki, kj] = (xd[:, ki:ki + H, kj:kj + W, :] * g).sum(axis=(0, 1, 2))
    return gd[:, p:p + H, p:p + W, :], dw, g.sum(axis=(0, 1, 2))


# ---- torch F.conv2d restatement (the reference's own check) ---------------------

def dw_forward_torch(x, w, bias=None, scale=None, shift=None, residual=None, act="none", dtype="float32",
                     channels_last=False):
    """F.conv2d(groups=C) on the fp16-rounded inputs, in float32 (or float64).

    Follows benchmark_sensitivity.py:254-259: permute NHWC -> NCHW, weights
    [K,K,C] -> [C,1,K,K], padding K//2, groups=C.  Returns NHWC numpy.
    """
    import torch
    import torch.nn.functional as F

    _check_shapes(x, w)
    td = torch.float64 if dtype == "float64" else torch.float32
    C = x.shape[3]
    K = w.shape[0]
    xt = torch.from_numpy(np.asarray(x, np.float16)).to(td).permute(0, 3, 1, 2)
    xt = xt.contiguous(memory_format=torch.channels_last) if channels_last else xt.contiguous()
    wt = torch.from_numpy(np.asarray(w, np.float16)).to(td).permute(2, 0, 1).unsqueeze(1).contiguous()
    with torch.no_grad():
        y = F.conv2d(xt, wt, padding=K // 2, groups=C)
        if bias is not None:
            y = y + torch.from_numpy(np.asarray(bias, np.float16)).to(td).view(1, C, 1, 1)
        if act == "relu":
            y = torch.relu(y)
        elif act == "gelu":
            y = F.gelu(y)
        if scale is not None:
            y = y * torch.from_numpy(np.asarray(scale, np.float16)).to(td).view(1, C, 1, 1)
        if shift is not None:
            y = y + torch.from_numpy(np.asarray(shift, np.float16)).to(td).view(1, C, 1, 1)
        if residual is not None:
            y = y + torch.from_numpy(np.asarray(residual, np.float16)).to(td).permute(0, 3, 1, 2)
    return y.permute(0, 2, 3, 1).contiguous().numpy()


# ---- parity metrics ------------------------------------------------------------

def parity(actual, expected):
    """(max |err|, rel-L2) of ``actual`` against ``expected`` (both cast to float64)."""
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    diff = a - e
    max_err = float(np.max(np.abs(diff))) if diff.size else 0.0
    denom = float(np.linalg.norm(e.ravel()))
    rel = float(np.linalg.norm(diff.ravel()) / denom) if denom > 0 else float(np.linalg.norm(diff.ravel()))
    return max_err, rel


# North-star tolerance for fp16 outputs against the exact result.
MAX_ABS_TOL = 1e-2
REL_L2_TOL = 1e-3
