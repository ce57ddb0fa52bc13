"""ctypes binding of ``libdwconv_b200.so``, the engine's C ABI (include/dwconv_b200.h).

The library is built in-tree by ``depthwise_conv_b200/csrc/build.py``.  There
is no fallback: if the library is missing or cannot be loaded, every entry
point raises ``RuntimeError`` naming the problem.
"""
from __future__ import annotations

import ctypes
import os
import threading

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libdwconv_b200.so")

ABI_VERSION = 6  # DWB_ABI_VERSION of include/dwconv_b200.h

# dwb_status
OK = 0
ERR_NULL_POINTER = 1
ERR_BAD_SHAPE = 2
ERR_BAD_ALIGN = 3
ERR_UNSUPPORTED = 4
ERR_CUDA = 5
ERR_NO_DEVICE = 6
ERR_DEVICE_TIMEOUT = 7
ERR_BAD_ARG = 8

# dwb_act / dwb_accum
ACT_NONE, ACT_RELU, ACT_GELU = 0, 1, 2
ACT_CODES = {"none": ACT_NONE, "relu": ACT_RELU, "gelu": ACT_GELU}
ACCUM_F32, ACCUM_MIXED = 0, 1
ACCUM_DEFAULT = ACCUM_MIXED  # DWB_ACCUM_DEFAULT

# Every entry point the header declares, with its ctypes signature.
_p, _i, _i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64


class Problem(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int64), ("height", ctypes.c_int64), ("width", ctypes.c_int64),
                ("channels", ctypes.c_int64), ("kernel_size", ctypes.c_int32), ("accum", ctypes.c_int32)]


class Plan(ctypes.Structure):
    _fields_ = [("kernel_size", ctypes.c_int32), ("cols_per_thread", ctypes.c_int32),
                ("rows_per_thread", ctypes.c_int32), ("channel_block", ctypes.c_int32),
                ("tile_h", ctypes.c_int32), ("tile_w", ctypes.c_int32), ("tile_w_in", ctypes.c_int32),
                ("ring_rows", ctypes.c_int32), ("ring_wrows", ctypes.c_int32), ("consumer_warps", ctypes.c_int32),
                ("threads", ctypes.c_int32), ("smem_bytes", ctypes.c_int32), ("ctas_per_sm", ctypes.c_int32),
                ("grid", ctypes.c_int64), ("tiles", ctypes.c_int64), ("accum", ctypes.c_int32), ("regs_estimate", ctypes.c_int32),
                ("model_cost", ctypes.c_double), ("row_splits", ctypes.c_int32), ("load_schedule", ctypes.c_int32),
                ("band_tiles", ctypes.c_int32)]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}

    @classmethod
    def from_dict(cls, d: dict) -> "Plan":
        p = cls()
        for name, _ in cls._fields_:
            if name in d:
                setattr(p, name, d[name])
        return p


SIGNATURES = {
    "dwb_abi_version": ([], _i),
    "dwb_status_string": ([_i], ctypes.c_char_p),
    "dwb_plan_query": ([ctypes.POINTER(Problem), _i, _i, ctypes.POINTER(Plan)], _i),
    "dwb_plan_select": ([ctypes.POINTER(Problem), ctypes.POINTER(Plan)], _i),
    "dwb_plan_candidates": ([ctypes.POINTER(Problem), _i, _i, ctypes.POINTER(Plan), _i, ctypes.POINTER(_i)], _i),
    "dwb_last_error": ([], ctypes.c_char_p),
    "dwb_conv2d_nhwc_fwd_planned": ([_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i, _i,
                                     ctypes.POINTER(Plan), _p], _i),
    "dwb_conv2d_nhwc_fwd": ([_p, _p, _p, _i64, _i64, _i64, _i64, _i, _p], _i),
    "dwb_conv2d_nhwc_fused_fwd": ([_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i, _i, _i, _p], _i),
    "dwb_depthwise_forward_32_768_7": ([_p, _p, _p, _i, _i, _i, _i, _i, _p], _i),
    "dwb_depthwise_forward_32_1536_9": ([_p, _p, _p, _i, _i, _i, _i, _i, _i, _p], _i),
    "dwb_depthwise_forward_32_1536_9_v2": ([_p, _p, _p, _i, _i, _i, _i, _i, _i, _p], _i),
    "dwb_depthwise_forward_16_1536_9": ([_p, _p, _p, _i, _i, _i, _i, _i, _p], _i),
    "dwb_depthwise_forward_32_1536_13": ([_p, _p, _p, _i, _i, _i, _i, _i, _p], _i),
    "dwb_depthwise_31x31_128_nhwc": ([_p, _p, _p, _p, _i, _i, _i, _i, _p], _i),
    "dwb_depthwise_29x29_256_nhwc": ([_p, _p, _p, _p, _i, _i, _i, _i, _p], _i),
    "dwb_depthwise_27x27_512_nhwc": ([_p, _p, _p, _p, _i, _i, _i, _i, _p], _i),
    "dwb_bias_act_affine_nhwc": ([_p, _p, _p, _p, _p, _i64, _i64, _i, _p], _i),
    "dwb_pointwise_conv_nhwc": ([_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i, _i, _p], _i),
    "dwb_device_error": ([ctypes.POINTER(ctypes.c_int), _i, _p], _i),
    "dwb_probe_fma_peak": ([ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double), _p], _i),
    "dwb_selftest_bounded_wait": ([_i64, _p], _i),
    "dwb_weight_rot180": ([_p, _p, _i64, _i, _p], _i),
    "dwb_conv2d_nhwc_bwd_data": ([_p, _p, _p, _i64, _i64, _i64, _i64, _i, _p], _i),
    "dwb_conv2d_nhwc_bwd_weight": ([_p, _p, _p, _i64, _i64, _i64, _i64, _i, _p], _i),
    "dwb_conv2d_nhwc_bwd_weight_workspace": ([_i64, _i64, _i64, _i64, _i, ctypes.POINTER(_i64)], _i),
    "dwb_conv2d_nhwc_bwd_weight_det": ([_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i, _p], _i),
    "dwb_conv2d_nhwc_bwd_data_noalloc": ([_p, _p, _p, _i64, _i64, _i64, _i64, _i, _p], _i),
}

_lib = None
_lock = threading.Lock()


class DwbError(RuntimeError):
    """A non-OK status returned by the engine's C ABI."""

    def __init__(self, fn: str, status: int):
        self.status = status
        detail = ""
        if status == ERR_CUDA:
            try:
                detail = ": " + load().dwb_last_error().decode()
            except Exception:  # pragma: no cover
                pass
        super().__init__(f"{fn} failed: status {status} ({status_string(status)}){detail}")


def load() -> ctypes.CDLL:
    """Load the C-ABI library (once).  Raises RuntimeError if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"depthwise_conv_b200: CUDA library {LIB_PATH} is missing; build it with "
                    "`python -m depthwise_conv_b200.csrc.build` (there is no CPU fallback)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (argtypes, restype) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = argtypes
                fn.restype = restype
            if lib.dwb_abi_version() != ABI_VERSION:
                raise RuntimeError("depthwise_conv_b200: ABI version mismatch")
            _lib = lib
    return _lib


def status_string(status: int) -> str:
    try:
        return load().dwb_status_string(status).decode()
    except Exception:  # pragma: no cover - library absent
        return "unknown"


def check(fn: str, status: int) -> None:
    if status != OK:
        raise DwbError(fn, status)


def call(fn: str, *args) -> None:
    """Call an entry point and raise DwbError on a non-OK status."""
    check(fn, getattr(load(), fn)(*args))


# Opt-in check of the device error word after every engine launch made through the torch ops.
# A kernel whose bounded wait expires (its data never arrived within ~1 s of SM clock) records a
# code in the word and returns with its output partly unwritten; without this check only an
# explicit device_error() call reveals it.  The check synchronises the launching stream, so it is
# for debugging and validation runs, and it is skipped while the stream is being captured into a
# CUDA graph (no synchronisation is allowed there).  Enabled by DWB_CHECK_DEVICE_ERROR=1 in the
# environment, or set_check_device_error(True).
_check_device_error = os.environ.get("DWB_CHECK_DEVICE_ERROR", "0") not in ("", "0")


def set_check_device_error(on: bool) -> bool:
    """Turn the post-launch device-error check on or off; returns the previous setting."""
    global _check_device_error
    prev, _check_device_error = _check_device_error, bool(on)
    return prev


def check_device_error_enabled() -> bool:
    return _check_device_error


class DeviceTimeoutError(RuntimeError):
    """A kernel's bounded wait expired: its output is incomplete (device error word set)."""

    def __init__(self, code: int, where: str):
        self.code = code
        super().__init__(f"{where}: a kernel's bounded wait expired (device error code {code}: "
                         f"{DEVICE_ERROR_CODES.get(code, 'unknown')}); its output is incomplete")


# Codes a kernel stores in the device error word (csrc/dw_device.cuh).
DEVICE_ERROR_CODES = {1: "stage wait before a tile's first step", 2: "stage wait of a step",
                      3: "producer's free-stage wait", 4: "row-split partial-sum hand-off",
                      5: "bounded-wait self-test", 6: "pointwise GEMM producer's free-stage wait",
                      7: "pointwise GEMM operand wait", 8: "pointwise GEMM accumulator wait"}


def after_launch(stream: int, where: str) -> None:
    """The opt-in post-launch check: raise DeviceTimeoutError if the device error word is set."""
    if not _check_device_error:
        return
    import torch
    if torch.cuda.is_current_stream_capturing():
        return
    code = device_error(stream, clear=True)
    if code:
        raise DeviceTimeoutError(code, where)


def plan_query(B: int, H: int, W: int, C: int, K: int, accum: int = ACCUM_DEFAULT, sm_count: int = 0,
               smem_optin: int = 0) -> dict:
    """The planner's choice for a problem (host arithmetic only, no GPU needed)."""
    pr = Problem(B, H, W, C, K, accum)
    out = Plan()
    check("dwb_plan_query", load().dwb_plan_query(ctypes.byref(pr), sm_count, smem_optin, ctypes.byref(out)))
    return out.as_dict()


def plan_select(B: int, H: int, W: int, C: int, K: int, accum: int = ACCUM_DEFAULT) -> dict:
    """The plan the launcher uses on the current device (tuned table, else the cost model)."""
    pr = Problem(B, H, W, C, K, accum)
    out = Plan()
    check("dwb_plan_select", load().dwb_plan_select(ctypes.byref(pr), ctypes.byref(out)))
    return out.as_dict()


def plan_candidates(B: int, H: int, W: int, C: int, K: int, accum: int = ACCUM_DEFAULT, sm_count: int = 0,
                    smem_optin: int = 0) -> list[dict]:
    """Every feasible plan of a problem with its modelled cost (host arithmetic only)."""
    pr = Problem(B, H, W, C, K, accum)
    n = ctypes.c_int(0)
    check("dwb_plan_candidates", load().dwb_plan_candidates(ctypes.byref(pr), sm_count, smem_optin, None, 0,
                                                            ctypes.byref(n)))
    arr = (Plan * max(1, n.value))()
    check("dwb_plan_candidates", load().dwb_plan_candidates(ctypes.byref(pr), sm_count, smem_optin, arr, n.value,
                                                            ctypes.byref(n)))
    return [arr[i].as_dict() for i in range(n.value)]


def device_error(stream: int = 0, clear: bool = True) -> int:
    """Device error word (0 = no bounded wait has expired); synchronises ``stream``."""
    code = ctypes.c_int(0)
    check("dwb_device_error", load().dwb_device_error(ctypes.byref(code), int(clear), stream))
    return code.value


def selftest_bounded_wait(limit_cycles: int = 2_000_000, stream: int = 0) -> int:
    """Run the bounded-wait self-test kernel and return the device error code it left (5 expected)."""
    check("dwb_selftest_bounded_wait", load().dwb_selftest_bounded_wait(int(limit_cycles), stream))
    return device_error(stream)


def probe_fma_peak(stream: int = 0) -> tuple[float, float]:
    """Measured (HFMA2, FFMA2) CUDA-core rates of the current device, TFLOP/s."""
    a, b = ctypes.c_double(0.0), ctypes.c_double(0.0)
    check("dwb_probe_fma_peak", load().dwb_probe_fma_peak(ctypes.byref(a), ctypes.byref(b), stream))
    return a.value, b.value
