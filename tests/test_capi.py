"""The C-ABI library on a machine without a GPU: it loads, exports every
declared symbol, validates arguments before touching a device, and plans
every benchmark configuration within the hardware limits."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "dwconv_b200.h")


@pytest.fixture(scope="module")
def lib():
    from depthwise_conv_b200 import _lib
    return _lib.load()


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"DWB_API\s+[\w\s\*]+?\b(dwb_\w+)\s*\(", text)))


def test_header_declares_the_abi():
    syms = declared_symbols()
    assert "dwb_conv2d_nhwc_fused_fwd" in syms and "dwb_depthwise_31x31_128_nhwc" in syms
    assert len(syms) >= 15


def test_every_declared_symbol_is_exported_and_bound(lib):
    from depthwise_conv_b200 import _lib
    for s in declared_symbols():
        assert hasattr(lib, s), f"{s} not exported by libdwconv_b200.so"
        assert s in _lib.SIGNATURES, f"{s} has no ctypes binding"


def test_abi_version_and_status_strings(lib):
    from depthwise_conv_b200 import _lib
    assert lib.dwb_abi_version() == 6
    for code in range(9):
        assert lib.dwb_status_string(code) and b"unknown" not in lib.dwb_status_string(code)
    assert lib.dwb_status_string(99) == b"unknown status"
    assert _lib.status_string(_lib.ERR_BAD_SHAPE).startswith("shape")


# Fake (never dereferenced) but 16-byte aligned addresses: every call below is
# rejected by argument validation before any CUDA call.
X, Wt, Y = 0x10000, 0x20000, 0x30000


def test_validation_statuses(lib):
    from depthwise_conv_b200 import _lib as L
    f = lib.dwb_conv2d_nhwc_fwd
    assert f(None, Wt, Y, 1, 8, 8, 64, 7, None) == L.ERR_NULL_POINTER
    assert f(X, None, Y, 1, 8, 8, 64, 7, None) == L.ERR_NULL_POINTER
    assert f(X, Wt, Y, 1, 8, 8, 64, 8, None) == L.ERR_BAD_SHAPE       # even K
    assert f(X, Wt, Y, 1, 8, 8, 64, 33, None) == L.ERR_BAD_SHAPE      # K > 31
    assert f(X, Wt, Y, 1, 8, 8, 60, 7, None) == L.ERR_BAD_SHAPE       # C % 8
    assert f(X, Wt, Y, 1, 0, 8, 64, 7, None) == L.ERR_BAD_SHAPE       # H = 0
    assert f(X + 2, Wt, Y, 1, 8, 8, 64, 7, None) == L.ERR_BAD_ALIGN
    assert f(X, Wt, Y + 8, 1, 8, 8, 64, 7, None) == L.ERR_BAD_ALIGN
    assert f(X, Wt, Y, 0, 8, 8, 64, 7, None) == L.OK                  # empty batch: no-op
    g = lib.dwb_conv2d_nhwc_fused_fwd
    assert g(X, Wt, None, None, None, None, Y, 1, 8, 8, 64, 7, 3, 0, None) == L.ERR_BAD_ARG   # act
    assert g(X, Wt, None, None, None, None, Y, 1, 8, 8, 64, 7, 0, 2, None) == L.ERR_BAD_ARG   # accum
    assert g(X, Wt, 0x40001, None, None, None, Y, 1, 8, 8, 64, 7, 0, 0, None) == L.ERR_BAD_ALIGN


def test_gradient_entry_points_validate(lib):
    """Shape, pointer and alignment checks of the gradient entry points answer without a device."""
    from depthwise_conv_b200 import _lib as L
    X, Y = ctypes.c_void_p(256), ctypes.c_void_p(512)
    assert lib.dwb_conv2d_nhwc_bwd_weight(X, Y, Y, 1, 8, 8, 64, 8, None) == L.ERR_BAD_SHAPE      # even K
    assert lib.dwb_conv2d_nhwc_bwd_weight(X, Y, Y, 1, 8, 8, 12, 7, None) == L.ERR_BAD_SHAPE      # C % 8
    assert lib.dwb_conv2d_nhwc_bwd_weight(None, Y, Y, 1, 8, 8, 64, 7, None) == L.ERR_NULL_POINTER
    assert lib.dwb_conv2d_nhwc_bwd_weight(ctypes.c_void_p(258), Y, Y, 1, 8, 8, 64, 7, None) == L.ERR_BAD_ALIGN
    assert lib.dwb_conv2d_nhwc_bwd_weight(None, None, None, 0, 8, 8, 64, 7, None) == L.OK         # empty batch
    assert lib.dwb_weight_rot180(X, Y, 64, 4, None) == L.ERR_BAD_SHAPE
    assert lib.dwb_weight_rot180(None, Y, 64, 5, None) == L.ERR_NULL_POINTER
    assert lib.dwb_conv2d_nhwc_bwd_data(X, Y, Y, 1, 8, 8, 64, 6, None) == L.ERR_BAD_SHAPE


def test_fixed_shape_launchers_reject_other_shapes(lib):
    from depthwise_conv_b200 import _lib as L
    assert lib.dwb_depthwise_forward_32_768_7(X, Wt, Y, 16, 32, 768, 7, 1, None) == L.ERR_BAD_SHAPE
    assert lib.dwb_depthwise_forward_32_1536_9(X, Wt, Y, 32, 32, 1536, 7, 1, 32 * 32 * 1536, None) == L.ERR_BAD_SHAPE
    assert lib.dwb_depthwise_forward_32_1536_9(X, Wt, Y, 32, 32, 1536, 9, 1, 12345, None) == L.ERR_BAD_SHAPE
    assert lib.dwb_depthwise_forward_32_1536_9_v2(X, Wt, Y, 32, 31, 1536, 9, 1, 0, None) == L.ERR_BAD_SHAPE
    assert lib.dwb_depthwise_forward_16_1536_9(X, Wt, Y, 16, 16, 1024, 9, 1, None) == L.ERR_BAD_SHAPE
    assert lib.dwb_depthwise_forward_32_1536_13(X, Wt, Y, 32, 32, 1536, 11, 1, None) == L.ERR_BAD_SHAPE
    assert lib.dwb_depthwise_31x31_128_nhwc(X, Wt, None, Y, 1, 128, 56, 55, None) == L.ERR_BAD_SHAPE
    assert lib.dwb_depthwise_29x29_256_nhwc(X, Wt, None, Y, 1, 128, 28, 28, None) == L.ERR_BAD_SHAPE
    assert lib.dwb_depthwise_27x27_512_nhwc(X, Wt, None, Y, 1, 512, 15, 14, None) == L.ERR_BAD_SHAPE
    # right shape, zero batch: accepted without a device
    assert lib.dwb_depthwise_31x31_128_nhwc(X, Wt, None, Y, 0, 128, 56, 56, None) == L.OK


BASELINE_SHAPES = [
    (1, 32, 32, 768, 7), (1, 32, 32, 1536, 9), (1, 56, 56, 128, 31), (1, 28, 28, 256, 29), (1, 14, 14, 512, 27),
    (1, 7, 7, 1024, 13), (16, 32, 32, 1536, 9), (64, 32, 32, 1536, 9), (256, 32, 32, 1536, 9),
    (1, 16, 16, 1536, 9), (1, 32, 32, 1536, 13),
] + [(64, 56, 56, 1024, k) for k in (7, 9, 13, 17, 21, 27, 29, 31)]


@pytest.mark.parametrize("B,H,W,C,K", BASELINE_SHAPES + [(2, 23, 17, 72, 5), (1, 1, 1, 8, 1), (3, 300, 500, 16, 31)])
@pytest.mark.parametrize("accum", [0, 1])
def test_plans_respect_hardware_limits(B, H, W, C, K, accum):
    from depthwise_conv_b200 import _lib
    p = _lib.plan_query(B, H, W, C, K, accum)
    assert p["kernel_size"] == K and p["accum"] == accum
    R, M = p["cols_per_thread"], p["rows_per_thread"]
    assert (R in (7, 8, 14, 16) or (R in (28, 32) and K <= 13)) and M in (1, 2)
    assert p["tile_w"] % R == 0 and p["tile_h"] % M == 0
    assert p["tile_w_in"] == p["tile_w"] + K - 1 <= 256                 # TMA box limit
    assert p["load_schedule"] in ((0, 1) if accum == 1 else (0,))
    S = p["row_splits"]
    assert 1 <= S <= K
    assert p["consumer_warps"] == S * (p["tile_w"] // R) * (p["tile_h"] // M)
    assert p["threads"] == 32 * (p["consumer_warps"] + 1) <= 1024
    # registers: per warp in units of 256, a CTA's warps spread over 4 sub-partitions of 16K each
    per_warp = -(-p["regs_estimate"] * 32 // 256) * 256
    assert -(-(p["consumer_warps"] + 1) // 4) * per_warp <= 16384
    assert p["smem_bytes"] <= 232448 and p["ctas_per_sm"] >= 1
    assert p["ring_wrows"] == 0
    slots = p["consumer_warps"] // S
    red = (S - 1) * slots * M * R * 32 * 8  # partial-sum exchange area
    tiles_h = -(-H // p["tile_h"])
    strips = B * -(-W // p["tile_w"]) * -(-C // 64)
    bt = p["band_tiles"]
    if bt == 0:  # tile mode: a stage holds an input row and a weight row
        assert p["ring_rows"] >= p["tile_h"]
        assert (2 * p["ring_rows"] + 2) * 8 <= 1024  # mbarrier area
        assert p["smem_bytes"] == 1024 + p["ring_rows"] * (p["tile_w_in"] + K) * 128 + red
        assert p["tiles"] == strips * tiles_h
    else:  # band mode (mixed, K <= 17): input rows only, two resident K x K weight buffers
        assert accum == 1 and K <= 17 and bt >= 1
        assert p["ring_rows"] >= p["tile_h"] + K - 1
        assert (2 * p["ring_rows"] + 6) * 8 <= 1024
        stages = 1024 + p["ring_rows"] * p["tile_w_in"] * 128 + red
        assert p["smem_bytes"] == -(-stages // 128) * 128 + 2 * K * K * 128
        assert p["tiles"] == strips * -(-tiles_h // bt)  # bands
    assert 1 <= p["grid"] <= min(p["tiles"], p["ctas_per_sm"] * 148) or (B == 0 and p["grid"] == 0)


def test_row_split_candidates_for_small_images():
    """Small images with large kernels get plans whose warps split the kernel rows; big batches do not."""
    from depthwise_conv_b200 import _lib
    small = _lib.plan_candidates(1, 14, 14, 512, 27, 1)
    splits = {c["row_splits"] for c in small}
    assert {1, 2, 4} <= splits
    for c in small:
        assert c["consumer_warps"] <= 31 and c["consumer_warps"] % c["row_splits"] == 0
        assert c["ring_rows"] >= c["tile_h"] + c["row_splits"] - 1 or c["ring_rows"] == c["tile_h"] + 26
    big = _lib.plan_candidates(64, 56, 56, 1024, 9, 1)
    assert {c["row_splits"] for c in big} == {1}


def test_plan_rejects_bad_problems():
    from depthwise_conv_b200 import _lib
    with pytest.raises(_lib.DwbError):
        _lib.plan_query(1, 8, 8, 64, 6)
    with pytest.raises(_lib.DwbError):
        _lib.plan_query(1, 8, 8, 12, 7)


def test_register_cap_table_is_consistent():
    """dw_regcaps.inc (generated by build.py --regcaps) names only compiled variants, and every cap is one
    of the occupancy steps the generator uses."""
    import os
    import re
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "depthwise_conv_b200", "csrc",
                        "dw_regcaps.inc")
    rows = [tuple(int(v) for v in m.groups())
            for m in re.finditer(r"\{(\d+), (\d+), (\d+), (\d+), (\d+), (\d+)\}", open(path).read())]
    assert rows, "empty register-cap table"
    assert len(set(r[:5] for r in rows)) == len(rows)  # one cap per variant
    for K, R, M, acc, pre, cap in rows:
        assert K % 2 == 1 and 1 <= K <= 31 and M in (1, 2) and acc in (0, 1) and pre in (0, 1)
        assert R in (7, 8, 14, 16) or (R in (28, 32) and K <= 13)
        assert pre == 0 or acc == 1  # the read-ahead schedule exists in mixed mode only
        assert cap in (64, 72, 80, 96, 128, 168)


def test_plans_respect_hardware_limits_on_random_problems():
    """The same invariants over seeded random problems the fixed list does not reach."""
    import numpy as np
    rng = np.random.default_rng(11)
    for _ in range(400):
        K = int(rng.choice(np.arange(1, 32, 2)))
        H, W = int(rng.integers(1, 601)), int(rng.integers(1, 601))
        C = 8 * int(rng.integers(1, 513))
        B = int(rng.choice([1, 2, 3, 8, 33, 512]))
        test_plans_respect_hardware_limits(B, H, W, C, K, int(rng.integers(0, 2)))
