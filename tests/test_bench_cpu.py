"""bench.py's roofline arithmetic and argument surface (CPU).

The algorithmic FLOP and byte counts behind `roofline.achieved` are checked
against an independent count (every in-image tap enumerated) and against the
per-layer figures the measurement plan tabulates for the benchmark shapes.
"""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


def _taps_enumerated(B, H, W, C, K):
    p = K // 2
    n = 0
    for h in range(H):
        for w in range(W):
            for i in range(K):
                for j in range(K):
                    if 0 <= h + i - p < H and 0 <= w + j - p < W:
                        n += 1
    return 2.0 * B * C * n


@pytest.mark.parametrize("B,H,W,C,K", [(1, 7, 9, 8, 3), (2, 5, 4, 16, 7), (1, 3, 3, 8, 31), (1, 10, 1, 8, 9)])
def test_valid_flops_counts_in_image_taps(B, H, W, C, K):
    assert bench.valid_flops(B, H, W, C, K) == _taps_enumerated(B, H, W, C, K)


@pytest.mark.parametrize("shape,flops", [((1, 32, 32, 1536, 9), 2.206e8), ((64, 56, 56, 1024, 31), 2.933e11),
                                          ((1, 56, 56, 128, 31), 5.729e8), ((1, 14, 14, 512, 27), 3.934e7),
                                          ((64, 56, 56, 1024, 7), 1.893e10)])
def test_valid_flops_of_benchmark_layers(shape, flops):
    assert abs(bench.valid_flops(*shape) / flops - 1) < 1e-3


def test_layer_bytes():
    # input + output once, weights once; the fused epilogue adds its three vectors and the residual read
    assert bench.dw_bytes(1, 32, 32, 1536, 9, epilogue=False) == 6540288
    assert bench.dw_bytes(1, 32, 32, 1536, 9) == 6540288 + 3 * 2 * 1536 + 2 * 32 * 32 * 1536


def test_cli_surface():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--help"], capture_output=True, text=True,
                         check=True).stdout
    for flag in ("--gpus", "--steps", "--warmup", "--impl", "--workload", "--shape", "--epilogue", "--backward"):
        assert flag in out


def test_reference_arm_line():
    """The reference arm runs the CPU model and prints one contract line (at least 3 warm-up steps)."""
    import json
    res = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "1"], capture_output=True, text=True, check=True, timeout=600)
    line = json.loads(res.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "img/s" and line["higher_is_better"] is True
    assert line["warmup"] >= 3 and line["steps"] == 1 and line["value"] > 0
    assert line["cpu_baseline"]["value"] == line["value"] and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"] == {"value": line["value"], "unit": "img/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_dw_configs_cover_every_baseline_layer():
    """18 layer entries: RepLKNet C3-C6 and the ConvMixer layers C1/C2 at B=1, the k9 batch sweep at
    B in {1, 16, 64, 256} and the k-sweep at B=64 with GELU+BN (BASELINE configs[1..4])."""
    names = [c[0] for c in bench.DW_CONFIGS]
    assert len(names) == len(set(names)) == 18
    shapes = {(B, H, W, C, K, epi) for _, B, H, W, C, K, epi, _ in bench.DW_CONFIGS}
    for s in [(1, 32, 32, 768, 7, "none"), (1, 32, 32, 1536, 9, "none"), (1, 56, 56, 128, 31, "none"),
              (1, 28, 28, 256, 29, "none"), (1, 14, 14, 512, 27, "none"), (1, 7, 7, 1024, 13, "none")]:
        assert s in shapes
    for b in (1, 16, 64, 256):
        assert (b, 32, 32, 1536, 9, "none") in shapes
    for k in (7, 9, 13, 17, 21, 27, 29, 31):
        assert (64, 56, 56, 1024, k, "gelu_bn") in shapes
    # batched configs shard over the ranks; batch-1 configs are per-GPU replicas
    for _, B, *_rest, shard in bench.DW_CONFIGS:
        assert shard == ("replica" if B == 1 else "batch")
