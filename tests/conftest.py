"""Shared test configuration.

Markers:
  gpu -- needs an sm_100 GPU and the built CUDA library; collected everywhere,
         skipped when no CUDA device is visible.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the built CUDA library")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device visible")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle as O
    O.build()
    return O


def make_problem(seed, B, H, W, C, K, wscale=None):
    """Seeded NHWC fp16 input and [K,K,C] fp16 weights (N(0,1) and N(0,1/K^2)), as numpy."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((B, H, W, C), dtype=np.float32).astype(np.float16)
    s = (1.0 / K) if wscale is None else wscale
    w = (rng.standard_normal((K, K, C), dtype=np.float32) * s).astype(np.float16)
    return x, w
