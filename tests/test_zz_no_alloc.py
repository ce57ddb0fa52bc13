"""The input gradient that allocates nothing (GPU).

Some callers cannot allocate device memory where they need the gradient (a
loop whose memory is fixed after warm-up, a host framework that owns every
allocation).  dwb_conv2d_nhwc_bwd_data_noalloc serves them: it takes the
unrotated weights and keeps the rotated taps in a buffer built into the
library.  Called here through the C ABI, twice in a row with different data,
and compared with the allocating path (dwb_weight_rot180 into a caller buffer
+ dwb_conv2d_nhwc_bwd_data), which runs the same kernel on the same rotated
taps and so must agree bit for bit, and with the exact float64 adjoint of
the oracle within the parity bar; a request larger than the
built-in buffer is refused with a message.  This file is collected last.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import make_problem

pytestmark = pytest.mark.gpu

MAX_TOL, REL_TOL = 1e-2, 1e-3


def _dev(a):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.permute(0, 3, 1, 2) if t.dim() == 4 else t


def test_input_gradient_without_allocation_matches_allocating_path(oracle_mod):
    import depthwise_conv_b200 as d
    from depthwise_conv_b200 import _lib
    lib = _lib.load()
    B, H, W, C, K = 2, 21, 19, 136, 13
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):  # the shared buffer is rewritten by each call
        _, w = make_problem(700 + call, B, H, W, C, K)
        dy = np.random.default_rng(800 + call).standard_normal((B, H, W, C)).astype(np.float16)
        dyd, wd = _dev(dy), _dev(w)
        expect = d.dw_ops.conv2d_nhwc_backward_input(dyd, wd)
        dx = torch.empty_like(dyd)
        rc = lib.dwb_conv2d_nhwc_bwd_data_noalloc(dyd.data_ptr(), wd.data_ptr(), dx.data_ptr(), B, H, W, C, K,
                                                  stream)
        assert rc == _lib.OK, _lib.load().dwb_status_string(rc)
        torch.cuda.synchronize()
        # the same kernel on the same rotated taps: bit-identical to the allocating path
        assert torch.equal(dx, expect), f"call {call}: differs from the allocating path"
        # and within the parity bar of the exact (float64) adjoint
        x0 = np.zeros((B, H, W, C), np.float16)
        exact_dx, _, _ = oracle_mod.dw_backward_numpy(x0, w, dy)
        a = dx.permute(0, 2, 3, 1).contiguous().cpu().numpy().astype(np.float64)
        max_err, rel = oracle_mod.parity(a, exact_dx)
        assert max_err <= MAX_TOL and rel <= REL_TOL, f"call {call}: max {max_err:.3e} rel {rel:.3e}"
    assert d.device_error() == 0


def test_oversize_request_is_refused():
    from depthwise_conv_b200 import _lib
    lib = _lib.load()
    K, C = 31, 4096  # 31 * 31 * 4096 taps > 2**21
    dy = torch.empty((1, C, 4, 4), dtype=torch.float16, device="cuda").contiguous(memory_format=torch.channels_last)
    w = torch.empty((K, K, C), dtype=torch.float16, device="cuda")
    dx = torch.empty_like(dy)
    rc = lib.dwb_conv2d_nhwc_bwd_data_noalloc(dy.data_ptr(), w.data_ptr(), dx.data_ptr(), 1, 4, 4, C, K,
                                              torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.ERR_BAD_SHAPE
    assert b"exceeds the built-in buffer" in lib.dwb_last_error()
