"""B200-native (sm_100a) engine for the FP16 NHWC large-kernel depthwise convolution.

Importing the package registers the torch ops of both reference modules
(``depthwise::*`` and ``replknet_dw::*``) plus the generic
``depthwise::conv2d_nhwc`` / ``depthwise::conv2d_nhwc_fused`` ops.  All of
them run through the C ABI of ``libdwconv_b200.so`` (include/dwconv_b200.h).
"""
from . import _lib
from . import dw_ops
from . import depthwise_torch_ops
from . import depthwise_replknet_nhwc_ops
from .dw_ops import conv2d_nhwc, conv2d_nhwc_fused
from ._lib import plan_query, device_error, probe_fma_peak, DwbError

__all__ = ["conv2d_nhwc", "conv2d_nhwc_fused", "plan_query", "device_error", "probe_fma_peak", "DwbError",
           "dw_ops", "depthwise_torch_ops", "depthwise_replknet_nhwc_ops"]
