"""``depthwise_torch_ops`` under the reference's bare module name.

The reference's callers import the ConvMixer op module by its bare name
(``from depthwise_torch_ops import CustomDepthwiseConv2d``,
bench_custom_warm.py:42-43; ``replace_depthwise_convs``,
benchmark_compile_modes.py:28, convmixer/benchmark.py:31).  Putting this
directory first on ``sys.path`` makes that import return the engine's
``depthwise_conv_b200.depthwise_torch_ops`` itself -- the same module object,
so every name (ops, fake impls, ``CustomDepthwiseConv2d``,
``replace_depthwise_convs``, ``SUPPORTED_CONFIGS``, ``_load_kernels``) is the
engine's and the ``depthwise::*`` ops are registered once.
"""
import os
import sys

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if _ROOT not in sys.path:
    sys.path.append(_ROOT)

from depthwise_conv_b200 import depthwise_torch_ops as _engine_module  # noqa: E402

sys.modules[__name__] = _engine_module
