"""``depthwise_replknet_nhwc_ops`` under the reference's bare module name.

The reference's RepLKNet benchmark imports the op module by its bare name
(``from depthwise_replknet_nhwc_ops import replace_replknet_depthwise_nhwc``,
replknet/benchmark.py:84,215).  Putting this directory first on ``sys.path``
makes that import return the engine's
``depthwise_conv_b200.depthwise_replknet_nhwc_ops`` itself -- the same module
object, so the ``replknet_dw::*`` ops, the ``NHWCDepthwise*`` modules and the
swapper are the engine's and are registered once.
"""
import os
import sys

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if _ROOT not in sys.path:
    sys.path.append(_ROOT)

from depthwise_conv_b200 import depthwise_replknet_nhwc_ops as _engine_module  # noqa: E402

sys.modules[__name__] = _engine_module
