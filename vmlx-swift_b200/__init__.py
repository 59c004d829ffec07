"""vmlx-swift_b200: B200-native (sm_100a) affine-quantized linear decode path.

Host-side mirror of vmlx-swift's QuantizedLinear / SwitchGLU / MLXDistributedTP
layers over the C ABI in include/vmlx_cuda.h (libvmlx_cuda.so, built in-tree).
The directory name contains a hyphen, so load it with ``load_package()`` from
the repository root helpers or importlib under the module name ``vmlx_b200``.
"""
from ._lib import VMLXError, build, lib  # noqa: F401
from . import ops, nn, switch_layers  # noqa: F401
from .ops import dequantized, gather_quantized_mm, quantized, quantized_mm  # noqa: F401
from .nn import QuantizedLinear  # noqa: F401
from .switch_layers import (QuantizedSwitchLinear, SwitchGLU, Qwen3MoESparseMoeBlock, gather_sort,  # noqa: F401
                            scatter_unsort)
from .ops import moe_combine, moe_route, moe_sort  # noqa: F401
from . import fast, llama, qwen3  # noqa: F401,E402
from . import distributed, load  # noqa: F401,E402
