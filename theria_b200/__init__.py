"""theria_b200: B200-native (sm_100a) higher-order scaled dot-product attention.

A drop-in for the higher-order SDPA path of alexgabel/theria: the
``theria.attention`` entry points, the ``theria.autograd`` Function
contracts (with create_graph=True double-backward) and the
``theria.maml.loops`` callers, running on hand-written CUDA kernels behind
a C ABI (include/theria_sdpa.h, libtheria_sm100.so).
"""

from theria_b200._lib import check_device_error  # noqa: F401
from theria_b200.autograd.sdpa_function import sdpa  # noqa: F401

__version__ = "0.1.0"
