"""Higher-order SDPA on B200 (sm_100a): the ``theria.attention`` surface.

Stable names, as in ``theria/attention/__init__.py:10-26``:
``triton_sdpa_fused``, ``sdpa_bwd_dq``, ``sdpa_bwd_dk``, ``sdpa_bwd_dv``,
``sdpa_jvp``.  Each runs hand-written CUDA kernels from libtheria_sm100.so.
"""

from .fused import triton_sdpa_fused, sdpa_fused, SDPAFunction
from .triton_sdpa_backward import sdpa_bwd_dq, sdpa_bwd_dk, sdpa_bwd_dv, sdpa_jvp
from .hvp_utils import hvp_fd_vjp, sdpa_hvp

__all__ = [
    "triton_sdpa_fused",
    "sdpa_bwd_dq",
    "sdpa_bwd_dk",
    "sdpa_bwd_dv",
    "sdpa_jvp",
    "sdpa_fused",
    "sdpa_hvp",
    "hvp_fd_vjp",
    "SDPAFunction",
]
