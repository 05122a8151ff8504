"""Import-path alias of ``theria/attention/triton_qk.py`` for the fused path.

The reference module holds the Triton forward and its autograd wrapper; the
same names here resolve to the sm_100a kernels (no Triton is involved).
The legacy partial kernels of that module (``triton_qk``,
``triton_qk_fast``, ``triton_qk_softmax``) are not on the fused path and are
not provided.
"""

from theria_b200.attention.fused import (  # noqa: F401
    SDPAFunction,
    TritonFusedSDPAFunction,
    triton_sdpa_fused,
    triton_sdpa_fused_autograd,
)
