"""Public SDPA entry point with the reference's names.

Mirrors ``theria/attention/custom.py:15-71``.  The reference's
``backend=`` switch selected among CPU reference math and several Triton
kernels; this library has one implementation (the sm_100a kernels), so the
switch keeps only the names that denoted the fused, higher-order-capable
operator and rejects the rest loudly instead of falling back.
"""

from __future__ import annotations

from theria_b200.attention.fused import SDPAFunction
from theria_b200.autograd.sdpa_custom_function import SDPACustom

FUSED_BACKENDS = ("triton_full_fused", "triton_full_fused_phase8", "custom", "fused")


def sdpa_custom(q, k, v, *, backend: str = "triton_full_fused", causal: bool = False):
    """softmax(q k^T / sqrt(D)) v on the CUDA kernels, returning q.dtype.

    Twice differentiable (``create_graph=True`` keeps the attention's own
    curvature).  ``causal=True`` applies a top-left-aligned causal mask.
    """
    if backend not in FUSED_BACKENDS:
        raise ValueError(
            f"Unsupported sdpa_custom backend: {backend} (theria_b200 provides only the "
            f"fused CUDA operator: {', '.join(FUSED_BACKENDS)})")
    if backend == "custom":
        return SDPACustom.apply(q, k, v, causal)
    return SDPAFunction.apply(q, k, v, causal, None)


def sdpa_custom_hvp(q, k, v, dq, dk, dv):
    """HVP of L = sum(O) along (dq, dk, dv) (reference custom.py:60-64)."""
    return SDPACustom.hvp(q, k, v, dq, dk, dv)


def sdpa_custom_jvp(q, k, v, dq, dk, dv):
    """Tangent of O along (dq, dk, dv) (reference custom.py:67-71)."""
    return SDPACustom.jvp(q, k, v, dq, dk, dv)
