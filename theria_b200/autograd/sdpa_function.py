"""``theria.autograd.sdpa_function`` surface (reference file :1-44).

In the reference ``SDPAFunction`` is the documented *failing* boundary
(autograd-in-backward without create_graph).  Here the name resolves to the
twice-differentiable fused function, so ``sdpa`` supports grad-of-grad.
"""

from theria_b200.attention.fused import SDPAFunction, sdpa_apply


def sdpa(q, k, v, causal: bool = False):
    """Public SDPA entry point: q, k (B, H, T|M, D), v (B, H, M, Dv) -> (B, H, T, Dv)."""
    return sdpa_apply(q, k, v, causal, None)


__all__ = ["SDPAFunction", "sdpa"]
