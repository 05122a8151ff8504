"""Public SDPA entry point with the reference's names.

Mirrors ``theria/attention/custom.py:15-71``.  The ``backend=`` switch keeps
the reference's names:

* ``triton_full_fused`` (default here; the reference defaults to
  ``reference``, and ``theria.attention.custom.sdpa_custom`` installed by
  ``theria_b200.compat.install_as_theria`` keeps that default),
  ``triton_full_fused_phase8``,
  ``fused``: the fused sm_100a operator (twice differentiable, forward-mode
  capable);
* ``custom``: ``SDPACustom`` (the same kernels behind the reference's
  Function contract with explicit ``hvp`` / ``jvp``);
* ``triton_qk`` / ``triton_ref`` / ``triton``, ``triton_fast``: scores from
  the dense score kernel, then PyTorch softmax and PV, as the reference did;
* ``triton_qk_softmax``: probabilities from the dense probability kernel,
  then PyTorch PV;
* ``reference``: the reference's formula softmax(q k^T / sqrt(D)) v in
  PyTorch operations on the inputs' device (the comparison arm of the
  reference's own tests, not a fallback: it runs only when asked for).

Unknown names raise ``ValueError`` like the reference.
"""

from __future__ import annotations

import torch

from theria_b200.attention.fused import sdpa_apply
from theria_b200.attention.reference import reference_attention
from theria_b200.attention.triton_qk import triton_qk, triton_qk_fast, triton_qk_softmax
from theria_b200.autograd.sdpa_custom_function import SDPACustom

FUSED_BACKENDS = ("triton_full_fused", "triton_full_fused_phase8", "custom", "fused")
PARTIAL_BACKENDS = ("triton_qk", "triton_ref", "triton", "triton_fast", "triton_qk_softmax")
BACKENDS = FUSED_BACKENDS + PARTIAL_BACKENDS + ("reference",)


def sdpa_custom(q, k, v, *, backend: str = "triton_full_fused", causal: bool = False):
    """softmax(q k^T / sqrt(D)) v, returning q.dtype.

    The fused backends are twice differentiable (``create_graph=True`` keeps
    the attention's own curvature); ``causal=True`` (top-left aligned mask)
    is available on the fused backends.
    """
    if backend not in BACKENDS:
        raise ValueError(f"Unsupported sdpa_custom backend: {backend}")
    if causal and backend not in FUSED_BACKENDS:
        raise ValueError(f"causal=True needs a fused backend ({', '.join(FUSED_BACKENDS)})")
    if backend == "custom":
        return SDPACustom.apply(q, k, v, causal)
    if backend in FUSED_BACKENDS:
        return sdpa_apply(q, k, v, causal, None)
    if backend == "reference":
        return reference_attention(q, k, v)
    if backend == "triton_qk_softmax":
        probs = triton_qk_softmax(q, k).to(torch.float32)
        return torch.matmul(probs, v.to(probs.dtype)).to(q.dtype)
    # custom.py:30-43: scores from the kernel, PyTorch softmax and PV
    qk = triton_qk_fast if backend == "triton_fast" else triton_qk
    scores = qk(q, k).to(torch.float32) / (q.shape[-1] ** 0.5)
    probs = torch.softmax(scores, dim=-1)
    return torch.matmul(probs, v.to(probs.dtype)).to(q.dtype)


def sdpa_custom_hvp(q, k, v, dq, dk, dv):
    """HVP of L = sum(O) along (dq, dk, dv) (reference custom.py:60-64)."""
    return SDPACustom.hvp(q, k, v, dq, dk, dv)


def sdpa_custom_jvp(q, k, v, dq, dk, dv):
    """Tangent of O along (dq, dk, dv) (reference custom.py:67-71)."""
    return SDPACustom.jvp(q, k, v, dq, dk, dv)
