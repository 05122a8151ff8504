"""Hessian-vector products of SDPA on the CUDA kernels.

``hvp_fd_vjp`` keeps the reference's finite-difference utility
(``theria/attention/hvp_utils.py:17-49``): a central difference of the
explicit VJP of L = sum(O), composed from the forward and backward kernels.
``sdpa_hvp`` is the analytic HVP of L = <O, W> in one kernel pipeline, which
replaces the finite difference on the hot path.
"""

from __future__ import annotations

import torch

from theria_b200.attention import ops


def _explicit_grads_sum(q, k, v):
    """Grads of sum(O) w.r.t. q, k, v from the forward + backward kernels."""
    _, lse = ops.forward(q, k, v, out_dtype=q.dtype)
    dout = torch.ones_like(q)
    return ops.backward(q, k, v, dout, lse)


def hvp_fd_vjp(q, k, v, dq, dk, dv, eps=1e-3):
    """Central difference of the explicit VJP along (dq, dk, dv)."""
    with torch.no_grad():
        gp = _explicit_grads_sum((q + eps * dq).contiguous(), (k + eps * dk).contiguous(),
                                 (v + eps * dv).contiguous())
        gm = _explicit_grads_sum((q - eps * dq).contiguous(), (k - eps * dk).contiguous(),
                                 (v - eps * dv).contiguous())
    inv = 0.5 / eps
    return tuple((a - b) * inv for a, b in zip(gp, gm))


def sdpa_hvp(q, k, v, tq, tk, tv, w=None, causal: bool = False, scale=None):
    """Analytic H u of L = <O, w> (w = ones gives the reference's L = sum(O)).

    Returns (hq, hk, hv), each in q.dtype.
    """
    w = torch.ones_like(q) if w is None else w.to(q.dtype).contiguous()
    _, lse = ops.forward(q, k, v, causal=causal, scale=scale)
    hq, hk, hv, _ = ops.hvp(q, k, v, w, lse, tq.to(q.dtype).contiguous(),
                            tk.to(q.dtype).contiguous(), tv.to(q.dtype).contiguous(),
                            causal=causal, scale=scale, need=(True, True, True, False))
    return hq, hk, hv


__all__ = ["hvp_fd_vjp", "sdpa_hvp"]
