"""``SDPACustom`` contract on the CUDA kernels.

Mirrors ``theria/autograd/sdpa_custom_function.py:14-70``: an
``autograd.Function`` whose backward stays differentiable under
``create_graph=True`` (so HVPs and full-MAML meta-gradients include the
attention's own curvature), plus static analytic ``hvp`` / ``jvp`` helpers.
The reference builds its backward by autograd-in-backward over torch ops;
here forward, backward, JVP and HVP are kernels (see
``theria_b200.attention.fused``).
"""

from __future__ import annotations

import torch

from theria_b200.attention import ops
from theria_b200.attention.fused import SDPABackward


class SDPACustom(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal=False):
        scale = ops.default_scale(q)
        # Save the inputs themselves (not packed copies): the backward
        # Function must stay connected to them for second order.
        o, lse = ops.forward(q.contiguous(), k.contiguous(), v.contiguous(), causal=causal,
                             scale=scale)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.causal, ctx.scale = causal, scale
        return o

    @staticmethod
    def backward(ctx, grad_out):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = SDPABackward.apply(q, k, v, o, lse, grad_out, ctx.causal, ctx.scale)
        return dq, dk, dv, None

    @staticmethod
    def hvp(q, k, v, dq, dk, dv):
        """H u of L = sum(O) along u = (dq, dk, dv) (reference_hvp_sdpa.py:46-97)."""
        from theria_b200.attention.hvp_utils import sdpa_hvp
        return sdpa_hvp(q.contiguous(), k.contiguous(), v.contiguous(), dq, dk, dv)

    @staticmethod
    def jvp(q, k, v, dq, dk, dv):
        """Tangent of O along (dq, dk, dv) (reference_jvp_sdpa.py:21-44)."""
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        _, lse = ops.forward(q, k, v)
        dt = q.dtype
        return ops.jvp(q, k, v, dq.to(dt).contiguous(), dk.to(dt).contiguous(),
                       dv.to(dt).contiguous(), lse)


__all__ = ["SDPACustom"]
