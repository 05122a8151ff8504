"""Fused SDPA with first- AND second-order autograd on the CUDA kernels.

Mirrors ``theria/attention/triton_qk.py:307-391`` (``triton_sdpa_fused``,
``TritonFusedSDPAFunction``, ``triton_sdpa_fused_autograd``) with one
deliberate difference: the reference's backward Function is not itself
differentiable, so ``create_graph=True`` silently drops the attention's own
curvature in full MAML.  Here the backward is a Function too, whose
backward is the HVP kernel:

    SDPAFunction.forward(q, k, v)          -> O           (saves q,k,v,O,lse)
    SDPAFunction.backward(dO)              -> SDPABackward.apply(q,k,v,O,lse,dO)
    SDPABackward.forward(...)              -> dQ, dK, dV  (backward kernel)
    SDPABackward.backward(gQ, gK, gV)      -> H u for u = (gQ,gK,gV) with
                                              respect to (q,k,v), and J u
                                              with respect to dO (HVP kernel)

O and lse enter SDPABackward as functions of (q, k, v): the HVP kernel
differentiates through them, so their own gradient slots are None.
"""

from __future__ import annotations

import torch
from torch.autograd.function import once_differentiable

from theria_b200.attention import ops


def _c(t, dtype):
    return t.to(dtype).contiguous()


class SDPABackward(torch.autograd.Function):
    """(q, k, v, O, lse, dO) -> (dQ, dK, dV); differentiable once more."""

    @staticmethod
    def forward(ctx, q, k, v, o, lse, dout, causal, scale, packed=None):
        # q, k, v are the forward's own inputs (possibly strided views): they
        # must stay the tensors autograd knows, or the second-order path
        # through them is cut.  Packed copies feed the kernels only; the
        # forward's own packed copies come in `packed` (no second packing).
        qc, kc, vc = packed if packed is not None else (q.contiguous(), k.contiguous(),
                                                        v.contiguous())
        dout = _c(dout, q.dtype)
        dq, dk, dv = ops.backward(qc, kc, vc, dout, lse, o=o, causal=causal, scale=scale)
        ctx.save_for_backward(qc, kc, vc, lse, dout)
        ctx.causal, ctx.scale = causal, scale
        return dq, dk, dv

    @staticmethod
    @once_differentiable
    def backward(ctx, gq, gk, gv):
        q, k, v, lse, dout = ctx.saved_tensors
        tq = torch.zeros_like(q) if gq is None else _c(gq, q.dtype)
        tk = torch.zeros_like(k) if gk is None else _c(gk, k.dtype)
        tv = torch.zeros_like(v) if gv is None else _c(gv, v.dtype)
        need = ctx.needs_input_grad
        hq, hk, hv, ot = ops.hvp(q, k, v, dout, lse, tq, tk, tv, causal=ctx.causal,
                                 scale=ctx.scale,
                                 need=(need[0], need[1], need[2], need[5]))
        return hq, hk, hv, None, None, ot, None, None, None


class SDPAFunction(torch.autograd.Function):
    """O = softmax(scale q k^T) v on the CUDA kernels; twice differentiable."""

    @staticmethod
    def forward(ctx, q, k, v, causal=False, scale=None):
        scale = ops.default_scale(q) if scale is None else float(scale)
        # Strided views (e.g. heads split out of a fused projection) are
        # packed for the kernels, but the saved q, k, v are the inputs
        # themselves so that the backward Function stays connected to them.
        qc, kc, vc = q.contiguous(), k.contiguous(), v.contiguous()
        o, lse = ops.forward(qc, kc, vc, causal=causal, scale=scale)
        ctx.save_for_backward(q, k, v, o, lse, qc, kc, vc)
        ctx.save_for_forward(q, k, v, lse, qc, kc, vc)
        ctx.causal, ctx.scale = causal, scale
        return o

    @staticmethod
    def jvp(ctx, tq, tk, tv, _causal=None, _scale=None):
        """Forward-mode rule (torch.autograd.forward_ad): the JVP kernel."""
        _, _, _, lse, q, k, v = ctx.saved_tensors
        tq = torch.zeros_like(q) if tq is None else _c(tq, q.dtype)
        tk = torch.zeros_like(k) if tk is None else _c(tk, k.dtype)
        tv = torch.zeros_like(v) if tv is None else _c(tv, v.dtype)
        return ops.jvp(q, k, v, tq, tk, tv, lse, causal=ctx.causal, scale=ctx.scale)

    @staticmethod
    def backward(ctx, grad_out):
        q, k, v, o, lse, qc, kc, vc = ctx.saved_tensors
        dq, dk, dv = SDPABackward.apply(q, k, v, o, lse, grad_out, ctx.causal, ctx.scale,
                                        (qc, kc, vc))
        return dq, dk, dv, None, None

    @staticmethod
    def jvp_rule(q, k, v, tq, tk, tv, causal=False, scale=None):
        """Forward-mode tangent of O (exact; P from the forward's lse)."""
        _, lse = ops.forward(q, k, v, causal=causal, scale=scale)
        return ops.jvp(q, k, v, tq, tk, tv, lse, causal=causal, scale=scale)


# Name kept from the reference (triton_qk.py:372); the class is the
# twice-differentiable function above.
TritonFusedSDPAFunction = SDPAFunction


def _padded_head_dim(q, d):
    # 16-bit inputs pad to the tensor-core head dims, others to the larger dim
    if q.dtype in (torch.float16, torch.bfloat16):
        for cand in (64, 128):
            if d <= cand:
                return cand
    return d


def sdpa_apply(q, k, v, causal: bool = False, scale=None):
    """SDPAFunction with a value head dim Dv that may differ from D.

    The kernels take one head dim for q, k and v.  For Dv != D the smaller
    side is padded with zero columns to a common width (for 16-bit inputs
    the next tensor-core width, 64 or 128): zero columns of q and k leave the
    scores unchanged (the scale stays 1/sqrt(D) of the real D), zero columns
    of v add zero output columns, and the output is sliced back to Dv.  Pad
    and slice are linear, so first and second derivatives and forward-mode
    tangents pass through them exactly.  This generalises the reference,
    whose fused path asserts Dv == D (``theria/attention/triton_qk.py:318``)
    and lists Dv != D as future work.
    """
    D, Dv = q.shape[-1], v.shape[-1]
    if Dv == D:
        return SDPAFunction.apply(q, k, v, causal, scale)
    scale = ops.default_scale(q) if scale is None else float(scale)
    Dp = _padded_head_dim(q, max(D, Dv))
    pad = torch.nn.functional.pad
    if Dp > D:
        q, k = pad(q, (0, Dp - D)), pad(k, (0, Dp - D))
    if Dp > Dv:
        v = pad(v, (0, Dp - Dv))
    return SDPAFunction.apply(q, k, v, causal, scale)[..., :Dv]


def sdpa_fused(q, k, v, causal: bool = False, scale=None):
    """Differentiable fused SDPA returning q.dtype (Dv may differ from D)."""
    return sdpa_apply(q, k, v, causal, scale)


def triton_sdpa_fused_autograd(q, k, v, causal: bool = False):
    """Reference name (triton_qk.py:390-391)."""
    return sdpa_apply(q, k, v, causal, None)


def triton_sdpa_fused(q, k, v, return_stats: bool = False, causal: bool = False):
    """Fused forward, float32 output, optional stats.

    Mirrors ``theria/attention/triton_qk.py:307-369``: output is float32 and
    ``return_stats=True`` returns ``(out, m, l)``.  The kernel saves the row
    logsumexp, so the stats come back as ``m = lse`` and ``l = ones``, which
    satisfy the reference's convention P = exp(s - m) / l exactly.
    """
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise AssertionError("triton_sdpa_fused requires CUDA tensors")
    if v.shape[-1] != q.shape[-1]:
        raise AssertionError("v0 fused path currently requires Dv == D")
    out, lse = ops.forward(q, k, v, causal=causal, out_dtype=torch.float32,
                           need_lse=return_stats)
    if return_stats:
        return out, lse, torch.ones_like(lse)
    return out
