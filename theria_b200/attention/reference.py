"""The reference library's plain-PyTorch attention math, as importable names.

These are the comparison arms the reference exposes next to its kernels
(``theria/attention/reference.py:1-26`` re-exports them): the attention
formula, its explicit backward, the fp64 forward-mode tangent and the
analytic sum-loss Hessian-vector product.  They run ordinary PyTorch
operations on whatever device the inputs are on; nothing in this package's
kernel path calls them.  They exist so that code written against
``theria.attention.reference*`` (the reference's tests, notebooks and
``sdpa_custom(backend="reference")``) keeps working after
``theria_b200.compat.install_as_theria()``.
"""

from __future__ import annotations

import math

import torch


def _probs(q, k, scale):
    return torch.softmax(torch.matmul(q, k.transpose(-2, -1)) * scale, dim=-1)


def reference_attention(q, k, v):
    """softmax(q k^T / sqrt(D)) v (``reference_attention.py:9-19``)."""
    return torch.matmul(_probs(q, k, 1.0 / math.sqrt(q.shape[-1])), v)


sdpa_reference = reference_attention  # legacy name (reference_attention.py:22-24)


def softmax_jvp(scores, dscores, p):
    """Tangent of softmax: p * (dscores - <dscores, p>) (``reference_jvp_sdpa.py:12-18``)."""
    del scores
    return p * (dscores - (dscores * p).sum(dim=-1, keepdim=True))


def sdpa_backward_reference(q, k, v, dout, scale):
    """dQ, dK, dV without autograd (``reference_backward_sdpa.py:12-53``)."""
    with torch.no_grad():
        q, k, v, dout = q.detach(), k.detach(), v.detach(), dout.detach()
        p = _probs(q, k, scale)
        dp = torch.matmul(dout, v.transpose(-2, -1))
        ds = p * (dp - (dp * p).sum(dim=-1, keepdim=True))
        return (torch.matmul(ds, k) * scale, torch.matmul(ds.transpose(-2, -1), q) * scale,
                torch.matmul(p.transpose(-2, -1), dout))


def sdpa_jvp_reference(q, k, v, dq, dk, dv, scale):
    """Forward-mode tangent of O in fp64, returned in q.dtype
    (``reference_jvp_sdpa.py:21-44``)."""
    qf, kf, vf, tq, tk, tv = (t.double() for t in (q, k, v, dq, dk, dv))
    p = _probs(qf, kf, scale)
    ds = (torch.matmul(tq, kf.transpose(-2, -1)) + torch.matmul(qf, tk.transpose(-2, -1))) * scale
    return (torch.matmul(softmax_jvp(None, ds, p), vf) + torch.matmul(p, tv)).to(q.dtype)


def sdpa_jvp(q, k, v, dq, dk, dv):
    """Forward-mode tangent of O in the inputs' precision
    (``reference_hvp_sdpa.py:20-43``)."""
    scale = 1.0 / math.sqrt(q.shape[-1])
    p = _probs(q, k, scale)
    ds = (torch.matmul(dq, k.transpose(-2, -1)) + torch.matmul(q, dk.transpose(-2, -1))) * scale
    return torch.matmul(softmax_jvp(None, ds, p), v) + torch.matmul(p, dv)


def sdpa_hvp(q, k, v, vq, vk, vv):
    """Analytic H u of L = sum(O) along (vq, vk, vv) (``reference_hvp_sdpa.py:46-97``).

    With upstream ones, dP_ij = sum_d V_jd; its tangent uses tV the same way."""
    scale = 1.0 / math.sqrt(q.shape[-1])
    p = _probs(q, k, scale)
    pd = softmax_jvp(None, (torch.matmul(vq, k.transpose(-2, -1))
                            + torch.matmul(q, vk.transpose(-2, -1))) * scale, p)
    g = v.sum(dim=-1).unsqueeze(-2).expand_as(p)
    gd = vv.sum(dim=-1).unsqueeze(-2).expand_as(p)
    z = (g * p).sum(dim=-1, keepdim=True)
    zd = (gd * p + g * pd).sum(dim=-1, keepdim=True)
    ds = p * (g - z)
    dsd = pd * (g - z) + p * (gd - zd)
    hq = scale * (torch.matmul(dsd, k) + torch.matmul(ds, vk))
    hk = scale * (torch.matmul(dsd.transpose(-2, -1), q) + torch.matmul(ds.transpose(-2, -1), vq))
    hv = pd.sum(dim=-2).unsqueeze(-1).expand_as(v)
    return hq, hk, hv


sdpa_hvp_reference = sdpa_hvp

__all__ = ["reference_attention", "sdpa_reference", "softmax_jvp", "sdpa_backward_reference",
           "sdpa_jvp_reference", "sdpa_jvp", "sdpa_hvp", "sdpa_hvp_reference"]
