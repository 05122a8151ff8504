"""Self-attention on a packed projection ``qkv [B, T, 3, H, D]``, twice
differentiable, without head-layout copies.

``sdpa_qkv(qkv)`` equals
``sdpa_fused(*qkv.permute(2, 0, 3, 1, 4).unbind(0)).transpose(1, 2)``,
i.e. O as ``[B, T, H, D]``.  The whole-head kernels read q, k and v in place
from the projection and write O, dqkv and the HVP's hqkv in these layouts
(``theria_sdpa_qkv_*`` in ``include/theria_sdpa.h``), so the transposes and
packing copies around the attention disappear from the forward, the
backward and the double backward.  It serves T <= 64 and D <= 64; other
shapes take the general path (the same kernel families through
``sdpa_fused`` on unpacked heads).
"""

from __future__ import annotations

import torch
from torch.autograd.function import once_differentiable

from theria_b200 import _lib
from theria_b200.attention import ops
from theria_b200.attention.fused import sdpa_fused

_SMALL = 64


def _dims(qkv):
    B, T, three, H, D = qkv.shape
    if three != 3:
        raise AssertionError(f"qkv must be [B, T, 3, H, D], got {tuple(qkv.shape)}")
    return B, H, T, D


def _call(name, *args):
    _lib.check(getattr(_lib.load(), name)(*args), name)


def _fwd(qkv, causal, scale):
    B, H, T, D = _dims(qkv)
    o = torch.empty(B, T, H, D, dtype=qkv.dtype, device=qkv.device)
    lse = torch.empty(B, H, T, dtype=torch.float32, device=qkv.device)
    with torch.cuda.device(qkv.device):
        _call("theria_sdpa_qkv_fwd", _lib.ptr(qkv), _lib.ptr(o), _lib.ptr(lse), B, H, T, D,
              _lib.DTYPE_CODE[qkv.dtype], scale, int(causal), _lib.stream_of(qkv))
    return o, lse


class _QKVBackward(torch.autograd.Function):
    """(qkv, lse, dO) -> dqkv; its backward is the HVP kernel (H u for qkv,
    J u for dO)."""

    @staticmethod
    def forward(ctx, qkv, lse, dout, causal, scale):
        B, H, T, D = _dims(qkv)
        dout = dout.to(qkv.dtype).contiguous()
        dqkv = torch.empty_like(qkv)
        with torch.cuda.device(qkv.device):
            _call("theria_sdpa_qkv_bwd", _lib.ptr(qkv), _lib.ptr(dout), _lib.ptr(lse),
                  _lib.ptr(dqkv), B, H, T, D, _lib.DTYPE_CODE[qkv.dtype], scale, int(causal),
                  _lib.stream_of(qkv))
        ctx.save_for_backward(qkv, lse, dout)
        ctx.causal, ctx.scale = causal, scale
        return dqkv

    @staticmethod
    @once_differentiable
    def backward(ctx, g):
        qkv, lse, dout = ctx.saved_tensors
        B, H, T, D = _dims(qkv)
        need_h, need_o = ctx.needs_input_grad[0], ctx.needs_input_grad[2]
        tqkv = g.to(qkv.dtype).contiguous()
        hqkv = torch.empty_like(qkv) if need_h else None
        ot = torch.empty_like(dout) if need_o else None
        if need_h or need_o:
            with torch.cuda.device(qkv.device):
                _call("theria_sdpa_qkv_hvp", _lib.ptr(qkv), _lib.ptr(dout), _lib.ptr(lse),
                      _lib.ptr(tqkv), _lib.ptr(hqkv), _lib.ptr(ot), B, H, T, D,
                      _lib.DTYPE_CODE[qkv.dtype], ctx.scale, int(ctx.causal),
                      _lib.stream_of(qkv))
        return hqkv, None, ot, None, None


class _QKVFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, causal, scale):
        o, lse = _fwd(qkv, causal, scale)
        ctx.save_for_backward(qkv, lse)
        ctx.causal, ctx.scale = causal, scale
        return o

    @staticmethod
    def backward(ctx, dout):
        qkv, lse = ctx.saved_tensors
        return _QKVBackward.apply(qkv, lse, dout, ctx.causal, ctx.scale), None, None


def sdpa_qkv(qkv, causal: bool = False, scale=None):
    """Attention of a packed projection: qkv [B, T, 3, H, D] -> O [B, T, H, D]."""
    if not qkv.is_cuda:
        raise AssertionError("sdpa_qkv requires CUDA tensors")
    B, H, T, D = _dims(qkv)
    scale = 1.0 / D ** 0.5 if scale is None else float(scale)
    if qkv.dtype not in _lib.DTYPE_CODE:
        raise AssertionError(f"Unsupported dtype for qkv: {qkv.dtype}")
    small = 32 if qkv.dtype == torch.float64 else _SMALL  # fp64 heads must fit as doubles
    if T > small or D > small:
        # general path: unpacked heads through the same operator family
        q, k, v = qkv.permute(2, 0, 3, 1, 4).unbind(0)
        return sdpa_fused(q, k, v, causal=causal, scale=scale).transpose(1, 2)
    return _QKVFunction.apply(qkv.contiguous(), bool(causal), scale)


__all__ = ["sdpa_qkv"]
