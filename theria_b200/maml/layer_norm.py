"""Task-batched LayerNorm with per-task affine parameters, twice
differentiable, on the fused kernels of libtheria_sm100.so
(``include/theria_ln.h``).

``layer_norm(x, w, b)`` with x ``[nt, ..., D]`` and w, b ``[nt, D]`` (one
row of fast weights per task) equals
``F.layer_norm(x, (D,)) * w[:, None, ...] + b[:, None, ...]``.  On CUDA
tensors the forward is one kernel, the backward one kernel plus a
deterministic column sum, and the backward's own backward (what the outer
step of full MAML differentiates through) the same; composed from torch
operators, that second derivative is several dozen small kernels per call.
CPU tensors take the composed torch form (the CPU model of the tests); on a
CUDA tensor the fused kernels are the only path and a missing library
raises.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch.autograd.function import once_differentiable

from theria_b200 import _lib

EPS = 1e-5


def _rows(x, w):
    nt, D = w.shape
    return nt, x.numel() // (nt * D), D


def _ldw(w):
    if w.stride(1) != 1:
        raise ValueError("layer_norm: affine rows must be contiguous")
    return w.shape[1] if w.shape[0] == 1 else w.stride(0)  # one row: its stride is unused


def _rowwise(t):
    # [nt, D] with unit column stride (rows may be strided views of a flat
    # per-task buffer); anything else is packed
    if t.shape[0] == 1 and t.stride(1) == 1:
        # one row: only row 0 is read, so its row stride is irrelevant; give
        # the kernels a view whose stride satisfies their ld >= D check
        return t.as_strided(t.shape, (t.shape[1], 1))
    return t if t.stride(1) == 1 and (t.stride(0) >= t.shape[1] or t.stride(0) == 0) \
        else t.contiguous()


def _ws(nt, R, D, like):
    n = _lib.load().theria_ln_workspace_bytes(nt, R, D)
    return torch.empty(max(n, 4) // 4, dtype=torch.float32, device=like.device)


class _LayerNormBackward(torch.autograd.Function):
    """(x, w, gy) -> (gx, gw, gb); its backward is the second derivative."""

    @staticmethod
    def forward(ctx, x, w, gy):
        gy = gy.contiguous()
        nt, R, D = _rows(x, w)
        gx = torch.empty_like(x)
        gw = torch.empty(nt, D, dtype=x.dtype, device=x.device)
        gb = torch.empty_like(gw)
        ws = _ws(nt, R, D, x)
        _lib.check(_lib.load().theria_ln_bwd(
            _lib.ptr(x), _lib.ptr(w), _ldw(w), _lib.ptr(gy), _lib.ptr(gx), _lib.ptr(gw),
            _lib.ptr(gb), _lib.ptr(ws), ws.numel() * 4, nt, R, D, EPS, _lib.stream_of(x)),
            "theria_ln_bwd")
        ctx.save_for_backward(x, w, gy)
        return gx, gw, gb

    @staticmethod
    @once_differentiable
    def backward(ctx, u, a, c):
        x, w, gy = ctx.saved_tensors
        nt, R, D = _rows(x, w)
        u = None if u is None else u.contiguous()
        a = None if a is None else _rowwise(a)
        c = None if c is None else _rowwise(c)
        dx = torch.empty_like(x)
        dgy = torch.empty_like(x)
        dw = torch.empty(nt, D, dtype=x.dtype, device=x.device)
        ws = _ws(nt, R, D, x)
        _lib.check(_lib.load().theria_ln_bwd2(
            _lib.ptr(x), _lib.ptr(w), _ldw(w), _lib.ptr(gy), _lib.ptr(u), _lib.ptr(a),
            0 if a is None else a.stride(0), _lib.ptr(c), 0 if c is None else c.stride(0),
            _lib.ptr(dx), _lib.ptr(dw), _lib.ptr(dgy), _lib.ptr(ws),
            ws.numel() * 4, nt, R, D, EPS, _lib.stream_of(x)), "theria_ln_bwd2")
        return dx, dw, dgy


class _LayerNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b):
        nt, R, D = _rows(x, w)
        if b.stride() != w.stride():
            b = b.clone(memory_format=torch.contiguous_format)
            w = w.contiguous()
        y = torch.empty_like(x)
        _lib.check(_lib.load().theria_ln_fwd(
            _lib.ptr(x), _lib.ptr(w), _lib.ptr(b), _ldw(w), _lib.ptr(y), nt, R, D, EPS,
            _lib.stream_of(x)), "theria_ln_fwd")
        ctx.save_for_backward(x, w)
        return y

    @staticmethod
    def backward(ctx, gy):
        x, w = ctx.saved_tensors
        gx, gw, gb = _LayerNormBackward.apply(x, w, gy)
        return gx, gw, gb


class _GeluBackward(torch.autograd.Function):
    """(x, gy) -> gy * gelu'(x) (torch's kernel); its backward is one kernel."""

    @staticmethod
    def forward(ctx, x, gy):
        gy = gy.contiguous()
        ctx.save_for_backward(x, gy)
        return torch.ops.aten.gelu_backward(gy, x)

    @staticmethod
    @once_differentiable
    def backward(ctx, u):
        x, gy = ctx.saved_tensors
        u = u.contiguous()
        dx, dgy = torch.empty_like(x), torch.empty_like(x)
        _lib.check(_lib.load().theria_gelu_bwd2(
            _lib.ptr(x), _lib.ptr(gy), _lib.ptr(u), _lib.ptr(dx), _lib.ptr(dgy), x.numel(),
            _lib.stream_of(x)), "theria_gelu_bwd2")
        return dx, dgy


class _Gelu(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        ctx.save_for_backward(x)
        return F.gelu(x)

    @staticmethod
    def backward(ctx, gy):
        (x,) = ctx.saved_tensors
        return _GeluBackward.apply(x, gy)


def gelu(x):
    """Exact GELU; on CUDA float32 its second derivative is one kernel."""
    if not x.is_cuda or x.dtype != torch.float32:
        return F.gelu(x)
    return _Gelu.apply(x.contiguous())


def layer_norm_reference(x, w, b):
    """The composed torch form (CPU tensors, and the tests' reference)."""
    h = F.layer_norm(x, (x.shape[-1],), eps=EPS)
    view = (x.shape[0],) + (1,) * (x.ndim - 2) + (x.shape[-1],)
    return h * w.view(view) + b.view(view)


def layer_norm(x, w, b):
    """LayerNorm over the last dim of x [nt, ..., D] with per-task w, b [nt, D]."""
    if not x.is_cuda:
        return layer_norm_reference(x, w, b)
    if x.dtype != torch.float32 or w.dtype != torch.float32 or b.dtype != torch.float32:
        raise ValueError("layer_norm: the fused kernels take float32")
    if w.shape != (x.shape[0], x.shape[-1]) or b.shape != w.shape:
        raise ValueError(f"layer_norm: w, b must be [nt, D], got {tuple(w.shape)}")
    return _LayerNorm.apply(x.contiguous(), w, b)


__all__ = ["layer_norm", "layer_norm_reference", "gelu", "EPS"]
