"""Batched matmul for the task-batched MAML model, differentiable to any
order, that splits long reductions.

The weight gradients of the model (``h^T @ gy`` per task) reduce over every
token row of a task (1,600 support / 4,800 query rows) while their outputs
are tiny (64 x 256 at most); with a handful of tasks per GPU, a plain
``bmm`` runs a few dozen CTAs and reaches a few TFLOP/s.  ``tbmm`` splits
such a reduction into S chunks that become extra batch entries (views, no
copies, when the operands are row-major as here) and adds the partial
products.  Its backward is written with ``tbmm`` again, so the second-order
MAML step (whose double backward produces the same shapes) splits as well.
"""

from __future__ import annotations

import torch

from theria_b200 import _lib

_TARGET_CTAS = 296  # two waves of 64 x 64 output tiles on 148 SMs
_MIN_CHUNK = 128


def _split(n, m, k, p):
    tiles = ((m + 63) // 64) * ((p + 63) // 64)
    want = -(-_TARGET_CTAS // max(1, n * tiles))
    s = 1
    while 2 * s <= want and k % (2 * s) == 0 and k // (2 * s) >= _MIN_CHUNK:
        s *= 2
    return s


def _k_major(x):
    # [n, r, k] stored k-major (x.transpose(1, 2) row-major): the rows of
    # every k-chunk are then a plain batch of views
    return x.stride(1) == 1 and x.stride(0) == x.shape[2] * x.stride(2)


def _row_major(x):
    return x.stride(2) == 1 and x.stride(0) == x.shape[1] * x.stride(1)


def _transposed(x):
    return x.stride(1) == 1 and x.stride(2) != 1


def _bmm(a, b):
    n, m, k = a.shape
    p = b.shape[2]
    s = _split(n, m, k, p)
    if s == 1 or not (_k_major(a) and _row_major(b)):
        return torch.bmm(a, b)
    at = a.transpose(1, 2).reshape(n * s, k // s, m).transpose(1, 2)
    bt = b.reshape(n * s, k // s, p)
    part = torch.bmm(at, bt)  # [n * s, m, p]
    if not (part.is_cuda and part.dtype == torch.float32):
        return part.view(n, s, m, p).sum(1)
    out = torch.empty(n, m, p, dtype=part.dtype, device=part.device)
    _lib.check(_lib.load().theria_chunk_sum(_lib.ptr(part), _lib.ptr(out), n, s, m * p,
                                            _lib.stream_of(part)), "theria_chunk_sum")
    return out


class _TaskBmm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b):
        ctx.save_for_backward(a, b)
        return _bmm(a, b)

    @staticmethod
    def backward(ctx, g):
        # Each gradient is produced in its input's layout (a transposed view
        # gets a transposed view back), so no copy follows in autograd.
        a, b = ctx.saved_tensors
        ga = gb = None
        if ctx.needs_input_grad[0]:
            ga = (tbmm(b, g.transpose(1, 2)).transpose(1, 2) if _transposed(a)
                  else tbmm(g, b.transpose(1, 2)))
        if ctx.needs_input_grad[1]:
            gb = (tbmm(g.transpose(1, 2), a).transpose(1, 2) if _transposed(b)
                  else tbmm(a.transpose(1, 2), g))
        return ga, gb


def tbmm(a, b):
    """``torch.bmm(a, b)`` (a [n, m, k], b [n, k, p]) with long-k splitting."""
    return _TaskBmm.apply(a, b)


class _RowSum(torch.autograd.Function):
    """x [n, R, C] -> sum over R, one deterministic kernel on CUDA."""

    @staticmethod
    def forward(ctx, x):
        x = x.contiguous()
        ctx.shape = x.shape
        if not x.is_cuda:
            return x.sum(1)
        n, r, c = x.shape
        out = torch.empty(n, c, dtype=x.dtype, device=x.device)
        lib = _lib.load()
        wsb = lib.theria_rowsum_workspace_bytes(n, r, c)
        ws = torch.empty(max(wsb, 4) // 4, dtype=torch.float32, device=x.device)
        _lib.check(lib.theria_rowsum(_lib.ptr(x), _lib.ptr(out), _lib.ptr(ws), ws.numel() * 4,
                                     n, r, c, _lib.stream_of(x)), "theria_rowsum")
        return out

    @staticmethod
    def backward(ctx, g):
        return g.unsqueeze(1).expand(ctx.shape)


class _AddBias(torch.autograd.Function):
    """x [n, R, C] + b [n, C] broadcast over R (+ an optional residual of x's
    shape, added in the same kernel); the bias gradient is a row sum
    (differentiable: its backward is a broadcast)."""

    @staticmethod
    def forward(ctx, x, b, res):
        ctx.has_res = res is not None
        x = x.contiguous()
        res = None if res is None else res.contiguous()
        if b.stride(1) != 1:
            b = b.contiguous()
        n, r, c = x.shape
        out = torch.empty_like(x)
        _lib.check(_lib.load().theria_add_bias(
            _lib.ptr(x), _lib.ptr(b), b.stride(0), _lib.ptr(res), _lib.ptr(out), n, r, c,
            _lib.stream_of(x)), "theria_add_bias")
        return out

    @staticmethod
    def backward(ctx, g):
        gb = _RowSum.apply(g) if ctx.needs_input_grad[1] else None
        return g, gb, (g if ctx.has_res else None)


def add_bias(x, b, res=None):
    """``[res +] x + b[:, None, :]`` for x [n, R, C] float32, with a fused
    bias gradient."""
    if x.dtype != torch.float32 or not x.is_cuda:
        out = x + b.unsqueeze(1)
        return out if res is None else res.reshape(out.shape) + out
    return _AddBias.apply(x, b, None if res is None else res.reshape(x.shape))


__all__ = ["tbmm", "add_bias"]
