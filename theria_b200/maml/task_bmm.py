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

_TARGET_CTAS = 296  # two waves of 64 x 64 output tiles on 148 SMs
_MIN_CHUNK = 128


def _split(n, m, k, p):
    tiles = ((m + 63) // 64) * ((p + 63) // 64)
    want = -(-_TARGET_CTAS // max(1, n * tiles))
    s = 1
    while 2 * s <= want and k % (2 * s) == 0 and k // (2 * s) >= _MIN_CHUNK:
        s *= 2
    return s


def _bmm(a, b):
    n, m, k = a.shape
    p = b.shape[2]
    s = _split(n, m, k, p)
    if s == 1:
        return torch.bmm(a, b)
    at = a.transpose(1, 2).reshape(n * s, k // s, m).transpose(1, 2)
    bt = b.reshape(n * s, k // s, p)
    return torch.bmm(at, bt).view(n, s, m, p).sum(1)


class _TaskBmm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b):
        ctx.save_for_backward(a, b)
        return _bmm(a, b)

    @staticmethod
    def backward(ctx, g):
        a, b = ctx.saved_tensors
        ga = tbmm(g, b.transpose(1, 2)) if ctx.needs_input_grad[0] else None
        gb = tbmm(a.transpose(1, 2), g) if ctx.needs_input_grad[1] else None
        return ga, gb


def tbmm(a, b):
    """``torch.bmm(a, b)`` (a [n, m, k], b [n, k, p]) with long-k splitting."""
    return _TaskBmm.apply(a, b)


__all__ = ["tbmm"]
