"""Full-MAML loops (``theria.maml.loops``), same API as the reference.

``named_params``, ``named_buffers``, ``loss_fn``, ``inner_adapt``,
``outer_loss`` and ``meta_loss_on_tasks`` follow
``theria/maml/loops.py:28-123``: functional inner SGD with
``create_graph=not fo`` so the meta-gradient is second order, and the mean
query loss over tasks.  With this library's attention the second-order
terms include the attention's own curvature (its backward is differentiable
through the HVP kernel).

``meta_loss_batched`` is an addition: the same meta-loss for a task-stacked
batch, all tasks adapted at once with per-task parameters (models that
implement ``forward_tasks``).  Because task losses are independent, the
gradient of their sum gives every task its own inner-step gradient, so the
result equals the sequential loop's.
"""

from __future__ import annotations

from collections import OrderedDict
from typing import Mapping

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.func import functional_call

from theria_b200.maml.tasks import TaskBatch

Params = "OrderedDict[str, torch.Tensor]"


def named_params(model: nn.Module):
    return OrderedDict((k, v) for k, v in model.named_parameters())


def named_buffers(model: nn.Module):
    return OrderedDict((k, v) for k, v in model.named_buffers())


def loss_fn(logits: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    return F.cross_entropy(logits, y)


def inner_adapt(model: nn.Module, params: Mapping[str, torch.Tensor],
                buffers: Mapping[str, torch.Tensor], task: TaskBatch, *,
                inner_lr: float = 0.1, inner_steps: int = 1, fo: bool = False):
    """phi <- phi - lr * grad L_support(phi), ``inner_steps`` times."""
    phi = OrderedDict(params.items())
    for _ in range(inner_steps):
        loss_s = loss_fn(functional_call(model, (phi, buffers), (task.x_s,)), task.y_s)
        grads = torch.autograd.grad(loss_s, tuple(phi.values()), create_graph=not fo,
                                    retain_graph=True, allow_unused=False)
        phi = OrderedDict((n, p - inner_lr * g) for (n, p), g in zip(phi.items(), grads))
    return phi


def outer_loss(model, phi, buffers, task: TaskBatch) -> torch.Tensor:
    return loss_fn(functional_call(model, (phi, buffers), (task.x_q,)), task.y_q)


def meta_loss_on_tasks(model: nn.Module, tasks: list[TaskBatch], *, inner_lr: float = 0.1,
                       inner_steps: int = 1, fo: bool = False, fo_strict: bool = False,
                       return_metrics: bool = False):
    """J(theta) = mean over tasks of L_query(phi_K(theta; support); query)."""
    params = named_params(model)
    buffers = named_buffers(model)
    losses, accs = [], []
    for task in tasks:
        phi = inner_adapt(model, params, buffers, task, inner_lr=inner_lr,
                          inner_steps=inner_steps, fo=fo)
        if fo_strict:
            phi = OrderedDict((k, v.detach().clone()) for k, v in phi.items())
        logits_q = functional_call(model, (phi, buffers), (task.x_q,))
        losses.append(loss_fn(logits_q, task.y_q))
        accs.append((logits_q.argmax(dim=-1) == task.y_q).float().mean())
    outer = torch.stack(losses).mean()
    if return_metrics:
        return outer, {"post_adapt_loss": outer.item(),
                       "post_adapt_acc": torch.stack(accs).mean().item()}
    return outer


def _task_losses(logits, y):
    # logits (nt, n, C), y (nt, n) -> per-task mean cross-entropy (nt,)
    nt, n, c = logits.shape
    return F.cross_entropy(logits.reshape(nt * n, c), y.reshape(nt * n),
                           reduction="none").view(nt, n).mean(dim=1)


_ALIGN = 32  # floats: parameter alignment inside the flat fast weights


def meta_loss_batched(model: nn.Module, tasks: TaskBatch, *, inner_lr: float = 0.1,
                      inner_steps: int = 1, fo: bool = False, reduction: str = "mean",
                      denom: int | None = None):
    """Meta-loss of a task-stacked batch (leading task axis on every field).

    ``model.forward_tasks(params, x)`` must accept parameters with a leading
    task axis.  Returns the mean (or sum / ``denom``) of the per-task query
    losses.

    The fast weights of all tasks live in ONE tensor phi [n_tasks, n_params]
    (the parameters concatenated), viewed per parameter through ``split``:
    an inner SGD step is then a single update of phi, and its gradient one
    concatenation, instead of a chain of small kernels per parameter.
    """
    nt = tasks.x_s.shape[0]
    names = [n for n, _ in model.named_parameters()]
    params = [p for _, p in model.named_parameters()]
    shapes = [p.shape for p in params]
    sizes = [p.numel() for p in params]
    # Every parameter starts on a 128-byte boundary of phi's rows (zero
    # padding between them): with an odd row length the per-task views are
    # misaligned and every GEMM and elementwise kernel on them falls back to
    # its unvectorised, 1-element-aligned variant (several times slower).
    padded = [-(-n // _ALIGN) * _ALIGN for n in sizes]
    parts = []
    for p, n, m in zip(params, sizes, padded):
        parts.append(p.reshape(-1))
        if m > n:
            parts.append(p.new_zeros(m - n))
    theta = torch.cat(parts)
    phi = theta.unsqueeze(0).expand(nt, theta.numel())

    def views(flat):
        return OrderedDict((n, c[:, :k].view(nt, *shp)) for n, c, k, shp in
                           zip(names, flat.split(padded, dim=1), sizes, shapes))

    for _ in range(inner_steps):
        ls = _task_losses(model.forward_tasks(views(phi), tasks.x_s), tasks.y_s).sum()
        (g,) = torch.autograd.grad(ls, (phi,), create_graph=not fo, retain_graph=True)
        phi = phi - inner_lr * g
    lq = _task_losses(model.forward_tasks(views(phi), tasks.x_q), tasks.y_q)
    if reduction == "sum":
        return lq.sum() / (denom if denom is not None else 1)
    return lq.mean()


__all__ = ["named_params", "named_buffers", "loss_fn", "inner_adapt", "outer_loss",
           "meta_loss_on_tasks", "meta_loss_batched"]
