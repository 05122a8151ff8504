"""Synthetic sequence-classification tasks for the full-MAML benchmark.

``TaskBatch`` keeps the reference's field names
(``theria/tasks/synthetic_seqcls.py:8-13``).  The sampler is new (the
reference's Gaussian-prototype tasks are a different benchmark): each task
draws, for each of its ``n_way`` classes, a token distribution from a
Dirichlet(alpha) over the vocabulary; every sequence of a class is ``seq_len``
i.i.d. tokens from that distribution.  Sampling runs on the host with a
seeded numpy Generator, so a (seed, task index) pair always yields the same
task on every rank and device.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch


@dataclass(frozen=True)
class TaskBatch:
    x_s: torch.Tensor  # (n_way * k_shot, L) int64 tokens
    y_s: torch.Tensor  # (n_way * k_shot,)
    x_q: torch.Tensor  # (n_way * n_query, L)
    y_q: torch.Tensor  # (n_way * n_query,)

    def to(self, device, non_blocking: bool = False) -> "TaskBatch":
        return TaskBatch(*(t.to(device, non_blocking=non_blocking)
                           for t in (self.x_s, self.y_s, self.x_q, self.y_q)))


@dataclass(frozen=True)
class TaskConfig:
    vocab: int = 32
    seq_len: int = 64
    n_way: int = 5
    k_shot: int = 5
    n_query: int = 15
    alpha: float = 0.5


def sample_task(rng: np.random.Generator, cfg: TaskConfig = TaskConfig()) -> TaskBatch:
    probs = rng.dirichlet(np.full(cfg.vocab, cfg.alpha), size=cfg.n_way)  # (C, V)

    def split(n):
        y = np.repeat(np.arange(cfg.n_way), n)
        x = np.stack([rng.choice(cfg.vocab, size=cfg.seq_len, p=probs[c]) for c in y])
        return torch.from_numpy(x.astype(np.int64)), torch.from_numpy(y.astype(np.int64))

    xs, ys = split(cfg.k_shot)
    xq, yq = split(cfg.n_query)
    return TaskBatch(xs, ys, xq, yq)


def sample_tasks(seed: int, n: int, cfg: TaskConfig = TaskConfig(), start: int = 0):
    """Tasks ``start .. start+n-1`` of the meta-batch drawn from ``seed``.

    Task ``i`` depends only on (seed, i), so ranks can each draw their shard.
    """
    return [sample_task(np.random.default_rng([seed, start + i]), cfg) for i in range(n)]


def stack_tasks(tasks: list[TaskBatch], pin: bool = False) -> TaskBatch:
    """Stack a list of tasks along a leading task axis (for batched MAML)."""
    out = TaskBatch(*(torch.stack([getattr(t, f) for t in tasks])
                      for f in ("x_s", "y_s", "x_q", "y_q")))
    if pin:
        out = TaskBatch(*(t.pin_memory() for t in (out.x_s, out.y_s, out.x_q, out.y_q)))
    return out
