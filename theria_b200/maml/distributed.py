"""Task-sharded full-MAML meta-step across ranks (one process per GPU).

The meta-batch of T tasks is split evenly over W ranks; each rank adapts
its T/W tasks locally (batched, per-task parameters) and back-propagates
sum(query losses) / T, so the per-rank gradients add up to the gradient of
the meta-batch mean.  One ``all_reduce(SUM)`` of a single flat fp32 bucket
holding every parameter's gradient (about 0.43 MB for the benchmark model)
then gives every rank the full meta-gradient, and each rank applies the
same Adam step, so parameters stay identical without a broadcast.  Initial
parameters are broadcast from rank 0 once.

The reference runs tasks sequentially on one device
(``theria/maml/loops.py:108-123``); this is the added exchange step, over
NCCL on GPUs or gloo for the CPU tests.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from theria_b200.maml.loops import meta_loss_batched
from theria_b200.maml.tasks import TaskBatch


def broadcast_params(model: torch.nn.Module, src: int = 0) -> None:
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        with torch.no_grad():
            for p in model.parameters():
                dist.broadcast(p.data, src)


def shard_range(meta_batch: int, rank: int, world: int) -> tuple[int, int]:
    if meta_batch % world != 0:
        raise ValueError(f"meta_batch {meta_batch} must divide evenly over {world} ranks")
    per = meta_batch // world
    return rank * per, per


class MetaStep:
    """One outer step: local batched adaptation, one gradient all-reduce, Adam."""

    def __init__(self, model, *, meta_batch=32, inner_lr=0.4, inner_steps=5, fo=False,
                 outer_lr=1e-3, world=1, capturable=False):
        self.model = model
        self.meta_batch = meta_batch
        self.inner_lr = inner_lr
        self.inner_steps = inner_steps
        self.fo = fo
        self.world = world
        self.params = [p for p in model.parameters()]
        # one fused kernel per step on the GPU (foreach kernels elsewhere)
        fused = self.params[0].is_cuda
        self.opt = torch.optim.Adam(self.params, lr=outer_lr, capturable=capturable,
                                    fused=fused or None)
        n = sum(p.numel() for p in self.params)
        self.bucket = torch.zeros(n, dtype=torch.float32, device=self.params[0].device)

    def loss_and_grad(self, tasks: TaskBatch) -> torch.Tensor:
        """Local share of the meta-loss; fills the flat gradient bucket."""
        loss = meta_loss_batched(self.model, tasks, inner_lr=self.inner_lr,
                                 inner_steps=self.inner_steps, fo=self.fo,
                                 reduction="sum", denom=self.meta_batch)
        grads = torch.autograd.grad(loss, self.params)
        torch.cat([g.reshape(-1) for g in grads], out=self.bucket)  # one copy kernel
        return loss.detach()

    def exchange(self) -> None:
        if self.world > 1:
            dist.all_reduce(self.bucket, op=dist.ReduceOp.SUM)

    def apply(self) -> None:
        if self.params[0].grad is None:
            off = 0
            for p in self.params:
                n = p.numel()
                p.grad = self.bucket[off:off + n].view_as(p)  # views of the bucket
                off += n
        self.opt.step()

    def step(self, tasks: TaskBatch) -> torch.Tensor:
        loss = self.loss_and_grad(tasks)
        self.exchange()
        self.apply()
        return loss


class GraphedMetaStep:
    """A MetaStep captured once into a CUDA graph and replayed every step.

    The meta-step is hundreds of small kernels (two encoder layers, five
    inner SGD steps with create_graph=True, the query loss, the
    second-order backward, the gradient all-reduce and Adam); at this
    model size launching them costs more than running them.  Capture
    records the whole step once; each call then copies the new task batch
    into the captured input buffers and replays the graph.

    The wrapped MetaStep's optimizer must be built with capturable=True
    (``MetaStep(..., capturable=True)``); the task batch shapes are fixed
    at capture.  Under torch.distributed the all-reduce is captured too
    (NCCL supports capture; the communicator is warmed up first).

    Construction is not free of side effects: the ``warmup`` eager
    meta-steps run before capture are real steps on ``example``, so they
    update the model's parameters and the optimizer's state (Adam moments
    and step count) ``warmup`` times.  Save and restore both around the
    constructor if the model must start from its current state.
    """

    def __init__(self, meta_step: "MetaStep", example: TaskBatch, warmup: int = 3):
        self.ms = meta_step
        dev = meta_step.bucket.device
        self.static = TaskBatch(*(t.to(dev).clone() for t in
                                  (example.x_s, example.y_s, example.x_q, example.y_q)))
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.ms.step(self.static)
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.loss = self.ms.step(self.static)

    def step(self, tasks: TaskBatch) -> torch.Tensor:
        for dst, src in zip((self.static.x_s, self.static.y_s, self.static.x_q, self.static.y_q),
                            (tasks.x_s, tasks.y_s, tasks.x_q, tasks.y_q)):
            dst.copy_(src, non_blocking=True)
        self.graph.replay()
        return self.loss
