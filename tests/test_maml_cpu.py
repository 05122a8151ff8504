"""MAML host logic on the CPU: model, sampler, batched-vs-sequential
equivalence, FULL vs FO, and the task-sharded all-reduce over gloo ranks.
Attention here is the CPU oracle (the CUDA path is exercised by the -m gpu
tests)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import sdpa_oracle as orc
from theria_b200.maml.distributed import MetaStep, broadcast_params, shard_range
from theria_b200.maml.loops import meta_loss_batched, meta_loss_on_tasks
from theria_b200.maml.model import MAMLClassifier, ModelConfig
from theria_b200.maml.tasks import TaskConfig, sample_tasks, stack_tasks


def _model(seed=0, dtype=torch.float32):
    torch.manual_seed(seed)
    return MAMLClassifier(ModelConfig(), attn_fn=orc.attention).to(dtype)


def _flat_grad(model, loss):
    return torch.cat([g.reshape(-1) for g in torch.autograd.grad(loss, list(model.parameters()))])


def test_param_count():
    assert sum(p.numel() for p in _model().parameters()) == 106565


def test_sampler_is_deterministic_and_shaped():
    a = sample_tasks(7, 3)
    b = sample_tasks(7, 3)
    c = sample_tasks(7, 2, start=1)
    assert torch.equal(a[1].x_s, b[1].x_s) and torch.equal(a[1].x_s, c[0].x_s)
    assert a[0].x_s.shape == (25, 64) and a[0].x_q.shape == (75, 64)
    assert int(a[0].x_s.max()) < TaskConfig().vocab
    assert torch.equal(a[0].y_s, torch.arange(5).repeat_interleave(5))


def test_batched_meta_loss_equals_sequential():
    m = _model(dtype=torch.float64)
    tasks = sample_tasks(0, 3, TaskConfig(seq_len=16))
    m.cfg = ModelConfig(seq_len=64)
    seq = meta_loss_on_tasks(m, tasks, inner_lr=0.4, inner_steps=2, fo=False)
    bat = meta_loss_batched(m, stack_tasks(tasks), inner_lr=0.4, inner_steps=2, fo=False)
    assert abs(seq.item() - bat.item()) <= 1e-10 * max(1.0, abs(seq.item()))
    gs, gb = _flat_grad(m, seq), _flat_grad(m, bat)
    assert (gs - gb).abs().max().item() <= 1e-9 * gs.abs().max().item()


def test_full_and_first_order_meta_gradients_differ():
    m = _model(dtype=torch.float64)
    tasks = stack_tasks(sample_tasks(1, 2, TaskConfig(seq_len=16)))
    g_full = _flat_grad(m, meta_loss_batched(m, tasks, inner_lr=0.4, inner_steps=2, fo=False))
    g_fo = _flat_grad(m, meta_loss_batched(m, tasks, inner_lr=0.4, inner_steps=2, fo=True))
    rel = (g_full - g_fo).norm() / g_full.norm()
    assert rel.item() > 1e-3


def test_shard_range():
    assert shard_range(32, 3, 8) == (12, 4)
    with pytest.raises(ValueError):
        shard_range(32, 0, 3)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.manual_seed(100 + rank)  # different init on purpose: broadcast fixes it
    m = MAMLClassifier(ModelConfig(), attn_fn=orc.attention)
    broadcast_params(m)
    meta_batch = 4
    start, per = shard_range(meta_batch, rank, world)
    tasks = stack_tasks(sample_tasks(3, per, TaskConfig(seq_len=16), start=start))
    step = MetaStep(m, meta_batch=meta_batch, inner_steps=1, world=world)
    step.loss_and_grad(tasks)
    step.exchange()
    if rank == 0:
        torch.save(step.bucket.clone(), out)
    dist.destroy_process_group()


def test_task_sharded_allreduce_matches_single_process(tmp_path):
    out = str(tmp_path / "g.pt")
    mp.spawn(_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    g2 = torch.load(out)
    torch.manual_seed(100)
    m = MAMLClassifier(ModelConfig(), attn_fn=orc.attention)
    step = MetaStep(m, meta_batch=4, inner_steps=1, world=1)
    step.loss_and_grad(stack_tasks(sample_tasks(3, 4, TaskConfig(seq_len=16))))
    g1 = step.bucket
    assert (g1 - g2).abs().max().item() <= 1e-5 * g1.abs().max().item()


def test_task_bmm_split_reduction_and_its_derivatives():
    # tbmm splits a long reduction into batch entries (views) and adds the
    # partials; equal to bmm, and differentiable twice through its own
    # backward (which calls tbmm again), for row-major and transposed inputs
    from theria_b200.maml.task_bmm import _split, tbmm
    assert _split(4, 64, 1600, 256) == 8 and _split(32, 64, 1600, 256) == 2
    g = torch.Generator().manual_seed(0)
    a = torch.randn(1, 2, 256, generator=g, dtype=torch.float64, requires_grad=True)
    b = torch.randn(1, 256, 2, generator=g, dtype=torch.float64, requires_grad=True)
    assert _split(1, 2, 256, 2) == 2
    assert torch.allclose(tbmm(a, b), torch.bmm(a, b))
    assert torch.autograd.gradgradcheck(tbmm, (a, b))
    at = torch.randn(1, 256, 2, generator=g, dtype=torch.float64, requires_grad=True)
    assert torch.autograd.gradgradcheck(lambda x, y: tbmm(x.transpose(1, 2), y), (at, b))
