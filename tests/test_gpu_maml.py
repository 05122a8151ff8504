"""Full-MAML on the CUDA attention: meta-loss and meta-gradient equal the
same computation with the CPU oracle's attention (fp64 on the CPU), and
second order differs from first order (test_maml_full_vs_fo.py pattern)."""

import pytest
import torch

from oracle import sdpa_oracle as orc

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():
    pytest.skip("CUDA not available", allow_module_level=True)

from theria_b200.maml.loops import meta_loss_batched, meta_loss_on_tasks  # noqa: E402
from theria_b200.maml.model import MAMLClassifier, ModelConfig  # noqa: E402
from theria_b200.maml.tasks import TaskConfig, sample_tasks, stack_tasks  # noqa: E402


def _grad(model, loss):
    return torch.cat([g.reshape(-1) for g in torch.autograd.grad(loss, list(model.parameters()))])


@pytest.mark.parametrize("fo", [False, True])
def test_meta_gradient_matches_cpu_oracle(fo):
    torch.manual_seed(0)
    m_gpu = MAMLClassifier(ModelConfig()).cuda()
    m_cpu = MAMLClassifier(ModelConfig(), attn_fn=orc.attention).double()
    m_cpu.load_state_dict({k: v.double().cpu() for k, v in m_gpu.state_dict().items()})
    tasks = stack_tasks(sample_tasks(0, 2))
    lg = meta_loss_batched(m_gpu, tasks.to("cuda"), inner_lr=0.4, inner_steps=5, fo=fo)
    lc = meta_loss_batched(m_cpu, tasks, inner_lr=0.4, inner_steps=5, fo=fo)
    assert abs(lg.item() - lc.item()) <= 1e-4 * abs(lc.item())
    gg, gc = _grad(m_gpu, lg).cpu().double(), _grad(m_cpu, lc)
    rel = (gg - gc).abs().max() / gc.abs().max()
    assert rel.item() <= 1e-3


def test_full_vs_first_order_differ_and_sequential_matches_batched():
    torch.manual_seed(1)
    m = MAMLClassifier(ModelConfig()).cuda()
    tasks = [t.to("cuda") for t in sample_tasks(5, 2)]
    full = meta_loss_on_tasks(m, tasks, inner_lr=0.4, inner_steps=2, fo=False)
    bat = meta_loss_batched(m, stack_tasks(tasks), inner_lr=0.4, inner_steps=2, fo=False)
    g_seq, g_bat = _grad(m, full), _grad(m, bat)
    assert ((g_seq - g_bat).abs().max() / g_seq.abs().max()).item() <= 1e-4
    fo = meta_loss_batched(m, stack_tasks(tasks), inner_lr=0.4, inner_steps=2, fo=True)
    g_fo = _grad(m, fo)
    assert ((g_bat - g_fo).norm() / g_bat.norm()).item() > 1e-3
    assert torch.isfinite(g_bat).all()


def test_graphed_meta_step_matches_eager():
    from theria_b200.maml.distributed import GraphedMetaStep, MetaStep
    torch.manual_seed(2)
    m1 = MAMLClassifier(ModelConfig()).cuda()
    m2 = MAMLClassifier(ModelConfig()).cuda()
    m2.load_state_dict(m1.state_dict())
    batches = [stack_tasks(sample_tasks(40 + i, 4)).to("cuda") for i in range(3)]
    eager = MetaStep(m1, meta_batch=4, inner_steps=2, capturable=True)
    graphed_ms = MetaStep(m2, meta_batch=4, inner_steps=2, capturable=True)
    # capture warms up on the first batch (3 steps); mirror that in eager
    g = GraphedMetaStep(graphed_ms, batches[0], warmup=3)
    for _ in range(3):
        eager.step(batches[0])
    for b in batches:
        l1 = eager.step(b)
        l2 = g.step(b)
    torch.cuda.synchronize()
    assert abs(l1.item() - l2.item()) <= 1e-4 * abs(l1.item())
    for p1, p2 in zip(m1.parameters(), m2.parameters()):
        assert (p1 - p2).abs().max().item() <= 1e-4 * max(1.0, p1.abs().max().item())
