"""Second-order boundary on the GPU backend, with negative controls.

Pattern of the reference's boundary tests (tests/test_attention_boundary.py:
42-151, tests/_graph_inspect.py:36-52) and of its Phase-11 "bad backend"
diagnostics (experiments/phase11/scripts/bad_backends.py,
run_bad_backend_diagnostics.py:54-87): a probe asks whether grad-of-grad
exists and is non-zero at the attention inputs.  This library's operator
must pass it; wrappers that cut the second-order path (detach, no_grad in
backward, once_differentiable) must fail it -- so the probe is shown to
detect the failure the reference's fused Triton backend had.  The
full-MAML FULL-vs-FO relative difference is then compared with the same
computation on the CPU oracle's attention (the reference backend's math).
"""

import pytest
import torch
from torch.autograd.function import once_differentiable

from oracle import sdpa_oracle as orc

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():
    pytest.skip("CUDA not available", allow_module_level=True)

from theria_b200.attention import ops  # noqa: E402
from theria_b200.attention.custom import sdpa_custom  # noqa: E402


def can_double_backward(fn, inputs):
    """True if grad-of-grad exists and is not identically zero."""
    out = fn(*inputs)
    grads = torch.autograd.grad(out.sum() + (out ** 2).sum(), inputs, create_graph=True)
    if not all(g.requires_grad for g in grads):
        return False
    dummy = sum((g ** 2).sum() for g in grads)
    try:
        gg = torch.autograd.grad(dummy, inputs, allow_unused=True)
    except RuntimeError:
        return False
    return any(x is not None and x.abs().sum().item() > 0 for x in gg)


class _OnceDifferentiable(torch.autograd.Function):
    """Negative control: kernel forward/backward, backward not differentiable."""

    @staticmethod
    def forward(ctx, q, k, v):
        o, lse = ops.forward(q, k, v)
        ctx.save_for_backward(q, k, v, o, lse)
        return o

    @staticmethod
    @once_differentiable
    def backward(ctx, g):
        q, k, v, o, lse = ctx.saved_tensors
        return ops.backward(q, k, v, g.contiguous(), lse, o=o)


def _detached(q, k, v):
    # Negative control: attention weights detached, gradient reaches v only
    return sdpa_custom(q.detach(), k.detach(), v)


def _inputs():
    g = torch.Generator("cpu").manual_seed(0)
    return [torch.randn(2, 2, 32, 16, generator=g).cuda().requires_grad_(True) for _ in range(3)]


def test_fused_backend_has_attention_curvature():
    assert can_double_backward(lambda q, k, v: sdpa_custom(q, k, v), _inputs())
    assert can_double_backward(lambda q, k, v: sdpa_custom(q, k, v, causal=True), _inputs())


def test_probe_detects_once_differentiable_backend():
    assert not can_double_backward(_OnceDifferentiable.apply, _inputs())


def test_probe_detects_detached_attention_weights():
    q, k, v = _inputs()
    out = _detached(q, k, v)
    grads = torch.autograd.grad(out.sum(), (q, k, v), allow_unused=True)
    assert grads[0] is None and grads[1] is None


def test_full_vs_fo_rel_diff_matches_reference_math():
    # rel_diff = |g_full - g_fo| / |g_full| of the meta-gradient (Phase-10
    # diagnostic).  With the attention's curvature kept it must equal the
    # value computed with the CPU oracle's attention, not a smaller one.
    from theria_b200.maml.loops import meta_loss_batched
    from theria_b200.maml.model import MAMLClassifier, ModelConfig
    from theria_b200.maml.tasks import TaskConfig, sample_tasks, stack_tasks

    torch.manual_seed(0)
    m_gpu = MAMLClassifier(ModelConfig()).cuda()
    m_cpu = MAMLClassifier(ModelConfig(), attn_fn=orc.attention).double()
    m_cpu.load_state_dict({k: v.double().cpu() for k, v in m_gpu.state_dict().items()})
    tasks = stack_tasks(sample_tasks(7, 2, TaskConfig(seq_len=32)))

    def rel_diff(model, t):
        gs = []
        for fo in (False, True):
            loss = meta_loss_batched(model, t, inner_lr=0.4, inner_steps=3, fo=fo)
            gs.append(torch.cat([g.reshape(-1) for g in
                                 torch.autograd.grad(loss, list(model.parameters()))]))
        return ((gs[0] - gs[1]).norm() / gs[0].norm()).item()

    r_gpu = rel_diff(m_gpu, tasks.to("cuda"))
    r_cpu = rel_diff(m_cpu, tasks)
    assert r_gpu > 1e-3
    assert abs(r_gpu - r_cpu) <= 1e-3 * max(1.0, r_cpu) + 1e-4
