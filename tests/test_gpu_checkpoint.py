"""Activation checkpointing and torch.compile over the fused operator.

The reference's Phase-11 diagnostics wrap the attention in checkpoint
variants (``experiments/phase11/scripts/bad_backends.py:222-268``):
recompute under checkpoint with grad enabled must keep the second-order
path; recompute under ``no_grad`` or a detached recompute must lose it, and
the grad-of-grad probe must tell the two apart.  torch.compile is exercised
with the ``eager`` backend (graph capture by dynamo, no code generation):
the Functions must trace or fall back cleanly and give the eager results.
"""

import pytest
import torch
from torch.utils.checkpoint import checkpoint

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():
    pytest.skip("CUDA not available", allow_module_level=True)

from theria_b200.attention.custom import sdpa_custom  # noqa: E402
from theria_b200.attention.fused import sdpa_fused  # noqa: E402
from tests.test_gpu_boundary import can_double_backward  # noqa: E402


def _inputs(seed=0, shape=(2, 2, 32, 16)):
    g = torch.Generator("cpu").manual_seed(seed)
    return [torch.randn(*shape, generator=g).cuda().requires_grad_(True) for _ in range(3)]


def checkpoint_attention(q, k, v):
    return checkpoint(lambda a, b, c: sdpa_custom(a, b, c), q, k, v, use_reentrant=False)


def checkpoint_no_grad(q, k, v):
    def fn(a, b, c):
        with torch.no_grad():
            return sdpa_custom(a, b, c)
    return checkpoint(fn, q, k, v, use_reentrant=False)


def checkpoint_detach_recompute(q, k, v):
    out = checkpoint(lambda a, b, c: sdpa_custom(a, b, c), q, k, v, use_reentrant=False)
    return out.detach() + out * 0.0


def _grads(fn, inputs, create_graph):
    out = fn(*inputs)
    loss = (out * torch.linspace(-1, 1, out.numel(), device=out.device).view_as(out)).sum()
    return torch.autograd.grad(loss, inputs, create_graph=create_graph)


def test_checkpointed_attention_keeps_curvature():
    assert can_double_backward(checkpoint_attention, _inputs())


def test_checkpointed_attention_matches_plain_first_and_second_order():
    ins = _inputs(1)
    g_plain = _grads(lambda q, k, v: sdpa_custom(q, k, v), ins, True)
    g_ckpt = _grads(checkpoint_attention, ins, True)
    for a, b in zip(g_plain, g_ckpt):
        torch.testing.assert_close(a, b, rtol=1e-6, atol=1e-6)
    # second order: gradient of sum(g^2) through both paths
    h_plain = torch.autograd.grad(sum((g ** 2).sum() for g in g_plain), ins)
    h_ckpt = torch.autograd.grad(sum((g ** 2).sum() for g in g_ckpt), ins)
    for a, b in zip(h_plain, h_ckpt):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("bad", [checkpoint_no_grad, checkpoint_detach_recompute])
def test_probe_detects_broken_checkpoint_variants(bad):
    ins = _inputs(2)
    try:
        ok = can_double_backward(bad, ins)
    except RuntimeError:
        ok = False  # no graph at all: the first-order grad is already gone
    assert not ok


def test_torch_compile_eager_backend_matches_eager():
    def block(q, k, v):
        o = sdpa_fused(q * 1.5, k, v)
        return torch.tanh(o).sum(dim=-1)

    ins = _inputs(3)
    ref = block(*ins)
    g_ref = torch.autograd.grad(ref.sum(), ins)
    compiled = torch.compile(block, backend="eager")
    out = compiled(*ins)
    g = torch.autograd.grad(out.sum(), ins)
    torch.testing.assert_close(out, ref, rtol=0, atol=0)
    for a, b in zip(g, g_ref):
        torch.testing.assert_close(a, b, rtol=0, atol=0)
