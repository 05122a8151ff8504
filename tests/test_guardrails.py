"""Loud host-side validation with the reference's messages (no GPU needed:
every check fires before a kernel is launched)."""

import pytest
import torch

from theria_b200.attention import (sdpa_bwd_dq, sdpa_bwd_dk, sdpa_bwd_dv, sdpa_jvp,
                                   triton_sdpa_fused)
from theria_b200.attention.custom import sdpa_custom
from theria_b200.attention import ops


def _cpu(shape=(1, 1, 4, 8)):
    return [torch.randn(*shape) for _ in range(3)]


def test_backward_requires_cuda():
    q, k, v = _cpu()
    m = torch.zeros(1, 1, 4)
    with pytest.raises(AssertionError, match="requires CUDA"):
        sdpa_bwd_dq(q, k, v, q, m, m + 1, 0.3)
    with pytest.raises(AssertionError, match="requires CUDA"):
        sdpa_bwd_dk(q, k, v, q, m, m + 1, 0.3)
    with pytest.raises(AssertionError, match="requires CUDA"):
        sdpa_bwd_dv(q, k, q, m, m + 1, 0.3)


def test_jvp_requires_cuda():
    q, k, v = _cpu()
    m = torch.zeros(1, 1, 4)
    with pytest.raises(AssertionError, match="requires CUDA"):
        sdpa_jvp(q, k, v, q, k, v, m, m + 1, 0.3)


def test_forward_requires_cuda():
    q, k, v = _cpu()
    with pytest.raises(AssertionError):
        triton_sdpa_fused(q, k, v)
    with pytest.raises(AssertionError, match="requires CUDA"):
        ops.forward(q, k, v)


def test_unknown_backend_is_rejected_not_rerouted():
    q, k, v = _cpu()
    for name in ("bogus", "triton_qk_fused", ""):
        with pytest.raises(ValueError, match="Unsupported sdpa_custom backend"):
            sdpa_custom(q, k, v, backend=name)


def test_partial_kernel_backends_require_cuda():
    # reference triton_qk.py:80, 193-194: the partial kernels assert CUDA
    q, k, v = _cpu()
    for name in ("triton_qk", "triton_ref", "triton", "triton_fast", "triton_qk_softmax"):
        with pytest.raises(AssertionError):
            sdpa_custom(q, k, v, backend=name)


def test_causal_needs_a_fused_backend():
    q, k, v = _cpu()
    with pytest.raises(ValueError, match="causal"):
        sdpa_custom(q, k, v, backend="triton_qk", causal=True)


def test_no_cpu_fallback_for_fused_backend():
    q, k, v = _cpu()
    with pytest.raises(AssertionError, match="requires CUDA"):
        sdpa_custom(q, k, v, backend="triton_full_fused")


def test_packed_attention_and_layer_norm_refuse_cpu_tensors_loudly():
    # the packed attention has no CPU path; the MAML LayerNorm / GELU use the
    # composed torch form only for CPU tensors (the CPU model of the tests)
    import torch.nn.functional as F
    from theria_b200.attention.packed import sdpa_qkv
    from theria_b200.maml.layer_norm import gelu, layer_norm, layer_norm_reference
    with pytest.raises(AssertionError, match="CUDA"):
        sdpa_qkv(torch.randn(1, 4, 3, 2, 8))
    x, w, b = torch.randn(2, 5, 16), torch.rand(2, 16) + 0.5, torch.randn(2, 16)
    assert torch.allclose(layer_norm(x, w, b), layer_norm_reference(x, w, b))
    assert torch.allclose(gelu(x), F.gelu(x))
