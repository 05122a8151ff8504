"""Packed self-attention (theria_sdpa_qkv_*): forward, gradient and second
derivative equal the unpacked operator on the same heads; fp64 gradcheck and
gradgradcheck of the packed kernels themselves."""

import pytest
import torch

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():
    pytest.skip("CUDA not available", allow_module_level=True)

from theria_b200.attention.fused import sdpa_fused  # noqa: E402
from theria_b200.attention.packed import sdpa_qkv  # noqa: E402


def _unpacked(qkv, causal):
    q, k, v = qkv.permute(2, 0, 3, 1, 4).unbind(0)
    return sdpa_fused(q, k, v, causal=causal).transpose(1, 2)


def _derivs(fn, qkv0, r0, v0, causal):
    qkv = qkv0.clone().requires_grad_(True)
    r = r0.clone().requires_grad_(True)
    o = fn(qkv, causal)
    (g,) = torch.autograd.grad((o * r).sum(), (qkv,), create_graph=True)
    return (o, g) + torch.autograd.grad((g * v0).sum(), (qkv, r))


@pytest.mark.parametrize("shape", [(6, 64, 4, 16), (3, 37, 2, 24), (2, 64, 1, 64)])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_packed_equals_unpacked(shape, causal, dtype):
    B, T, H, D = shape
    g = torch.Generator("cpu").manual_seed(T + D)
    qkv0 = torch.randn(B, T, 3, H, D, generator=g).to(dtype).cuda()
    r0 = torch.randn(B, T, H, D, generator=g).to(dtype).cuda()
    v0 = torch.randn(B, T, 3, H, D, generator=g).to(dtype).cuda()
    a = _derivs(sdpa_qkv, qkv0, r0, v0, causal)
    b = _derivs(_unpacked, qkv0, r0, v0, causal)
    for x, y in zip(a, b):
        assert x.shape == y.shape
        # same kernels, same arithmetic: only the memory layout differs
        assert torch.equal(x, y) or (x.float() - y.float()).abs().max() <= 1e-6 * (
            y.float().abs().max() + 1)


def test_packed_gradcheck_and_gradgradcheck_fp64():
    g = torch.Generator("cpu").manual_seed(5)
    qkv = torch.randn(2, 6, 3, 2, 8, generator=g, dtype=torch.float64).cuda().requires_grad_()
    for causal in (False, True):
        fn = lambda x: sdpa_qkv(x, causal=causal)  # noqa: E731
        assert torch.autograd.gradcheck(fn, (qkv,))
        assert torch.autograd.gradgradcheck(fn, (qkv,))


def test_long_sequences_take_the_general_path():
    qkv = torch.randn(1, 100, 3, 2, 16, device="cuda", requires_grad=True)
    o = sdpa_qkv(qkv)
    assert o.shape == (1, 100, 2, 16)
    assert torch.allclose(o, _unpacked(qkv, False), atol=1e-6)
