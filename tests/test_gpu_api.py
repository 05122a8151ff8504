"""The reference-facing API on the GPU: compat signatures with external
(m, l) stats, the autograd contracts (first and second order), the
finite-difference HVP utility, and full-MAML meta-gradients against the CPU
oracle.  Patterns follow the reference's own tests (test_triton_sdpa_dq.py,
test_triton_fused_backward_parity.py, test_triton_sdpa_jvp.py,
test_custom_attention_hvp.py, test_attention_boundary.py,
test_maml_full_vs_fo.py)."""

import pytest
import torch

from oracle import sdpa_oracle as orc
from tests._util import max_abs, max_rel

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():
    pytest.skip("CUDA not available", allow_module_level=True)

from theria_b200.attention import (hvp_fd_vjp, sdpa_bwd_dk, sdpa_bwd_dq,  # noqa: E402
                                   sdpa_bwd_dv, sdpa_jvp, triton_sdpa_fused)
from theria_b200.attention.custom import sdpa_custom, sdpa_custom_hvp, sdpa_custom_jvp  # noqa: E402
from theria_b200.autograd import SDPACustom, sdpa  # noqa: E402

DEV = "cuda"


def _qkv(shape, dtype=torch.float32, seed=0, n=3):
    g = torch.Generator("cpu").manual_seed(seed)
    return [torch.randn(*shape, generator=g).to(dtype) for _ in range(n)]


@pytest.mark.parametrize("shape", [(1, 1, 32, 32), (2, 4, 128, 64)])
def test_fused_forward_fp32_output_and_stats(shape):
    q, k, v = (t.to(DEV) for t in _qkv(shape, torch.float16))
    out, m, l = triton_sdpa_fused(q, k, v, return_stats=True)
    assert out.dtype == torch.float32 and m.shape == shape[:3] and l.shape == shape[:3]
    ref = orc.attention(q.float().cpu(), k.float().cpu(), v.float().cpu())
    assert max_abs(out, ref) <= 2e-2
    # (m, l) obey the reference convention P = exp(s - m) / l
    s = (q.float() @ k.float().transpose(-2, -1)) / shape[-1] ** 0.5
    p = torch.exp(s - m.unsqueeze(-1)) / l.unsqueeze(-1)
    assert max_abs(p.sum(-1), torch.ones_like(l)) <= 1e-3


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("shape", [(1, 1, 32, 32), (2, 4, 128, 64)])
def test_compat_backward_with_external_stats(dtype, shape):
    q, k, v, do = (t.to(DEV) for t in _qkv(shape, dtype, n=4))
    scale = 1.0 / shape[-1] ** 0.5
    s = (q.float() @ k.float().transpose(-2, -1)) * scale
    m = s.max(dim=-1).values
    l = torch.exp(s - m.unsqueeze(-1)).sum(dim=-1)
    ref = orc.backward(*(t.float().cpu() for t in (q, k, v, do)))
    tol = 2e-2 if dtype != torch.float32 else None
    got = (sdpa_bwd_dq(q, k, v, do, m, l, scale), sdpa_bwd_dk(q, k, v, do, m, l, scale),
           sdpa_bwd_dv(q, k, do, m, l, scale))
    for x, r in zip(got, ref):
        assert x.dtype == dtype
        if tol:
            assert max_abs(x, r) <= tol
        else:
            assert max_rel(x, r) <= 1e-5


def test_compat_jvp_with_external_stats_matches_exact():
    q, k, v, tq, tk, tv = (t.to(DEV) for t in _qkv((2, 4, 128, 64), torch.float32, n=6))
    scale = 1.0 / 8.0
    s = (q @ k.transpose(-2, -1)) * scale
    m = s.max(dim=-1).values
    l = torch.exp(s - m.unsqueeze(-1)).sum(dim=-1)
    got = sdpa_jvp(q, k, v, tq, tk, tv, m, l, scale)
    ref = orc.jvp(*(t.cpu() for t in (q, k, v, tq, tk, tv)))
    assert max_rel(got, ref) <= 1e-5
    with pytest.raises(AssertionError, match="l > 0"):
        sdpa_jvp(q, k, v, tq, tk, tv, m, torch.zeros_like(l), scale)


@pytest.mark.parametrize("backend", ["triton_full_fused", "custom"])
@pytest.mark.parametrize("causal", [False, True])
def test_double_backward_matches_oracle_hvp(backend, causal):
    q, k, v, w, tq, tk, tv = _qkv((2, 2, 64, 32), n=7, seed=3)
    qd, kd, vd = (t.to(DEV).requires_grad_(True) for t in (q, k, v))
    out = sdpa_custom(qd, kd, vd, backend=backend, causal=causal)
    loss = (out * w.to(DEV)).sum()
    g = torch.autograd.grad(loss, (qd, kd, vd), create_graph=True)
    assert all(x.requires_grad for x in g)
    dot = sum((a * t.to(DEV)).sum() for a, t in zip(g, (tq, tk, tv)))
    h = torch.autograd.grad(dot, (qd, kd, vd))
    ref = orc.hvp_autograd(q, k, v, w, tq, tk, tv, causal=causal)
    for a, b in zip(h, ref):
        assert max_rel(a, b) <= 1e-4
    gref = orc.backward(q, k, v, w, causal=causal)
    for a, b in zip(g, gref):
        assert max_rel(a, b) <= 1e-5


def test_double_backward_gradient_wrt_upstream_is_the_jvp():
    # d/d(dO) <grad, u> = J u: reach it by making the upstream gradient a leaf.
    q, k, v, w, tq, tk, tv = _qkv((1, 2, 48, 16), n=7, seed=4)
    qd, kd, vd = (t.to(DEV).requires_grad_(True) for t in (q, k, v))
    wd = w.to(DEV).requires_grad_(True)
    out = sdpa(qd, kd, vd)
    g = torch.autograd.grad(out, (qd, kd, vd), grad_outputs=wd, create_graph=True)
    dot = sum((a * t.to(DEV)).sum() for a, t in zip(g, (tq, tk, tv)))
    (gw,) = torch.autograd.grad(dot, (wd,))
    assert max_rel(gw, orc.jvp(q, k, v, tq, tk, tv)) <= 1e-5


def test_grad_of_grad_exists():
    # test_attention_boundary.py:42-93 pattern: sum of first grads is differentiable
    q, k, v = (t.to(DEV).requires_grad_(True) for t in _qkv((1, 1, 8, 16)))
    loss = sdpa_custom(q, k, v).sum()
    grads = torch.autograd.grad(loss, (q, k, v), create_graph=True)
    dummy = sum(g.sum() for g in grads)
    torch.autograd.grad(dummy, (q, k, v), allow_unused=False)


def test_custom_helpers_match_oracle():
    q, k, v, tq, tk, tv = _qkv((1, 2, 16, 8), n=6, seed=5)
    d = [t.to(DEV) for t in (q, k, v, tq, tk, tv)]
    for a, b in zip(sdpa_custom_hvp(*d), orc.hvp_sum(q, k, v, tq, tk, tv)):
        assert max_rel(a, b) <= 1e-4
    assert max_rel(sdpa_custom_jvp(*d), orc.jvp(q, k, v, tq, tk, tv)) <= 1e-5
    for a, b in zip(SDPACustom.hvp(*d), orc.hvp_sum(q, k, v, tq, tk, tv)):
        assert max_rel(a, b) <= 1e-4


def test_fd_hvp_agrees_with_analytic():
    # test_triton_fused_hvp_sanity.py pattern, tightened: FD of the kernel VJP
    # against the analytic HVP kernel (fp32, eps 1e-3).
    q, k, v, tq, tk, tv = _qkv((2, 2, 64, 32), n=6, seed=6)
    d = [t.to(DEV) for t in (q, k, v, tq, tk, tv)]
    fd = hvp_fd_vjp(*d, eps=1e-3)
    an = sdpa_custom_hvp(*d)
    ref = orc.hvp_sum(q, k, v, tq, tk, tv)
    for a, b, r in zip(fd, an, ref):
        assert torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0) > 0.999
        assert max_rel(a, r) <= 5e-2


def test_fp32_double_backward_cfg1():
    # BASELINE cfg1: [2,2,64,32] fp32, HVP of sum(O * dO) along v ~ N(0,1)
    q, k, v, do, vq, vk, vv = _qkv((2, 2, 64, 32), n=7, seed=0)
    qd, kd, vd = (t.to(DEV).requires_grad_(True) for t in (q, k, v))
    g = torch.autograd.grad((sdpa(qd, kd, vd) * do.to(DEV)).sum(), (qd, kd, vd),
                            create_graph=True)
    dot = sum((a * t.to(DEV)).sum() for a, t in zip(g, (vq, vk, vv)))
    h = torch.autograd.grad(dot, (qd, kd, vd))
    ref = orc.hvp(q.double(), k.double(), v.double(), do.double(), vq.double(), vk.double(),
                  vv.double())
    for a, b in zip(h, ref[:3]):
        assert max_rel(a, b) <= 1e-4

    def grad_fn(q_, k_, v_):
        q_, k_, v_ = (t.detach().requires_grad_(True) for t in (q_, k_, v_))
        loss = (orc.attention(q_, k_, v_) * do.double()).sum()
        return torch.autograd.grad(loss, (q_, k_, v_))

    fd = orc.hvp_fd(grad_fn, q.double(), k.double(), v.double(), vq.double(), vk.double(),
                    vv.double(), eps=1e-3)
    for a, b in zip(h, fd):
        assert max_rel(a, b) <= 1e-4


def test_double_backward_through_strided_views():
    # Heads split out of a fused projection arrive as non-contiguous views;
    # the second-order path must still reach the tensor they view.
    g = torch.Generator("cpu").manual_seed(7)
    x = torch.randn(2, 48, 3, 2, 16, generator=g)  # (B, T, qkv, H, D)
    w, tq = torch.randn(2, 2, 48, 16, generator=g), torch.randn(2, 48, 3, 2, 16, generator=g)
    xd = x.to(DEV).requires_grad_(True)
    q, k, v = xd.permute(2, 0, 3, 1, 4)
    assert not q.is_contiguous()
    out = sdpa(q, k, v)
    (gx,) = torch.autograd.grad((out * w.to(DEV)).sum(), (xd,), create_graph=True)
    (hx,) = torch.autograd.grad((gx * tq.to(DEV)).sum(), (xd,))
    xc = x.double().requires_grad_(True)
    qc, kc, vc = xc.permute(2, 0, 3, 1, 4)
    (gc,) = torch.autograd.grad((orc.attention(qc, kc, vc) * w.double()).sum(), (xc,),
                                create_graph=True)
    (hc,) = torch.autograd.grad((gc * tq.double()).sum(), (xc,))
    assert max_rel(gx, gc) <= 1e-5
    assert max_rel(hx, hc) <= 1e-4


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("shape", [(2, 2, 64, 32), (1, 2, 200, 64)])
def test_forward_mode_ad_uses_the_jvp_kernel(causal, shape):
    import torch.autograd.forward_ad as fwAD
    q, k, v, tq, tk, tv = _qkv(shape, n=6, seed=8)
    with fwAD.dual_level():
        duals = [fwAD.make_dual(x.to(DEV), t.to(DEV)) for x, t in ((q, tq), (k, tk), (v, tv))]
        out = sdpa(*duals, causal=causal)
        primal, tangent = fwAD.unpack_dual(out)
    assert max_rel(primal, orc.attention(q, k, v, causal=causal)) <= 1e-5
    assert max_rel(tangent, orc.jvp(q, k, v, tq, tk, tv, causal=causal)) <= 1e-5


def test_three_call_backward_computes_once():
    # the reference's pattern: sdpa_bwd_dq, _dk, _dv on the same inputs
    from theria_b200 import _lib
    from theria_b200.attention.triton_sdpa_backward import sdpa_bwd_dk, sdpa_bwd_dq, sdpa_bwd_dv
    g = torch.Generator("cpu").manual_seed(9)
    q, k, v, do = (torch.randn(2, 2, 200, 64, generator=g).to(torch.bfloat16).cuda()
                   for _ in range(4))
    scale = 64 ** -0.5
    s = torch.matmul(q.float(), k.float().transpose(-2, -1)) * scale
    m = s.max(dim=-1).values
    l = torch.exp(s - m.unsqueeze(-1)).sum(dim=-1)
    lib = _lib.load()
    n0 = lib.theria_launch_count()
    dq = sdpa_bwd_dq(q, k, v, do, m, l, scale)
    n1 = lib.theria_launch_count()
    dk = sdpa_bwd_dk(q, k, v, do, m, l, scale)
    dv = sdpa_bwd_dv(q, k, do, m, l, scale)
    assert n1 > n0 and lib.theria_launch_count() == n1  # dk, dv: no new launches
    ref = orc.backward(q.float().cpu(), k.float().cpu(), v.float().cpu(), do.float().cpu())
    for x, r in zip((dq, dk, dv), ref):
        assert (x.float().cpu() - r).abs().max().item() <= 2e-2
    # a modified input is never served from the kept results
    do.mul_(2.0)
    dk2 = sdpa_bwd_dk(q, k, v, do, m, l, scale)
    assert lib.theria_launch_count() > n1
    assert (dk2.float().cpu() - 2 * ref[1]).abs().max().item() <= 4e-2
