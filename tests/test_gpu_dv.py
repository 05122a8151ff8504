"""Value head dim Dv different from the query/key head dim D.

The reference's formula allows v of shape (B, H, M, Dv)
(``theria/attention/reference_attention.py:9-19``) while its fused path
asserts Dv == D.  Here the fused operator accepts Dv != D (zero-padding to a
common kernel width, exact); forward, gradients, the double-backward HVP and
the forward-mode tangent are compared with the CPU oracle."""

import pytest
import torch

from oracle import sdpa_oracle as orc
from tests._util import max_abs, max_rel

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():
    pytest.skip("CUDA not available", allow_module_level=True)

from theria_b200.attention.custom import sdpa_custom  # noqa: E402
from theria_b200.autograd.sdpa_function import sdpa  # noqa: E402

CASES = [  # (B, H, T, M, D, Dv, dtype, causal)
    (2, 2, 48, 40, 16, 48, torch.float32, False),     # whole-head kernels
    (1, 2, 130, 100, 64, 32, torch.float32, True),    # CUDA-core kernels
    (1, 2, 300, 257, 64, 128, torch.bfloat16, False),  # tensor cores, q/k padded
    (2, 1, 200, 200, 128, 64, torch.float16, True),   # tensor cores, v padded
    (1, 2, 256, 256, 96, 40, torch.bfloat16, False),  # both padded to 128
]


def _ok(x, r, dt, tol32):
    if dt == torch.float32:
        return max_rel(x, r) <= tol32
    return max_abs(x, r) <= 2e-2 if r.abs().max() < 8 else max_rel(x, r) <= 2e-2


@pytest.mark.parametrize("case", CASES)
def test_dv_differs_from_d(case):
    B, H, T, M, D, Dv, dt, causal = case
    g = torch.Generator("cpu").manual_seed(11)
    q, tq = (torch.randn(B, H, T, D, generator=g) for _ in range(2))
    k, tk = (torch.randn(B, H, M, D, generator=g) for _ in range(2))
    v, tv = (torch.randn(B, H, M, Dv, generator=g) for _ in range(2))
    w = torch.randn(B, H, T, Dv, generator=g)
    q, k, v, tq, tk, tv, w = (t.to(dt) for t in (q, k, v, tq, tk, tv, w))
    qd, kd, vd = (t.cuda().requires_grad_(True) for t in (q, k, v))
    out = sdpa_custom(qd, kd, vd, causal=causal)
    assert out.shape == (B, H, T, Dv) and out.dtype == dt
    grads = torch.autograd.grad((out * w.cuda()).sum(), (qd, kd, vd), create_graph=True)
    dot = sum((a * t.cuda()).sum() for a, t in zip(grads, (tq, tk, tv)))
    hvp = torch.autograd.grad(dot, (qd, kd, vd))
    f32 = [t.float() for t in (q, k, v, w, tq, tk, tv)]
    assert _ok(out.float().cpu(), orc.attention(*f32[:3], causal=causal), dt, 1e-5)
    for a, r in zip(grads, orc.backward(*f32[:4], causal=causal)):
        assert a.shape == r.shape
        assert _ok(a.float().cpu(), r, dt, 1e-5)
    for a, r in zip(hvp, orc.hvp(*f32, causal=causal)[:3]):
        assert _ok(a.float().cpu(), r.float(), dt, 1e-4)


def test_dv_forward_mode_tangent():
    g = torch.Generator("cpu").manual_seed(12)
    q, k, tq, tk = (torch.randn(1, 2, 70, 32, generator=g) for _ in range(4))
    v, tv = (torch.randn(1, 2, 70, 48, generator=g) for _ in range(2))
    import torch.autograd.forward_ad as fwAD
    with fwAD.dual_level():
        duals = [fwAD.make_dual(x.cuda(), t.cuda()) for x, t in ((q, tq), (k, tk), (v, tv))]
        jv = fwAD.unpack_dual(sdpa(*duals)).tangent
    assert max_rel(jv.cpu(), orc.jvp(q, k, v, tq, tk, tv)) <= 1e-5
