"""fp64 variant of the whole-head kernels: gradcheck and gradgradcheck on the
GPU, as the reference runs them on its CPU path
(``tests/test_sdpa_gradcheck.py:17-23``), plus direct parity with the fp64
oracle.  The saved row logsumexp is float32; the fp64 kernels rebuild it
from the scores in double precision so every derivative stays smooth.
"""

import pytest
import torch

from oracle import sdpa_oracle as orc
from tests._util import max_rel

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():
    pytest.skip("CUDA not available", allow_module_level=True)

from theria_b200 import _lib  # noqa: E402
from theria_b200.attention import ops  # noqa: E402
from theria_b200.attention.fused import sdpa_fused  # noqa: E402
from theria_b200.autograd.sdpa_function import sdpa  # noqa: E402


def _draw(shape_q, shape_k, n_q, n_k, seed=0, requires_grad=False):
    g = torch.Generator("cpu").manual_seed(seed)
    qs = [torch.randn(*shape_q, generator=g, dtype=torch.float64).cuda() for _ in range(n_q)]
    ks = [torch.randn(*shape_k, generator=g, dtype=torch.float64).cuda() for _ in range(n_k)]
    if requires_grad:
        for t in qs + ks:
            t.requires_grad_(True)
    return qs, ks


def test_sdpa_gradcheck_fp64():
    # reference tests/test_sdpa_gradcheck.py:17-23 (shape [1,1,4,8], double)
    (q,), (k, v) = _draw((1, 1, 4, 8), (1, 1, 4, 8), 1, 2, requires_grad=True)
    assert torch.autograd.gradcheck(lambda *xs: sdpa(*xs), (q, k, v))


@pytest.mark.parametrize("causal", [False, True])
def test_sdpa_gradgradcheck_fp64(causal):
    (q,), (k, v) = _draw((1, 2, 5, 6), (1, 2, 5, 6), 1, 2, seed=1, requires_grad=True)
    fn = lambda a, b, c: sdpa_fused(a, b, c, causal=causal)  # noqa: E731
    assert torch.autograd.gradcheck(fn, (q, k, v))
    assert torch.autograd.gradgradcheck(fn, (q, k, v))


@pytest.mark.parametrize("shape", [(2, 2, 16, 24, 8), (1, 3, 33, 20, 16), (1, 1, 40, 48, 32)])
@pytest.mark.parametrize("causal", [False, True])
def test_fp64_kernels_match_fp64_oracle(shape, causal):
    B, H, T, M, D = shape
    if causal and T > M:
        pytest.skip("causal rows past the last key have no valid key")
    (q, do, w, tq), (k, v, tk, tv) = _draw((B, H, T, D), (B, H, M, D), 4, 4, seed=2)
    # the C ABI carries the scale as float32: give the oracle the same value
    sc = float(torch.tensor(D ** -0.5, dtype=torch.float32))
    o, lse = ops.forward(q, k, v, causal=causal, scale=sc)
    assert o.dtype == torch.float64
    c = [t.cpu() for t in (q, k, v, do, w, tq, tk, tv)]
    assert max_rel(o, orc.attention(c[0], c[1], c[2], scale=sc, causal=causal)) <= 1e-10
    grads = ops.backward(q, k, v, do, lse, o=o, causal=causal, scale=sc)
    for x, r in zip(grads, orc.backward(c[0], c[1], c[2], c[3], scale=sc, causal=causal)):
        assert max_rel(x, r) <= 1e-10
    ot = ops.jvp(q, k, v, tq, tk, tv, lse, causal=causal, scale=sc)
    assert max_rel(ot, orc.jvp(c[0], c[1], c[2], c[5], c[6], c[7], scale=sc, causal=causal)) <= 1e-10
    h = ops.hvp(q, k, v, w, lse, tq, tk, tv, causal=causal, scale=sc)
    ref = orc.hvp(c[0], c[1], c[2], c[4], c[5], c[6], c[7], scale=sc, causal=causal)
    for x, r in zip(h, ref):
        assert max_rel(x, r) <= 1e-10


def test_fp64_outside_the_whole_head_kernels_is_refused():
    (q,), (k, v) = _draw((1, 1, 128, 16), (1, 1, 128, 16), 1, 2)
    with pytest.raises(_lib.TheriaError, match="status 2"):
        ops.forward(q, k, v)
