"""Dense score / probability kernels and the partial-kernel backends of
``sdpa_custom`` (the reference's ``triton_qk``, ``triton_fast``,
``triton_qk_softmax``), against the CPU oracle.

Reference tests followed: ``tests/test_triton_qk.py`` (scores vs
q @ k^T and the ``triton_qk`` backend vs ``reference``, atol 5e-3),
``tests/test_triton_fast_relaxed.py`` (cosine > 0.99, atol 1e-1),
``tests/test_triton_forward_matches_reference.py`` (``triton_ref``, fp16,
atol 2e-2), ``tests/test_triton_gradcheck.py`` (gradcheck of
``TritonQKFunction``).  Scores are exact products of the (rounded) inputs
accumulated in fp32, so fp32 and 16-bit inputs share the fp32 tolerance
when the output is fp32; 16-bit outputs add one rounding.
"""

import pytest
import torch

from oracle import sdpa_oracle as orc
from tests._util import max_abs, max_rel

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():
    pytest.skip("CUDA not available", allow_module_level=True)

from theria_b200 import _lib  # noqa: E402
from theria_b200.attention import ops  # noqa: E402
from theria_b200.attention.custom import sdpa_custom  # noqa: E402
from theria_b200.attention.triton_qk import (  # noqa: E402
    TritonQKFunction, triton_qk, triton_qk_fast, triton_qk_softmax)

DTYPES = [torch.float32, torch.bfloat16, torch.float16]
# (B, H, T, M, D): tcgen05 tiles (D 64/128, ragged edges) and CUDA-core tiles
SHAPES = [(1, 2, 128, 128, 64), (2, 1, 200, 130, 128), (1, 1, 4, 8, 8), (2, 2, 33, 70, 20),
          (1, 3, 257, 63, 64)]


def _qk(shape, dtype, seed=0):
    B, H, T, M, D = shape
    g = torch.Generator("cpu").manual_seed(seed)
    q = torch.randn(B, H, T, D, generator=g).to(dtype)
    k = torch.randn(B, H, M, D, generator=g).to(dtype)
    return q, k


def _ref_scores(q, k, scale=1.0):
    return torch.matmul(q.double(), k.double().transpose(-2, -1)) * scale


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("dtype", DTYPES)
def test_scores_fp32_out(shape, dtype):
    q, k = _qk(shape, dtype)
    s = ops.scores(q.cuda(), k.cuda(), scale=0.5)
    assert s.dtype == torch.float32 and s.shape == (*shape[:3], shape[3])
    assert max_rel(s, _ref_scores(q, k, 0.5)) <= 1e-5


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_scores_input_dtype_out(shape, dtype):
    q, k = _qk(shape, dtype, seed=1)
    s = ops.scores(q.cuda(), k.cuda(), out_dtype=dtype)
    assert s.dtype == dtype
    ref = _ref_scores(q, k)
    # one rounding of the result to the 16-bit type
    assert (s.double().cpu() - ref).abs().max().item() <= 8e-3 * ref.abs().max().item()


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("causal", [False, True])
def test_probs_match_oracle_softmax(shape, dtype, causal):
    q, k = _qk(shape, dtype, seed=2)
    if causal and shape[2] > shape[3]:
        pytest.skip("causal rows past the last key have no valid key")
    p = ops.probs(q.cuda(), k.cuda(), causal=causal)
    P = orc.probs(q.float(), k.float(), causal=causal)
    if dtype == torch.float32:
        assert max_rel(p, P) <= 1e-5
    else:
        assert max_abs(p, P) <= 2e-2
    rows = p.double().sum(-1).cpu()
    assert (rows - 1).abs().max().item() <= 1e-4


def test_scores_unaligned_output_and_strided_inputs():
    # an output row length that breaks 16-byte vector stores (M % 4 != 0),
    # and inputs that are views (made contiguous by the wrapper)
    q, k = _qk((1, 2, 40, 37, 64), torch.bfloat16, seed=3)
    qd = q.cuda().transpose(1, 2).contiguous().transpose(1, 2)
    s = triton_qk(qd, k.cuda())
    assert max_rel(s, _ref_scores(q, k)) <= 1e-5


def test_triton_qk_backend_matches_reference_backend():
    # reference tests/test_triton_qk.py:32-51
    g = torch.Generator("cpu").manual_seed(0)
    q, k, v = (torch.randn(1, 1, 4, 8, generator=g).cuda().requires_grad_(True) for _ in range(3))
    out = sdpa_custom(q, k, v, backend="triton_qk").float()
    ref = sdpa_custom(q, k, v, backend="reference").float()
    torch.testing.assert_close(out, ref, rtol=5e-3, atol=5e-3)
    assert max_rel(out, orc.attention(q.detach().cpu(), k.detach().cpu(), v.detach().cpu())) <= 1e-5
    # gradients flow through the scores kernel's backward
    gq, gk, gv = torch.autograd.grad(out.sum(), (q, k, v))
    rq, rk, rv = orc.backward(q.detach().cpu(), k.detach().cpu(), v.detach().cpu(),
                              torch.ones(1, 1, 4, 8))
    for x, r in ((gq, rq), (gk, rk), (gv, rv)):
        assert max_rel(x, r) <= 1e-5


@pytest.mark.parametrize("backend", ["triton_ref", "triton", "triton_qk_softmax"])
def test_partial_backends_fp16(backend):
    # reference tests/test_triton_forward_matches_reference.py:23-37
    g = torch.Generator("cpu").manual_seed(0)
    q, k, v = (torch.randn(2, 3, 64, 32, generator=g).to(torch.float16) for _ in range(3))
    out = sdpa_custom(q.cuda(), k.cuda(), v.cuda(), backend=backend)
    assert out.dtype == torch.float16
    assert max_abs(out, orc.attention(q.float(), k.float(), v.float())) <= 2e-2


def test_triton_fast_relaxed():
    # reference tests/test_triton_fast_relaxed.py:8-27
    g = torch.Generator("cpu").manual_seed(0)
    q, k, v = (torch.randn(1, 1, 4, 8, generator=g).to(torch.float16).cuda() for _ in range(3))
    out = sdpa_custom(q, k, v, backend="triton_fast").float()
    ref = sdpa_custom(q, k, v, backend="reference").float()
    cos = torch.nn.functional.cosine_similarity(out.flatten(), ref.flatten(), dim=0)
    assert cos > 0.99
    torch.testing.assert_close(out, ref, rtol=1e-1, atol=1e-1)
    s = triton_qk_fast(q, k)
    assert s.dtype == torch.float16


def test_triton_qk_gradcheck():
    # reference tests/test_triton_gradcheck.py:8-28
    g = torch.Generator("cpu").manual_seed(0)
    q = torch.randn(1, 1, 2, 3, generator=g).cuda().requires_grad_(True)
    k = torch.randn(1, 1, 2, 3, generator=g).cuda().requires_grad_(True)
    assert torch.autograd.gradcheck(lambda a, b: TritonQKFunction.apply(a, b), (q, k),
                                    eps=1e-3, atol=1e-3, rtol=1e-2, fast_mode=True)


def test_qk_softmax_contract():
    q, k = _qk((1, 2, 16, 24, 32), torch.float32, seed=4)
    p = triton_qk_softmax(q.cuda(), k.cuda())
    P = orc.probs(q, k)
    assert p.dtype == torch.float32 and max_rel(p, P) <= 1e-5
    with pytest.raises(AssertionError, match="contiguous"):
        triton_qk_softmax(q.cuda().transpose(2, 3), k.cuda().transpose(2, 3))


def test_scores_and_probs_launch_library_kernels():
    lib = _lib.load()
    n0 = lib.theria_launch_count()
    q, k = _qk((1, 1, 128, 128, 128), torch.bfloat16)
    ops.scores(q.cuda(), k.cuda())
    ops.probs(q.cuda(), k.cuda())
    torch.cuda.synchronize()
    assert lib.theria_launch_count() - n0 >= 3  # scores, forward (LSE), probs
