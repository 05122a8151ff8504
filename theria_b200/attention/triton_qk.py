"""Names of ``theria/attention/triton_qk.py``: the fused operator and the
partial score / probability kernels.

The fused forward and its autograd wrapper resolve to the sm_100a fused
kernels.  The partial kernels the reference kept next to them (scores
``Q K^T`` with PyTorch softmax and PV; fused ``QK^T`` + softmax with PyTorch
PV) resolve to the dense score / probability kernels of libtheria_sm100.so
(tcgen05 tiles for 16-bit inputs with head dim 64/128, CUDA-core tiles
otherwise).  No Triton is involved.
"""

from __future__ import annotations

import torch

from theria_b200.attention import ops
from theria_b200.attention.fused import (  # noqa: F401
    SDPAFunction,
    TritonFusedSDPAFunction,
    triton_sdpa_fused,
    triton_sdpa_fused_autograd,
)


def _scores_backward(q, k, grad_out):
    # d(q k^T): grad_q = G k, grad_k = G^T q (reference triton_qk.py:117-121,
    # with the operands brought to the gradient's dtype).
    g = grad_out
    grad_q = torch.matmul(g, k.to(g.dtype)).to(q.dtype)
    grad_k = torch.matmul(g.transpose(-2, -1), q.to(g.dtype)).to(k.dtype)
    return grad_q, grad_k


class TritonQKFunction(torch.autograd.Function):
    """scores = q k^T as float32 (reference ``triton_qk.py:73-121``)."""

    @staticmethod
    def forward(ctx, q, k):
        assert q.is_cuda and k.is_cuda, "TritonQKFunction requires CUDA tensors"
        assert q.shape[-1] == k.shape[-1], "Q and K last dimensions must match"
        ctx.save_for_backward(q, k)
        return ops.scores(q.contiguous(), k.contiguous(), scale=1.0, out_dtype=torch.float32)

    @staticmethod
    def backward(ctx, grad_out):
        q, k = ctx.saved_tensors
        return _scores_backward(q, k, grad_out)


def triton_qk(q, k):
    """Scores q k^T (float32) with autograd support (reference ``triton_qk.py:124-126``)."""
    return TritonQKFunction.apply(q, k)


class TritonQKFunctionFast(torch.autograd.Function):
    """scores = q k^T in the input dtype (reference ``triton_qk.py:458-520``).

    The reference accumulated in the 16-bit type ("expect numerical drift");
    here the accumulation is fp32 and only the result is rounded.
    """

    @staticmethod
    def forward(ctx, q, k):
        assert q.is_cuda and k.is_cuda, "TritonQKFunctionFast requires CUDA tensors"
        assert q.shape[-1] == k.shape[-1], "Q and K last dimensions must match"
        out_dtype = q.dtype if q.dtype in (torch.float16, torch.bfloat16) else torch.float32
        ctx.save_for_backward(q, k)
        return ops.scores(q.contiguous(), k.contiguous(), scale=1.0, out_dtype=out_dtype)

    @staticmethod
    def backward(ctx, grad_out):
        q, k = ctx.saved_tensors
        return _scores_backward(q, k, grad_out)


def triton_qk_fast(q, k):
    """Scores q k^T in the input dtype (reference ``triton_qk.py:523-525``)."""
    return TritonQKFunctionFast.apply(q, k)


def triton_qk_softmax(q, k):
    """softmax(q k^T / sqrt(D)) as float32 [B, H, T, M] (reference
    ``triton_qk.py:193-239``); forward only, like the reference."""
    assert q.is_cuda and k.is_cuda
    assert q.is_contiguous() and k.is_contiguous(), \
        "triton_qk_softmax requires contiguous inputs (v0)"
    assert q.shape[-1] == k.shape[-1]
    assert q.shape[-1] <= 128, "triton_qk_softmax supports D <= 128"
    return ops.probs(q, k)
