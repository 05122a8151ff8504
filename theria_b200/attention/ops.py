"""Tensor-level SDPA operators over the C ABI (forward, backward, JVP, HVP).

Each function validates its arguments with the reference's guardrail
messages (``theria/attention/triton_sdpa_backward.py:20-103``), allocates
its outputs with torch on the input's device, and launches on torch's
current stream.  Nothing here computes on the CPU: the CUDA library is the
only implementation, and a missing library raises.

Saved statistics are the row logsumexp ``lse = m + log(l)`` (float32,
``[B, H, T]``), from which P = exp(s q k^T - lse).
"""

from __future__ import annotations

import math

import torch

from theria_b200 import _lib

# float64 runs in double precision in the whole-head kernels only (T, M, D
# <= 64; other shapes raise), for gradcheck-style verification.
_ALLOWED_DTYPES = (torch.float16, torch.bfloat16, torch.float32, torch.float64)

# Each operator is one opaque library call: torch.compile (dynamo) runs it
# eagerly between the graphs it captures around it instead of tracing into
# the ctypes call.
_opaque = torch.compiler.disable
MAX_HEAD_DIM = 128


def default_scale(q: torch.Tensor) -> float:
    return 1.0 / math.sqrt(q.shape[-1])


def _check_tensor(name, t, what):
    if not t.is_cuda:
        raise AssertionError(f"{what} requires CUDA tensors")
    if t.dtype not in _ALLOWED_DTYPES:
        raise AssertionError(f"Unsupported dtype for {name}: {t.dtype}")
    if not t.is_contiguous():
        raise AssertionError(f"{name} must be contiguous for {what}")


def check_qkv(q, k, v, what="theria SDPA"):
    """Shape/dtype/device contract shared by every entry point."""
    for name, t in (("q", q), ("k", k), ("v", v)):
        _check_tensor(name, t, what)
    if q.ndim != 4:
        raise AssertionError("q must have shape (B,H,T,D)")
    B, H, T, D = q.shape
    if k.ndim != 4 or k.shape[0] != B or k.shape[1] != H or k.shape[3] != D:
        raise AssertionError("k must have shape (B,H,M,D) with D matching q")
    if v.ndim != 4 or tuple(v.shape) != tuple(k.shape):
        raise AssertionError("v must have shape (B,H,M,D) with D matching q")
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise AssertionError("q, k, v must share one dtype")
    if not (q.device == k.device == v.device):
        raise AssertionError("q, k, v must be on one device")
    if D > MAX_HEAD_DIM:
        raise AssertionError(f"theria_b200 supports D<={MAX_HEAD_DIM}")
    if k.shape[2] == 0 and T > 0:
        raise AssertionError("k must have at least one key row")
    return B, H, T, k.shape[2], D


def _like(name, t, ref, what):
    _check_tensor(name, t, what)
    if tuple(t.shape) != tuple(ref.shape):
        raise AssertionError(f"{name} shape must be {tuple(ref.shape)}")
    if t.dtype != ref.dtype:
        raise AssertionError(f"{name} dtype must be {ref.dtype}")


def _check_lse(lse, B, H, T):
    if lse.dtype != torch.float32 or tuple(lse.shape) != (B, H, T) or not lse.is_contiguous():
        raise AssertionError("lse must be float32 forward stats with shape (B,H,T)")


@_opaque
def forward(q, k, v, *, causal=False, scale=None, out_dtype=None, need_lse=True):
    """O = softmax(scale q k^T) v and the row logsumexp.

    Returns (o, lse); lse is None when ``need_lse`` is false.
    """
    B, H, T, M, D = check_qkv(q, k, v, "theria forward")
    scale = default_scale(q) if scale is None else float(scale)
    out_dtype = q.dtype if out_dtype is None else out_dtype
    if out_dtype not in (torch.float32, q.dtype):
        raise AssertionError("out_dtype must be float32 or q.dtype")
    o = torch.empty((B, H, T, D), device=q.device, dtype=out_dtype)
    lse = torch.empty((B, H, T), device=q.device, dtype=torch.float32) if need_lse else None
    lib = _lib.load()
    with torch.cuda.device(q.device):
        st = lib.theria_sdpa_fwd(
            _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(o), _lib.DTYPE_CODE[out_dtype],
            _lib.ptr(lse), B, H, T, M, D, _lib.DTYPE_CODE[q.dtype], scale, int(bool(causal)),
            _lib.stream_of(q))
    _lib.check(st, "theria_sdpa_fwd")
    return o, lse


def check_qk(q, k, what):
    """Contract of the dense score / probability kernels (q and k only)."""
    for name, t in (("q", q), ("k", k)):
        _check_tensor(name, t, what)
    if q.ndim != 4 or k.ndim != 4:
        raise AssertionError("q and k must have shape (B,H,T,D) and (B,H,M,D)")
    B, H, T, D = q.shape
    if k.shape[0] != B or k.shape[1] != H or k.shape[3] != D:
        raise AssertionError("Q and K last dimensions must match")
    if k.dtype != q.dtype or k.device != q.device:
        raise AssertionError("q and k must share one dtype and device")
    if D > MAX_HEAD_DIM:
        raise AssertionError(f"theria_b200 supports D<={MAX_HEAD_DIM}")
    return B, H, T, k.shape[2], D


@_opaque
def scores(q, k, *, scale=1.0, out_dtype=torch.float32):
    """Dense S = scale q k^T as [B, H, T, M] (fp32 accumulation)."""
    B, H, T, M, D = check_qk(q, k, "theria scores")
    if out_dtype not in (torch.float32, q.dtype):
        raise AssertionError("out_dtype must be float32 or q.dtype")
    out = torch.empty((B, H, T, M), device=q.device, dtype=out_dtype)
    lib = _lib.load()
    with torch.cuda.device(q.device):
        st = lib.theria_sdpa_scores(
            _lib.ptr(q), _lib.ptr(k), _lib.ptr(out), _lib.DTYPE_CODE[out_dtype], B, H, T, M, D,
            _lib.DTYPE_CODE[q.dtype], float(scale), _lib.stream_of(q))
    _lib.check(st, "theria_sdpa_scores")
    return out


@_opaque
def probs(q, k, *, causal=False, scale=None, lse=None):
    """Dense P = softmax(scale q k^T) as float32 [B, H, T, M].

    The row logsumexp comes from the forward kernel (run with k as values
    when ``lse`` is not given); the probabilities are then one tile pass.
    """
    B, H, T, M, D = check_qk(q, k, "theria probs")
    scale = default_scale(q) if scale is None else float(scale)
    if lse is None:
        _, lse = forward(q, k, k, causal=causal, scale=scale)
    _check_lse(lse, B, H, T)
    out = torch.empty((B, H, T, M), device=q.device, dtype=torch.float32)
    lib = _lib.load()
    with torch.cuda.device(q.device):
        st = lib.theria_sdpa_probs(
            _lib.ptr(q), _lib.ptr(k), _lib.ptr(lse), _lib.ptr(out), B, H, T, M, D,
            _lib.DTYPE_CODE[q.dtype], scale, int(bool(causal)), _lib.stream_of(q))
    _lib.check(st, "theria_sdpa_probs")
    return out


@_opaque
def backward(q, k, v, dout, lse, *, o=None, causal=False, scale=None,
             need=(True, True, True)):
    """dQ, dK, dV of <O, dout>; entries of ``need`` that are False return None."""
    B, H, T, M, D = check_qkv(q, k, v, "theria backward")
    _like("dout", dout, q, "theria backward")
    _check_lse(lse, B, H, T)
    if o is not None:
        _check_tensor("o", o, "theria backward")
        if tuple(o.shape) != tuple(q.shape):
            raise AssertionError("o shape must match q")
    scale = default_scale(q) if scale is None else float(scale)
    dq = torch.empty_like(q) if need[0] else None
    dk = torch.empty_like(k) if need[1] else None
    dv = torch.empty_like(v) if need[2] else None
    lib = _lib.load()
    ws_bytes = lib.theria_sdpa_bwd_workspace_bytes(B, H, T, M, D)
    ws = torch.empty(max(ws_bytes, 1), device=q.device, dtype=torch.uint8)
    o_code = _lib.DTYPE_CODE[o.dtype] if o is not None else 0
    with torch.cuda.device(q.device):
        st = lib.theria_sdpa_bwd(
            _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(o), o_code, _lib.ptr(dout),
            _lib.ptr(lse), _lib.ptr(dq), _lib.ptr(dk), _lib.ptr(dv), _lib.ptr(ws), ws_bytes,
            B, H, T, M, D, _lib.DTYPE_CODE[q.dtype], scale, int(bool(causal)),
            _lib.stream_of(q))
    _lib.check(st, "theria_sdpa_bwd")
    return dq, dk, dv


@_opaque
def jvp(q, k, v, tq, tk, tv, lse, *, causal=False, scale=None):
    """Tangent of O along (tq, tk, tv), P rebuilt from the saved lse."""
    B, H, T, M, D = check_qkv(q, k, v, "theria JVP")
    _like("dq", tq, q, "theria JVP")
    _like("dk", tk, k, "theria JVP")
    _like("dv", tv, v, "theria JVP")
    _check_lse(lse, B, H, T)
    scale = default_scale(q) if scale is None else float(scale)
    o_tan = torch.empty_like(q)
    lib = _lib.load()
    with torch.cuda.device(q.device):
        st = lib.theria_sdpa_jvp(
            _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(tq), _lib.ptr(tk), _lib.ptr(tv),
            _lib.ptr(lse), _lib.ptr(o_tan), B, H, T, M, D, _lib.DTYPE_CODE[q.dtype], scale,
            int(bool(causal)), _lib.stream_of(q))
    _lib.check(st, "theria_sdpa_jvp")
    return o_tan


@_opaque
def hvp(q, k, v, w, lse, tq, tk, tv, *, causal=False, scale=None,
        need=(True, True, True, True)):
    """H u of L = <O, w> along u = (tq, tk, tv), plus J u.

    Returns (hq, hk, hv, o_tan); entries of ``need`` that are False are None.
    """
    B, H, T, M, D = check_qkv(q, k, v, "theria HVP")
    _like("w", w, q, "theria HVP")
    _like("tq", tq, q, "theria HVP")
    _like("tk", tk, k, "theria HVP")
    _like("tv", tv, v, "theria HVP")
    _check_lse(lse, B, H, T)
    scale = default_scale(q) if scale is None else float(scale)
    hq = torch.empty_like(q) if need[0] else None
    hk = torch.empty_like(k) if need[1] else None
    hv = torch.empty_like(v) if need[2] else None
    ot = torch.empty_like(q) if need[3] else None
    lib = _lib.load()
    ws_bytes = lib.theria_sdpa_hvp_workspace_bytes(B, H, T, M, D)
    ws = torch.empty(max(ws_bytes, 1), device=q.device, dtype=torch.uint8)
    with torch.cuda.device(q.device):
        st = lib.theria_sdpa_hvp(
            _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(w), _lib.ptr(lse),
            _lib.ptr(tq), _lib.ptr(tk), _lib.ptr(tv), _lib.ptr(hq), _lib.ptr(hk),
            _lib.ptr(hv), _lib.ptr(ot), _lib.ptr(ws), ws_bytes, B, H, T, M, D,
            _lib.DTYPE_CODE[q.dtype], scale, int(bool(causal)), _lib.stream_of(q))
    _lib.check(st, "theria_sdpa_hvp")
    return hq, hk, hv, ot


def lse_from_ml(m, l):
    """Row logsumexp from the reference's (m, l) stats: lse = m + log(l)."""
    return (m.float() + torch.log(l.float())).contiguous()
