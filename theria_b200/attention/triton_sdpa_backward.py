"""Explicit backward and frozen-stats JVP with the reference's signatures.

Import-path and signature compatible with
``theria/attention/triton_sdpa_backward.py`` (``sdpa_bwd_dq`` :635-696,
``sdpa_bwd_dk`` :401-462, ``sdpa_bwd_dv`` :194-266, ``sdpa_jvp`` :465-503).
There is no Triton here: each call runs the sm_100a kernels of
libtheria_sm100.so.  Stats arrive as the reference's ``(m, l)`` (P =
exp(s q k^T - m) / l) and are folded into the row logsumexp m + log(l).
The head-dim limit is 128 (the reference stops at 64).
"""

from __future__ import annotations

import torch

from theria_b200.attention import ops

_ALLOWED_DTYPES = (torch.float16, torch.bfloat16, torch.float32)


def _assert_backward_contract(q, k, v, dout, m, l, require_v: bool = True):
    """Guardrails, same messages as the reference (:23-64)."""
    tensors = [("q", q), ("k", k), ("dout", dout)] + ([("v", v)] if require_v else [])
    for _, t in tensors:
        if t is None or not t.is_cuda:
            raise AssertionError("Phase9 backward requires CUDA tensors")
    for name, t in tensors:
        if t.dtype not in _ALLOWED_DTYPES:
            raise AssertionError(f"Unsupported dtype for {name}: {t.dtype}")
        if not t.is_contiguous():
            raise AssertionError(f"{name} must be contiguous for Phase9 backward")
    B, H, T, D = q.shape
    if k.ndim != 4 or k.shape[0] != B or k.shape[1] != H or k.shape[3] != D:
        raise AssertionError("k must have shape (B,H,M,D) with D matching q")
    if tuple(dout.shape) != (B, H, T, D):
        raise AssertionError("dout shape must be (B,H,T,D)")
    if require_v and (v.ndim != 4 or v.shape[0] != B or v.shape[1] != H or v.shape[3] != D):
        raise AssertionError("v must have shape (B,H,M,D) with D matching q")
    if tuple(m.shape) != (B, H, T) or tuple(l.shape) != (B, H, T):
        raise AssertionError("m,l must be saved forward stats with shape (B,H,T)")
    if D > ops.MAX_HEAD_DIM:
        raise AssertionError(f"theria_b200 supports D<={ops.MAX_HEAD_DIM}")


def _assert_jvp_contract(q, k, v, dq, dk, dv, m, l):
    """Guardrails, same messages as the reference (:66-103), incl. l > 0."""
    for name, t in (("q", q), ("k", k), ("v", v), ("dq", dq), ("dk", dk), ("dv", dv)):
        if not t.is_cuda:
            raise AssertionError("Phase9 JVP requires CUDA tensors")
        if t.dtype not in _ALLOWED_DTYPES:
            raise AssertionError(f"Unsupported dtype for {name}: {t.dtype}")
        if not t.is_contiguous():
            raise AssertionError(f"{name} must be contiguous for Phase9 JVP")
    B, H, T, D = q.shape
    if k.ndim != 4 or k.shape[0] != B or k.shape[1] != H or k.shape[3] != D:
        raise AssertionError("k must have shape (B,H,M,D) with D matching q")
    if v.ndim != 4 or v.shape[0] != B or v.shape[1] != H or v.shape[3] != D:
        raise AssertionError("v must have shape (B,H,M,D) with D matching q")
    if dq.shape != q.shape or dk.shape != k.shape or dv.shape != v.shape:
        raise AssertionError("dq, dk, dv must match q, k, v shapes respectively")
    if tuple(m.shape) != (B, H, T) or tuple(l.shape) != (B, H, T):
        raise AssertionError("m,l must be saved forward stats with shape (B,H,T)")
    if D > ops.MAX_HEAD_DIM:
        raise AssertionError(f"theria_b200 supports D<={ops.MAX_HEAD_DIM}")
    # The reference performs this host-synchronising check too (:102-103).
    if torch.any(l <= 0):
        raise AssertionError("Phase9 JVP requires l > 0 (forward sumexp stats)")


def _cast(t, dtype):
    return t if t.dtype == dtype else t.to(dtype)


# The reference's callers obtain a backward as three calls on the same
# inputs (sdpa_bwd_dq, sdpa_bwd_dk, sdpa_bwd_dv; ``theria/attention/
# triton_qk.py:384-386``, ``hvp_utils.py:22-26``).  One kernel call yields all
# three gradients at the cost of one, so the first call of such a sequence
# computes all three and keeps the two not asked for; a later call with the
# very same tensor objects, unmodified (version counters unchanged), takes
# its gradient from there, once.  The entry holds references to its inputs,
# so their memory cannot be reused while it lives; any other call replaces
# it.
_pending = {}


def _key(*ts):
    return tuple((id(t), t._version) for t in ts)


def _take(kind, base, v):
    if _pending.get("base") == base and (v is None or _pending.get("v") == v):
        got = _pending["grads"].pop(kind, None)
        if not _pending["grads"]:
            _pending.clear()  # all handed out: release the inputs
        return got
    return None


def _all_three(q, k, v, dout, m, l, scale, causal):
    dt = q.dtype
    dq, dk, dv = ops.backward(q, _cast(k, dt), _cast(v, dt), _cast(dout, dt).contiguous(),
                              ops.lse_from_ml(m, l), causal=causal, scale=float(scale))
    _pending.clear()
    _pending.update(base=_key(q, k, dout, m, l) + ((float(scale), bool(causal)),),
                    v=_key(v), grads={"dq": dq, "dk": dk.to(k.dtype), "dv": dv},
                    refs=(q, k, v, dout, m, l))
    return _pending["grads"]


def sdpa_bwd_dq(q, k, v, dout, m, l, scale, causal: bool = False):
    """dQ = scale * [P * (dP - z)] K, in q.dtype."""
    _assert_backward_contract(q, k, v, dout, m, l)
    base = _key(q, k, dout, m, l) + ((float(scale), bool(causal)),)
    got = _take("dq", base, _key(v))
    return got if got is not None else _all_three(q, k, v, dout, m, l, scale, causal).pop("dq")


def sdpa_bwd_dk(q, k, v, dout, m, l, scale, causal: bool = False):
    """dK = scale * dS^T Q, in k.dtype."""
    _assert_backward_contract(q, k, v, dout, m, l)
    base = _key(q, k, dout, m, l) + ((float(scale), bool(causal)),)
    got = _take("dk", base, _key(v))
    return got if got is not None else _all_three(q, k, v, dout, m, l, scale, causal).pop("dk")


def sdpa_bwd_dv(q, k, dout, m, l, scale, causal: bool = False):
    """dV = P^T dO, in q.dtype.

    dV does not depend on V, and this signature (like the reference's)
    has none; the kernel's V slot receives K, whose values only feed the
    dQ/dK terms that this call does not store.
    """
    _assert_backward_contract(q, k, None, dout, m, l, require_v=False)
    # dV does not depend on V: any pending sequence on these inputs serves
    got = _take("dv", _key(q, k, dout, m, l) + ((float(scale), bool(causal)),), None)
    if got is not None:
        return got
    dt = q.dtype
    kk = _cast(k, dt)
    _, _, dv = ops.backward(q, kk, kk, _cast(dout, dt).contiguous(), ops.lse_from_ml(m, l),
                            causal=causal, scale=float(scale), need=(False, False, True))
    return dv


def sdpa_jvp(q, k, v, dq, dk, dv, m, l, scale, causal: bool = False):
    """Frozen-stats JVP: dO = Pdot V + P dV with P rebuilt from (m, l)."""
    _assert_jvp_contract(q, k, v, dq, dk, dv, m, l)
    dt = q.dtype
    return ops.jvp(q, _cast(k, dt), _cast(v, dt), _cast(dq, dt), _cast(dk, dt),
                   _cast(dv, dt), ops.lse_from_ml(m, l), causal=causal, scale=float(scale))


__all__ = ["sdpa_bwd_dq", "sdpa_bwd_dk", "sdpa_bwd_dv", "sdpa_jvp"]
