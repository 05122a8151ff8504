"""CPU oracle for the higher-order SDPA path.

TEST INFRASTRUCTURE ONLY.  This module is the checker: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The product path (``theria_b200``) never
calls it and fails loudly when its CUDA library is missing.

It restates, in plain PyTorch on the CPU, the reference library's own math
for the path (alexgabel/theria).  Each function names the reference
file:line it follows (paths relative to the theria project root).

Parity pins: the restatement is checked in ``tests/test_oracle_golden.py``
against golden vectors that ``tests/golden/make_golden.py`` produced by
importing and running the reference itself (forward, explicit backward, the
fp64 JVP, the analytic sum-loss HVP and ``SDPACustom`` double-backward).
The causal mask and the general-W analytic HVP have no reference
counterpart; they are pinned by autograd of the restated forward.
"""

from __future__ import annotations

import math

import torch

__all__ = [
    "attention",
    "row_stats",
    "backward",
    "jvp",
    "jvp_frozen",
    "hvp",
    "hvp_sum",
    "hvp_autograd",
    "hvp_fd",
    "attention_rows",
    "jvp_rows",
]


def _scores(q, k, scale, causal):
    # reference_attention.py:16-17 -- scores = q k^T / sqrt(d)
    s = torch.matmul(q, k.transpose(-2, -1)) * scale
    if causal:
        # No reference counterpart (theria has no mask, docs/STATUS.md:61-64).
        # Top-left aligned causal mask: query i sees keys j <= i.
        T, M = s.shape[-2], s.shape[-1]
        mask = torch.ones(T, M, dtype=torch.bool).triu(1)
        s = s.masked_fill(mask, float("-inf"))
    return s


def _scale(q, scale):
    return 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale


def attention(q, k, v, scale=None, causal=False):
    """O = softmax(s Q K^T) V.

    Follows ``theria/attention/reference_attention.py:9-19`` (scale fixed to
    1/sqrt(D) there; here it defaults to the same).
    """
    s = _scores(q, k, _scale(q, scale), causal)
    return torch.matmul(torch.softmax(s, dim=-1), v)


def probs(q, k, scale=None, causal=False):
    """P = softmax(scale q k^T) in fp64 (the probabilities of
    ``theria/attention/reference_attention.py:9-19``, and what
    ``theria/attention/triton_qk.py:130-190`` writes)."""
    return torch.softmax(_scores(q.double(), k.double(), _scale(q, scale), causal), dim=-1)


def row_stats(q, k, scale=None, causal=False):
    """Row max ``m`` and sum-exp ``l`` of the scaled scores, and LSE = m + log l.

    The (m, l) convention is the one the reference's fused forward saves,
    ``theria/attention/triton_qk.py:281-304`` (P = exp(s - m) / l).
    """
    s = _scores(q.double(), k.double(), _scale(q, scale), causal)
    m = s.max(dim=-1).values
    l = torch.exp(s - m.unsqueeze(-1)).sum(dim=-1)
    return m.float(), l.float(), (m + torch.log(l)).float()


def backward(q, k, v, dout, scale=None, causal=False):
    """dQ, dK, dV of O against upstream dO, no autograd.

    Follows ``theria/attention/reference_backward_sdpa.py:12-53``:
    dV = P^T dO; dP = dO V^T; z = rowsum(dP * P); dS = P (dP - z);
    dQ = s dS K; dK = s dS^T Q.
    """
    scale = _scale(q, scale)
    with torch.no_grad():
        p = torch.softmax(_scores(q, k, scale, causal), dim=-1)
        dv = torch.matmul(p.transpose(-2, -1), dout)
        dp = torch.matmul(dout, v.transpose(-2, -1))
        z = (dp * p).sum(dim=-1, keepdim=True)
        ds = p * (dp - z)
        dq = torch.matmul(ds, k) * scale
        dk = torch.matmul(ds.transpose(-2, -1), q) * scale
    return dq, dk, dv


def jvp(q, k, v, tq, tk, tv, scale=None, causal=False):
    """Exact forward-mode tangent of O along (tQ, tK, tV), computed in fp64.

    Follows ``theria/attention/reference_jvp_sdpa.py:21-44`` (promotion to
    fp64 at :33-35, cast back to q.dtype at :44).
    """
    scale = _scale(q, scale)
    qf, kf, vf = q.double(), k.double(), v.double()
    tqf, tkf, tvf = tq.double(), tk.double(), tv.double()
    s = _scores(qf, kf, scale, causal)
    p = torch.softmax(s, dim=-1)
    ds = (torch.matmul(tqf, kf.transpose(-2, -1)) + torch.matmul(qf, tkf.transpose(-2, -1))) * scale
    ds = torch.where(torch.isfinite(s), ds, torch.zeros_like(ds))
    dp = p * (ds - (ds * p).sum(dim=-1, keepdim=True))
    return (torch.matmul(dp, vf) + torch.matmul(p, tvf)).to(q.dtype)


def jvp_frozen(q, k, v, tq, tk, tv, m, l, scale):
    """Frozen-stats JVP: P rebuilt from saved (m, l), centring term applied.

    Follows ``theria/attention/triton_sdpa_backward.py:465-503`` (fp32
    compute, result in q.dtype).
    """
    qf, kf, vf = q.float(), k.float(), v.float()
    tqf, tkf, tvf = tq.float(), tk.float(), tv.float()
    s = torch.matmul(qf, kf.transpose(-2, -1)) * scale
    p = torch.exp(s - m.unsqueeze(-1)) / l.unsqueeze(-1)
    ds = (torch.matmul(tqf, kf.transpose(-2, -1)) + torch.matmul(qf, tkf.transpose(-2, -1))) * scale
    dp = p * (ds - (ds * p).sum(dim=-1, keepdim=True))
    return (torch.matmul(dp, vf) + torch.matmul(p, tvf)).to(q.dtype)


def hvp(q, k, v, w, tq, tk, tv, scale=None, causal=False):
    """Analytic Hessian-vector product of L = <O, W> along u = (tQ, tK, tV), fp64.

    Generalises ``theria/attention/reference_hvp_sdpa.py:46-97`` (which fixes
    W = ones) to any W: with dP = W V^T, z = rowsum(P dP),
    dS = P (dP - z), Pdot = softmax-JVP(Sdot), Odot = Pdot V + P tV,
    dPdot = W tV^T, zdot = rowsum(W Odot),
    dSdot = Pdot (dP - z) + P (dPdot - zdot):

        hQ = s (dSdot K + dS tK)
        hK = s (dSdot^T Q + dS^T tQ)
        hV = Pdot^T W

    Returns (hQ, hK, hV, Odot) in q.dtype.  Odot is also the derivative of
    <grad L, u> with respect to W, which the double-backward needs.
    """
    scale = _scale(q, scale)
    qf, kf, vf, wf = q.double(), k.double(), v.double(), w.double()
    tqf, tkf, tvf = tq.double(), tk.double(), tv.double()
    s = _scores(qf, kf, scale, causal)
    p = torch.softmax(s, dim=-1)
    sd = (torch.matmul(tqf, kf.transpose(-2, -1)) + torch.matmul(qf, tkf.transpose(-2, -1))) * scale
    sd = torch.where(torch.isfinite(s), sd, torch.zeros_like(sd))
    pd = p * (sd - (sd * p).sum(dim=-1, keepdim=True))
    od = torch.matmul(pd, vf) + torch.matmul(p, tvf)
    dp = torch.matmul(wf, vf.transpose(-2, -1))
    z = (dp * p).sum(dim=-1, keepdim=True)
    ds = p * (dp - z)
    dpd = torch.matmul(wf, tvf.transpose(-2, -1))
    zd = (wf * od).sum(dim=-1, keepdim=True)
    dsd = pd * (dp - z) + p * (dpd - zd)
    hq = scale * (torch.matmul(dsd, kf) + torch.matmul(ds, tkf))
    hk = scale * (torch.matmul(dsd.transpose(-2, -1), qf) + torch.matmul(ds.transpose(-2, -1), tqf))
    hv = torch.matmul(pd.transpose(-2, -1), wf)
    dt = q.dtype
    return hq.to(dt), hk.to(dt), hv.to(dt), od.to(dt)


def hvp_sum(q, k, v, tq, tk, tv):
    """HVP for L = sum(O): the analytic reference ``sdpa_hvp``.

    Follows ``theria/attention/reference_hvp_sdpa.py:46-97``; equal to
    ``hvp`` with W = ones.
    """
    hq, hk, hv, _ = hvp(q, k, v, torch.ones_like(q), tq, tk, tv)
    return hq, hk, hv


def hvp_autograd(q, k, v, w, tq, tk, tv, scale=None, causal=False):
    """H u by autograd double-backward of the restated forward (fp64).

    The same construction the reference tests use
    (``tests/test_custom_attention_hvp.py:89-104``,
    ``tests/test_triton_fused_hvp_sanity.py:34-44``).
    """
    qd = q.detach().double().requires_grad_(True)
    kd = k.detach().double().requires_grad_(True)
    vd = v.detach().double().requires_grad_(True)
    out = attention(qd, kd, vd, scale, causal)
    loss = (out * w.double()).sum()
    g = torch.autograd.grad(loss, (qd, kd, vd), create_graph=True)
    dot = sum((gi * ti.double()).sum() for gi, ti in zip(g, (tq, tk, tv)))
    return torch.autograd.grad(dot, (qd, kd, vd))


def hvp_fd(grad_fn, q, k, v, tq, tk, tv, eps=1e-3):
    """Central finite difference of a gradient function along (tQ, tK, tV).

    Follows ``theria/attention/hvp_utils.py:30-49``:
    [grad(x + eps u) - grad(x - eps u)] / (2 eps).
    """
    gp = grad_fn(q + eps * tq, k + eps * tk, v + eps * tv)
    gm = grad_fn(q - eps * tq, k - eps * tk, v - eps * tv)
    return tuple((a - b) * (0.5 / eps) for a, b in zip(gp, gm))


def _row_mask(rows, M):
    # causal mask for query rows at absolute positions `rows` (top-left aligned)
    return torch.arange(M).unsqueeze(0) > rows.unsqueeze(1)


def attention_rows(q, k, v, rows, scale=None, causal=False):
    """Rows ``rows`` of O and of the row LSE, computed in fp64 from only those
    query rows: row i of ``reference_attention.py:9-19`` depends on q_i and
    all of K, V, so long sequences are checked on a sample of rows.

    q, k, v are one head each ([N, D] or [M, D]); returns (O[rows], LSE[rows]).
    """
    scale = _scale(q, scale)
    qr = q[rows].double()
    s = torch.matmul(qr, k.double().transpose(-2, -1)) * scale
    if causal:
        s = s.masked_fill(_row_mask(rows, k.shape[0]), float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    return torch.matmul(torch.exp(s - lse.unsqueeze(-1)), v.double()), lse


def jvp_rows(q, k, v, tq, tk, tv, rows, scale=None, causal=False):
    """Rows ``rows`` of the exact tangent Odot (fp64), as ``jvp`` computes it
    (``reference_jvp_sdpa.py:21-44``) but from only those query rows."""
    scale = _scale(q, scale)
    qr, tqr = q[rows].double(), tq[rows].double()
    kf, vf, tkf, tvf = k.double(), v.double(), tk.double(), tv.double()
    s = torch.matmul(qr, kf.transpose(-2, -1)) * scale
    sd = (torch.matmul(tqr, kf.transpose(-2, -1)) + torch.matmul(qr, tkf.transpose(-2, -1))) * scale
    if causal:
        mask = _row_mask(rows, k.shape[0])
        s = s.masked_fill(mask, float("-inf"))
        sd = sd.masked_fill(mask, 0.0)
    p = torch.softmax(s, dim=-1)
    pd = p * (sd - (sd * p).sum(dim=-1, keepdim=True))
    return torch.matmul(pd, vf) + torch.matmul(p, tvf)
