"""Pin the CPU oracle against golden vectors produced by the reference itself.

The fixtures (tests/golden/sdpa_*.npz) were written by
tests/golden/make_golden.py, which imports the reference library and runs
its own CPU functions; these tests need no GPU and do not import the
reference.
"""

import pytest
import torch

from oracle import sdpa_oracle as orc
from tests._util import load_golden, max_rel

CASES = ["cfg1", "maml"]


@pytest.mark.parametrize("case", CASES)
def test_oracle_forward_matches_reference(case):
    g = load_golden(case)
    o = orc.attention(g["in_q"], g["in_k"], g["in_v"])
    assert max_rel(o, g["out_o"]) <= 1e-6


@pytest.mark.parametrize("case", CASES)
def test_oracle_backward_matches_reference(case):
    g = load_golden(case)
    dq, dk, dv = orc.backward(g["in_q"], g["in_k"], g["in_v"], g["in_dout"])
    assert max_rel(dq, g["out_dq"]) <= 1e-6
    assert max_rel(dk, g["out_dk"]) <= 1e-6
    assert max_rel(dv, g["out_dv"]) <= 1e-6


@pytest.mark.parametrize("case", CASES)
def test_oracle_jvp_matches_reference(case):
    g = load_golden(case)
    t = orc.jvp(g["in_q"], g["in_k"], g["in_v"], g["in_tq"], g["in_tk"], g["in_tv"])
    assert max_rel(t, g["out_jvp"]) <= 1e-6


@pytest.mark.parametrize("case", CASES)
def test_oracle_hvp_sum_matches_reference_analytic(case):
    g = load_golden(case)
    h = orc.hvp_sum(g["in_q"], g["in_k"], g["in_v"], g["in_vq"], g["in_vk"], g["in_vv"])
    for x, n in zip(h, ("q", "k", "v")):
        assert max_rel(x, g[f"out_hvp_sum_{n}"]) <= 1e-5


@pytest.mark.parametrize("case", CASES)
def test_oracle_hvp_general_w_matches_reference_double_backward(case):
    g = load_golden(case)
    hq, hk, hv, _ = orc.hvp(g["in_q"], g["in_k"], g["in_v"], g["in_dout"],
                            g["in_vq"], g["in_vk"], g["in_vv"])
    for x, n in zip((hq, hk, hv), ("q", "k", "v")):
        assert max_rel(x, g[f"out_hvp_w_{n}"]) <= 1e-5


def _inputs(shape, seed=0):
    gen = torch.Generator("cpu").manual_seed(seed)
    return [torch.randn(*shape, generator=gen, dtype=torch.float64) for _ in range(7)]


@pytest.mark.parametrize("causal", [False, True])
def test_oracle_hvp_matches_autograd_and_fd(causal):
    q, k, v, w, tq, tk, tv = _inputs((1, 2, 24, 8))
    hq, hk, hv, od = orc.hvp(q, k, v, w, tq, tk, tv, causal=causal)
    ag = orc.hvp_autograd(q, k, v, w, tq, tk, tv, causal=causal)
    for a, b in zip((hq, hk, hv), ag):
        assert max_rel(a, b) <= 1e-10

    def grad_fn(q_, k_, v_):
        q_, k_, v_ = (t.detach().requires_grad_(True) for t in (q_, k_, v_))
        loss = (orc.attention(q_, k_, v_, causal=causal) * w).sum()
        return torch.autograd.grad(loss, (q_, k_, v_))

    fd = orc.hvp_fd(grad_fn, q, k, v, tq, tk, tv, eps=1e-4)
    for a, b in zip((hq, hk, hv), fd):
        assert max_rel(a, b) <= 1e-6
    # J u is the derivative of <grad L, u> with respect to w.
    assert max_rel(od, orc.jvp(q, k, v, tq, tk, tv, causal=causal)) <= 1e-12


@pytest.mark.parametrize("causal", [False, True])
def test_oracle_backward_and_jvp_match_autograd(causal):
    q, k, v, w, tq, tk, tv = _inputs((2, 1, 17, 8), seed=1)
    qd, kd, vd = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = orc.attention(qd, kd, vd, causal=causal)
    ga = torch.autograd.grad((o * w).sum(), (qd, kd, vd))
    gb = orc.backward(q, k, v, w, causal=causal)
    for a, b in zip(ga, gb):
        assert max_rel(b, a) <= 1e-12
    _, jv = torch.autograd.functional.jvp(
        lambda a, b, c: orc.attention(a, b, c, causal=causal), (q, k, v), (tq, tk, tv))
    assert max_rel(orc.jvp(q, k, v, tq, tk, tv, causal=causal), jv) <= 1e-12


def test_oracle_frozen_jvp_equals_exact_at_saved_stats():
    q, k, v, _, tq, tk, tv = _inputs((1, 2, 16, 8), seed=2)
    m, l, _ = orc.row_stats(q, k)
    a = orc.jvp_frozen(q.float(), k.float(), v.float(), tq.float(), tk.float(), tv.float(),
                       m, l, 1.0 / 8 ** 0.5)
    b = orc.jvp(q, k, v, tq, tk, tv)
    assert max_rel(a, b) <= 1e-5
