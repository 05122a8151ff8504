"""Fused task-batched LayerNorm (include/theria_ln.h): forward, gradient and
second derivative against the composed torch form in float64 on the CPU,
with affine rows taken as strided views of a padded flat buffer (the MAML
fast-weight layout) and head dims that do and do not fill the warp lanes."""

import pytest
import torch

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():
    pytest.skip("CUDA not available", allow_module_level=True)

from theria_b200.maml.layer_norm import layer_norm, layer_norm_reference  # noqa: E402


def _rel(a, b):
    return ((a.double().cpu() - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def _inputs(nt, rows, D, seed):
    g = torch.Generator("cpu").manual_seed(seed)
    x = torch.randn(nt, *rows, D, generator=g) * 2 + 0.5
    flat = torch.zeros(nt, 2 * D + 40)           # padded rows: stride != D
    flat[:, :D] = 1 + 0.3 * torch.randn(nt, D, generator=g)
    flat[:, D + 8:2 * D + 8] = torch.randn(nt, D, generator=g)
    r = torch.randn(nt, *rows, D, generator=g)
    vx = torch.randn(nt, *rows, D, generator=g)
    vw, vb = torch.randn(nt, D, generator=g), torch.randn(nt, D, generator=g)
    return x, flat, r, vx, vw, vb


def _run(fn, x, flat, r, vx, vw, vb, D):
    flat = flat.clone().requires_grad_(True)
    w, b = flat[:, :D], flat[:, D + 8:2 * D + 8]
    x = x.clone().requires_grad_(True)
    r = r.clone().requires_grad_(True)
    y = fn(x, w, b)
    gx, gw, gb = torch.autograd.grad((y * r).sum(), (x, w, b), create_graph=True)
    l2 = (gx * vx).sum() + (gw * vw).sum() + (gb * vb).sum()
    dx, dflat, dr = torch.autograd.grad(l2, (x, flat, r))
    return y, gx, gw, gb, dx, dflat[:, :D], dr


@pytest.mark.parametrize("nt,rows,D", [(3, (5, 7), 64), (2, (130,), 48), (1, (3, 64), 100),
                                       (4, (1,), 16)])
def test_layer_norm_matches_composed_torch(nt, rows, D):
    args = _inputs(nt, rows, D, seed=D)
    ref = _run(layer_norm_reference, *(t.double() for t in args), D)
    got = _run(layer_norm, *(t.cuda() for t in args), D)
    names = ["y", "gx", "gw", "gb", "d2x", "d2w", "d2gy"]
    for n, a, b in zip(names, got, ref):
        tol = 1e-5 if n in ("y", "gx", "gw", "gb") else 1e-4
        assert _rel(a, b) <= tol, (n, _rel(a, b))


def test_layer_norm_second_derivative_without_some_cotangents():
    # only gx is used downstream: the gw / gb cotangents arrive as None
    x, flat, r, vx, _, _ = _inputs(2, (9,), 64, seed=3)

    def run(fn, dev, dt):
        xx = x.to(dev, dt).requires_grad_(True)
        w = flat[:, :64].to(dev, dt).requires_grad_(True)
        b = flat[:, 72:136].to(dev, dt)
        y = fn(xx, w, b)
        (gx,) = torch.autograd.grad((y * r.to(dev, dt)).sum(), (xx,), create_graph=True)
        return torch.autograd.grad((gx * vx.to(dev, dt)).sum(), (xx, w))

    for a, b in zip(run(layer_norm, "cuda", torch.float32),
                    run(layer_norm_reference, "cpu", torch.float64)):
        assert _rel(a, b) <= 1e-4


def test_layer_norm_refuses_non_float32():
    x = torch.randn(2, 4, 64, device="cuda", dtype=torch.float16)
    w = torch.ones(2, 64, device="cuda", dtype=torch.float16)
    with pytest.raises(ValueError):
        layer_norm(x, w, w)


def test_task_linear_first_and_second_derivatives():
    # tbmm (split long reductions) + add_bias (row-sum bias gradient), as the
    # model's linears use them, against plain torch in float64
    from theria_b200.maml.task_bmm import add_bias, tbmm
    g = torch.Generator("cpu").manual_seed(7)
    h0 = torch.randn(3, 1600, 64, generator=g)
    flat0 = torch.randn(3, 70 * 64 + 70 + 30, generator=g)
    r0 = torch.randn(3, 1600, 70, generator=g)
    v0 = torch.randn(3, 1600, 64, generator=g)

    res0 = torch.randn(3, 1600, 70, generator=g)

    def run(lin, dev, dt):
        h = h0.to(dev, dt).requires_grad_(True)
        flat = flat0.to(dev, dt).requires_grad_(True)
        res = res0.to(dev, dt).requires_grad_(True)
        w = flat[:, :70 * 64].view(3, 70, 64)
        b = flat[:, 70 * 64 + 30:]
        y = lin(h, w, b, res)
        gh, gflat, gres = torch.autograd.grad((y.square() * r0.to(dev, dt)).sum(),
                                              (h, flat, res), create_graph=True)
        l2 = (gh * v0.to(dev, dt)).sum() + gflat.square().sum() + gres.square().sum()
        return (y, gh, gflat, gres) + torch.autograd.grad(l2, (h, flat, res))

    got = run(lambda h, w, b, res: add_bias(tbmm(h, w.transpose(1, 2)), b, res), "cuda",
              torch.float32)
    ref = run(lambda h, w, b, res: res + torch.bmm(h, w.transpose(1, 2)) + b.unsqueeze(1),
              "cpu", torch.float64)
    for a, b in zip(got, ref):
        assert _rel(a, b) <= 1e-5


def test_gelu_second_derivative_matches_torch():
    from theria_b200.maml.layer_norm import gelu
    g = torch.Generator("cpu").manual_seed(11)
    x0 = torch.randn(3, 50, 256, generator=g) * 2
    r0, v0 = torch.randn(3, 50, 256, generator=g), torch.randn(3, 50, 256, generator=g)

    def run(fn, dev, dt):
        x = x0.to(dev, dt).requires_grad_(True)
        r = r0.to(dev, dt).requires_grad_(True)
        y = fn(x)
        (gx,) = torch.autograd.grad((y * r).sum(), (x,), create_graph=True)
        return (y, gx) + torch.autograd.grad((gx * v0.to(dev, dt)).sum(), (x, r))

    for a, b in zip(run(gelu, "cuda", torch.float32),
                    run(torch.nn.functional.gelu, "cpu", torch.float64)):
        assert _rel(a, b) <= 1e-5


def test_layer_norm_single_task_with_degenerate_row_strides():
    # one task: affine rows taken from a transposed [D, 1] view have row
    # stride 1 < D (torch still calls them contiguous); only row 0 is read,
    # so the kernels must accept them (first and second derivatives)
    D = 64
    g = torch.Generator("cpu").manual_seed(5)
    x = (torch.randn(1, 7, D, generator=g) * 2).double()
    wcol = (1 + 0.3 * torch.randn(D, 1, generator=g)).double()
    bcol = torch.randn(D, 1, generator=g).double()
    r, vx = torch.randn(1, 7, D, generator=g).double(), torch.randn(1, 7, D, generator=g).double()
    outs = []
    for dev, fn in (("cuda", layer_norm), ("cpu", layer_norm_reference)):
        xd = x.to(dev).float().requires_grad_(True) if dev == "cuda" else x.clone().requires_grad_(True)
        wd = (wcol.to(dev).float() if dev == "cuda" else wcol.clone()).requires_grad_(True)
        bd = (bcol.to(dev).float() if dev == "cuda" else bcol.clone()).requires_grad_(True)
        w, b = wd.t(), bd.t()  # [1, D] views with stride (1, 1)
        assert w.stride() == (1, 1)
        y = fn(xd, w, b)
        gx, gw, gb = torch.autograd.grad((y * r.to(dev).to(y.dtype)).sum(), (xd, w, b),
                                         create_graph=True)
        l2 = (gx * vx.to(dev).to(gx.dtype)).sum() + gw.sum() + gb.sum()
        outs.append([y, gx, gw, gb] + list(torch.autograd.grad(l2, (xd, wd))))
    for a, b in zip(*outs):
        assert _rel(a, b.double()) <= 1e-4
