"""The drop-in switch on the CPU: after ``install_as_theria()`` the module
names the reference library's callers import resolve to this library, and
the plain-PyTorch comparison math it re-exposes (``theria.attention.
reference*``) agrees with the CPU oracle.  No kernel is launched here."""

import importlib

import pytest
import torch

from oracle import sdpa_oracle as orc
from tests._util import max_rel
from theria_b200.compat import install_as_theria

install_as_theria()

# (module, names) the reference's callers import (theria/attention/__init__.py:10-26,
# custom.py:15-71, triton_qk.py, triton_sdpa_backward.py, hvp_utils.py,
# reference*.py, autograd/sdpa_*.py, maml/loops.py)
SURFACE = [
    ("theria", ["sdpa"]),
    ("theria.attention", ["triton_sdpa_fused", "sdpa_bwd_dq", "sdpa_bwd_dk", "sdpa_bwd_dv",
                          "sdpa_jvp"]),
    ("theria.attention.triton_qk", ["triton_qk", "triton_qk_fast", "triton_qk_softmax",
                                    "TritonQKFunction", "triton_sdpa_fused",
                                    "TritonFusedSDPAFunction", "triton_sdpa_fused_autograd"]),
    ("theria.attention.triton_sdpa_backward", ["sdpa_bwd_dq", "sdpa_bwd_dk", "sdpa_bwd_dv",
                                               "sdpa_jvp"]),
    ("theria.attention.hvp_utils", ["hvp_fd_vjp"]),
    ("theria.attention.custom", ["sdpa_custom", "sdpa_custom_hvp", "sdpa_custom_jvp"]),
    ("theria.attention.reference", ["reference_attention", "sdpa_backward_reference",
                                    "sdpa_jvp_reference", "sdpa_hvp_reference"]),
    ("theria.attention.reference_attention", ["reference_attention", "sdpa_reference"]),
    ("theria.attention.reference_backward_sdpa", ["sdpa_backward_reference"]),
    ("theria.attention.reference_jvp_sdpa", ["sdpa_jvp_reference", "softmax_jvp"]),
    ("theria.attention.reference_hvp_sdpa", ["sdpa_jvp", "sdpa_hvp"]),
    ("theria.autograd.sdpa_function", ["sdpa", "SDPAFunction"]),
    ("theria.autograd.sdpa_custom_function", ["SDPACustom"]),
    ("theria.maml.loops", ["inner_adapt", "outer_loss", "meta_loss_on_tasks", "named_params",
                           "named_buffers", "loss_fn"]),
]


@pytest.mark.parametrize("mod,names", SURFACE)
def test_reference_import_names_resolve_here(mod, names):
    m = importlib.import_module(mod)
    assert getattr(m, "__theria_b200__", False) or m.__name__.startswith("theria_b200")
    for n in names:
        assert hasattr(m, n), (mod, n)


def test_kernel_names_are_this_librarys():
    import theria.attention.triton_qk as tq
    from theria_b200.attention import fused
    assert tq.triton_sdpa_fused is fused.triton_sdpa_fused
    from theria.autograd.sdpa_custom_function import SDPACustom
    assert SDPACustom.__module__.startswith("theria_b200")


def test_sdpa_custom_keeps_the_reference_default_backend():
    from theria.attention.custom import sdpa_custom
    g = torch.Generator("cpu").manual_seed(0)
    q, k, v = (torch.randn(2, 2, 16, 8, generator=g, dtype=torch.float64) for _ in range(3))
    # default = "reference": plain PyTorch on the inputs' device (CPU here)
    assert max_rel(sdpa_custom(q, k, v), orc.attention(q, k, v)) <= 1e-12
    with pytest.raises(ValueError):
        sdpa_custom(q, k, v, backend="nope")


def test_reference_math_agrees_with_the_oracle():
    from theria.attention.reference_backward_sdpa import sdpa_backward_reference
    from theria.attention.reference_hvp_sdpa import sdpa_hvp, sdpa_jvp
    from theria.attention.reference_jvp_sdpa import sdpa_jvp_reference
    g = torch.Generator("cpu").manual_seed(1)
    q, k, v, w, a, b, c = (torch.randn(2, 3, 20, 8, generator=g, dtype=torch.float64)
                           for _ in range(7))
    s = 8 ** -0.5
    for x, r in zip(sdpa_backward_reference(q, k, v, w, s), orc.backward(q, k, v, w)):
        assert max_rel(x, r) <= 1e-12
    assert max_rel(sdpa_jvp_reference(q, k, v, a, b, c, s), orc.jvp(q, k, v, a, b, c)) <= 1e-12
    assert max_rel(sdpa_jvp(q, k, v, a, b, c), orc.jvp(q, k, v, a, b, c)) <= 1e-12
    for x, r in zip(sdpa_hvp(q, k, v, a, b, c), orc.hvp_sum(q, k, v, a, b, c)):
        assert max_rel(x, r) <= 1e-12


def test_install_refuses_to_shadow_another_theria(monkeypatch):
    import sys
    import types

    import theria_b200.compat as compat
    monkeypatch.setattr(compat, "_INSTALLED", False)
    monkeypatch.setitem(sys.modules, "theria", types.ModuleType("theria"))
    with pytest.raises(RuntimeError, match="different `theria`"):
        compat.install_as_theria()
