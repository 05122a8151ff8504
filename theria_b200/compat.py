"""Make ``import theria...`` resolve to this library (the drop-in switch).

``install_as_theria()`` registers, in ``sys.modules``, the module names the
reference library's callers import (paths inside the theria project):

=========================================  ==========================================
``theria``                                 ``sdpa`` (``theria/__init__.py:1``)
``theria.attention``                       ``triton_sdpa_fused``, ``sdpa_bwd_dq/dk/dv``,
                                           ``sdpa_jvp`` (``attention/__init__.py:10-26``)
``theria.attention.triton_qk``             ``triton_qk``, ``triton_qk_fast``,
                                           ``triton_qk_softmax``, ``TritonQKFunction``,
                                           ``TritonQKFunctionFast``, ``triton_sdpa_fused``,
                                           ``TritonFusedSDPAFunction``,
                                           ``triton_sdpa_fused_autograd``
``theria.attention.triton_sdpa_backward``  ``sdpa_bwd_dq/dk/dv``, ``sdpa_jvp``
``theria.attention.hvp_utils``             ``hvp_fd_vjp``, ``_explicit_grads_sum``
``theria.attention.custom``                ``sdpa_custom`` (default backend
                                           ``"reference"``, as ``custom.py:15``),
                                           ``sdpa_custom_hvp``, ``sdpa_custom_jvp``
``theria.attention.reference*``            the plain-PyTorch comparison math
``theria.autograd.sdpa_function``          ``sdpa``, ``SDPAFunction``
``theria.autograd.sdpa_custom_function``   ``SDPACustom``
``theria.maml`` / ``theria.maml.loops``    the MAML loops
=========================================  ==========================================

Every kernel-backed name is this library's (hand-written sm_100a kernels
behind libtheria_sm100.so); the ``reference*`` modules are the reference's
own PyTorch formulas, kept for the comparisons its callers make.  The
reference's ``theria.models`` / ``theria.tasks`` demo code is not provided.

Call it once, before the first ``import theria``::

    import theria_b200.compat
    theria_b200.compat.install_as_theria()
    from theria.attention.custom import sdpa_custom   # -> theria_b200

or run an unchanged pytest suite with ``-p theria_b200.pytest_theria``.
"""

from __future__ import annotations

import sys
import types

_INSTALLED = False


def _module(name, doc, **attrs):
    m = types.ModuleType(name, doc)
    m.__dict__.update(attrs)
    m.__all__ = [k for k in attrs if not k.startswith("_")]
    m.__theria_b200__ = True
    return m


def install_as_theria(force: bool = False) -> None:
    """Register the ``theria.*`` module names listed in this module's doc.

    Raises ``RuntimeError`` if another ``theria`` package is already imported
    (unless ``force``, which replaces it).  Idempotent."""
    global _INSTALLED
    if _INSTALLED:
        return
    have = sys.modules.get("theria")
    if have is not None and not getattr(have, "__theria_b200__", False) and not force:
        raise RuntimeError("a different `theria` package is already imported; call "
                           "install_as_theria() before importing it, or pass force=True")

    from theria_b200.attention import custom as _custom
    from theria_b200.attention import fused, hvp_utils, reference, triton_qk
    from theria_b200.attention import triton_sdpa_backward as tsb
    from theria_b200.autograd import sdpa_custom_function as scf
    from theria_b200.autograd import sdpa_function as sf
    from theria_b200.maml import loops

    def sdpa_custom(q, k, v, *, backend: str = "reference", causal: bool = False):
        """``theria.attention.custom.sdpa_custom``: the reference's default
        backend ("reference", ``custom.py:15``); every other name runs this
        library's kernels (see ``theria_b200.attention.custom``)."""
        return _custom.sdpa_custom(q, k, v, backend=backend, causal=causal)

    bwd = dict(sdpa_bwd_dq=tsb.sdpa_bwd_dq, sdpa_bwd_dk=tsb.sdpa_bwd_dk,
               sdpa_bwd_dv=tsb.sdpa_bwd_dv, sdpa_jvp=tsb.sdpa_jvp)
    mods = {
        "theria.attention.triton_qk": _module(
            "theria.attention.triton_qk", triton_qk.__doc__,
            triton_qk=triton_qk.triton_qk, triton_qk_fast=triton_qk.triton_qk_fast,
            triton_qk_softmax=triton_qk.triton_qk_softmax,
            TritonQKFunction=triton_qk.TritonQKFunction,
            TritonQKFunctionFast=triton_qk.TritonQKFunctionFast,
            triton_sdpa_fused=fused.triton_sdpa_fused,
            TritonFusedSDPAFunction=fused.TritonFusedSDPAFunction,
            triton_sdpa_fused_autograd=fused.triton_sdpa_fused_autograd),
        "theria.attention.triton_sdpa_backward": _module(
            "theria.attention.triton_sdpa_backward", tsb.__doc__, **bwd),
        "theria.attention.hvp_utils": _module(
            "theria.attention.hvp_utils", hvp_utils.__doc__, hvp_fd_vjp=hvp_utils.hvp_fd_vjp,
            _explicit_grads_sum=hvp_utils._explicit_grads_sum),
        "theria.attention.custom": _module(
            "theria.attention.custom", _custom.__doc__, sdpa_custom=sdpa_custom,
            sdpa_custom_hvp=_custom.sdpa_custom_hvp, sdpa_custom_jvp=_custom.sdpa_custom_jvp),
        "theria.attention.reference_attention": _module(
            "theria.attention.reference_attention", reference.__doc__,
            reference_attention=reference.reference_attention,
            sdpa_reference=reference.sdpa_reference),
        "theria.attention.reference_backward_sdpa": _module(
            "theria.attention.reference_backward_sdpa", reference.__doc__,
            sdpa_backward_reference=reference.sdpa_backward_reference),
        "theria.attention.reference_jvp_sdpa": _module(
            "theria.attention.reference_jvp_sdpa", reference.__doc__,
            softmax_jvp=reference.softmax_jvp, sdpa_jvp_reference=reference.sdpa_jvp_reference,
            sdpa_jvp=reference.sdpa_jvp_reference),
        "theria.attention.reference_hvp_sdpa": _module(
            "theria.attention.reference_hvp_sdpa", reference.__doc__,
            sdpa_jvp=reference.sdpa_jvp, sdpa_hvp=reference.sdpa_hvp,
            sdpa_hvp_reference=reference.sdpa_hvp_reference),
        "theria.attention.reference": _module(
            "theria.attention.reference", reference.__doc__,
            reference_attention=reference.reference_attention,
            sdpa_reference=reference.sdpa_reference,
            sdpa_backward_reference=reference.sdpa_backward_reference,
            sdpa_jvp_reference=reference.sdpa_jvp_reference,
            sdpa_hvp_reference=reference.sdpa_hvp_reference),
        "theria.autograd.sdpa_function": _module(
            "theria.autograd.sdpa_function", sf.__doc__, sdpa=sf.sdpa,
            SDPAFunction=sf.SDPAFunction),
        "theria.autograd.sdpa_custom_function": _module(
            "theria.autograd.sdpa_custom_function", scf.__doc__, SDPACustom=scf.SDPACustom),
        "theria.maml.loops": loops,
    }
    pkgs = {
        "theria": _module("theria", __doc__, sdpa=sf.sdpa),
        "theria.attention": _module("theria.attention", None,
                                    triton_sdpa_fused=fused.triton_sdpa_fused, **bwd),
        "theria.autograd": _module("theria.autograd", None),
        "theria.maml": _module("theria.maml", None),
    }
    for name, m in pkgs.items():
        m.__path__ = []  # a package: submodules resolve through sys.modules
    allm = {**pkgs, **mods}
    for name, m in allm.items():
        sys.modules[name] = m
    for name, m in allm.items():  # attribute access: theria.attention.custom, ...
        if "." in name:
            parent, child = name.rsplit(".", 1)
            setattr(allm[parent], child, m)
    _INSTALLED = True


__all__ = ["install_as_theria"]
