"""The C-ABI library loads and exports every entry point the headers in
include/ declare; host-only calls (status strings, workspace sizes, argument
rejection) behave.  No kernel is launched, so no GPU is needed."""

import ctypes
import os
import re

import pytest

from theria_b200 import _lib

INCLUDE = os.path.join(os.path.dirname(__file__), "..", "include")
HEADERS = sorted(os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h"))


def declared_functions():
    names = set()
    for h in HEADERS:
        src = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        names.update(re.findall(r"\b(theria_\w+)\s*\(", src))
    return sorted(names)


def test_header_declares_the_entry_points():
    names = declared_functions()
    for n in ("theria_sdpa_fwd", "theria_sdpa_bwd", "theria_sdpa_jvp", "theria_sdpa_hvp",
              "theria_ln_fwd", "theria_ln_bwd", "theria_ln_bwd2"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_binding_covers_every_declared_symbol():
    assert set(declared_functions()) == set(_lib.SIGNATURES)


def test_status_strings_and_version():
    lib = _lib.load()
    assert lib.theria_version().decode().startswith("theria-sm100")
    for code in range(6):
        assert lib.theria_status_string(code)
    assert lib.theria_status_string(0).decode() == "ok"


def test_workspace_sizes():
    lib = _lib.load()
    b = lib.theria_sdpa_bwd_workspace_bytes(4, 16, 4096, 4096, 128)
    assert b >= 4 * 16 * 4096 * 4 and b % 256 == 0
    h = lib.theria_sdpa_hvp_workspace_bytes(2, 8, 2048, 2048, 64)
    assert h >= 3 * 2 * 8 * 2048 * 4 and h % 256 == 0


@pytest.mark.parametrize("bad", [
    dict(D=0), dict(D=129), dict(dtype=7), dict(T=-1), dict(B=70000, H=1), dict(M=0),
])
def test_fwd_rejects_bad_arguments_before_touching_the_device(bad):
    lib = _lib.load()
    a = dict(B=1, H=1, T=4, M=4, D=16, dtype=0)
    a.update(bad)
    p = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    st = lib.theria_sdpa_fwd(p, p, p, p, 0, None, a["B"], a["H"], a["T"], a["M"], a["D"],
                             a["dtype"], 0.25, 0, None)
    assert st in (_lib.THERIA_ERR_INVALID_ARG, _lib.THERIA_ERR_UNSUPPORTED)


def test_null_pointers_rejected():
    lib = _lib.load()
    st = lib.theria_sdpa_jvp(None, None, None, None, None, None, None, None,
                             1, 1, 4, 4, 16, 0, 0.25, 0, None)
    assert st == _lib.THERIA_ERR_INVALID_ARG


def test_bwd_without_workspace_rejected():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    st = lib.theria_sdpa_bwd(p, p, p, None, 0, p, p, p, p, p, None, 0,
                             1, 1, 4, 4, 16, 0, 0.25, 0, None)
    assert st == _lib.THERIA_ERR_WORKSPACE


def test_empty_problem_is_a_no_op():
    lib = _lib.load()
    st = lib.theria_sdpa_fwd(None, None, None, None, 0, None, 0, 4, 4, 4, 16, 0, 0.25, 0,
                             None)
    assert st == _lib.THERIA_OK


def test_layer_norm_arguments_checked_on_the_host():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    assert lib.theria_ln_fwd(p, p, p, 512, p, 4, 100, 512, 1e-5, None) == \
        _lib.THERIA_ERR_UNSUPPORTED
    assert lib.theria_ln_fwd(p, p, p, 32, p, 4, 100, 64, 1e-5, None) == \
        _lib.THERIA_ERR_INVALID_ARG  # ldw < D
    assert lib.theria_ln_bwd(p, p, 64, p, p, p, p, None, 0, 4, 100, 64, 1e-5, None) == \
        _lib.THERIA_ERR_WORKSPACE
    assert lib.theria_ln_workspace_bytes(4, 100, 64) == 4 * 7 * 2 * 64 * 4  # ceil(100 / 16) CTAs


def test_packed_attention_arguments_checked_on_the_host():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    # beyond the whole-head kernels (T or D > 64): unsupported, not rerouted
    assert lib.theria_sdpa_qkv_fwd(p, p, p, 2, 4, 65, 16, 0, 0.25, 0, None) == \
        _lib.THERIA_ERR_UNSUPPORTED
    assert lib.theria_sdpa_qkv_bwd(p, p, p, p, 2, 4, 64, 96, 0, 0.25, 0, None) in \
        (_lib.THERIA_ERR_UNSUPPORTED, _lib.THERIA_ERR_INVALID_ARG)
    assert lib.theria_sdpa_qkv_fwd(None, p, p, 2, 4, 64, 16, 0, 0.25, 0, None) == \
        _lib.THERIA_ERR_INVALID_ARG
    # the HVP needs at least one output
    assert lib.theria_sdpa_qkv_hvp(p, p, p, p, None, None, 2, 4, 64, 16, 0, 0.25, 0, None) == \
        _lib.THERIA_ERR_INVALID_ARG
    assert lib.theria_sdpa_qkv_fwd(p, p, p, 0, 4, 64, 16, 0, 0.25, 0, None) == _lib.THERIA_OK


def test_maml_helper_arguments_checked_on_the_host():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    assert lib.theria_rowsum(p, p, None, 0, 4, 100, 64, None) == _lib.THERIA_ERR_WORKSPACE
    assert lib.theria_rowsum(p, p, p, 1 << 20, 4, 100, 2048, None) == _lib.THERIA_ERR_UNSUPPORTED
    assert lib.theria_rowsum_workspace_bytes(4, 300, 64) == 4 * 3 * 64 * 4
    assert lib.theria_add_bias(p, p, 32, None, p, 4, 10, 64, None) == \
        _lib.THERIA_ERR_INVALID_ARG  # ldb < C
    assert lib.theria_chunk_sum(None, p, 4, 8, 100, None) == _lib.THERIA_ERR_INVALID_ARG
    assert lib.theria_gelu_bwd2(p, p, None, p, p, 10, None) == _lib.THERIA_ERR_INVALID_ARG
    assert lib.theria_gelu_bwd2(None, None, None, None, None, 0, None) == _lib.THERIA_OK
    assert lib.theria_ln_bwd2(p, p, 64, p, p, p, 8, p, 64, p, p, p, p, 1 << 20, 4, 100, 64,
                              1e-5, None) == _lib.THERIA_ERR_INVALID_ARG  # lda < D


def test_diag_wait_and_noalloc_query_checked_on_the_host():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    assert lib.theria_diag_bounded_wait(0, p, None) == _lib.THERIA_ERR_INVALID_ARG
    assert lib.theria_diag_bounded_wait(1 << 21, p, None) == _lib.THERIA_ERR_INVALID_ARG
    assert lib.theria_diag_bounded_wait(5, None, None) == _lib.THERIA_ERR_INVALID_ARG
    # which backward the allocation-free entry point runs, from sizes alone
    assert lib.theria_sdpa_bwd_noalloc_uses_tc(1, 2, 257, 257, 128, _lib.BF16) == 1
    assert lib.theria_sdpa_bwd_noalloc_uses_tc(1, 4, 2048, 2048, 128, _lib.BF16) == 0
    assert lib.theria_sdpa_bwd_noalloc_uses_tc(1, 2, 200, 200, 64, _lib.F32) == 0
    assert lib.theria_sdpa_bwd_noalloc_uses_tc(4, 16, 4096, 4096, 128, _lib.BF16) == 0
    assert lib.theria_sdpa_bwd_noalloc_uses_tc(1, 16, 131072, 131072, 64, _lib.BF16) == \
        -_lib.THERIA_ERR_SCRATCH_LIMIT
    assert lib.theria_sdpa_bwd_noalloc_uses_tc(1, 1, 8, 8, 0, _lib.BF16) == \
        -_lib.THERIA_ERR_INVALID_ARG
