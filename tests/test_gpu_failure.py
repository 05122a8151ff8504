"""Failure detection without a GPU fault: a bounded device-side wait that
must run out.

Every tensor-core kernel bounds its mbarrier waits; when one gives up it
sets the library's device error word to THERIA_ERR_DEVICE_TIMEOUT, raises
its CTA's abort flag so the other warps unwind, and returns.  Here
theria_diag_bounded_wait waits on a phase nothing completes with a short
poll limit, so the timeout path runs for real while the context stays
usable: the test checks the status, that Python callers see it through
check_device_error, that clearing resets it, and that kernels still run
correctly afterwards.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():
    pytest.skip("CUDA not available", allow_module_level=True)

from oracle import sdpa_oracle as orc  # noqa: E402
from tests._util import max_rel  # noqa: E402
from theria_b200 import _lib  # noqa: E402
from theria_b200.attention import ops  # noqa: E402


@pytest.mark.parametrize("polls", [1, 1000])
def test_bounded_wait_times_out_and_unwinds(polls):
    lib = _lib.load()
    _lib.clear_device_error()
    assert _lib.device_error() == _lib.THERIA_OK
    out = torch.zeros(2, dtype=torch.int32, device="cuda")
    st = lib.theria_diag_bounded_wait(polls, ctypes.c_void_p(out.data_ptr()),
                                      _lib.stream_of(out))
    assert st == _lib.THERIA_OK
    torch.cuda.synchronize()  # the kernel returned: no wait hung
    assert out.tolist() == [1, 1]  # first wait gave up, second unwound on abort
    assert _lib.device_error() == _lib.THERIA_ERR_DEVICE_TIMEOUT
    with pytest.raises(_lib.TheriaError, match="timed out"):
        _lib.check_device_error()  # raises and clears
    assert _lib.device_error() == _lib.THERIA_OK


def test_context_usable_after_timeout():
    lib = _lib.load()
    out = torch.zeros(2, dtype=torch.int32, device="cuda")
    assert lib.theria_diag_bounded_wait(10, ctypes.c_void_p(out.data_ptr()),
                                        _lib.stream_of(out)) == _lib.THERIA_OK
    _lib.clear_device_error()
    g = torch.Generator("cpu").manual_seed(3)
    q, k, v = (torch.randn(1, 2, 300, 128, generator=g).to(torch.bfloat16) for _ in range(3))
    o, _ = ops.forward(q.cuda(), k.cuda(), v.cuda())
    torch.cuda.synchronize()
    ref = orc.attention(q.float(), k.float(), v.float())
    assert (o.float().cpu() - ref).abs().max().item() <= 2e-2
    assert _lib.device_error() == _lib.THERIA_OK

