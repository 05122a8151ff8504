"""Test configuration: the repository root on sys.path, the `gpu` marker,
and a check of the library's device-side error word after every GPU test
(a kernel whose bounded wait gave up leaves partial outputs; no GPU test may
pass over one)."""

import sys
from pathlib import Path

import pytest

_ROOT = Path(__file__).resolve().parents[1]
if str(_ROOT) not in sys.path:
    sys.path.insert(0, str(_ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(autouse=True)
def _device_error_word_stays_clear(request):
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import torch
    if not torch.cuda.is_available():
        return
    from theria_b200 import _lib
    if _lib._lib is None:  # the test never loaded the library
        return
    for d in range(torch.cuda.device_count()):
        _lib.check_device_error(d)
