"""The allocation-free backward entry point, theria_sdpa_bwd_noalloc.

Some callers cannot allocate device memory when they call the backward:
code that runs under a memory pool or foreign allocator which forbids
cudaMalloc, or a plain C host that holds only raw device pointers and has no
allocator to make a workspace with.  theria_sdpa_bwd_noalloc serves them by
using a fixed scratch array inside the library instead of a caller-provided
workspace.  These tests call it through the C ABI and check that two calls
in a row give the same dQ/dK/dV as the regular entry point (with its own
workspace), within the suite's tolerances, and that problems too large for
the fixed scratch are refused with THERIA_ERR_SCRATCH_LIMIT.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test.
"""

import ctypes

import pytest
import torch

from oracle import sdpa_oracle as orc
from tests._util import max_abs, max_rel

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():
    pytest.skip("CUDA not available", allow_module_level=True)

from theria_b200 import _lib  # noqa: E402
from theria_b200.attention import ops  # noqa: E402

CODE = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}


def _inputs(shape, dtype, seed):
    g = torch.Generator("cpu").manual_seed(seed)
    return [torch.randn(*shape, generator=g).to(dtype).cuda() for _ in range(4)]


def _bwd_regular(lib, q, k, v, o, do, lse, causal):
    B, H, T, D = q.shape
    M = k.shape[2]
    outs = [torch.empty_like(t) for t in (q, k, v)]
    ws_bytes = lib.theria_sdpa_bwd_workspace_bytes(B, H, T, M, D)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    st = lib.theria_sdpa_bwd(
        _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(o), CODE[o.dtype], _lib.ptr(do),
        _lib.ptr(lse), *(_lib.ptr(t) for t in outs), _lib.ptr(ws), ws_bytes, B, H, T, M, D,
        CODE[q.dtype], 1.0 / D ** 0.5, int(causal), _lib.stream_of(q))
    assert st == _lib.THERIA_OK
    return outs


def _bwd_noalloc(lib, q, k, v, o, do, lse, causal):
    B, H, T, D = q.shape
    M = k.shape[2]
    outs = [torch.empty_like(t) for t in (q, k, v)]
    st = lib.theria_sdpa_bwd_noalloc(
        _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(o), CODE[o.dtype], _lib.ptr(do),
        _lib.ptr(lse), *(_lib.ptr(t) for t in outs), B, H, T, M, D, CODE[q.dtype],
        1.0 / D ** 0.5, int(causal), _lib.stream_of(q))
    assert st == _lib.THERIA_OK, lib.theria_status_string(st)
    return outs


# (dtype, shape, causal, path the noalloc entry point should take): 1 = the
# tensor-core backward, 0 = whole-head or CUDA-core kernels.  fp32 T > 64
# and the bf16 (1, 4, 2048, 128) case keep their row terms in the scratch
# array; the latter's fp32 dQ accumulator does not fit beside them, so it
# runs the CUDA-core kernels.
CASES = [
    (torch.float32, (2, 2, 64, 32), False, 0),
    (torch.float32, (1, 4, 64, 16), True, 0),
    (torch.float32, (1, 2, 200, 64), True, 0),
    (torch.bfloat16, (1, 2, 257, 128), False, 1),
    (torch.float16, (2, 2, 130, 64), True, 1),
    (torch.bfloat16, (1, 4, 2048, 128), False, 0),
]


@pytest.mark.parametrize("dtype,shape,causal,tc", CASES)
def test_noalloc_matches_regular_backward_twice(dtype, shape, causal, tc):
    lib = _lib.load()
    B, H, T, D = shape
    assert lib.theria_sdpa_bwd_noalloc_uses_tc(B, H, T, T, D, CODE[dtype]) == tc
    for call, seed in enumerate((11, 12)):  # two calls in a row, different data
        q, k, v, do = _inputs(shape, dtype, seed)
        o, lse = ops.forward(q, k, v, causal=causal)
        want = _bwd_regular(lib, q, k, v, o, do, lse, causal)
        got = _bwd_noalloc(lib, q, k, v, o, do, lse, causal)
        torch.cuda.synchronize()
        for a, b, name in zip(got, want, ("dq", "dk", "dv")):
            if dtype == torch.float32:
                assert max_rel(a, b) <= 1e-5, (call, name)
            else:
                assert max_abs(a, b) <= 2e-2, (call, name)
        if call == 0:
            # the first call also against the CPU oracle (two heads at most)
            hs = slice(0, 2)
            qc, kc, vc, dc = (t[:1, hs].float().cpu() for t in (q, k, v, do))
            ref = orc.backward(qc, kc, vc, dc, causal=causal)
            for a, b, name in zip(got, ref, ("dq", "dk", "dv")):
                a = a[:1, hs].float().cpu()
                if dtype == torch.float32:
                    assert max_rel(a, b) <= 1e-5, ("oracle", name)
                else:
                    assert max_abs(a, b) <= 2e-2, ("oracle", name)


def test_noalloc_refuses_problems_beyond_its_scratch():
    lib = _lib.load()
    # B*H*T*4 bytes = 8 MiB > the 4 MiB scratch; refused before any launch.
    p = ctypes.c_void_p(256)
    st = lib.theria_sdpa_bwd_noalloc(p, p, p, None, 0, p, p, p, p, p,
                                     1, 16, 131072, 128, 64, _lib.BF16, 0.125, 0, None)
    assert st == _lib.THERIA_ERR_SCRATCH_LIMIT
    assert b"scratch" in lib.theria_status_string(st)
    assert lib.theria_sdpa_bwd_noalloc_uses_tc(1, 16, 131072, 131072, 64, _lib.BF16) == \
        -_lib.THERIA_ERR_SCRATCH_LIMIT
