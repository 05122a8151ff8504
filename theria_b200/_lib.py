"""ctypes binding of libtheria_sm100.so (the C ABI in include/theria_sdpa.h).

There is no fallback: if the library is missing or fails to load, every
operator raises.  ``THERIA_LIB`` may point at another build of the library.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("THERIA_LIB", os.path.join(HERE, "libtheria_sm100.so"))

THERIA_OK = 0
THERIA_ERR_INVALID_ARG = 1
THERIA_ERR_UNSUPPORTED = 2
THERIA_ERR_LAUNCH = 3
THERIA_ERR_WORKSPACE = 4
THERIA_ERR_DEVICE_TIMEOUT = 5
THERIA_ERR_SCRATCH_LIMIT = 6
NOALLOC_SCRATCH_BYTES = 4 * 1024 * 1024

F32, F16, BF16, F64 = 0, 1, 2, 3
DTYPE_CODE = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16, torch.float64: F64}

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i = ctypes.c_int
_f = ctypes.c_float

# name -> (restype, argtypes); must mirror include/theria_sdpa.h and
# include/theria_ln.h exactly.
SIGNATURES = {
    "theria_status_string": (ctypes.c_char_p, [_i]),
    "theria_version": (ctypes.c_char_p, []),
    "theria_sdpa_fwd": (_i, [_vp, _vp, _vp, _vp, _i, _vp,
                             _i64, _i64, _i64, _i64, _i64, _i, _f, _i, _vp]),
    "theria_sdpa_bwd_workspace_bytes": (_i64, [_i64] * 5),
    "theria_sdpa_hvp_workspace_bytes": (_i64, [_i64] * 5),
    "theria_sdpa_bwd": (_i, [_vp, _vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _vp, _vp, _i64,
                             _i64, _i64, _i64, _i64, _i64, _i, _f, _i, _vp]),
    "theria_sdpa_jvp": (_i, [_vp] * 8 + [_i64] * 5 + [_i, _f, _i, _vp]),
    "theria_sdpa_hvp": (_i, [_vp] * 12 + [_vp, _i64] + [_i64] * 5 + [_i, _f, _i, _vp]),
    "theria_sdpa_bwd_noalloc": (_i, [_vp] * 10 + [_i64] * 5 + [_i, _f, _i, _vp]),
    "theria_sdpa_bwd_noalloc_uses_tc": (_i, [_i64] * 5 + [_i]),
    "theria_sdpa_scores": (_i, [_vp, _vp, _vp, _i] + [_i64] * 5 + [_i, _f, _vp]),
    "theria_sdpa_probs": (_i, [_vp] * 4 + [_i64] * 5 + [_i, _f, _i, _vp]),
    "theria_sdpa_qkv_fwd": (_i, [_vp] * 3 + [_i64] * 4 + [_i, _f, _i, _vp]),
    "theria_sdpa_qkv_bwd": (_i, [_vp] * 4 + [_i64] * 4 + [_i, _f, _i, _vp]),
    "theria_sdpa_qkv_hvp": (_i, [_vp] * 6 + [_i64] * 4 + [_i, _f, _i, _vp]),
    "theria_launch_count": (_i64, []),
    "theria_ln_workspace_bytes": (_i64, [_i64] * 3),
    "theria_rowsum_workspace_bytes": (_i64, [_i64] * 3),
    "theria_gelu_bwd2": (_i, [_vp] * 5 + [_i64, _vp]),
    "theria_chunk_sum": (_i, [_vp, _vp, _i64, _i64, _i64, _vp]),
    "theria_add_bias": (_i, [_vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _vp]),
    "theria_rowsum": (_i, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp]),
    "theria_ln_fwd": (_i, [_vp, _vp, _vp, _i64, _vp, _i64, _i64, _i64, _f, _vp]),
    "theria_ln_bwd": (_i, [_vp, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _i64,
                           _i64, _i64, _i64, _f, _vp]),
    "theria_ln_bwd2": (_i, [_vp, _vp, _i64, _vp, _vp, _vp, _i64, _vp, _i64, _vp, _vp, _vp,
                            _vp, _i64, _i64, _i64, _i64, _f, _vp]),
    "theria_get_device_error": (_i, [ctypes.POINTER(ctypes.c_int), _vp]),
    "theria_clear_device_error": (_i, [_vp]),
    "theria_diag_bounded_wait": (_i, [_i, _vp, _vp]),
}

_lib = None
_lock = threading.Lock()


class TheriaError(RuntimeError):
    """A C-ABI call returned a non-zero THERIA_* status."""


def load():
    """Load (once) and return the library; raises if it is unavailable."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"theria_b200: CUDA library not built ({LIB_PATH}); run "
                    "`python -m theria_b200.build` (there is no CPU fallback)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(status: int, what: str) -> None:
    if status != THERIA_OK:
        msg = load().theria_status_string(status).decode()
        raise TheriaError(f"{what}: {msg} (status {status})")


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def device_error(device=None) -> int:
    """The device-side error word of `device` (synchronises its current stream)."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
    flag = ctypes.c_int(0)
    with torch.cuda.device(dev):
        st = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        check(load().theria_get_device_error(ctypes.byref(flag), st), "theria_get_device_error")
    return flag.value


def clear_device_error(device=None) -> None:
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
    with torch.cuda.device(dev):
        st = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        check(load().theria_clear_device_error(st), "theria_clear_device_error")


def check_device_error(device=None, clear: bool = True) -> None:
    """Raise TheriaError if a kernel's bounded device-side wait gave up on
    `device` since the word was last cleared (its outputs are then partly
    written).  Clears the word before raising when `clear` is set."""
    flag = device_error(device)
    if flag != THERIA_OK:
        if clear:
            clear_device_error(device)
        msg = load().theria_status_string(flag).decode()
        raise TheriaError(f"device-side error: {msg} (status {flag})")
