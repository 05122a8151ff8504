"""Autograd contracts (``theria/autograd``) on the CUDA kernels."""

from .sdpa_custom_function import SDPACustom
from .sdpa_function import SDPAFunction, sdpa

__all__ = ["SDPACustom", "SDPAFunction", "sdpa"]
