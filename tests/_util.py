"""Shared helpers of the test suite."""

import numpy as np
import torch

GOLDEN = __import__("os").path.join(__import__("os").path.dirname(__file__), "golden")


def max_rel(x, ref):
    """max|x - ref| / max|ref| over the whole tensor (the contract's metric)."""
    x = x.detach().double().cpu()
    ref = ref.detach().double().cpu()
    den = ref.abs().max().item()
    return (x - ref).abs().max().item() / (den if den > 0 else 1.0)


def max_abs(x, ref):
    return (x.detach().double().cpu() - ref.detach().double().cpu()).abs().max().item()


def load_golden(name):
    z = np.load(f"{GOLDEN}/sdpa_{name}.npz")
    return {k: torch.from_numpy(z[k]) for k in z.files}


def randn(shape, seed, dtype=torch.float32, gen=None):
    g = gen if gen is not None else torch.Generator("cpu").manual_seed(seed)
    return torch.randn(*shape, generator=g, dtype=torch.float32).to(dtype)
