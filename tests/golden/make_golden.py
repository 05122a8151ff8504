"""Generate the golden vectors in this folder by running the reference itself.

Run in a container where the reference project (alexgabel/theria) is
importable:

    python tests/golden/make_golden.py --reference <path to theria checkout>

It draws seeded CPU inputs, calls the reference's own CPU functions and
writes ``sdpa_<case>.npz``.  Those files are committed; the tests read them
and never import the reference (it is absent on the GPU box).

Reference functions exercised (paths inside the theria project):
  theria/attention/reference_attention.py:9-19        reference_attention
  theria/attention/reference_backward_sdpa.py:12-53   sdpa_backward_reference
  theria/attention/reference_jvp_sdpa.py:21-44        sdpa_jvp_reference (fp64)
  theria/attention/reference_hvp_sdpa.py:46-97        sdpa_hvp (loss = sum(O))
  theria/autograd/sdpa_custom_function.py:14-53       SDPACustom double-backward
"""

from __future__ import annotations

import argparse
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# case name -> (B, H, N, D): cfg1 of the benchmark plan, and the per-head
# shape the MAML classifier's attention runs at (d_model 64, 4 heads).
CASES = {
    "cfg1": (2, 2, 64, 32),
    "maml": (1, 4, 64, 16),
}


def make_case(name, shape, seed=0):
    from theria.attention.reference_attention import reference_attention
    from theria.attention.reference_backward_sdpa import sdpa_backward_reference
    from theria.attention.reference_jvp_sdpa import sdpa_jvp_reference
    from theria.attention.reference_hvp_sdpa import sdpa_hvp
    from theria.autograd.sdpa_custom_function import SDPACustom

    g = torch.Generator("cpu").manual_seed(seed)
    names = ["q", "k", "v", "dout", "tq", "tk", "tv", "vq", "vk", "vv"]
    x = {n: torch.randn(*shape, generator=g, dtype=torch.float32) for n in names}
    scale = 1.0 / math.sqrt(shape[-1])
    out = {}
    out["o"] = reference_attention(x["q"], x["k"], x["v"])
    out["dq"], out["dk"], out["dv"] = sdpa_backward_reference(
        x["q"], x["k"], x["v"], x["dout"], scale)
    out["jvp"] = sdpa_jvp_reference(
        x["q"], x["k"], x["v"], x["tq"], x["tk"], x["tv"], scale)
    hs = sdpa_hvp(x["q"], x["k"], x["v"], x["vq"], x["vk"], x["vv"])
    out["hvp_sum_q"], out["hvp_sum_k"], out["hvp_sum_v"] = hs

    # H u of L = sum(O * dout) through the reference's double-backward
    # Function, along u = (vq, vk, vv) -- in fp64 so the fixture itself is
    # accurate to well below the fp32 tolerance.
    qd, kd, vd = (x[n].double().requires_grad_(True) for n in ("q", "k", "v"))
    o = SDPACustom.apply(qd, kd, vd)
    loss = (o * x["dout"].double()).sum()
    gr = torch.autograd.grad(loss, (qd, kd, vd), create_graph=True)
    dot = sum((a * x[n].double()).sum() for a, n in zip(gr, ("vq", "vk", "vv")))
    hq, hk, hv = torch.autograd.grad(dot, (qd, kd, vd))
    out["hvp_w_q"], out["hvp_w_k"], out["hvp_w_v"] = hq.float(), hk.float(), hv.float()

    arrs = {f"in_{n}": t.numpy() for n, t in x.items()}
    arrs.update({f"out_{n}": t.detach().float().numpy() for n, t in out.items()})
    arrs["scale"] = np.float32(scale)
    path = os.path.join(HERE, f"sdpa_{name}.npz")
    np.savez_compressed(path, **arrs)
    print(f"wrote {path}: {len(arrs)} arrays")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="path of the theria project root to import")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    for name, shape in CASES.items():
        make_case(name, shape)


if __name__ == "__main__":
    main()
