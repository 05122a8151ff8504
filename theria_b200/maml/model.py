"""The full-MAML benchmark model: a tiny pre-LN transformer classifier.

2 encoder layers, d_model 64, 4 heads (head dim 16), FFN 256 (GELU),
learned token and position embeddings, final LayerNorm, mean-pool over the
sequence and a linear head; fp32 parameters, Xavier-uniform matrices and
zero biases (106,565 parameters at the default sizes).  This model is not in
the reference library; its closest template there is the pre-LN decoder of
``examples/minimal_decoder_transformer.py:82-263``.  Attention runs through
``attn_fn`` (default: this library's twice-differentiable fused SDPA).

Every layer is written once for a leading *task* axis (``forward_tasks``),
so a meta-batch of tasks can be adapted in one pass with per-task
parameters; ``forward`` is the same code with a task axis of one, which is
what ``torch.func.functional_call`` drives in the reference-style loops.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from theria_b200.attention.fused import sdpa_fused
from theria_b200.attention.packed import sdpa_qkv
from theria_b200.maml.layer_norm import gelu, layer_norm
from theria_b200.maml.task_bmm import add_bias, tbmm


@dataclass(frozen=True)
class ModelConfig:
    vocab: int = 32
    seq_len: int = 64
    d_model: int = 64
    n_heads: int = 4
    d_ff: int = 256
    n_layers: int = 2
    n_classes: int = 5


def _linear(h, w, b, res=None):
    # h (nt, ..., din), w (nt, dout, din), b (nt, dout); res: an optional
    # residual added in the bias kernel.  tbmm: the weight gradients reduce
    # over all rows of a task, which tbmm splits.
    nt = h.shape[0]
    shp = h.shape
    out = add_bias(tbmm(h.reshape(nt, -1, shp[-1]), w.transpose(1, 2)), b, res)
    return out.view(*shp[:-1], w.shape[1])


def _layer_norm(h, w, b):
    # fused kernels on CUDA tensors (twice differentiable), torch ops on CPU
    return layer_norm(h, w, b)


class MAMLClassifier(nn.Module):
    def __init__(self, cfg: ModelConfig = ModelConfig(), attn_fn=None):
        super().__init__()
        self.cfg = cfg
        self.attn_fn = attn_fn if attn_fn is not None else sdpa_fused
        D, F_ = cfg.d_model, cfg.d_ff
        self.tok = nn.Parameter(torch.empty(cfg.vocab, D))
        self.pos = nn.Parameter(torch.empty(cfg.seq_len, D))
        self.blocks = nn.ModuleList()
        for _ in range(cfg.n_layers):
            blk = nn.Module()
            blk.ln1_w = nn.Parameter(torch.ones(D))
            blk.ln1_b = nn.Parameter(torch.zeros(D))
            blk.qkv_w = nn.Parameter(torch.empty(3 * D, D))
            blk.qkv_b = nn.Parameter(torch.zeros(3 * D))
            blk.out_w = nn.Parameter(torch.empty(D, D))
            blk.out_b = nn.Parameter(torch.zeros(D))
            blk.ln2_w = nn.Parameter(torch.ones(D))
            blk.ln2_b = nn.Parameter(torch.zeros(D))
            blk.ff1_w = nn.Parameter(torch.empty(F_, D))
            blk.ff1_b = nn.Parameter(torch.zeros(F_))
            blk.ff2_w = nn.Parameter(torch.empty(D, F_))
            blk.ff2_b = nn.Parameter(torch.zeros(D))
            self.blocks.append(blk)
        self.lnf_w = nn.Parameter(torch.ones(D))
        self.lnf_b = nn.Parameter(torch.zeros(D))
        self.head_w = nn.Parameter(torch.empty(cfg.n_classes, D))
        self.head_b = nn.Parameter(torch.zeros(cfg.n_classes))
        for name, p in self.named_parameters():
            if p.ndim == 2:
                nn.init.xavier_uniform_(p)

    # -- task-batched forward -------------------------------------------
    def forward_tasks(self, params, x):
        """params: name -> tensor with a leading task axis nt; x (nt, n, L)."""
        cfg = self.cfg
        nt, n, L = x.shape
        D, H = cfg.d_model, cfg.n_heads
        Dh = D // H
        # Token embedding as a one-hot product: its gradient (and the
        # gradient's gradient) is then a batched GEMM, not a sort-based
        # scatter-add; exact in fp32 (one nonzero term per output).
        onehot = F.one_hot(x.reshape(nt, n * L), cfg.vocab).to(params["tok"].dtype)
        h = tbmm(onehot, params["tok"]).view(nt, n, L, D)
        h = h + params["pos"][:, :L].unsqueeze(1)
        for i in range(cfg.n_layers):
            p = lambda s: params[f"blocks.{i}.{s}"]  # noqa: E731
            a = _layer_norm(h, p("ln1_w"), p("ln1_b"))
            qkv = _linear(a, p("qkv_w"), p("qkv_b")).view(nt * n, L, 3, H, Dh)
            if self.attn_fn is sdpa_fused and qkv.is_cuda:
                # the default attention, on the packed projection: q, k, v
                # read in place, O written token-major (no layout copies)
                o = sdpa_qkv(qkv).reshape(nt, n, L, D)
            else:
                q, k, v = qkv.permute(2, 0, 3, 1, 4).unbind(0)  # (nt*n, H, L, Dh) each
                o = self.attn_fn(q, k, v).transpose(1, 2).reshape(nt, n, L, D)
            h = _linear(o, p("out_w"), p("out_b"), res=h)
            f = _layer_norm(h, p("ln2_w"), p("ln2_b"))
            f = gelu(_linear(f, p("ff1_w"), p("ff1_b")))
            h = _linear(f, p("ff2_w"), p("ff2_b"), res=h)
        h = _layer_norm(h, params["lnf_w"], params["lnf_b"]).mean(dim=2)  # (nt, n, D)
        return _linear(h, params["head_w"], params["head_b"])  # (nt, n, C)

    def _current_params(self):
        # Attribute lookups, so torch.func.functional_call substitutions apply.
        out = {}
        for name, _ in self.named_parameters():
            obj = self
            for part in name.split("."):
                obj = getattr(obj, part)
            out[name] = obj
        return out

    def forward(self, x):
        """x (n, L) int tokens -> logits (n, C)."""
        params = {k: v.unsqueeze(0) for k, v in self._current_params().items()}
        return self.forward_tasks(params, x.unsqueeze(0)).squeeze(0)
