"""GDN-2 language model (atomic_gdn2/training/model.py:6-20): byte embedding, n_layers GDN-2
layers, final normalisation and a dense head.  At the benchmark configuration (d_model 512,
6 heads of 128, 8 layers, vocab 256, MLP expansion 4) it has 39,121,152 parameters, the count of
the reference's layer.py model (the README's 34.9M-parameter model is a different notebook
architecture)."""
from __future__ import annotations

import math

import torch

from ..layer import GDN2Layer, dense_init, lnorm
from ..pipeline import make_blr_trainable


def lm_config():
    """The BASELINE LM: width 512, H 6, D 128, 8 layers, byte vocabulary."""
    return dict(d_model=512, n_heads=6, d_head=128, n_layers=8, vocab=256, expansion=4)


class GDN2LM(torch.nn.Module):
    """init_model + model_fwd.  `blr_fn` defaults to the CUDA operator
    make_blr_trainable(cfg, 1/sqrt(d_head)) (model.py:13) and `prologue_fn` to the fused CUDA
    prologue; CPU tests pass restatements of both."""

    def __init__(self, cfg, d_model, n_heads, d_head, n_layers, vocab=256, expansion=4, g_init=0.05, seed=0,
                 blr_fn=None, l2norm_k=True, prologue_fn=None):
        super().__init__()
        gen = torch.Generator().manual_seed(seed)
        self.cfg, self.l2norm_k = cfg, l2norm_k
        self.embed = torch.nn.Parameter(torch.randn(vocab, d_model, generator=gen) * 0.02)
        self.layers = torch.nn.ModuleList(
            GDN2Layer(d_model, n_heads, d_head, expansion, g_init, generator=gen, prologue_fn=prologue_fn)
            for _ in range(n_layers))
        w, b = dense_init(d_model, vocab, generator=gen)
        self.head_w, self.head_b = torch.nn.Parameter(w), torch.nn.Parameter(b)
        self.blr_fn = blr_fn if blr_fn is not None else make_blr_trainable(cfg, 1.0 / math.sqrt(d_head))

    def forward(self, tokens: torch.Tensor, stats: bool = False):
        x = self.embed[tokens]
        st = []
        for layer in self.layers:
            r = layer(x, self.blr_fn, self.cfg, l2norm_k=self.l2norm_k, stats=stats)
            x, s = r if stats else (r, None)
            st.append(s)
        B, L, d = x.shape
        logits = torch.addmm(self.head_b, lnorm(x).reshape(B * L, d), self.head_w).view(B, L, -1)
        return (logits, st) if stats else logits


def n_params(model: torch.nn.Module) -> int:
    return sum(p.numel() for n, p in model.named_parameters())
