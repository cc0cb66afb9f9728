"""Domain of correctness and guards (atomic_gdn2/domain.py:1-62), torch versions.

I-1: g <= 0.   I-2: beta*||k||^2 <= 2.   I-3 (reference BTL diagonal): half_span < 88.
This build's kernels rescale each channel of a chunk by one reference point when the channel's
span of gc = cumsum(g) inside the chunk is <= SPAN_LIMIT (128) and evaluate wider channels'
intra-chunk terms exactly on the CUDA cores, so every span the reference accepts (g_max up to
5) is computed; only positive gates (I-1) are refused by the operator.
"""
from __future__ import annotations

import math

import torch

from .config import BTL_HARD_LIMIT, BTL_STOP, BTL_WARN

SPAN_LIMIT = 128.0


def half_span_max(gc_chunks: torch.Tensor, bs2: int) -> float:
    """domain.py:14-20: gc_chunks (B,H,nc,bt,D) cumsum inside chunk -> max half-span over bs2 blocks."""
    lead = gc_chunks.shape[:-2]
    bt, D = gc_chunks.shape[-2:]
    blk = gc_chunks.reshape(lead + (bt // bs2, bs2, D))
    span = blk[..., 0, :] - blk[..., -1, :]
    return float(0.5 * span.max())


def half_span_from_g(g_hm: torch.Tensor, bt: int, bs2: int) -> float:
    """domain.py:23-27: g (B,H,L,D) -> max half span."""
    b, h, L, d = g_hm.shape
    gc = torch.cumsum(g_hm.float().reshape(b, h, L // bt, bt, d), dim=-2)
    return half_span_max(gc, bs2)


def chunk_span_max(g_hm: torch.Tensor, bt: int) -> float:
    """Largest per-channel span (max - min of gc) inside one chunk; channels above SPAN_LIMIT take
    the kernels' exact wide-channel path."""
    b, h, L, d = g_hm.shape
    gc = torch.cumsum(g_hm.float().reshape(b, h, L // bt, bt, d), dim=-2)
    return float((gc.amax(-2) - gc.amin(-2)).max())


def bk2_stat(k: torch.Tensor, b: torch.Tensor):
    """domain.py:30-33: max/mean of sum_d b*k^2 (I-2)."""
    x = (b * k * k).sum(-1)
    return float(x.max()), float(x.mean())


def clamp_g(g_neg: torch.Tensor, g_max: float) -> torch.Tensor:
    """domain.py:36-38: enforce |g| <= g_max on g <= 0."""
    return torch.clamp(g_neg, min=-g_max)


def init_g_bias(target: float = 0.05) -> float:
    """domain.py:41-43: bias so that softplus(bias) = target."""
    return math.log(math.expm1(target))


def check_preconditions(g_hm: torch.Tensor, cfg, strict: bool = True) -> dict:
    """domain.py:46-55: BTL half-span status (reference semantics) plus this build's chunk span."""
    hs = half_span_from_g(g_hm, cfg.bt, cfg.bs2) if cfg.diag == "btl" else 0.0
    status = "ok"
    if hs > BTL_STOP:
        status = "STOP"
    elif hs > BTL_WARN:
        status = "warn"
    if strict and status == "STOP":
        raise RuntimeError(f"BTL half_span={hs:.1f} > {BTL_STOP} (limit {BTL_HARD_LIMIT}); reduce bs2 or clamp g")
    span = chunk_span_max(g_hm, cfg.bt)
    return {"half_span_max": hs, "status": status, "chunk_span_max": span, "wide_channels": span > SPAN_LIMIT,
            "kernel_ok": bool((g_hm <= 0).all())}


def safe_bs2_for(g_max: float, candidates=(128, 64, 32, 16, 8)) -> int:
    """domain.py:58-62."""
    for c in candidates:
        if g_max * c / 2.0 < BTL_STOP:
            return c
    return candidates[-1]
