"""gdn2_forward / gdn2_forward_trainable (atomic_ops/fallback.py:9-22) on the B200 operator."""
from __future__ import annotations

import torch

from atomic_gdn2 import make_blr_trainable, make_cfg

from .configs import DEFAULT_CONFIG, KernelConfig, validate_inputs

_T = 128  # the operator's chunk length


def _operator(config: KernelConfig, L: int, scale: float):
    cfg = make_cfg(bt=_T, wy_eps=config.wy_eps, clip=config.clip, dot_mode="highest",
                   solve_dot_mode="highest", b3_dot_mode="highest", max_chunks_per_call=max(1, L // _T))
    return make_blr_trainable(cfg, scale)


def gdn2_forward_trainable(q, k, v, w, b, g, scale, h0=None, config: KernelConfig = None):
    """(B, L, H, D) inputs -> (o (B, L, H, D) fp32, h_final (B, H, D, D) fp32); differentiable
    w.r.t. q, k, v, w, b, g and h0 (atomic_ops/gdn2_pipeline.py:145-152).

    With wy_eps > 0 the reference damps every interaction inside one config.bt-token chunk
    (A = (I + (1 - eps) Akk)^-1 over the whole chunk), so the result depends on the chunk length;
    this operator's chunk is 128 tokens, so such configs are accepted only with bt = 128.  With
    wy_eps = 0 the chunked-WY result is the same for every chunk length and any bt works."""
    config = config or DEFAULT_CONFIG
    validate_inputs(q, k, v, w, b, g, scale, h0, config)
    if config.wy_eps > 0 and config.bt != _T:
        raise NotImplementedError(
            f"wy_eps={config.wy_eps} damps within {config.bt}-token chunks; the B200 operator's chunk is {_T} "
            f"tokens: use bt={_T} (e.g. KAGGLE_SMALL) or wy_eps=0")
    L = q.shape[1]
    fn = _operator(config, L, float(scale))
    hm = [t.transpose(1, 2).contiguous() for t in (q, k, v, w, b, g)]
    o, h_final = fn(*hm, h0)
    return o.transpose(1, 2), h_final


def gdn2_forward(q, k, v, w, b, g, scale, h0=None, config: KernelConfig = None):
    """Forward only (atomic_ops/fallback.py:9-14, gdn2_fwd.py:340-361)."""
    with torch.no_grad():
        return gdn2_forward_trainable(q, k, v, w, b, g, scale, h0=h0, config=config)
