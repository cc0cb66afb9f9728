"""KernelConfig, presets, sanitize and input validation of the legacy API
(atomic_ops/configs.py:16-136): same fields, defaults, checks and messages."""
from __future__ import annotations

import dataclasses as dc

import torch


@dc.dataclass(frozen=True)
class KernelConfig:
    bt: int = 256
    bc: int = 128
    mb: int = 16
    clip: float = 1e4
    wy_eps: float = 0.0

    @property
    def n_sub(self) -> int:
        return self.bt // self.bc

    @property
    def n_micro(self) -> int:
        return self.bc // self.mb

    def __post_init__(self):
        if self.bt % self.bc != 0:
            raise ValueError(f"bt={self.bt} must be divisible by bc={self.bc}")
        if self.bt != 2 * self.bc:
            raise ValueError(f"bt={self.bt} must equal 2*bc (top-level WY-solve split supports only the "
                             f"2-block case); got bc={self.bc}.")
        if self.bc % self.mb != 0:
            raise ValueError(f"bc={self.bc} must be divisible by mb={self.mb}")
        if not (0.0 <= self.wy_eps < 1.0):
            raise ValueError(f"wy_eps={self.wy_eps} must be in [0, 1)")


KAGGLE_SMALL = KernelConfig(bt=128, bc=64, mb=16, clip=1e4, wy_eps=1e-3)
KAGGLE_MEDIUM = KernelConfig(bt=256, bc=128, mb=16, clip=1e4, wy_eps=1e-3)
KAGGLE_LARGE = KernelConfig(bt=256, bc=128, mb=16, clip=5e3, wy_eps=1e-3)
DEFAULT_CONFIG = KAGGLE_MEDIUM


def sanitize(x: torch.Tensor, config: KernelConfig = DEFAULT_CONFIG) -> torch.Tensor:
    """configs.py:56-59: clip to +-clip, NaN -> 0, +-inf -> +-clip."""
    c = config.clip
    return torch.nan_to_num(torch.clamp(x, -c, c), nan=0.0, posinf=c, neginf=-c)


def validate_inputs(q, k, v, w, b, g, scale, h0, config: KernelConfig):
    """configs.py:116-136: shape checks shared by forward and backward entry points."""
    if q.ndim != 4:
        raise ValueError(f"q must be (batch, seq_len, heads, d_head); got shape {tuple(q.shape)}")
    bsz, L, H, D = q.shape
    if D != 128:
        raise ValueError(f"Kernels assume d_head=128; got D={D}.")
    if L % config.bt != 0:
        raise ValueError(f"seq_len={L} must be divisible by config.bt={config.bt}.")
    for name, t in (("k", k), ("v", v), ("w", w), ("b", b), ("g", g)):
        if t.shape != q.shape:
            raise ValueError(f"{name}.shape={tuple(t.shape)} must match q.shape={tuple(q.shape)}")
    if h0 is not None and tuple(h0.shape) != (bsz, H, D, D):
        raise ValueError(f"h0.shape={tuple(h0.shape)} must be {(bsz, H, D, D)}")
    return bsz, L, H, D, L // config.bt
