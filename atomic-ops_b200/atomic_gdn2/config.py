"""Operator configuration: the reference's BLRConfig / make_cfg surface, field for field.

Mirrors atomic_gdn2/config.py:1-83 (same fields, defaults, validation and errors).  How each
field maps onto the B200 kernels:

  bt, D          chunk length and head dim; this build implements bt = 128, D = 128
                 (other values raise NotImplementedError at call time, ValueError as in the
                 reference for invalid combinations here).
  clip           sanitize bound of intermediates and outputs (precision.py:50-51).
  wy_eps         WY damping A = (I + (1 - wy_eps) Akk)^-1 (fwd/solve.py:21-28).
  dot_mode       precision of scores, recompute, the forward state scan and B4-adjacent
  solve_dot_mode precision of the WY-inverse products
  b3_dot_mode    precision of backward stages B1-B3 (incl. the reverse state scan)
                 ("highest" = 3 x tf32, "bf16x3" = 3 x bf16, "default" = 1 x bf16, and the
                 extra "tf32" = 1 x tf32, which the reference does not have).
  max_chunks_per_call  segment length of a call in chunks; h is carried across segments.
  bc, mb, score_bs, bs2, diag, diff_clip, group, interpret, vmem_mb, g_max
                 TPU tiling / Pallas execution knobs of the reference.  They are accepted and
                 validated exactly as in the reference; the B200 kernels compute the gated
                 scores with one exact per-channel reference point per chunk (see
                 csrc/gdn2_fwd.cu), so these fields do not change the arithmetic.  g_max and bs2
                 keep their meaning for the layer-side gate clamp and the domain helpers.
"""
from __future__ import annotations

import dataclasses as dc

from .precision import DOT_MODES, EXTRA_DOT_MODES  # the mode table

MB = 1024 * 1024
DIAGS = ("btl", "lean")
BTL_HARD_LIMIT = 88.0     # exp overflow of one BTL leg (f32)
BTL_WARN = 60.0
BTL_STOP = 80.0


def _default_interpret() -> bool:
    # Pallas interpret mode has no meaning here; the field is kept for API compatibility.
    return False


def effective_group(n_chunks: int, requested):
    """config.py:19-25: largest divisor of n_chunks not above `requested`."""
    if requested is None or requested >= n_chunks:
        return n_chunks
    g = int(requested)
    while g > 1 and n_chunks % g:
        g -= 1
    return max(1, g)


@dc.dataclass(frozen=True)
class BLRConfig:
    # geometry
    bt: int = 128
    bc: int = 64
    mb: int = 8
    score_bs: int = 128
    bs2: int = 32
    diag: str = "btl"
    diff_clip: float = 20.0
    # numerics
    clip: float = 1e4
    wy_eps: float = 1e-3
    dot_mode: str = "highest"
    solve_dot_mode: str = "bf16x3"
    b3_dot_mode: str = "bf16x3"
    # execution
    group: int | None = None
    max_chunks_per_call: int = 32
    interpret: bool = dc.field(default_factory=_default_interpret)
    vmem_mb: float = 150.0
    # domain
    g_max: float = 160.0 / 32

    def __post_init__(self):
        # config.py:52-65, same checks and messages
        if self.bt != 2 * self.bc:
            raise ValueError(f"bt={self.bt} must equal 2*bc")
        if self.bt % self.score_bs or self.score_bs % self.bs2:
            raise ValueError("need bt % score_bs == 0 and score_bs % bs2 == 0")
        if self.mb & (self.mb - 1) or self.bt % self.mb or (self.bt // self.mb) & (self.bt // self.mb - 1):
            raise ValueError("mb and bt/mb must be powers of two dividing bt")
        if not 0.0 <= self.wy_eps < 1.0:
            raise ValueError("wy_eps in [0,1)")
        for m in (self.dot_mode, self.solve_dot_mode, self.b3_dot_mode):
            if m not in DOT_MODES + EXTRA_DOT_MODES:
                raise ValueError(f"dot mode {m} not in {DOT_MODES}")
        if self.diag not in DIAGS:
            raise ValueError(f"diag must be in {DIAGS}")
        if self.max_chunks_per_call < 1:
            raise ValueError("max_chunks_per_call must be >= 1")

    @property
    def n_sub(self):
        return self.bt // self.score_bs

    @property
    def n_inner(self):
        return self.score_bs // self.bs2

    @property
    def btl_half_span_limit(self):
        return self.g_max * self.bs2 / 2.0

    def with_(self, **kw):
        return dc.replace(self, **kw)


def make_cfg(**kw) -> BLRConfig:
    """PROD preset: bt=128, sbs=128, bs2=32, mb=8, btl, bf16x3 (B3), g_max tied to bs2
    (config.py:76-80)."""
    bs2 = kw.get("bs2", 32)
    kw.setdefault("g_max", 160.0 / bs2)
    return BLRConfig(**kw)


PROD = make_cfg
