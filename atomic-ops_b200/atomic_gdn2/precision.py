"""Precision modes (atomic_gdn2/precision.py:1-52) as this build realises them on the tensor core.

    mode       reference meaning (TPU)                 B200 realisation (tcgen05)
    highest    f32 dot (Precision.HIGHEST)             3 x kind::tf32: hi*hi + hi*lo + lo*hi
    bf16x3     dot_bf16x3: hi/lo bf16, 3 products      3 x kind::f16 (bf16 operands), same split
    default    1 bf16 pass (Precision.DEFAULT)         1 x kind::f16 (bf16 operands)
    tf32       (not in the reference)                  1 x kind::tf32

Accumulation is always fp32 in tensor memory.  `sanitize` is applied by the kernels at the same
stages as the reference (scores, WY inverse, wp/u/kg/qg, the state update, o and every gradient);
the host applies it once more only where a caller's clip is looser than the final bound.

This module is the single table of modes: config.py validates against it, _lib.py passes its
C-ABI values (gdn2_precision in include/gdn2_b200.h) to the kernels, pipeline.py uses `sanitize`.
"""
import torch

DOT_MODES = ("highest", "bf16x3", "default")   # the reference's modes (precision.py:8-37)
EXTRA_DOT_MODES = ("tf32",)                    # B200-only mode (1 x kind::tf32)
ALL_MODES = DOT_MODES + EXTRA_DOT_MODES
ENUM = {"highest": 0, "bf16x3": 1, "default": 2, "tf32": 3}   # gdn2_precision
PASSES = {"highest": 3, "bf16x3": 3, "default": 1, "tf32": 1}
OPERAND = {"highest": "tf32", "bf16x3": "bf16", "default": "bf16", "tf32": "tf32"}


def sanitize(x: torch.Tensor, clip: float) -> torch.Tensor:
    """precision.py:50-51: nan_to_num(clip(x, -c, c))."""
    return torch.nan_to_num(x.clamp(-clip, clip), nan=0.0, posinf=clip, neginf=-clip)
