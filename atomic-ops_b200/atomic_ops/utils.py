"""atomic_ops/utils.py:1-36: device probe, memory estimate, preset picker."""
from __future__ import annotations

from .configs import KAGGLE_LARGE, KAGGLE_MEDIUM, KAGGLE_SMALL, KernelConfig


def is_tpu_available() -> bool:
    """There is no TPU in a B200 deployment; the operator runs on CUDA."""
    return False


def estimate_memory(batch: int, seq_len: int, heads: int, d_head: int = 128, bt: int = 256,
                    bytes_per_param: int = 4) -> float:
    """Rough residual footprint in MB (utils.py:14-24, the reference's formula)."""
    n_chunks = seq_len // bt
    per_chunk = (bt * bt * 3) + (bt * d_head * 7) + (d_head * d_head * 2)
    return batch * heads * n_chunks * per_chunk * bytes_per_param / (1024 * 1024)


def get_recommended_config(batch: int, seq_len: int, heads: int, d_head: int = 128) -> KernelConfig:
    """utils.py:27-35."""
    mem = estimate_memory(batch, seq_len, heads, d_head)
    if mem > 6000:
        return KAGGLE_LARGE
    if mem > 2500:
        return KAGGLE_MEDIUM
    return KAGGLE_SMALL
