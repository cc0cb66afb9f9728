"""Batch x head sharding across GPUs (one process per GPU).

Every (b, h) pair of the operator is an independent recurrence (the reference's Pallas grids are
(B, H) for the scans, fwd/cd_slim.py:43, bwd/mega.py:71), so the operator shards over the
flattened B*H axis with no communication inside the kernels.  A rank's shard is presented to the
operator as a (1, n_local, L, D) tensor (B = 1, H = n_local heads).  NCCL (or gloo on CPU) is
only used to gather results when a caller wants the full tensor back.
"""
from __future__ import annotations

import torch


def bh_range(B: int, H: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [start, end) range of flattened heads owned by `rank` (sizes differ by <= 1)."""
    n = B * H
    base, rem = divmod(n, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def shard_heads(t: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """(B, H, ...) -> this rank's (1, n_local, ...) view of the flattened heads."""
    B, H = t.shape[:2]
    s, e = bh_range(B, H, rank, world)
    return t.reshape((1, B * H) + tuple(t.shape[2:]))[:, s:e]


def gather_heads(local: torch.Tensor, B: int, H: int, world: int, group=None) -> torch.Tensor:
    """Inverse of shard_heads over a process group: all ranks receive the full (B, H, ...)."""
    import torch.distributed as dist
    sizes = [bh_range(B, H, r, world) for r in range(world)]
    n_max = max(e - s for s, e in sizes)
    tail = tuple(local.shape[2:])
    buf = local.new_zeros((n_max,) + tail)
    buf[: local.shape[1]] = local[0]
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf.contiguous(), group=group)
    full = torch.cat([p[: e - s] for p, (s, e) in zip(parts, sizes)], 0)
    return full.reshape((B, H) + tail)
