"""(batch x head) slice sharding across ranks, and the gather used to verify it.

Attention over [B, H, N, d] is independent per (b, h) slice, so a multi-GPU run
gives each rank a contiguous range of the B*H flattened slices (a contiguous
byte range of every contiguous [B, H, N, d] tensor) and needs no communication
while computing.  The only collective is the all-gather of O and LSE after the
timed region, to check the sharded result (NCCL over NVLink on the GPU box, gloo
in the CPU tests).  The reference has no multi-GPU code; this module is new.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist


def slice_range(num_slices: int, rank: int, world: int) -> Tuple[int, int]:
    """[lo, hi) of the flattened (b, h) slices owned by `rank`; sizes differ by at most 1."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    base, extra = divmod(num_slices, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def shard(t: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's slices of a contiguous [B, H, N, d] (or [B, H, N]) tensor, as [1, S_r, ...]."""
    if not t.is_contiguous():
        raise RuntimeError("shard() needs a contiguous tensor")
    b, h = t.shape[0], t.shape[1]
    lo, hi = slice_range(b * h, rank, world)
    return t.reshape(b * h, *t.shape[2:])[lo:hi].unsqueeze(0)


def gather(local: torch.Tensor, num_slices: int, group: Optional[dist.ProcessGroup] = None) -> torch.Tensor:
    """All-gather every rank's [1, S_r, ...] shard into [num_slices, ...] on every rank.

    Shards are padded to the largest shard so the collective has equal counts.
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    lo, hi = slice_range(num_slices, rank, world)
    if local.shape[1] != hi - lo:
        raise RuntimeError(f"rank {rank} holds {local.shape[1]} slices, expected {hi - lo}")
    width = max(slice_range(num_slices, r, world)[1] - slice_range(num_slices, r, world)[0] for r in range(world))
    tail = local.shape[2:]
    pad = torch.zeros((width, *tail), dtype=local.dtype, device=local.device)
    pad[: hi - lo] = local[0]
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    out = []
    for r in range(world):
        a, b = slice_range(num_slices, r, world)
        out.append(parts[r][: b - a])
    return torch.cat(out, dim=0)
