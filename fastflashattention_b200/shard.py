"""Batch x head data parallelism: which (batch, head) slices a rank owns.

Attention is independent per (batch, head) slice, so a job spread over P GPUs (one
process per GPU) gives every rank a contiguous block of the flattened b*H + h slice
index and needs no communication on the data path.  Rank r owns
``[r * ceil(BH / P), min((r + 1) * ceil(BH / P), BH))``.  On a contiguous ``[B, H, S, D]``
tensor that block is a dim-0 slice of the ``[B*H, S, D]`` view, so a rank's shard is a
view, not a copy.  The only collective a job needs is for reporting, such as the maximum
of the ranks' device times (``max_over_ranks``).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def bh_range(bh: int, rank: int, world: int) -> tuple[int, int]:
    """[start, end) of the flattened (batch, head) slices rank `rank` of `world` owns."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} is not in a world of {world}")
    per = -(-bh // world)
    start = min(rank * per, bh)
    return start, min(start + per, bh)


def shard_heads(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's slices of a ``[B, H, S, D]`` tensor, as a ``[1, n, S, D]`` tensor
    (a view when `x` is contiguous) that ``fast_attention`` accepts directly."""
    B, H, S, D = x.shape
    start, end = bh_range(B * H, rank, world)
    return x.reshape(B * H, S, D)[start:end].unsqueeze(0)


def unshard_heads(shards: list[torch.Tensor], B: int, H: int) -> torch.Tensor:
    """Inverse of ``shard_heads`` given every rank's shard, in rank order."""
    flat = torch.cat([s.reshape(-1, *s.shape[-2:]) for s in shards], dim=0)
    if flat.shape[0] != B * H:
        raise ValueError(f"shards hold {flat.shape[0]} slices, expected B*H = {B * H}")
    return flat.reshape(B, H, *flat.shape[-2:])


def max_over_ranks(value: float, group=None) -> float:
    """The maximum of `value` over the ranks of `group` (the job's time is the slowest
    rank's).  Without an initialised process group it returns `value`."""
    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else torch.device("cpu")
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
