"""Row sharding of the op path across ranks (one process per GPU).

The ops are row-wise, so a job over T token rows splits into contiguous row
ranges with no exchange on the hot path.  The only collectives are outside
it: the max over ranks of a measured time, and an all-gather of sampled rows
for a correctness check on rank 0.  Works with any torch.distributed backend
(NCCL on GPUs, gloo on CPU for tests).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def row_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """(first row, row count) of `rank`: contiguous ranges, sizes differing
    by at most one, earlier ranks taking the remainder."""
    if world < 1 or not 0 <= rank < world or total < 0:
        raise ValueError(f"bad split: total={total} world={world} rank={rank}")
    base, rem = divmod(total, world)
    start = rank * base + min(rank, rem)
    return start, base + (1 if rank < rem else 0)


def positions(total: int, world: int, rank: int, device=None) -> torch.Tensor:
    """Global token positions of the rank's rows (RoPE uses global positions)."""
    start, n = row_range(total, world, rank)
    return torch.arange(start, start + n, device=device)


def max_over_ranks(value: float, device=None) -> float:
    """The maximum of `value` over all ranks (identity without a process group)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_rows(sample: torch.Tensor) -> torch.Tensor:
    """All-gather equally shaped per-rank tensors into [world, *sample.shape]."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return sample.unsqueeze(0)
    world = dist.get_world_size()
    flat = sample.reshape(-1).contiguous()
    out = torch.empty(world * flat.numel(), dtype=flat.dtype, device=flat.device)
    dist.all_gather_into_tensor(out, flat)
    return out.view(world, *sample.shape)
