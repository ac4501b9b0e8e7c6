"""Token-row sharding across GPUs and the final output all-gather.

The projection path is independent per token row, so a latent of M rows is
split into contiguous per-rank row blocks, every rank runs the W8A8 path on its
block with the int8 weights replicated, and the only collective is one
all-gather of the bf16 output rows at the end (NCCL over NVLink/NVSwitch on a
B200 node). Shards differ by at most one row; the gather pads every shard to
the largest one and strips the padding afterwards.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_bounds(total: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of this rank's contiguous row block (first ranks get the remainder)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"invalid rank {rank} of world {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_rows(x: torch.Tensor, world: int, rank: int, dim: int = -2) -> torch.Tensor:
    """This rank's row block of ``x`` along ``dim`` (a view)."""
    start, stop = shard_bounds(x.shape[dim], world, rank)
    return x.narrow(dim, start, stop - start)


def gather_rows(local: torch.Tensor, total: int, group=None) -> torch.Tensor:
    """All-gather the row blocks of every rank into the full [total, ...] tensor.

    ``local`` is this rank's block (rows on dim 0). One all_gather_into_tensor
    of equally padded shards; the result is identical on every rank.
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    start, stop = shard_bounds(total, world, rank)
    if local.shape[0] != stop - start:
        raise ValueError(f"rank {rank} holds {local.shape[0]} rows, expected {stop - start}")
    width = -(-total // world)
    padded = local.new_zeros((width, *local.shape[1:]))
    padded[: local.shape[0]] = local
    out = local.new_empty((world * width, *local.shape[1:]))
    dist.all_gather_into_tensor(out, padded.contiguous(), group=group)
    if total % world == 0:
        return out
    parts = []
    for r in range(world):
        s, e = shard_bounds(total, world, r)
        parts.append(out[r * width: r * width + (e - s)])
    return torch.cat(parts, dim=0)
