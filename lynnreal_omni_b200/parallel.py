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


def frame_bounds(frames: int, frame_rows: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) rows of this rank when whole frames of ``frame_rows`` rows
    are distributed (first ranks get the remainder). Token compression selects
    and restores within a frame, so frame-aligned shards compress exactly as
    the whole sequence does."""
    f0, f1 = shard_bounds(frames, world, rank)
    return f0 * frame_rows, f1 * frame_rows


def gather_rows(local: torch.Tensor, total: int, group=None, bounds=None) -> torch.Tensor:
    """All-gather the row blocks of every rank into the full [total, ...] tensor.

    ``local`` is this rank's block (rows on dim 0); ``bounds[r]`` is rank r's
    [start, stop) (default: ``shard_bounds``). One all_gather_into_tensor of
    equally padded shards; the result is identical on every rank.
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    bounds = bounds or [shard_bounds(total, world, r) for r in range(world)]
    if len(bounds) != world or bounds[0][0] != 0 or bounds[-1][1] != total or any(
            bounds[r][1] != bounds[r + 1][0] for r in range(world - 1)):
        raise ValueError("row bounds must tile [0, total) in rank order")
    start, stop = bounds[rank]
    if local.shape[0] != stop - start:
        raise ValueError(f"rank {rank} holds {local.shape[0]} rows, expected {stop - start}")
    width = max(e - s for s, e in bounds)
    padded = local.new_zeros((width, *local.shape[1:]))
    padded[: local.shape[0]] = local
    out = local.new_empty((world * width, *local.shape[1:]))
    dist.all_gather_into_tensor(out, padded.contiguous(), group=group)
    if all(e - s == width for s, e in bounds):
        return out
    return torch.cat([out[r * width: r * width + (e - s)] for r, (s, e) in enumerate(bounds)], dim=0)
